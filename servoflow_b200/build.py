"""Builds libsfb200.so in-tree for sm_100a with nvcc (no GPU needed).

    python -m servoflow_b200.build
"""
from __future__ import annotations

import fcntl
import hashlib
import os
import subprocess
import sys

_HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(_HERE, "csrc")
OUT_DIR = os.path.join(_HERE, "_lib")
LIB = os.path.join(OUT_DIR, "libsfb200.so")
STAMP = LIB + ".sources"          # digest of the sources the library was built from

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    # a soname, so that a library linked against libsfb200 (the servoflow
    # binding) shares the copy a process has already loaded
    "-Xlinker", "-soname=libsfb200.so",
]


def _sources():
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC))
            if f.endswith((".cu", ".cuh", ".h"))] + [
        os.path.join(_HERE, "..", "include", "sfb200.h")]


def _digest() -> str:
    h = hashlib.sha256()
    for f in _sources():
        with open(f, "rb") as fh:
            h.update(os.path.basename(f).encode() + b"\0" + fh.read())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def up_to_date() -> bool:
    """The library exists and was built from the current sources (by content:
    copies of the tree onto another machine keep a valid build)."""
    if not os.path.exists(LIB) or not os.path.exists(STAMP):
        return False
    with open(STAMP) as f:
        return f.read().strip() == _digest()


def build_library(force: bool = False, verbose: bool = False) -> str:
    """Compiles csrc/sfb200.cu (the single translation unit) to _lib/libsfb200.so.
    Safe to call from several processes at once: builds are serialised by a
    lock file and each writes its own temporary file."""
    if not force and up_to_date():
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    with open(os.path.join(OUT_DIR, ".build.lock"), "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if not force and up_to_date():          # another process built it meanwhile
            return LIB
        digest = _digest()
        tmp = f"{LIB}.{os.getpid()}.tmp"
        nvcc = os.environ.get("NVCC", "nvcc")
        cmd = [nvcc, *NVCC_FLAGS, os.path.join(CSRC, "sfb200.cu"), "-o", tmp]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("nvcc failed:\n" + r.stdout + r.stderr)
        if verbose:
            sys.stderr.write(r.stderr)
        os.replace(tmp, LIB)
        with open(STAMP, "w") as f:
            f.write(digest + "\n")
    return LIB


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose="-v" in sys.argv))
