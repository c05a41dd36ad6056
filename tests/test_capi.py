"""CPU checks of the C ABI: the library loads, exports every function that
include/sfb200.h declares, and its host-only helpers behave. No kernel is
launched here."""
import ctypes
import os
import re
import subprocess

from servoflow_b200 import _capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for f in os.listdir(os.path.join(ROOT, "include")):
        if f.endswith(".h"):
            src = open(os.path.join(ROOT, "include", f)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(sfb_\w+)\s*\(", src))
    return sorted(names)


def test_header_declares_the_boundary():
    names = declared_functions()
    for n in ("sfb_attention_fwd", "sfb_attention_bhsd", "sfb_dequantize_int8", "sfb_device_error",
              "sfb_status_string", "sfb_version"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = _capi.lib()
    for n in declared_functions():
        assert hasattr(lib, n), f"{n} declared in include/ but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", _capi.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (sfb_\w+)", out))
    assert set(declared_functions()) <= exported


def test_status_strings_and_version():
    assert _capi.status_string(0) == "ok"
    assert "16-byte" in _capi.status_string(_capi.SFB_ERR_ALIGN)
    assert _capi.status_string(12345) == "unknown status"
    assert _capi.lib().sfb_version().decode().endswith("sm_100a")


def test_args_struct_layout_matches_header():
    # offsets of sfb_attn_args as laid out by the C compiler
    src = r'''
#include <stddef.h>
#include <stdio.h>
#include "sfb200.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu %zu\n", offsetof(sfb_attn_args, q_stride), offsetof(sfb_attn_args, batch),
         offsetof(sfb_attn_args, scale), offsetof(sfb_attn_args, key_mask_stride_b),
         offsetof(sfb_attn_args, attn_mask), offsetof(sfb_attn_args, attn_mask_stride),
         sizeof(sfb_attn_args));
  return 0;
}
'''
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        open(c, "w").write(src)
        exe = os.path.join(d, "t")
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        got = list(map(int, subprocess.run([exe], capture_output=True, text=True).stdout.split()))
    A = _capi.AttnArgs
    want = [A.q_stride.offset, A.batch.offset, A.scale.offset, A.key_mask_stride_b.offset,
            A.attn_mask.offset, A.attn_mask_stride.offset, ctypes.sizeof(A)]
    assert got == want


def _c_offsets(struct: str, fields):
    """Offsets of `fields` and the size of `struct` as the C compiler lays them out."""
    import tempfile
    prints = ", ".join(f"offsetof({struct}, {f})" for f in fields)
    src = ("#include <stddef.h>\n#include <stdio.h>\n#include \"sfb200.h\"\n"
           f"int main(void) {{ printf(\"{'%zu ' * (len(fields) + 1)}\\n\", {prints}, sizeof({struct})); "
           "return 0; }\n")
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        open(c, "w").write(src)
        exe = os.path.join(d, "t")
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        return list(map(int, subprocess.run([exe], capture_output=True, text=True).stdout.split()))


def test_model_config_structs_match_header():
    """The ctypes mirrors of sfb_rdt1b_config and sfb_octo_config have the C layout."""
    from servoflow_b200.octo import OctoConfig
    from servoflow_b200.rdt1b import RDT1BConfig
    for struct, py in (("sfb_rdt1b_config", RDT1BConfig), ("sfb_octo_config", OctoConfig)):
        fields = [f for f, _ in py._fields_]
        want = [getattr(py, f).offset for f in fields] + [ctypes.sizeof(py)]
        assert _c_offsets(struct, fields) == want, struct


def test_null_args_rejected_without_device():
    # argument validation runs before any CUDA call
    assert _capi.lib().sfb_attention_fwd(None, None) == _capi.SFB_ERR_INVALID
    assert _capi.lib().sfb_dequantize_int8(None, None, 1, 1, None, 1, 0, 0, None) == _capi.SFB_OK
    assert _capi.lib().sfb_dequantize_int8(None, None, 1, 1, None, 1, 2, 2, None) == \
        _capi.SFB_ERR_INVALID


def test_model_api_argument_checks_without_a_gpu():
    """The RDT-1B entry points reject bad arguments before touching a device
    (the same statuses a servoflow binding turns into exceptions)."""
    from servoflow_b200.rdt1b import RDT1BConfig, _declare, default_config
    lib = _capi.lib()
    _declare(lib)
    h = ctypes.c_void_p()
    cfg = default_config()
    assert lib.sfb_rdt1b_create(None, 0, ctypes.byref(h)) == _capi.SFB_ERR_INVALID
    assert lib.sfb_rdt1b_create(ctypes.byref(cfg), 0, None) == _capi.SFB_ERR_INVALID
    for bad in (dict(hidden=2000), dict(heads=31), dict(num_layers=0), dict(max_sessions=0),
                dict(num_steps=0), dict(num_steps=65), dict(action_dim=100), dict(lang_dim=100),
                dict(state_dim=64)):
        c = default_config(**bad)
        assert lib.sfb_rdt1b_create(ctypes.byref(c), 0, ctypes.byref(h)) == _capi.SFB_ERR_SHAPE, bad
    x = ctypes.c_void_p(1)
    assert lib.sfb_rdt1b_encode(None, 1, x, x, x, x, None) == _capi.SFB_ERR_INVALID
    assert lib.sfb_rdt1b_forward(None, 1, x, 0.0, x, None) == _capi.SFB_ERR_INVALID
    assert lib.sfb_rdt1b_sample(None, 1, x, x, 1, None) == _capi.SFB_ERR_INVALID
    assert lib.sfb_rdt1b_destroy(None) == _capi.SFB_ERR_INVALID
    n = ctypes.c_int64()
    assert lib.sfb_rdt1b_graph_kernels(None, 1, ctypes.byref(n)) == _capi.SFB_ERR_INVALID
    assert lib.sfb_rdt1b_schedule(None, None, None, None, None, 5) == _capi.SFB_ERR_INVALID
    n32 = ctypes.c_int32()
    assert lib.sfb_rdt1b_profile_dense(None, 999.0, 0, ctypes.byref(n32), None, None, None) == _capi.SFB_ERR_INVALID
