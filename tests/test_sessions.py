"""CPU tests of the multi-GPU layer (servoflow_b200/sessions.py): session
sharding, per-session seeds, and the only collectives of the path (barrier and
max over ranks), run as world-size-2 gloo process groups; and the reference
arm of bench.py, which only rank 0 runs."""
import os
import socket
import subprocess
import sys

import pytest
import torch.multiprocessing as mp

from servoflow_b200.sessions import RankInfo, rank_env, session_ids, session_seed

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_shards_are_disjoint_and_cover():
    for world in (1, 2, 4, 8):
        ids = [list(session_ids(world, r, 32)) for r in range(world)]
        flat = [i for part in ids for i in part]
        assert flat == list(range(32 * world))
    assert list(session_ids(2, 1, 1)) == [1]
    for bad in ((0, 0, 1), (2, 2, 1), (2, -1, 1), (2, 0, 0)):
        with pytest.raises(ValueError):
            session_ids(*bad)


def test_seeds_follow_the_session_not_the_world():
    # session 3 gets the same seeds as rank 3 of 8 and as the 4th session of rank 1 of 2
    assert session_seed(session_ids(8, 3, 1)[0], "weights") == session_seed(session_ids(2, 1, 2)[1], "weights")
    seeds = {session_seed(s, k) for s in range(64) for k in ("weights", "inputs", "serving")}
    assert len(seeds) == 3 * 64


def test_rank_env(monkeypatch):
    for k in ("WORLD_SIZE", "RANK", "LOCAL_RANK"):
        monkeypatch.delenv(k, raising=False)
    assert rank_env() == RankInfo(1, 0, 0)
    monkeypatch.setenv("WORLD_SIZE", "4"); monkeypatch.setenv("RANK", "3"); monkeypatch.setenv("LOCAL_RANK", "3")
    assert rank_env() == RankInfo(4, 3, 3)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import torch.distributed as dist
    from servoflow_b200 import sessions
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        info = sessions.rank_env()
        ids = list(sessions.session_ids(info.world, info.rank, 3))
        sessions.barrier()
        # per-rank device-timed statistics; the report is their max over ranks
        stats = sessions.max_over_ranks([float(rank), 5.0 - rank, 2.5, 10.0 * (rank + 1)])
        out.put((rank, ids, stats))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_reduce():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[0] for r in res] == [0, 1]
    assert res[0][1] + res[1][1] == list(range(6))           # disjoint, covering shards
    for _, _, stats in res:
        assert stats == [1.0, 5.0, 2.5, 20.0]                # identical max on every rank


def test_reference_arm_runs_on_rank_zero_only():
    env = dict(os.environ, WORLD_SIZE="2", RANK="1", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "2",
                        "--warmup", "3"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""
