"""Multi-rank batch sharding on the CPU (gloo, world size 2): each rank compiles the program for
its shard, runs it through the cuda target's planner (host-side stand-in device), and the gathered
output equals the single-process reference cpu run bit for bit.  A rank that dies before the
gather makes the other rank's collective fail with an error instead of waiting forever."""
import datetime
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, n_global, mode, outdir):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from fake_device import FakeDevice
    from mira_b200 import configs, shard
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    try:
        a, b = shard.shard_bounds(n_global, rank, world)
        prog = configs.compile_w8a8("mlp", b - a, "cuda", calib_batch=4, n_calib=2, executor=FakeDevice())
        x = np.random.default_rng(7).standard_normal((n_global, 784)).astype(np.float32)
        local = prog.run({"x": x[a:b]})
        if mode == "die" and rank == 1:
            os._exit(0)      # leaves between steps, no collective in flight
        try:
            full = shard.gather_rows(local, n_global, world)
            np.save(os.path.join(outdir, f"out{rank}.npy"), full)
        except Exception as e:  # the peer is gone: the collective must fail, not hang
            with open(os.path.join(outdir, f"err{rank}.txt"), "w") as f:
                f.write(type(e).__name__ + ": " + str(e)[:200])
    finally:
        if not (mode == "die" and rank == 1):
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _spawn(mode, n_global, tmp_path):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_global, mode, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    return procs


def test_sharded_batch_matches_single_process(tmp_path):
    sys.path.insert(0, str(ROOT))
    from mira_b200 import configs
    n = 13   # uneven shards: 7 + 6
    procs = _spawn("ok", n, tmp_path)
    assert all(p.exitcode == 0 for p in procs)
    want = configs.compile_w8a8("mlp", n, "cpu", calib_batch=4, n_calib=2).run(
        {"x": np.random.default_rng(7).standard_normal((n, 784)).astype(np.float32)})
    for r in range(2):
        np.testing.assert_array_equal(np.load(tmp_path / f"out{r}.npy"), want)


def test_dead_rank_fails_the_gather_instead_of_hanging(tmp_path):
    _spawn("die", 10, tmp_path)
    assert (tmp_path / "err0.txt").exists(), "rank 0 should have seen the collective fail"


def test_shard_bounds_cover_the_batch():
    sys.path.insert(0, str(ROOT))
    from mira_b200.shard import shard_bounds
    for n in (1, 7, 256, 257):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1
