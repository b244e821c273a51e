"""Multi-rank host logic on CPU: world-size-2 gloo process groups.

The GPU path shards the batch across ranks with no collective on the hot path;
what the ranks share is the measurement plumbing (barrier, max over ranks of
the device times) and the shard arithmetic. These tests run it with the gloo
backend in two processes, and run bench.py's reference arm under torchrun with
two ranks (rank 0 measures and prints, rank 1 exits without work).
"""

import json
import os
import socket
import subprocess
import sys

import pytest
import torch.multiprocessing as mp

from mdlc_b200 import dist as mdist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    d = mdist.from_env(backend="gloo", timeout_s=60)
    try:
        d.barrier()
        got_max = d.max(10.0 + rank)           # per-rank "device time"
        got_sum = d.sum(rank + 1)
        lo, hi = mdist.shard(512, world, rank)
        covered = d.sum(hi - lo)
        import numpy as np
        part = np.full((3, 4), rank, np.float32) + np.arange(12, dtype=np.float32).reshape(3, 4)
        whole = d.gather(part)
        d.barrier()
        out.put((rank, got_max, got_sum, lo, hi, covered, whole.tolist()))
    finally:
        d.close()


def test_gloo_two_ranks_max_and_shards():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    import numpy as np
    base = np.arange(12, dtype=np.float32).reshape(3, 4)
    for rank, got_max, got_sum, lo, hi, covered, whole in res:
        assert got_max == 11.0 and got_sum == 3.0
        assert covered == 512
        # the output gather: every rank's shard, in rank order, on every rank
        np.testing.assert_array_equal(np.asarray(whole, np.float32), np.concatenate([base, base + 1]))
    assert [(r[3], r[4]) for r in res] == [(0, 256), (256, 512)]


def test_shard_rules():
    assert mdist.shard(256, 1, 0) == (0, 256)
    assert mdist.shard(1024, 8, 7) == (896, 1024)
    with pytest.raises(ValueError):
        mdist.shard(10, 4, 0)
    with pytest.raises(ValueError):
        mdist.shard(8, 2, 2)


def test_world_of_one_needs_no_group():
    d = mdist.from_env(backend="gloo")
    assert (d.rank, d.world) == (0, 1)
    assert d.max(3.5) == 3.5 and d.sum(2) == 2.0
    d.barrier()
    d.close()


def test_bench_reference_arm_two_ranks_rank0_only():
    """``bench.py --impl reference`` under torchrun with 2 ranks (gloo on CPU):
    exactly one JSON line, from rank 0, with the reference-arm keys."""
    env = dict(os.environ, OMP_NUM_THREADS="1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}", "bench.py", "--impl", "reference",
           "--gpus", "2", "--steps", "1", "--warmup", "1", "--ref-procs", "2"]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["n_gpus"] == 2 and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"
