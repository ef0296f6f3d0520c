"""The N-GPU host logic on CPU: row-shard ranges, and barrier / max-over-ranks
across two real processes over gloo (127.0.0.1)."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from ako_b200.sharding import shard_range


@pytest.mark.parametrize("total", [0, 1, 7, 32768, 32769])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_ranges_cover_rows_once(total: int, world: int) -> None:
    ranges = [shard_range(total, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == total
    for (a0, a1), (b0, _) in zip(ranges, ranges[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_rank() -> None:
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    import numpy as np

    import bench
    from ako_b200 import sharding
    from oracle import c_oracle as C

    w, r, _ = sharding.init("gloo", timeout_s=60)
    # Each rank generates only its rows of the seeded global batch (by global
    # row index, as bench.py does on the GPU), runs the fused residual
    # RMSNorm on them with no data exchange (the C oracle stands in for the
    # kernel), and reports a rank-dependent "time"; the job time is the max,
    # the bytes the sum, and the parity check the AND over ranks.
    rows, h = 2500, 64
    lo, hi = sharding.shard_range(rows, w, r)
    x, res = bench.global_rows(lo, hi, h, torch.bfloat16, "cpu", 0)
    wt = bench.weight(h, torch.bfloat16, "cpu", 0)
    host = lambda t: t.view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    y, ro = C.rmsnorm_residual(host(x), host(res), host(wt), 1e-5, "bfloat16", threads=1)
    sharding.barrier()
    job = sharding.max_over_ranks(1.5 + r)
    total = sharding.sum_over_ranks(hi - lo)
    ok = sharding.all_over_ranks(r == 0)
    out.put((r, lo, hi, y, ro, job, total, ok))
    sharding.finish()


def test_two_ranks_over_gloo() -> None:
    """Two ranks each normalize their shard; the concatenation equals the
    unsharded result bit for bit."""
    import numpy as np

    import bench
    from oracle import c_oracle as C

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    got.sort(key=lambda g: g[0])
    assert [g[5] for g in got] == [2.5, 2.5]  # max over ranks
    assert [g[6] for g in got] == [2500, 2500]  # sum over ranks
    assert [g[7] for g in got] == [False, False]  # AND over ranks: rank 1 said False
    assert got[0][1:3] == (0, 1250) and got[1][1:3] == (1250, 2500)
    x, res = bench.global_rows(0, 2500, 64, torch.bfloat16, "cpu", 0)
    wt = bench.weight(64, torch.bfloat16, "cpu", 0)
    host = lambda t: t.view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    y, ro = C.rmsnorm_residual(host(x), host(res), host(wt), 1e-5, "bfloat16")
    np.testing.assert_array_equal(np.concatenate([g[3] for g in got]), y)
    np.testing.assert_array_equal(np.concatenate([g[4] for g in got]), ro)
