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
    from ako_b200 import sharding
    from ako_b200.reference import ops

    w, r, _ = sharding.init("gloo", timeout_s=60)
    # Each rank normalizes its own block of a global batch, with no data
    # exchange, and reports a rank-dependent "time"; the job time is the max.
    g = torch.Generator().manual_seed(0)
    x = torch.randn(10, 64, generator=g)
    wt = torch.randn(64, generator=g)
    lo, hi = sharding.shard_range(x.shape[0], w, r)
    local = ops().rmsnorm_ref(x[lo:hi], wt)
    sharding.barrier()
    job = sharding.max_over_ranks(1.5 + r)
    out.put((r, lo, hi, local, job))
    sharding.finish()


def test_two_ranks_over_gloo() -> None:
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
    got.sort()
    assert [g[4] for g in got] == [2.5, 2.5]
    from ako_b200.reference import ops

    g = torch.Generator().manual_seed(0)
    x = torch.randn(10, 64, generator=g)
    wt = torch.randn(64, generator=g)
    whole = torch.cat([g_[3] for g_ in got])
    assert torch.equal(whole, ops().rmsnorm_ref(x, wt)) or torch.allclose(whole, ops().rmsnorm_ref(x, wt), atol=1e-6)
    assert got[0][1:3] == (0, 5) and got[1][1:3] == (5, 10)
