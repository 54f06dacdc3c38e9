"""Multi-rank host logic on CPU (world_size 2, gloo backend): batch sharding,
max-over-ranks timing, bitwise digest agreement and shard gathering.  The
per-row computation used here is the fp64 oracle applied row by row, so the
gathered shards must reproduce the single-process result bit for bit."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from batch_invariant_ops import sharding


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n, k, m = 7, 16, 5
        gen = torch.Generator().manual_seed(0)
        x = torch.randn(n, k, generator=gen, dtype=torch.float64)
        w = torch.randn(m, k, generator=gen, dtype=torch.float64)
        start, end = sharding.shard_range(n, world, rank)
        # row-wise product: each row's result depends on that row only
        mine = torch.stack([(x[i] * w).sum(dim=1) for i in range(start, end)])
        full = sharding.gather_rows(mine, n)
        expected = torch.stack([(x[i] * w).sum(dim=1) for i in range(n)])
        t = sharding.max_over_ranks(float(rank + 1))
        agree_same = sharding.ranks_agree(sharding.bit_digest(expected))
        other = expected.clone()
        if rank == 1:
            other[0, 0] = other[0, 0].item() + 1e-3
        agree_diff = sharding.ranks_agree(sharding.bit_digest(other))
        q.put((rank, torch.equal(full, expected), t, agree_same, agree_diff))
    finally:
        dist.destroy_process_group()


def test_shard_range_covers_rows():
    for n in (0, 1, 7, 8, 1000):
        for world in (1, 2, 3, 8):
            spans = [sharding.shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharding.shard_range(4, 2, 2)


def test_bit_digest_detects_one_ulp():
    x = torch.randn(64, dtype=torch.float32)
    y = x.clone()
    y[3] = torch.nextafter(y[3], torch.tensor(float("inf")))
    assert not torch.equal(sharding.bit_digest(x), sharding.bit_digest(y))
    assert torch.equal(sharding.bit_digest(x), sharding.bit_digest(x.clone()))


def test_two_rank_gloo_sharding_round_trip():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, gathered_ok, tmax, agree_same, agree_diff in results:
        assert gathered_ok
        assert tmax == 2.0
        assert agree_same
        assert not agree_diff
