"""Sharding / gather logic on world_size-2 gloo CPU ranks.  The compute step
is a CPU stand-in (the partition and the gather are what is tested); the GPU
kernels themselves are covered by the -m gpu tests."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from jules_b200 import shard


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_row_range_partition():
    for total in (0, 1, 7, 4096, 4097):
        for world in (1, 2, 3, 8):
            ranges = [shard.row_range(total, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            for (a, b), (c, d) in zip(ranges, ranges[1:]):
                assert b == c
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1


def _ref_attention(Q, K, V, causal):
    B, Hq, S, D = Q.shape
    g = Hq // K.shape[1]
    Kr = K.repeat_interleave(g, dim=1)
    Vr = V.repeat_interleave(g, dim=1)
    s = Q @ Kr.transpose(-1, -2) / D ** 0.5
    if causal:
        s = s + torch.triu(torch.full((S, S), float("-inf")), 1)
    return torch.softmax(s, -1) @ Vr


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        # rows (fused GEMM / MLP block): GELU(X W + b)
        X = torch.randn(37, 16)
        W = torch.randn(16, 24)
        b = torch.randn(24)
        fn = lambda x: torch.nn.functional.gelu(x @ W + b, approximate="tanh")
        full = shard.sharded_rows(fn, X, rank, world, dist)
        ok_rows = torch.allclose(full, fn(X), atol=1e-5)
        # attention units with grouped-query heads
        Q = torch.randn(3, 8, 20, 16)
        K = torch.randn(3, 2, 20, 16)
        V = torch.randn(3, 2, 20, 16)
        att = lambda q, k, v: _ref_attention(q, k, v, True)
        O = shard.sharded_attention(att, Q, K, V, rank, world, dist)
        ok_attn = torch.allclose(O, _ref_attention(Q, K, V, True), atol=1e-5)
        q.put((rank, bool(ok_rows), bool(ok_attn)))
    finally:
        dist.destroy_process_group()


def test_sharded_gather_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert res == [(0, True, True), (1, True, True)]


def test_rank_failure_is_reported():
    """A rank that dies before the collective: the survivor's gather fails
    with an error (short process-group timeout) instead of hanging."""
    ctx = mp.get_context("spawn")
    port = _free_port()
    q = ctx.Queue()
    procs = [ctx.Process(target=_dying_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert procs[1].exitcode != 0
    res = q.get(timeout=10)
    assert res[0] == 0 and res[1] == "error"


def _dying_worker(rank, port, q):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # leaves between steps, before the gather
    try:
        shard.sharded_rows(lambda x: x * 2, torch.ones(8, 4), rank, 2, dist)
        q.put((rank, "no error"))
    except Exception:
        q.put((rank, "error"))
