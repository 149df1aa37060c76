"""Multi-GPU sharding of the hot path (one process per GPU).

The work splits into independent units with no exchange on the data path:
token rows for the fused GEMM / MLP block, (batch, kv-head group) units for
attention (each unit is one kv head and the Hq/Hkv query heads that read it,
contiguous in [B, H, S, D] memory).  Each rank computes its slice with the
CUDA kernels; the only collective is the output gather (NCCL all-gather over
NVLink on GPUs, gloo on CPU).

The compute step is a parameter so the partition/gather logic can be tested
on CPU ranks.
"""
from __future__ import annotations


def row_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Balanced contiguous [start, stop) of `total` rows for `rank`."""
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def attention_units(B: int, Hq: int, Hkv: int) -> int:
    """Number of (batch, kv-head group) units."""
    assert Hq % Hkv == 0
    return B * Hkv


def _gather_rows(local, total_rows: int, rank: int, world: int, dist, group=None):
    """All-gather row slices of sizes given by row_range into [total_rows, ...]."""
    import torch
    sizes = [row_range(total_rows, r, world) for r in range(world)]
    maxn = max(b - a for a, b in sizes)
    pad = torch.zeros((maxn,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([parts[r][: b - a] for r, (a, b) in enumerate(sizes)], dim=0)


def sharded_rows(fn, X, rank: int, world: int, dist=None, gather: bool = True, group=None):
    """Apply a row-wise op (fused GEMM, MLP block, LayerNorm) to this rank's
    rows of X; optionally all-gather the full result."""
    a, b = row_range(X.shape[0], rank, world)
    local = fn(X[a:b].contiguous())
    if not gather or world == 1:
        return local
    return _gather_rows(local, X.shape[0], rank, world, dist, group)


def sharded_attention(fn, Q, K, V, rank: int, world: int, dist=None, gather: bool = True,
                      group=None):
    """Causal/non-causal attention over this rank's (batch, kv-group) units.

    fn(Qs, Ks, Vs) computes attention for views shaped [units, Hq/Hkv, S, D]
    (queries) and [units, 1, S, D] (keys/values); returns O shaped like Qs.
    The gathered result has Q's shape."""
    B, Hq, S, D = Q.shape
    Hkv = K.shape[1]
    grp = Hq // Hkv
    n = attention_units(B, Hq, Hkv)
    a, b = row_range(n, rank, world)
    Qu = Q.reshape(n, grp, S, D)[a:b]
    Ku = K.reshape(n, 1, S, D)[a:b]
    Vu = V.reshape(n, 1, S, D)[a:b]
    Ou = fn(Qu, Ku, Vu)
    if not gather or world == 1:
        return Ou
    return _gather_rows(Ou, n, rank, world, dist, group).reshape(B, Hq, S, D)
