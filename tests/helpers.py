"""Seeded input generators (shapes and distributions of the configs) and
torch <-> numpy bf16 plumbing for the parity tests."""
import numpy as np


def rng(seed):
    return np.random.default_rng(seed)


def bf16_np(x):
    """float32 array rounded to bf16 (RNE), kept as float32."""
    import oracle
    return oracle.bf16_round(np.ascontiguousarray(x, np.float32))


def f16_np(x):
    """float32 array rounded to IEEE half (RNE), kept as float32."""
    return np.ascontiguousarray(x, np.float32).astype(np.float16).astype(np.float32)


def to_dev(x, dtype="bf16"):
    """numpy float32 -> CUDA tensor (bf16 / f16 keep the exact RNE-rounded bits)."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x, np.float32))
    if dtype == "bf16":
        t = t.to(torch.bfloat16)
    elif dtype == "f16":
        t = t.to(torch.float16)
    return t.cuda()


def to_np(t):
    import torch
    return t.detach().to(torch.float32).cpu().numpy()


def gemm_inputs(M, N, K, seed=0, bias=True):
    """Config C2 distributions: A, W ~ U(-1,1)/sqrt(K) (bf16), bias ~ N(0, 0.02)."""
    g = rng(seed)
    s = 1.0 / np.sqrt(K)
    A = bf16_np(g.uniform(-1, 1, (M, K)).astype(np.float32) * s)
    W = bf16_np(g.uniform(-1, 1, (K, N)).astype(np.float32) * s)
    b = (g.standard_normal(N) * 0.02).astype(np.float32) if bias else None
    return A, W, b


def attn_inputs(B, Hq, Hkv, S, D, seed=0, bf16=True):
    """Q, K, V iid N(0,1)."""
    g = rng(seed)
    Q = g.standard_normal((B, Hq, S, D), dtype=np.float32)
    K = g.standard_normal((B, Hkv, S, D), dtype=np.float32)
    V = g.standard_normal((B, Hkv, S, D), dtype=np.float32)
    if bf16:
        Q, K, V = bf16_np(Q), bf16_np(K), bf16_np(V)
    return Q, K, V


_KEEP = []


def arg_buffer(nbytes=1 << 20):
    """Pointer for argument-validation tests, whose calls must fail before
    any kernel runs.  With a GPU present it is a real device allocation of
    nbytes (kept alive for the session), so that a validation regression
    would launch on valid memory instead of a made-up address; without one
    the library cannot launch anything and a placeholder address is used."""
    import ctypes
    try:
        import torch
        gpu = torch.cuda.is_available()
    except Exception:
        gpu = False
    if not gpu:
        return ctypes.c_void_p(256)
    t = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device="cuda")
    _KEEP.append(t)
    return ctypes.c_void_p(t.data_ptr())
