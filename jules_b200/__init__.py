"""jules_b200 - B200 (sm_100a) implementation of the Jules fused-kernel layer.

The product is the shared library ``jules_b200/_lib/libjules_b200.so``
(C ABI in ``include/jules_kernels.h``, reference-signature C++ API in
``include/jules/Kernel/*.h``).  This module loads it with ctypes and offers
thin torch-tensor wrappers (device memory and streams come from torch; the
arithmetic is the library's CUDA kernels).

There is no CPU fallback: if the library is missing or no GPU is present the
calls raise.
"""
from __future__ import annotations

import ctypes
import os

__all__ = [
    "lib", "JulesError", "ACT", "gemm_bias_act", "flash_attention_fwd", "layernorm", "gelu",
    "mlp_block", "mlp_block_workspace_bytes", "sgemm", "device_error", "kernel_by_name",
    "kernel_names", "LIB_PATH", "gemm_fp8", "cast", "matmul_int8", "softmax",
    "cross_entropy_loss", "custom_call", "mlp_fwd_bwd", "flash_attention_bwd", "attention",
    "Dist", "mlp_block_fold_weights", "mlp_block_folded",
]

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libjules_b200.so")

ACT = {"none": 0, "relu": 1, "sigmoid": 2, "tanh": 3, "gelu": 4}
DT_F32, DT_BF16, DT_FP8E4M3, DT_FP8E5M2, DT_F16 = 0, 1, 2, 3, 4

_c_vp = ctypes.c_void_p
_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_c_f = ctypes.c_float

_SIGNATURES = {
    "jules_version": ([], _c_int),
    "jules_last_error_string": ([], ctypes.c_char_p),
    "jules_status_string": ([_c_int], ctypes.c_char_p),
    "jules_device_error": ([ctypes.POINTER(ctypes.c_uint32), _c_int], _c_int),
    "jules_selftest_bounded_wait": ([ctypes.c_uint64, _c_vp], _c_int),
    "jules_gemm_f32_tc_workspace_bytes": ([_c_i64, _c_i64, _c_i64], ctypes.c_size_t),
    "jules_gemm_f32_tc": ([_c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_int, _c_vp,
                           ctypes.c_size_t, _c_vp], _c_int),
    "jules_gemm_bias_act": ([_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_int,
                             _c_int, _c_int, _c_vp], _c_int),
    "jules_sgemm": ([_c_int, _c_int, _c_i64, _c_i64, _c_i64, _c_f, _c_vp, _c_i64, _c_vp, _c_i64,
                     _c_f, _c_vp, _c_i64, _c_vp], _c_int),
    "jules_flash_attention_bwd_workspace_bytes": ([_c_int] * 5, ctypes.c_size_t),
    "jules_flash_attention_bwd": ([_c_vp] * 9 + [_c_int] * 5 + [_c_f, _c_int, _c_int, _c_vp,
                                                               ctypes.c_size_t, _c_vp], _c_int),
    "jules_flash_attention_fwd": ([_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int,
                                   _c_int, _c_int, _c_f, _c_int, _c_int, _c_vp], _c_int),
    "jules_layernorm": ([_c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_f, _c_int, _c_int, _c_vp,
                         _c_vp, _c_vp], _c_int),
    "jules_gelu": ([_c_vp, _c_vp, _c_i64, _c_int, _c_vp], _c_int),
    "jules_softmax": ([_c_vp, _c_vp, _c_i64, _c_i64, _c_int, _c_int, _c_vp], _c_int),
    "jules_mlp_fwd_bwd_workspace_bytes": ([_c_i64, _c_i64, _c_i64], ctypes.c_size_t),
    "jules_mlp_fwd_bwd": ([_c_vp] * 13 + [_c_i64] * 4 + [_c_vp, ctypes.c_size_t, _c_vp], _c_int),
    "jules_matmul_int8": ([_c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_f, _c_f, _c_vp, _c_vp],
                          _c_int),
    "jules_gemm_fp8": ([_c_vp] * 5 + [_c_i64] * 3 + [_c_f] + [_c_int] * 4 + [_c_vp], _c_int),
    "jules_cast": ([_c_vp, _c_vp, _c_i64, _c_int, _c_int, _c_vp], _c_int),
    "jules_cross_entropy_loss": ([_c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_int, _c_vp],
                                 _c_int),
    "jules_mlp_block_workspace_bytes": ([_c_i64, _c_i64, _c_i64], ctypes.c_size_t),
    "jules_mlp_block": ([_c_vp] * 8 + [_c_int, _c_i64, _c_i64, _c_i64, _c_f, _c_vp,
                                       ctypes.c_size_t, _c_vp], _c_int),
    "jules_custom_call": ([ctypes.c_char_p, _c_vp, ctypes.POINTER(_c_vp), _c_int, _c_vp,
                           ctypes.c_size_t], _c_int),
    "jules_kernel_by_name": ([ctypes.c_char_p], _c_int),
    "jules_kernel_name": ([_c_int], ctypes.c_char_p),
    "jules_kernel_count": ([], _c_int),
    "jules_kernel_implemented": ([_c_int], _c_int),
    "jules_mlp_block_fold_weights": ([_c_vp] * 7 + [_c_i64, _c_i64, _c_vp], _c_int),
    "jules_mlp_block_folded_workspace_bytes": ([_c_i64, _c_i64, _c_i64], ctypes.c_size_t),
    "jules_mlp_block_folded": ([_c_vp] * 7 + [_c_int, _c_i64, _c_i64, _c_i64, _c_f, _c_vp,
                                              ctypes.c_size_t, _c_vp], _c_int),
    "jules_dist_shard": ([_c_i64, _c_int, _c_int, ctypes.POINTER(_c_i64), ctypes.POINTER(_c_i64)],
                         _c_int),
    "jules_dist_unique_id": ([_c_vp], _c_int),
    "jules_dist_init": ([ctypes.POINTER(_c_vp), _c_int, _c_int, _c_vp], _c_int),
    "jules_dist_destroy": ([_c_vp], _c_int),
    "jules_dist_barrier": ([_c_vp, _c_vp], _c_int),
    "jules_dist_multicast": ([_c_vp, ctypes.POINTER(_c_int)], _c_int),
    "jules_dist_gather_route": ([_c_vp, ctypes.c_size_t, ctypes.POINTER(_c_int)], _c_int),
    "jules_dist_alloc_shared": ([_c_vp, ctypes.c_size_t, ctypes.POINTER(_c_vp)], _c_int),
    "jules_dist_free_shared": ([_c_vp, _c_vp], _c_int),
    "jules_dist_gemm_bias_act": ([_c_vp] * 6 + [_c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int,
                                                _c_vp], _c_int),
    "jules_dist_flash_attention_fwd": ([_c_vp] * 6 + [_c_int] * 5 + [_c_f, _c_int, _c_int, _c_vp],
                                       _c_int),
}


class CallDesc(ctypes.Structure):
    """jules_call_desc (include/jules_kernels.h): shapes and scalars of a
    custom call, passed as the opaque bytes."""
    _fields_ = [("dims", ctypes.c_int64 * 6), ("fparams", ctypes.c_float * 2),
                ("dtype", ctypes.c_int32), ("flags", ctypes.c_int32)]


class JulesError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(what)


_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} missing: build it with `python -m jules_b200.build`")
        h = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(h, name)
            fn.argtypes = args
            fn.restype = res
        _lib = h
    return _lib


def _check(rc: int, what: str) -> None:
    if rc != 0:
        h = lib()
        raise JulesError(rc, f"{what}: {h.jules_status_string(rc).decode()}: "
                             f"{h.jules_last_error_string().decode()}")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _dtype_code(t) -> int:
    import torch
    if t.dtype == torch.float32:
        return DT_F32
    if t.dtype == torch.bfloat16:
        return DT_BF16
    if t.dtype == torch.float16:
        return DT_F16
    if t.dtype == torch.float8_e4m3fn:
        return DT_FP8E4M3
    if t.dtype == torch.float8_e5m2:
        return DT_FP8E5M2
    raise TypeError(f"unsupported dtype {t.dtype}")


def _stream(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _dense(t, name):
    if not t.is_cuda or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous CUDA tensor")
    return t


def device_error(clear: bool = True) -> int:
    """Synchronise and return the device error word (0 = no error)."""
    w = ctypes.c_uint32(0)
    lib().jules_device_error(ctypes.byref(w), 1 if clear else 0)
    return int(w.value)


def gemm_bias_act(A, W, bias=None, residual=None, act="none", out=None, out_dtype=None,
                  stream=None):
    """C = act(A @ W + bias) (+ residual); A [M,K], W [K,N] (same dtype: fp32,
    bf16, or an fp8 type with a bf16 residual and bf16 C by default)."""
    import torch
    _dense(A, "A"), _dense(W, "W")
    M, K = A.shape
    K2, N = W.shape
    if K2 != K or W.dtype != A.dtype:
        raise ValueError("A/W shape or dtype mismatch")
    fp8 = A.dtype in (torch.float8_e4m3fn, torch.float8_e5m2)
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype or (torch.bfloat16 if fp8 else A.dtype),
                          device=A.device)
    if bias is not None:
        _dense(bias, "bias")
        if bias.dtype != torch.float32 or bias.numel() != N:
            raise ValueError("bias must be fp32 with N elements")
    if residual is not None:
        _dense(residual, "residual")
        if residual.dtype != (torch.bfloat16 if fp8 else A.dtype) or residual.shape != out.shape:
            raise ValueError("residual must have A's dtype (bf16 for fp8 A) and C's shape")
    rc = lib().jules_gemm_bias_act(_ptr(A), _ptr(W), _ptr(bias), _ptr(residual), _ptr(out), M, N,
                                   K, ACT[act] if isinstance(act, str) else int(act),
                                   _dtype_code(A), _dtype_code(out), _stream(stream))
    _check(rc, "jules_gemm_bias_act")
    return out


def gemm_f32_tc(A, W, bias=None, act="none", out=None, workspace=None, stream=None):
    """fp32 C = act(A @ W + bias) on tensor cores with fp32-level accuracy
    (3xTF32, jules_gemm_f32_tc).  workspace: a uint8 CUDA tensor of at least
    gemm_f32_tc_workspace_bytes(M, N, K) bytes (allocated here if None)."""
    import torch
    _dense(A, "A"), _dense(W, "W")
    M, K = A.shape
    K2, N = W.shape
    if K2 != K or A.dtype != torch.float32 or W.dtype != torch.float32:
        raise ValueError("A [M,K] and W [K,N] must be fp32")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=A.device)
    if bias is not None:
        _dense(bias, "bias")
        if bias.dtype != torch.float32 or bias.numel() != N:
            raise ValueError("bias must be fp32 with N elements")
    need = gemm_f32_tc_workspace_bytes(M, N, K)
    if workspace is None:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=A.device)
    rc = lib().jules_gemm_f32_tc(_ptr(A), _ptr(W), _ptr(bias), _ptr(out), M, N, K,
                                 ACT[act] if isinstance(act, str) else int(act), _ptr(workspace),
                                 workspace.numel() * workspace.element_size(), _stream(stream))
    _check(rc, "jules_gemm_f32_tc")
    return out


def gemm_f32_tc_workspace_bytes(M, N, K):
    return int(lib().jules_gemm_f32_tc_workspace_bytes(M, N, K))


def sgemm(A, B, C=None, alpha=1.0, beta=0.0, transA=False, transB=False, stream=None):
    """Row-major fp32 C = alpha op(A) op(B) + beta C."""
    import torch
    M = A.shape[1] if transA else A.shape[0]
    K = A.shape[0] if transA else A.shape[1]
    N = B.shape[0] if transB else B.shape[1]
    if C is None:
        C = torch.zeros((M, N), dtype=torch.float32, device=A.device)
    rc = lib().jules_sgemm(int(transA), int(transB), M, N, K, alpha, _ptr(A), A.shape[1], _ptr(B),
                           B.shape[1], beta, _ptr(C), C.shape[1], _stream(stream))
    _check(rc, "jules_sgemm")
    return C


def flash_attention_fwd(Q, K, V, causal=False, scale=0.0, out=None, lse=True, stream=None):
    """Q [B,Hq,S,D], K/V [B,Hkv,S,D] (fp32 or bf16).  Returns (O, lse|None)."""
    import torch
    for t, n in ((Q, "Q"), (K, "K"), (V, "V")):
        _dense(t, n)
    B, Hq, S, D = Q.shape
    Hkv = K.shape[1]
    if out is None:
        out = torch.empty_like(Q)
    l = torch.empty((B, Hq, S), dtype=torch.float32, device=Q.device) if lse else None
    rc = lib().jules_flash_attention_fwd(_ptr(Q), _ptr(K), _ptr(V), _ptr(out), _ptr(l), B, Hq, Hkv,
                                         S, D, float(scale), int(bool(causal)), _dtype_code(Q),
                                         _stream(stream))
    _check(rc, "jules_flash_attention_fwd")
    return out, l


def flash_attention_bwd(Q, K, V, O, dO, lse, causal=False, scale=0.0, workspace=None,
                        out=None, stream=None):
    """Gradients (dQ, dK, dV) of flash_attention_fwd for dO, from its O and
    lse.  Q, O, dO [B,Hq,S,D]; K, V [B,Hkv,S,D]; one dtype (fp32 or bf16);
    lse [B,Hq,S] fp32.  out: optional (dQ, dK, dV) tensors."""
    import torch
    for t, n in ((Q, "Q"), (K, "K"), (V, "V"), (O, "O"), (dO, "dO"), (lse, "lse")):
        _dense(t, n)
    B, Hq, S, D = Q.shape
    Hkv = K.shape[1]
    dt = _dtype_code(Q)
    if any(t.dtype != Q.dtype for t in (K, V, O, dO)) or lse.dtype != torch.float32:
        raise ValueError("flash_attention_bwd: Q, K, V, O, dO share one dtype; lse is fp32")
    dQ, dK, dV = out if out is not None else (torch.empty_like(Q), torch.empty_like(K),
                                              torch.empty_like(V))
    need = lib().jules_flash_attention_bwd_workspace_bytes(B, Hq, S, D, dt)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=Q.device)
    rc = lib().jules_flash_attention_bwd(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), _ptr(dO), _ptr(lse),
                                         _ptr(dQ), _ptr(dK), _ptr(dV), B, Hq, Hkv, S, D,
                                         float(scale), int(bool(causal)), dt, _ptr(workspace),
                                         workspace.numel() * workspace.element_size(),
                                         _stream(stream))
    _check(rc, "jules_flash_attention_bwd")
    return dQ, dK, dV


def attention(Q, K, V, causal=False, scale=0.0):
    """Differentiable attention: forward jules_flash_attention_fwd, backward
    jules_flash_attention_bwd (torch.autograd.Function)."""
    return _attention_fn().apply(Q, K, V, bool(causal), float(scale))


_ATTN_FN = None


def _attention_fn():
    global _ATTN_FN
    if _ATTN_FN is None:
        import torch

        class _Attention(torch.autograd.Function):
            @staticmethod
            def forward(ctx, Q, K, V, causal, scale):
                Q, K, V = Q.contiguous(), K.contiguous(), V.contiguous()
                O, lse = flash_attention_fwd(Q, K, V, causal=causal, scale=scale)
                ctx.save_for_backward(Q, K, V, O, lse)
                ctx.causal, ctx.scale = causal, scale
                return O

            @staticmethod
            def backward(ctx, dO):
                Q, K, V, O, lse = ctx.saved_tensors
                dQ, dK, dV = flash_attention_bwd(Q, K, V, O, dO.contiguous(), lse,
                                                 causal=ctx.causal, scale=ctx.scale)
                return dQ, dK, dV, None, None

        _ATTN_FN = _Attention
    return _ATTN_FN


def layernorm(x, gamma, beta, eps=1e-5, out=None, out_dtype=None, stats=False, stream=None):
    import torch
    _dense(x, "x")
    M, N = x.shape
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype or x.dtype, device=x.device)
    mean = torch.empty(M, dtype=torch.float32, device=x.device) if stats else None
    rstd = torch.empty(M, dtype=torch.float32, device=x.device) if stats else None
    rc = lib().jules_layernorm(_ptr(x), _ptr(gamma), _ptr(beta), _ptr(out), M, N, float(eps),
                               _dtype_code(x), _dtype_code(out), _ptr(mean), _ptr(rstd),
                               _stream(stream))
    _check(rc, "jules_layernorm")
    return (out, mean, rstd) if stats else out


def gelu(x, out=None, stream=None):
    import torch
    _dense(x, "x")
    if out is None:
        out = torch.empty_like(x)
    rc = lib().jules_gelu(_ptr(x), _ptr(out), x.numel(), _dtype_code(x), _stream(stream))
    _check(rc, "jules_gelu")
    return out


def mlp_fwd_bwd(X, W1, b1, W2, b2, targets, want_dx=True, workspace=None, stream=None):
    """2-layer ReLU MLP training step in fp32 (the reference's
    interleavedMLPForwardBackward): returns dict(loss (0-d device tensor),
    out, dW1, db1, dW2, db2, dX)."""
    import torch
    M, K1 = X.shape
    N1, N2 = W1.shape[1], W2.shape[1]
    dev = X.device
    e = lambda *s: torch.empty(s, dtype=torch.float32, device=dev)
    r = dict(out=e(M, N2), loss=e(), dW1=e(K1, N1), db1=e(N1), dW2=e(N1, N2), db2=e(N2),
             dX=e(M, K1) if want_dx else None)
    need = int(lib().jules_mlp_fwd_bwd_workspace_bytes(M, N1, N2))
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    rc = lib().jules_mlp_fwd_bwd(_ptr(X), _ptr(W1), _ptr(b1), _ptr(W2), _ptr(b2), _ptr(targets),
                                 _ptr(r["out"]), _ptr(r["loss"]), _ptr(r["dW1"]), _ptr(r["db1"]),
                                 _ptr(r["dW2"]), _ptr(r["db2"]), _ptr(r["dX"]), M, K1, N1, N2,
                                 _ptr(workspace), workspace.numel(), _stream(stream))
    _check(rc, "jules_mlp_fwd_bwd")
    return r


def matmul_int8(A, B, scale_a=1.0, scale_b=1.0, bias=None, out=None, stream=None):
    """C = float(A @ B) * scale_a * scale_b (+ bias); A [M,K], B [K,N] int8,
    int32 accumulation, fp32 C."""
    import torch
    for t, n in ((A, "A"), (B, "B")):
        _dense(t, n)
        if t.dtype != torch.int8:
            raise ValueError(f"matmul_int8: {n} must be int8")
    M, K = A.shape
    N = B.shape[1]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=A.device)
    rc = lib().jules_matmul_int8(_ptr(A), _ptr(B), _ptr(out), M, N, K, scale_a, scale_b,
                                 _ptr(bias), _stream(stream))
    _check(rc, "jules_matmul_int8")
    return out


def gemm_fp8(A, W, bias=None, residual=None, act="none", scale=1.0, out=None, out_dtype=None,
             stream=None):
    """C = act((A @ W) * scale + bias) (+ residual); A [M,K], W [K,N] in
    torch.float8_e4m3fn / float8_e5m2 (each its own), fp32 accumulation;
    residual bf16; C bf16 (default) or fp32."""
    import torch
    _dense(A, "A"), _dense(W, "W")
    M, K = A.shape
    K2, N = W.shape
    if K2 != K:
        raise ValueError("gemm_fp8: A/W shape mismatch")
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype or torch.bfloat16, device=A.device)
    if bias is not None:
        _dense(bias, "bias")
        if bias.dtype != torch.float32 or bias.numel() != N:
            raise ValueError("bias must be fp32 with N elements")
    if residual is not None:
        _dense(residual, "residual")
        if residual.dtype != torch.bfloat16 or residual.shape != out.shape:
            raise ValueError("residual must be bf16 with C's shape")
    rc = lib().jules_gemm_fp8(_ptr(A), _ptr(W), _ptr(bias), _ptr(residual), _ptr(out), M, N, K,
                              float(scale), ACT[act] if isinstance(act, str) else int(act),
                              _dtype_code(A), _dtype_code(W), _dtype_code(out), _stream(stream))
    _check(rc, "jules_gemm_fp8")
    return out


def cast(x, dtype, out=None, stream=None):
    """Element type conversion among fp32, bf16, float8_e4m3fn and
    float8_e5m2 (to fp8: round to nearest even, saturating to the largest
    finite value)."""
    import torch
    _dense(x, "x")
    if out is None:
        out = torch.empty(x.shape, dtype=dtype, device=x.device)
    elif out.numel() != x.numel():
        raise ValueError("cast: out must have x's size")
    rc = lib().jules_cast(_ptr(x), _ptr(out), x.numel(), _dtype_code(x), _dtype_code(out),
                          _stream(stream))
    _check(rc, "jules_cast")
    return out


def softmax(x, out=None, out_dtype=None, stream=None):
    """Row softmax of a 2-D tensor (fp32 or bf16; fp32 arithmetic)."""
    import torch
    _dense(x, "x")
    if x.dim() != 2:
        raise ValueError("softmax: x must be 2-D [M, N]")
    if out is None:
        out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    M, N = x.shape
    rc = lib().jules_softmax(_ptr(x), _ptr(out), M, N, _dtype_code(x), _dtype_code(out),
                             _stream(stream))
    _check(rc, "jules_softmax")
    return out


def cross_entropy_loss(logits, targets, grad=True, stream=None):
    """Fused softmax + cross-entropy.  Returns (loss as a 0-d fp32 device
    tensor, grad [M, N] in the logits' dtype or None)."""
    import torch
    _dense(logits, "logits")
    if logits.dim() != 2:
        raise ValueError("cross_entropy_loss: logits must be 2-D [M, N]")
    if targets.dtype != torch.int32 or not targets.is_contiguous():
        raise ValueError("cross_entropy_loss: targets must be contiguous int32")
    M, N = logits.shape
    g = torch.empty_like(logits) if grad else None
    loss = torch.empty((), dtype=torch.float32, device=logits.device)
    rc = lib().jules_cross_entropy_loss(_ptr(logits), _ptr(targets), _ptr(g) if g is not None else None,
                                        _ptr(loss), M, N, _dtype_code(logits), _stream(stream))
    _check(rc, "jules_cross_entropy_loss")
    return loss, g


def custom_call(name, buffers, dims=(), fparams=(), dtype=DT_BF16, flags=0, stream=None, check=True):
    """Run a registered kernel the way a runtime's custom-call handler does:
    a name, device buffers (tensors or raw addresses, inputs then outputs) and
    one CallDesc as the opaque bytes.  Returns the status code."""
    d = CallDesc()
    for i, v in enumerate(dims):
        d.dims[i] = int(v)
    for i, v in enumerate(fparams):
        d.fparams[i] = float(v)
    d.dtype, d.flags = int(dtype), int(flags)
    arr = (_c_vp * max(1, len(buffers)))(
        *[b if isinstance(b, int) or b is None else b.data_ptr() for b in buffers])
    rc = lib().jules_custom_call(name.encode(), _stream(stream), arr, len(buffers),
                                 ctypes.cast(ctypes.pointer(d), _c_vp), ctypes.sizeof(d))
    if check:
        _check(rc, f"jules_custom_call({name})")
    return rc


def mlp_block_workspace_bytes(T, d, dff) -> int:
    return int(lib().jules_mlp_block_workspace_bytes(T, d, dff))


def mlp_block(X, gamma, beta, W1, b1, W2, b2, eps=1e-5, out=None, workspace=None, stream=None,
              out_dtype=None):
    """out = GELU(LN(X) @ W1 + b1) @ W2 + b2 + X  (bf16 operands; bf16 or
    fp32 output)."""
    import torch
    T, d = X.shape
    dff = W1.shape[1]
    if out is None:
        out = torch.empty((T, d), dtype=out_dtype or X.dtype, device=X.device)
    need = mlp_block_workspace_bytes(T, d, dff)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=X.device)
    rc = lib().jules_mlp_block(_ptr(X), _ptr(gamma), _ptr(beta), _ptr(W1), _ptr(b1), _ptr(W2),
                               _ptr(b2), _ptr(out), _dtype_code(out), T, d, dff, float(eps),
                               _ptr(workspace),
                               workspace.numel() * workspace.element_size(), _stream(stream))
    _check(rc, "jules_mlp_block")
    return out


def mlp_block_fold_weights(gamma, beta, W1, b1, stream=None):
    """Folded LayerNorm weights of the MLP block (once per weights):
    (W1f = bf16(diag(gamma) W1), colsum(W1f), c = beta . W1 + b1)."""
    import torch
    d, dff = W1.shape
    W1f = torch.empty_like(W1)
    colsum = torch.empty(dff, dtype=torch.float32, device=W1.device)
    c = torch.empty(dff, dtype=torch.float32, device=W1.device)
    rc = lib().jules_mlp_block_fold_weights(_ptr(gamma), _ptr(beta), _ptr(W1), _ptr(b1), _ptr(W1f),
                                            _ptr(colsum), _ptr(c), d, dff, _stream(stream))
    _check(rc, "jules_mlp_block_fold_weights")
    return W1f, colsum, c


def mlp_block_folded(X, folded, W2, b2, eps=1e-5, out=None, workspace=None, stream=None,
                     out_dtype=None):
    """mlp_block with the LayerNorm folded into GEMM1's epilogue; `folded` is
    mlp_block_fold_weights(gamma, beta, W1, b1)."""
    import torch
    W1f, colsum, c = folded
    T, d = X.shape
    dff = W1f.shape[1]
    if out is None:
        out = torch.empty((T, d), dtype=out_dtype or X.dtype, device=X.device)
    need = int(lib().jules_mlp_block_folded_workspace_bytes(T, d, dff))
    if workspace is None:
        workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=X.device)
    rc = lib().jules_mlp_block_folded(_ptr(X), _ptr(W1f), _ptr(colsum), _ptr(c), _ptr(W2), _ptr(b2),
                                      _ptr(out), _dtype_code(out), T, d, dff, float(eps),
                                      _ptr(workspace), workspace.numel() * workspace.element_size(),
                                      _stream(stream))
    _check(rc, "jules_mlp_block_folded")
    return out


def kernel_by_name(name: str) -> int:
    return int(lib().jules_kernel_by_name(name.encode()))


def kernel_names():
    h = lib()
    return [h.jules_kernel_name(i).decode() for i in range(h.jules_kernel_count())]


# ---------------------------------------------------------------------------
# Multi-GPU (one process per GPU): the jules_dist_* entry points.
# ---------------------------------------------------------------------------
DIST_ID_BYTES = 128


def dist_shard(units: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of `units` owned by `rank` (the library's partition)."""
    b, e = _c_i64(0), _c_i64(0)
    _check(lib().jules_dist_shard(units, world, rank, ctypes.byref(b), ctypes.byref(e)),
           "jules_dist_shard")
    return b.value, e.value


class _DevArray:
    """__cuda_array_interface__ over library-owned device memory."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


class Dist:
    """A communicator of the multi-GPU entry points.  Every rank constructs
    one with the same id (see unique_id / from_torch) and its own device
    current; all methods are collective."""

    def __init__(self, world: int, rank: int, uid: bytes):
        self.world, self.rank = world, rank
        self.h = _c_vp()
        buf = ctypes.create_string_buffer(bytes(uid), DIST_ID_BYTES)
        _check(lib().jules_dist_init(ctypes.byref(self.h), world, rank, buf), "jules_dist_init")
        self._shared = {}

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(DIST_ID_BYTES)
        _check(lib().jules_dist_unique_id(buf), "jules_dist_unique_id")
        return buf.raw

    @classmethod
    def from_torch(cls, group=None):
        """Rank 0's id sent to all ranks over an initialised torch.distributed
        group (plumbing only)."""
        import torch.distributed as tdist
        obj = [cls.unique_id() if tdist.get_rank(group) == 0 else None]
        tdist.broadcast_object_list(obj, src=0, group=group)
        return cls(tdist.get_world_size(group), tdist.get_rank(group), obj[0])

    def close(self):
        if self.h:
            lib().jules_dist_destroy(self.h)
            self.h = _c_vp()
            self._shared.clear()

    @property
    def multicast(self):
        """True when shared buffers have an NVLink multicast address (the
        fused gathers store each chunk once; the NVSwitch replicates it)."""
        on = _c_int(0)
        _check(lib().jules_dist_multicast(self.h, ctypes.byref(on)), "jules_dist_multicast")
        return bool(on.value)

    def gather_route(self, out_bytes):
        """"stores", "multicast" or "pull": how a sharded call gathers a
        shared output of out_bytes (jules_dist_gather_route)."""
        r = _c_int(0)
        _check(lib().jules_dist_gather_route(self.h, int(out_bytes), ctypes.byref(r)),
               "jules_dist_gather_route")
        return ("stores", "multicast", "pull")[r.value]

    def barrier(self, stream=None):
        _check(lib().jules_dist_barrier(self.h, _stream(stream)), "jules_dist_barrier")

    def alloc_shared(self, shape, dtype):
        """A zeroed tensor whose memory every rank can write (the output of a
        fused-gather call).  Valid until free_shared / close."""
        import torch
        elt = torch.empty((), dtype=dtype).element_size()
        n = 1
        for d in shape:
            n *= int(d)
        p = _c_vp()
        _check(lib().jules_dist_alloc_shared(self.h, max(n * elt, 16), ctypes.byref(p)),
               "jules_dist_alloc_shared")
        code = {1: "|u1", 2: "<i2", 4: "<f4"}[elt]
        t = torch.as_tensor(_DevArray(p.value, shape, code))
        if t.dtype != dtype:
            t = t.view(dtype)
        self._shared[p.value] = t
        return t

    def free_shared(self, t):
        ptr = t.data_ptr()
        self._shared.pop(ptr, None)
        _check(lib().jules_dist_free_shared(self.h, _c_vp(ptr)), "jules_dist_free_shared")

    def gemm_bias_act(self, A, W, bias=None, residual=None, act="none", out=None, out_dtype=None,
                      stream=None):
        """Sharded jules_gemm_bias_act: this rank computes its rows of C and every
        rank's `out` holds the whole C afterwards (fused gather when `out` came
        from alloc_shared)."""
        import torch
        _dense(A, "A"), _dense(W, "W")
        M, K = A.shape
        N = W.shape[1]
        if out is None:
            out = torch.empty((M, N), dtype=out_dtype or A.dtype, device=A.device)
        rc = lib().jules_dist_gemm_bias_act(self.h, _ptr(A), _ptr(W), _ptr(bias), _ptr(residual),
                                            _ptr(out), M, N, K,
                                            ACT[act] if isinstance(act, str) else int(act),
                                            _dtype_code(A), _dtype_code(out), _stream(stream))
        _check(rc, "jules_dist_gemm_bias_act")
        return out

    def flash_attention_fwd(self, Q, K, V, causal=False, scale=0.0, out=None, lse=None,
                            stream=None):
        """Sharded jules_flash_attention_fwd over (batch, kv head) units; every
        rank's `out` (and `lse`) holds the whole result afterwards."""
        import torch
        B, Hq, S, D = Q.shape
        Hkv = K.shape[1]
        if out is None:
            out = torch.empty_like(Q)
        rc = lib().jules_dist_flash_attention_fwd(self.h, _ptr(Q), _ptr(K), _ptr(V), _ptr(out),
                                                  _ptr(lse), B, Hq, Hkv, S, D, float(scale),
                                                  int(bool(causal)), _dtype_code(Q),
                                                  _stream(stream))
        _check(rc, "jules_dist_flash_attention_fwd")
        return out, lse
