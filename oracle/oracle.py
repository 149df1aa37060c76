"""ctypes front end for the parity oracle.

TEST INFRASTRUCTURE ONLY.  Only tests/, ``__graft_entry__.smoke()`` and the
CPU legs of ``bench.py`` import this module.  The shipped library
(``jules_b200``) never imports it and has no CPU fallback.

Two oracles:

* ``Restated`` - oracle/restate.c, a C restatement of the reference kernels
  (causal / grouped-query / logsumexp and the MLP-block composition are
  extensions written into the reference's loop structure).
* ``Reference`` - the reference's own ``include/jules/Kernel`` headers
  compiled unmodified by oracle/Makefile into oracle/_ref (needs the
  reference source at build time; the built .so travels without it).

Inputs and outputs are numpy float32 arrays (bf16 data is carried as
bf16-rounded float32, the same bits the GPU consumes).
"""
from __future__ import annotations

import ctypes
import glob
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")
REF = os.path.join(HERE, "_ref")

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int)
_i64p = ctypes.POINTER(ctypes.c_int64)

ACT = {"none": 0, "relu": 1, "sigmoid": 2, "tanh": 3, "gelu": 4}
FP8_FMT = {"e4m3": 0, "e5m2": 1}


def reference_dir() -> str:
    """Checkout of the reference project: $JULES_REFERENCE_DIR, else a
    `reference` directory beside this repository."""
    return os.environ.get("JULES_REFERENCE_DIR") or os.path.join(os.path.dirname(os.path.dirname(HERE)),
                                                                 "reference")


def build(reference_root: str | None = None) -> None:
    """Compile the oracle (restatement always; reference when present)."""
    subprocess.run(["make", "-s", f"REF={reference_root or reference_dir()}"], cwd=HERE, check=True)


def _fp(a: np.ndarray | None):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def _i8(a: np.ndarray):
    assert a.dtype == np.int8 and a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.c_void_p)


def _ip(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(_i32p)


def _cpu_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    flags = line.split()
                    return all(x in flags for x in ("avx512f", "avx512dq", "avx512vl", "avx512bw"))
    except OSError:
        pass
    return False


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bf16 precision, returned as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7F800000) == 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    r = np.where(nan, (u & 0xFFFF0000).astype(np.uint32) | np.where((u & 0x7FFFFF) != 0, 0x00400000, 0).astype(np.uint32), r)
    return r.view(np.float32).reshape(x.shape)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def _mlp_fwd_bwd(fn, X, W1, b1, W2, b2, targets, want_dx):
    X, W1, b1, W2, b2 = (np.ascontiguousarray(a, np.float32) for a in (X, W1, b1, W2, b2))
    t = np.ascontiguousarray(targets, np.int32)
    M, K1 = X.shape
    N1, N2 = W1.shape[1], W2.shape[1]
    r = dict(out=np.empty((M, N2), np.float32), dW1=np.empty((K1, N1), np.float32),
             db1=np.empty(N1, np.float32), dW2=np.empty((N1, N2), np.float32),
             db2=np.empty(N2, np.float32), dX=np.empty((M, K1), np.float32) if want_dx else None)
    r["loss"] = float(fn(_fp(X), _fp(W1), _fp(b1), _fp(W2), _fp(b2), _ip(t), _fp(r["out"]),
                         _fp(r["dW1"]), _fp(r["db1"]), _fp(r["dW2"]), _fp(r["db2"]), _fp(r["dX"]),
                         M, K1, N1, N2))
    return r


class Restated:
    """oracle/restate.c via ctypes."""

    def __init__(self):
        path = os.path.join(BUILD, "liboracle.so")
        if not os.path.exists(path):
            build()
        lib = ctypes.CDLL(path)
        lib.orc_gemm_bias_act.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_int64,
                                          ctypes.c_int64, ctypes.c_int64, ctypes.c_int]
        lib.orc_layernorm.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int64, ctypes.c_int64,
                                      ctypes.c_float, _f32p, _f32p]
        lib.orc_gelu.argtypes = [_f32p, _f32p, ctypes.c_int64]
        lib.orc_flash_attention.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p] + [ctypes.c_int] * 5 + [
            ctypes.c_float, ctypes.c_int, _i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.c_int, ctypes.c_int]
        lib.orc_mlp_block.argtypes = [_f32p] * 8 + [ctypes.c_int64] * 3 + [ctypes.c_float, _i64p,
                                                                          ctypes.c_int64]
        lib.orc_attention_bwd.argtypes = [_f32p] * 7 + [ctypes.c_int] * 5 + [ctypes.c_float,
                                                                             ctypes.c_int]
        lib.orc_fp8_decode.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int64, ctypes.c_int]
        lib.orc_fp8_encode.argtypes = [_f32p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int]
        lib.orc_gemm_fp8.argtypes = [ctypes.c_void_p, ctypes.c_void_p, _f32p, _f32p, _f32p,
                                     ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_float,
                                     ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.orc_matmul_int8.argtypes = [ctypes.c_void_p, ctypes.c_void_p, _f32p, ctypes.c_int64,
                                        ctypes.c_int64, ctypes.c_int64, ctypes.c_float,
                                        ctypes.c_float, _f32p]
        lib.orc_mlp_fwd_bwd.argtypes = [_f32p] * 5 + [_i32p] + [_f32p] * 6 + [ctypes.c_int64] * 4
        lib.orc_mlp_fwd_bwd.restype = ctypes.c_float
        lib.orc_softmax.argtypes = [_f32p, _f32p, ctypes.c_int64, ctypes.c_int64]
        lib.orc_cross_entropy.argtypes = [_f32p, _i32p, _f32p, ctypes.c_int64, ctypes.c_int64]
        lib.orc_cross_entropy.restype = ctypes.c_float
        lib.orc_num_threads.restype = ctypes.c_int
        self.lib = lib

    def num_threads(self) -> int:
        return self.lib.orc_num_threads()

    def gemm_bias_act(self, A, W, bias=None, residual=None, act="none"):
        M, K = A.shape
        N = W.shape[1]
        C = np.empty((M, N), np.float32)
        self.lib.orc_gemm_bias_act(_fp(A), _fp(W), _fp(bias), _fp(residual), _fp(C), M, N, K,
                                   ACT[act] if isinstance(act, str) else int(act))
        return C

    def layernorm(self, x, gamma, beta, eps=1e-5, stats=False):
        M, N = x.shape
        out = np.empty_like(x)
        mean = np.empty(M, np.float32) if stats else None
        rstd = np.empty(M, np.float32) if stats else None
        self.lib.orc_layernorm(_fp(out), _fp(x), _fp(gamma), _fp(beta), M, N, eps, _fp(mean), _fp(rstd))
        return (out, mean, rstd) if stats else out

    def gelu(self, x):
        out = np.empty_like(x)
        self.lib.orc_gelu(_fp(out), _fp(x), x.size)
        return out

    def softmax(self, x):
        x = np.ascontiguousarray(x, np.float32)
        M, N = x.shape
        out = np.empty_like(x)
        self.lib.orc_softmax(_fp(out), _fp(x), M, N)
        return out

    def mlp_fwd_bwd(self, X, W1, b1, W2, b2, targets, want_dx=True):
        """Returns dict(loss, out, dW1, db1, dW2, db2, dX)."""
        return _mlp_fwd_bwd(self.lib.orc_mlp_fwd_bwd, X, W1, b1, W2, b2, targets, want_dx)

    def matmul_int8(self, A, B, scale_a=1.0, scale_b=1.0, bias=None):
        A = np.ascontiguousarray(A, np.int8)
        B = np.ascontiguousarray(B, np.int8)
        M, K = A.shape
        N = B.shape[1]
        C = np.empty((M, N), np.float32)
        self.lib.orc_matmul_int8(_i8(A), _i8(B), _fp(C), M, N, K, scale_a, scale_b,
                                 _fp(None if bias is None else np.ascontiguousarray(bias, np.float32)))
        return C

    def fp8_decode(self, codes, fmt):
        """8-bit float codes (uint8) -> fp32; fmt "e4m3" or "e5m2"."""
        codes = np.ascontiguousarray(codes, np.uint8)
        out = np.empty(codes.shape, np.float32)
        self.lib.orc_fp8_decode(codes.ctypes.data_as(ctypes.c_void_p), _fp(out), codes.size,
                                FP8_FMT[fmt])
        return out

    def fp8_encode(self, x, fmt):
        """fp32 -> 8-bit float codes (uint8): nearest-even, saturating."""
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(x.shape, np.uint8)
        self.lib.orc_fp8_encode(_fp(x), out.ctypes.data_as(ctypes.c_void_p), x.size, FP8_FMT[fmt])
        return out

    def gemm_fp8(self, A, W, a_fmt="e4m3", w_fmt="e4m3", bias=None, residual=None, act="none",
                 scale=1.0):
        """A, W: uint8 codes of 8-bit floats.  Returns fp32 C."""
        A = np.ascontiguousarray(A, np.uint8)
        W = np.ascontiguousarray(W, np.uint8)
        M, K = A.shape
        N = W.shape[1]
        C = np.empty((M, N), np.float32)
        vp = lambda a: a.ctypes.data_as(ctypes.c_void_p)
        self.lib.orc_gemm_fp8(vp(A), vp(W),
                              _fp(None if bias is None else np.ascontiguousarray(bias, np.float32)),
                              _fp(None if residual is None else np.ascontiguousarray(residual, np.float32)),
                              _fp(C), M, N, K, scale, ACT[act] if isinstance(act, str) else int(act),
                              FP8_FMT[a_fmt], FP8_FMT[w_fmt])
        return C

    def cross_entropy(self, logits, targets):
        """Returns (mean loss, grad)."""
        logits = np.ascontiguousarray(logits, np.float32)
        targets = np.ascontiguousarray(targets, np.int32)
        M, N = logits.shape
        grad = np.empty_like(logits)
        loss = self.lib.orc_cross_entropy(_fp(logits), _ip(targets), _fp(grad), M, N)
        return float(loss), grad

    def flash_attention(self, Q, K, V, causal=False, scale=None, units=None, q_begin=0, q_end=0,
                        tile_q=32, tile_k=64, want_lse=True):
        """Q [B,Hq,S,D], K/V [B,Hkv,S,D].  Returns (O, lse); rows outside the
        computed units / window are left at zero."""
        B, Hq, S, D = Q.shape
        Hkv = K.shape[1]
        if scale is None:
            scale = 1.0 / np.sqrt(D)
        O = np.zeros_like(Q)
        lse = np.zeros((B, Hq, S), np.float32) if want_lse else None
        if units is not None:
            u = np.ascontiguousarray(np.asarray(units, dtype=np.int32))
            up, nu = u.ctypes.data_as(_i32p), len(u)
        else:
            up, nu = None, 0
        self.lib.orc_flash_attention(_fp(O), _fp(lse), _fp(Q), _fp(K), _fp(V), B, Hq, Hkv, S, D,
                                     float(scale), int(bool(causal)), up, nu, int(q_begin),
                                     int(q_end), int(tile_q), int(tile_k))
        return O, lse

    def attention_bwd(self, Q, K, V, dO, causal=False, scale=None):
        """Exact (double) gradients (dQ, dK, dV) of the attention forward for
        dO; shapes as flash_attention."""
        Q, K, V, dO = (np.ascontiguousarray(a, np.float32) for a in (Q, K, V, dO))
        B, Hq, S, D = Q.shape
        Hkv = K.shape[1]
        if scale is None:
            scale = 1.0 / np.sqrt(D)
        dQ, dK, dV = np.empty_like(Q), np.empty_like(K), np.empty_like(V)
        self.lib.orc_attention_bwd(_fp(dQ), _fp(dK), _fp(dV), _fp(Q), _fp(K), _fp(V), _fp(dO),
                                   B, Hq, Hkv, S, D, float(scale), int(bool(causal)))
        return dQ, dK, dV

    def mlp_block(self, X, gamma, beta, W1, b1, W2, b2, eps=1e-5, rows=None):
        T, d = X.shape
        dff = W1.shape[1]
        if rows is not None:
            r = np.ascontiguousarray(np.asarray(rows, dtype=np.int64))
            rp, nr = r.ctypes.data_as(_i64p), len(r)
        else:
            rp, nr = None, T
        out = np.empty((nr, d), np.float32)
        self.lib.orc_mlp_block(_fp(out), _fp(X), _fp(gamma), _fp(beta), _fp(W1), _fp(b1), _fp(W2),
                               _fp(b2), T, d, dff, eps, rp, nr)
        return out


def find_openblas_sgemm64():
    """Address of numpy's bundled ILP64 cblas_sgemm, or None."""
    try:
        import numpy as _np
        libdir = os.path.join(os.path.dirname(os.path.dirname(_np.__file__)), "numpy.libs")
        cands = sorted(glob.glob(os.path.join(libdir, "libscipy_openblas64_*.so")))
        if not cands:
            return None
        ob = ctypes.CDLL(cands[0])
        return ctypes.cast(ob.scipy_cblas_sgemm64_, ctypes.c_void_p).value
    except (OSError, AttributeError):
        return None


class Reference:
    """The reference's own kernels (oracle/_ref), compiled from its sources."""

    def __init__(self, use_openblas: bool = False, variant: str | None = None):
        if variant is None:
            variant = "avx512" if _cpu_has_avx512() else "avx2"
        path = os.path.join(REF, f"libjules_ref_{variant}.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"reference oracle not built: {path} (run make in oracle/ where "
                                    "the reference source is present)")
        lib = ctypes.CDLL(path)
        self.variant = variant
        lib.ref_flash_attention.argtypes = [_f32p] * 4 + [ctypes.c_int] * 4
        lib.ref_standard_attention.argtypes = [_f32p] * 4 + [ctypes.c_int] * 4
        lib.ref_attention.argtypes = [_f32p] * 4 + [ctypes.c_int] * 4
        lib.ref_should_use_flash.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_size_t]
        lib.ref_tile_config.argtypes = [ctypes.c_int] * 3 + [_i32p]
        lib.ref_tiled_matmul_act.argtypes = [_f32p] * 3 + [ctypes.c_int] * 7
        lib.ref_fused_matmul_relu.argtypes = [_f32p] * 3 + [ctypes.c_int] * 3
        lib.ref_fused_matmul_bias_relu.argtypes = [_f32p] * 4 + [ctypes.c_int] * 3
        lib.ref_fused_layernorm.argtypes = [_f32p] * 4 + [ctypes.c_int] * 2 + [ctypes.c_float]
        lib.ref_fused_gelu.argtypes = [_f32p, _f32p, ctypes.c_int]
        lib.ref_fused_softmax.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int]
        lib.ref_fused_cross_entropy.argtypes = [_f32p, _i32p, _f32p, ctypes.c_int, ctypes.c_int]
        lib.ref_matmul_int8.argtypes = [ctypes.c_void_p, ctypes.c_void_p, _f32p] + [ctypes.c_int] * 3 + [
            ctypes.c_float, ctypes.c_float, _f32p]
        lib.ref_interleaved_mlp.argtypes = [_f32p] * 5 + [_i32p] + [_f32p] * 6 + [ctypes.c_int] * 4
        lib.ref_interleaved_mlp.restype = ctypes.c_float
        lib.ref_fused_cross_entropy.restype = ctypes.c_float
        lib.ref_blas_matmul.argtypes = [_f32p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_float] * 2 + [
            ctypes.c_int] * 2
        lib.ref_fused_mlp_forward.argtypes = [_f32p] * 6 + [ctypes.c_int] * 4
        lib.ref_cache_info.argtypes = [ctypes.POINTER(ctypes.c_size_t)]
        lib.oracle_set_sgemm64.argtypes = [ctypes.c_void_p]
        lib.ref_set_threads.argtypes = [ctypes.c_int]
        self.lib = lib
        self.openblas = False
        if use_openblas:
            fn = find_openblas_sgemm64()
            if fn:
                lib.oracle_set_sgemm64(fn)
                self.openblas = True

    def set_threads(self, n: int) -> None:
        self.lib.ref_set_threads(int(n))

    def cache_info(self):
        out = (ctypes.c_size_t * 4)()
        self.lib.ref_cache_info(out)
        return {"l1d": out[0], "l2": out[1], "l3": out[2], "cores": out[3]}

    def flash_attention(self, Q, K, V):
        B, H, S, D = Q.shape
        O = np.empty_like(Q)
        self.lib.ref_flash_attention(_fp(O), _fp(Q), _fp(K), _fp(V), B, H, S, D)
        return O

    def standard_attention(self, Q, K, V):
        B, H, S, D = Q.shape
        O = np.empty_like(Q)
        self.lib.ref_standard_attention(_fp(O), _fp(Q), _fp(K), _fp(V), B, H, S, D)
        return O

    def attention(self, Q, K, V):
        B, H, S, D = Q.shape
        O = np.empty_like(Q)
        self.lib.ref_attention(_fp(O), _fp(Q), _fp(K), _fp(V), B, H, S, D)
        return O

    def should_use_flash(self, S, D, l3):
        return bool(self.lib.ref_should_use_flash(S, D, l3))

    def tile_config(self, M, N, K):
        out = (ctypes.c_int * 3)()
        self.lib.ref_tile_config(M, N, K, out)
        return tuple(out)

    def tiled_matmul_act(self, A, B, act="none", tile=None):
        M, K = A.shape
        N = B.shape[1]
        tm, tn, tk = tile or self.tile_config(M, N, K)
        C = np.empty((M, N), np.float32)
        self.lib.ref_tiled_matmul_act(_fp(A), _fp(B), _fp(C), M, N, K, tm, tn, tk,
                                      ACT[act] if isinstance(act, str) else int(act))
        return C

    def fused_matmul_relu(self, X, W):
        M, K = X.shape
        N = W.shape[1]
        out = np.empty((M, N), np.float32)
        self.lib.ref_fused_matmul_relu(_fp(X), _fp(W), _fp(out), M, K, N)
        return out

    def fused_matmul_bias_relu(self, X, W, b):
        M, K = X.shape
        N = W.shape[1]
        out = np.empty((M, N), np.float32)
        self.lib.ref_fused_matmul_bias_relu(_fp(X), _fp(W), _fp(b), _fp(out), M, K, N)
        return out

    def layernorm(self, x, gamma, beta, eps=1e-5):
        M, N = x.shape
        out = np.empty_like(x)
        self.lib.ref_fused_layernorm(_fp(out), _fp(x), _fp(gamma), _fp(beta), M, N, eps)
        return out

    def gelu(self, x):
        out = np.empty_like(x)
        self.lib.ref_fused_gelu(_fp(out), _fp(x), x.size)
        return out

    def softmax(self, x):
        x = np.ascontiguousarray(x, np.float32)
        M, N = x.shape
        out = np.empty_like(x)
        self.lib.ref_fused_softmax(_fp(out), _fp(x), M, N)
        return out

    def mlp_fwd_bwd(self, X, W1, b1, W2, b2, targets, want_dx=True):
        """The reference's interleavedMLPForwardBackward; dict(loss, out, dW1,
        db1, dW2, db2, dX)."""
        return _mlp_fwd_bwd(self.lib.ref_interleaved_mlp, X, W1, b1, W2, b2, targets, want_dx)

    def matmul_int8(self, A, B, scale_a=1.0, scale_b=1.0, bias=None):
        """The reference's matmulInt8.  Only the "avx2" variant (compiled
        without AVX-512, so its scalar branch) computes the documented product."""
        A = np.ascontiguousarray(A, np.int8)
        B = np.ascontiguousarray(B, np.int8)
        M, K = A.shape
        N = B.shape[1]
        C = np.empty((M, N), np.float32)
        self.lib.ref_matmul_int8(_i8(A), _i8(B), _fp(C), M, N, K, scale_a, scale_b,
                                 _fp(None if bias is None else np.ascontiguousarray(bias, np.float32)))
        return C

    def cross_entropy(self, logits, targets):
        """Returns (mean loss, grad) from the reference's fusedCrossEntropyLoss."""
        logits = np.ascontiguousarray(logits, np.float32)
        targets = np.ascontiguousarray(targets, np.int32)
        M, N = logits.shape
        grad = np.empty_like(logits)
        loss = self.lib.ref_fused_cross_entropy(_fp(logits), _ip(targets), _fp(grad), M, N)
        return float(loss), grad

    def blas_matmul(self, A, B, alpha=1.0, beta=0.0):
        M, K = A.shape
        N = B.shape[1]
        C = np.zeros((M, N), np.float32)
        self.lib.ref_blas_matmul(_fp(A), _fp(B), _fp(C), M, N, K, alpha, beta, 0, 0)
        return C

    def mlp_forward(self, X, W1, b1, W2, b2):
        M, K1 = X.shape
        N1 = W1.shape[1]
        N2 = W2.shape[1]
        out = np.empty((M, N2), np.float32)
        self.lib.ref_fused_mlp_forward(_fp(out), _fp(X), _fp(W1), _fp(b1), _fp(W2), _fp(b2), M, K1,
                                       N1, N2)
        return out

    def gemm_bias_gelu(self, A, W, bias, tile=None):
        """Config C2 composed from reference pieces: tiled GEMM (no act,
        FusedKernels.h:378-458) -> bias add (the :309-311 loop) -> fusedGelu
        (:606-627)."""
        C = self.tiled_matmul_act(A, W, "none", tile)
        C += bias[None, :]
        return self.gelu(np.ascontiguousarray(C))
