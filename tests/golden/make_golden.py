"""Generate the golden fixtures in tests/golden/ from the reference itself.

Runs the reference's own kernels (include/jules/Kernel/*.h of
AVmakeralt/jules, compiled unmodified into oracle/_ref by oracle/Makefile)
on seeded inputs and stores their outputs.  The reference ships no test
vectors of its own (its only tests parse .jules files,
test/CMakeLists.txt:4-15), so these fixtures are what pins the oracle.

Inputs are not stored: each case records its generator (numpy PCG64 seed,
shape, distribution) and a checksum of the inputs, and the tests regenerate
them.  Large outputs are stored as a strided sample plus per-row sums.

Run from the repository root where the reference source is present:
    python tests/golden/make_golden.py
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle  # noqa: E402


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()[:16]


# name -> (kind, params).  Generators live in golden_cases() so the tests use
# the same code.
def golden_cases():
    cases = {}
    # flashAttention / standardAttention: bench_kernel.cpp:502-556 style
    # shapes; config C1 uses N(0,1).
    cases["attn_small"] = dict(kind="attn", B=2, H=2, S=40, D=16, seed=101, dist="uniform")
    cases["attn_ragged"] = dict(kind="attn", B=1, H=3, S=77, D=32, seed=102, dist="normal")
    cases["attn_c1"] = dict(kind="attn", B=1, H=8, S=512, D=64, seed=1, dist="normal")
    # tiledMatmulWithActivation for every ActivationType.
    for act in ("none", "relu", "sigmoid", "tanh", "gelu"):
        cases[f"tiled_{act}"] = dict(kind="tiled", M=48, N=56, K=40, act=act, seed=200)
    cases["tiled_big"] = dict(kind="tiled", M=128, N=512, K=512, act="gelu", seed=201)
    cases["bias_relu"] = dict(kind="bias_relu", M=64, K=48, N=80, seed=300)
    cases["layernorm"] = dict(kind="layernorm", M=64, N=256, seed=400)
    cases["layernorm_ragged"] = dict(kind="layernorm", M=9, N=1000, seed=401)
    cases["gelu"] = dict(kind="gelu", N=1000, seed=500)
    # fusedMLPForward on the bench_kernel.cpp:166-256 shape.
    cases["mlp_forward"] = dict(kind="mlp", M=64, K1=784, N1=256, N2=10, seed=600)
    # Config C2's composition (GEMM -> bias -> GELU) on bf16-valued inputs.
    cases["gemm_bias_gelu"] = dict(kind="gemm_bias_gelu", M=32, N=384, K=512, seed=700)
    # bench_kernel.cpp:396-400 softmax shapes, plus a ragged row length
    cases["softmax_mlp"] = dict(kind="softmax", M=64, N=256, seed=800)
    cases["softmax_cls"] = dict(kind="softmax", M=64, N=10, seed=801)
    cases["softmax_ragged"] = dict(kind="softmax", M=7, N=1000, seed=802)
    cases["xent"] = dict(kind="xent", M=64, N=1000, seed=900)
    cases["xent_ragged"] = dict(kind="xent", M=13, N=37, seed=901)
    # matmulInt8 (FusedKernels.h:867-1073), from the reference build's scalar branch
    cases["int8"] = dict(kind="int8", M=64, N=96, K=200, seed=1000)
    cases["int8_bias"] = dict(kind="int8", M=33, N=40, K=77, seed=1001, bias=True)
    # interleavedMLPForwardBackward (InterleavedAutodiff.h:55-160), bench_kernel.cpp-style shape
    cases["mlp_train"] = dict(kind="mlp_train", M=64, K1=100, N1=48, N2=10, seed=1100)
    return cases


def make_inputs(c):
    g = np.random.default_rng(c["seed"])
    k = c["kind"]
    if k == "attn":
        shape = (c["B"], c["H"], c["S"], c["D"])
        if c["dist"] == "uniform":
            return [g.uniform(-1, 1, shape).astype(np.float32) for _ in range(3)]
        return [g.standard_normal(shape, dtype=np.float32) for _ in range(3)]
    if k == "tiled":
        return [g.uniform(-1, 1, (c["M"], c["K"])).astype(np.float32),
                g.uniform(-1, 1, (c["K"], c["N"])).astype(np.float32)]
    if k == "bias_relu":
        return [g.uniform(-1, 1, (c["M"], c["K"])).astype(np.float32),
                g.uniform(-1, 1, (c["K"], c["N"])).astype(np.float32),
                g.uniform(-1, 1, c["N"]).astype(np.float32)]
    if k == "layernorm":
        return [g.uniform(-1, 1, (c["M"], c["N"])).astype(np.float32),
                (1 + 0.02 * g.standard_normal(c["N"])).astype(np.float32),
                (0.02 * g.standard_normal(c["N"])).astype(np.float32)]
    if k == "gelu":
        return [g.uniform(-6, 6, c["N"]).astype(np.float32)]
    if k == "mlp":
        return [g.uniform(-1, 1, (c["M"], c["K1"])).astype(np.float32),
                (g.uniform(-1, 1, (c["K1"], c["N1"])) / np.sqrt(c["K1"])).astype(np.float32),
                g.uniform(-1, 1, c["N1"]).astype(np.float32),
                (g.uniform(-1, 1, (c["N1"], c["N2"])) / np.sqrt(c["N1"])).astype(np.float32),
                g.uniform(-1, 1, c["N2"]).astype(np.float32)]
    if k == "gemm_bias_gelu":
        s = 1.0 / np.sqrt(c["K"])
        return [oracle.bf16_round(g.uniform(-1, 1, (c["M"], c["K"])).astype(np.float32) * s),
                oracle.bf16_round(g.uniform(-1, 1, (c["K"], c["N"])).astype(np.float32) * s),
                (0.02 * g.standard_normal(c["N"])).astype(np.float32)]
    if k == "softmax":
        return [(3 * g.standard_normal((c["M"], c["N"]))).astype(np.float32)]
    if k == "xent":
        return [(3 * g.standard_normal((c["M"], c["N"]))).astype(np.float32),
                g.integers(0, c["N"], c["M"]).astype(np.int32)]
    if k == "mlp_train":
        M, K1, N1, N2 = c["M"], c["K1"], c["N1"], c["N2"]
        return [g.uniform(-1, 1, (M, K1)).astype(np.float32),
                (g.uniform(-1, 1, (K1, N1)) / np.sqrt(K1)).astype(np.float32),
                (0.1 * g.standard_normal(N1)).astype(np.float32),
                (g.uniform(-1, 1, (N1, N2)) / np.sqrt(N1)).astype(np.float32),
                (0.1 * g.standard_normal(N2)).astype(np.float32),
                g.integers(0, N2, M).astype(np.int32)]
    if k == "int8":
        ins = [g.integers(-128, 128, (c["M"], c["K"])).astype(np.int8),
               g.integers(-128, 128, (c["K"], c["N"])).astype(np.int8)]
        if c.get("bias"):
            ins.append(g.standard_normal(c["N"]).astype(np.float32))
        return ins
    raise ValueError(k)


def run_reference(ref, c, ins):
    k = c["kind"]
    if k == "attn":
        return {"flash": ref.flash_attention(*ins), "standard": ref.standard_attention(*ins)}
    if k == "tiled":
        return {"out": ref.tiled_matmul_act(ins[0], ins[1], c["act"])}
    if k == "bias_relu":
        return {"out": ref.fused_matmul_bias_relu(*ins)}
    if k == "layernorm":
        return {"out": ref.layernorm(*ins)}
    if k == "gelu":
        return {"out": ref.gelu(ins[0])}
    if k == "mlp":
        return {"out": ref.mlp_forward(*ins)}
    if k == "gemm_bias_gelu":
        return {"out": ref.gemm_bias_gelu(*ins)}
    if k == "softmax":
        return {"out": ref.softmax(ins[0])}
    if k == "xent":
        loss, grad = ref.cross_entropy(ins[0], ins[1])
        return {"grad": grad, "loss": np.array([loss], np.float32)}
    if k == "mlp_train":
        r = ref.mlp_fwd_bwd(*ins)
        r["loss"] = np.array([r["loss"]], np.float32)
        return r
    if k == "int8":
        scalar = ref if ref.variant == "avx2" else oracle.Reference(variant="avx2")
        return {"out": scalar.matmul_int8(ins[0], ins[1], 0.02, 0.03,
                                          ins[2] if len(ins) > 2 else None)}
    raise ValueError(k)


SAMPLE_STRIDE = 37  # outputs above this size keep every 37th element + row sums
FULL_LIMIT = 20000


def pack(name, arr):
    flat = arr.ravel()
    if flat.size <= FULL_LIMIT:
        return {f"{name}": arr}
    rows = arr.reshape(-1, arr.shape[-1])
    return {f"{name}__sample": flat[::SAMPLE_STRIDE].copy(),
            f"{name}__rowsum": rows.astype(np.float64).sum(axis=1)}


def main():
    ref = oracle.Reference()
    out = {}
    for name, c in golden_cases().items():
        ins = make_inputs(c)
        res = run_reference(ref, c, ins)
        out[f"{name}/input_digest"] = np.array(digest(*ins))
        for key, arr in res.items():
            for k2, v in pack(key, arr).items():
                out[f"{name}/{k2}"] = v
    out["_meta/variant"] = np.array(ref.variant)
    path = os.path.join(HERE, "reference_outputs.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(golden_cases())} cases)")


if __name__ == "__main__":
    main()
