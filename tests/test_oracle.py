"""Pins the oracle: the C restatement (oracle/restate.c) against the golden
fixtures produced by the reference's own kernels (tests/golden), the
reference build against the same fixtures, and the causal / grouped-query /
lse extensions against an independent float64 computation."""
import os

import numpy as np
import pytest

from conftest import F32_REL_L2, ROOT, max_abs, rel_l2

import sys
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
import make_golden as mg  # noqa: E402

GOLD = np.load(os.path.join(ROOT, "tests", "golden", "reference_outputs.npz"))
CASES = mg.golden_cases()


def _compare(name, key, arr, tol):
    if f"{name}/{key}" in GOLD.files:
        want = GOLD[f"{name}/{key}"]
        assert rel_l2(arr, want) <= tol, (name, key, rel_l2(arr, want))
    else:
        samp = GOLD[f"{name}/{key}__sample"]
        rows = GOLD[f"{name}/{key}__rowsum"]
        assert rel_l2(arr.ravel()[::mg.SAMPLE_STRIDE], samp) <= tol
        got_rows = arr.reshape(-1, arr.shape[-1]).astype(np.float64).sum(axis=1)
        assert max_abs(got_rows, rows) <= 1e-3


def _restated(orc, c, ins):
    k = c["kind"]
    if k == "attn":
        o, _ = orc.flash_attention(*ins, causal=False)
        return {"flash": o, "standard": o}
    if k == "tiled":
        return {"out": orc.gemm_bias_act(ins[0], ins[1], None, None, c["act"])}
    if k == "bias_relu":
        return {"out": orc.gemm_bias_act(ins[0], ins[1], ins[2], None, "relu")}
    if k == "layernorm":
        return {"out": orc.layernorm(*ins)}
    if k == "gelu":
        return {"out": orc.gelu(ins[0])}
    if k == "mlp":
        X, W1, b1, W2, b2 = ins
        h = orc.gemm_bias_act(X, W1, b1, None, "relu")
        return {"out": orc.gemm_bias_act(h, W2, b2, None, "none")}
    if k == "gemm_bias_gelu":
        return {"out": orc.gemm_bias_act(ins[0], ins[1], ins[2], None, "gelu")}
    if k == "softmax":
        return {"out": orc.softmax(ins[0])}
    if k == "xent":
        loss, grad = orc.cross_entropy(ins[0], ins[1])
        return {"grad": grad, "loss": np.array([loss], np.float32)}
    if k == "mlp_train":
        r = orc.mlp_fwd_bwd(*ins)
        r["loss"] = np.array([r["loss"]], np.float32)
        return r
    if k == "int8":
        return {"out": orc.matmul_int8(ins[0], ins[1], 0.02, 0.03, ins[2] if len(ins) > 2 else None)}
    raise ValueError(k)


@pytest.mark.parametrize("name", sorted(CASES))
def test_inputs_regenerate(name):
    c = CASES[name]
    assert mg.digest(*mg.make_inputs(c)) == str(GOLD[f"{name}/input_digest"])


@pytest.mark.parametrize("name", sorted(CASES))
def test_restated_matches_reference_fixture(orc, name):
    c = CASES[name]
    ins = mg.make_inputs(c)
    # The reference's exp is a polynomial (FusedKernels.h:90-133) accurate to
    # ~4e-6 relative; the restatement uses expf.  Everything else agrees to
    # summation-order noise.
    tol = F32_REL_L2
    for key, arr in _restated(orc, c, ins).items():
        _compare(name, key, arr, tol)


@pytest.mark.parametrize("name", sorted(CASES))
def test_reference_build_matches_fixture(ref, name):
    c = CASES[name]
    ins = mg.make_inputs(c)
    for key, arr in mg.run_reference(ref, c, ins).items():
        _compare(name, key, arr, 1e-6)


def test_reference_flash_vs_standard_fixture():
    for name in ("attn_small", "attn_ragged"):
        assert rel_l2(GOLD[f"{name}/flash"], GOLD[f"{name}/standard"]) <= 1e-5


def _attn_f64(Q, K, V, causal, scale=None):
    B, Hq, S, D = Q.shape
    g = Hq // K.shape[1]
    Kr = np.repeat(K, g, axis=1).astype(np.float64)
    Vr = np.repeat(V, g, axis=1).astype(np.float64)
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    s = np.einsum("bhqd,bhkd->bhqk", Q.astype(np.float64), Kr) * scale
    if causal:
        s = s + np.triu(np.full((S, S), -np.inf), 1)
    m = s.max(-1, keepdims=True)
    lse = np.log(np.exp(s - m).sum(-1)) + m[..., 0]
    return np.exp(s - lse[..., None]) @ Vr, lse


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("Hq,Hkv,S", [(4, 4, 64), (8, 2, 100), (6, 1, 33), (2, 2, 1)])
def test_restated_attention_extensions_vs_float64(orc, causal, Hq, Hkv, S):
    g = np.random.default_rng(S + Hq)
    D = 32
    Q = g.standard_normal((2, Hq, S, D), dtype=np.float32)
    K = g.standard_normal((2, Hkv, S, D), dtype=np.float32)
    V = g.standard_normal((2, Hkv, S, D), dtype=np.float32)
    o, lse = orc.flash_attention(Q, K, V, causal=causal)
    o2, lse2 = _attn_f64(Q, K, V, causal)
    assert rel_l2(o, o2) <= 2e-6
    assert max_abs(lse, lse2) <= 2e-5


def test_restated_attention_windows_and_units(orc):
    g = np.random.default_rng(0)
    Q, K, V = (g.standard_normal((2, 4, 96, 16), dtype=np.float32) for _ in range(3))
    full, lf = orc.flash_attention(Q, K, V, causal=True)
    part, lp = orc.flash_attention(Q, K, V, causal=True, units=[5], q_begin=40, q_end=70)
    assert np.array_equal(part[1, 1, 40:70], full[1, 1, 40:70])
    assert np.array_equal(lp[1, 1, 40:70], lf[1, 1, 40:70])
    assert not part[0].any()


def test_attention_known_answers(orc):
    """S=1 gives O = V; identical keys give O = mean(V)."""
    g = np.random.default_rng(1)
    Q, K, V = (g.standard_normal((1, 2, 1, 8), dtype=np.float32) for _ in range(3))
    o, lse = orc.flash_attention(Q, K, V)
    assert np.allclose(o, V, rtol=1e-6, atol=1e-7)
    Q = g.standard_normal((1, 1, 5, 8), dtype=np.float32)
    K = np.repeat(g.standard_normal((1, 1, 1, 8), dtype=np.float32), 5, axis=2)
    V = g.standard_normal((1, 1, 5, 8), dtype=np.float32)
    o, _ = orc.flash_attention(Q, K, V)
    assert np.allclose(o[0, 0], V[0, 0].mean(0, keepdims=True), rtol=1e-5, atol=1e-6)


def test_bf16_round_matches_torch():
    import torch
    import oracle
    g = np.random.default_rng(3)
    x = np.concatenate([g.standard_normal(10000).astype(np.float32) * 10 ** g.uniform(-30, 30, 10000).astype(np.float32),
                        np.array([0.0, -0.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, np.inf, -np.inf,
                                  3.4e38, 1e-40], np.float32)])
    want = torch.from_numpy(x).to(torch.bfloat16).to(torch.float32).numpy()
    got = oracle.bf16_round(x)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_mlp_block_composition(orc):
    """The C4 oracle is LN -> bf16 -> GEMM+b1+GELU -> bf16 -> GEMM+b2+X (fp32)."""
    import oracle
    g = np.random.default_rng(2)
    T, d, dff = 8, 32, 64
    X = oracle.bf16_round(g.standard_normal((T, d)).astype(np.float32))
    gam = (1 + 0.02 * g.standard_normal(d)).astype(np.float32)
    bet = (0.02 * g.standard_normal(d)).astype(np.float32)
    W1 = oracle.bf16_round((0.1 * g.standard_normal((d, dff))).astype(np.float32))
    b1 = (0.02 * g.standard_normal(dff)).astype(np.float32)
    W2 = oracle.bf16_round((0.1 * g.standard_normal((dff, d))).astype(np.float32))
    b2 = (0.02 * g.standard_normal(d)).astype(np.float32)
    out = orc.mlp_block(X, gam, bet, W1, b1, W2, b2)
    xn = oracle.bf16_round(orc.layernorm(X, gam, bet))
    h = oracle.bf16_round(orc.gemm_bias_act(xn, W1, b1, None, "gelu"))
    want = orc.gemm_bias_act(h, W2, b2, X, "none")
    assert np.array_equal(out, want)
    part = orc.mlp_block(X, gam, bet, W1, b1, W2, b2, rows=[3, 6])
    assert np.array_equal(part, out[[3, 6]])
