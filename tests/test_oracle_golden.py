"""Pin the CPU oracle before trusting it as the parity checker.

1. The reference's own known-answer tests for this path
   (aptransformerTests/ESPrimitivesTests.mm):
   * testGeluTanhMatchesFormula (:44-56): 5 points vs the double formula, 1e-5.
   * testGeluTanhBf16DoesNotQuantiseItsConstants (:71-91): >=99 % identical
     results for bf16 input vs the same values as f32 input over 512 points.
   * testMoERouterTopKWeights (:171-189): H=64, E=16, K=4, T=3, unit scales;
     exactly K nonzeros per routeWeights row and a row sum of 1 within 1e-4.
2. Golden vectors from HF transformers' Gemma4TextRouter / Gemma4TextExperts
   run in f32 (tests/golden/make_golden.py).
"""
import math
import os

import numpy as np
import pytest

from tests.helpers import block_close, router_index_check

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLDEN, f"hf_moe_{name}.npz")))


# ------------------------------------------------------------- reference KATs

def test_gelu_matches_formula(oracle):
    for v in (-2.0, -0.5, 0.0, 0.5, 2.0):
        inner = 0.7978845608028654 * (v + 0.044715 * v ** 3)
        ref = 0.5 * v * (1.0 + math.tanh(inner))
        assert abs(oracle.gelu_tanh_f32(v) - ref) <= 1e-5


def test_gelu_bf16_does_not_quantise_constants(oracle):
    n = 512
    xs = (-6.0 + 12.0 * np.arange(n, dtype=np.float32) / np.float32(n - 1)).astype(np.float32)
    xb = oracle.f32_to_bf16(xs)
    via_bf16 = oracle.bf16_to_f32(oracle.gelu_tanh_bf16(xb))
    via_f32 = oracle.bf16_to_f32(oracle.f32_to_bf16(
        np.array([oracle.gelu_tanh_f32(float(v)) for v in oracle.bf16_to_f32(xb)], np.float32)))
    same = np.mean(via_bf16 == via_f32)
    assert same >= 0.99


def test_router_topk_weights_structure(oracle):
    H, E, K, T = 64, 16, 4, 3
    rng = np.random.default_rng(0)
    proj = oracle.f32_to_bf16(rng.standard_normal((E, H), dtype=np.float32))
    x = oracle.f32_to_bf16(rng.standard_normal((T, H), dtype=np.float32))
    ones_h = oracle.f32_to_bf16(np.ones(H, np.float32))
    ones_e = oracle.f32_to_bf16(np.ones(E, np.float32))
    idx, w = oracle.route_topk(x, proj, ones_h, ones_e, K)
    W = oracle.bf16_to_f32(oracle.route_weights(idx, w, E))
    assert W.shape == (T, E)
    for t in range(T):
        assert int(np.sum(W[t] > 0)) == K
        # w is rounded to bf16 (ESRouter.mm:31): K values each within half a
        # bf16 ulp of ~1/K, so the row sum stays within 1e-4 .. K*2^-9/K.
        assert abs(float(W[t].sum()) - 1.0) <= max(1e-4, K * 2.0 ** -9)


# ------------------------------------------------------------- HF golden vectors

@pytest.mark.parametrize("case", ["unit", "small", "gemma"])
def test_router_vs_hf(oracle, case):
    d = load(case)
    idx, w, aux = oracle.route_topk(d["x"], d["proj"], d["scale"], d["pes"], int(d["K"]),
                                    return_scores=True)
    # logits agree to f32 summation-order noise
    np.testing.assert_allclose(aux["scores"], d["hf_scores"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(aux["probs"], d["hf_probs"], rtol=1e-4, atol=1e-7)
    bad, exempt = router_index_check(idx, d["hf_idx"], d["hf_scores"])
    assert bad == 0, f"{bad} rows with non-tie index mismatches"
    same = np.all(idx == d["hf_idx"], axis=1)
    np.testing.assert_allclose(aux["w_f32"][same], d["hf_w"][same], rtol=1e-5, atol=1e-7)


def _expert_bank(oracle, d):
    if "gate_up" in d:
        return d["gate_up"], d["down"]
    from tests.golden.make_golden import expert_weights  # regenerates per expert
    import torch
    E, I, H = int(d["E"]), int(d["I"]), int(d["H"])
    gu = np.zeros((E, 2 * I, H), np.uint16)
    dn = np.zeros((E, H, I), np.uint16)
    for e in np.unique(d["hf_idx"]):
        g, dd = expert_weights(int(d["seed"]), int(e), I, H)
        gu[e] = g.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        dn[e] = dd.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    return gu, dn


@pytest.mark.parametrize("case", ["unit", "small", "gemma"])
def test_experts_vs_hf(oracle, case):
    d = load(case)
    gu, dn = _expert_bank(oracle, d)
    # HF ran with f32 weights: feed the oracle HF's own top-k (bf16-rounded w)
    w_bf = oracle.f32_to_bf16(d["hf_w"])
    out = oracle.bf16_to_f32(oracle.experts_sparse(d["x"], gu, dn, d["hf_idx"], w_bf))
    ok, ma, cos = block_close(out, d["hf_out"])
    assert ok, (ma, cos)
    # the bf16 rounding points cost a few bf16 ulps at most
    scale = np.abs(d["hf_out"]).max()
    assert ma <= 0.02 * scale, (ma, scale)


def test_dense_equals_sparse(oracle):
    d = load("small")
    idx, w = oracle.route_topk(d["x"], d["proj"], d["scale"], d["pes"], int(d["K"]))
    W = oracle.route_weights(idx, w, int(d["E"]))
    sp = oracle.bf16_to_f32(oracle.experts_sparse(d["x"], d["gate_up"], d["down"], idx, w))
    de = oracle.bf16_to_f32(oracle.experts_dense(d["x"], d["gate_up"], d["down"], W))
    # same terms, summed in expert order instead of k order: <= 1 bf16 ulp apart
    diff = np.abs(sp - de)
    assert np.all(diff <= np.abs(sp) * 2.0 ** -7 + 1e-6)


def _mlx_affine_py(wf, gs, bits):
    """MLX's affine_quantize rule (mlx/fast.cpp at ml-explore/mlx @ 057cdc9ec,
    the call behind mx::quantize at ESExperts.mm:14,16), restated in numpy
    float32 independently of the C oracle."""
    f = np.float32
    n = f((1 << bits) - 1)
    g = wf.reshape(wf.shape[0], -1, gs).astype(f)
    mx, mn = g.max(-1), g.min(-1)
    mask = np.abs(mn) > np.abs(mx)
    sc = np.maximum((mx - mn) / n, f(1e-7)).astype(f)
    sc = np.where(mask, sc, -sc).astype(f)
    edge = np.where(mask, mn, mx).astype(f)
    q0 = np.rint(edge / sc).astype(f)
    sc = np.where(q0 != 0, edge / np.where(q0 != 0, q0, f(1)), sc).astype(f)
    bi = np.where(q0 == 0, f(0), edge).astype(f)
    q = np.clip(np.rint((g - bi[..., None]) / sc[..., None]), 0, n).astype(np.uint32)
    return q.reshape(wf.shape), sc, bi


def test_quantize_matches_mlx_rule(oracle):
    rng = np.random.default_rng(5)
    w = oracle.f32_to_bf16(rng.standard_normal((64, 256), dtype=np.float32) * 0.02)
    w[3, :64] = oracle.f32_to_bf16(np.abs(rng.standard_normal(64, dtype=np.float32)))  # all > 0
    w[4, :64] = 0  # a constant group: scale 1e-7 path
    wf = oracle.bf16_to_f32(w)
    for bits in (4, 8):
        q, s, b = oracle.quantize_affine(w, 64, bits)
        qr, sr, br = _mlx_affine_py(wf, 64, bits)
        per = 32 // bits
        codes = np.stack([(q >> (bits * l)) & ((1 << bits) - 1) for l in range(per)], -1)
        codes = codes.reshape(q.shape[0], -1)  # low bits first
        np.testing.assert_array_equal(codes, qr)
        np.testing.assert_array_equal(s, oracle.f32_to_bf16(sr))
        np.testing.assert_array_equal(b, oracle.f32_to_bf16(br))
        # the scale is negative exactly where the group's max has the larger magnitude
        g = wf.reshape(64, -1, 64)
        neg = np.abs(g.min(-1)) <= np.abs(g.max(-1))
        sf = oracle.bf16_to_f32(s)
        assert np.all((sf < 0)[neg & (sf != 0)]) and np.all((sf > 0)[~neg])


def test_quantize_roundtrip(oracle):
    rng = np.random.default_rng(5)
    w = oracle.f32_to_bf16(rng.standard_normal((8, 256), dtype=np.float32) * 0.02)
    for bits in (4, 8):
        q, s, b = oracle.quantize_affine(w, 64, bits)
        assert q.shape == (8, 256 * bits // 32) and s.shape == (8, 4)
        deq = oracle.dequantize_affine(q, s, b, 64, bits)
        wf = oracle.bf16_to_f32(w)
        step = np.abs(oracle.bf16_to_f32(s)).repeat(64, axis=1)
        # within one step (half a step, plus the clip at the far end after the
        # scale was moved so that zero falls on a code) + bf16 rounding
        assert np.all(np.abs(deq - wf) <= step + 2e-4)
        assert np.mean(np.abs(deq - wf) <= 0.5 * step + 2e-4) > 0.99
        # packing: element 0 of row 0 sits in the low bits of word 0
        q0 = int(q[0, 0]) & ((1 << bits) - 1)
        ref = (wf[0, 0] - oracle.bf16_to_f32(b)[0, 0]) / oracle.bf16_to_f32(s)[0, 0]
        assert abs(q0 - ref) <= 0.5 + 2e-2


def test_quantized_experts_close_to_bf16(oracle):
    """testQuantizedLinearCloseToBf16 (ESPrimitivesTests.mm:157-169) for experts:
    the quantised block stays within 5 % of peak of the bf16 block (8-bit)
    and 20 % (4-bit: MLX moves each group's scale so that zero is a code, which
    clips the far end of some groups by up to ~0.7 of a step)."""
    d = load("small")
    idx, w = oracle.route_topk(d["x"], d["proj"], d["scale"], d["pes"], int(d["K"]))
    ref = oracle.bf16_to_f32(oracle.experts_sparse(d["x"], d["gate_up"], d["down"], idx, w))
    peak = np.abs(ref).max()
    for bits, tol in ((8, 0.05), (4, 0.20)):
        gq = oracle.quantize_affine(d["gate_up"], 64, bits)
        dq = oracle.quantize_affine(d["down"], 64, bits)
        got = oracle.bf16_to_f32(oracle.experts_sparse_q(d["x"], *gq, *dq, bits, 64, idx, w,
                                                         int(d["I"])))
        assert np.abs(got - ref).max() <= tol * peak
