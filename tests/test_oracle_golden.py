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


def test_quantize_roundtrip(oracle):
    rng = np.random.default_rng(5)
    w = oracle.f32_to_bf16(rng.standard_normal((8, 256), dtype=np.float32) * 0.02)
    for bits in (4, 8):
        q, s, b = oracle.quantize_affine(w, 64, bits)
        assert q.shape == (8, 256 * bits // 32) and s.shape == (8, 4)
        deq = oracle.dequantize_affine(q, s, b, 64, bits)
        wf = oracle.bf16_to_f32(w)
        step = oracle.bf16_to_f32(s).repeat(64, axis=1)
        # every element within half a step (+ bf16 rounding of scale/bias)
        assert np.all(np.abs(deq - wf) <= 0.5 * step + 2e-4)
        # packing: element 0 of row 0 sits in the low bits of word 0
        q0 = int(q[0, 0]) & ((1 << bits) - 1)
        ref = (wf[0, 0] - oracle.bf16_to_f32(b)[0, 0]) / oracle.bf16_to_f32(s)[0, 0]
        assert abs(q0 - ref) <= 0.5 + 1e-3


def test_quantized_experts_close_to_bf16(oracle):
    """testQuantizedLinearCloseToBf16 (ESPrimitivesTests.mm:157-169) for experts:
    the quantised block stays within 5 % of peak of the bf16 block (8-bit)
    and 15 % (4-bit)."""
    d = load("small")
    idx, w = oracle.route_topk(d["x"], d["proj"], d["scale"], d["pes"], int(d["K"]))
    ref = oracle.bf16_to_f32(oracle.experts_sparse(d["x"], d["gate_up"], d["down"], idx, w))
    peak = np.abs(ref).max()
    for bits, tol in ((8, 0.05), (4, 0.15)):
        gq = oracle.quantize_affine(d["gate_up"], 64, bits)
        dq = oracle.quantize_affine(d["down"], 64, bits)
        got = oracle.bf16_to_f32(oracle.experts_sparse_q(d["x"], *gq, *dq, bits, 64, idx, w,
                                                         int(d["I"])))
        assert np.abs(got - ref).max() <= tol * peak
