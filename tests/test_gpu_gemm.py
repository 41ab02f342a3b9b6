"""tcgen05 grouped-GEMM path (prefill-sized groups) vs the CPU oracle and vs
the GEMV path.  The GEMM path is forced with set_gemv_max_tokens(0)."""
import numpy as np
import pytest
import torch

from tests.helpers import bf16_to_f32, block_close

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import apertura_b200 as A  # noqa: E402
from apertura_b200.synthetic import block_inputs, to_numpy_bits as _np  # noqa: E402

DEV = torch.device("cuda", 0)
TIGHT_REL = 2.0 ** -6


def _block(d, T):
    cfg = A.ESModelConfig(hidden_size=d["H"], num_experts=d["E"], top_k_experts=d["K"],
                          moe_intermediate_size=d["I"], moe_sparse=True, max_tokens=T)
    return A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], d["gate_up"], d["down"])


def _run(blk, x, gemv_max):
    blk.handle.set_gemv_max_tokens(gemv_max)
    out, tk = blk.forward(x, return_routing=True)
    torch.cuda.synchronize()
    blk.handle.sync()  # raises if a bounded device wait gave up
    return out, tk


@pytest.mark.parametrize("shape,T", [((256, 32, 8, 128), 100), ((2816, 128, 8, 704), 48),
                                     ((2816, 128, 8, 704), 300)])
def test_gemm_vs_oracle(oracle, shape, T):
    H, E, K, I = shape
    d = block_inputs(T, seed=60 + T, device=DEV, H=H, E=E, K=K, I=I)
    blk = _block(d, T)
    out, tk = _run(blk, d["x"], 0)
    ref = oracle.experts_sparse(_np(d["x"]), _np(d["gate_up"]), _np(d["down"]),
                                tk.idx.cpu().numpy(), _np(tk.w))
    got, refv = bf16_to_f32(_np(out)), bf16_to_f32(ref)
    ok, ma, cos = block_close(got, refv)
    assert ok and ma <= TIGHT_REL * np.abs(refv).max(), (ma, cos)


def test_gemm_matches_gemv_zipf():
    """Skewed routing (Zipf 1.1): hot experts span many m-tiles, cold ones one
    partial tile; both paths must agree to a few bf16 ulps."""
    T = 2048
    d = block_inputs(T, seed=3, device=DEV, routing="zipf")
    blk = _block(d, T)
    a, tk = _run(blk, d["x"], 0)
    a = a.clone()
    b, tk2 = _run(blk, d["x"], 1 << 30)
    assert torch.equal(tk.idx, tk2.idx)
    fa, fb = bf16_to_f32(_np(a)), bf16_to_f32(_np(b))
    ok, ma, cos = block_close(fa, fb)
    assert ok and ma <= TIGHT_REL * np.abs(fb).max(), (ma, cos)
    counts = blk.handle.last_counts().numpy()
    assert counts.max() > 4 * 128  # the hot expert really spans several m-tiles


def test_gemm_prefill_vs_oracle(oracle):
    """BASELINE config 3 (T=8192, Zipf s=1.1) through the tensor-core router
    and the tcgen05 experts: every token's indices against the oracle's
    ESRouter::routeTopK (bit-exact but for one-bf16-ulp ties, whose share is
    reported), then the block on 256 sampled tokens against the oracle's
    experts run on the ORACLE's own routing."""
    from tests.helpers import router_index_check
    T = 8192
    d = block_inputs(T, seed=9, device=DEV, routing="zipf")
    blk = _block(d, T)
    out, tk = _run(blk, d["x"], 0)
    idx = tk.idx.cpu().numpy()
    idx_o, w_o, aux = oracle.route_topk(_np(d["x"]), _np(d["proj"]), _np(d["scale"]),
                                        _np(d["pes"]), 8, return_scores=True)
    bad, exempt = router_index_check(idx, idx_o, aux["scores"])
    print(f"T=8192 Zipf: {exempt} of {T} tokens exempt as one-ulp ties "
          f"({100.0 * exempt / T:.2f} %)")
    assert bad == 0, f"{bad} non-tie index mismatches (exempt {exempt})"
    assert exempt <= T // 20
    same = np.nonzero(np.all(idx == idx_o, axis=1))[0]
    rng = np.random.default_rng(0)
    rows = np.sort(rng.choice(same, 256, replace=False))
    ref = oracle.experts_sparse(_np(d["x"][rows]), _np(d["gate_up"]), _np(d["down"]),
                                idx_o[rows], w_o[rows])
    got, refv = bf16_to_f32(_np(out))[rows], bf16_to_f32(ref)
    ok, ma, cos = block_close(got, refv)
    assert ok and ma <= TIGHT_REL * np.abs(refv).max(), (ma, cos)


def test_experts_grouped_in_place(oracle):
    """apt_moe_experts_grouped (the expert-parallel remote step): rows in G
    groups, group g on expert g2e[g], unweighted outputs in row order."""
    import ctypes
    H, E, I = 2816, 16, 704
    d = block_inputs(4, seed=31, device=DEV, H=H, E=E, K=4, I=I)
    rng = np.random.default_rng(4)
    G = 32
    counts = rng.integers(0, 40, size=G).astype(np.int32)
    counts[5] = 0
    g2e = rng.integers(0, E, size=G).astype(np.int32)
    R = int(counts.sum())
    rows = torch.randn(R, H, device=DEV).to(torch.bfloat16)
    cfg = A.ESModelConfig(hidden_size=H, num_experts=E, top_k_experts=1, moe_intermediate_size=I,
                          moe_sparse=True, max_tokens=R)
    h = A.Handle(cfg)
    ex = A.ESExperts(d["gate_up"], d["down"], handle=h)
    out = torch.empty_like(rows)
    c_t = torch.from_numpy(counts).to(DEV)
    g_t = torch.from_numpy(g2e).to(DEV)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    h.check(A.lib().apt_moe_experts_grouped(h.h, P(rows), R, P(c_t), P(g_t), G, P(out), None))
    torch.cuda.synchronize()
    h.sync()
    ids = np.repeat(g2e, counts).reshape(R, 1).astype(np.int32)
    ones = oracle.f32_to_bf16(np.ones((R, 1), np.float32))
    ref = oracle.experts_sparse(_np(rows), _np(d["gate_up"]), _np(d["down"]), ids, ones)
    got, refv = bf16_to_f32(_np(out)), bf16_to_f32(ref)
    ok, ma, cos = block_close(got, refv)
    assert ok and ma <= TIGHT_REL * np.abs(refv).max(), (ma, cos)
    del ex


def test_prefill_outputs_bitwise_deterministic():
    """Rows take atomically claimed slots inside their expert group, so the
    row order varies between calls; the outputs must not."""
    T = 2048
    d = block_inputs(T, seed=8, device=DEV, routing="zipf")
    blk = _block(d, T)
    a, _ = _run(blk, d["x"], 0)
    a = a.clone()
    for _ in range(2):
        b, _ = _run(blk, d["x"], 0)
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
