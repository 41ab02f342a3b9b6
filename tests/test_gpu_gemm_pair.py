"""CTA-pair tcgen05 GEMM (cta_group::2, M=256 tiles over two SMs) against
the single-CTA GEMM, the GEMV path and the CPU oracle."""
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


def _run(blk, x, pair, gemv_max=0):
    blk.handle.set_gemv_max_tokens(gemv_max)
    blk.handle.set_gemm_pair(pair)
    out, tk = blk.forward(x, return_routing=True)
    torch.cuda.synchronize()
    blk.handle.sync()  # raises if a bounded device wait gave up
    return out.clone(), tk


@pytest.mark.parametrize("shape,T", [((256, 32, 8, 128), 100), ((2816, 128, 8, 704), 48),
                                     ((2816, 128, 8, 704), 300)])
def test_pair_vs_oracle(oracle, shape, T):
    H, E, K, I = shape
    d = block_inputs(T, seed=70 + T, device=DEV, H=H, E=E, K=K, I=I)
    blk = _block(d, T)
    out, tk = _run(blk, d["x"], 1)
    ref = oracle.experts_sparse(_np(d["x"]), _np(d["gate_up"]), _np(d["down"]),
                                tk.idx.cpu().numpy(), _np(tk.w))
    got, refv = bf16_to_f32(_np(out)), bf16_to_f32(ref)
    ok, ma, cos = block_close(got, refv)
    assert ok and ma <= TIGHT_REL * np.abs(refv).max(), (ma, cos)


@pytest.mark.parametrize("T,routing", [(300, "uniform"), (2048, "zipf"), (8192, "zipf")])
def test_pair_matches_single(T, routing):
    """Same k order and rounding points: the two tile forms agree bitwise."""
    d = block_inputs(T, seed=5 + T, device=DEV, routing=routing)
    blk = _block(d, T)
    a, tk = _run(blk, d["x"], 1)
    b, tk2 = _run(blk, d["x"], 0)
    assert torch.equal(tk.idx, tk2.idx)
    if not torch.equal(a, b):
        fa, fb = bf16_to_f32(_np(a)), bf16_to_f32(_np(b))
        ok, ma, cos = block_close(fa, fb)
        assert ok and ma <= TIGHT_REL * np.abs(fb).max(), (ma, cos)


def test_pair_grouped_in_place(oracle):
    """apt_moe_experts_grouped (the expert-parallel step) on the pair kernel:
    groups map to experts out of order and repeat; vs the oracle and the
    single-CTA kernel."""
    import ctypes
    H, E, I = 2816, 16, 704
    d = block_inputs(4, seed=32, device=DEV, H=H, E=E, K=4, I=I)
    rng = np.random.default_rng(5)
    G = 32
    counts = rng.integers(0, 300, size=G).astype(np.int32)
    counts[3] = 0
    g2e = rng.integers(0, E, size=G).astype(np.int32)
    R = int(counts.sum())
    rows = torch.randn(R, H, device=DEV).to(torch.bfloat16)
    cfg = A.ESModelConfig(hidden_size=H, num_experts=E, top_k_experts=1, moe_intermediate_size=I,
                          moe_sparse=True, max_tokens=R)
    h = A.Handle(cfg)
    ex = A.ESExperts(d["gate_up"], d["down"], handle=h)
    c_t = torch.from_numpy(counts).to(DEV)
    g_t = torch.from_numpy(g2e).to(DEV)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    outs = []
    for pair in (1, 0):
        h.set_gemm_pair(pair)
        out = torch.empty_like(rows)
        h.check(A.lib().apt_moe_experts_grouped(h.h, P(rows), R, P(c_t), P(g_t), G, P(out), None))
        torch.cuda.synchronize()
        h.sync()
        outs.append(out)
    ids = np.repeat(g2e, counts).reshape(R, 1).astype(np.int32)
    ones = oracle.f32_to_bf16(np.ones((R, 1), np.float32))
    sel = np.sort(rng.choice(R, 256, replace=False))
    ref = oracle.experts_sparse(_np(rows[sel]), _np(d["gate_up"]), _np(d["down"]), ids[sel],
                                ones[sel])
    got, refv = bf16_to_f32(_np(outs[0]))[sel], bf16_to_f32(ref)
    ok, ma, cos = block_close(got, refv)
    assert ok and ma <= TIGHT_REL * np.abs(refv).max(), (ma, cos)
    assert torch.equal(outs[0], outs[1])
    del ex
