"""The MoE half of ESDecoderLayer::forward with its norms
(apt_moe_layer_forward): post_ff_ln_2(experts(pre_ff_ln_2(x1), router(x1)))
vs the oracle, on the fused decode router, the tensor-core prefill router and
the small-shape path (standalone RMSNorm)."""
import numpy as np
import pytest
import torch

from tests.helpers import bf16_to_f32, block_close, router_index_check

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import apertura_b200 as A  # noqa: E402
from apertura_b200.synthetic import block_inputs, to_numpy_bits as _np  # noqa: E402

DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("shape,T,sparse", [((2816, 128, 8, 704), 3, True),
                                            ((2816, 128, 8, 704), 100, True),
                                            ((2816, 128, 8, 704), 5, False),
                                            ((2816, 128, 8, 704), 400, True),
                                            ((64, 16, 4, 64), 7, True)])
def test_layer_forward_with_norms(oracle, shape, T, sparse):
    H, E, K, I = shape
    d = block_inputs(T, seed=T + H, device=DEV, H=H, E=E, K=K, I=I, nonunit=True)
    g = torch.Generator(device=DEV).manual_seed(5)
    pre = (1 + 0.2 * torch.randn(H, generator=g, device=DEV)).to(torch.bfloat16)
    post = (1 + 0.2 * torch.randn(H, generator=g, device=DEV)).to(torch.bfloat16)
    cfg = A.ESModelConfig(hidden_size=H, num_experts=E, top_k_experts=K, moe_intermediate_size=I,
                          moe_sparse=sparse, max_tokens=T)
    blk = A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], d["gate_up"], d["down"])
    out = blk.forward_with_norms(d["x"], pre, post)
    # routing of the same call, for the tie-aware comparison
    _, tk = blk.forward(d["x"], return_routing=True)
    torch.cuda.synchronize()
    ref, idx_ref, _ = oracle.layer_moe(_np(d["x"]), _np(pre), _np(post), _np(d["proj"]),
                                       _np(d["scale"]), _np(d["pes"]), _np(d["gate_up"]),
                                       _np(d["down"]), K)
    _, _, aux = oracle.route_topk(_np(d["x"]), _np(d["proj"]), _np(d["scale"]), _np(d["pes"]), K,
                                  return_scores=True)
    bad, _ = router_index_check(tk.idx.cpu().numpy(), idx_ref, aux["scores"])
    assert bad == 0
    same = np.all(tk.idx.cpu().numpy() == idx_ref, axis=1)
    got, refv = bf16_to_f32(_np(out))[same], bf16_to_f32(ref)[same]
    # post_ff_ln_2 renormalises each row to unit RMS (times the weight): the
    # outputs are O(1), where one bf16 ulp exceeds the block bar's 2e-2, so
    # max-abs is held to a couple of ulps of the largest output instead
    peak = np.abs(refv).max()
    ok, ma, cos = block_close(got, refv, max_abs=2.0 ** -6 * peak)
    assert ok, (ma, cos, peak)


@pytest.mark.parametrize("shape,T", [((2816, 128, 8, 704), 4), ((2816, 128, 8, 704), 80),
                                     ((2816, 128, 8, 704), 400), ((64, 16, 4, 64), 7)])
def test_decoder_ff_tail(oracle, shape, T):
    """apt_moe_decoder_ff: x2 = x1 + post_ff_ln(post_ff_ln_1(hmlp) + post_ff_ln_2(MoE(x1)))."""
    H, E, K, I = shape
    d = block_inputs(T, seed=3 * T + H, device=DEV, H=H, E=E, K=K, I=I, nonunit=True)
    g = torch.Generator(device=DEV).manual_seed(6)
    ws = [(1 + 0.2 * torch.randn(H, generator=g, device=DEV)).to(torch.bfloat16) for _ in range(4)]
    pre, ln1, post, lnf = ws
    hmlp = (0.5 * torch.randn(T, H, generator=g, device=DEV)).to(torch.bfloat16)
    cfg = A.ESModelConfig(hidden_size=H, num_experts=E, top_k_experts=K, moe_intermediate_size=I,
                          moe_sparse=True, max_tokens=T)
    blk = A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], d["gate_up"], d["down"])
    x2 = blk.forward_decoder_ff(d["x"], hmlp, pre, ln1, post, lnf)
    _, tk = blk.forward(d["x"], return_routing=True)
    torch.cuda.synchronize()
    ref, idx_ref, _ = oracle.decoder_ff(_np(d["x"]), _np(hmlp), _np(pre), _np(ln1), _np(post),
                                        _np(lnf), _np(d["proj"]), _np(d["scale"]), _np(d["pes"]),
                                        _np(d["gate_up"]), _np(d["down"]), K)
    _, _, aux = oracle.route_topk(_np(d["x"]), _np(d["proj"]), _np(d["scale"]), _np(d["pes"]), K,
                                  return_scores=True)
    bad, _ = router_index_check(tk.idx.cpu().numpy(), idx_ref, aux["scores"])
    assert bad == 0
    same = np.all(tk.idx.cpu().numpy() == idx_ref, axis=1)
    got, refv = bf16_to_f32(_np(x2))[same], bf16_to_f32(ref)[same]
    peak = np.abs(refv).max()
    ok, ma, cos = block_close(got, refv, max_abs=2.0 ** -6 * peak)
    assert ok, (ma, cos, peak)


@pytest.mark.parametrize("T", [1, 5, 96])
def test_dense_mlp(oracle, T):
    """MLPBlock (ESMLPBlock): GEMV path for small T, tensor-core path above."""
    H, I = 2816, 2112
    g = torch.Generator(device=DEV).manual_seed(7 + T)
    gate = (0.02 * torch.randn(I, H, generator=g, device=DEV)).to(torch.bfloat16)
    up = (0.02 * torch.randn(I, H, generator=g, device=DEV)).to(torch.bfloat16)
    down = (0.02 * torch.randn(H, I, generator=g, device=DEV)).to(torch.bfloat16)
    x = torch.randn(T, H, generator=g, device=DEV).to(torch.bfloat16)
    mlp = A.MLPBlock(gate, up, down, hidden_size=H, intermediate_size=I, max_tokens=128)
    out = mlp(x)
    torch.cuda.synchronize()
    mlp.handle.sync()
    ref = oracle.mlp(_np(x), _np(gate), _np(up), _np(down))
    got, refv = bf16_to_f32(_np(out)), bf16_to_f32(ref)
    ok, ma, cos = block_close(got, refv)
    assert ok and ma <= 2.0 ** -6 * np.abs(refv).max(), (ma, cos)


@pytest.mark.parametrize("T", [4, 80, 320])
def test_decoder_ff_full(oracle, T):
    """apt_moe_decoder_ff_full: the layer's whole feed-forward half from x1."""
    H, E, K, I, Id = 2816, 128, 8, 704, 2112
    d = block_inputs(T, seed=11 * T, device=DEV, H=H, E=E, K=K, I=I, nonunit=True)
    g = torch.Generator(device=DEV).manual_seed(9)
    ws = [(1 + 0.2 * torch.randn(H, generator=g, device=DEV)).to(torch.bfloat16) for _ in range(5)]
    pre_ff, pre2, ln1, post, lnf = ws
    gate = (0.02 * torch.randn(Id, H, generator=g, device=DEV)).to(torch.bfloat16)
    up = (0.02 * torch.randn(Id, H, generator=g, device=DEV)).to(torch.bfloat16)
    down = (0.02 * torch.randn(H, Id, generator=g, device=DEV)).to(torch.bfloat16)
    cfg = A.ESModelConfig(hidden_size=H, num_experts=E, top_k_experts=K, moe_intermediate_size=I,
                          moe_sparse=True, max_tokens=T)
    blk = A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], d["gate_up"], d["down"])
    mlp = A.MLPBlock(gate, up, down, hidden_size=H, intermediate_size=Id, max_tokens=T)
    x2 = blk.forward_decoder_ff_full(d["x"], mlp, pre_ff, pre2, ln1, post, lnf)
    _, tk = blk.forward(d["x"], return_routing=True)
    torch.cuda.synchronize()
    ref, idx_ref, _ = oracle.decoder_ff_full(_np(d["x"]), _np(pre_ff), _np(gate), _np(up),
                                             _np(down), _np(pre2), _np(ln1), _np(post), _np(lnf),
                                             _np(d["proj"]), _np(d["scale"]), _np(d["pes"]),
                                             _np(d["gate_up"]), _np(d["down"]), K)
    _, _, aux = oracle.route_topk(_np(d["x"]), _np(d["proj"]), _np(d["scale"]), _np(d["pes"]), K,
                                  return_scores=True)
    bad, _ = router_index_check(tk.idx.cpu().numpy(), idx_ref, aux["scores"])
    assert bad == 0
    same = np.all(tk.idx.cpu().numpy() == idx_ref, axis=1)
    got, refv = bf16_to_f32(_np(x2))[same], bf16_to_f32(ref)[same]
    peak = np.abs(refv).max()
    ok, ma, cos = block_close(got, refv, max_abs=2.0 ** -6 * peak)
    assert ok, (ma, cos, peak)
