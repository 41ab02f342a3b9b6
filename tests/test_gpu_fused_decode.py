"""The one-kernel decode block (decode_fused.cu: router, dispatch, gate_up,
down and the k-order combine in one persistent launch, T <= 8) against the
CPU oracle and against the kernel chain it replaces.

Calls are repeated with new tokens so the kernel's self re-arming counters
are exercised, and the router and expert inputs are also given as distinct
tensors (the MoE section of ESDecoderLayer::forward, ESDecoderLayer.mm:67-75)."""
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
TIGHT_REL = 2.0 ** -6


def _block(d, T):
    cfg = A.ESModelConfig(hidden_size=d["H"], num_experts=d["E"], top_k_experts=d["K"],
                          moe_intermediate_size=d["I"], moe_sparse=True, max_tokens=T)
    return A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], d["gate_up"], d["down"])


@pytest.mark.parametrize("T", [1, 2, 3, 4, 5, 8])
def test_fused_decode_vs_oracle_repeated(oracle, T):
    d = block_inputs(3 * T, seed=500 + T, device=DEV, nonunit=True)
    blk = _block(d, T)
    for call in range(3):
        x = d["x"][call * T:(call + 1) * T].contiguous()
        out, tk = blk.forward(x, return_routing=True)
        torch.cuda.synchronize()
        blk.handle.sync()
        assert blk.handle.last_launches() == 1  # the whole block is one kernel
        idx = tk.idx.cpu().numpy()
        idx_o, w_o, aux = oracle.route_topk(_np(x), _np(d["proj"]), _np(d["scale"]),
                                            _np(d["pes"]), d["K"], return_scores=True)
        bad, exempt = router_index_check(idx, idx_o, aux["scores"])
        assert bad == 0, (bad, exempt)
        same = np.all(idx == idx_o, axis=1)
        w = bf16_to_f32(_np(tk.w))
        wo = bf16_to_f32(w_o)
        assert np.all(np.abs(w[same] - wo[same]) <= np.abs(wo[same]) * 2.0 ** -7 + 1e-9)
        ref = oracle.experts_sparse(_np(x), _np(d["gate_up"]), _np(d["down"]), idx, _np(tk.w))
        got, refv = bf16_to_f32(_np(out)), bf16_to_f32(ref)
        ok, ma, cos = block_close(got, refv)
        assert ok and ma <= TIGHT_REL * np.abs(refv).max(), (call, ma, cos)


@pytest.mark.parametrize("T", [1, 4, 8])
def test_fused_decode_matches_chain(T):
    d = block_inputs(T, seed=900 + T, device=DEV)
    blk = _block(d, T)
    a, ta = blk.forward(d["x"], return_routing=True)
    a = a.clone()
    blk.handle.set_fused_decode(False)
    b, tb = blk.forward(d["x"], return_routing=True)
    torch.cuda.synchronize()
    assert blk.handle.last_launches() > 1
    blk.handle.set_fused_decode(True)
    same = torch.all(ta.idx == tb.idx, dim=1).cpu().numpy()
    assert same.mean() >= 0.75  # the rest: router ties broken by f32 summation order
    fa, fb = bf16_to_f32(_np(a))[same], bf16_to_f32(_np(b))[same]
    assert np.abs(fa - fb).max() <= TIGHT_REL * np.abs(fb).max()


def test_fused_decode_distinct_expert_input(oracle):
    """Router on x1, experts on another tensor (apt_moe_forward's two inputs)."""
    T = 6
    d = block_inputs(T, seed=77, device=DEV)
    xe = (d["x"].float() * 0.5 + 0.1).to(torch.bfloat16)
    blk = _block(d, T)
    out, tk = blk.forward_layer(d["x"], xe, return_routing=True)
    torch.cuda.synchronize()
    blk.handle.sync()
    ref = oracle.experts_sparse(_np(xe), _np(d["gate_up"]), _np(d["down"]), tk.idx.cpu().numpy(),
                                _np(tk.w))
    got, refv = bf16_to_f32(_np(out)), bf16_to_f32(ref)
    ok, ma, cos = block_close(got, refv)
    assert ok and ma <= TIGHT_REL * np.abs(refv).max(), (ma, cos)


def test_fused_decode_host_graph_replay():
    """apt_moe_forward_host replays a captured graph of the fused kernel."""
    T = 4
    d = block_inputs(2 * T, seed=31, device=DEV)
    blk = _block(d, T)
    for call in range(2):
        xh = d["x"][call * T:(call + 1) * T].cpu().pin_memory()
        oh = torch.empty(T, d["H"], dtype=torch.bfloat16).pin_memory()
        for _ in range(2):
            blk.forward_host(xh, oh)
        ref_out = blk.forward(xh.to(DEV))
        torch.cuda.synchronize()
        assert torch.equal(oh.view(torch.int16), ref_out.cpu().view(torch.int16))


def _quant_block(oracle, d, T, bits):
    gq = oracle.quantize_affine(_np(d["gate_up"]), 64, bits)
    dq = oracle.quantize_affine(_np(d["down"]), 64, bits)

    def dev(a):
        a = np.ascontiguousarray(a)
        if a.dtype == np.uint16:
            return torch.from_numpy(a.view(np.int16)).to(DEV).view(torch.bfloat16)
        return torch.from_numpy(a.view(np.int32)).to(DEV)

    cfg = A.ESModelConfig(hidden_size=d["H"], num_experts=d["E"], top_k_experts=d["K"],
                          moe_intermediate_size=d["I"], moe_sparse=True, max_tokens=T)
    q = dict(gu_q=dev(gq[0]), gu_s=dev(gq[1]), gu_b=dev(gq[2]), dn_q=dev(dq[0]),
             dn_s=dev(dq[1]), dn_b=dev(dq[2]), bits=bits, group_size=64)
    return A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], quantized=q), gq, dq


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("T", [1, 3, 8])
def test_fused_decode_quant_vs_oracle(oracle, bits, T):
    """MLX affine experts (gather_qmm, ESExperts.mm:50-57) through the one-kernel
    block: repeated calls against the oracle on the same packed weights."""
    d = block_inputs(2 * T, seed=700 + T + bits, device=DEV)
    blk, gq, dq = _quant_block(oracle, d, T, bits)
    for call in range(2):
        x = d["x"][call * T:(call + 1) * T].contiguous()
        out, tk = blk.forward(x, return_routing=True)
        torch.cuda.synchronize()
        blk.handle.sync()
        assert blk.handle.last_launches() == 1
        ref = oracle.experts_sparse_q(_np(x), *gq, *dq, bits, 64, tk.idx.cpu().numpy(),
                                      _np(tk.w), d["I"])
        got, refv = bf16_to_f32(_np(out)), bf16_to_f32(ref)
        ok, ma, cos = block_close(got, refv)
        assert ok and ma <= TIGHT_REL * np.abs(refv).max(), (call, ma, cos)


@pytest.mark.parametrize("bits", [4, 8])
def test_fused_decode_quant_matches_chain(oracle, bits):
    T = 4
    d = block_inputs(T, seed=910 + bits, device=DEV)
    blk, _, _ = _quant_block(oracle, d, T, bits)
    a, ta = blk.forward(d["x"], return_routing=True)
    a = a.clone()
    blk.handle.set_fused_decode(False)
    b, tb = blk.forward(d["x"], return_routing=True)
    torch.cuda.synchronize()
    assert blk.handle.last_launches() > 1
    blk.handle.set_fused_decode(True)
    same = torch.all(ta.idx == tb.idx, dim=1).cpu().numpy()
    assert same.mean() >= 0.75
    fa, fb = bf16_to_f32(_np(a))[same], bf16_to_f32(_np(b))[same]
    assert np.abs(fa - fb).max() <= TIGHT_REL * np.abs(fb).max()
