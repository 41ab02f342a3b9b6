"""MLX-format affine expert weights (gather_qmm path of ESExperts::sparseForward,
aptransformer/ESExperts.mm:50-57) through the CUDA path vs the CPU oracle.

Both sides consume the same packed (q, scales, biases): quantised once by the
oracle and adopted verbatim (the bundle constructor), or quantised on the
device at load (the quantBits > 0 constructor), which must reproduce the
oracle's packing bit for bit."""
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


def _dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).to(DEV).view(torch.bfloat16)
    return torch.from_numpy(a.view(np.int32)).to(DEV)


def _quantize(oracle, d, bits):
    gq = oracle.quantize_affine(_np(d["gate_up"]), 64, bits)
    dq = oracle.quantize_affine(_np(d["down"]), 64, bits)
    return gq, dq


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("shape,T", [((256, 32, 8, 128), 5), ((2816, 128, 8, 704), 1),
                                     ((2816, 128, 8, 704), 4)])
def test_bundle_quant_parity(oracle, bits, shape, T):
    H, E, K, I = shape
    d = block_inputs(T, seed=21 + T, device=DEV, H=H, E=E, K=K, I=I)
    gq, dq = _quantize(oracle, d, bits)
    cfg = A.ESModelConfig(hidden_size=H, num_experts=E, top_k_experts=K, moe_intermediate_size=I,
                          moe_sparse=True, max_tokens=T)
    q = dict(gu_q=_dev(gq[0]), gu_s=_dev(gq[1]), gu_b=_dev(gq[2]), dn_q=_dev(dq[0]),
             dn_s=_dev(dq[1]), dn_b=_dev(dq[2]), bits=bits, group_size=64)
    blk = A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], quantized=q)
    out, tk = blk.forward(d["x"], return_routing=True)
    torch.cuda.synchronize()
    ref = oracle.experts_sparse_q(_np(d["x"]), *gq, *dq, bits, 64, tk.idx.cpu().numpy(),
                                  _np(tk.w), I)
    got, refv = bf16_to_f32(_np(out)), bf16_to_f32(ref)
    ok, ma, cos = block_close(got, refv)
    assert ok and ma <= TIGHT_REL * np.abs(refv).max(), (ma, cos)


@pytest.mark.parametrize("bits", [4, 8])
def test_device_quantize_matches_oracle(oracle, bits):
    """quantBits>0 ctor: the device quantiser must equal the oracle's packing,
    so the block equals the oracle run on oracle-quantised weights."""
    H, E, K, I, T = 256, 32, 8, 128, 6
    d = block_inputs(T, seed=5, device=DEV, H=H, E=E, K=K, I=I)
    gq, dq = _quantize(oracle, d, bits)
    cfg = A.ESModelConfig(hidden_size=H, num_experts=E, top_k_experts=K, moe_intermediate_size=I,
                          moe_sparse=True, quant_bits=bits, max_tokens=T)
    blk = A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], d["gate_up"], d["down"])
    out, tk = blk.forward(d["x"], return_routing=True)
    torch.cuda.synchronize()
    ref = oracle.experts_sparse_q(_np(d["x"]), *gq, *dq, bits, 64, tk.idx.cpu().numpy(),
                                  _np(tk.w), I)
    got, refv = bf16_to_f32(_np(out)), bf16_to_f32(ref)
    assert np.abs(got - refv).max() <= TIGHT_REL * np.abs(refv).max()


def test_quant_bundle_has_no_dense_path():
    H, E, K, I, T = 256, 32, 8, 128, 2
    d = block_inputs(T, seed=1, device=DEV, H=H, E=E, K=K, I=I)
    from oracle import oracle as O
    gq = O.quantize_affine(_np(d["gate_up"]), 64, 4)
    dq = O.quantize_affine(_np(d["down"]), 64, 4)
    cfg = A.ESModelConfig(hidden_size=H, num_experts=E, top_k_experts=K, moe_intermediate_size=I,
                          moe_sparse=False, max_tokens=T)
    q = dict(gu_q=_dev(gq[0]), gu_s=_dev(gq[1]), gu_b=_dev(gq[2]), dn_q=_dev(dq[0]),
             dn_s=_dev(dq[1]), dn_b=_dev(dq[2]), bits=4, group_size=64)
    blk = A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], quantized=q)
    with pytest.raises(A.AptError) as ei:
        blk.forward(d["x"])
    assert ei.value.status == 6


@pytest.mark.parametrize("bits", [4, 8])
def test_quant_prefill_tensor_core_path(oracle, bits):
    """Prefill-sized T with quantised experts: the touched experts are expanded
    to bf16 (w = bf16(scale*q + bias)) and run on the tcgen05 GEMM.  Compared
    with the oracle's f32 dequantisation on a sample of tokens; the extra bf16
    rounding of w stays inside a few output ulps."""
    H, E, K, I, T = 2816, 128, 8, 704, 1024
    d = block_inputs(T, seed=77, device=DEV, routing="zipf", H=H, E=E, K=K, I=I)
    gq, dq = _quantize(oracle, d, bits)
    cfg = A.ESModelConfig(moe_sparse=True, max_tokens=T)
    q = dict(gu_q=_dev(gq[0]), gu_s=_dev(gq[1]), gu_b=_dev(gq[2]), dn_q=_dev(dq[0]),
             dn_s=_dev(dq[1]), dn_b=_dev(dq[2]), bits=bits, group_size=64)
    blk = A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], quantized=q)
    out, tk = blk.forward(d["x"], return_routing=True)
    torch.cuda.synchronize()
    blk.handle.sync()
    rows = np.sort(np.random.default_rng(1).choice(T, 16, replace=False))
    ref = oracle.experts_sparse_q(_np(d["x"][rows]), *gq, *dq, bits, 64,
                                  tk.idx.cpu().numpy()[rows], _np(tk.w)[rows], I)
    got, refv = bf16_to_f32(_np(out))[rows], bf16_to_f32(ref)
    ok, ma, cos = block_close(got, refv)
    assert ok and ma <= TIGHT_REL * np.abs(refv).max(), (ma, cos)


def test_quant4_prefill_T4096_zipf_vs_oracle(oracle):
    """BASELINE config 4 at T=4096: 4-bit MLX-affine experts (group 64),
    Zipf-skewed routing, the block's prefill path against the oracle's
    gather_qmm restatement on 128 sampled tokens with the oracle's routing
    (indices first checked on every token)."""
    from tests.helpers import router_index_check
    H, E, K, I, T = 2816, 128, 8, 704, 4096
    d = block_inputs(T, seed=4096, device=DEV, routing="zipf", H=H, E=E, K=K, I=I)
    gq, dq = _quantize(oracle, d, 4)
    cfg = A.ESModelConfig(moe_sparse=True, max_tokens=T)
    q = dict(gu_q=_dev(gq[0]), gu_s=_dev(gq[1]), gu_b=_dev(gq[2]), dn_q=_dev(dq[0]),
             dn_s=_dev(dq[1]), dn_b=_dev(dq[2]), bits=4, group_size=64)
    blk = A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], quantized=q)
    out, tk = blk.forward(d["x"], return_routing=True)
    torch.cuda.synchronize()
    blk.handle.sync()
    idx = tk.idx.cpu().numpy()
    idx_o, w_o, aux = oracle.route_topk(_np(d["x"]), _np(d["proj"]), _np(d["scale"]),
                                        _np(d["pes"]), K, return_scores=True)
    bad, exempt = router_index_check(idx, idx_o, aux["scores"])
    assert bad == 0, f"{bad} non-tie index mismatches (exempt {exempt})"
    same = np.nonzero(np.all(idx == idx_o, axis=1))[0]
    rows = np.sort(np.random.default_rng(2).choice(same, 128, replace=False))
    ref = oracle.experts_sparse_q(_np(d["x"][rows]), *gq, *dq, 4, 64, idx_o[rows], w_o[rows], I)
    got, refv = bf16_to_f32(_np(out))[rows], bf16_to_f32(ref)
    ok, ma, cos = block_close(got, refv)
    assert ok and ma <= TIGHT_REL * np.abs(refv).max(), (ma, cos)


@pytest.mark.parametrize("shape,T,routing", [((2816, 128, 8, 704), 16, "uniform"),
                                             ((2816, 128, 8, 704), 300, "zipf"),
                                             ((2816, 128, 8, 704), 4096, "zipf"),
                                             ((256, 32, 8, 128), 64, "uniform")])
def test_quant4_gemm_equals_expansion(shape, T, routing):
    """4-bit experts on the tensor cores: the GEMMs that dequantise each B tile
    in shared memory (apt_moe_set_q4_gemm 1) must give the same bits as
    expanding the touched experts to a bf16 bank first (0) -- both feed the
    tensor cores w = bf16(scale * q + bias) -- and the same bits on a repeat
    call.  Covers the narrow last gate_up tile (I = 704) and I = 128 (none)."""
    from oracle import oracle as O
    H, E, K, I = shape
    d = block_inputs(T, seed=400 + T, device=DEV, routing=routing, H=H, E=E, K=K, I=I)
    gq = O.quantize_affine(_np(d["gate_up"]), 64, 4)
    dq = O.quantize_affine(_np(d["down"]), 64, 4)
    cfg = A.ESModelConfig(hidden_size=H, num_experts=E, top_k_experts=K, moe_intermediate_size=I,
                          moe_sparse=True, max_tokens=T)
    q = dict(gu_q=_dev(gq[0]), gu_s=_dev(gq[1]), gu_b=_dev(gq[2]), dn_q=_dev(dq[0]),
             dn_s=_dev(dq[1]), dn_b=_dev(dq[2]), bits=4, group_size=64)
    blk = A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], quantized=q)
    outs = []
    for on in (1, 1, 0):
        blk.handle.set_q4_gemm(on)
        outs.append(blk.forward(d["x"]))
        torch.cuda.synchronize()
        blk.handle.sync()
    assert torch.isfinite(outs[0].float()).all()
    assert torch.equal(outs[0], outs[1]), "dequantising GEMM not deterministic"
    diff = (outs[0].float() - outs[2].float()).abs().max().item()
    assert torch.equal(outs[0], outs[2]), f"dequantising GEMM != expansion path (max {diff})"
