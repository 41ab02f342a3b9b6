"""apt_moe_clone_shared: a second handle on the same device weights (as
several sessions of one model share its mx::arrays)."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import apertura_b200 as A  # noqa: E402
from apertura_b200.synthetic import block_inputs  # noqa: E402

DEV = torch.device("cuda", 0)
P = lambda t: ctypes.c_void_p(t.data_ptr())


def _fwd(h, x):
    out = torch.empty_like(x)
    h.check(A.lib().apt_moe_forward(h.h, P(x), P(x), x.shape[0], P(out), None, None, None))
    torch.cuda.synchronize()
    h.sync()
    return out


@pytest.mark.parametrize("quant_bits", [0, 4])
def test_clone_shares_weights(quant_bits):
    d = block_inputs(16, seed=4, device=DEV)
    cfg = A.ESModelConfig(moe_sparse=True, max_tokens=64, quant_bits=quant_bits)
    blk = A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], d["gate_up"], d["down"])
    x = d["x"]
    ref = _fwd(blk.handle, x)
    small = A.ESModelConfig(moe_sparse=True, max_tokens=16, quant_bits=quant_bits)
    h2 = blk.handle.clone_shared(small)
    assert torch.equal(_fwd(h2, x), ref)
    # shared weights are read-only on both handles
    for h in (blk.handle, h2):
        st = A.lib().apt_moe_load_router(h.h, P(d["proj"]), P(d["scale"]), P(d["pes"]), 1)
        assert st == 6  # APT_ERR_STATE
    # a clone outlives its source
    blk.handle.close()
    assert torch.equal(_fwd(h2, x), ref)
    # and a clone of a clone
    h3 = h2.clone_shared()
    h2.close()
    assert torch.equal(_fwd(h3, x), ref)
    h3.close()


def test_clone_rejects_other_shapes():
    d = block_inputs(4, seed=5, device=DEV)
    cfg = A.ESModelConfig(moe_sparse=True, max_tokens=8)
    blk = A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], d["gate_up"], d["down"])
    bad = A.ESModelConfig(moe_sparse=True, max_tokens=8, num_experts=64)
    with pytest.raises(A.AptError):
        blk.handle.clone_shared(bad)
