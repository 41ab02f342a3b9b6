"""Failure detection without a GPU fault: a bounded device wait that nothing
satisfies expires, the handle reports APT_ERR_TIMEOUT, and the context keeps
working (the same helper bounds every wait in the library's pipelines)."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import apertura_b200 as A  # noqa: E402
from apertura_b200.synthetic import block_inputs  # noqa: E402

DEV = torch.device("cuda", 0)


def test_bounded_wait_expires_and_context_survives():
    d = block_inputs(4, seed=8, device=DEV)
    cfg = A.ESModelConfig(moe_sparse=True, max_tokens=8)
    blk = A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], d["gate_up"], d["down"])
    ref = blk.forward(d["x"]).clone()
    blk.handle.sync()
    t0 = time.perf_counter()
    blk.handle.check(A.lib().apt_moe_selftest_wait(blk.handle.h, 200000, None))  # ~0.2 s
    with pytest.raises(A.AptError, match="TIMEOUT"):
        blk.handle.sync()
    assert time.perf_counter() - t0 < 10.0
    # the error word was cleared and the context still computes the same result
    out = blk.forward(d["x"])
    blk.handle.sync()
    assert torch.equal(out, ref)
