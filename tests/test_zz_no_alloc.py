"""apt_moe_route_noalloc: the router for callers that may not allocate device
memory (a host runtime that owns every device byte, a plugin handed only its
buffers).  Called through the C ABI it must match apt_moe_route, the handle
-based router, on two calls in a row -- the second with different tokens, so
stale contents of its shared fixed scratch would show.

Kept in its own file, collected last, so a run that stops at the first failure
has already run every other test; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest
import torch

from tests.helpers import bf16_to_f32

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import apertura_b200 as A  # noqa: E402
from apertura_b200.synthetic import block_inputs, to_numpy_bits  # noqa: E402

DEV = torch.device("cuda", 0)
H, E, K = 2816, 128, 8


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _noalloc(d, x):
    T = x.shape[0]
    idx = torch.full((T, K), -7, dtype=torch.int32, device=DEV)
    w = torch.zeros(T, K, dtype=torch.bfloat16, device=DEV)
    st = A.lib().apt_moe_route_noalloc(
        _p(x), T, _p(d["proj"]), _p(d["scale"]), _p(d["pes"]), H, E, K, 1e-6, _p(idx), _p(w),
        ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream))
    assert st == 0, A._lib.STATUS_NAMES.get(st, st)
    return idx, w


@pytest.mark.parametrize("T", [16, 64])
def test_noalloc_matches_route_twice(T):
    d = block_inputs(2 * T, seed=40 + T, device=DEV, with_experts=False, nonunit=True)
    router = A.ESRouter(d["proj"], d["scale"], d["pes"], E, K, H,
                        handle=A.Handle(A.ESModelConfig(moe_intermediate_size=64, max_tokens=T)))
    for call in range(2):
        x = d["x"][call * T:(call + 1) * T].contiguous()
        ref = router.route_top_k(x)
        idx, w = _noalloc(d, x)
        torch.cuda.synchronize()
        # same kernels, same order of work: indices equal, weights within the
        # router tests' tolerance (one bf16 rounding step)
        np.testing.assert_array_equal(idx.cpu().numpy(), ref.idx.cpu().numpy())
        a = bf16_to_f32(to_numpy_bits(w))
        b = bf16_to_f32(to_numpy_bits(ref.w))
        assert np.all(np.abs(a - b) <= np.abs(b) * 2.0 ** -7 + 1e-9)


def test_noalloc_rejects_oversize():
    x = torch.zeros(129, H, dtype=torch.bfloat16, device=DEV)  # 129*128 > 16384 scores
    d = block_inputs(1, seed=1, device=DEV, with_experts=False)
    idx = torch.zeros(129, K, dtype=torch.int32, device=DEV)
    w = torch.zeros(129, K, dtype=torch.bfloat16, device=DEV)
    st = A.lib().apt_moe_route_noalloc(_p(x), 129, _p(d["proj"]), _p(d["scale"]), _p(d["pes"]),
                                       H, E, K, 1e-6, _p(idx), _p(w), None)
    assert st == 2  # APT_ERR_UNSUPPORTED
