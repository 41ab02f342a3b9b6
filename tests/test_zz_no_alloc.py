"""apt_moe_route_noalloc: the router for callers that may not allocate device
memory (a host runtime whose pool owns every device byte, a plugin handed only
its buffers).  Called through the C ABI it must match apt_moe_route, the
handle-based router, and the CPU oracle's ESRouter::routeTopK restatement, on
two calls in a row -- the second with different tokens, so stale contents of
its shared fixed scratch would show.  Cases cover both score kernels: the
bulk-copy kernel (T <= 64, H a multiple of 256) and the register-tiled one
(T = 128 at E = 128, exactly the scratch limit; H = 2880, a multiple of 64 but
not of 256).

Kept in its own file, collected last, so a run that stops at the first failure
has already run every other test; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest
import torch

from tests.helpers import bf16_to_f32, router_index_check

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import apertura_b200 as A  # noqa: E402
from apertura_b200.synthetic import block_inputs, to_numpy_bits  # noqa: E402

DEV = torch.device("cuda", 0)
E, K = 128, 8
W_REL = 2.0 ** -7  # one bf16 rounding step of w (f32 summation order)


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _noalloc(d, x, H):
    T = x.shape[0]
    idx = torch.full((T, K), -7, dtype=torch.int32, device=DEV)
    w = torch.zeros(T, K, dtype=torch.bfloat16, device=DEV)
    st = A.lib().apt_moe_route_noalloc(
        _p(x), T, _p(d["proj"]), _p(d["scale"]), _p(d["pes"]), H, E, K, 1e-6, _p(idx), _p(w),
        ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream))
    assert st == 0, A._lib.STATUS_NAMES.get(st, st)
    return idx, w


def _wf(t):
    return bf16_to_f32(to_numpy_bits(t))


@pytest.mark.parametrize("T,H", [(16, 2816), (64, 2816), (128, 2816), (40, 2880)])
def test_noalloc_matches_route_and_oracle_twice(oracle, T, H):
    d = block_inputs(2 * T, seed=40 + T, device=DEV, H=H, with_experts=False, nonunit=True)
    router = A.ESRouter(d["proj"], d["scale"], d["pes"], E, K, H,
                        handle=A.Handle(A.ESModelConfig(hidden_size=H, moe_intermediate_size=64,
                                                        max_tokens=T)))
    for call in range(2):
        x = d["x"][call * T:(call + 1) * T].contiguous()
        ref = router.route_top_k(x)
        idx, w = _noalloc(d, x, H)
        torch.cuda.synchronize()
        got = idx.cpu().numpy()
        idx_o, w_o, aux = oracle.route_topk(to_numpy_bits(x), to_numpy_bits(d["proj"]),
                                            to_numpy_bits(d["scale"]), to_numpy_bits(d["pes"]), K,
                                            return_scores=True)
        # against the handle path (above T = 64 its scores come from the
        # tensor-core router, another f32 summation order): bit-exact indices
        # except one-bf16-ulp ties of the oracle's scores
        ref_idx = ref.idx.cpu().numpy()
        bad, exempt = router_index_check(got, ref_idx, aux["scores"])
        assert bad == 0, f"{bad} non-tie mismatches vs apt_moe_route (exempt {exempt})"
        eq = np.all(got == ref_idx, axis=1)
        a, b = _wf(w), _wf(ref.w)
        assert np.all(np.abs(a[eq] - b[eq]) <= np.abs(b[eq]) * W_REL + 1e-9)
        # against the oracle: bit-exact indices except one-bf16-ulp ties
        bad, exempt = router_index_check(got, idx_o, aux["scores"])
        assert bad == 0, f"{bad} non-tie index mismatches (exempt {exempt} of {T})"
        same = np.all(got == idx_o, axis=1)
        wo = bf16_to_f32(w_o)
        assert np.all(np.abs(a[same] - wo[same]) <= np.abs(wo[same]) * W_REL + 1e-9)


def test_noalloc_rejects_oversize():
    H = 2816
    x = torch.zeros(129, H, dtype=torch.bfloat16, device=DEV)  # 129*128 > 16384 scores
    d = block_inputs(1, seed=1, device=DEV, with_experts=False)
    idx = torch.zeros(129, K, dtype=torch.int32, device=DEV)
    w = torch.zeros(129, K, dtype=torch.bfloat16, device=DEV)
    st = A.lib().apt_moe_route_noalloc(_p(x), 129, _p(d["proj"]), _p(d["scale"]), _p(d["pes"]),
                                       H, E, K, 1e-6, _p(idx), _p(w), None)
    assert st == 2  # APT_ERR_UNSUPPORTED
