"""Generate the golden vectors that pin the CPU oracle.

The reference (Objective-C++ on MLX) cannot be compiled or run here, and it
ships no router or expert fixtures.  The model it re-implements is HF
``Gemma4TextForCausalLM``; its MoE modules ``Gemma4TextRouter`` and
``Gemma4TextExperts`` (transformers 5.5.0,
``transformers/models/gemma4/modeling_gemma4.py``) are importable here and are
the same block the reference's conformance fixtures were captured from
(Tools/generate_fixtures.py).  This script runs them in f32 on torch CPU on
seeded bf16-representable inputs and stores inputs and outputs as small
``.npz`` fixtures.  Re-run with ``python tests/golden/make_golden.py``.

Cases:
  ``unit``   H=64,  E=16, K=4, I=32,  T=3   (the shape of the reference's
             testMoERouterTopKWeights, ESPrimitivesTests.mm:171-189)
  ``small``  H=256, E=32, K=8, I=128, T=24, non-unit router scales
  ``gemma``  H=2816, E=128, K=8, I=704, T=2, the real Gemma-4-26B block
             shape; expert weights are not stored but regenerated per
             selected expert by ``expert_weights`` (numpy PCG64 streams)

Unselected experts are zero in every case (never evaluated by either side).
"""
from __future__ import annotations

import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16).copy()


def expert_weights(seed, e, I, H):
    """Expert e's (gate_up [2I,H], down [H,I]) as f32 tensors holding bf16 values.

    Each expert has its own numpy PCG64 stream, so a test can regenerate just
    the experts a token selected without storing the full bank.
    """
    rng = np.random.default_rng([seed, 1000 + e])
    gu = rng.standard_normal((2 * I, H), dtype=np.float32) * np.float32(0.02)
    dn = rng.standard_normal((H, I), dtype=np.float32) * np.float32(0.02)
    return (torch.from_numpy(gu).to(torch.bfloat16).to(torch.float32),
            torch.from_numpy(dn).to(torch.bfloat16).to(torch.float32))


def make_case(name, T, H, E, K, I, seed, unit_scales=True, compact=False):
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig
    from transformers.models.gemma4.modeling_gemma4 import Gemma4TextExperts, Gemma4TextRouter

    g = torch.Generator().manual_seed(seed)
    cfg = Gemma4TextConfig(hidden_size=H, num_experts=E, top_k_experts=K,
                           moe_intermediate_size=I, rms_norm_eps=1e-6,
                           hidden_activation="gelu_pytorch_tanh", enable_moe_block=True)

    def bf(t):  # make every input exactly bf16-representable, keep f32 storage
        return t.to(torch.bfloat16).to(torch.float32)

    x = bf(torch.randn(T, H, generator=g))
    proj = bf(torch.randn(E, H, generator=g) / float(np.sqrt(H)))
    if unit_scales:
        scale = torch.ones(H)
        pes = torch.ones(E)
    else:
        scale = bf(1.0 + 0.1 * torch.randn(H, generator=g))
        pes = bf(1.0 + 0.1 * torch.randn(E, generator=g))
    gate_up = torch.zeros(E, 2 * I, H)
    down = torch.zeros(E, H, I)

    router = Gemma4TextRouter(cfg)
    experts = Gemma4TextExperts(cfg)
    with torch.no_grad():
        router.proj.weight.copy_(proj)
        router.scale.copy_(scale)
        router.per_expert_scale.copy_(pes)
        experts.gate_up_proj.copy_(gate_up)
        experts.down_proj.copy_(down)
        probs, top_w, top_i = router(x)
        # Only the selected experts are ever evaluated; the rest stay zero.
        for e in np.unique(top_i.numpy()):
            gate_up[e], down[e] = expert_weights(seed, int(e), I, H)
        experts.gate_up_proj.copy_(gate_up)
        experts.down_proj.copy_(down)
        # logits, for the tie analysis
        h = router.norm(x) * router.scale * router.scalar_root_size
        scores = router.proj(h)
        out = experts(x, top_i, top_w)

    d = dict(
        T=T, H=H, E=E, K=K, I=I, seed=seed,
        x=bf16_bits(x), proj=bf16_bits(proj), scale=bf16_bits(scale), pes=bf16_bits(pes),
        hf_scores=scores.numpy().astype(np.float32),
        hf_probs=probs.numpy().astype(np.float32),
        hf_idx=top_i.numpy().astype(np.int32),
        hf_w=top_w.numpy().astype(np.float32),
        hf_out=out.numpy().astype(np.float32),
    )
    if not compact:
        d["gate_up"] = bf16_bits(gate_up)
        d["down"] = bf16_bits(down)
    path = os.path.join(HERE, f"hf_moe_{name}.npz")
    np.savez_compressed(path, **d)
    print(path, os.path.getsize(path))


if __name__ == "__main__":
    torch.set_num_threads(8)
    make_case("unit", T=3, H=64, E=16, K=4, I=32, seed=1)
    make_case("small", T=24, H=256, E=32, K=8, I=128, seed=2, unit_scales=False)
    make_case("gemma", T=2, H=2816, E=128, K=8, I=704, seed=3, compact=True)
