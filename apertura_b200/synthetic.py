"""Seeded synthetic inputs with BASELINE.json's shapes and distributions.

The reference publishes no dataset for this path, so every config is restated
as seeded synthetic tensors:

* hidden ~ N(0,1) [T,H]; router proj ~ N(0, 1/sqrt(H)) [E,H] (std convention);
  router scale = ones [H], per_expert_scale = ones [E] (HF init values, since
  the configs do not give them; ``nonunit=True`` draws N(1, 0.1) instead);
* expert gate_up [E,2I,H] and down [E,H,I] ~ N(0, 0.02); all stored as bf16
  after f32 sampling.
* ``routing="zipf"`` (configs 3 and 5): a fixed per-expert logit bias makes
  expert popularity follow Zipf(s) over a seeded random permutation of expert
  ids.  The router math is left untouched: the bias is folded into the data
  by adding alpha*d (d a seeded unit vector) to every hidden row and beta_e*d
  to router row e; beta is calibrated by fixed-point iteration until the
  top-K selection frequencies match the (capped) Zipf targets.

Tensors are generated on the target device with a seeded torch.Generator.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

GEMMA = dict(H=2816, E=128, K=8, I=704)


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _randn(shape, g, device, std=1.0, mean=0.0):
    t = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    if std != 1.0:
        t.mul_(std)
    if mean != 0.0:
        t.add_(mean)
    return t.to(torch.bfloat16)


def expert_bank(E, H, I, seed=0, device="cuda"):
    """gate_up [E,2I,H], down [E,H,I] bf16 ~ N(0, 0.02)."""
    g = _gen(device, seed * 7919 + 17)
    gate_up = torch.empty(E, 2 * I, H, dtype=torch.bfloat16, device=device)
    down = torch.empty(E, H, I, dtype=torch.bfloat16, device=device)
    for e in range(E):  # per-expert draws keep peak f32 scratch small
        gate_up[e] = _randn((2 * I, H), g, device, 0.02)
        down[e] = _randn((H, I), g, device, 0.02)
    return gate_up, down


def zipf_targets(E, K, s=1.1, seed=0):
    """Per-expert selection frequency (fraction of tokens choosing e), Zipf(s)
    over a seeded permutation, capped at 1 and renormalised to sum K."""
    g = torch.Generator().manual_seed(seed + 12345)
    perm = torch.randperm(E, generator=g)
    p = torch.tensor([(r + 1) ** (-s) for r in range(E)], dtype=torch.float64)
    f = K * p / p.sum()
    for _ in range(64):  # water-fill the cap
        over = f > 1.0
        if not over.any():
            break
        excess = float((f[over] - 1.0).sum())
        f[over] = 1.0
        free = ~over & (f < 1.0)
        f[free] += excess * f[free] / f[free].sum()
    out = torch.empty(E, dtype=torch.float64)
    out[perm] = f
    return out


def _route_f32(x, proj, scale, K, eps=1e-6):
    xf = x.float()
    h = xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + eps)
    h = h * scale.float() * (x.shape[1] ** -0.5)
    probs = torch.softmax(h @ proj.float().t(), -1)
    return torch.topk(probs, K, dim=-1).indices


def block_inputs(T: int, seed: int = 0, device="cuda", H=2816, E=128, K=8, I=704,
                 routing: str = "uniform", zipf_s: float = 1.1, with_experts: bool = True,
                 nonunit: bool = False, calib_tokens: Optional[int] = None):
    g = _gen(device, seed)
    x = _randn((T, H), g, device)
    proj = _randn((E, H), g, device, 1.0 / math.sqrt(H))
    if nonunit:
        scale = _randn((H,), g, device, 0.1, 1.0)
        pes = _randn((E,), g, device, 0.1, 1.0)
    else:
        scale = torch.ones(H, dtype=torch.bfloat16, device=device)
        pes = torch.ones(E, dtype=torch.bfloat16, device=device)
    out = dict(x=x, proj=proj, scale=scale, pes=pes, T=T, H=H, E=E, K=K, I=I)
    if routing == "zipf":
        x, proj, info = _fold_zipf(x, proj, scale, K, zipf_s, seed, device, calib_tokens)
        out.update(x=x, proj=proj, zipf=info)
    if with_experts:
        out["gate_up"], out["down"] = expert_bank(E, H, I, seed, device)
    return out


def _fold_zipf(x, proj, scale, K, s, seed, device, calib_tokens=None, iters=80):
    T, H = x.shape
    E = proj.shape[0]
    g = _gen(device, seed + 99)
    d = torch.randn(H, generator=g, device=device)
    d = d / d.norm()
    alpha = 8.0
    xb = (x.float() + alpha * d).to(torch.bfloat16)
    target = zipf_targets(E, K, s, seed).to(device)
    # calibrate on a fixed sample of the tokens
    n = min(T, calib_tokens or 4096)
    xs = xb[:n]
    beta = torch.zeros(E, device=device, dtype=torch.float64)
    projf = proj.float()
    # step size in bias units that moves a logit by ~0.3 of its spread
    xf = xs.float()
    h = xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + 1e-6) * scale.float() * H ** -0.5
    spread = float((h @ projf.t()).std())
    hd = float((h @ d).mean())
    step = 0.3 * spread / hd
    for it in range(iters):
        pb = (projf + beta.float()[:, None] * d[None, :]).to(torch.bfloat16)
        idx = _route_f32(xs, pb, scale, K)
        freq = torch.bincount(idx.flatten(), minlength=E).double() / n
        err = torch.log(target.clamp_min(1e-6)) - torch.log(freq.clamp_min(0.5 / n))
        beta += step * (1.0 - 0.5 * it / iters) * err.clamp(-3, 3)
        beta -= beta.mean()
    pb = (projf + beta.float()[:, None] * d[None, :]).to(torch.bfloat16)
    idx = _route_f32(xb, pb, scale, K)
    freq = torch.bincount(idx.flatten(), minlength=E).double() / T
    info = dict(target=target.cpu(), achieved=freq.cpu(), alpha=alpha)
    return xb, pb, info


def to_numpy_bits(t: torch.Tensor):
    """bf16 tensor -> numpy uint16 bits (CPU copy) for the oracle."""
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view("uint16")


def router_tie_tokens(x, proj, scale, K, eps=1e-6):
    """Tokens whose K-th and (K+1)-th router scores lie within one bf16 ulp
    of each other (f32 restatement of ESRouter.mm:14-24 in torch): their
    selected set may differ between two correct implementations, e.g. when
    the expert ids are relabelled for expert parallelism.  For checks only."""
    xf = x.float()
    h = xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + eps)
    h = h * scale.float() * (x.shape[1] ** -0.5)
    s = torch.sort(h @ proj.float().t(), dim=-1, descending=True).values
    a, b = s[:, K - 1], s[:, K]
    ulp = torch.exp2(torch.floor(torch.log2(a.abs().clamp_min(1e-30))) - 7)
    return (a - b) <= ulp
