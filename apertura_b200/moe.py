"""Host-side mirror of the reference's MoE interface over torch device tensors.

Same names, argument meaning and error behaviour as the reference classes
(paths within the reference project):

* :class:`ESModelConfig`  -- MoE subset of es::ESModelConfig
  (aptransformer/ESModelConfig.h:135-157, parsed at ESModelConfig.mm:46-49)
* :class:`ESRouter`       -- es::ESRouter (aptransformer/ESRouter.h:17-34):
  ``route_top_k`` = routeTopK, ``route_weights`` = routeWeights
* :class:`ESExperts`      -- es::ESExperts (aptransformer/ESExperts.h:17-41):
  ``forward(x, W)`` = forward (dense), ``sparse_forward(x, idx, w)`` =
  sparseForward; ``ESExperts.from_quantized`` = the bundle constructor
* :func:`make_experts`    -- esMakeExperts (aptransformer/ESWeightLoader.mm:145-154)
* :class:`MoEBlock`       -- the MoE section of ESDecoderLayer::forward
  (aptransformer/ESDecoderLayer.mm:67-75): ``forward(hidden) -> hidden``

Torch only supplies device memory and the current stream.  Every compute call
goes through libapt_moe.so's C ABI; there is no other implementation, so a
missing library or a CPU tensor raises instead of falling back.
"""
from __future__ import annotations

import ctypes
import json
import os
from dataclasses import dataclass, field
from typing import NamedTuple, Optional

import torch

from ._lib import AptMoeConfig, check, lib


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _bits(t: torch.Tensor) -> torch.Tensor:
    """bf16 tensor -> same storage seen as int16 (the ABI passes raw bf16 bits)."""
    return t if t.dtype == torch.int16 else t.view(torch.int16)


def _need_cuda_bf16(name, t, shape=None):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be bfloat16, got {t.dtype}")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} shape {tuple(t.shape)} != {tuple(shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


@dataclass
class ESModelConfig:
    """MoE fields of the model config plus the reference's runtime knobs."""
    hidden_size: int = 2816
    num_experts: int = 128
    top_k_experts: int = 8
    moe_intermediate_size: int = 704
    rms_norm_eps: float = 1e-6
    enable_moe_block: bool = True
    moe_sparse: bool = False      # reference default: dense (MoE_REFERENCE.md section 5)
    quant_bits: int = 0
    quant_group_size: int = 64
    max_tokens: int = 8192
    device: int = 0

    @classmethod
    def from_config_json(cls, path_or_text: str, **runtime) -> "ESModelConfig":
        """ESModelConfig::fromConfigJSON for the MoE keys (text_config preferred)."""
        text = path_or_text
        if os.path.exists(path_or_text):
            with open(path_or_text) as f:
                text = f.read()
        c = AptMoeConfig()
        check(lib().apt_moe_config_from_json(text.encode(), ctypes.byref(c)))
        cfg = cls(hidden_size=c.hidden_size, num_experts=c.num_experts,
                  top_k_experts=c.top_k_experts, moe_intermediate_size=c.moe_intermediate_size,
                  rms_norm_eps=c.rms_norm_eps, enable_moe_block=bool(c.enable_moe_block),
                  moe_sparse=bool(c.moe_sparse), quant_bits=c.quant_bits,
                  quant_group_size=c.quant_group_size, max_tokens=c.max_tokens, device=c.device)
        for k, v in runtime.items():
            if not hasattr(cfg, k):
                raise TypeError(f"unknown config field {k}")
            setattr(cfg, k, v)
        return cfg

    def to_c(self) -> AptMoeConfig:
        return AptMoeConfig(self.hidden_size, self.num_experts, self.top_k_experts,
                            self.moe_intermediate_size, float(self.rms_norm_eps),
                            int(self.enable_moe_block), int(self.moe_sparse), int(self.quant_bits),
                            int(self.quant_group_size), int(self.max_tokens), int(self.device))


class Handle:
    """Owns one apt_moe_handle (device weights + workspace)."""

    def __init__(self, cfg: ESModelConfig):
        self.cfg = cfg
        self.device = torch.device("cuda", cfg.device)
        h = ctypes.c_void_p()
        c = cfg.to_c()
        check(lib().apt_moe_create(ctypes.byref(c), ctypes.byref(h)))
        self.h = h

    def clone_shared(self, cfg: Optional[ESModelConfig] = None) -> "Handle":
        """A second handle on the same device weights (own workspace and
        settings; the shared weights are read-only).  cfg may change only
        max_tokens, moe_sparse, rms_norm_eps and enable_moe_block."""
        out = Handle.__new__(Handle)
        out.cfg = cfg or self.cfg
        out.device = self.device
        h = ctypes.c_void_p()
        c = out.cfg.to_c() if cfg is not None else None
        self.check(lib().apt_moe_clone_shared(self.h, ctypes.byref(c) if c is not None else None,
                                              ctypes.byref(h)))
        out.h = h
        return out

    def close(self):
        if getattr(self, "h", None):
            lib().apt_moe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, status):
        check(status, self.h)

    def set_gemv_max_tokens(self, t: int):
        self.check(lib().apt_moe_set_gemv_max_tokens(self.h, int(t)))

    def set_sm_limit(self, n: int):
        """Cap on the SMs the persistent kernels of this handle fill (0 = all)."""
        self.check(lib().apt_moe_set_sm_limit(self.h, int(n)))

    def set_fused_decode(self, on: bool):
        """Decode (T <= 8) as one persistent kernel (default) or the kernel chain."""
        self.check(lib().apt_moe_set_fused_decode(self.h, int(bool(on))))

    def set_q4_gemm(self, on: bool):
        """4-bit experts above decode sizes: dequantise B tiles inside the
        tensor-core GEMMs (default) or expand the touched experts to bf16 first."""
        self.check(lib().apt_moe_set_q4_gemm(self.h, int(bool(on))))

    def last_counts(self) -> torch.Tensor:
        out = torch.zeros(self.cfg.num_experts, dtype=torch.int32)
        self.check(lib().apt_moe_last_counts(self.h, ctypes.c_void_p(out.data_ptr())))
        return out

    def last_launches(self) -> int:
        return lib().apt_moe_last_launches(self.h)

    def set_timing(self, enable: bool = True):
        self.check(lib().apt_moe_set_timing(self.h, int(enable)))

    def stage_times(self) -> dict:
        """Per-stage CUDA-event durations (ms) of the last call; needs set_timing."""
        from ._lib import STAGES
        buf = (ctypes.c_float * len(STAGES))()
        self.check(lib().apt_moe_stage_times(self.h, ctypes.cast(buf, ctypes.c_void_p)))
        return {n: float(buf[i]) for i, n in enumerate(STAGES) if buf[i] >= 0}

    def sync(self):
        self.check(lib().apt_moe_sync(self.h))


class TopK(NamedTuple):
    idx: torch.Tensor  # [T, K] int32, descending probability
    w: torch.Tensor    # [T, K] bf16


class ESRouter:
    """es::ESRouter(proj, scale, perExpertScale, numExperts, topK, hiddenSize, eps)."""

    def __init__(self, proj, scale, per_expert_scale, num_experts, top_k, hidden_size, eps=1e-6,
                 handle: Optional[Handle] = None, max_tokens: int = 8192):
        if handle is None:
            dev = proj.device.index or 0
            handle = Handle(ESModelConfig(hidden_size=hidden_size, num_experts=num_experts,
                                          top_k_experts=top_k, moe_intermediate_size=64,
                                          rms_norm_eps=eps, max_tokens=max_tokens, device=dev))
        self.handle = handle
        self.num_experts, self.top_k, self.hidden_size = num_experts, top_k, hidden_size
        _need_cuda_bf16("proj", proj, (num_experts, hidden_size))
        _need_cuda_bf16("scale", scale, (hidden_size,))
        _need_cuda_bf16("per_expert_scale", per_expert_scale, (num_experts,))
        handle.check(lib().apt_moe_load_router(handle.h, _ptr(proj), _ptr(scale),
                                               _ptr(per_expert_scale), 1))

    def route_top_k(self, x: torch.Tensor) -> TopK:
        _need_cuda_bf16("x", x)
        T = x.shape[0]
        idx = torch.empty(T, self.top_k, dtype=torch.int32, device=x.device)
        w = torch.empty(T, self.top_k, dtype=torch.bfloat16, device=x.device)
        self.handle.check(lib().apt_moe_route(self.handle.h, _ptr(x), T, _ptr(idx), _ptr(w),
                                              _stream(x.device)))
        return TopK(idx, w)

    # reference spelling
    routeTopK = route_top_k

    def route_weights(self, x: torch.Tensor) -> torch.Tensor:
        _need_cuda_bf16("x", x)
        T = x.shape[0]
        W = torch.empty(T, self.num_experts, dtype=torch.bfloat16, device=x.device)
        self.handle.check(lib().apt_moe_route_weights(self.handle.h, _ptr(x), T, _ptr(W),
                                                      _stream(x.device)))
        return W

    routeWeights = route_weights


class ESExperts:
    """es::ESExperts(gateUp [E,2I,H], down [E,H,I], quantBits=0, groupSize=64)."""

    def __init__(self, gate_up, down, quant_bits: int = 0, group_size: int = 64,
                 handle: Optional[Handle] = None, max_tokens: int = 8192, _quantized=None):
        if _quantized is None:
            E, I2, H = gate_up.shape
            I = I2 // 2
        else:
            E, I, H = _quantized["shape"]
        if handle is None:
            dev = (gate_up if gate_up is not None else _quantized["gu_q"]).device.index or 0
            handle = Handle(ESModelConfig(hidden_size=H, num_experts=E, top_k_experts=min(8, E),
                                          moe_intermediate_size=I, quant_bits=quant_bits,
                                          quant_group_size=group_size, max_tokens=max_tokens,
                                          device=dev))
        self.handle = handle
        self.num_experts, self.hidden_size, self.inter = E, H, I
        self.quant_bits, self.group_size = quant_bits, group_size
        if _quantized is None:
            _need_cuda_bf16("gate_up", gate_up, (E, 2 * I, H))
            _need_cuda_bf16("down", down, (E, H, I))
            if quant_bits and handle.cfg.quant_bits != quant_bits:
                raise ValueError("handle config quant_bits differs from quant_bits")
            handle.check(lib().apt_moe_load_experts_bf16(handle.h, _ptr(gate_up), _ptr(down), 1))
        else:
            q = _quantized
            handle.check(lib().apt_moe_load_experts_quant(
                handle.h, _ptr(q["gu_q"]), _ptr(q["gu_s"]), _ptr(q["gu_b"]), _ptr(q["dn_q"]),
                _ptr(q["dn_s"]), _ptr(q["dn_b"]), quant_bits, group_size, 1))

    @classmethod
    def from_quantized(cls, gu_q, gu_s, gu_b, dn_q, dn_s, dn_b, bits: int, group_size: int = 64,
                       handle: Optional[Handle] = None, max_tokens: int = 8192):
        """Adopt MLX-format packed experts verbatim (ESExperts bundle ctor)."""
        E, I2, _ = gu_q.shape
        H = dn_q.shape[1]
        q = dict(gu_q=gu_q, gu_s=gu_s, gu_b=gu_b, dn_q=dn_q, dn_s=dn_s, dn_b=dn_b,
                 shape=(E, I2 // 2, H))
        for k in ("gu_q", "dn_q"):
            if q[k].dtype not in (torch.int32, torch.uint32) or not q[k].is_cuda:
                raise ValueError(f"{k} must be a CUDA int32/uint32 tensor")
        return cls(None, None, bits, group_size, handle=handle, max_tokens=max_tokens,
                   _quantized=q)

    def sparse_forward(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        _need_cuda_bf16("x", x)
        _need_cuda_bf16("w", w)
        if idx.dtype != torch.int32 or not idx.is_cuda or not idx.is_contiguous():
            raise ValueError("idx must be a contiguous CUDA int32 tensor")
        T = x.shape[0]
        out = torch.empty(T, self.hidden_size, dtype=torch.bfloat16, device=x.device)
        self.handle.check(lib().apt_moe_experts(self.handle.h, _ptr(x), _ptr(idx), _ptr(w), T,
                                                _ptr(out), _stream(x.device)))
        return out

    sparseForward = sparse_forward

    def forward(self, x: torch.Tensor, W: torch.Tensor) -> torch.Tensor:
        _need_cuda_bf16("x", x)
        _need_cuda_bf16("W", W)
        T = x.shape[0]
        out = torch.empty(T, self.hidden_size, dtype=torch.bfloat16, device=x.device)
        self.handle.check(lib().apt_moe_experts_dense(self.handle.h, _ptr(x), _ptr(W), T,
                                                      _ptr(out), _stream(x.device)))
        return out


def make_experts(weights: dict, gate_up_name: str, down_name: str, quant_bits: int = 0,
                 group_size: int = 64, **kw) -> ESExperts:
    """esMakeExperts: adopt `<name>.scales/.biases` triples when present, else
    build from bf16 (quantising at load when quant_bits > 0).  The width of
    adopted codes is the bundle's (`bundle_bits`, ESWeightLoader::bundleBits,
    as ESWeightLoader.mm:149-150 passes it); when not given it follows from
    the triple's shapes: in = groups x group_size, bits = 32 x words / in."""
    if gate_up_name + ".scales" in weights:
        g = gate_up_name
        d = down_name
        bits = kw.pop("bundle_bits", None)
        if bits is None:
            words, groups = weights[g].shape[-1], weights[g + ".scales"].shape[-1]
            if (32 * words) % (groups * group_size):
                raise ValueError(f"{g}: {words} code words for {groups} groups of {group_size}")
            bits = 32 * words // (groups * group_size)
        return ESExperts.from_quantized(weights[g], weights[g + ".scales"], weights[g + ".biases"],
                                        weights[d], weights[d + ".scales"], weights[d + ".biases"],
                                        bits, group_size, **kw)
    return ESExperts(weights[gate_up_name], weights[down_name], quant_bits, group_size, **kw)


class MoEBlock:
    """Router + experts sharing one handle: the MoE section of ESDecoderLayer.

    ``forward(hidden)`` runs the whole block (router on ``hidden``, experts on
    ``hidden``), which is the BASELINE block harness; ``forward_layer(x1,
    expert_in)`` is the decoder-layer form (router on the raw residual x1,
    experts on pre_ff_ln_2(x1))."""

    def __init__(self, cfg: ESModelConfig, proj, scale, per_expert_scale, gate_up=None, down=None,
                 quantized: Optional[dict] = None):
        self.cfg = cfg
        self.handle = Handle(cfg)
        self.router = ESRouter(proj, scale, per_expert_scale, cfg.num_experts, cfg.top_k_experts,
                               cfg.hidden_size, cfg.rms_norm_eps, handle=self.handle)
        if quantized is not None:
            self.experts = ESExperts.from_quantized(**quantized, handle=self.handle)
        else:
            self.experts = ESExperts(gate_up, down, cfg.quant_bits, cfg.quant_group_size,
                                     handle=self.handle)

    def forward(self, hidden: torch.Tensor, return_routing: bool = False):
        return self.forward_layer(hidden, hidden, return_routing)

    __call__ = forward

    def forward_layer(self, x1: torch.Tensor, expert_in: torch.Tensor, return_routing=False):
        _need_cuda_bf16("x1", x1)
        _need_cuda_bf16("expert_in", expert_in)
        T = x1.shape[0]
        out = torch.empty(T, self.cfg.hidden_size, dtype=torch.bfloat16, device=x1.device)
        idx = w = None
        if return_routing:
            idx = torch.empty(T, self.cfg.top_k_experts, dtype=torch.int32, device=x1.device)
            w = torch.empty(T, self.cfg.top_k_experts, dtype=torch.bfloat16, device=x1.device)
        self.handle.check(lib().apt_moe_forward(self.handle.h, _ptr(x1), _ptr(expert_in), T,
                                                _ptr(out), _ptr(idx), _ptr(w), _stream(x1.device)))
        return (out, TopK(idx, w)) if return_routing else out

    def forward_with_norms(self, x1: torch.Tensor, pre_ff_ln_2_w: torch.Tensor,
                           post_ff_ln_2_w: torch.Tensor) -> torch.Tensor:
        """post_ff_ln_2(experts(pre_ff_ln_2(x1), router(x1))): the MoE half of
        ESDecoderLayer::forward (ESDecoderLayer.mm:69-74) with both norms fused."""
        _need_cuda_bf16("x1", x1)
        H = self.cfg.hidden_size
        _need_cuda_bf16("pre_ff_ln_2_w", pre_ff_ln_2_w, (H,))
        _need_cuda_bf16("post_ff_ln_2_w", post_ff_ln_2_w, (H,))
        T = x1.shape[0]
        out = torch.empty(T, H, dtype=torch.bfloat16, device=x1.device)
        self.handle.check(lib().apt_moe_layer_forward(self.handle.h, _ptr(x1), _ptr(pre_ff_ln_2_w),
                                                      _ptr(post_ff_ln_2_w), T, _ptr(out),
                                                      _stream(x1.device)))
        return out

    def forward_decoder_ff(self, x1: torch.Tensor, hmlp: torch.Tensor,
                           pre_ff_ln_2_w: torch.Tensor, post_ff_ln_1_w: torch.Tensor,
                           post_ff_ln_2_w: torch.Tensor, post_ff_ln_w: torch.Tensor) -> torch.Tensor:
        """x2 = x1 + post_ff_ln(post_ff_ln_1(hmlp) + post_ff_ln_2(MoE(x1))): the
        feed-forward tail of an MoE ESDecoderLayer (ESDecoderLayer.mm:61-78),
        hmlp being the dense MLP's output; all trailing norms fused."""
        _need_cuda_bf16("x1", x1)
        H = self.cfg.hidden_size
        T = x1.shape[0]
        _need_cuda_bf16("hmlp", hmlp, (T, H))
        for name, t in (("pre_ff_ln_2_w", pre_ff_ln_2_w), ("post_ff_ln_1_w", post_ff_ln_1_w),
                        ("post_ff_ln_2_w", post_ff_ln_2_w), ("post_ff_ln_w", post_ff_ln_w)):
            _need_cuda_bf16(name, t, (H,))
        x2 = torch.empty(T, H, dtype=torch.bfloat16, device=x1.device)
        self.handle.check(lib().apt_moe_decoder_ff(
            self.handle.h, _ptr(x1), _ptr(hmlp), _ptr(pre_ff_ln_2_w), _ptr(post_ff_ln_1_w),
            _ptr(post_ff_ln_2_w), _ptr(post_ff_ln_w), T, _ptr(x2), _stream(x1.device)))
        return x2

    def forward_decoder_ff_full(self, x1: torch.Tensor, mlp: "MLPBlock", pre_ff_ln_w,
                                pre_ff_ln_2_w, post_ff_ln_1_w, post_ff_ln_2_w,
                                post_ff_ln_w) -> torch.Tensor:
        """The whole feed-forward half of an MoE ESDecoderLayer (ESDecoderLayer.mm:
        61-78), dense MLP included: x2 = x1 + post_ff_ln(post_ff_ln_1(mlp(
        pre_ff_ln(x1))) + post_ff_ln_2(MoE(x1)))."""
        _need_cuda_bf16("x1", x1)
        H = self.cfg.hidden_size
        T = x1.shape[0]
        for name, t in (("pre_ff_ln_w", pre_ff_ln_w), ("pre_ff_ln_2_w", pre_ff_ln_2_w),
                        ("post_ff_ln_1_w", post_ff_ln_1_w), ("post_ff_ln_2_w", post_ff_ln_2_w),
                        ("post_ff_ln_w", post_ff_ln_w)):
            _need_cuda_bf16(name, t, (H,))
        x2 = torch.empty(T, H, dtype=torch.bfloat16, device=x1.device)
        self.handle.check(lib().apt_moe_decoder_ff_full(
            self.handle.h, mlp.handle.h, _ptr(x1), _ptr(pre_ff_ln_w), _ptr(pre_ff_ln_2_w),
            _ptr(post_ff_ln_1_w), _ptr(post_ff_ln_2_w), _ptr(post_ff_ln_w), T, _ptr(x2),
            _stream(x1.device)))
        return x2

    def forward_host(self, x_host: torch.Tensor, out_host: Optional[torch.Tensor] = None,
                     asynchronous: bool = False):
        """End-to-end call with host buffers (pinned for speed).  With
        asynchronous=True the copies and the block are only queued on the
        current stream (apt_moe_forward_host_async): synchronise before reading
        out_host or reusing x_host."""
        if x_host.is_cuda or x_host.dtype != torch.bfloat16:
            raise ValueError("x_host must be a CPU bfloat16 tensor")
        T = x_host.shape[0]
        if out_host is None:
            out_host = torch.empty(T, self.cfg.hidden_size, dtype=torch.bfloat16,
                                   pin_memory=x_host.is_pinned())
        fn = lib().apt_moe_forward_host_async if asynchronous else lib().apt_moe_forward_host
        self.handle.check(fn(self.handle.h, _ptr(x_host), T, _ptr(out_host),
                             _stream(self.handle.device)))
        return out_host


class MLPBlock:
    """ESMLPBlock (ESMLPBlock.mm:11-15): down(gelu(gate(x)) * up(x)), the dense
    GeGLU MLP that an MoE layer adds to the expert output.  Runs on the
    expert kernels as a one-expert handle; gate/up/down are the [I, H], [I, H]
    and [H, I] bf16 Linear weights (quantised at load when quant_bits > 0)."""

    def __init__(self, gate, up, down, hidden_size: int = 2816, intermediate_size: int = 2112,
                 rms_norm_eps: float = 1e-6, quant_bits: int = 0, max_tokens: int = 8192,
                 device: int = 0):
        I, H = intermediate_size, hidden_size
        for name, t, shp in (("gate", gate, (I, H)), ("up", up, (I, H)), ("down", down, (H, I))):
            _need_cuda_bf16(name, t, shp)
        self.cfg = ESModelConfig(hidden_size=H, num_experts=1, top_k_experts=1,
                                 moe_intermediate_size=I, rms_norm_eps=rms_norm_eps,
                                 moe_sparse=True, quant_bits=quant_bits, max_tokens=max_tokens,
                                 device=device)
        self.handle = Handle(self.cfg)
        gu = torch.cat([gate, up], 0).unsqueeze(0).contiguous()
        dn = down.unsqueeze(0).contiguous()
        self.handle.check(lib().apt_moe_load_experts_bf16(self.handle.h, _ptr(gu), _ptr(dn), 1))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _need_cuda_bf16("x", x)
        T = x.shape[0]
        out = torch.empty_like(x)
        self.handle.check(lib().apt_moe_mlp_forward(self.handle.h, _ptr(x), T, _ptr(out),
                                                    _stream(x.device)))
        return out

    __call__ = forward

