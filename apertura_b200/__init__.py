"""apertura_b200 -- B200-native (sm_100a) Gemma-4 MoE block for Apertura.

The product is libapt_moe.so (C ABI in include/apt_moe.h, CUDA kernels in
csrc/).  This package builds it and mirrors the reference's ESRouter /
ESExperts interface over torch device tensors.
"""
from ._lib import AptError, lib  # noqa: F401
from .moe import (ESExperts, ESModelConfig, ESRouter, Handle, MLPBlock, MoEBlock, TopK,  # noqa: F401
                  make_experts)

__all__ = ["AptError", "ESExperts", "ESModelConfig", "ESRouter", "Handle", "MLPBlock", "MoEBlock", "TopK",
           "make_experts", "lib"]
