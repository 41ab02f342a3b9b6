"""Expert-weight ingest for the MoE block: HF safetensors checkpoints and
Apertura `.apml` bundles (the on-disk formats feeding the kernels).

Restates the parts of es::ESWeightLoader that concern the MoE block
(aptransformer/ESWeightLoader.mm, ESWeightLoader.h):

* HF directory (ESWeightLoader.mm:24-61): `model.safetensors.index.json`
  weight_map (or a single `model.safetensors`); keys under the text prefix
  `model.language_model.` are kept with the prefix stripped and cast to the
  compute dtype (bf16).
* Bundle (ESWeightLoader.mm:77-110): `manifest.json` -> default variant ->
  its `path` and `files`; tensors adopted verbatim (packed uint32 stays
  uint32); quantisation bits / group size from the variant.
* Layer keys `layers.{i}.{suffix}` (ESWeightLoader.h:53-55); a tensor is
  pre-quantised iff `<name>.scales` exists (ESWeightLoader.h:46), which is
  what esMakeExperts (ESWeightLoader.mm:145-154) dispatches on.

Only the tensors of the requested MoE layer are read (safetensors lazy
access), so building one block does not load a 50 GB checkpoint.
"""
from __future__ import annotations

import json
import os
from typing import Dict, Optional

import torch

TEXT_PREFIX = "model.language_model."
MOE_SUFFIXES = ("router.proj.weight", "router.scale", "router.per_expert_scale",
                "experts.gate_up_proj", "experts.down_proj")


def layer_key(i: int, suffix: str) -> str:
    return f"layers.{i}.{suffix}"


class MoEWeightLoader:
    """Lazy reader of the MoE tensors of one checkpoint or bundle."""

    def __init__(self, path: str):
        from safetensors import safe_open  # noqa: F401  (fail early if missing)
        self.path = path
        self.is_bundle = False
        self.bits = 0
        self.group_size = 64
        self._where: Dict[str, tuple] = {}  # key -> (file, stored name)
        manifest = os.path.join(path, "manifest.json")
        if os.path.exists(manifest):
            with open(manifest) as f:
                m = json.load(f)
            if m.get("kind") not in (None, "apertura-model"):
                raise ValueError(f"{manifest}: not an Apertura model bundle")
            self._index_bundle(m)
        else:
            self._index_hf()

    # ------------------------------------------------------------------ indexing
    def _index_hf(self):
        idx = os.path.join(self.path, "model.safetensors.index.json")
        if os.path.exists(idx):
            with open(idx) as f:
                wmap = json.load(f)["weight_map"]
            for name, shard in wmap.items():
                if name.startswith(TEXT_PREFIX):
                    self._where[name[len(TEXT_PREFIX):]] = (os.path.join(self.path, shard), name)
        else:
            from safetensors import safe_open
            single = os.path.join(self.path, "model.safetensors")
            if not os.path.exists(single):
                raise FileNotFoundError(f"no model.safetensors(.index.json) in {self.path}")
            with safe_open(single, "pt") as f:
                for name in f.keys():
                    if name.startswith(TEXT_PREFIX):
                        self._where[name[len(TEXT_PREFIX):]] = (single, name)

    def _index_bundle(self, manifest: dict):
        from safetensors import safe_open
        self.is_bundle = True
        default = manifest.get("default_variant")
        variant = next((v for v in manifest.get("variants", []) if v.get("id") == default), None)
        if variant is None:
            raise ValueError("bundle manifest: default_variant not found")
        q = variant.get("quantization", {})
        self.bits = int(q.get("bits", 0))
        self.group_size = int(q.get("group_size", 64))
        base = os.path.join(self.path, variant["path"])
        for fname in variant["files"]:
            fp = os.path.join(base, fname)
            with safe_open(fp, "pt") as f:
                for name in f.keys():
                    self._where[name] = (fp, name)

    # ------------------------------------------------------------------ access
    def has(self, key: str) -> bool:
        return key in self._where

    def has_quantized(self, key: str) -> bool:
        return (key + ".scales") in self._where

    def get(self, key: str, device="cpu") -> torch.Tensor:
        from safetensors import safe_open
        if key not in self._where:
            raise KeyError(f"{key} not found in {self.path}")
        fp, name = self._where[key]
        with safe_open(fp, "pt") as f:
            t = f.get_tensor(name)
        if not self.is_bundle and t.is_floating_point():
            t = t.to(torch.bfloat16)  # computeDtype cast (ESWeightLoader.mm:52)
        return t.to(device)

    def moe_layer(self, i: int, device="cpu") -> Dict[str, torch.Tensor]:
        """The MoE tensors of decoder layer i, keyed by their layer suffix;
        quantised expert triples add `<suffix>.scales` / `.biases`."""
        out = {}
        for suf in MOE_SUFFIXES:
            key = layer_key(i, suf)
            out[suf] = self.get(key, device)
            if suf.startswith("experts.") and self.has_quantized(key):
                out[suf + ".scales"] = self.get(key + ".scales", device)
                out[suf + ".biases"] = self.get(key + ".biases", device)
        return out


def block_from_checkpoint(path: str, layer: int, cfg=None, device: int = 0,
                          quant_bits: Optional[int] = None, max_tokens: int = 8192):
    """MoEBlock of one decoder layer, built from a checkpoint or bundle (the
    router and esMakeExperts part of the ESDecoderLayer ctor, ESDecoderLayer.mm:35-43)."""
    from .moe import ESModelConfig, MoEBlock
    if cfg is None:
        cfg = ESModelConfig.from_config_json(os.path.join(path, "config.json"))
    cfg.max_tokens, cfg.device = max_tokens, device
    ld = MoEWeightLoader(path)
    dev = torch.device("cuda", device)
    w = ld.moe_layer(layer, dev)
    r = (w["router.proj.weight"].contiguous(), w["router.scale"].contiguous(),
         w["router.per_expert_scale"].contiguous())
    gu, dn = "experts.gate_up_proj", "experts.down_proj"
    if gu + ".scales" in w:
        q = dict(gu_q=w[gu].contiguous(), gu_s=w[gu + ".scales"].contiguous(),
                 gu_b=w[gu + ".biases"].contiguous(), dn_q=w[dn].contiguous(),
                 dn_s=w[dn + ".scales"].contiguous(), dn_b=w[dn + ".biases"].contiguous(),
                 bits=ld.bits, group_size=ld.group_size)
        return MoEBlock(cfg, *r, quantized=q)
    if quant_bits is not None:
        cfg.quant_bits = quant_bits
    return MoEBlock(cfg, *r, w[gu].contiguous(), w[dn].contiguous())
