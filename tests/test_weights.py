"""Expert-weight ingest (apertura_b200/weights.py) against synthetic HF and
bundle directories laid out as ESWeightLoader expects."""
import json
import os

import numpy as np
import pytest
import torch
from safetensors.torch import save_file

from apertura_b200.weights import MoEWeightLoader, layer_key

H, E, I = 64, 16, 64
P = "model.language_model."


def _hf_dir(tmp_path):
    g = torch.Generator().manual_seed(0)
    t = lambda *s: torch.randn(*s, generator=g)
    shard0 = {P + "layers.0.router.proj.weight": t(E, H), P + "layers.0.router.scale": t(H),
              P + "layers.0.router.per_expert_scale": t(E),
              P + "layers.0.experts.gate_up_proj": t(E, 2 * I, H).to(torch.bfloat16),
              "model.vision_tower.patch.weight": t(4, 4)}
    shard1 = {P + "layers.0.experts.down_proj": t(E, H, I), P + "layers.1.router.scale": t(H)}
    save_file(shard0, os.path.join(tmp_path, "model-00001.safetensors"))
    save_file(shard1, os.path.join(tmp_path, "model-00002.safetensors"))
    wmap = {k: "model-00001.safetensors" for k in shard0}
    wmap.update({k: "model-00002.safetensors" for k in shard1})
    with open(os.path.join(tmp_path, "model.safetensors.index.json"), "w") as f:
        json.dump({"weight_map": wmap}, f)
    return shard0, shard1


def test_hf_layer_keys_prefix_and_cast(tmp_path):
    s0, s1 = _hf_dir(tmp_path)
    ld = MoEWeightLoader(str(tmp_path))
    assert not ld.is_bundle
    assert ld.has(layer_key(0, "experts.down_proj"))
    assert not ld.has("vision_tower.patch.weight")  # outside the text prefix
    w = ld.moe_layer(0)
    assert set(w) == {"router.proj.weight", "router.scale", "router.per_expert_scale",
                      "experts.gate_up_proj", "experts.down_proj"}
    for v in w.values():
        assert v.dtype == torch.bfloat16  # cast to the compute dtype
    assert torch.equal(w["experts.down_proj"], s1[P + "layers.0.experts.down_proj"].to(torch.bfloat16))
    assert not ld.has_quantized(layer_key(0, "experts.gate_up_proj"))
    with pytest.raises(KeyError):
        ld.moe_layer(1)  # layer 1 has only a scale


def test_bundle_quantised_triples(tmp_path):
    from oracle import oracle as O
    rng = np.random.default_rng(1)
    gu = O.f32_to_bf16(0.02 * rng.standard_normal((E, 2 * I, H)))
    dn = O.f32_to_bf16(0.02 * rng.standard_normal((E, H, I)))
    gq, dq = O.quantize_affine(gu, 64, 4), O.quantize_affine(dn, 64, 4)
    tb = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)
    tu = lambda a: torch.from_numpy(a.astype(np.uint32))
    tensors = {"layers.0.router.proj.weight": torch.zeros(E, H, dtype=torch.bfloat16),
               "layers.0.router.scale": torch.ones(H, dtype=torch.bfloat16),
               "layers.0.router.per_expert_scale": torch.ones(E, dtype=torch.bfloat16),
               "layers.0.experts.gate_up_proj": tu(gq[0]),
               "layers.0.experts.gate_up_proj.scales": tb(gq[1]),
               "layers.0.experts.gate_up_proj.biases": tb(gq[2]),
               "layers.0.experts.down_proj": tu(dq[0]),
               "layers.0.experts.down_proj.scales": tb(dq[1]),
               "layers.0.experts.down_proj.biases": tb(dq[2])}
    os.makedirs(os.path.join(tmp_path, "weights", "mlx-q4"))
    save_file(tensors, os.path.join(tmp_path, "weights", "mlx-q4", "model.safetensors"))
    manifest = {"kind": "apertura-model", "default_variant": "q4",
                "variants": [{"id": "q4", "path": "weights/mlx-q4", "files": ["model.safetensors"],
                              "quantization": {"bits": 4, "group_size": 64, "embed_bits": 0}}]}
    with open(os.path.join(tmp_path, "manifest.json"), "w") as f:
        json.dump(manifest, f)
    ld = MoEWeightLoader(str(tmp_path))
    assert ld.is_bundle and ld.bits == 4 and ld.group_size == 64
    w = ld.moe_layer(0)
    assert w["experts.gate_up_proj"].dtype == torch.uint32  # verbatim
    assert "experts.down_proj.scales" in w and "experts.down_proj.biases" in w
    assert np.array_equal(w["experts.gate_up_proj"].numpy(), gq[0])


def test_bundle_rejects_foreign_manifest(tmp_path):
    with open(os.path.join(tmp_path, "manifest.json"), "w") as f:
        json.dump({"kind": "something-else"}, f)
    with pytest.raises(ValueError):
        MoEWeightLoader(str(tmp_path))


@pytest.mark.gpu
def test_block_from_checkpoint_matches_direct(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import apertura_b200 as A
    from apertura_b200.synthetic import block_inputs
    from apertura_b200.weights import block_from_checkpoint
    dev = torch.device("cuda", 0)
    Hb, Eb, Kb, Ib, T = 256, 32, 8, 128, 6
    d = block_inputs(T, seed=3, device=dev, H=Hb, E=Eb, K=Kb, I=Ib, nonunit=True)
    names = {"router.proj.weight": d["proj"], "router.scale": d["scale"],
             "router.per_expert_scale": d["pes"], "experts.gate_up_proj": d["gate_up"],
             "experts.down_proj": d["down"]}
    save_file({P + "layers.3." + k: v.cpu().contiguous() for k, v in names.items()},
              os.path.join(tmp_path, "model.safetensors"))
    with open(os.path.join(tmp_path, "config.json"), "w") as f:
        json.dump({"text_config": {"hidden_size": Hb, "num_experts": Eb, "top_k_experts": Kb,
                                   "moe_intermediate_size": Ib, "enable_moe_block": True}}, f)
    blk = block_from_checkpoint(str(tmp_path), 3, max_tokens=T)
    cfg = A.ESModelConfig(hidden_size=Hb, num_experts=Eb, top_k_experts=Kb,
                          moe_intermediate_size=Ib, moe_sparse=False, max_tokens=T)
    ref = A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], d["gate_up"], d["down"])
    # the checkpoint's config keeps the reference default (dense, moeSparse=false)
    assert blk.cfg.moe_sparse is False
    a, b = blk.forward(d["x"]), ref.forward(d["x"])
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_make_experts_bits_from_triple_shapes(monkeypatch):
    """esMakeExperts adopts a bundle's triples at the bundle's width; without
    an explicit bundle_bits it follows from the shapes (4-bit and 8-bit)."""
    import apertura_b200.moe as M
    seen = {}
    monkeypatch.setattr(M.ESExperts, "from_quantized",
                        classmethod(lambda cls, *a, **kw: seen.setdefault("bits", a[6])))
    for bits in (4, 8):
        seen.clear()
        w = {"g": torch.zeros(2, 8, 256 * bits // 32, dtype=torch.int32),
             "g.scales": torch.zeros(2, 8, 4, dtype=torch.bfloat16),
             "g.biases": torch.zeros(2, 8, 4, dtype=torch.bfloat16),
             "d": torch.zeros(2, 256, 4 * bits // 32 * 8, dtype=torch.int32),
             "d.scales": torch.zeros(2, 256, 1), "d.biases": torch.zeros(2, 256, 1)}
        M.make_experts(w, "g", "d")
        assert seen["bits"] == bits
    seen.clear()
    M.make_experts(w, "g", "d", bundle_bits=8)
    assert seen["bits"] == 8
