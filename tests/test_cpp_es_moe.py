"""The C++ host side: include/es_weight_loader.hpp (ESWeightLoader's MoE
subset: HF safetensors checkpoints, .apml bundles) and include/es_moe.hpp
(es::ESRouter / es::ESExperts with the reference constructor signatures,
esMakeExperts), driven by tests/cpp/es_moe_driver.cpp.

CPU: the loader reads a sharded HF checkpoint (text prefix stripped, f32 cast
to bf16, vision tensors ignored) and a quantised bundle (triples adopted
verbatim) exactly as apertura_b200/weights.py does.
GPU: router + experts built from those directories match the CPU oracle."""
import json
import os
import subprocess

import numpy as np
import pytest
import torch
from safetensors.torch import save_file

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "es_moe_driver.cpp")
H, E, K, I, T = 256, 32, 8, 128, 5
P = "model.language_model."


def _gcc():
    cmd = ["g++", "-O2", "-std=c++17", "-I", os.path.join(ROOT, "include")]
    lib = "/usr/lib/gcc/x86_64-linux-gnu/13/"
    if os.path.isdir(lib):
        cmd.insert(1, "-B" + lib)
    return cmd


def build(out_dir, cuda):
    exe = os.path.join(out_dir, "es_moe_driver" + ("" if cuda else "_cpu"))
    cmd = _gcc() + [SRC, "-o", exe]
    if cuda:
        from apertura_b200 import build as B
        B.build()
        libdir = os.path.join(ROOT, "apertura_b200")
        cmd += ["-I", "/usr/local/cuda/include", "-L", libdir, "-lapt_moe",
                "-L", "/usr/local/cuda/lib64", "-lcudart",
                "-Wl,-rpath," + libdir + ":/usr/local/cuda/lib64"]
    else:
        cmd.insert(-3, "-DES_DRIVER_CPU_ONLY")
    subprocess.run(cmd, check=True)
    return exe


def _tensors(seed=0):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s, std=1.0: torch.randn(*s, generator=g) * std
    return dict(proj=r(E, H, std=H ** -0.5), scale=1.0 + 0.1 * r(H), pes=1.0 + 0.1 * r(E),
                gate_up=r(E, 2 * I, H, std=0.02).to(torch.bfloat16),
                down=r(E, H, I, std=0.02).to(torch.bfloat16))


def _config(d):
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump({"text_config": {"hidden_size": H, "num_experts": E, "top_k_experts": K,
                                   "moe_intermediate_size": I, "rms_norm_eps": 1e-6,
                                   "enable_moe_block": True}}, f)


def make_hf(d, t):
    """Two shards: f32 router tensors, bf16 experts, a vision tensor."""
    s0 = {P + "layers.0.router.proj.weight": t["proj"], P + "layers.0.router.scale": t["scale"],
          P + "layers.0.experts.gate_up_proj": t["gate_up"],
          "model.vision_tower.patch.weight": torch.zeros(4, 4)}
    s1 = {P + "layers.0.router.per_expert_scale": t["pes"],
          P + "layers.0.experts.down_proj": t["down"]}
    save_file(s0, os.path.join(d, "model-00001.safetensors"))
    save_file(s1, os.path.join(d, "model-00002.safetensors"))
    wmap = {k: "model-00001.safetensors" for k in s0}
    wmap.update({k: "model-00002.safetensors" for k in s1})
    with open(os.path.join(d, "model.safetensors.index.json"), "w") as f:
        json.dump({"weight_map": wmap}, f)
    _config(d)


def make_bundle(d, t, oracle, bits=4):
    gq = oracle.quantize_affine(t["gate_up"].view(torch.int16).numpy().view(np.uint16), 64, bits)
    dq = oracle.quantize_affine(t["down"].view(torch.int16).numpy().view(np.uint16), 64, bits)
    tb = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)
    tu = lambda a: torch.from_numpy(a.view(np.int32))
    L = "layers.0."
    tensors = {L + "router.proj.weight": t["proj"].to(torch.bfloat16),
               L + "router.scale": t["scale"].to(torch.bfloat16),
               L + "router.per_expert_scale": t["pes"].to(torch.bfloat16),
               L + "experts.gate_up_proj": tu(gq[0]), L + "experts.gate_up_proj.scales": tb(gq[1]),
               L + "experts.gate_up_proj.biases": tb(gq[2]), L + "experts.down_proj": tu(dq[0]),
               L + "experts.down_proj.scales": tb(dq[1]), L + "experts.down_proj.biases": tb(dq[2])}
    os.makedirs(os.path.join(d, "weights", "mlx-q4"))
    save_file(tensors, os.path.join(d, "weights", "mlx-q4", "model.safetensors"))
    with open(os.path.join(d, "manifest.json"), "w") as f:
        json.dump({"kind": "apertura-model", "default_variant": "mlx-q4",
                   "variants": [{"id": "mlx-q4", "path": "weights/mlx-q4",
                                 "files": ["model.safetensors"],
                                 "quantization": {"bits": bits, "group_size": 64,
                                                  "embed_bits": 8}}]}, f)
    _config(d)
    return gq, dq


def _fnv(b: bytes) -> int:
    s = 0
    for x in b:
        s = (s * 1099511628211 + x) & 0xFFFFFFFFFFFFFFFF
    return s


def _listing(exe, d):
    r = subprocess.run([exe, "list", d, "0"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    rows = {}
    for ln in r.stdout.splitlines()[:-1]:
        f = ln.split()
        rows[f[0]] = (f[1], tuple(int(v) for v in f[2:-1]), int(f[-1]))
    return rows, r.stdout.splitlines()[-1]


def test_cpp_loader_hf_and_bundle(tmp_path, oracle):
    from apertura_b200.weights import MoEWeightLoader
    exe = build(str(tmp_path), cuda=False)
    t = _tensors()
    hf = tmp_path / "hf"
    hf.mkdir()
    make_hf(str(hf), t)
    rows, tail = _listing(exe, str(hf))
    assert tail == "bundle=0 bits=0 group=64 quantized=0"
    py = MoEWeightLoader(str(hf)).moe_layer(0)
    assert set(rows) == {"layers.0." + k for k in py}
    for k, v in py.items():
        dt, shape, chk = rows["layers.0." + k]
        assert dt == "bf16" and shape == tuple(v.shape)  # f32 cast to the compute dtype
        assert chk == _fnv(v.contiguous().view(torch.int16).numpy().tobytes()), k
    bd = tmp_path / "bundle"
    bd.mkdir()
    make_bundle(str(bd), t, oracle)
    rows, tail = _listing(exe, str(bd))
    assert tail == "bundle=1 bits=4 group=64 quantized=1"
    pyb = MoEWeightLoader(str(bd)).moe_layer(0)
    for k, v in pyb.items():
        dt, shape, chk = rows["layers.0." + k]
        # packed codes keep their stored 32-bit type (u32 from MLX, i32 here)
        assert dt == ("i32" if v.dtype == torch.int32 else "bf16") and shape == tuple(v.shape)
        raw = v.contiguous().view(torch.int32 if v.dtype == torch.int32 else torch.int16)
        assert chk == _fnv(raw.numpy().tobytes()), k


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["hf", "bundle"])
def test_cpp_es_classes_vs_oracle(tmp_path, oracle, kind):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from tests.helpers import bf16_to_f32, block_close, router_index_check
    exe = build(str(tmp_path), cuda=True)
    t = _tensors(seed=3)
    d = tmp_path / kind
    d.mkdir()
    if kind == "hf":
        make_hf(str(d), t)
    else:
        gq, dq = make_bundle(str(d), t, oracle)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
    xb = x.view(torch.int16).numpy().view(np.uint16)
    xb.tofile(str(tmp_path / "x.bin"))
    outp = str(tmp_path / "out")
    r = subprocess.run([exe, "run", str(d), "0", str(T), str(tmp_path / "x.bin"), outp],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    idx = np.fromfile(outp + ".idx", np.int32).reshape(T, K)
    w = np.fromfile(outp + ".w", np.uint16).reshape(T, K)
    bf = lambda a: a.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    proj, scale, pes = bf(t["proj"]), bf(t["scale"]), bf(t["pes"])
    idx_o, w_o, aux = oracle.route_topk(xb, proj, scale, pes, K, return_scores=True)
    bad, _ = router_index_check(idx, idx_o, aux["scores"])
    assert bad == 0
    got = bf16_to_f32(np.fromfile(outp + ".sparse", np.uint16)).reshape(T, H)
    gu, dn = bf(t["gate_up"]), bf(t["down"])
    if kind == "hf":
        ref = oracle.experts_sparse(xb, gu, dn, idx, w)
        dense = bf16_to_f32(np.fromfile(outp + ".dense", np.uint16)).reshape(T, H)
        W = oracle.route_weights(idx, w, E)
        refd = bf16_to_f32(oracle.experts_dense(xb, gu, dn, W))
        ok, ma, cos = block_close(dense, refd)
        assert ok, ("dense", ma, cos)
    else:
        ref = oracle.experts_sparse_q(xb, *gq, *dq, 4, 64, idx, w, I)
    refv = bf16_to_f32(ref)
    ok, ma, cos = block_close(got, refv)
    assert ok and ma <= 2.0 ** -6 * np.abs(refv).max(), (ma, cos)
