"""The C++ boundary: tests/cpp/moe_cpp_driver.cpp (g++, include/es_moe_cuda.hpp,
linked against libapt_moe.so) runs the block from host buffers; its output
must match the CPU oracle.  The build half runs on CPU; the run half on GPU."""
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "moe_cpp_driver.cpp")


def build_driver(out_dir):
    from apertura_b200 import build as B
    B.build()
    exe = os.path.join(out_dir, "moe_cpp_driver")
    gcc_lib = "/usr/lib/gcc/x86_64-linux-gnu/13/"
    cmd = ["g++", "-O2", "-std=c++17", "-I", os.path.join(ROOT, "include"), SRC, "-o", exe,
           "-L", os.path.join(ROOT, "apertura_b200"), "-lapt_moe",
           "-Wl,-rpath," + os.path.join(ROOT, "apertura_b200")]
    if os.path.isdir(gcc_lib):
        cmd.insert(1, "-B" + gcc_lib)
    subprocess.run(cmd, check=True)
    return exe


def test_cpp_driver_builds(tmp_path):
    exe = build_driver(str(tmp_path))
    r = subprocess.run([exe], capture_output=True, text=True)
    assert r.returncode == 2 and "usage" in r.stderr


@pytest.mark.gpu
def test_cpp_driver_matches_oracle(tmp_path, oracle):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    exe = build_driver(str(tmp_path))
    H, E, K, I, T = 256, 32, 8, 128, 5
    rng = np.random.default_rng(9)
    bf = lambda a: oracle.f32_to_bf16(np.asarray(a, np.float32))
    data = dict(proj=bf(rng.standard_normal((E, H)) / np.sqrt(H)), scale=bf(np.ones(H)),
                pes=bf(np.ones(E)), gate_up=bf(0.02 * rng.standard_normal((E, 2 * I, H))),
                down=bf(0.02 * rng.standard_normal((E, H, I))), x=bf(rng.standard_normal((T, H))))
    for k, v in data.items():
        v.tofile(os.path.join(tmp_path, f"{k}.bin"))
    cfgp = os.path.join(tmp_path, "config.json")
    with open(cfgp, "w") as f:
        f.write('{"text_config": {"hidden_size": %d, "num_experts": %d, "top_k_experts": %d, '
                '"moe_intermediate_size": %d, "enable_moe_block": true}}' % (H, E, K, I))
    r = subprocess.run([exe, cfgp, str(tmp_path), str(T)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    got = oracle.bf16_to_f32(np.fromfile(os.path.join(tmp_path, "out.bin"), np.uint16))
    idx, w = oracle.route_topk(data["x"], data["proj"], data["scale"], data["pes"], K)
    ref = oracle.bf16_to_f32(oracle.experts_sparse(data["x"], data["gate_up"], data["down"], idx, w))
    from tests.helpers import block_close
    ok, ma, cos = block_close(got, ref.ravel())
    assert ok, (ma, cos)
