"""Expert parallelism on 2 GPUs (NCCL): the EP block equals the single-GPU
block on every rank's tokens.  Skipped when fewer than 2 GPUs are visible."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r'''
import os, sys, numpy as np, torch, torch.distributed as dist
sys.path.insert(0, os.environ["APT_ROOT"])
import apertura_b200 as A
from apertura_b200.ep import ExpertParallelMoE, NativeExpertParallelMoE
from apertura_b200.synthetic import block_inputs, expert_bank
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank); dev = torch.device("cuda", rank)
dist.init_process_group("nccl", device_id=dev)
T = int(os.environ["APT_T"])
# one Zipf-routed token set and router, split over the ranks
r0 = block_inputs(T * world, seed=1000, device=dev, routing="zipf", with_experts=False)
d = dict(x=r0["x"][rank * T:(rank + 1) * T].contiguous())
gu, dn = expert_bank(128, 2816, 704, 7, dev)
cfg = A.ESModelConfig(moe_sparse=True, max_tokens=T, device=rank)
loads = r0["zipf"]["target"].tolist()  # the expected loads of this routing
make = NativeExpertParallelMoE if os.environ.get("APT_NATIVE") == "1" else ExpertParallelMoE
ep = make(cfg, r0["proj"], r0["scale"], r0["pes"], gu, dn, loads=loads, max_tokens_per_rank=T)
out = ep(d["x"])
recv, hot = ep.stats() if make is NativeExpertParallelMoE else (ep.last_recv_rows, ep.last_hot_rows)
ref_blk = A.MoEBlock(cfg, r0["proj"], r0["scale"], r0["pes"], gu, dn)
ref = ref_blk.forward(d["x"])
torch.cuda.synchronize()
ma = float((out.float() - ref.float()).abs().max()); peak = float(ref.float().abs().max())
cos = float(torch.nn.functional.cosine_similarity(out.float().flatten(), ref.float().flatten(), 0))
print(f"\nRESULT rank={rank} max_abs={ma:.3e} peak={peak:.3e} cos={cos:.6f} recv={recv} hot={hot}")
ok = ma <= 2e-2 and cos >= 0.9999
dist.destroy_process_group()
sys.exit(0 if ok else 3)
'''


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
@pytest.mark.parametrize("T,native", [(64, False), (2048, False), (64, True), (2048, True)])
def test_ep_two_gpus_matches_single_gpu(tmp_path, T, native):
    """Python-orchestrated (ExpertParallelMoE) and C-ABI (apt_moe_create_ep) forms."""
    script = tmp_path / "ep_worker.py"
    script.write_text(WORKER)
    env = dict(os.environ, APT_ROOT=ROOT, APT_T=str(T), NCCL_NVLS_ENABLE="0",
               APT_NATIVE="1" if native else "0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(29600 + T % 97 + (7 if native else 0)), str(script)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    # each rank exits 3 if its outputs miss the bar; ranks' lines may interleave
    assert r.returncode == 0 and r.stdout.count("RESULT rank=") == 2, (
        r.returncode, r.stdout[-2000:], r.stderr[-3000:])
