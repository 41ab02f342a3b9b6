"""Benchmark of the B200 Gemma-4 MoE block (ESRouter + ESExperts).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--no-prefill] [--no-cpu-baseline]

Workload (the decode sweep): one step is one
MoE-block forward at each T in {1, 4, 16, 64} on the Gemma-4-26B block shape
(H=2816, E=128, top-8, I=704, bf16), seeded synthetic inputs, uniform-ish
routing.  value = tokens/s over the whole job (85 tokens per step per GPU).
L2 is flushed (a 256 MiB read, which also writes back dirty lines) before
every timed forward and the flush is outside the timed events.  The prefill config (T=8192, Zipf(1.1) routing) is
reported as an extra object.

``--impl reference`` times the CPU oracle (the C restatement of the
reference's mx:: op sequence; MLX itself is not installed) on the host cores
for the same workload.  Under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE-block tokens/s (decode T=1..64, prefill T=8192); % of HBM / TC roofline"
SWEEP = (1, 4, 16, 64)
H, E, K, I = 2816, 128, 8, 704
EXPERT_BYTES = (2 * I * H + H * I) * 2          # 11,894,784 B per touched expert
GATEUP_BYTES = 2 * I * H * 2                    # gate_up part of it
# DRAM bytes read by the four expert-stage launches of one sweep step (T=1,4,16,64),
# from an ncu capture (dram__bytes_read.sum); the command and the per-T figures
# are in profiles/decode_sweep_traffic.txt.
GATEUP_SWEEP_TRAFFIC = 2149.07e6  # dram__bytes_read.sum, profiles/decode_sweep_traffic.txt
ROUTER_BYTES = E * H * 2                        # 720,896 B


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return dict(hbm=d["hbm_gbs"], tc=d["bf16_tflops"], tc_sust=d["bf16_tflops_sustained"],
                    src="measured")
    return dict(hbm=6650.0, tc=1590.0, tc_sust=1400.0, src="fallback")


class ClockSampler:
    """SM clock, max clock and clock-event (throttle) reasons of one GPU, read
    every ~10 ms from a thread while the timed region runs: through NVML when
    the bindings are importable, else nvidia-smi every ~200 ms.  Read-only."""

    # NVML clocks-event reason bits
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
            "hw_thermal_slowdown": 0x40}
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.sm, self.mx, self.reasons = [], None, set()
        self.stop = threading.Event()

    def _poll_nvml(self, nv):
        # the CUDA device's own GPU (NVML numbers all GPUs of the machine)
        h = None
        try:
            import torch
            uuid = getattr(torch.cuda.get_device_properties(self.index), "uuid", None)
            if uuid is not None:
                h = nv.nvmlDeviceGetHandleByUUID(f"GPU-{uuid}")
        except Exception:
            h = None
        if h is None:
            h = nv.nvmlDeviceGetHandleByIndex(self.index)
        self.mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons")
        while not self.stop.is_set():
            self.sm.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
            bits = get_reasons(h)
            for n, b in self.BITS.items():
                if bits & b:
                    self.reasons.add(n)
            self.stop.wait(0.01)

    def _poll_smi(self):
        cmd = ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
               "--format=csv,noheader,nounits"]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        while not self.stop.is_set():
            try:
                r = subprocess.run(cmd, capture_output=True, text=True, timeout=5)
            except Exception:
                return
            for ln in r.stdout.splitlines():
                f = [x.strip() for x in ln.split(",")]
                if len(f) < 8:
                    continue
                try:
                    self.sm.append(float(f[1]))
                    self.mx = float(f[2])
                except ValueError:
                    continue
                for n, v in zip(names, f[4:8]):
                    if v.lower().startswith("active"):
                        self.reasons.add(n)
            self.stop.wait(0.2)

    def _poll(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
        except Exception:
            return self._poll_smi()
        try:
            self._poll_nvml(nv)
        except Exception:
            if not self.sm:
                self._poll_smi()
        finally:
            try:
                nv.nvmlShutdown()
            except Exception:
                pass

    def __enter__(self):
        self.t = threading.Thread(target=self._poll, daemon=True)
        self.t.start()
        return self

    def __exit__(self, *a):
        self.stop.set()
        self.t.join(timeout=10)

    def summary(self):
        if not self.sm:
            return {"sm_mhz": None, "sm_max_mhz": self.mx, "reasons": [], "samples": 0}
        sm = sorted(self.sm)
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": self.mx, "reasons": sorted(self.reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------- helpers

def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def n_unique(idx):
    import torch
    return int(torch.unique(idx).numel())


def oracle_sweep_inputs(d_by_T, gate_up, down):
    """CPU copies (numpy bf16 bits) for the oracle."""
    from apertura_b200.synthetic import to_numpy_bits as nb
    xs = {T: nb(d["x"]) for T, d in d_by_T.items()}
    d0 = next(iter(d_by_T.values()))
    return dict(xs=xs, proj=nb(d0["proj"]), scale=nb(d0["scale"]), pes=nb(d0["pes"]),
                gate_up=nb(gate_up), down=nb(down))


def time_oracle_sweep(o, budget_s=12.0, max_passes=400):
    """Oracle (route + sparse experts) over the sweep until `budget_s` elapses.
    Returns (tokens/s, passes, seconds, threads)."""
    from oracle import oracle as O
    O.build()
    O.set_num_threads(host_cores())
    passes, t0 = 0, time.perf_counter()
    while True:
        for T, x in o["xs"].items():
            idx, w = O.route_topk(x, o["proj"], o["scale"], o["pes"], K)
            O.experts_sparse(x, o["gate_up"], o["down"], idx, w)
        passes += 1
        el = time.perf_counter() - t0
        if el >= budget_s or passes >= max_passes:
            break
    return passes * sum(SWEEP) / el, passes, el, O.num_threads()


def make_sweep_inputs(dev, seed=0):
    from apertura_b200.synthetic import block_inputs, expert_bank
    gate_up, down = expert_bank(E, H, I, seed, dev)
    # one router and 85 distinct tokens, split over the sweep's T values
    d = block_inputs(sum(SWEEP), seed=seed, device=dev, with_experts=False)
    d_by_T, t0 = {}, 0
    for T in SWEEP:
        d_by_T[T] = dict(d, x=d["x"][t0:t0 + T].contiguous(), T=T)
        t0 += T
    return d_by_T, gate_up, down


# --------------------------------------------------------------------- reference arm

def run_reference(args):
    world, rank, local = dist_env()
    if rank != 0:
        return 0
    import torch
    dev = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    d_by_T, gate_up, down = make_sweep_inputs(dev)
    o = oracle_sweep_inputs(d_by_T, gate_up, down)
    from oracle import oracle as O
    O.build()
    # every host core (torchrun starts ranks with one OpenMP thread)
    O.set_num_threads(host_cores())
    # warm-up passes (untimed), then K timed sweep passes, each its own step
    for _ in range(max(args.warmup, 0)):
        x = o["xs"][1]
        idx, w = O.route_topk(x, o["proj"], o["scale"], o["pes"], K)
        O.experts_sparse(x, o["gate_up"], o["down"], idx, w)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for T, x in o["xs"].items():
            idx, w = O.route_topk(x, o["proj"], o["scale"], o["pes"], K)
            O.experts_sparse(x, o["gate_up"], o["down"], idx, w)
    el = time.perf_counter() - t0
    tps = args.steps * sum(SWEEP) / el
    sample = (f"{args.steps} passes of the decode sweep T in {SWEEP} (route + sparse experts), "
              f"C restatement of ESRouter.mm/ESExperts.mm with OpenMP (MLX not installed)")
    line = {
        "metric": METRIC, "value": tps, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": "decode sweep T in {1,4,16,64}, Gemma-4-26B MoE block "
                               "(H=2816,E=128,K=8,I=704), bf16, uniform routing, CPU"},
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": O.num_threads(),
                         "per_core": tps / O.num_threads(), "kind": "port", "sample": sample},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------- our arm

def run_ours(args):
    import torch
    import torch.distributed as dist
    import apertura_b200 as A
    from apertura_b200 import build as B

    world, rank, local = dist_env()
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B.build()
    peaks = load_peaks()

    d_by_T, gate_up, down = make_sweep_inputs(dev, seed=rank)
    d0 = d_by_T[SWEEP[0]]
    cfg = A.ESModelConfig(moe_sparse=True, max_tokens=8192 if args.prefill else max(SWEEP),
                          device=local)
    blk = A.MoEBlock(cfg, d0["proj"], d0["scale"], d0["pes"], gate_up, down)
    if args.gemv_max_tokens is not None:
        blk.handle.set_gemv_max_tokens(args.gemv_max_tokens)
    flush = torch.ones(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def forward_T(T):
        return blk.forward(d_by_T[T]["x"])

    # routing stats per T (U = distinct experts touched)
    U = {}
    for T in SWEEP:
        _, tk = blk.forward(d_by_T[T]["x"], return_routing=True)
        U[T] = n_unique(tk.idx)
    launches_per_step = 0
    for T in SWEEP:
        forward_T(T)
        launches_per_step += blk.handle.last_launches()
    for _ in range(args.warmup):
        for T in SWEEP:
            forward_T(T)
    torch.cuda.synchronize()

    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps * len(SWEEP))]
    per_T_ms = {T: 0.0 for T in SWEEP}
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        i = 0
        for _ in range(args.steps):
            for T in SWEEP:
                flush.sum()                         # evict L2 (outside the events)
                a, b = evs[i]
                a.record(stream)
                forward_T(T)
                b.record(stream)
                i += 1
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
    i = 0
    total_ms = 0.0
    for _ in range(args.steps):
        for T in SWEEP:
            ms = evs[i][0].elapsed_time(evs[i][1])
            per_T_ms[T] += ms / args.steps
            total_ms += ms
            i += 1
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    value = world * sum(SWEEP) / (ms_per_step / 1e3)

    # per-stage times (separate untimed-for-value pass with stage events on)
    blk.handle.set_timing(True)
    stage = {T: {} for T in SWEEP}
    reps = 5
    for _ in range(reps):
        for T in SWEEP:
            flush.sum()
            forward_T(T)
            for k, v in blk.handle.stage_times().items():
                stage[T][k] = stage[T].get(k, 0.0) + v / reps
    blk.handle.set_timing(False)

    # roofline of the dominant kernel over the sweep: the weight-streaming
    # expert stage.  T <= 8 runs the whole block as one kernel
    # (decode_fused_kernel, its only stage): its bytes are the block's; T > 8
    # runs the tcgen05 gate_up GEMM: its bytes are the gate_up weights + rows.
    block_bytes = {T: U[T] * EXPERT_BYTES + ROUTER_BYTES + T * H * 2 * 2 + T * K * 6
                   for T in SWEEP}
    fused = {T: "down" not in stage[T] for T in SWEEP}
    gu_bytes = sum(block_bytes[T] if fused[T] else U[T] * GATEUP_BYTES + T * H * 2 + T * K * I * 2
                   for T in SWEEP)
    gu_ms = sum(stage[T].get("gate_up", 0.0) for T in SWEEP)
    achieved = gu_bytes / (gu_ms / 1e3) / 1e9
    sweep_detail = {
        str(T): {"ms": per_T_ms[T], "tokens_per_s": T / (per_T_ms[T] / 1e3), "U": U[T],
                 "block_GBps": block_bytes[T] / (per_T_ms[T] / 1e3) / 1e9,
                 "block_hbm_frac": block_bytes[T] / (per_T_ms[T] / 1e3) / 1e9 / peaks["hbm"],
                 "stages_ms": stage[T]}
        for T in SWEEP}

    # e2e through the C ABI with host buffers (pinned), copies inside the events
    xh = {T: d_by_T[T]["x"].cpu().pin_memory() for T in SWEEP}
    oh = {T: torch.empty(T, H, dtype=torch.bfloat16).pin_memory() for T in SWEEP}
    for T in SWEEP:
        blk.forward_host(xh[T], oh[T])
    # Each timed forward: pinned host x -> device -> block -> host out, queued
    # through apt_moe_forward_host_async; the step's result is read on the host
    # after one synchronisation per step (a decode engine's pattern).  The L2
    # flush before each forward stays outside the events.
    e2e_ms = 0.0
    for _ in range(args.steps):
        evs = []
        for T in SWEEP:
            flush.sum()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            blk.forward_host(xh[T], oh[T], asynchronous=True)
            b.record(stream)
            evs.append((a, b))
        evs[-1][1].synchronize()
        checksum = float(sum(oh[T][0, :8].float().sum() for T in SWEEP))  # read the results
        e2e_ms += sum(a.elapsed_time(b) for a, b in evs)
        assert checksum == checksum, "NaN in the block output"
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = {"value": world * sum(SWEEP) * args.steps / (e2e_ms / 1e3), "unit": "tokens/s",
           "h2d_bytes_per_step": sum(SWEEP) * H * 2, "d2h_bytes_per_step": sum(SWEEP) * H * 2}

    prefill = run_prefill(blk, dev, peaks, flush) if args.prefill else None
    ep = None
    if args.ep:
        try:
            ep = run_ep(args, dev, world, rank)
        except Exception as e:  # the EP extra must not cost the headline line
            ep = {"error": f"{type(e).__name__}: {e}"[:300]}
    quant = run_quant(dev, peaks, flush) if args.quant else None

    cpu = None
    if rank == 0 and world == 1 and args.cpu_baseline:
        o = oracle_sweep_inputs(d_by_T, gate_up, down)
        tps, passes, el, thr = time_oracle_sweep(o)
        cpu = {"value": tps, "unit": "tokens/s", "cores": thr, "per_core": tps / thr,
               "kind": "port",
               "sample": f"{passes} passes of the decode sweep T in {SWEEP} ({el:.1f} s), C "
                         f"restatement of ESRouter.mm/ESExperts.mm, OpenMP"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": "decode sweep T in {1,4,16,64}, Gemma-4-26B MoE block "
                                   "(H=2816,E=128,K=8,I=704), bf16, uniform routing",
                       "l2": "flushed before every timed forward (256 MiB read, untimed)",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
            "roofline": {"bound": "hbm",
                         "kernel": "expert stage: decode_fused_kernel, the whole block (T<=8); "
                                   "moe_gemm_kernel gate_up (T>8)",
                         "achieved": achieved, "peak": peaks["hbm"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm"], "peak_source": peaks["src"],
                         "traffic": args.traffic if args.traffic else GATEUP_SWEEP_TRAFFIC,
                         "traffic_source": ("--traffic argument" if args.traffic else
                                            "fixed figure from one ncu capture (dram__bytes_read"
                                            ".sum) of the expert-stage launches, "
                                            "profiles/decode_sweep_traffic.txt; not "
                                            "measured by this run"),
                         "scope": "sums over the 4 gate_up launches of one sweep step",
                         "algorithmic_bytes": gu_bytes},
            "sweep": sweep_detail,
            "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks.summary(),
        }
        if prefill:
            line["prefill"] = prefill
        if ep:
            line["ep"] = ep
        if quant:
            line["quant"] = quant
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def _timed(fn, dev, steps, warmup, world):
    """ms per call: CUDA events around each call, barrier + sync on both sides,
    mean over `steps`, max over ranks."""
    import torch
    import torch.distributed as dist
    stream = torch.cuda.current_stream(dev)
    for _ in range(warmup):
        fn()
    ms = 0.0
    for _ in range(steps):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        torch.cuda.synchronize()
        ms += a.elapsed_time(b) / steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def _parity(out, ref, ties, dev, world):
    """EP output vs the single-GPU block on the same tokens: max-abs over the
    tokens without a router tie (max over ranks), tie-exempt token count,
    cosine (min over ranks); ok = every non-tie token within 2e-2 and
    cosine >= 0.9999."""
    import torch
    import torch.distributed as dist
    err = (out.float() - ref.float()).abs().max(dim=1).values
    ma = float(err.masked_fill(ties, 0).max())
    cos = float(torch.nn.functional.cosine_similarity(out.float().flatten(),
                                                      ref.float().flatten(), 0))
    over = err > 2e-2
    n_over, n_over_tie = float(over.sum()), float((over & ties).sum())
    if world > 1:
        t = torch.tensor([ma, -cos], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ma, cos = float(t[0]), -float(t[1])
        t2 = torch.tensor([n_over, n_over_tie], device=dev)
        dist.all_reduce(t2)
        n_over, n_over_tie = float(t2[0]), float(t2[1])
    # tokens outside 2e-2 must all sit on a router tie (K-th vs K+1-th score
    # within one bf16 ulp), broken the other way by the relabelled expert ids
    return {"max_abs_non_tie": ma, "cos": cos, "tokens_over_tol": int(n_over),
            "tokens_over_tol_on_ties": int(n_over_tie),
            "ok": ma <= 2e-2 and cos >= 0.9999 and n_over == n_over_tie}


def run_ep(args, dev, world, rank, T=4096, steps=5, warmup=3):
    """expert parallelism over N GPUs, T tokens per GPU with
    Zipf(1.1) routing.  The N=1 point is the single-GPU block on the same
    tokens (every rank measures it on its own tokens, max over ranks), so
    efficiency = tput(N) / (N * tput(1)) comes from one run.  Forms: the C-ABI
    handle over NVLink peer memory (the EP value), the same over NCCL, and the
    Python host flow over NCCL.  Each form's output is checked against the
    single-GPU block on the rank's tokens."""
    import torch
    import torch.distributed as dist
    import apertura_b200 as A
    from apertura_b200.ep import ExpertParallelMoE, NativeExpertParallelMoE
    from apertura_b200.synthetic import block_inputs, expert_bank, router_tie_tokens
    d = block_inputs(T * world, seed=5, device=dev, routing="zipf", with_experts=False,
                     calib_tokens=4096)
    x = d["x"][rank * T:(rank + 1) * T].contiguous()
    ties = router_tie_tokens(x, d["proj"], d["scale"], K)
    gu, dn = expert_bank(E, H, I, 0, dev)
    cfg = A.ESModelConfig(moe_sparse=True, max_tokens=T, device=dev.index)
    loads = d["zipf"]["target"].tolist()
    # the N=1 point: the single-GPU block on this rank's tokens
    blk = A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], gu, dn)
    ref = blk.forward(x).clone()
    ms1 = _timed(lambda: blk.forward(x), dev, steps, warmup, world)
    del blk
    res = {"tokens_per_gpu": T, "routing": "zipf s=1.1",
           "single_gpu": {"ms_per_step": ms1, "tokens_per_s": T / (ms1 / 1e3)}}
    forms = {}
    if world > 1 or args.ep_one_rank:
        for transport in ("p2p", "nccl"):
            try:
                nep = NativeExpertParallelMoE(cfg, d["proj"], d["scale"], d["pes"], gu, dn,
                                              loads=loads, max_tokens_per_rank=T,
                                              transport=transport)
            except RuntimeError as e:
                forms[transport] = {"error": str(e)[:200]}
                continue
            out = nep(x)
            nep.sync()
            par = _parity(out, ref, ties, dev, world)
            ms = _timed(lambda: nep(x), dev, steps, warmup, world)
            nep.sync()
            recv, hot = nep.stats()
            rv = torch.tensor([float(recv)], device=dev)
            allr = [rv]
            if world > 1:
                allr = [torch.zeros_like(rv) for _ in range(world)]
                dist.all_gather(allr, rv)
            forms[transport] = {"ms_per_step": ms, "tokens_per_s": world * T / (ms / 1e3),
                                "efficiency": ms1 / ms, "parity_vs_single_gpu": par,
                                "recv_rows_per_rank": [int(v.item()) for v in allr],
                                "hot_rows": hot}
            nep.close()
    if world > 1:
        ep = ExpertParallelMoE(cfg, d["proj"], d["scale"], d["pes"], gu, dn, loads=loads,
                               max_tokens_per_rank=T)
        out = ep(x)
        par = _parity(out, ref, ties, dev, world)
        ms = _timed(lambda: ep(x), dev, steps, warmup, world)
        ep.timing = True
        ep(x)
        ep.timing = False
        names = list(ep.last_phase_ms)
        ph = torch.tensor([ep.last_phase_ms[n] for n in names], device=dev)
        dist.all_reduce(ph, op=dist.ReduceOp.MAX)
        hph = torch.tensor([ep.last_host_ms[n] for n in names], device=dev)
        dist.all_reduce(hph, op=dist.ReduceOp.MAX)
        forms["python_nccl"] = {
            "ms_per_step": ms, "tokens_per_s": world * T / (ms / 1e3),
            "efficiency": ms1 / ms, "parity_vs_single_gpu": par,
            "phases_ms_max_over_ranks": {n: float(v) for n, v in zip(names, ph.tolist())},
            "host_enqueue_ms_max_over_ranks": {n: float(v) for n, v in zip(names, hph.tolist())}}
        del ep
    res["forms"] = forms
    best = forms.get("p2p", {})
    if "ms_per_step" in best:
        res.update(tokens_per_s=best["tokens_per_s"], efficiency=best["efficiency"],
                   form="c-abi, NVLink peer memory")
    del gu, dn
    torch.cuda.empty_cache()
    return res


def run_quant(dev, peaks, flush, bits=4, Ts=(1, 4096), steps=5):
    """experts in MLX affine 4-bit (group 64), quantised on
    the device at load as ESExperts does with quantBits > 0; T=1 and T=4096."""
    import torch
    import apertura_b200 as A
    from apertura_b200.synthetic import block_inputs, expert_bank
    gu, dn = expert_bank(E, H, I, 0, dev)
    res = {}
    for T in Ts:
        d = block_inputs(T, seed=11, device=dev, routing="zipf" if T > 64 else "uniform",
                         with_experts=False)
        cfg = A.ESModelConfig(moe_sparse=True, quant_bits=bits, max_tokens=T, device=dev.index)
        blk = A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], gu, dn)
        out, tk = blk.forward(d["x"], return_routing=True)
        U = n_unique(tk.idx)
        stream = torch.cuda.current_stream(dev)

        def timed():
            ms = 0.0
            for _ in range(steps):
                flush.sum()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                blk.forward(d["x"])
                b.record(stream)
                b.synchronize()
                ms += a.elapsed_time(b) / steps
            return ms

        ms = timed()
        ms_expand = None
        if T > 64 and bits == 4:  # the other tensor-core form, for comparison
            blk.handle.set_q4_gemm(False)
            blk.forward(d["x"])
            ms_expand = timed()
            blk.handle.set_q4_gemm(True)
        qbytes = U * ((2 * I * H + H * I) * bits // 8 + (2 * I * H + H * I) // 64 * 4)
        res[str(T)] = {"ms": ms, "tokens_per_s": T / (ms / 1e3), "U": U,
                       "expert_bytes": qbytes,
                       "block_hbm_frac": qbytes / (ms / 1e3) / 1e9 / peaks["hbm"]}
        if T > 64:  # tensor-bound: the expansion of the touched experts is inside the timing
            blk.handle.set_timing(True)
            flush.sum()
            blk.forward(d["x"])
            st = blk.handle.stage_times()
            blk.handle.set_timing(False)
            flops = 2.0 * T * K * (2 * I * H + I * H)
            gemm_ms = st.get("gate_up", 0.0) + st.get("down", 0.0)
            res[str(T)].update(
                block_tflops=flops / (ms / 1e3) / 1e12,
                block_tc_frac=flops / (ms / 1e3) / 1e12 / peaks["tc"],
                expert_kernels_tflops=flops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else None,
                stages_ms=st,
                kernel=("moe_gemm_kernel QB=4: B tiles dequantised in shared memory"
                        if bits == 4 else
                        "dequant_active_kernel (touched experts, every call) + bf16 moe_gemm_kernel"),
                ms_expansion_path=ms_expand)
        del blk
    return {"bits": bits, "group": 64, **res}


def run_prefill(blk, dev, peaks, flush, T=8192, steps=3):
    """T=8192 with Zipf(1.1) routing; tensor-pipe roofline."""
    import torch
    from apertura_b200.synthetic import block_inputs
    d = block_inputs(T, seed=1, device=dev, routing="zipf", with_experts=False)
    # router weights of the Zipf config go into the same handle
    from apertura_b200.moe import ESRouter
    ESRouter(d["proj"], d["scale"], d["pes"], E, K, H, handle=blk.handle)
    out = blk.forward(d["x"])
    torch.cuda.synchronize()
    ms = 0.0
    stream = torch.cuda.current_stream(dev)
    for _ in range(steps):
        flush.sum()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        blk.forward(d["x"])
        b.record(stream)
        b.synchronize()
        ms += a.elapsed_time(b) / steps
    blk.handle.set_timing(True)
    blk.forward(d["x"])
    st = blk.handle.stage_times()
    blk.handle.set_timing(False)
    flops = 2.0 * T * K * (2 * I * H + I * H)
    gemm_ms = st.get("gate_up", 0.0) + st.get("down", 0.0)
    counts = blk.handle.last_counts()
    return {"T": T, "ms": ms, "tokens_per_s": T / (ms / 1e3),
            "block_tflops": flops / (ms / 1e3) / 1e12,
            "block_tc_frac": flops / (ms / 1e3) / 1e12 / peaks["tc"],
            "expert_kernels_tflops": flops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else None,
            "stages_ms": st, "max_expert_rows": int(counts.max()),
            "zipf_top_share": float(d["zipf"]["achieved"].max()), "routing": "zipf s=1.1"}


def run_prefill_only(args):
    """Prefill config alone at T tokens (the small case the ncu captures use);
    --bits 4/8 quantises the experts at load (MLX affine, group 64)."""
    import torch
    import apertura_b200 as A
    from apertura_b200 import build as B
    from apertura_b200.synthetic import expert_bank
    B.build()
    dev = torch.device("cuda", 0)
    gate_up, down = expert_bank(E, H, I, 0, dev)
    T = args.prefill_only
    ones_h = torch.ones(H, dtype=torch.bfloat16, device=dev)
    ones_e = torch.ones(E, dtype=torch.bfloat16, device=dev)
    proj = torch.zeros(E, H, dtype=torch.bfloat16, device=dev)
    cfg = A.ESModelConfig(moe_sparse=True, quant_bits=args.bits, max_tokens=T)
    blk = A.MoEBlock(cfg, proj, ones_h, ones_e, gate_up, down)
    flush = torch.ones(256 << 20, dtype=torch.uint8, device=dev)
    res = run_prefill(blk, dev, load_peaks(), flush, T=T, steps=args.steps)
    print(json.dumps({"prefill_only": res}), flush=True)
    return 0


def run_decode_only(args):
    """One decode forward at T tokens (bf16, or MLX affine --bits), repeated
    warmup + steps times with the L2 flushed before each: the case the ncu
    captures of decode_fused_kernel use (every forward is one launch)."""
    import torch
    import apertura_b200 as A
    from apertura_b200 import build as B
    from apertura_b200.synthetic import block_inputs, expert_bank
    B.build()
    dev = torch.device("cuda", 0)
    gu, dn = expert_bank(E, H, I, 0, dev)
    T = args.decode_only
    d = block_inputs(T, seed=11, device=dev, with_experts=False)
    cfg = A.ESModelConfig(moe_sparse=True, quant_bits=args.bits, max_tokens=T)
    blk = A.MoEBlock(cfg, d["proj"], d["scale"], d["pes"], gu, dn)
    flush = torch.ones(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    ms = 0.0
    for i in range(args.warmup + args.steps):
        flush.sum()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        blk.forward(d["x"])
        b.record(stream)
        b.synchronize()
        if i >= args.warmup:
            ms += a.elapsed_time(b) / args.steps
    blk.handle.sync()
    print(json.dumps({"decode_only": {"T": T, "bits": args.bits, "ms": ms,
                                      "launches": blk.handle.last_launches()}}), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-prefill", dest="prefill", action="store_false")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--no-quant", dest="quant", action="store_false",
                    help="skip the 4-bit expert measurement")
    ap.add_argument("--no-ep", dest="ep", action="store_false",
                    help="skip the expert-parallel measurement (and its 1-GPU point)")
    ap.add_argument("--ep-one-rank", action="store_true",
                    help="also run the EP handle with a single rank (N=1)")
    ap.add_argument("--gemv-max-tokens", type=int, default=None,
                    help="largest T that uses the GEMV expert kernels (default: library's)")
    ap.add_argument("--prefill-only", type=int, default=0, metavar="T",
                    help="only run the prefill config at T tokens (profiling case)")
    ap.add_argument("--decode-only", type=int, default=0, metavar="T",
                    help="only repeat one decode forward at T tokens (profiling case)")
    ap.add_argument("--bits", type=int, default=0, choices=[0, 4, 8],
                    help="with --decode-only / --prefill-only: MLX affine expert bits (0: bf16)")
    ap.add_argument("--traffic", type=float, default=None,
                    help="dram bytes per gate_up launch from an ncu capture (reported as is)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.prefill_only:
        return run_prefill_only(args)
    if args.decode_only:
        return run_decode_only(args)
    return run_reference(args) if args.impl == "reference" else run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
