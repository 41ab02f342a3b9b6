"""Expert-parallel exchange logic on CPU ranks (gloo, world_size 2).

The compute steps are stood in for by the CPU oracle (a test-only backend),
so these tests check what the EP layer itself owns: LPT placement, relabelled
routing, count exchange, split sizes, the row all-to-all both ways, local
expert ids, and the k-order combine.  The result must equal the oracle's
single-device block on every rank's tokens.  The CUDA backend is exercised by
the GPU test of the same flow (test_gpu_ep.py)."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from apertura_b200.ep import hot_cold_placement, lpt_placement

H, E, K, I = 64, 16, 4, 64


def test_lpt_placement_balances():
    loads = [100.0 / (r + 1) ** 1.1 for r in range(16)]
    perm = lpt_placement(loads, 4)
    assert sorted(perm) == list(range(16))
    per_rank = [sum(loads[e] for e in perm[r * 4:(r + 1) * 4]) for r in range(4)]
    # LPT bound: no rank exceeds the mean by more than the largest single load,
    # and a contiguous split of the sorted ids would be far worse
    assert max(per_rank) <= sum(loads) / 4 + max(loads)
    naive = [sum(loads[r * 4:(r + 1) * 4]) for r in range(4)]
    assert max(per_rank) < 0.75 * max(naive)
    # every rank owns exactly E/N experts, listed ascending within the rank
    for r in range(4):
        block = perm[r * 4:(r + 1) * 4]
        assert block == sorted(block)


def test_lpt_rejects_uneven():
    with pytest.raises(ValueError):
        lpt_placement([1.0] * 10, 4)


def test_hot_cold_placement():
    loads = [1.0 / (e + 1) for e in range(16)]
    perm = hot_cold_placement(loads, 2, 4)
    assert sorted(perm) == list(range(16))
    assert sorted(perm[:4]) == [0, 1, 2, 3]  # the 4 heaviest are replicated
    assert len(hot_cold_placement(loads, 3, 4)) == 16  # 12 cold over 3 ranks
    with pytest.raises(ValueError):
        hot_cold_placement(loads, 3, 3)       # 13 cold experts do not split over 3
    with pytest.raises(ValueError):
        hot_cold_placement(loads, 2, 5)       # 11 cold experts do not split over 2


def test_native_placement_matches_python():
    """apt_moe_ep_placement (the C-ABI EP's placement) = hot_cold_placement."""
    import ctypes
    from apertura_b200._lib import lib
    rng = np.random.default_rng(3)
    for E, N, R in ((128, 2, 24), (128, 8, 24), (128, 4, 0), (16, 2, 4)):
        loads = rng.pareto(1.1, E).astype(np.float32)
        loads[5] = loads[6]  # a tie
        out = np.zeros(E, np.int32)
        st = lib().apt_moe_ep_placement(ctypes.c_void_p(loads.ctypes.data), E, N, R,
                                        ctypes.c_void_p(out.ctypes.data))
        assert st == 0
        assert out.tolist() == hot_cold_placement([float(v) for v in loads], N, R)


class OracleBackend:
    """CPU stand-in for CudaBackend, built on the oracle."""

    def __init__(self, cfg, proj, scale, pes, gu_loc, dn_loc, max_recv, n_hot=0):
        from oracle import oracle as O
        self.hot_base = gu_loc.shape[0] - n_hot  # hot bank follows the cold one
        self.O = O
        b = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)
        self.proj, self.scale, self.pes = b(proj), b(scale), b(pes)
        self.gu, self.dn = b(gu_loc), b(dn_loc)
        self.K, self.E = cfg.top_k_experts, cfg.num_experts

    def dispatch(self, x):
        xb = x.contiguous().view(torch.int16).numpy().view(np.uint16)
        idx, w = self.O.route_topk(xb, self.proj, self.scale, self.pes, self.K)
        flat = idx.ravel()
        order = np.argsort(flat, kind="stable")       # expert order, stable in pair order
        self.inv = np.empty_like(order)
        self.inv[order] = np.arange(order.size)
        rows = xb[order // self.K]
        counts = np.bincount(flat, minlength=self.E).astype(np.int32)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
        return (torch.from_numpy(idx), t(w), t(rows), torch.from_numpy(counts))

    def experts(self, rows, group_counts, group_expert, out=None, hot=False):
        R = int(group_counts.sum())  # rows past the groups are left untouched
        if R == 0:
            return rows.clone() if out is None else out
        rows = rows[:R]
        rb = rows.contiguous().view(torch.int16).numpy().view(np.uint16)
        ge = group_expert.numpy() + (self.hot_base if hot else 0)
        ids = np.repeat(ge, group_counts.numpy()).astype(np.int32).reshape(R, 1)
        ones = self.O.f32_to_bf16(np.ones((R, 1), np.float32))
        res = torch.from_numpy(self.O.experts_sparse(rb, self.gu, self.dn, ids, ones).view(np.int16))
        res = res.view(torch.bfloat16)
        if out is None:
            return res
        out[:R].copy_(res)
        return out

    def combine(self, back, idx, w):
        O = self.O
        bb = O.bf16_to_f32(back.contiguous().view(torch.int16).numpy().view(np.uint16))
        wf = O.bf16_to_f32(w.contiguous().view(torch.int16).numpy().view(np.uint16))
        T = idx.shape[0]
        acc = np.zeros((T, bb.shape[1]), np.float32)
        for k in range(self.K):
            rows = bb[self.inv[np.arange(T) * self.K + k]]
            prod = O.bf16_to_f32(O.f32_to_bf16(wf[:, k:k + 1] * rows))
            acc = (acc + prod).astype(np.float32)
        return torch.from_numpy(O.f32_to_bf16(acc).view(np.int16)).view(torch.bfloat16)


def _worker(rank, world, port, result_q, n_hot):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O
        from apertura_b200.moe import ESModelConfig
        from apertura_b200.ep import ExpertParallelMoE
        g = torch.Generator().manual_seed(0)
        bf = lambda t: t.to(torch.bfloat16)
        proj = bf(torch.randn(E, H, generator=g) / H ** 0.5)
        scale = bf(1 + 0.1 * torch.randn(H, generator=g))
        pes = bf(1 + 0.1 * torch.randn(E, generator=g))
        gu = bf(0.02 * torch.randn(E, 2 * I, H, generator=g))
        dn = bf(0.02 * torch.randn(E, H, I, generator=g))
        gx = torch.Generator().manual_seed(100 + rank)
        T = 10 + 3 * rank  # ragged token counts per rank
        x = bf(torch.randn(T, H, generator=gx))
        loads = [1.0 / (e + 1) for e in range(E)]
        cfg = ESModelConfig(hidden_size=H, num_experts=E, top_k_experts=K, moe_intermediate_size=I,
                            moe_sparse=True, max_tokens=64, device=0)
        ep = ExpertParallelMoE(cfg, proj, scale, pes, gu, dn, loads=loads, max_tokens_per_rank=64,
                               backend=OracleBackend, replicate_hot=n_hot)
        assert ep.n_hot == n_hot
        out = ep(x)
        b = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)
        idx, w = O.route_topk(b(x), b(proj), b(scale), b(pes), K)
        ref = O.experts_sparse(b(x), b(gu), b(dn), idx, w)
        got = O.bf16_to_f32(b(out))
        refv = O.bf16_to_f32(ref)
        result_q.put((rank, float(np.abs(got - refv).max()), float(np.abs(refv).max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_hot", [0, 4])
def test_ep_exchange_matches_single_device(n_hot):
    """Pure sharding, and 4 of 16 experts replicated on both ranks (their rows
    computed at home, the rest exchanged)."""
    from oracle import oracle as O
    O.build()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() + 7 * n_hot) % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, n_hot)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=5) for _ in range(2))
    for rank, ma, peak in res:
        # same arithmetic, same order: identical up to relabelled tie-breaking
        assert ma <= 2.0 ** -7 * peak, (rank, ma, peak)


def _failing_worker(rank, world, port, result_q):
    """Rank 1 leaves between steps (no exchange in flight); rank 0's next
    exchange must end with an error from the process-group timeout, not hang."""
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=8))
    from apertura_b200.moe import ESModelConfig
    from apertura_b200.ep import ExpertParallelMoE
    g = torch.Generator().manual_seed(0)
    bf = lambda t: t.to(torch.bfloat16)
    proj = bf(torch.randn(E, H, generator=g) / H ** 0.5)
    scale, pes = bf(torch.ones(H)), bf(torch.ones(E))
    gu = bf(0.02 * torch.randn(E, 2 * I, H, generator=g))
    dn = bf(0.02 * torch.randn(E, H, I, generator=g))
    cfg = ESModelConfig(hidden_size=H, num_experts=E, top_k_experts=K, moe_intermediate_size=I,
                        moe_sparse=True, max_tokens=64, device=0)
    ep = ExpertParallelMoE(cfg, proj, scale, pes, gu, dn, max_tokens_per_rank=64,
                           backend=OracleBackend, replicate_hot=0)
    x = bf(torch.randn(8, H, generator=g))
    ep(x)  # one good step on both ranks
    if rank == 1:
        result_q.put((rank, "left"))
        result_q.close()
        result_q.join_thread()
        os._exit(0)  # leaves without a goodbye, between steps
    import time
    t0 = time.time()
    try:
        ep(x)
        result_q.put((rank, "no error"))
    except Exception as e:  # gloo reports the lost peer or the timeout
        result_q.put((rank, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))
    result_q.close()
    result_q.join_thread()
    os._exit(0)


def test_ep_lost_rank_is_detected():
    from oracle import oracle as O
    O.build()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() + 311) % 1000
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p.is_alive() for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert not any(alive), "a rank hung instead of failing"
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res[1] == "left"
    assert res[0].startswith("error after"), res[0]
