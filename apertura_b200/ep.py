"""Expert parallelism for the MoE block: the cold experts sharded over the
GPUs, the hottest few replicated on every GPU, NCCL all-to-all token dispatch
and combine over NVLink.

The reference runs on one device and has no collective; this mode is new.
It reduces exactly to the single-GPU block: every (token, k) row is computed
by one holder of its expert, returned unweighted, and the home rank applies
the reference's combine (bf16(w * out) summed in k order, ESExperts.mm:58-59).

Placement.  Experts are relabelled once at load.  With R replicated ("hot")
experts and C = E - R cold ones, every rank holds the hot ids [0, R) and rank r
owns the cold ids [R + r*C/N, R + (r+1)*C/N).  The hot set is the R experts with the
largest expected load, the cold ones are spread by a longest-processing-time
assignment of their loads, so Zipf-skewed routing neither piles hot experts on
one rank nor ships their rows at all: under capped Zipf(1.1) the top 8 of 128
experts take half of all (token, k) pairs and the top 24 about 70 %, which stay
on their home GPU.  (Measured at 2 GPUs, 4096 Zipf tokens each: 1.40 ms per step
with pure sharding, 1.09 ms with 8 replicated experts, 0.95 ms with 24; every
replicated expert costs 11.9 MB per GPU.)  The
router's proj rows and per_expert_scale are permuted the same way, which leaves
the selected experts and their weights unchanged (only exact probability ties
could order differently).  With that numbering the dispatch's expert-sorted
rows are [hot rows | cold rows grouped by destination rank]: the hot part starts
at row 0 and its group sizes are on the device, so its compute is queued right
after the dispatch, before the host learns any split; the second part is the
send buffer.

Per step (one process per GPU, torch.distributed over NCCL for the plumbing):
  1. apt_moe_ep_dispatch: route, top-K, dispatch, gather rows
  2. all_to_all of the per-expert cold counts
  3. hot rows: apt_moe_experts_grouped on a side stream, straight into the
     return buffer, overlapping 4-6; then one host sync for the splits
  4. all_to_all of the cold rows to their owners
  5. apt_moe_experts_grouped on the received rows, grouped by (source rank,
     local expert), in place -> unweighted expert rows
  6. all_to_all of the cold result rows back (reverse splits)
  7. apt_moe_ep_combine: weighted k-order combine on the home rank
The compute steps go through a backend object built by a factory; the default
is the C ABI (libapt_moe.so).  Tests substitute a CPU factory to exercise the
exchange logic on gloo ranks.
"""
from __future__ import annotations

import ctypes
import time
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from ._lib import lib
from .moe import ESModelConfig, Handle, _ptr, _stream


def lpt_placement(loads: Sequence[float], n_ranks: int) -> List[int]:
    """Longest-processing-time placement with E/N experts per rank.

    Returns perm with perm[new_id] = original expert id, rank r owning new ids
    [r*E/N, (r+1)*E/N).  Experts are taken by descending load and given to the
    least-loaded rank that still has room; ties break by lower id / rank."""
    E = len(loads)
    if E % n_ranks:
        raise ValueError(f"{E} experts do not split over {n_ranks} ranks")
    cap = E // n_ranks
    order = sorted(range(E), key=lambda e: (-float(loads[e]), e))
    rank_load = [0.0] * n_ranks
    members: List[List[int]] = [[] for _ in range(n_ranks)]
    for e in order:
        r = min((r for r in range(n_ranks) if len(members[r]) < cap),
                key=lambda r: (rank_load[r], r))
        members[r].append(e)
        rank_load[r] += float(loads[e])
    perm: List[int] = []
    for r in range(n_ranks):
        perm.extend(sorted(members[r]))
    return perm


def hot_cold_placement(loads: Sequence[float], n_ranks: int, n_hot: int) -> List[int]:
    """perm[new_id] = original id: the n_hot hottest experts (replicated),
    followed by an LPT placement of the others over the ranks."""
    E = len(loads)
    if n_hot < 0 or n_hot >= E or (E - n_hot) % n_ranks:
        raise ValueError(f"{E} experts minus {n_hot} replicated do not split over {n_ranks} ranks")
    order = sorted(range(E), key=lambda e: (-float(loads[e]), e))
    hot = sorted(order[:n_hot])
    cold = sorted(order[n_hot:])
    sub = lpt_placement([loads[e] for e in cold], n_ranks)
    return hot + [cold[i] for i in sub]


class CudaBackend:
    """The product path: every compute step is a libapt_moe.so call.  Holds a
    router handle (all E experts) and one handle per local expert bank (the
    rank's cold experts; the replicated hot experts), so the hot compute can run
    on its own stream beside the cold exchange without sharing a workspace."""

    def __init__(self, cfg: ESModelConfig, proj, scale, pes, local_gate_up, local_down,
                 max_recv_rows: int, n_hot: int = 0, hot_sm_limit: int = 0):
        E_loc = local_gate_up.shape[0]
        self.cfg = cfg
        self.n_hot = n_hot
        self.router = Handle(cfg)
        self.router.check(lib().apt_moe_load_router(self.router.h, _ptr(proj), _ptr(scale),
                                                     _ptr(pes), 1))

        def bank(gu, dn, rows):
            c = ESModelConfig(hidden_size=cfg.hidden_size, num_experts=gu.shape[0],
                              top_k_experts=1, moe_intermediate_size=cfg.moe_intermediate_size,
                              moe_sparse=True, max_tokens=max(1, rows), device=cfg.device)
            h = Handle(c)
            h.check(lib().apt_moe_load_experts_bf16(h.h, _ptr(gu.contiguous()),
                                                    _ptr(dn.contiguous()), 1))
            return h

        n_cold = E_loc - n_hot
        self.cold = bank(local_gate_up[:n_cold], local_down[:n_cold], max_recv_rows) \
            if n_cold > 0 else None
        self.hot = bank(local_gate_up[n_cold:], local_down[n_cold:],
                        cfg.max_tokens * cfg.top_k_experts) if n_hot > 0 else None
        if self.hot is not None and hot_sm_limit > 0:
            self.hot.set_sm_limit(hot_sm_limit)  # SMs left free for the exchange
        self.device = torch.device("cuda", cfg.device)

    def dispatch(self, x):
        T, H = x.shape
        K, E = self.cfg.top_k_experts, self.cfg.num_experts
        idx = torch.empty(T, K, dtype=torch.int32, device=x.device)
        w = torch.empty(T, K, dtype=torch.bfloat16, device=x.device)
        rows = torch.empty(T * K, H, dtype=torch.bfloat16, device=x.device)
        counts = torch.empty(E, dtype=torch.int32, device=x.device)
        self.router.check(lib().apt_moe_ep_dispatch(self.router.h, _ptr(x), T, _ptr(idx), _ptr(w),
                                                    _ptr(rows), _ptr(counts), _stream(x.device)))
        return idx, w, rows, counts

    def experts(self, rows, group_counts, group_expert, out=None, hot=False):
        """Rows grouped as in group_counts, group g on bank expert group_expert[g]
        (the hot bank when hot=True); unweighted outputs in row order."""
        R, H = rows.shape
        if out is None:
            out = torch.empty_like(rows)
        if R == 0:
            return out
        h = self.hot if hot else self.cold
        G = group_counts.numel()
        h.check(lib().apt_moe_experts_grouped(
            h.h, _ptr(rows), R, _ptr(group_counts), _ptr(group_expert), G, _ptr(out),
            _stream(rows.device)))
        return out

    def combine(self, back, idx, w):
        T, K = idx.shape
        out = torch.empty(T, back.shape[1], dtype=torch.bfloat16, device=back.device)
        self.router.check(lib().apt_moe_ep_combine(self.router.h, _ptr(back), _ptr(idx), _ptr(w),
                                                   T, _ptr(out), _stream(back.device)))
        return out


class ExpertParallelMoE:
    """The MoE block with experts sharded over the ranks of `group`.

    Parameters are the full router weights (replicated, 0.72 MB) and the full
    expert banks (on the local device or the host); `loads` (expected tokens per
    expert) drives the placement (uniform if None); `replicate_hot` experts
    with the largest loads are held by every rank (0: pure sharding); the
    replicated experts' kernels leave `exchange_sms` SMs free for NCCL."""

    def __init__(self, cfg: ESModelConfig, proj, scale, pes, gate_up, down,
                 group=None, loads: Optional[Sequence[float]] = None,
                 max_tokens_per_rank: int = 4096, capacity_factor: float = 4.0,
                 backend=None, replicate_hot: int = 24, exchange_sms: int = 24):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        E, K = cfg.num_experts, cfg.top_k_experts
        R = replicate_hot if self.world > 1 else 0
        if R and (R >= E or (E - R) % self.world):
            R = 0  # the cold part must split evenly; fall back to pure sharding
        if (E - R) % self.world:
            raise ValueError(f"{E} experts do not split over {self.world} ranks")
        self.n_hot, self.n_cold = R, E - R
        self.C_loc = self.n_cold // self.world
        self.cfg = cfg
        loads = list(loads) if loads is not None else [1.0] * E
        self.perm = hot_cold_placement(loads, self.world, R)
        pidx = torch.tensor(self.perm, dtype=torch.long, device=proj.device)
        proj_r = proj.index_select(0, pidx).contiguous()
        pes_r = pes.index_select(0, pidx).contiguous()
        lo, hi = R + self.rank * self.C_loc, R + (self.rank + 1) * self.C_loc
        mine = torch.cat([pidx[lo:hi], pidx[:R]])  # local bank: [owned cold | hot]
        gu_loc = gate_up.index_select(0, mine.to(gate_up.device)).contiguous()
        dn_loc = down.index_select(0, mine.to(down.device)).contiguous()
        dev = proj.device
        if gu_loc.device != dev:
            gu_loc, dn_loc = gu_loc.to(dev), dn_loc.to(dev)
        self.max_recv = int(capacity_factor * max_tokens_per_rank * K)
        cfg_r = ESModelConfig(**{**cfg.__dict__, "moe_sparse": True,
                                 "max_tokens": max_tokens_per_rank})
        # cold group g = (source rank g // C_loc, local expert g % C_loc)
        self.cold_expert = torch.arange(self.C_loc, dtype=torch.int32).repeat(self.world).to(dev)
        self.hot_expert = torch.arange(R, dtype=torch.int32).to(dev)
        if backend is None:
            sms = torch.cuda.get_device_properties(dev).multi_processor_count
            self.backend = CudaBackend(cfg_r, proj_r, scale, pes_r, gu_loc, dn_loc, self.max_recv,
                                       R, max(1, sms - exchange_sms) if exchange_sms else 0)
        else:  # a factory with CudaBackend's signature (tests: a CPU stand-in)
            self.backend = backend(cfg_r, proj_r, scale, pes_r, gu_loc, dn_loc, self.max_recv, R)
        self.last_recv_rows = 0
        self.last_hot_rows = 0
        self._side = torch.cuda.Stream(dev) if dev.type == "cuda" and R else None
        # per-phase CUDA-event timing of the last forward (set timing = True)
        self.timing = False
        self.last_phase_ms = {}
        self.last_host_ms = {}  # host time between the same marks (enqueue cost)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        N, C_loc = self.world, self.C_loc
        T, H = x.shape
        marks: List[Tuple[str, torch.cuda.Event]] = []

        host: List[float] = []

        def mark(name):
            if self.timing and x.is_cuda:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append((name, ev))
                host.append(time.perf_counter())

        mark("start")
        idx, w, rows, counts = self.backend.dispatch(x)
        mark("dispatch")
        Rh = self.n_hot
        back = torch.empty_like(rows)
        # 1. per-(destination rank, local cold expert) counts, exchanged first:
        #    a small NCCL op that must not queue behind the replicated experts
        cold_counts = counts[Rh:].contiguous()
        recv_counts = torch.empty_like(cold_counts)
        dist.all_to_all_single(recv_counts, cold_counts, group=self.group)
        # 2. replicated experts: their rows open the sorted buffer and their group
        #    sizes are on the device, so this is queued before the host sync and
        #    runs beside the exchange below
        hot_side = Rh > 0 and self._side is not None
        if Rh:
            hot_counts = counts[:Rh].contiguous()
            if hot_side:
                self._side.wait_stream(torch.cuda.current_stream(x.device))
                with torch.cuda.stream(self._side):
                    self.backend.experts(rows, hot_counts, self.hot_expert, out=back, hot=True)
                rows.record_stream(self._side)
                back.record_stream(self._side)
                hot_counts.record_stream(self._side)
            else:
                self.backend.experts(rows, hot_counts, self.hot_expert, out=back, hot=True)
        both = torch.cat([cold_counts.view(N, C_loc).sum(1), recv_counts.view(N, C_loc).sum(1),
                          counts[:Rh].sum().view(1)]).cpu()  # one host sync for the splits
        mark("counts")
        send_splits = both[:N].tolist()
        recv_splits = both[N:2 * N].tolist()
        n_hot_rows = int(both[2 * N])
        S = int(sum(send_splits))
        R = int(sum(recv_splits))
        if R > self.max_recv:
            raise RuntimeError(f"rank {self.rank} receives {R} rows > capacity {self.max_recv}; "
                               f"raise capacity_factor")
        lo, hi = n_hot_rows, n_hot_rows + S
        # 3. cold token rows to their owners
        recv_rows = torch.empty(R, H, dtype=rows.dtype, device=rows.device)
        dist.all_to_all_single(recv_rows, rows[lo:hi], recv_splits, send_splits, group=self.group)
        mark("rows_out")
        # 4. owned cold experts, unweighted: rows from each source arrive
        #    grouped by local expert, so (source, expert) groups run in place
        out_rows = self.backend.experts(recv_rows, recv_counts, self.cold_expert)
        mark("experts")
        # 5. back to the home ranks, in the send order
        dist.all_to_all_single(back[lo:hi], out_rows, send_splits, recv_splits, group=self.group)
        mark("rows_back")
        if hot_side:
            torch.cuda.current_stream(x.device).wait_stream(self._side)
        self.last_recv_rows = R
        self.last_hot_rows = n_hot_rows
        # 6. weighted combine in k order
        out = self.backend.combine(back, idx, w)
        mark("combine")
        if marks:
            marks[-1][1].synchronize()
            self.last_phase_ms = {b[0]: a[1].elapsed_time(b[1]) for a, b in zip(marks, marks[1:])}
            self.last_host_ms = {b[0]: 1e3 * (hb - ha)
                                 for a, b, ha, hb in zip(marks, marks[1:], host, host[1:])}
        return out

    __call__ = forward


class NativeExpertParallelMoE:
    """The same expert-parallel block with the whole step inside the library
    (apt_moe_create_ep: C++ host flow, NCCL resolved by the library): what a
    C or C++ host would call.  Construction is collective over `group` (its
    NCCL communicator is made from an id that rank 0 creates and the group
    broadcasts).  Parameters as ExpertParallelMoE."""

    TRANSPORTS = {"nccl": 0, "p2p": 1}

    def __init__(self, cfg: ESModelConfig, proj, scale, pes, gate_up, down, group=None,
                 loads: Optional[Sequence[float]] = None, max_tokens_per_rank: int = 4096,
                 replicate_hot: int = 24, transport: Optional[str] = None):
        import numpy as np
        from ._lib import check as _check
        single = not (dist.is_available() and dist.is_initialized())
        self.rank = 0 if single else dist.get_rank(group)
        self.world = 1 if single else dist.get_world_size(group)
        self.cfg = cfg
        idbuf = ctypes.create_string_buffer(128)
        if self.rank == 0:
            _check(lib().apt_moe_nccl_unique_id(idbuf))
        if self.world > 1:
            obj = [idbuf.raw if self.rank == 0 else None]
            dist.broadcast_object_list(obj, src=0, group=group)
            idbuf = ctypes.create_string_buffer(obj[0], 128)
        self._loads = None if loads is None else np.asarray(loads, dtype=np.float32)
        c = ESModelConfig(**{**cfg.__dict__, "moe_sparse": True,
                             "max_tokens": max_tokens_per_rank}).to_c()
        ep = ctypes.c_void_p()
        lp = None if self._loads is None else ctypes.c_void_p(self._loads.ctypes.data)
        _check(lib().apt_moe_create_ep(ctypes.byref(c), idbuf, self.rank, self.world, lp,
                                       int(replicate_hot), ctypes.byref(ep)))
        self.ep = ep
        self._check(lib().apt_moe_ep_load_router(ep, _ptr(proj), _ptr(scale), _ptr(pes), 1))
        self._check(lib().apt_moe_ep_load_experts_bf16(ep, _ptr(gate_up), _ptr(down), 1))
        if transport is not None:
            self._check(lib().apt_moe_ep_set_transport(ep, self.TRANSPORTS[transport]))

    @property
    def transport(self) -> str:
        t = ctypes.c_int()
        self._check(lib().apt_moe_ep_get_transport(self.ep, ctypes.byref(t)))
        return {v: k for k, v in self.TRANSPORTS.items()}[t.value]

    def sync(self):
        """Wait for the device; raises if a bounded wait of the exchange gave up."""
        self._check(lib().apt_moe_ep_sync(self.ep))

    def _check(self, status):
        if status != 0:
            msg = lib().apt_moe_ep_last_error(self.ep)
            raise RuntimeError(f"apt_moe_ep: status {status}: {msg.decode() if msg else ''}")

    def stats(self):
        r, h = ctypes.c_int(), ctypes.c_int()
        self._check(lib().apt_moe_ep_stats(self.ep, ctypes.byref(r), ctypes.byref(h)))
        return r.value, h.value

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        out = torch.empty_like(x)
        self._check(lib().apt_moe_ep_forward(self.ep, _ptr(x), T, _ptr(out), _stream(x.device)))
        return out

    __call__ = forward

    def close(self):
        if getattr(self, "ep", None):
            lib().apt_moe_ep_destroy(self.ep)
            self.ep = None

    # No __del__: destroying the handle is collective (its buffers stay mapped
    # by the other ranks until all of them destroy), so it happens only in an
    # explicit close() that every rank calls.

