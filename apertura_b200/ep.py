"""Expert parallelism for the MoE block: 128/N experts per GPU, NCCL
all-to-all token dispatch and combine over NVLink.

The reference runs on one device and has no collective; this mode is new.
It reduces exactly to the single-GPU block: every (token, k) row is computed
by the rank owning its expert, returned unweighted, and the home rank applies
the reference's combine (bf16(w * out) summed in k order, ESExperts.mm:58-59).

Placement.  Experts are relabelled once at load so that rank r owns the
contiguous id range [r*E/N, (r+1)*E/N); the permutation comes from a
longest-processing-time assignment of measured (or expected) expert loads, so
Zipf-skewed routing does not pile the hot experts on one rank.  The router's
proj rows and per_expert_scale are permuted the same way, which leaves the
selected experts and their weights unchanged (only exact probability ties
could order differently).  With that numbering the dispatch's expert-sorted
rows are already grouped by destination rank: they are the send buffer.

Per step (one process per GPU, torch.distributed over NCCL for the plumbing):
  1. apt_moe_ep_dispatch: route, top-K, dispatch, gather rows (send buffer)
  2. all_to_all of the per-expert counts (E ints), then of the rows
  3. apt_moe_experts_grouped on the local experts: the received rows, grouped
     by (source rank, local expert), run in place -> unweighted expert rows
  4. all_to_all of the result rows back (reverse splits)
  5. apt_moe_ep_combine: weighted k-order combine on the home rank
The compute steps go through a backend object built by a factory; the
default is the C ABI (libapt_moe.so).  Tests substitute a CPU factory to
exercise the exchange logic on gloo ranks.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

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


class CudaBackend:
    """The product path: every compute step is a libapt_moe.so call."""

    def __init__(self, cfg: ESModelConfig, proj, scale, pes, local_gate_up, local_down,
                 max_recv_rows: int):
        E_loc = local_gate_up.shape[0]
        self.cfg = cfg
        self.router = Handle(cfg)
        self.router.check(lib().apt_moe_load_router(self.router.h, _ptr(proj), _ptr(scale),
                                                     _ptr(pes), 1))
        lcfg = ESModelConfig(hidden_size=cfg.hidden_size, num_experts=E_loc, top_k_experts=1,
                             moe_intermediate_size=cfg.moe_intermediate_size, moe_sparse=True,
                             max_tokens=max(1, max_recv_rows), device=cfg.device)
        self.local = Handle(lcfg)
        self.local.check(lib().apt_moe_load_experts_bf16(self.local.h, _ptr(local_gate_up),
                                                         _ptr(local_down), 1))
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

    def experts(self, rows, group_counts, group_expert):
        """Rows grouped as (source rank, local expert): apt_moe_experts_grouped
        consumes them in place."""
        R, H = rows.shape
        out = torch.empty_like(rows)
        if R == 0:
            return out
        G = group_counts.numel()
        self.local.check(lib().apt_moe_experts_grouped(
            self.local.h, _ptr(rows), R, _ptr(group_counts), _ptr(group_expert), G, _ptr(out),
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
    expert banks on the local device or only this rank's slice; `loads`
    (expected tokens per expert) drives the placement (uniform if None)."""

    def __init__(self, cfg: ESModelConfig, proj, scale, pes, gate_up, down,
                 group=None, loads: Optional[Sequence[float]] = None,
                 max_tokens_per_rank: int = 4096, capacity_factor: float = 4.0,
                 backend=None, banks_are_local: bool = False):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        E, K = cfg.num_experts, cfg.top_k_experts
        if E % self.world:
            raise ValueError(f"{E} experts do not split over {self.world} ranks")
        self.E_loc = E // self.world
        self.cfg = cfg
        self.perm = lpt_placement(loads if loads is not None else [1.0] * E, self.world)
        pidx = torch.tensor(self.perm, dtype=torch.long, device=proj.device)
        proj_r = proj.index_select(0, pidx).contiguous()
        pes_r = pes.index_select(0, pidx).contiguous()
        lo, hi = self.rank * self.E_loc, (self.rank + 1) * self.E_loc
        if banks_are_local:
            gu_loc, dn_loc = gate_up, down
        else:
            mine = pidx[lo:hi].to(gate_up.device)
            gu_loc = gate_up.index_select(0, mine).contiguous()
            dn_loc = down.index_select(0, mine).contiguous()
        self.max_recv = int(capacity_factor * max_tokens_per_rank * K)
        cfg_r = ESModelConfig(**{**cfg.__dict__, "moe_sparse": True,
                                 "max_tokens": max_tokens_per_rank})
        # group g = (source rank g // E_loc, local expert g % E_loc)
        self.group_expert = torch.arange(self.E_loc, dtype=torch.int32).repeat(self.world).to(
            proj.device)
        make = backend or CudaBackend  # a factory with CudaBackend's signature
        self.backend = make(cfg_r, proj_r, scale, pes_r, gu_loc, dn_loc, self.max_recv)
        self.last_recv_rows = 0

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        N, E_loc = self.world, self.E_loc
        T, H = x.shape
        idx, w, rows, counts = self.backend.dispatch(x)
        # 1. per-(destination rank, local expert) counts, exchanged
        recv_counts = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        send_splits = counts.view(N, E_loc).sum(1)
        both = torch.cat([send_splits, recv_counts]).cpu()  # one host sync for the splits
        send_splits = both[:N].tolist()
        recv_per = both[N:].view(N, E_loc)
        recv_splits = recv_per.sum(1).tolist()
        R = int(sum(recv_splits))
        if R > self.max_recv:
            raise RuntimeError(f"rank {self.rank} receives {R} rows > capacity {self.max_recv}; "
                               f"raise capacity_factor")
        # 2. token rows to the expert owners
        recv_rows = torch.empty(R, H, dtype=rows.dtype, device=rows.device)
        dist.all_to_all_single(recv_rows, rows, recv_splits, send_splits, group=self.group)
        # 3. local experts, unweighted: rows from each source arrive grouped by
        #    local expert, so (source, expert) groups run in place
        out_rows = self.backend.experts(recv_rows, recv_counts, self.group_expert)
        # 4. back to the home ranks, in the send order
        back = torch.empty_like(rows)
        dist.all_to_all_single(back, out_rows, send_splits, recv_splits, group=self.group)
        self.last_recv_rows = R
        # 5. weighted combine in k order
        return self.backend.combine(back, idx, w)

    __call__ = forward
