"""Expert-parallel MoE forward over the GPUs of one node.

Tokens are sharded (T/G per rank: router, top-k and sort run locally), experts are
sharded (E/G per rank, expert e lives on rank e // (E/G)).  The one exchange step each
way is an all_to_all_single: per-expert counts first, then the expert-sorted activation
rows (dispatch), and after the expert GEMMs the output rows back (combine).

Because the local sort is expert-major and experts are dealt out in contiguous runs, the
compactly sorted rows are already grouped by destination rank: the gather kernel writes
the send buffer, the collective moves it, no separate pack pass exists.  Received rows
arrive grouped by source rank; one row gather regroups them by expert for the grouped
GEMM, and its inverse puts the outputs back in arrival order for the return trip.

The arithmetic is injected as an `ops` object so that the same host logic (split sizes,
regroup plan, collectives) runs on GPUs over NCCL with the C-ABI kernels and, in the CPU
tests, over gloo with stand-in arithmetic.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist


def experts_per_rank(experts: int, world: int) -> int:
    if experts % world != 0:
        raise ValueError(f"{experts} experts do not split over {world} ranks")
    return experts // world


def expert_owner(expert: int, experts: int, world: int) -> int:
    return expert // experts_per_rank(experts, world)


def send_splits(expert_counts: np.ndarray, world: int) -> np.ndarray:
    """Rows this rank sends to each destination: sums of its per-expert counts."""
    counts = np.asarray(expert_counts, dtype=np.int64)
    return counts.reshape(world, -1).sum(axis=1)


@dataclass
class RegroupPlan:
    """Received rows are src-major (all rows from rank 0, then rank 1, ...; per source in
    local-expert order).  The grouped GEMM wants them expert-major."""

    gather: np.ndarray          # [R] grouped position -> arrival position
    scatter: np.ndarray         # [R] arrival position -> grouped position (inverse)
    expert_offsets: np.ndarray  # [E_l + 1] first grouped row of each local expert
    expert_counts: np.ndarray   # [E_l]
    recv_splits: np.ndarray     # [G] rows received from each source


def regroup_plan(recv_counts: np.ndarray) -> RegroupPlan:
    """recv_counts[src, e] = rows that rank `src` sends for this rank's local expert e."""
    rc = np.asarray(recv_counts, dtype=np.int64)
    world, e_local = rc.shape
    recv_splits = rc.sum(axis=1)
    total = int(recv_splits.sum())
    # arrival order: (src, e) segments
    seg_arrival_start = np.concatenate([[0], np.cumsum(rc.reshape(-1))])[:-1].reshape(world, e_local)
    expert_counts = rc.sum(axis=0)
    expert_offsets = np.concatenate([[0], np.cumsum(expert_counts)])
    # grouped order: (e, src) segments; within an expert the sources keep rank order.
    # Position g of the grouped buffer lies in segment k: it reads arrival row
    # seg_arrival_start[k] + (g - seg_grouped_start[k]).
    seg_len = rc.T.reshape(-1)                                   # (e, src) order
    seg_grouped_start = np.concatenate([[0], np.cumsum(seg_len)])[:-1]
    shift = seg_arrival_start.T.reshape(-1) - seg_grouped_start
    gather = (np.repeat(shift, seg_len) + np.arange(total, dtype=np.int64)).astype(np.int32)
    scatter = np.empty(total, dtype=np.int32)
    scatter[gather] = np.arange(total, dtype=np.int32)
    return RegroupPlan(gather=gather, scatter=scatter,
                       expert_offsets=expert_offsets.astype(np.int32),
                       expert_counts=expert_counts.astype(np.int32),
                       recv_splits=recv_splits)


class ExpertParallelMoE:
    """One rank's side of the expert-parallel forward.

    ops must provide (all on this rank's device):
      route(x, logits | w_router) -> (topk_ids [T,k] i32, topk_weights [T,k] f32)
      sort(topk_ids, topk_weights, experts) -> object with .expert_counts [E], .route_pos [T*k]
            and whatever permute() needs; compact layout (no padding between experts)
      permute(x, routes) -> rows [T*k, H] in sorted order
      gather(rows, index [R] i32) -> rows[index]
      expert_ffn(rows [R,H], expert_offsets [E_l+1] i32, expert_counts [E_l] i32, w13_l, w2_l) -> [R,H]
      combine(rows [T*k,H], routes, topk_weights, tokens) -> [T,H]
      to_host(tensor) -> numpy,  from_host(np array, dtype) -> tensor on the device
      empty(shape, dtype) -> tensor on the device
    """

    def __init__(self, *, experts: int, topk: int, group=None, ops=None):
        self.E, self.k = experts, topk
        self.group = group
        self.ops = ops
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.e_local = experts_per_rank(experts, self.world)
        self.last_plan: RegroupPlan | None = None
        self.last_send_splits: np.ndarray | None = None

    def forward(self, x, w13_local, w2_local, *, logits=None, w_router=None):
        ops, G, El = self.ops, self.world, self.e_local
        T, H = x.shape
        ids, wts = ops.route(x, logits=logits, w_router=w_router)
        routes = ops.sort(ids, wts, self.E)
        rows = ops.permute(x, routes)  # [T*k, H], grouped by destination rank already

        # 1) exchange per-expert counts: I send counts[g*El:(g+1)*El] to rank g
        counts = routes.expert_counts
        recv_counts = ops.empty((G * El,), counts.dtype)
        dist.all_to_all_single(recv_counts, counts.contiguous(), group=self.group)
        both = ops.to_host(torch.cat([counts.view(-1), recv_counts.view(-1)]))  # the one host sync
        counts_h = both[: self.E]
        plan = regroup_plan(both[self.E:].reshape(G, El))
        in_splits = send_splits(counts_h, G)
        self.last_plan, self.last_send_splits = plan, in_splits
        R = int(plan.recv_splits.sum())

        # 2) dispatch the rows
        recv = ops.empty((R, H), rows.dtype)
        dist.all_to_all_single(recv, rows[: int(in_splits.sum())], plan.recv_splits.tolist(),
                               in_splits.tolist(), group=self.group)

        # 3) regroup by expert, run the experts, restore arrival order
        if R > 0:
            # one upload: [gather | scatter | expert_offsets | expert_counts]
            packed = ops.from_host(np.concatenate([plan.gather, plan.scatter, plan.expert_offsets,
                                                   plan.expert_counts]), torch.int32)
            gather_d, scatter_d = packed[:R], packed[R:2 * R]
            offsets_d, counts_d = packed[2 * R:2 * R + El + 1], packed[2 * R + El + 1:]
            grouped = ops.gather(recv, gather_d)
            y = ops.expert_ffn(grouped, offsets_d, counts_d, w13_local, w2_local)
            y_back = ops.gather(y, scatter_d)
        else:
            y_back = recv

        # 4) send the outputs home (the splits swap roles)
        ret = ops.empty((int(in_splits.sum()), H), rows.dtype)
        dist.all_to_all_single(ret, y_back, in_splits.tolist(), plan.recv_splits.tolist(),
                               group=self.group)

        # 5) weighted combine over each token's k routes
        return ops.combine(ret, routes, wts, T)


class CudaOps:
    """The C-ABI kernels behind ExpertParallelMoE on one GPU."""

    def __init__(self, device: torch.device, *, tokens_global: int, experts: int, topk: int):
        from . import moe

        self.moe = moe
        self.dev = device
        self.topk = topk
        self.rows_hint = max(1, (tokens_global * topk + experts - 1) // experts)

    def route(self, x, *, logits=None, w_router=None):
        if logits is None:
            logits = self.moe.router_logits(x, w_router)
        return self.moe.route_topk(logits, self.topk)

    def sort(self, ids, wts, experts):
        return self.moe.build_sorted_routes(topk_ids=ids, topk_weights=wts, experts=experts, group=1)

    def permute(self, x, routes):
        return self.moe.permute_rows(x, routes)

    def gather(self, rows, index):
        return self.moe.gather_rows(rows, index)

    def expert_ffn(self, rows, expert_offsets, expert_counts, w13, w2):
        class _R:
            pass

        r = _R()
        r.expert_offsets, r.expert_counts = expert_offsets, expert_counts
        h = self.moe.grouped_gemm(rows, w13, r, gated=True, rows_hint=self.rows_hint)
        return self.moe.grouped_gemm(h, w2, r, gated=False, rows_hint=self.rows_hint)

    def combine(self, rows, routes, wts, tokens):
        return self.moe.combine(rows, routes, wts, tokens)

    def to_host(self, t):
        return t.cpu().numpy()

    def from_host(self, a, dtype):
        t = torch.from_numpy(np.ascontiguousarray(a)).to(dtype)
        return t.pin_memory().to(self.dev, non_blocking=True)

    def empty(self, shape, dtype):
        return torch.empty(shape, dtype=dtype, device=self.dev)
