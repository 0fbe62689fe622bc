"""Expert-parallel MoE forward over the GPUs of one node.

Tokens are sharded (T/G per rank: router, top-k and sort run locally), experts are
sharded (E/G per rank, expert e lives on rank e // (E/G)).  There is one exchange step each
way: the expert-sorted activation rows go to the GPUs that own their experts (dispatch) and
the expert outputs come back (return), before the local weighted combine.

Two transports implement the exchange.  PeerExpertParallelMoE (the default choice on
NVLink-connected GPUs) uses this library's own kernels, which store rows directly into the
peers' buffers.  ExpertParallelMoE uses all_to_all_single collectives: per-expert counts
first, one host read, then the rows with split sizes; the notes below describe it.

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


@dataclass
class PeerPlan:
    """What lumen_b200_moe_ep_plan computes on the device, restated in numpy (used by the
    tests and as the specification of the kernel)."""

    send_dst_start: np.ndarray  # [E]
    local_offsets: np.ndarray   # [El + 1]
    local_counts: np.ndarray    # [El]
    seg_start: np.ndarray       # [El * G + 1], index le * G + s
    seg_home_row: np.ndarray    # [El * G]


def peer_plan(counts: np.ndarray, rank: int) -> PeerPlan:
    """counts[s, e] = routes of GPU s for global expert e."""
    c = np.asarray(counts, dtype=np.int64)
    G, E = c.shape
    El = experts_per_rank(E, G)
    total = c.sum(axis=0)
    prefix = np.concatenate([[0], np.cumsum(total)])
    owner_base = prefix[(np.arange(E) // El) * El]
    before_me = c[:rank].sum(axis=0)
    send_dst_start = prefix[:-1] - owner_base + before_me
    mine = slice(rank * El, (rank + 1) * El)
    local_counts = total[mine]
    local_offsets = np.concatenate([[0], np.cumsum(local_counts)])
    before_src = np.cumsum(c[:, mine], axis=0) - c[:, mine]          # [G, El]
    seg_start = (local_offsets[:-1][:, None] + before_src.T).reshape(-1)  # (le, s) order
    seg_start = np.concatenate([seg_start, [local_offsets[-1]]])
    home = np.cumsum(c, axis=1) - c                                     # [G, E] exclusive over experts
    seg_home_row = home[:, mine].T.reshape(-1)
    i32 = np.int32
    return PeerPlan(send_dst_start.astype(i32), local_offsets.astype(i32), local_counts.astype(i32),
                    seg_start.astype(i32), seg_home_row.astype(i32))


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

    def forward(self, x, w13_local, w2_local, *, logits=None, w_router=None, marks=None):
        """`marks`, if a list, receives (label, CUDA event) pairs recorded on the current
        stream after each phase (measurement aid; events need a CUDA device)."""
        ops, G, El = self.ops, self.world, self.e_local
        T, H = x.shape

        def mark(label):
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append((label, ev))

        mark("start")
        ids, wts = ops.route(x, logits=logits, w_router=w_router)
        routes = ops.sort(ids, wts, self.E)
        rows = ops.permute(x, routes)  # [T*k, H], grouped by destination rank already
        mark("route+sort+permute")

        # 1) exchange per-expert counts: I send counts[g*El:(g+1)*El] to rank g
        counts = routes.expert_counts
        recv_counts = ops.empty((G * El,), counts.dtype)
        dist.all_to_all_single(recv_counts, counts.contiguous(), group=self.group)
        both = ops.to_host(torch.cat([counts.view(-1), recv_counts.view(-1)]))  # the one host sync
        counts_h = both[: self.E]
        plan = regroup_plan(both[self.E:].reshape(G, El))
        in_splits = send_splits(counts_h, G)
        self.last_plan, self.last_send_splits = plan, in_splits
        # The split sizes every rank derives must describe the rows it really holds; a rank
        # whose counts and rows disagree stops here, before the payload collective (its peers
        # then run into the process group's timeout instead of receiving misplaced rows).
        if int(in_splits.sum()) != T * self.k or int(in_splits.sum()) > rows.shape[0]:
            raise ValueError(f"rank {self.rank}: per-expert counts add up to {int(in_splits.sum())} routes, "
                             f"but {T} tokens x top-{self.k} = {T * self.k} routes were sorted")
        R = int(plan.recv_splits.sum())
        mark("counts exchange + host plan")

        # 2) dispatch the rows
        recv = ops.empty((R, H), rows.dtype)
        dist.all_to_all_single(recv, rows[: int(in_splits.sum())], plan.recv_splits.tolist(),
                               in_splits.tolist(), group=self.group)
        mark("dispatch all_to_all")

        # 3) regroup by expert, run the experts, restore arrival order
        if R > 0:
            # one upload: [gather | scatter | expert_offsets | expert_counts]
            packed = ops.from_host(np.concatenate([plan.gather, plan.scatter, plan.expert_offsets,
                                                   plan.expert_counts]), torch.int32)
            gather_d, scatter_d = packed[:R], packed[R:2 * R]
            offsets_d, counts_d = packed[2 * R:2 * R + El + 1], packed[2 * R + El + 1:]
            grouped = ops.gather(recv, gather_d)
            mark("regroup gather")
            y = ops.expert_ffn(grouped, offsets_d, counts_d, w13_local, w2_local)
            mark("expert GEMMs")
            y_back = ops.gather(y, scatter_d)
            mark("restore gather")
        else:
            y_back = recv

        # 4) send the outputs home (the splits swap roles)
        ret = ops.empty((int(in_splits.sum()), H), rows.dtype)
        dist.all_to_all_single(ret, y_back, in_splits.tolist(), plan.recv_splits.tolist(),
                               group=self.group)

        mark("return all_to_all")

        # 5) weighted combine over each token's k routes
        out = ops.combine(ret, routes, wts, T)
        mark("combine")
        return out


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


class PeerExpertParallelMoE:
    """Expert-parallel forward whose dispatch and return are this library's own kernels
    writing over NVLink into the peers' buffers (symmetric memory), instead of a packed send
    buffer plus all_to_all.  The host reads nothing during a forward: every GPU derives the
    same offsets from the all-gathered G x E count matrix on the device.

      route -> compact sort -> counts to every peer + barrier -> plan -> dispatch (peer
      stores) -> barrier -> grouped GEMMs on the received rows -> return (peer stores)
      -> barrier -> weighted combine

    Buffers are sized for the worst case (every route of every GPU lands on one GPU).
    Construction is collective (symmetric-memory rendezvous)."""

    def __init__(self, *, tokens_local: int, hidden: int, inter: int, experts: int, topk: int,
                 device: torch.device, group=None, fused_return: bool = False, sync: str = "signals"):
        import ctypes
        import os

        import torch.distributed._symmetric_memory as symm_mem

        from . import _cabi, moe

        # plain peer loads/stores only: no NVLink multicast binding of these buffers
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        self.moe, self._cabi = moe, _cabi
        self.group = group if group is not None else dist.group.WORLD
        self.G = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.T, self.H, self.I, self.E, self.k = tokens_local, hidden, inter, experts, topk
        self.El = experts_per_rank(experts, self.G)
        self.dev = device
        self.capacity = tokens_local * self.G * topk
        self.home_rows = moe.max_padded_routes(tokens_local, topk, experts, 1)
        bf16, i32 = torch.bfloat16, torch.int32
        self.recv = symm_mem.empty((self.capacity, hidden), dtype=bf16, device=device)
        self.ret = symm_mem.empty((self.home_rows, hidden), dtype=bf16, device=device)
        self._recv_hdl = symm_mem.rendezvous(self.recv, self.group)
        self._ret_hdl = symm_mem.rendezvous(self.ret, self.group)
        ptr_array = ctypes.c_void_p * self.G
        self._recv_peers = ptr_array(*[int(p) for p in self._recv_hdl.buffer_ptrs])
        self._ret_peers = ptr_array(*[int(p) for p in self._ret_hdl.buffer_ptrs])
        self.routes = moe.alloc_sorted_routes(tokens_local, topk, experts, device, group=1)
        need = int(_cabi.load().lumen_b200_moe_sort_scratch_bytes(tokens_local, experts, topk))
        self.scratch = torch.empty((max(need, 4),), dtype=torch.uint8, device=device)
        self.topk_ids = torch.empty((tokens_local, topk), dtype=i32, device=device)
        self.topk_weights = torch.empty((tokens_local, topk), dtype=torch.float32, device=device)
        self.logits = torch.empty((tokens_local, experts), dtype=torch.float32, device=device)
        # sync = "signals": the GPUs meet through flags in each other's memory (this library's
        # barrier kernel) and exchange their expert counts with peer stores, so a forward
        # contains no collective-library call at all; sync = "nccl": all_gather + all_reduce
        if sync not in ("signals", "nccl"):
            raise ValueError("sync must be 'signals' or 'nccl'")
        self.sync = sync
        self.count_matrix = symm_mem.empty((self.G, experts), dtype=i32, device=device)
        self.signals = symm_mem.empty((64,), dtype=i32, device=device)
        self.count_matrix.zero_()
        self.signals.zero_()
        self._cm_hdl = symm_mem.rendezvous(self.count_matrix, self.group)
        self._sig_hdl = symm_mem.rendezvous(self.signals, self.group)
        self._cm_peers = ptr_array(*[int(p) for p in self._cm_hdl.buffer_ptrs])
        self._sig_peers = ptr_array(*[int(p) for p in self._sig_hdl.buffer_ptrs])
        self.epochs = torch.zeros((4,), dtype=i32, device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)  # every GPU's flags are zero before anybody signals
        self.send_dst_start = torch.zeros((experts,), dtype=i32, device=device)
        self.local_offsets = torch.zeros((self.El + 1,), dtype=i32, device=device)
        self.local_counts = torch.zeros((self.El,), dtype=i32, device=device)
        self.seg_start = torch.zeros((self.El * self.G + 1,), dtype=i32, device=device)
        self.seg_home_row = torch.zeros((self.El * self.G,), dtype=i32, device=device)
        self.h = torch.empty((self.capacity, inter), dtype=bf16, device=device)
        self.y = torch.empty((self.capacity, hidden), dtype=bf16, device=device)
        self.out = torch.empty((tokens_local, hidden), dtype=bf16, device=device)
        # fused_return: the second expert GEMM stores each output row straight into its home
        # GPU's buffer (row address table), instead of a local y followed by a return kernel.
        # Same bits either way; off by default because the epilogue's row-wise peer stores
        # slow the GEMM by more than the bulk return kernel costs (2 GPUs, 8192 tokens, 256
        # experts: 4.33 ms fused against 3.99 ms separate; equal for 8 large experts).
        self.fused_return = fused_return
        self.row_ptrs = torch.zeros((self.capacity,), dtype=torch.int64, device=device)
        self._flag = torch.zeros((1,), dtype=torch.float32, device=device)
        # page-locked copy of the device status word, refreshed at the end of every forward
        self._status_host = torch.zeros((1,), dtype=torch.int32).pin_memory()
        self.rows_hint = max(1, (tokens_local * self.G * topk + experts - 1) // experts)

        class _Local:
            pass

        self._local = _Local()
        self._local.expert_offsets, self._local.expert_counts = self.local_offsets, self.local_counts

    def _gpu_barrier(self, slot: int):
        # stream-ordered rendezvous of all GPUs: nobody passes before everybody's earlier
        # kernels (the peer stores) have completed
        if self.sync == "nccl":
            dist.all_reduce(self._flag, group=self.group)
            return
        with self._cabi.on_device(self.dev):
            self._cabi.check("lumen_b200_moe_ep_barrier", self._cabi.load().lumen_b200_moe_ep_barrier(
                self.rank, self.G, self._sig_peers, self.epochs.data_ptr(), slot,
                torch.cuda.current_stream(self.dev).cuda_stream))

    def check_status(self) -> None:
        """Raises if a kernel of an earlier forward recorded a wait that gave up (e.g. a peer
        GPU that was more than the barrier's wait limit late).  Reads the page-locked copy the
        previous forward left behind: no synchronisation, so the newest forward may not be
        covered yet; device_status() synchronises and covers everything."""
        code = int(self._status_host[0])
        if code != 0:
            raise self._cabi.LumenB200Error(
                f"expert-parallel forward (status word {code:#x}: site {code >> 16}, "
                f"slot {(code >> 8) & 0xff}, peer {code & 0xff})", self._cabi.EDEVICE)

    def forward(self, x, w13_local, w2_local, *, logits=None, w_router=None, marks=None):
        moe, lib = self.moe, self._cabi.load()
        stream = torch.cuda.current_stream(self.dev).cuda_stream
        self.check_status()

        def mark(label):
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append((label, ev))

        mark("start")
        if logits is None:
            logits = moe.router_logits(x, w_router, out=self.logits)
        moe.route_topk(logits, self.k, ids_out=self.topk_ids, weights_out=self.topk_weights)
        r = moe.build_sorted_routes(topk_ids=self.topk_ids, topk_weights=self.topk_weights,
                                    experts=self.E, out=self.routes, scratch=self.scratch, group=1)
        mark("route+sort")
        if self.sync == "nccl":
            dist.all_gather_into_tensor(self.count_matrix.view(-1), r.expert_counts, group=self.group)
        else:
            with self._cabi.on_device(self.dev):
                self._cabi.check("lumen_b200_moe_ep_exchange_counts", lib.lumen_b200_moe_ep_exchange_counts(
                    r.expert_counts.data_ptr(), self.E, self.rank, self.G, self._cm_peers, self._sig_peers,
                    self.epochs.data_ptr(), 0, stream))
        with self._cabi.on_device(self.dev):
            self._cabi.check("lumen_b200_moe_ep_plan", lib.lumen_b200_moe_ep_plan(
                self.count_matrix.data_ptr(), self.G, self.E, self.rank, self.send_dst_start.data_ptr(),
                self.local_offsets.data_ptr(), self.local_counts.data_ptr(), self.seg_start.data_ptr(),
                self.seg_home_row.data_ptr(), stream))
            mark("counts all_gather + plan")
            self._cabi.check("lumen_b200_moe_ep_dispatch", lib.lumen_b200_moe_ep_dispatch(
                x.data_ptr(), r.sorted_token_ids.data_ptr(), r.sorted_expert_ids.data_ptr(),
                r.expert_offsets.data_ptr(), self.send_dst_start.data_ptr(), r.num_valid_ids.data_ptr(),
                self._recv_peers, self.G, self.T, self.H, self.E, self.T * self.k, self.capacity, stream))
        self._gpu_barrier(1)
        mark("dispatch (peer stores) + barrier")
        moe.grouped_gemm(self.recv, w13_local, self._local, gated=True, rows_hint=self.rows_hint, out=self.h)
        if self.fused_return:
            with self._cabi.on_device(self.dev):
                self._cabi.check("lumen_b200_moe_ep_row_ptrs", lib.lumen_b200_moe_ep_row_ptrs(
                    self.seg_start.data_ptr(), self.seg_home_row.data_ptr(), self._ret_peers, self.G,
                    self.El, self.H, self.capacity, self.home_rows, self.row_ptrs.data_ptr(), stream))
            moe.grouped_gemm_to_rows(self.h, w2_local, self.row_ptrs, self._local, gated=False,
                                     rows_hint=self.rows_hint)
            mark("expert GEMMs (second one stores to the home GPUs)")
        else:
            moe.grouped_gemm(self.h, w2_local, self._local, gated=False, rows_hint=self.rows_hint, out=self.y)
            mark("expert GEMMs")
            with self._cabi.on_device(self.dev):
                self._cabi.check("lumen_b200_moe_ep_return", lib.lumen_b200_moe_ep_return(
                    self.y.data_ptr(), self.seg_start.data_ptr(), self.seg_home_row.data_ptr(),
                    self._ret_peers, self.G, self.El, self.H, self.capacity, self.home_rows, stream))
        self._gpu_barrier(2)
        mark("return + barrier")
        out = moe.combine(self.ret, r, self.topk_weights, self.T, out=self.out)
        with self._cabi.on_device(self.dev):
            self._cabi.check("lumen_b200_status_snapshot", lib.lumen_b200_status_snapshot(
                self._status_host.data_ptr(), stream))
        mark("combine")
        return out
