"""The expert-parallel exchange kernels on ONE GPU: G "virtual ranks" share cuda:0.

The C-ABI takes the peers' buffers as a plain array of device pointers, so the buffers of
G ranks can all live on one device.  Every rank's kernels are launched in turn on one
stream (stream order stands in for the barriers between GPUs; no kernel here waits for
another one), which exercises lumen_b200_moe_ep_plan / _dispatch / _return / _row_ptrs and
lumen_b200_moe_grouped_gemm_to_rows exactly as PeerExpertParallelMoE.forward drives them:

  per rank: top-k -> compact sort         (counts gathered into the G x E matrix)
  per rank: plan (checked against moe_ep.peer_plan) -> dispatch into the owners' buffers
  per rank: grouped GEMMs on the received rows -> return (bulk kernel, or the second
            GEMM's epilogue through the row-address table)
  per rank: weighted combine, compared with the CPU oracle

The barrier and count-exchange kernels are run with G = 1 (a rank that is its own only
peer); a barrier whose peer never signals is covered in test_failure_paths_gpu.py.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import ATOL, RTOL
from oracle import moe_oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _ptr_array(tensors):
    arr = (ctypes.c_void_p * len(tensors))(*[t.data_ptr() for t in tensors])
    return arr


class VirtualRank:
    """Buffers of one rank (the ones PeerExpertParallelMoE allocates per GPU)."""

    def __init__(self, pkg, rank, G, Tl, H, I, E, k):
        moe = pkg.moe
        i32 = dict(dtype=torch.int32, device=DEV)
        self.rank = rank
        self.capacity = Tl * G * k
        self.home_rows = moe.max_padded_routes(Tl, k, E, 1)
        self.recv = torch.full((self.capacity, H), float("nan"), dtype=torch.bfloat16, device=DEV)
        self.ret = torch.full((self.home_rows, H), float("nan"), dtype=torch.bfloat16, device=DEV)
        self.routes = moe.alloc_sorted_routes(Tl, k, E, DEV, group=1)
        El = E // G
        self.send_dst_start = torch.zeros((E,), **i32)
        self.local_offsets = torch.zeros((El + 1,), **i32)
        self.local_counts = torch.zeros((El,), **i32)
        self.seg_start = torch.zeros((El * G + 1,), **i32)
        self.seg_home_row = torch.zeros((El * G,), **i32)
        self.h = torch.empty((self.capacity, I), dtype=torch.bfloat16, device=DEV)
        self.y = torch.empty((self.capacity, H), dtype=torch.bfloat16, device=DEV)
        self.row_ptrs = torch.zeros((self.capacity,), dtype=torch.int64, device=DEV)
        self.topk_ids = torch.empty((Tl, k), **i32)
        self.topk_weights = torch.empty((Tl, k), dtype=torch.float32, device=DEV)

        class _Local:
            pass

        self.local = _Local()
        self.local.expert_offsets, self.local.expert_counts = self.local_offsets, self.local_counts


def _run(pkg, G, T, H, I, E, k, *, skew, fused_return, seed):
    moe, lib, check = pkg.moe, pkg._cabi.load(), pkg._cabi.check
    stream = torch.cuda.current_stream(DEV).cuda_stream
    d = moe_oracle.moe_inputs(T, H, I, E, seed, with_router=False)
    logits = d["logits"].clone()
    if skew:  # most routes land on the last rank's experts; expert 0 receives nothing
        logits[:, E - E // G:] += 3.0
        logits[:, 0] = -50.0
    Tl, El = T // G, E // G
    ranks = [VirtualRank(pkg, r, G, Tl, H, I, E, k) for r in range(G)]
    xs = [d["x"][r * Tl:(r + 1) * Tl].to(DEV) for r in range(G)]
    w13 = [d["w13"][r * El:(r + 1) * El].to(DEV) for r in range(G)]
    w2 = [d["w2"][r * El:(r + 1) * El].to(DEV) for r in range(G)]
    rows_hint = max(1, (T * k + E - 1) // E)

    # 1) route and sort locally; gather the counts (host stands in for the count exchange)
    for r, vr in enumerate(ranks):
        moe.route_topk(logits[r * Tl:(r + 1) * Tl].to(DEV), k, ids_out=vr.topk_ids, weights_out=vr.topk_weights)
        moe.build_sorted_routes(topk_ids=vr.topk_ids, topk_weights=vr.topk_weights, experts=E,
                                out=vr.routes, group=1)
    torch.cuda.synchronize()
    counts = np.stack([vr.routes.expert_counts.cpu().numpy() for vr in ranks])
    count_matrix = torch.from_numpy(counts).to(DEV)
    recv_peers = _ptr_array([vr.recv for vr in ranks])
    ret_peers = _ptr_array([vr.ret for vr in ranks])

    # 2) plan + dispatch of every rank
    for r, vr in enumerate(ranks):
        check("plan", lib.lumen_b200_moe_ep_plan(
            count_matrix.data_ptr(), G, E, r, vr.send_dst_start.data_ptr(), vr.local_offsets.data_ptr(),
            vr.local_counts.data_ptr(), vr.seg_start.data_ptr(), vr.seg_home_row.data_ptr(), stream))
        rt = vr.routes
        check("dispatch", lib.lumen_b200_moe_ep_dispatch(
            xs[r].data_ptr(), rt.sorted_token_ids.data_ptr(), rt.sorted_expert_ids.data_ptr(),
            rt.expert_offsets.data_ptr(), vr.send_dst_start.data_ptr(), rt.num_valid_ids.data_ptr(),
            recv_peers, G, Tl, H, E, Tl * k, vr.capacity, stream))
    torch.cuda.synchronize()
    for r, vr in enumerate(ranks):
        ref = pkg.moe_ep.peer_plan(counts, r)
        assert np.array_equal(vr.send_dst_start.cpu().numpy(), ref.send_dst_start)
        assert np.array_equal(vr.local_offsets.cpu().numpy(), ref.local_offsets)
        assert np.array_equal(vr.local_counts.cpu().numpy(), ref.local_counts)
        assert np.array_equal(vr.seg_start.cpu().numpy(), ref.seg_start)
        assert np.array_equal(vr.seg_home_row.cpu().numpy(), ref.seg_home_row)

    # every received row is the row of the token the oracle's routing sends there:
    # rank r's grouped buffer holds, per local expert, the rows of source 0, 1, ... in
    # each source's (token ascending, slot ascending) order
    ids, w = moe_oracle.route_topk(logits, k)
    for r, vr in enumerate(ranks):
        want_rows = []
        for le in range(El):
            e = r * El + le
            for s in range(G):
                tok, _slot = np.nonzero(ids[s * Tl:(s + 1) * Tl].numpy() == e)
                want_rows.append(d["x"][s * Tl + torch.from_numpy(tok)])
        want_rows = torch.cat(want_rows) if want_rows else torch.empty((0, H), dtype=torch.bfloat16)
        got = vr.recv[: want_rows.shape[0]].cpu()
        assert torch.equal(got.view(torch.int16), want_rows.view(torch.int16)), f"rank {r} received rows"

    # 3) expert GEMMs on the received rows and the trip home
    for r, vr in enumerate(ranks):
        moe.grouped_gemm(vr.recv, w13[r], vr.local, gated=True, rows_hint=rows_hint, out=vr.h)
        if fused_return:
            check("row_ptrs", lib.lumen_b200_moe_ep_row_ptrs(
                vr.seg_start.data_ptr(), vr.seg_home_row.data_ptr(), ret_peers, G, El, H, vr.capacity,
                vr.home_rows, vr.row_ptrs.data_ptr(), stream))
            moe.grouped_gemm_to_rows(vr.h, w2[r], vr.row_ptrs, vr.local, gated=False, rows_hint=rows_hint)
        else:
            moe.grouped_gemm(vr.h, w2[r], vr.local, gated=False, rows_hint=rows_hint, out=vr.y)
            check("return", lib.lumen_b200_moe_ep_return(
                vr.y.data_ptr(), vr.seg_start.data_ptr(), vr.seg_home_row.data_ptr(), ret_peers, G, El, H,
                vr.capacity, vr.home_rows, stream))

    # 4) combine at home and compare with the oracle
    want = moe_oracle.moe_reference(d["x"], d["w13"], d["w2"], ids, w)
    outs = []
    for r, vr in enumerate(ranks):
        out = moe.combine(vr.ret, vr.routes, vr.topk_weights, Tl)
        torch.cuda.synchronize()
        assert torch.equal(vr.topk_ids.cpu(), ids[r * Tl:(r + 1) * Tl])
        torch.testing.assert_close(out.cpu().float(), want[r * Tl:(r + 1) * Tl].float(), rtol=RTOL, atol=ATOL)
        outs.append(out.cpu())
    assert pkg.device_status() == 0
    return torch.cat(outs)


@pytest.mark.parametrize("G", [2, 4, 8])
@pytest.mark.parametrize("skew", [False, True])
def test_virtual_ranks_match_oracle(cuda_pkg, G, skew):
    """Both return paths give the oracle's result and the same bits as each other, and the
    same bits as the single-GPU forward (the exchange moves rows, it changes no arithmetic
    except the tile a row falls into)."""
    T, H, I, E, k = 256, 512, 384, 16, 4
    a = _run(cuda_pkg, G, T, H, I, E, k, skew=skew, fused_return=False, seed=20260319 + G)
    b = _run(cuda_pkg, G, T, H, I, E, k, skew=skew, fused_return=True, seed=20260319 + G)
    assert torch.equal(a, b)


def test_virtual_ranks_fine_grained_shape(cuda_pkg):
    """Eight ranks, 256 experts, top-8 at the fine-grained configuration's hidden sizes
    (32 experts per rank, 7168 -> 2048 -> 7168), fewer tokens."""
    _run(cuda_pkg, 8, 512, 7168, 2048, 256, 8, skew=False, fused_return=False, seed=5)


def test_count_exchange_and_barrier_with_one_rank(cuda_pkg):
    """G = 1: the rank is its own only peer, so the barrier's wait is satisfied by its own
    signal and the count exchange is a copy; epochs advance by one per call."""
    lib, check = cuda_pkg._cabi.load(), cuda_pkg._cabi.check
    stream = torch.cuda.current_stream(DEV).cuda_stream
    E = 256
    counts = torch.arange(E, dtype=torch.int32, device=DEV) * 3 + 1
    matrix = torch.zeros((1, E), dtype=torch.int32, device=DEV)
    signals = torch.zeros((64,), dtype=torch.int32, device=DEV)
    epochs = torch.zeros((4,), dtype=torch.int32, device=DEV)
    mats, sigs = _ptr_array([matrix]), _ptr_array([signals])
    for i in range(3):
        check("exchange", lib.lumen_b200_moe_ep_exchange_counts(
            counts.data_ptr(), E, 0, 1, mats, sigs, epochs.data_ptr(), 0, stream))
        check("barrier", lib.lumen_b200_moe_ep_barrier(0, 1, sigs, epochs.data_ptr(), 2, stream))
    torch.cuda.synchronize()
    assert torch.equal(matrix[0], counts)
    assert epochs.cpu().tolist() == [3, 0, 3, 0]
    sig = signals.cpu().view(4, 16)
    assert sig[0, 0].item() == 3 and sig[2, 0].item() == 3
    assert cuda_pkg.device_status() == 0
