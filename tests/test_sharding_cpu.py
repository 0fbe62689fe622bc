"""Host logic of the multi-GPU paths, on CPU: shard arithmetic, and the expert-parallel MoE
driven end to end over a world_size-2 (and 4) gloo group with the oracle standing in for the
kernels.  The same ExpertParallelMoE code runs over NCCL with the C-ABI kernels on GPUs."""
from __future__ import annotations

import importlib
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))
from oracle import moe_oracle  # noqa: E402

PKG = "lumen-sosp26-ae_b200"


def _pkg():
    return importlib.import_module(PKG)


# ------------------------------------------------------------------ shard arithmetic
@pytest.mark.parametrize("n", [4096, 6144, 14336, 520])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_gemm_column_ranges_tile_the_columns(n, world):
    sh = _pkg().sharding
    ranges = [sh.gemm_column_range(n, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0 and a1 > a0
    assert all(lo % 8 == 0 for lo, _ in ranges)
    sizes = [hi - lo for lo, hi in ranges]
    assert max(sizes) - min(sizes) <= 8


@pytest.mark.parametrize("batch,kv_heads", [(8, 8), (2, 16), (16, 1)])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_attention_shards_cover_every_unit_once(batch, kv_heads, world):
    sh = _pkg().sharding
    if world > batch and (world % batch != 0 or kv_heads % (world // batch) != 0):
        with pytest.raises(ValueError):
            sh.attention_shard(batch, kv_heads, world, 0)
        return
    seen = np.zeros((batch, kv_heads), dtype=np.int32)
    for r in range(world):
        s = sh.attention_shard(batch, kv_heads, world, r)
        seen[s.b0:s.b1, s.hk0:s.hk1] += 1
    assert (seen == 1).all()
    assert len({sh.attention_shard(batch, kv_heads, world, r).units() for r in range(world)}) == 1


def test_sliced_attention_inputs_keep_heads_with_their_kv_head():
    sh = _pkg().sharding
    q = torch.arange(2 * 3 * 8 * 4, dtype=torch.float32).view(2, 3, 8, 4)
    k = torch.arange(2 * 3 * 4 * 4, dtype=torch.float32).view(2, 3, 4, 4)
    s = sh.attention_shard(2, 4, 4, 3)  # second batch entry, KV heads 2..3
    qs, ks, vs = sh.slice_attention_inputs(q, k, k, s)
    assert qs.shape == (1, 3, 4, 4) and ks.shape == (1, 3, 2, 4)
    assert torch.equal(qs, q[1:2, :, 4:8]) and torch.equal(ks, k[1:2, :, 2:4])
    assert qs.is_contiguous() and ks.is_contiguous()


def test_regroup_plan_is_a_permutation_grouped_by_expert():
    ep = _pkg().moe_ep
    rc = np.array([[3, 0, 2], [1, 4, 0]])  # 2 sources, 3 local experts
    plan = ep.regroup_plan(rc)
    assert plan.recv_splits.tolist() == [5, 5]
    assert plan.expert_counts.tolist() == [4, 4, 2] and plan.expert_offsets.tolist() == [0, 4, 8, 10]
    # arrival order: src0: e0 e0 e0 e2 e2 | src1: e0 e1 e1 e1 e1
    arrival_expert = np.array([0, 0, 0, 2, 2, 0, 1, 1, 1, 1])
    grouped = arrival_expert[plan.gather]
    assert grouped.tolist() == [0, 0, 0, 0, 1, 1, 1, 1, 2, 2]
    assert plan.gather.tolist() == [0, 1, 2, 5, 6, 7, 8, 9, 3, 4]  # sources keep rank order
    assert np.array_equal(plan.gather[plan.scatter], np.arange(10))
    assert ep.send_splits(np.array([1, 2, 3, 4, 5, 6]), 2).tolist() == [6, 15]
    empty = ep.regroup_plan(np.zeros((2, 3), dtype=np.int64))
    assert empty.gather.size == 0 and empty.expert_offsets.tolist() == [0, 0, 0, 0]


def test_peer_plan_moves_every_row_there_and_back():
    """Simulate G GPUs in numpy: dispatch with send_dst_start, return with seg_start /
    seg_home_row; every route's row must land in its expert's group and come home."""
    ep = _pkg().moe_ep
    rng = np.random.default_rng(3)
    G, E, k, T = 4, 16, 3, 37
    El = E // G
    ids = [np.stack([rng.choice(E, size=k, replace=False) for _ in range(T)]).astype(np.int32) for _ in range(G)]
    ids[1][:, 0] = 5  # skew: one hot expert
    sorted_ = [moe_oracle.build_sorted_routes(ids[g], np.ones((T, k), np.float32), E, group=1) for g in range(G)]
    counts = np.stack([s[5] for s in sorted_])
    plans = [ep.peer_plan(counts, g) for g in range(G)]
    cap = T * k * G
    recv = [np.full((cap, 3), -1, dtype=np.int64) for _ in range(G)]  # payload: (src gpu, src pos, expert)
    for g in range(G):
        tok_ids, _, row_expert, nv, off, cnt, _ = sorted_[g]
        for pos in range(int(nv[0])):
            e = int(row_expert[pos])
            dst = int(plans[g].send_dst_start[e]) + pos - int(off[e])
            assert (recv[e // El][dst] == -1).all(), "two rows landed on one slot"
            recv[e // El][dst] = (g, pos, e)
    for g in range(G):
        p = plans[g]
        total = int(p.local_offsets[-1])
        assert total == int(counts[:, g * El:(g + 1) * El].sum())
        assert (recv[g][:total, 0] >= 0).all() and (recv[g][total:, 0] == -1).all()
        for le in range(El):  # grouped by expert, sources in rank order
            a, n = int(p.local_offsets[le]), int(p.local_counts[le])
            assert (recv[g][a:a + n, 2] == g * El + le).all()
            assert (np.diff(recv[g][a:a + n, 0]) >= 0).all()
        # return trip
        for row in range(total):
            kseg = int(np.searchsorted(p.seg_start, row, side="right")) - 1
            src = kseg % G
            home = int(p.seg_home_row[kseg]) + row - int(p.seg_start[kseg])
            assert recv[g][row, 0] == src and recv[g][row, 1] == home
    # the two formulations of the grouped layout agree
    for g in range(G):
        rp = ep.regroup_plan(counts[:, g * El:(g + 1) * El])
        assert np.array_equal(rp.expert_offsets, plans[g].local_offsets)
        assert np.array_equal(rp.expert_counts, plans[g].local_counts)


# ------------------------------------------------------------------ expert parallel over gloo
class OracleOps:
    """Stand-in arithmetic for ExpertParallelMoE: the CPU oracle (test infrastructure)."""

    def __init__(self, topk):
        self.topk = topk

    def route(self, x, *, logits=None, w_router=None):
        if logits is None:
            logits = moe_oracle.router_logits(x, w_router)
        return moe_oracle.route_topk(logits, self.topk)

    def sort(self, ids, wts, experts):
        o = moe_oracle.build_sorted_routes(ids.numpy(), wts.numpy(), experts, group=1)

        class R:
            pass

        r = R()
        r.sorted_token_ids = torch.from_numpy(o[0])
        r.expert_counts = torch.from_numpy(o[5])
        r.route_pos = torch.from_numpy(o[6])
        return r

    def permute(self, x, routes):
        tok = (routes.sorted_token_ids & 0xFFFFFF).long()
        out = torch.zeros((tok.numel(), x.shape[1]), dtype=x.dtype)
        valid = tok < x.shape[0]
        out[valid] = x[tok[valid]]
        return out

    def gather(self, rows, index):
        return rows[index.long()]

    def expert_ffn(self, rows, expert_offsets, expert_counts, w13, w2):
        out = torch.zeros((rows.shape[0], w2.shape[1]), dtype=torch.bfloat16)
        inter = w13.shape[1] // 2
        for e in range(w13.shape[0]):
            a, n = int(expert_offsets[e]), int(expert_counts[e])
            if n == 0:
                continue
            s1 = rows[a:a + n].float() @ w13[e].float().T
            h = torch.nn.functional.silu(s1[:, :inter]) * s1[:, inter:]
            out[a:a + n] = (h @ w2[e].float().T).to(torch.bfloat16)
        return out

    def combine(self, rows, routes, wts, tokens):
        k = wts.shape[1]
        pos = routes.route_pos.long().view(tokens, k)
        acc = (rows[pos].float() * wts.unsqueeze(-1)).sum(dim=1)
        return acc.to(torch.bfloat16)

    def to_host(self, t):
        return t.numpy()

    def from_host(self, a, dtype):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dtype)

    def empty(self, shape, dtype):
        return torch.empty(shape, dtype=dtype)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ep_worker(rank, world, port, T, H, I, E, k, skew, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ep = importlib.import_module(PKG).moe_ep
        d = moe_oracle.moe_inputs(T, H, I, E, 20260319, with_router=False)
        logits = d["logits"].clone()
        if skew:  # every token prefers experts owned by the last rank; some experts stay empty
            logits[:, E - E // world:] += 4.0
            logits[:, 1] = -50.0
        t0, t1 = rank * T // world, (rank + 1) * T // world
        el = E // world
        op = ep.ExpertParallelMoE(experts=E, topk=k, ops=OracleOps(k))
        out = op.forward(d["x"][t0:t1], d["w13"][rank * el:(rank + 1) * el],
                         d["w2"][rank * el:(rank + 1) * el], logits=logits[t0:t1])
        ids, w = moe_oracle.route_topk(logits, k)
        want = moe_oracle.moe_reference(d["x"], d["w13"], d["w2"], ids, w)[t0:t1]
        torch.testing.assert_close(out.float(), want.float(), rtol=2e-2, atol=2e-2)
        # what crossed the wire matches the routing
        counts = np.bincount(ids[t0:t1].numpy().reshape(-1), minlength=E)
        assert op.last_send_splits.tolist() == counts.reshape(world, el).sum(1).tolist()
        (Path(result_dir) / f"ok{rank}").write_text("ok")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,skew", [(2, False), (2, True), (4, False)])
def test_expert_parallel_forward_over_gloo(tmp_path, world, skew):
    T, H, I, E, k = 48, 64, 32, 8, 2
    mp.spawn(_ep_worker, args=(world, _free_port(), T, H, I, E, k, skew, str(tmp_path)),
             nprocs=world, join=True)
    assert sorted(p.name for p in tmp_path.iterdir()) == [f"ok{r}" for r in range(world)]


# ------------------------------------------------------------------ failures, made on the host
class _InflatedCounts(OracleOps):
    """A rank whose per-expert counts do not describe its rows (a corrupted histogram)."""

    def sort(self, ids, wts, experts):
        r = super().sort(ids, wts, experts)
        r.expert_counts = r.expert_counts.clone()
        r.expert_counts[0] += 3
        return r


def _ep_failure_worker(rank, world, port, mode, result_dir):
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=6))
    note = Path(result_dir) / f"rank{rank}"
    try:
        ep = importlib.import_module(PKG).moe_ep
        T, H, I, E, k = 32, 64, 32, 8, 2
        d = moe_oracle.moe_inputs(T, H, I, E, 7, with_router=False)
        t0, t1 = rank * T // world, (rank + 1) * T // world
        el = E // world
        args = (d["x"][t0:t1], d["w13"][rank * el:(rank + 1) * el], d["w2"][rank * el:(rank + 1) * el])
        bad = mode == "splits" and rank == 1
        op = ep.ExpertParallelMoE(experts=E, topk=k, ops=_InflatedCounts(k) if bad else OracleOps(k))
        try:
            if mode == "leave":
                op.forward(*args, logits=d["logits"][t0:t1])  # one good forward together
                if rank == 1:
                    note.write_text("left")
                    return  # leaves between forwards, nothing of its own in flight
            op.forward(*args, logits=d["logits"][t0:t1])
            note.write_text("finished")
        except Exception as exc:  # what the surviving / inconsistent rank must see
            note.write_text(f"raised:{type(exc).__name__}")
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


@pytest.mark.parametrize("mode", ["splits", "leave"])
def test_exchange_failures_surface_as_exceptions_not_hangs(tmp_path, mode):
    """Host-made failures of the collective transport: a rank whose split sizes disagree with
    its rows raises before it sends anything, a rank that has left makes the next forward of
    the others raise (process-group timeout or closed connection); nobody returns a result."""
    world = 2
    mp.spawn(_ep_failure_worker, args=(world, _free_port(), mode, str(tmp_path)), nprocs=world, join=True)
    notes = {p.name: p.read_text() for p in tmp_path.iterdir()}
    if mode == "splits":
        assert notes["rank1"] == "raised:ValueError"
        assert notes["rank0"].startswith("raised:")
    else:
        assert notes["rank1"] == "left"
        assert notes["rank0"].startswith("raised:")


# ------------------------------------------------------------------ property checks
def test_exchange_plans_hold_for_random_loads():
    """Random count matrices (empty experts, empty senders, one hot expert): both plans are
    permutations that group by expert with sources in rank order, and they agree."""
    from hypothesis import given, settings
    from hypothesis import strategies as st

    ep = _pkg().moe_ep

    @settings(max_examples=60, deadline=None)
    @given(st.integers(1, 4).flatmap(lambda g: st.tuples(
        st.just(g), st.integers(1, 5).map(lambda el: el * g))).flatmap(lambda ge: st.tuples(
            st.just(ge[0]), st.just(ge[1]),
            st.lists(st.lists(st.integers(0, 7), min_size=ge[1], max_size=ge[1]), min_size=ge[0], max_size=ge[0]))))
    def check(args):
        G, E, rows = args
        counts = np.array(rows, dtype=np.int64)
        El = E // G
        for rank in range(G):
            mine = counts[:, rank * El:(rank + 1) * El]
            rp = ep.regroup_plan(mine)
            pp = ep.peer_plan(counts, rank)
            total = int(mine.sum())
            assert sorted(rp.gather.tolist()) == list(range(total))
            assert np.array_equal(rp.gather[rp.scatter], np.arange(total))
            assert np.array_equal(rp.expert_offsets, pp.local_offsets)
            assert np.array_equal(rp.expert_counts, pp.local_counts)
            assert int(pp.seg_start[-1]) == total and (np.diff(pp.seg_start) >= 0).all()
            # segment (le, s) holds exactly the rows sender s has for local expert le
            assert np.array_equal(np.diff(pp.seg_start).reshape(El, G), mine.T)
            # a sender's rows of expert e start where the rows of its earlier experts end
            assert np.array_equal(pp.seg_home_row.reshape(El, G),
                                  (np.cumsum(counts, axis=1) - counts)[:, rank * El:(rank + 1) * El].T)
        # every sender's destination ranges tile the owners' grouped buffers without overlap
        for owner in range(G):
            spans = []
            for s in range(G):
                p = ep.peer_plan(counts, s)
                for e in range(owner * El, (owner + 1) * El):
                    if counts[s, e]:
                        spans.append((int(p.send_dst_start[e]), int(p.send_dst_start[e]) + int(counts[s, e])))
            spans.sort()
            pos = 0
            for a, b in spans:
                assert a == pos
                pos = b
            assert pos == int(counts[:, owner * El:(owner + 1) * El].sum())

    check()
