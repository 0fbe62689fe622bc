"""GPU parity of the MoE kernels (through the C-ABI) against the CPU oracle: routing and
the token permutation bit-exact, expert compute within tolerance."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import ATOL, RTOL, load_golden
from oracle import moe_oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def check_routes(pkg, ids, w, experts):
    r = pkg.moe.build_sorted_routes(topk_ids=ids.to(DEV), topk_weights=w.to(DEV), experts=experts)
    torch.cuda.synchronize()
    o = moe_oracle.build_sorted_routes(ids.numpy(), w.numpy(), experts)
    got = (r.sorted_token_ids, r.sorted_weights, r.sorted_expert_ids, r.num_valid_ids,
           r.expert_offsets, r.expert_counts, r.route_pos)
    names = ("sorted_token_ids", "sorted_weights", "sorted_expert_ids", "num_valid_ids",
             "expert_offsets", "expert_counts", "route_pos")
    for name, a, b in zip(names, got, o):
        assert np.array_equal(a.cpu().numpy(), b), name
    return r


@pytest.mark.parametrize("case,k", [("mixtral_like", 2), ("fine_grained", 8)])
def test_routing_golden_bit_exact(cuda_pkg, case, k):
    g = load_golden("moe")
    ids, w = cuda_pkg.moe.route_topk(g[f"{case}_logits"].to(DEV), k)
    torch.cuda.synchronize()
    assert torch.equal(ids.cpu(), g[f"{case}_topk_ids"])
    torch.testing.assert_close(w.cpu(), g[f"{case}_topk_weights"], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("T,E,k", [(1, 256, 8), (64, 256, 8), (512, 256, 8), (8192, 256, 8),
                                   (4096, 8, 2), (7, 5, 5), (300, 1000, 3), (33, 32, 1)])
def test_routing_matches_oracle(cuda_pkg, T, E, k):
    g = torch.Generator().manual_seed(20260319 + T)
    logits = torch.randn((T, E), generator=g)
    ids, w = cuda_pkg.moe.route_topk(logits.to(DEV), k)
    torch.cuda.synchronize()
    want_ids, want_w = moe_oracle.route_topk(logits, k)
    assert torch.equal(ids.cpu(), want_ids)
    torch.testing.assert_close(w.cpu(), want_w, rtol=1e-6, atol=1e-7)


def test_routing_ties_take_lower_index(cuda_pkg):
    logits = torch.zeros((3, 40))
    logits[1, 7] = 1.0
    logits[2, 35] = logits[2, 2] = 2.0
    ids, w = cuda_pkg.moe.route_topk(logits.to(DEV), 4)
    torch.cuda.synchronize()
    want_ids, want_w = moe_oracle.route_topk(logits, 4)
    assert ids.cpu().tolist() == [[0, 1, 2, 3], [7, 0, 1, 2], [2, 35, 0, 1]]
    assert torch.equal(ids.cpu(), want_ids)
    torch.testing.assert_close(w.cpu(), want_w, rtol=1e-6, atol=1e-7)


def test_router_logits(cuda_pkg):
    d = moe_oracle.moe_inputs(515, 4096, 128, 8, 20260319, with_router=True)
    got = cuda_pkg.moe.router_logits(d["x"].to(DEV), d["w_router"].to(DEV))
    torch.cuda.synchronize()
    want = moe_oracle.router_logits(d["x"], d["w_router"])
    torch.testing.assert_close(got.cpu(), want, rtol=1e-4, atol=1e-4)
    # expert assignment is bit-exact on identical logits
    ids, _ = cuda_pkg.moe.route_topk(got, 2)
    want_ids, _ = moe_oracle.route_topk(got.cpu(), 2)
    assert torch.equal(ids.cpu(), want_ids)


@pytest.mark.parametrize("case,experts", [("mixtral_like", 8), ("fine_grained", 32), ("routes", 256)])
def test_sorted_routes_golden_bit_exact(cuda_pkg, case, experts):
    g = load_golden("moe")
    r = check_routes(cuda_pkg, g[f"{case}_topk_ids"], g[f"{case}_topk_weights"], experts)
    assert torch.equal(r.sorted_token_ids.cpu(), g[f"{case}_sorted_token_ids"])
    assert torch.equal(r.sorted_weights.cpu(), g[f"{case}_sorted_weights"])
    assert torch.equal(r.sorted_expert_ids.cpu(), g[f"{case}_sorted_expert_ids"])
    assert torch.equal(r.num_valid_ids.cpu(), g[f"{case}_num_valid_ids"])


@pytest.mark.parametrize("T,E,k", [(1, 256, 8), (64, 256, 8), (512, 256, 8), (8192, 256, 8),
                                   (4096, 8, 2), (129, 3, 2), (1000, 1024, 4)])
def test_sorted_routes_random(cuda_pkg, T, E, k):
    g = torch.Generator().manual_seed(T * 31 + E)
    ids, w = moe_oracle.route_topk(torch.randn((T, E), generator=g), k)
    check_routes(cuda_pkg, ids, w, E)


@pytest.mark.parametrize("T,E,k", [(1, 256, 8), (100, 16, 4), (128, 8, 8), (2000, 64, 2)])
def test_compact_sort_for_expert_parallel_dispatch(cuda_pkg, T, E, k):
    """route_group = 1: experts back to back, one expert id per sorted row (both the one-CTA
    and the three-kernel form)."""
    g = torch.Generator().manual_seed(T + E)
    ids, w = moe_oracle.route_topk(torch.randn((T, E), generator=g), k)
    r = cuda_pkg.moe.build_sorted_routes(topk_ids=ids.to(DEV), topk_weights=w.to(DEV), experts=E, group=1)
    torch.cuda.synchronize()
    o = moe_oracle.build_sorted_routes(ids.numpy(), w.numpy(), E, group=1)
    got = (r.sorted_token_ids, r.sorted_weights, r.sorted_expert_ids, r.num_valid_ids,
           r.expert_offsets, r.expert_counts, r.route_pos)
    for a, b in zip(got, o):
        assert np.array_equal(a.cpu().numpy(), b)
    assert int(r.num_valid_ids[0]) == T * k


def test_sorted_routes_skewed_and_empty_experts(cuda_pkg):
    ids = torch.full((2100, 1), 3, dtype=torch.int32)  # every route on one expert, 3 chunks
    check_routes(cuda_pkg, ids, torch.ones((2100, 1)), 6)
    ids = torch.tensor([[5, 2]], dtype=torch.int32)
    check_routes(cuda_pkg, ids, torch.tensor([[0.75, 0.25]]), 8)


def moe_case(pkg, T, H, I, E, k, seed, with_router):
    d = moe_oracle.moe_inputs(T, H, I, E, seed, with_router=with_router)
    op = pkg.moe.FusedMoE(tokens=T, hidden=H, inter=I, experts=E, topk=k, device=DEV)
    x, w13, w2 = d["x"].to(DEV), d["w13"].to(DEV), d["w2"].to(DEV)
    if with_router:
        out = op.forward(x, w13, w2, w_router=d["w_router"].to(DEV))
    else:
        out = op.forward(x, w13, w2, logits=d["logits"].to(DEV))
    torch.cuda.synchronize()
    assert pkg.device_status() == 0
    # the oracle consumes the ids the device chose (bit-exact on identical logits, checked above)
    ids, w = op.topk_ids.cpu(), op.topk_weights.cpu()
    return d, op, out.cpu(), ids, w


@pytest.mark.parametrize("case,k,router", [("mixtral_like", 2, True), ("fine_grained", 8, False)])
def test_forward_golden(cuda_pkg, case, k, router):
    g = load_golden("moe")
    x, w13, w2 = g[f"{case}_x"], g[f"{case}_w13"], g[f"{case}_w2"]
    T, H = x.shape
    E, two_i, _ = w13.shape
    op = cuda_pkg.moe.FusedMoE(tokens=T, hidden=H, inter=two_i // 2, experts=E, topk=k, device=DEV)
    out = op.forward_routed(x.to(DEV), g[f"{case}_topk_ids"].to(DEV), g[f"{case}_topk_weights"].to(DEV),
                            w13.to(DEV), w2.to(DEV))
    torch.cuda.synchronize()
    assert cuda_pkg.device_status() == 0
    torch.testing.assert_close(out.cpu().float(), g[f"{case}_out"].float(), rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("T,H,I,E,k,router", [
    (1, 512, 256, 16, 4, False),        # one token
    (64, 1024, 512, 32, 8, False),      # a few rows per expert: weight-streaming orientation
    (200, 512, 384, 8, 2, True),        # ~50 rows per expert
    (400, 512, 256, 8, 2, True),        # 100 rows per expert: weight-major, MMA N sized per unit
    (1024, 512, 256, 8, 2, True),       # 256 rows per expert: token-major orientation
    (700, 384, 640, 4, 2, True),        # ragged tiles in every dimension
    (3300, 256, 384, 4, 1, True),       # ~825 rows per expert: CTA pairs, 256-row token tiles, ragged
    (1500, 320, 192, 2, 2, False),      # 1500 rows per expert, columns that do not fill a tile
])
def test_forward_matches_oracle(cuda_pkg, T, H, I, E, k, router):
    d, op, out, ids, w = moe_case(cuda_pkg, T, H, I, E, k, 20260319 + T, router)
    logits = moe_oracle.router_logits(d["x"], d["w_router"]) if router else d["logits"]
    want_ids, _ = moe_oracle.route_topk(op.logits.cpu() if router else logits, k)
    assert torch.equal(ids, want_ids)
    want = moe_oracle.moe_reference(d["x"], d["w13"], d["w2"], ids, w)
    torch.testing.assert_close(out.float(), want.float(), rtol=RTOL, atol=ATOL)


def test_grouped_gemm_rows_are_independent(cuda_pkg):
    """Rows of one expert's tile that belong to another expert (or are padding) must not
    leak into stored rows: permuting the tokens permutes the outputs."""
    d, op, out, ids, w = moe_case(cuda_pkg, 96, 256, 256, 8, 2, 99, False)
    perm = torch.randperm(96, generator=torch.Generator().manual_seed(4))
    op2 = cuda_pkg.moe.FusedMoE(tokens=96, hidden=256, inter=256, experts=8, topk=2, device=DEV)
    out2 = op2.forward(d["x"][perm].to(DEV), d["w13"].to(DEV), d["w2"].to(DEV), logits=d["logits"][perm].to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(out2.cpu(), out[perm])


@pytest.mark.parametrize("T,H,I,E,k", [(1, 512, 256, 16, 4), (200, 512, 384, 8, 2), (700, 384, 640, 4, 2)])
def test_single_call_forward_equals_the_launch_sequence(cuda_pkg, T, H, I, E, k):
    """lumen_b200_moe_forward (one C call, intermediates in one scratch buffer) launches the
    same kernels as FusedMoE: identical bits, from logits and from precomputed routing, with
    a scratch pointer that is not 256-byte aligned and holds garbage."""
    d, op, out, ids, w = moe_case(cuda_pkg, T, H, I, E, k, 20260319 + T, False)
    moe = cuda_pkg.moe
    need = moe.moe_forward_scratch_bytes(T, H, I, E, k)
    scratch = torch.full((need + 16,), 0xA5, dtype=torch.uint8, device=DEV)[16:]
    x, w13, w2 = d["x"].to(DEV), d["w13"].to(DEV), d["w2"].to(DEV)
    got = moe.moe_forward(x, w13, w2, topk=k, logits=d["logits"].to(DEV), scratch=scratch)
    got_routed = moe.moe_forward(x, w13, w2, topk=k, topk_ids=ids.to(DEV), topk_weights=w.to(DEV))
    torch.cuda.synchronize()
    assert cuda_pkg.device_status() == 0
    assert torch.equal(got.cpu(), out)
    assert torch.equal(got_routed.cpu(), out)
    with pytest.raises(cuda_pkg._cabi.LumenB200Error):
        moe.moe_forward(x, w13, w2, topk=k, logits=d["logits"].to(DEV), scratch=scratch[: need // 2])
    with pytest.raises(ValueError):
        moe.moe_forward(x, w13, w2, topk=k)
