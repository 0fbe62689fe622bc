"""GPU parity of the fused MoE forward at the full benchmark sizes against the CPU oracle.

  Mixtral-like:  T=4096, H=4096, I=14336, E=8, top-2, router matrix inside the operator
  fine-grained:  E=256, top-8, H=7168, I=2048, T in {1, 64, 512, 8192}, logits given

The oracle loops over experts in fp32 on the host, so it is run on a sample of token rows
(all of a token's experts are needed for its output row) and only the experts those tokens
touch are copied to the host; besides whole output rows, single rows of the second grouped
GEMM's result are checked at the edges of the experts' row tiles (first and last row, rows
127/128/255/256 of an expert), where a tiling mistake would show.  Expert ids are compared
bit-exactly on identical logits, and the smallest top-k gap of each seed is printed.
The reference checks on the full workload too: scripts/benchmark/backend_moe.py:422-466.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import ATOL, RTOL
from oracle import moe_oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
SEED = 20260319


def _device_weights(E, H, I, seed):
    """w13 [E,2I,H], w2 [E,H,I] ~ N(0, 0.02) bf16, drawn on the device one expert at a time
    (21 GiB for the 256-expert configuration: generating them on the host would take minutes)."""
    g = torch.Generator(device=DEV).manual_seed(seed + 17)
    w13 = torch.empty((E, 2 * I, H), device=DEV, dtype=torch.bfloat16)
    w2 = torch.empty((E, H, I), device=DEV, dtype=torch.bfloat16)
    for e in range(E):
        w13[e] = (torch.randn((2 * I, H), device=DEV, dtype=torch.float32, generator=g) * 0.02).to(torch.bfloat16)
        w2[e] = (torch.randn((H, I), device=DEV, dtype=torch.float32, generator=g) * 0.02).to(torch.bfloat16)
    return w13, w2


def _oracle_rows(x_rows, ids_rows, w_rows, w13, w2):
    """moe_oracle.moe_reference on a few token rows: only the experts they touch are copied
    to the host, under compact expert numbers."""
    touched = sorted(set(ids_rows.reshape(-1).tolist()))
    remap = {e: i for i, e in enumerate(touched)}
    idx = torch.tensor(touched, device=DEV)
    w13_c = w13.index_select(0, idx).cpu()
    w2_c = w2.index_select(0, idx).cpu()
    ids_c = torch.tensor([[remap[int(e)] for e in row] for row in ids_rows.tolist()], dtype=torch.int32)
    return moe_oracle.moe_reference(x_rows, w13_c, w2_c, ids_c, w_rows)


def _edge_routes(counts, offsets, rng, per_expert=3, experts=6):
    """Sorted positions at the edges of row tiles of a few experts (largest, smallest
    non-empty, random ones)."""
    nz = np.nonzero(counts)[0]
    if nz.size == 0:
        return []
    picks = {int(nz[np.argmax(counts[nz])]), int(nz[np.argmin(counts[nz])])}
    picks.update(int(e) for e in rng.choice(nz, size=min(experts, nz.size), replace=False))
    pos = []
    for e in sorted(picks):
        n = int(counts[e])
        local = {0, n - 1, n // 2}
        for edge in (63, 64, 127, 128, 255, 256):
            if edge < n:
                local.add(edge)
        local = sorted(local)
        if len(local) > per_expert + 4:
            local = local[:2] + local[-(per_expert + 2):]
        pos.extend((e, int(offsets[e]) + r) for r in local)
    return pos


def _check_forward(pkg, T, H, I, E, k, w13, w2, *, router, n_tokens):
    g = torch.Generator().manual_seed(SEED + T)
    x = torch.randn((T, H), generator=g, dtype=torch.float32).to(torch.bfloat16)
    op = pkg.moe.FusedMoE(tokens=T, hidden=H, inter=I, experts=E, topk=k, device=DEV)
    xd = x.to(DEV)
    if router:
        gw = torch.Generator().manual_seed(SEED + 17)
        w_router = (torch.randn((E, H), generator=gw, dtype=torch.float32) * 0.02).to(torch.bfloat16)
        out = op.forward(xd, w13, w2, w_router=w_router.to(DEV))
        torch.cuda.synchronize()
        logits = op.logits.cpu()
        torch.testing.assert_close(logits, moe_oracle.router_logits(x, w_router), rtol=1e-4, atol=1e-4)
    else:
        logits = torch.randn((T, E), generator=g, dtype=torch.float32)
        out = op.forward(xd, w13, w2, logits=logits.to(DEV))
        torch.cuda.synchronize()
    assert pkg.device_status() == 0
    print(f"\nT={T} E={E} top-{k}: smallest gap among the top {k + 1} logits of any token = "
          f"{moe_oracle.min_topk_gap(logits, k):.3e}")

    # expert assignment and weights: bit-exact ids on identical logits
    ids, w = op.topk_ids.cpu(), op.topk_weights.cpu()
    want_ids, want_w = moe_oracle.route_topk(logits, k)
    assert torch.equal(ids, want_ids)
    torch.testing.assert_close(w, want_w, rtol=1e-6, atol=1e-7)
    # the permutation the expert GEMMs consumed
    r = op.routes
    o = moe_oracle.build_sorted_routes(ids.numpy(), w.numpy(), E)
    got = (r.sorted_token_ids, r.sorted_weights, r.sorted_expert_ids, r.num_valid_ids,
           r.expert_offsets, r.expert_counts, r.route_pos)
    for a, b in zip(got, o):
        assert np.array_equal(a.cpu().numpy(), b)

    rng = np.random.default_rng(T)
    # whole output rows of sampled tokens
    tok = np.sort(rng.choice(T, size=min(n_tokens, T), replace=False))
    tok_t = torch.from_numpy(tok)
    want = _oracle_rows(x[tok_t], ids[tok_t], w[tok_t], w13, w2)
    torch.testing.assert_close(out.cpu()[tok_t].float(), want.float(), rtol=RTOL, atol=ATOL)

    # single rows of y = (silu(x W1^T) * (x W3^T)) W2^T at tile edges of a few experts
    counts, offsets = o[5], o[4]
    sorted_ids = o[0]
    by_expert: dict[int, list[int]] = {}
    for e, pos in _edge_routes(counts, offsets, rng):
        by_expert.setdefault(e, []).append(pos)
    y = op.y
    for e, positions in by_expert.items():
        toks = torch.tensor([int(sorted_ids[p]) & 0xFFFFFF for p in positions])
        n = len(positions)
        want_rows = moe_oracle.moe_reference(x[toks], w13[e:e + 1].cpu(), w2[e:e + 1].cpu(),
                                             torch.zeros((n, 1), dtype=torch.int32), torch.ones((n, 1)))
        got_rows = y[torch.tensor(positions, device=DEV)].cpu()
        torch.testing.assert_close(got_rows.float(), want_rows.float(), rtol=RTOL, atol=ATOL)


@pytest.fixture(scope="module")
def fine_grained_weights():
    w = _device_weights(256, 7168, 2048, SEED)
    yield w
    del w
    torch.cuda.empty_cache()


def test_mixtral_like_full_size(cuda_pkg):
    T, H, I, E, k = 4096, 4096, 14336, 8, 2
    w13, w2 = _device_weights(E, H, I, SEED)
    _check_forward(cuda_pkg, T, H, I, E, k, w13, w2, router=True, n_tokens=48)
    del w13, w2
    torch.cuda.empty_cache()


@pytest.mark.parametrize("T,n_tokens", [(1, 1), (64, 4), (512, 4), (8192, 6)])
def test_fine_grained_full_size(cuda_pkg, fine_grained_weights, T, n_tokens):
    w13, w2 = fine_grained_weights
    _check_forward(cuda_pkg, T, 7168, 2048, 256, 8, w13, w2, router=False, n_tokens=n_tokens)
