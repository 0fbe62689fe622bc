"""The CPU oracle replays the fixtures that tests/golden/make_golden.py produced by
running the reference's own functions (GEMM Model, _attention_reference, the attention
Model, _moe_reference, _build_sorted_routes, torch.topk + softmax routing)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import attention_oracle, gemm_oracle, moe_oracle


@pytest.mark.parametrize("case", ["small", "ragged"])
def test_gemm_oracle_matches_reference_model(case):
    g = load_golden("gemm")
    out = gemm_oracle.gemm_reference(g[f"{case}_a"], g[f"{case}_b"])
    # the reference Model rounds a bf16 CPU matmul; at most one bf16 ulp apart
    torch.testing.assert_close(out.float(), g[f"{case}_out"].float(), rtol=1e-2, atol=1e-2)
    assert (out == g[f"{case}_out"]).float().mean() > 0.99


@pytest.mark.parametrize("case", ["gqa", "mqa"])
@pytest.mark.parametrize("causal", [True, False])
def test_attention_oracle_matches_harness_reference(case, causal):
    g = load_golden("attention")
    out = attention_oracle.attention_reference(g[f"{case}_q"], g[f"{case}_k"], g[f"{case}_v"],
                                               causal=causal, q_chunk=32)
    want = g[f"{case}_out_{'causal' if causal else 'full'}"]
    torch.testing.assert_close(out.float(), want.float(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("case", ["gqa", "mqa"])
def test_attention_oracle_matches_prompt_model(case):
    g = load_golden("attention")
    out = attention_oracle.attention_reference(
        g[f"{case}_q"], g[f"{case}_k"], g[f"{case}_v"], causal=True,
        scale=attention_oracle.SM_SCALE_D128, q_chunk=16)
    torch.testing.assert_close(out.float(), g[f"{case}_out_model_causal"].float(), rtol=1e-2, atol=1e-2)


def test_attention_oracle_chunking_is_invisible():
    q, k, v = attention_oracle.attention_inputs(1, 70, 2, 1, 128, 7)
    a = attention_oracle.attention_reference(q, k, v, causal=True, q_chunk=7)
    b = attention_oracle.attention_reference(q, k, v, causal=True, q_chunk=1024)
    torch.testing.assert_close(a.float(), b.float(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("case,k", [("mixtral_like", 2), ("fine_grained", 8)])
def test_moe_routing_bit_exact(case, k):
    g = load_golden("moe")
    ids, w = moe_oracle.route_topk(g[f"{case}_logits"], k)
    assert torch.equal(ids, g[f"{case}_topk_ids"])
    assert torch.equal(w, g[f"{case}_topk_weights"])


def test_moe_router_logits_oracle():
    g = load_golden("moe")
    logits = moe_oracle.router_logits(g["mixtral_like_x"], g["mixtral_like_w_router"])
    torch.testing.assert_close(logits, g["mixtral_like_logits"], rtol=0, atol=0)


@pytest.mark.parametrize("case,experts", [("mixtral_like", 8), ("fine_grained", 32), ("routes", 256)])
def test_sorted_routes_bit_exact(case, experts):
    g = load_golden("moe")
    o = moe_oracle.build_sorted_routes(g[f"{case}_topk_ids"].numpy(), g[f"{case}_topk_weights"].numpy(), experts)
    assert np.array_equal(o[0], g[f"{case}_sorted_token_ids"].numpy())
    assert np.array_equal(o[1], g[f"{case}_sorted_weights"].numpy())
    assert np.array_equal(o[2], g[f"{case}_sorted_expert_ids"].numpy())
    assert np.array_equal(o[3], g[f"{case}_num_valid_ids"].numpy())
    # derived tables are consistent with the reference arrays
    off, cnt, pos = o[4], o[5], o[6]
    assert off[-1] == o[3][0]
    ids = g[f"{case}_topk_ids"].numpy()
    T, k = ids.shape
    for r in range(T * k):
        packed = o[0][pos[r]]
        assert packed & 0xFFFFFF == r // k and packed >> 24 == r % k
    assert np.array_equal(cnt, np.bincount(ids.reshape(-1), minlength=experts))


def test_sorted_routes_edge_cases():
    # a single token, and every route on one expert
    ids = np.array([[5, 2]], dtype=np.int32)
    w = np.array([[0.75, 0.25]], dtype=np.float32)
    o = moe_oracle.build_sorted_routes(ids, w, 8)
    assert o[3].tolist() == [64, 1]
    assert o[0][0] == (1 << 24) | 0 and o[0][32] == 0
    assert o[2][:3].tolist() == [2, 5, -1]
    ids = np.full((70, 1), 3, dtype=np.int32)
    o = moe_oracle.build_sorted_routes(ids, np.ones((70, 1), np.float32), 4)
    assert o[3][0] == 96 and o[5].tolist() == [0, 0, 0, 70]
    assert o[0][69] == 69 and o[0][70] == (1 << 24) | 70


@pytest.mark.parametrize("case", ["mixtral_like", "fine_grained"])
def test_moe_oracle_matches_reference(case):
    g = load_golden("moe")
    out = moe_oracle.moe_reference(g[f"{case}_x"], g[f"{case}_w13"], g[f"{case}_w2"],
                                   g[f"{case}_topk_ids"], g[f"{case}_topk_weights"])
    assert torch.equal(out, g[f"{case}_out"])
