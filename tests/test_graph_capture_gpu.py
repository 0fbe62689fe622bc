"""The reference times every system under CUDA-graph replay
(scripts/benchmark/cudagraph_timer.py:33-55): each operator must be capturable (no host
synchronisation, no allocation that moves, no host read of device data) and a replay with new
input values in the same buffers must give the new result."""
from __future__ import annotations

import pytest
import torch

from conftest import ATOL, RTOL
from oracle import attention_oracle, gemm_oracle, moe_oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def capture(fn):
    fn()  # first call outside capture: sets kernel attributes, sizes scratch
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = fn()
    torch.cuda.synchronize()
    return graph, out


@pytest.mark.parametrize("m,n,k", [(16, 4096, 4096), (1024, 1024, 1024)])
def test_gemm_replays_with_new_inputs(cuda_pkg, m, n, k):
    a, b = gemm_oracle.gemm_inputs(m, n, k, 1)
    ad, bd = a.to(DEV), b.to(DEV)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=DEV)
    graph, _ = capture(lambda: cuda_pkg.gemm_pipeline_transposed_b(ad, bd, out))
    a2, b2 = gemm_oracle.gemm_inputs(m, n, k, 2)
    ad.copy_(a2.to(DEV))
    bd.copy_(b2.to(DEV))
    for _ in range(3):  # split-K counters must be left reusable by every replay
        graph.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(out.cpu().float(), gemm_oracle.gemm_reference(a2, b2).float(), rtol=RTOL, atol=ATOL)
    assert cuda_pkg.device_status() == 0


def test_attention_replays_with_new_inputs(cuda_pkg):
    q, k, v = attention_oracle.attention_inputs(2, 300, 4, 2, 128, 1)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    out = torch.empty_like(qd)
    graph, _ = capture(lambda: cuda_pkg.flash_attn(qd, kd, vd, causal=True, out=out))
    q2, k2, v2 = attention_oracle.attention_inputs(2, 300, 4, 2, 128, 2)
    qd.copy_(q2.to(DEV)); kd.copy_(k2.to(DEV)); vd.copy_(v2.to(DEV))
    graph.replay()
    torch.cuda.synchronize()
    want = attention_oracle.attention_reference(q2, k2, v2, causal=True)
    torch.testing.assert_close(out.cpu().float(), want.float(), rtol=RTOL, atol=ATOL)


def test_moe_forward_replays_with_new_routing(cuda_pkg):
    """Router, sort, gather, both grouped GEMMs and the combine in one graph: the expert loads
    change between replays and are never read on the host."""
    T, H, I, E, k = 256, 512, 256, 16, 4
    d = moe_oracle.moe_inputs(T, H, I, E, 3, with_router=False)
    op = cuda_pkg.moe.FusedMoE(tokens=T, hidden=H, inter=I, experts=E, topk=k, device=DEV)
    x, lg = d["x"].to(DEV), d["logits"].to(DEV)
    w13, w2 = d["w13"].to(DEV), d["w2"].to(DEV)
    graph, out = capture(lambda: op.forward(x, w13, w2, logits=lg))
    d2 = moe_oracle.moe_inputs(T, H, I, E, 4, with_router=False)
    logits2 = d2["logits"].clone()
    logits2[:, :3] += 5.0  # skew the loads: three hot experts
    x.copy_(d2["x"].to(DEV))
    lg.copy_(logits2.to(DEV))
    graph.replay()
    torch.cuda.synchronize()
    ids, w = moe_oracle.route_topk(logits2, k)
    assert torch.equal(op.topk_ids.cpu(), ids)
    want = moe_oracle.moe_reference(d2["x"], d["w13"], d["w2"], ids, w)
    torch.testing.assert_close(out.cpu().float(), want.float(), rtol=RTOL, atol=ATOL)
    assert cuda_pkg.device_status() == 0
