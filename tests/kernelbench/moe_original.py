"""KernelBench-style original for the evaluator tests: routed SiLU-gated MoE with per-128
block scales on small tensors, in the argument order of the reference's MoE task
(prompts/kernelbench/3_fused_moe.py: input_q, w1_q, w2_q, topk_weights, topk_ids,
input_scale, fc1_scale, fc2_scale).  Scales differ from 1 so that a candidate that caches
dequantised weights by the identity of the codes alone gives stale results."""
import torch
import torch.nn as nn
import torch.nn.functional as F

T, DIM, INTER, E, K, BLK = 192, 512, 256, 8, 2, 128


def _expand(scale, rows, cols):
    return scale.float().view(rows // BLK, cols // BLK).repeat_interleave(BLK, 0).repeat_interleave(BLK, 1)


class Model(nn.Module):
    def forward(self, input_q, w1_q, w2_q, topk_weights, topk_ids, input_scale, fc1_scale, fc2_scale):
        # every expert on every token, weighted by the routing (zero where the expert was not
        # chosen): no data-dependent shapes, so the evaluator can capture it in a CUDA graph
        x = input_q.float() * input_scale.float().repeat_interleave(BLK, dim=1)
        out = torch.zeros_like(x)
        for e in range(w1_q.shape[0]):
            w1 = w1_q[e].float() * _expand(fc1_scale[e], 2 * INTER, DIM)
            w2 = w2_q[e].float() * _expand(fc2_scale[e], DIM, INTER)
            gate, up = (x @ w1.T).split(INTER, dim=-1)
            y = (F.silu(gate) * up) @ w2.T
            route_weight = (topk_weights.float() * (topk_ids == e)).sum(dim=1, keepdim=True)
            out += y * route_weight
        return out.to(torch.bfloat16)


def get_inputs():
    x = torch.randn(T, DIM, dtype=torch.bfloat16)
    w1 = (torch.randn(E, 2 * INTER, DIM) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, DIM, INTER) * 0.02).to(torch.bfloat16)
    tv, ti = torch.topk(torch.randn(T, E), k=K, dim=-1)
    return [x, w1, w2, torch.softmax(tv, dim=-1), ti.to(torch.int32),
            0.5 + torch.rand(T, DIM // BLK), 0.5 + torch.rand(E, (2 * INTER // BLK) * (DIM // BLK)),
            0.5 + torch.rand(E, (DIM // BLK) * (INTER // BLK))]


def get_init_inputs():
    return []
