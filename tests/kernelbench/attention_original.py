"""KernelBench-style original for the evaluator tests: causal grouped-query attention on
small bf16 tensors in the harness layout [B, S, H, D] (the contract of
prompts/kernelbench/2_attention.py of the reference: Model, get_inputs, get_init_inputs)."""
import math

import torch
import torch.nn as nn

B, S, HQ, HKV, D = 2, 384, 8, 2, 128


class Model(nn.Module):
    def forward(self, q_bshd, k_bshd, v_bshd):
        group = q_bshd.shape[2] // k_bshd.shape[2]
        q = q_bshd.float().permute(0, 2, 1, 3)
        k = k_bshd.float().permute(0, 2, 1, 3).repeat_interleave(group, dim=1)
        v = v_bshd.float().permute(0, 2, 1, 3).repeat_interleave(group, dim=1)
        scores = q @ k.transpose(-1, -2) / math.sqrt(q.shape[-1])
        keep = torch.ones(scores.shape[-2:], dtype=torch.bool, device=scores.device).tril()
        probs = torch.softmax(scores.masked_fill(~keep, float("-inf")), dim=-1)
        return (probs @ v).permute(0, 2, 1, 3).to(q_bshd.dtype)


def get_inputs():
    return [torch.randn(B, S, HQ, D, dtype=torch.bfloat16), torch.randn(B, S, HKV, D, dtype=torch.bfloat16),
            torch.randn(B, S, HKV, D, dtype=torch.bfloat16)]


def get_init_inputs():
    return []
