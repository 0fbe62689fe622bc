"""KernelBench-style original for the evaluator tests: C = A B^T on small bf16 matrices
(the layout of prompts/kernelbench/1_gemm.py of the reference: Model, get_inputs,
get_init_inputs at module level; inputs drawn from torch's global generator, which the
evaluator seeds per trial)."""
import torch
import torch.nn as nn

M, N, K = 512, 640, 384


class Model(nn.Module):
    def forward(self, a_mk, b_nk):
        return torch.matmul(a_mk, b_nk.T)


def get_inputs():
    return [torch.randn(M, K, dtype=torch.bfloat16), torch.randn(N, K, dtype=torch.bfloat16)]


def get_init_inputs():
    return []
