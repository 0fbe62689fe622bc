"""Oracle for C = A * B^T (bf16 inputs, fp32 accumulation, bf16 output).

Follows `Model.forward` (prompts/kernelbench/1_gemm.py:5-10: torch.matmul(A, B.T)) and
the harness check (scripts/benchmark/backend_gemm.py:135-137) of the reference, with
the accumulation done in fp32 as the reference's kernels do
(datasets/inference/gemm/lumen/amdgpu_gemm.py:247-248: bf16 MFMA into fp32).
"""
from __future__ import annotations

import torch


def gemm_fp32(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """fp32 result of A[M,K] @ B[N,K]^T; inputs are upcast first."""
    return a.to(torch.float32) @ b.to(torch.float32).transpose(0, 1)


def gemm_reference(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """bf16 (round-to-nearest-even) result of the fp32-accumulated product."""
    return gemm_fp32(a, b).to(torch.bfloat16)


def gemm_inputs(m: int, n: int, k: int, seed: int, b_std: float = 1.0):
    """Seeded stand-in inputs: A ~ N(0,1), B ~ N(0, b_std), drawn in fp32 on the CPU
    generator and cast to bf16 (scripts/benchmark/backend_gemm.py:58-69 draws A then B
    from one generator; its generator lives on the device, so the streams differ)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    a = torch.randn((m, k), generator=g, dtype=torch.float32).to(torch.bfloat16)
    b = (torch.randn((n, k), generator=g, dtype=torch.float32) * b_std).to(torch.bfloat16)
    return a, b
