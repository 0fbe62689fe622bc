"""B200 system for datasets/inference/gemm: C[M,N] = A[M,K] * B[N,K]^T in bf16.

Loaded by the reference harness like any other system directory
(scripts/benchmark/backends.py:95-143 looks for ModelNew, then Model, then
kernel_function; scripts/benchmark/backend_gemm.py:100-103 uses build_call when present):

    python scripts/benchmark/bench_gemm.py --backend lumen \
        --model-path <this file> --check-correctness
"""
from __future__ import annotations

import importlib.util
import os
from pathlib import Path

import torch
import torch.nn as nn


def _find_loader() -> Path:
    """_loader.py sits two directories above this file.  An evaluator that executes this
    file's source text instead of importing it by path (no usable __file__, the
    KernelBench way: python/lumen/harness/datasets/kernelbench/evaluator.py:158-167) names
    the directory that contains the package in the environment variable LUMEN_B200_ROOT."""
    places = []
    here = globals().get("__file__")
    if here:
        places += [p / "_loader.py" for p in list(Path(here).resolve().parents)[2:3]]
    if os.environ.get("LUMEN_B200_ROOT"):
        places.append(Path(os.environ["LUMEN_B200_ROOT"]) / "lumen-sosp26-ae_b200" / "datasets" / "inference" / "_loader.py")
    for place in places:
        if place.is_file():
            return place
    raise ImportError("cannot locate the lumen-sosp26-ae_b200 package: import this file by its path "
                      "inside the package, or set LUMEN_B200_ROOT to the directory that contains the package")


_spec = importlib.util.spec_from_file_location("_b200_dataset_loader", _find_loader())
_loader = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(_loader)
_pkg = _loader.load_b200_package()

kernel_function = _pkg.gemm_pipeline_transposed_b


class ModelNew(nn.Module):
    """forward(a_mk [M,K], b_nk [N,K]) -> [M,N], same dtype (bf16), fp32 accumulation."""

    def __init__(self):
        super().__init__()
        self._out_cache: dict = {}

    def build_call(self, *, a_mk: torch.Tensor, b_nk: torch.Tensor):
        """Zero-argument closure for CUDA-graph capture: the output buffer is allocated
        here, once, so that replays write to a fixed address."""
        key = (a_mk.shape[0], b_nk.shape[0], a_mk.device)
        out = self._out_cache.get(key)
        if out is None:
            out = torch.empty((a_mk.shape[0], b_nk.shape[0]), dtype=torch.bfloat16, device=a_mk.device)
            self._out_cache[key] = out
        # first call outside capture: sizes the split-K scratch for this shape
        kernel_function(a_mk, b_nk, out)
        return lambda: kernel_function(a_mk, b_nk, out)

    def forward(self, a_mk: torch.Tensor, b_nk: torch.Tensor) -> torch.Tensor:
        return kernel_function(a_mk, b_nk)


Model = ModelNew

M = 4096
K = 4096
N = 4096


def get_inputs():
    """Seeded stand-ins with the harness' distribution (A, B ~ N(0,1), bf16)."""
    g = torch.Generator().manual_seed(20260312)
    a = torch.randn((M, K), generator=g, dtype=torch.float32).to(torch.bfloat16)
    b = torch.randn((N, K), generator=g, dtype=torch.float32).to(torch.bfloat16)
    return [a, b]


def get_init_inputs():
    return []


__all__ = ["ModelNew", "Model", "kernel_function", "get_inputs", "get_init_inputs"]
