"""B200 system for datasets/inference/attention: GQA flash-attention forward, bf16.

    python scripts/benchmark/bench_attn.py --backend lumen \
        --model-path <this file> --check-correctness

The harness contract has no `causal` argument (scripts/benchmark/backend_attn.py:131-134);
it is a constructor default here, True like ATTENTION_DEFAULTS
(scripts/benchmark/config.py:13-20).
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

flash_attn = _pkg.attention.flash_attn


class ModelNew(nn.Module):
    """forward(q [B,S,Hq,D], k [B,S,Hkv,D], v [B,S,Hkv,D]) -> [B,S,Hq,D] bf16."""

    def __init__(self, causal: bool = True):
        super().__init__()
        self.causal = bool(causal)
        self._out_cache: dict = {}

    def build_call(self, *, q_bshd: torch.Tensor, k_bshd: torch.Tensor, v_bshd: torch.Tensor):
        if q_bshd.dtype != torch.bfloat16:
            raise ValueError("B200 attention supports only bf16")
        if q_bshd.ndim != 4 or k_bshd.ndim != 4 or v_bshd.ndim != 4:
            raise ValueError("B200 attention expects q/k/v in [B,S,H,D] layout")
        q, k, v = q_bshd.contiguous(), k_bshd.contiguous(), v_bshd.contiguous()
        key = (tuple(q.shape), q.device, q.dtype)
        out = self._out_cache.get(key)
        if out is None:
            out = torch.empty_like(q)
            self._out_cache[key] = out
        causal = self.causal
        return lambda: flash_attn(q, k, v, causal=causal, out=out)

    def forward(self, q_bshd: torch.Tensor, k_bshd: torch.Tensor, v_bshd: torch.Tensor) -> torch.Tensor:
        return self.build_call(q_bshd=q_bshd, k_bshd=k_bshd, v_bshd=v_bshd)()


Model = ModelNew

batch_size = 8
num_q_heads = 32
num_kv_heads = 8
sequence_length = 4096
head_dim = 128


def get_inputs():
    g = torch.Generator().manual_seed(20260314)
    shape_q = (batch_size, sequence_length, num_q_heads, head_dim)
    shape_kv = (batch_size, sequence_length, num_kv_heads, head_dim)
    q = torch.randn(shape_q, generator=g, dtype=torch.float32).to(torch.bfloat16)
    k = torch.randn(shape_kv, generator=g, dtype=torch.float32).to(torch.bfloat16)
    v = torch.randn(shape_kv, generator=g, dtype=torch.float32).to(torch.bfloat16)
    return [q, k, v]


def get_init_inputs():
    return []


__all__ = ["ModelNew", "Model", "flash_attn", "get_inputs", "get_init_inputs"]
