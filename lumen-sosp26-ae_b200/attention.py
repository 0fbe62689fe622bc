"""Host side of the GQA flash-attention forward (bf16, head dimension 128).

`flash_attn` takes the harness layout q [B,S,Hq,D], k/v [B,S,Hkv,D]
(scripts/benchmark/backend_attn.py:74-94 of the reference) and validates like the
reference's host wrapper (datasets/inference/attention/lumen/attn_06_inst_scheduling.py:
2144-2193: TypeError for a wrong dtype of `out`, ValueError for shapes/devices), then calls
lumen_b200_fa_fwd_bf16 on the current CUDA stream.
"""
from __future__ import annotations

import math

import torch

from . import _cabi

HEAD_DIM = 128


def flash_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, causal: bool = True,
               scale: float | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.dtype != torch.bfloat16:
            raise TypeError(f"{name} must be torch.bfloat16 (got {t.dtype})")
        if t.ndim != 4:
            raise ValueError(f"{name} must be [B,S,H,D] (got shape {tuple(t.shape)})")
        if not t.is_cuda:
            raise ValueError("flash_attn needs CUDA tensors: there is no CPU path")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    B, S, Hq, D = q.shape
    if D != HEAD_DIM:
        raise ValueError(f"head_dim must be {HEAD_DIM} (got {D})")
    if k.shape != v.shape:
        raise ValueError("k and v must have identical shape")
    if k.shape[0] != B or k.shape[1] != S or k.shape[3] != D:
        raise ValueError("q and k must share batch, sequence length and head_dim")
    Hkv = k.shape[2]
    if Hq % Hkv != 0:
        raise ValueError(f"query heads ({Hq}) must be divisible by KV heads ({Hkv})")
    if k.device != q.device or v.device != q.device:
        raise ValueError("q, k and v must be on one device")
    if out is None:
        out = torch.empty_like(q)
    else:
        if out.shape != q.shape:
            raise ValueError(f"out must have shape {q.shape} (got {out.shape})")
        if out.dtype != torch.bfloat16:
            raise TypeError(f"out must be torch.bfloat16 (got {out.dtype})")
        if out.device != q.device:
            raise ValueError(f"out must be on {q.device} (got {out.device})")
        if not out.is_contiguous():
            raise ValueError("out must be contiguous")
    if B == 0 or S == 0:
        return out
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    with _cabi.on_device(q.device):
        rc = _cabi.load().lumen_b200_fa_fwd_bf16(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, S, Hq, Hkv, D,
            float(scale), 1 if causal else 0, torch.cuda.current_stream(q.device).cuda_stream)
    _cabi.check("lumen_b200_fa_fwd_bf16", rc)
    return out
