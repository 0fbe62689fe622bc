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


def flash_attn_packed(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seq_ptr: torch.Tensor,
                      max_seq_len: int, out: torch.Tensor | None = None, *, causal: bool = True,
                      scale: float | None = None) -> torch.Tensor:
    """Variable-length sequences packed along the token dimension: q [tokens,Hq,D],
    k/v [tokens,Hkv,D], seq_ptr [num_seqs+1] prefix sums.  Same positional arguments and
    checks as the reference's flash_attn(q, k, v, seq_ptr, max_seq_len, out=)
    (datasets/inference/attention/lumen/attn_06_inst_scheduling.py:108-165,2144-2193), without
    its restriction to 8 query heads and 1 KV head."""
    if q.ndim != 3 or k.ndim != 3 or v.ndim != 3:
        raise ValueError("q, k, and v must be rank-3 packed tensors shaped [tokens, heads, dim] "
                         f"(got q.ndim={q.ndim}, k.ndim={k.ndim}, v.ndim={v.ndim})")
    if q.shape[-1] != HEAD_DIM or k.shape[-1] != HEAD_DIM or v.shape[-1] != HEAD_DIM:
        raise ValueError(f"BF16 flash attention currently requires head_dim={HEAD_DIM} "
                         f"(got q={q.shape[-1]}, k={k.shape[-1]}, v={v.shape[-1]})")
    if q.shape[0] != k.shape[0] or q.shape[0] != v.shape[0]:
        raise ValueError("q, k, and v must have the same token dimension "
                         f"(got {q.shape[0]}, {k.shape[0]}, {v.shape[0]})")
    if k.shape[1] != v.shape[1]:
        raise ValueError(f"k and v must have the same number of KV heads (got {k.shape[1]}, {v.shape[1]})")
    if q.shape[1] == 0 or k.shape[1] == 0:
        raise ValueError("q_heads and kv_heads must be nonzero")
    if q.shape[1] % k.shape[1] != 0:
        raise ValueError(f"q_heads must be divisible by kv_heads (got {q.shape[1]} and {k.shape[1]})")
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise TypeError(f"q, k, and v must be torch.bfloat16 (got q={q.dtype}, k={k.dtype}, v={v.dtype})")
    if q.device.type != "cuda" or k.device.type != "cuda" or v.device.type != "cuda":
        raise ValueError(f"q, k, and v must be CUDA tensors (got q={q.device}, k={k.device}, v={v.device})")
    if q.device != k.device or q.device != v.device:
        raise ValueError(f"q, k, and v must be on the same device (got {q.device}, {k.device}, {v.device})")
    if not q.is_contiguous() or not k.is_contiguous() or not v.is_contiguous():
        raise ValueError("q, k, and v must be contiguous")
    if not isinstance(seq_ptr, torch.Tensor):
        raise TypeError("seq_ptr must be torch.Tensor")
    if seq_ptr.ndim != 1:
        raise ValueError(f"seq_ptr must be rank-1 (got seq_ptr.ndim={seq_ptr.ndim})")
    if seq_ptr.numel() < 2:
        raise ValueError("seq_ptr must have at least two elements")
    if seq_ptr.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"seq_ptr must be torch.int32 or torch.int64 (got {seq_ptr.dtype})")
    if seq_ptr.device != q.device:
        raise ValueError(f"seq_ptr must be on {q.device} (got {seq_ptr.device})")
    if not seq_ptr.is_contiguous():
        raise ValueError("seq_ptr must be contiguous")
    if not isinstance(max_seq_len, int) or max_seq_len < 0:
        raise ValueError(f"max_seq_len must be a non-negative int (got {max_seq_len!r})")
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
    total_tokens = q.shape[0]
    if total_tokens > 0 and max_seq_len > total_tokens:
        raise ValueError(f"max_seq_len ({max_seq_len}) cannot exceed total_tokens ({total_tokens})")
    if total_tokens == 0 or max_seq_len == 0:
        return out
    seq_ptr_i32 = seq_ptr if seq_ptr.dtype == torch.int32 else seq_ptr.to(torch.int32)
    if scale is None:
        scale = 1.0 / math.sqrt(HEAD_DIM)
    with _cabi.on_device(q.device):
        rc = _cabi.load().lumen_b200_fa_fwd_varlen_bf16(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), seq_ptr_i32.data_ptr(),
            seq_ptr.numel() - 1, total_tokens, int(max_seq_len), q.shape[1], k.shape[1], HEAD_DIM,
            float(scale), 1 if causal else 0, torch.cuda.current_stream(q.device).cuda_stream)
    _cabi.check("lumen_b200_fa_fwd_varlen_bf16", rc)
    return out
