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
from ._checks import Operand, check_operands, check_output, require

HEAD_DIM = 128


def _check_heads(op: str, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> int:
    """Head geometry shared by both layouts (heads are dimension -2, the head size -1)."""
    require(tuple(k.shape) == tuple(v.shape), op, f"k is {tuple(k.shape)} but v is {tuple(v.shape)}")
    require(q.shape[-1] == HEAD_DIM and k.shape[-1] == HEAD_DIM, op,
            f"the kernel is built for a head size of {HEAD_DIM}; q has {q.shape[-1]}, k has {k.shape[-1]}")
    hq, hkv = q.shape[-2], k.shape[-2]
    require(hq > 0 and hkv > 0 and hq % hkv == 0, op,
            f"{hq} query heads cannot share {hkv} KV heads evenly")
    return hkv


def flash_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, causal: bool = True,
               scale: float | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    op = "flash_attn"
    dev = check_operands(op, [Operand("q", q, "[B, S, Hq, D]"), Operand("k", k, "[B, S, Hkv, D]"),
                              Operand("v", v, "[B, S, Hkv, D]")], dtype=torch.bfloat16, dtype_error=TypeError)
    B, S, Hq, D = q.shape
    Hkv = _check_heads(op, q, k, v)
    require(k.shape[0] == B and k.shape[1] == S, op,
            f"q is {tuple(q.shape)} and k is {tuple(k.shape)}: batch and sequence length must agree")
    out = check_output(op, out, tuple(q.shape), dev, dtype=torch.bfloat16, dtype_error=TypeError)
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
    k/v [tokens,Hkv,D], seq_ptr [num_seqs+1] prefix sums.  Same positional arguments and the
    same exception type per kind of mistake as the reference's flash_attn(q, k, v, seq_ptr,
    max_seq_len, out=) (datasets/inference/attention/lumen/attn_06_inst_scheduling.py:108-165,
    2144-2193), without its restriction to 8 query heads and 1 KV head."""
    op = "flash_attn_packed"
    dev = check_operands(op, [Operand("q", q, "[tokens, Hq, D]"), Operand("k", k, "[tokens, Hkv, D]"),
                              Operand("v", v, "[tokens, Hkv, D]")], dtype=torch.bfloat16, dtype_error=TypeError)
    _check_heads(op, q, k, v)
    total_tokens = q.shape[0]
    require(k.shape[0] == total_tokens, op, f"q holds {total_tokens} tokens, k and v hold {k.shape[0]}")
    require(isinstance(seq_ptr, torch.Tensor), op, "seq_ptr is not a torch.Tensor", TypeError)
    require(seq_ptr.dtype in (torch.int32, torch.int64), op,
            f"seq_ptr holds {seq_ptr.dtype}; prefix sums are int32 or int64", TypeError)
    require(seq_ptr.ndim == 1 and seq_ptr.numel() >= 2 and seq_ptr.is_contiguous(), op,
            f"seq_ptr is the dense 1-D list of num_seqs + 1 prefix sums, got shape {tuple(seq_ptr.shape)}")
    require(seq_ptr.device == dev, op, f"seq_ptr lives on {seq_ptr.device}, the tokens on {dev}")
    require(isinstance(max_seq_len, int) and max_seq_len >= 0, op,
            f"max_seq_len is the longest sequence's length (an int >= 0), got {max_seq_len!r}")
    out = check_output(op, out, tuple(q.shape), dev, dtype=torch.bfloat16, dtype_error=TypeError)
    require(total_tokens == 0 or max_seq_len <= total_tokens, op,
            f"the longest sequence ({max_seq_len}) cannot be longer than all {total_tokens} packed tokens")
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
