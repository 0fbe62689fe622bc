"""Oracle for the GQA attention forward  O = softmax(scale * Q K^T + mask) V.

Follows `Model.forward` of prompts/kernelbench/2_attention.py:11-50 (explicit fp32
scores, -inf above the diagonal, softmax, fp32 P*V, bf16 out; KV head of query head
h is h // (Hq // Hkv), the `repeat_interleave` at :29-32) generalised to any Hq/Hkv
and to the non-causal case, as the harness oracle `_attention_reference`
(scripts/benchmark/backend_attn.py:197-211) is.  Works one (batch, kv-head) group at
a time and in query chunks so that the [S,S] fp32 score matrix is never held whole.
"""
from __future__ import annotations

import math

import torch

SM_SCALE_D128 = 0.08838834764831843  # prompts/kernelbench/2_attention.py:38


def attention_reference(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, causal: bool,
                        scale: float | None = None, q_chunk: int = 1024) -> torch.Tensor:
    """q [B,S,Hq,D], k/v [B,S,Hkv,D] -> bf16 [B,S,Hq,D]."""
    B, S, Hq, D = q.shape
    Hkv = k.shape[2]
    if Hq % Hkv != 0:
        raise ValueError(f"query heads ({Hq}) must be divisible by KV heads ({Hkv})")
    groups = Hq // Hkv
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    out = torch.empty((B, S, Hq, D), dtype=torch.bfloat16)
    for b in range(B):
        for hk in range(Hkv):
            kf = k[b, :, hk, :].to(torch.float32)  # [S,D]
            vf = v[b, :, hk, :].to(torch.float32)
            for g in range(groups):
                h = hk * groups + g
                for s0 in range(0, S, q_chunk):
                    s1 = min(S, s0 + q_chunk)
                    qf = q[b, s0:s1, h, :].to(torch.float32) * scale
                    kv_end = s1 if causal else S
                    scores = qf @ kf[:kv_end].transpose(0, 1)  # [chunk, kv_end]
                    if causal:
                        rows = torch.arange(s0, s1).unsqueeze(1)
                        cols = torch.arange(0, kv_end).unsqueeze(0)
                        scores = scores.masked_fill(cols > rows, float("-inf"))
                    probs = torch.softmax(scores, dim=-1)
                    out[b, s0:s1, h, :] = (probs @ vf[:kv_end]).to(torch.bfloat16)
    return out


def attention_inputs(B: int, S: int, Hq: int, Hkv: int, D: int, seed: int):
    """q, k, v ~ N(0,1) bf16, drawn in that order from one CPU generator
    (scripts/benchmark/backend_attn.py:74-94 draws them in the same order)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    q = torch.randn((B, S, Hq, D), generator=g, dtype=torch.float32).to(torch.bfloat16)
    k = torch.randn((B, S, Hkv, D), generator=g, dtype=torch.float32).to(torch.bfloat16)
    v = torch.randn((B, S, Hkv, D), generator=g, dtype=torch.float32).to(torch.bfloat16)
    return q, k, v
