#!/usr/bin/env python3
"""Attention benchmark (GQA flash-attention forward, bf16, [B,S,H,D]), CUDA-graph timing.

Same flags and JSONL record as the reference's scripts/benchmark/bench_attn.py (q, k, v drawn
in that order per sequence length from one device generator, backend_attn.py:60-95; check
against scaled_dot_product_attention with its tolerance, :45-48,197-211), plus --no-causal
(the reference hard-wires causal=True, config.py:13-20) and a `torch` backend (SDPA)."""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import torch
import torch.nn.functional as F

sys.path.insert(0, str(Path(__file__).resolve().parent))
import core  # noqa: E402

TOL = {"bf16": 2e-2, "fp16": 1e-2}
SEQ_LENS = [1024, 2048, 4096, 8192, 16384]


def sdpa(q, k, v, causal: bool):
    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    if qt.shape[1] != kt.shape[1]:
        if qt.shape[1] % kt.shape[1]:
            raise ValueError(f"query heads ({qt.shape[1]}) must be divisible by KV heads ({kt.shape[1]})")
        g = qt.shape[1] // kt.shape[1]
        kt, vt = kt.repeat_interleave(g, dim=1), vt.repeat_interleave(g, dim=1)
    return F.scaled_dot_product_attention(qt, kt, vt, is_causal=causal).transpose(1, 2).contiguous()


class TorchAttention(torch.nn.Module):
    def __init__(self, causal=True):
        super().__init__()
        self.causal = causal

    def forward(self, q, k, v):
        return sdpa(q, k, v, self.causal)


def attention_tflops(batch, heads, seq, dim, ms, causal) -> float:
    """The reference's conversion (scripts/table2/benchmark.py:274-285): 4*2*B*H*S^2*D,
    halved when causal."""
    flop = 4.0 * 2.0 * batch * heads * seq * seq * dim
    return (flop / 2.0 if causal else flop) / (ms / 1e3) / 1e12


def run(argv=None) -> list[dict]:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--backend", choices=["b200", "torch"], default="b200")
    p.add_argument("--seed", type=int, default=20260314)
    p.add_argument("--dtype", choices=["bf16"], default="bf16")
    p.add_argument("--seq-lens", type=int, nargs="+", default=SEQ_LENS)
    p.add_argument("--batch-size", type=int, default=16)
    p.add_argument("--num-q-heads", type=int, default=8)
    p.add_argument("--num-kv-heads", type=int, default=1)
    p.add_argument("--head-dim", type=int, default=128)
    p.add_argument("--no-causal", dest="causal", action="store_false")
    p.add_argument("--check-correctness", action="store_true")
    p.add_argument("--model-path", type=Path, default=None)
    core.add_timer_flags(p)
    a = p.parse_args(argv)

    torch.manual_seed(a.seed)
    dev, dtype = torch.device("cuda"), torch.bfloat16
    gen = torch.Generator(device=dev).manual_seed(a.seed)
    data = {}
    for s in a.seq_lens:
        shape_q = (a.batch_size, s, a.num_q_heads, a.head_dim)
        shape_kv = (a.batch_size, s, a.num_kv_heads, a.head_dim)
        data[s] = tuple(torch.randn(sh, device=dev, dtype=dtype, generator=gen) for sh in (shape_q, shape_kv, shape_kv))
    if a.backend == "torch":
        model = TorchAttention(a.causal)
    else:
        model = core.instantiate(core.import_by_path(a.model_path or core.default_model_path("attention", "b200")),
                                 device=dev, dtype=dtype)
        if hasattr(model, "causal"):
            model.causal = a.causal
    records = []
    for s in a.seq_lens:
        q, k, v = data[s]
        if a.check_correctness:
            with torch.inference_mode():
                core.check_tensor(model(q, k, v), sdpa(q, k, v, a.causal),
                                  f"Attention correctness failed for seq_len {s}", TOL[a.dtype], TOL[a.dtype])
        if hasattr(model, "build_call"):
            call = model.build_call(q_bshd=q, k_bshd=k, v_bshd=v)
        else:
            call = lambda q=q, k=k, v=v: model(q, k, v)  # noqa: E731
        ms = core.time_with_cudagraph(call, warmup=a.warmup, repeat=a.repeat, graph_iters=a.graph_iters)
        rec = {"domain": "attention", "backend": a.backend, "seq_len": s, "batch_size": a.batch_size,
               "num_q_heads": a.num_q_heads, "num_kv_heads": a.num_kv_heads, "head_dim": a.head_dim,
               "causal": a.causal, "dtype": a.dtype, "mean_ms": ms,
               "tflops": attention_tflops(a.batch_size, a.num_q_heads, s, a.head_dim, ms, a.causal)}
        if a.check_correctness:
            rec["correctness"] = True
        core.emit(rec)
        records.append(rec)
    return records


if __name__ == "__main__":
    run()
