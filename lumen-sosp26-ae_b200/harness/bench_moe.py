#!/usr/bin/env python3
"""Fused-MoE benchmark (bf16 or fp8 storage, precomputed top-k routing), CUDA-graph timing.

Same flags and JSONL record as the reference's scripts/benchmark/bench_moe.py: inputs and weights follow backend_moe.py:86-210 (x = randn + 0.1, positive
per-128-block scales, scores ~ N(0,1) -> topk(sorted) -> softmax of the k values; weights from
seed + 17, randn * 8, positive block scales), the check is the routed fp32 reference of
:469-525 with its tolerance (:22-25), and a backend is a `Model(variant=).build_cases(...)`."""
from __future__ import annotations

import argparse
import sys
from pathlib import Path
from types import SimpleNamespace

import torch
import torch.nn.functional as F

sys.path.insert(0, str(Path(__file__).resolve().parent))
import core  # noqa: E402

BLOCK = 128
TOL = 1e-1
TOKENS = [1024, 2048, 4096, 8192, 16384]


def fp8_dtype():
    """The harness picks e4m3fnuz when torch has it, else e4m3fn (backend_moe.py:65-73)."""
    dt = getattr(torch, "float8_e4m3fnuz", None) or getattr(torch, "float8_e4m3fn", None)
    if dt is None:
        raise RuntimeError("torch float8 dtype is unavailable")
    return dt


def make_inputs(tokens, dim, experts, topk, dev, seed, dtype=torch.bfloat16):
    gen = torch.Generator(device=dev).manual_seed(seed)
    out = {}
    for t in tokens:
        x = torch.randn((t, dim), dtype=torch.float32, device=dev, generator=gen).add_(0.1).to(dtype)
        xs = torch.randn((t, dim // BLOCK), dtype=torch.float32, device=dev, generator=gen).mul_(2e-2).add_(1e-1)
        scores = torch.randn((t, experts), dtype=torch.float32, device=dev, generator=gen)
        val, idx = torch.topk(scores, k=topk, dim=-1, largest=True, sorted=True)
        out[t] = SimpleNamespace(input_q=x.contiguous(), input_scale=xs.clamp_min_(1e-8).contiguous(),
                                 topk_ids=idx.to(torch.int32).contiguous(),
                                 topk_weights=torch.softmax(val, dim=-1).to(torch.float32).contiguous())
    return out


def make_weights(dim, inter, experts, dev, seed, dtype=torch.bfloat16):
    gen = torch.Generator(device=dev).manual_seed(seed + 17)

    def rnd(shape):
        return torch.randn(shape, dtype=torch.float32, device=dev, generator=gen)

    w1 = rnd((experts, 2 * inter, dim)).mul_(8.0).to(dtype)
    w2 = rnd((experts, dim, inter)).mul_(8.0).to(dtype)
    s1 = rnd((experts, (2 * inter // BLOCK) * (dim // BLOCK))).mul_(2e-3).add_(1e-2).clamp_min_(1e-8)
    s2 = rnd((experts, (dim // BLOCK) * (inter // BLOCK))).mul_(2e-3).add_(1e-2).clamp_min_(1e-8)
    return {"w1_q": w1.contiguous(), "w2_q": w2.contiguous(), "fc1_scale": s1.contiguous(), "fc2_scale": s2.contiguous()}


def block_dequant(w, scale):
    rows, cols = w.shape
    s = scale.to(torch.float32).view(rows // BLOCK, 1, cols // BLOCK, 1)
    return (w.to(torch.float32).view(rows // BLOCK, BLOCK, cols // BLOCK, BLOCK) * s).view(rows, cols)


def expert_routes(x, experts):
    """Per expert, the (token, slot) index tensors of its routes; None where the expert is idle."""
    routes = []
    for e in range(experts):
        tok, slot = torch.nonzero(x.topk_ids == e, as_tuple=True)
        routes.append((tok, slot) if tok.numel() else None)
    return routes


def routed_reference(x, w, dim, inter, experts, routes=None):
    """fp32 expert-by-expert forward on the dequantised operands; `routes` (from expert_routes) may be
    passed in so that the call itself reads nothing back to the host and can be captured in a graph."""
    routes = expert_routes(x, experts) if routes is None else routes
    xf = (x.input_q.to(torch.float32).view(-1, dim // BLOCK, BLOCK) * x.input_scale.unsqueeze(-1)).reshape(-1, dim)
    out = torch.zeros_like(xf)
    for e, route in enumerate(routes):
        if route is None:
            continue
        tok, slot = route
        s1 = xf[tok] @ block_dequant(w["w1_q"][e], w["fc1_scale"][e]).T
        h = F.silu(s1[:, :inter]) * s1[:, inter:]
        out.index_add_(0, tok, (h @ block_dequant(w["w2_q"][e], w["fc2_scale"][e]).T)
                       * x.topk_weights[tok, slot].unsqueeze(1))
    return out.to(torch.bfloat16)


class TorchMoE:
    """PyTorch (cuBLAS) implementation of the same routed computation, the library baseline: bf16
    matmuls expert by expert on weights dequantised once.  The routes of each expert are found
    once per workload, outside the timed call, which keeps the call capturable; the baseline is
    therefore timed without its routing step and without the dequantisation."""

    def __init__(self, *, variant="torch"):
        self._out_cache = {}
        self._weights = None

    def _dense_weights(self, w):
        if self._weights is None:
            experts = w["w1_q"].shape[0]
            self._weights = (
                torch.stack([block_dequant(w["w1_q"][e], w["fc1_scale"][e]).to(torch.bfloat16) for e in range(experts)]),
                torch.stack([block_dequant(w["w2_q"][e], w["fc2_scale"][e]).to(torch.bfloat16) for e in range(experts)]))
        return self._weights

    def build_cases(self, *, seq_len, shared_input, shared_weights, dim, inter_dim, experts, topk, input_dtype):
        routes = expert_routes(shared_input, experts)
        w13, w2 = self._dense_weights(shared_weights)
        x = shared_input

        def forward():
            xb = (x.input_q.to(torch.float32).view(-1, dim // BLOCK, BLOCK)
                  * x.input_scale.unsqueeze(-1)).reshape(-1, dim).to(torch.bfloat16)
            out = torch.zeros(xb.shape, dtype=torch.float32, device=xb.device)
            for e, route in enumerate(routes):
                if route is None:
                    continue
                tok, slot = route
                s1 = xb[tok] @ w13[e].T
                h = F.silu(s1[:, :inter_dim].float()).mul_(s1[:, inter_dim:].float()).to(torch.bfloat16)
                out.index_add_(0, tok, (h @ w2[e].T).float() * x.topk_weights[tok, slot].unsqueeze(1))
            return out.to(torch.bfloat16)

        return [forward]


def run(argv=None) -> list[dict]:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--backend", choices=["b200", "torch"], default="b200")
    p.add_argument("--seed", type=int, default=20260319)
    p.add_argument("--tokens", type=int, nargs="+", default=TOKENS)
    p.add_argument("--dim", type=int, default=7168)
    p.add_argument("--inter-dim", type=int, default=2048)
    p.add_argument("--experts", type=int, default=32)
    p.add_argument("--topk", type=int, default=4)
    p.add_argument("--input-dtype", choices=["fp8", "bf16"], default="bf16")
    p.add_argument("--check-correctness", action="store_true")
    p.add_argument("--model-path", type=Path, default=None)
    core.add_timer_flags(p)
    a = p.parse_args(argv)
    if a.topk > a.experts:
        raise ValueError(f"topk ({a.topk}) must be <= experts ({a.experts})")
    if a.dim % BLOCK or a.inter_dim % BLOCK:
        raise ValueError(f"dim and inter_dim must be divisible by {BLOCK}")

    torch.manual_seed(a.seed)
    dev = torch.device("cuda")
    storage = torch.bfloat16 if a.input_dtype == "bf16" else fp8_dtype()
    inputs = make_inputs(a.tokens, a.dim, a.experts, a.topk, dev, a.seed, storage)
    weights = make_weights(a.dim, a.inter_dim, a.experts, dev, a.seed, storage)
    if a.backend == "torch":
        model = TorchMoE()
    else:
        mod = core.import_by_path(a.model_path or core.default_model_path("moe", "b200"))
        model = mod.Model(variant=a.backend)
    records = []
    for t in a.tokens:
        cases = model.build_cases(seq_len=t, shared_input=inputs[t], shared_weights=weights, dim=a.dim,
                                  inter_dim=a.inter_dim, experts=a.experts, topk=a.topk, input_dtype=a.input_dtype)
        for fn in cases:
            if a.check_correctness:
                with torch.inference_mode():
                    core.check_tensor(fn(), routed_reference(inputs[t], weights, a.dim, a.inter_dim, a.experts),
                                      f"MoE correctness failed for {t} tokens", TOL, TOL)
            ms = core.time_with_cudagraph(fn, warmup=a.warmup, repeat=a.repeat, graph_iters=a.graph_iters)
            rec = {"domain": "moe", "backend": a.backend, "tokens": t, "dim": a.dim, "inter_dim": a.inter_dim,
                   "experts": a.experts, "topk": a.topk, "input_dtype": a.input_dtype, "mean_ms": ms,
                   "tflops": 6.0 * t * a.topk * a.dim * a.inter_dim / (ms / 1e3) / 1e12}
            if a.check_correctness:
                rec["correctness"] = True
            core.emit(rec)
            records.append(rec)
        cache = getattr(model, "_out_cache", None)
        if isinstance(cache, dict):
            cache.clear()
    return records


if __name__ == "__main__":
    run()
