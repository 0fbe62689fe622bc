#!/usr/bin/env python3
"""GEMM benchmark, C[M,N] = A[M,K] * B[N,K]^T in bf16, CUDA-graph timing.

Same flags and JSONL record as the reference's scripts/benchmark/bench_gemm.py (inputs of
--matrix-sizes are drawn in sequence from one device generator like backend_gemm.py:58-69,
check against torch.matmul(a, b.T) with its tolerance, :43-46,135-137), plus --shapes MxNxK
for rectangular problems and a `torch` backend (cuBLAS) for comparison."""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))
import core  # noqa: E402

TOL = {"bf16": 1e-1, "fp16": 1e-2}
DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16}
SQUARE_SIZES = [1024, 2048, 4096, 8192, 16384]  # scripts/benchmark/config.py:4


class TorchGemm(torch.nn.Module):
    def forward(self, a_mk, b_nk):
        return torch.matmul(a_mk, b_nk.transpose(0, 1))


def run(argv=None) -> list[dict]:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--backend", choices=["b200", "torch"], default="b200")
    p.add_argument("--seed", type=int, default=20260312)
    p.add_argument("--dtype", choices=sorted(DTYPES), default="bf16")
    p.add_argument("--matrix-sizes", type=int, nargs="+", default=None)
    p.add_argument("--shapes", type=str, nargs="+", default=None, help="rectangular problems MxNxK")
    p.add_argument("--check-correctness", action="store_true")
    p.add_argument("--model-path", type=Path, default=None)
    core.add_timer_flags(p)
    a = p.parse_args(argv)

    torch.manual_seed(a.seed)
    dev, dtype = torch.device("cuda"), DTYPES[a.dtype]
    shapes = [(s, s, s) for s in (a.matrix_sizes or ([] if a.shapes else SQUARE_SIZES))]
    shapes += [tuple(int(x) for x in s.lower().split("x")) for s in (a.shapes or [])]
    gen = torch.Generator(device=dev).manual_seed(a.seed)
    inputs = [(torch.randn((m, k), device=dev, dtype=dtype, generator=gen),
               torch.randn((n, k), device=dev, dtype=dtype, generator=gen)) for (m, n, k) in shapes]
    if a.backend == "torch":
        model = TorchGemm()
    else:
        model = core.instantiate(core.import_by_path(a.model_path or core.default_model_path("gemm", "b200")),
                                 device=dev, dtype=dtype)
    records = []
    for (m, n, k), (x, w) in zip(shapes, inputs):
        if a.check_correctness:
            with torch.inference_mode():
                core.check_tensor(model(x, w), torch.matmul(x, w.transpose(0, 1)),
                                  f"GEMM correctness failed for {m}x{n}x{k}", TOL[a.dtype], TOL[a.dtype])
        call = model.build_call(a_mk=x, b_nk=w) if hasattr(model, "build_call") else (lambda x=x, w=w: model(x, w))
        ms = core.time_with_cudagraph(call, warmup=a.warmup, repeat=a.repeat, graph_iters=a.graph_iters)
        rec = {"domain": "gemm", "backend": a.backend, "matrix_size": m if m == n == k else None, "m": m, "n": n,
               "k": k, "dtype": a.dtype, "mean_ms": ms, "tflops": 2.0 * m * n * k / (ms / 1e3) / 1e12}
        if a.check_correctness:
            rec["correctness"] = True
        core.emit(rec)
        records.append(rec)
    return records


if __name__ == "__main__":
    run()
