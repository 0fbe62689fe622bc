#!/usr/bin/env python3
"""Table of TFLOP/s per operator, workload and backend on this machine.

Runs the three benchmark CLIs of this directory over the workload grid of the reference's
paper table (scripts/table2/benchmark.py:17,154-231 of the reference: square GEMMs, causal
attention with batch 16 / 8 query heads / 1 KV head / head size 128, and the MoE with hidden
7168, intermediate 2048, 32 experts, top-4, all at workloads 1024 ... 16384), one subprocess
per (operator, backend), collects their JSONL records in a workspace directory and renders
one CSV: a row per (domain, workload), a column per backend, `-` where a backend produced no
record.  TFLOP/s are recomputed from `mean_ms` with the reference's conventions
(scripts/table2/benchmark.py:266-296): GEMM 2MNK; attention 8*B*Hq*S^2*D, halved for a
causal mask; MoE 6*T*topk*dim*inter_dim.

    python table2.py [--workloads 1024 4096] [--backends b200 torch] [--moe-input-dtype bf16]
    python table2.py --workspace-dir DIR --skip-run      # re-render records written earlier

The backends are the ones these CLIs know: `b200` (this library) and `torch` (cuBLAS, SDPA,
a per-expert loop) as the same-machine comparison column.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import math
import subprocess
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
WORKLOADS = (1024, 2048, 4096, 8192, 16384)
BACKENDS = ("b200", "torch")
DOMAINS = ("gemm", "attention", "moe")


def cli_command(domain: str, backend: str, workloads, *, python: str, moe_input_dtype: str,
                warmup: int, repeat: int, graph_iters: int, check: bool) -> list[str]:
    """Argument vector of one benchmark subprocess (same flags as the reference's CLIs)."""
    sizes = [str(w) for w in workloads]
    timer = ["--warmup", str(warmup), "--repeat", str(repeat), "--graph-iters", str(graph_iters)]
    if domain == "gemm":
        cmd = [python, str(HERE / "bench_gemm.py"), "--backend", backend, "--dtype", "bf16", "--matrix-sizes", *sizes]
    elif domain == "attention":
        cmd = [python, str(HERE / "bench_attn.py"), "--backend", backend, "--dtype", "bf16", "--seq-lens", *sizes,
               "--batch-size", "16", "--num-q-heads", "8", "--num-kv-heads", "1", "--head-dim", "128"]
    elif domain == "moe":
        cmd = [python, str(HERE / "bench_moe.py"), "--backend", backend, "--tokens", *sizes, "--dim", "7168",
               "--inter-dim", "2048", "--experts", "32", "--topk", "4", "--input-dtype", moe_input_dtype]
    else:
        raise ValueError(f"no such domain: {domain}")
    return cmd + timer + (["--check-correctness"] if check else [])


def collect(cmd: list[str], sink: Path, *, timeout: float, runner=subprocess.run) -> int:
    """Run one CLI; append every JSON object it printed to `sink`.  A failing or slow backend
    costs its cells, not the table (the reference's driver continues the same way,
    scripts/table2/benchmark.py:109-140)."""
    try:
        done = runner(cmd, capture_output=True, text=True, timeout=timeout)
        stdout, stderr, rc = done.stdout, done.stderr, done.returncode
    except subprocess.TimeoutExpired as exc:
        stdout, stderr, rc = (exc.stdout or ""), f"timed out after {timeout:.0f} s", -1
        if isinstance(stdout, bytes):
            stdout = stdout.decode(errors="replace")
    kept = 0
    with sink.open("a", encoding="utf-8") as out:
        for line in stdout.splitlines():
            line = line.strip()
            if line.startswith("{"):
                try:
                    json.loads(line)
                except json.JSONDecodeError:
                    continue
                out.write(line + "\n")
                kept += 1
    if rc != 0:
        print(f"[table2] {' '.join(cmd[1:4])} ... ended with code {rc}; kept {kept} record(s)\n{stderr}",
              file=sys.stderr)
    return kept


def workload_of(rec: dict) -> int:
    return int(rec[{"gemm": "matrix_size", "attention": "seq_len", "moe": "tokens"}[rec["domain"]]])


def tflops_of(rec: dict) -> float:
    ms = float(rec["mean_ms"])
    if not ms > 0.0:
        return math.nan
    d = rec["domain"]
    if d == "gemm":
        work = 2.0 * rec["m"] * rec["n"] * rec["k"]
    elif d == "attention":
        work = 8.0 * rec["batch_size"] * rec["num_q_heads"] * float(rec["seq_len"]) ** 2 * rec["head_dim"]
        if rec.get("causal", True):
            work *= 0.5
    else:
        work = 6.0 * rec["tokens"] * rec["topk"] * rec["dim"] * rec["inter_dim"]
    return work / (ms * 1e-3) / 1e12


def read_records(workspace: Path) -> list[dict]:
    recs = []
    for domain in DOMAINS:
        path = workspace / f"{domain}.jsonl"
        if path.exists():
            recs += [json.loads(line) for line in path.read_text().splitlines() if line.strip()]
    return recs


def render(records: list[dict], workloads, backends) -> str:
    cells: dict[tuple, float] = {}
    for rec in records:
        if rec.get("domain") in DOMAINS and (rec["domain"] != "gemm" or rec.get("matrix_size")):
            cells[(rec["domain"], workload_of(rec), rec.get("backend"))] = tflops_of(rec)
    buf = io.StringIO()
    w = csv.writer(buf, lineterminator="\n")
    w.writerow(["domain", "workload", *backends])
    for domain in DOMAINS:
        for wl in workloads:
            w.writerow([domain, wl, *[f"{cells[(domain, wl, b)]:.2f}" if (domain, wl, b) in cells else "-"
                                      for b in backends]])
    return buf.getvalue()


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--workspace-dir", type=Path, default=None)
    p.add_argument("--python", default=sys.executable)
    p.add_argument("--workloads", type=int, nargs="+", default=list(WORKLOADS))
    p.add_argument("--backends", nargs="+", choices=BACKENDS, default=list(BACKENDS))
    p.add_argument("--domains", nargs="+", choices=DOMAINS, default=list(DOMAINS))
    p.add_argument("--moe-input-dtype", choices=["fp8", "bf16"], default="bf16")
    p.add_argument("--check-correctness", action="store_true")
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--repeat", type=int, default=100)
    p.add_argument("--graph-iters", type=int, default=1)
    p.add_argument("--timeout", type=float, default=1800.0, help="seconds per subprocess")
    p.add_argument("--skip-run", action="store_true", help="render the records already in the workspace")
    a = p.parse_args(argv)
    ws = a.workspace_dir or HERE / "workspace" / time.strftime("%Y%m%d_%H%M%S", time.gmtime())
    ws.mkdir(parents=True, exist_ok=True)
    if not a.skip_run:
        for domain in a.domains:
            (ws / f"{domain}.jsonl").write_text("")
            for backend in a.backends:
                collect(cli_command(domain, backend, a.workloads, python=a.python,
                                    moe_input_dtype=a.moe_input_dtype, warmup=a.warmup, repeat=a.repeat,
                                    graph_iters=a.graph_iters, check=a.check_correctness),
                        ws / f"{domain}.jsonl", timeout=a.timeout)
    text = render(read_records(ws), a.workloads, a.backends)
    (ws / "table2.csv").write_text(text)
    sys.stdout.write(text)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
