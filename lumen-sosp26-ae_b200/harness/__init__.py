"""Benchmark harness for the B200 box with the command line and JSONL records of the
reference's scripts/benchmark (bench_gemm.py, bench_attn.py, bench_moe.py), extended with
rectangular GEMMs, --no-causal and a `torch` library backend for comparison."""
