"""The harness CLIs (reference flags, reference JSONL records) drive the B200 systems through
the model.py contract with --check-correctness, i.e. the reference's own parity check."""
from __future__ import annotations

import importlib.util
import json
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
HARNESS = Path(__file__).resolve().parents[1] / "lumen-sosp26-ae_b200" / "harness"


def load(name):
    spec = importlib.util.spec_from_file_location(f"harness_{name}", HARNESS / f"{name}.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


FAST = ["--warmup", "2", "--repeat", "3"]


def test_gemm_cli(cuda_pkg, capsys):
    recs = load("bench_gemm").run(["--matrix-sizes", "1024", "--shapes", "16x1024x512", "300x520x136",
                                   "--check-correctness", *FAST])
    lines = [json.loads(l) for l in capsys.readouterr().out.splitlines() if l.startswith("{")]
    assert [r["m"] for r in recs] == [1024, 16, 300] and all(r["correctness"] for r in lines)
    assert set(lines[0]) >= {"domain", "backend", "matrix_size", "m", "n", "k", "dtype", "mean_ms", "tflops"}
    assert cuda_pkg.device_status() == 0


@pytest.mark.parametrize("extra", [[], ["--no-causal"]])
def test_attention_cli(cuda_pkg, capsys, extra):
    recs = load("bench_attn").run(["--seq-lens", "512", "1000", "--batch-size", "2", "--num-q-heads", "8",
                                   "--num-kv-heads", "2", "--check-correctness", *extra, *FAST])
    assert [r["seq_len"] for r in recs] == [512, 1000] and all(r["correctness"] for r in recs)
    assert recs[0]["causal"] == (not extra)
    assert cuda_pkg.device_status() == 0


def test_moe_cli_with_block_scales(cuda_pkg, capsys):
    """The harness' bf16 mode keeps per-block scales; the B200 system folds them in."""
    recs = load("bench_moe").run(["--tokens", "64", "700", "--dim", "512", "--inter-dim", "256", "--experts", "8",
                                  "--topk", "2", "--check-correctness", *FAST])
    assert [r["tokens"] for r in recs] == [64, 700] and all(r["correctness"] for r in recs)
    assert cuda_pkg.device_status() == 0


def test_moe_cli_fp8_storage(cuda_pkg, capsys):
    """The reference harness' default storage: fp8 codes + block scales (compute stays bf16)."""
    recs = load("bench_moe").run(["--tokens", "300", "--dim", "512", "--inter-dim", "256", "--experts", "8",
                                  "--topk", "2", "--input-dtype", "fp8", "--check-correctness", *FAST])
    assert recs[0]["input_dtype"] == "fp8" and recs[0]["correctness"]
    assert cuda_pkg.device_status() == 0
