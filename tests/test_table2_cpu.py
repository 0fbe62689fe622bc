"""The table driver without a GPU: command lines carry the reference's grid and shapes,
records are re-rated with the reference's FLOP conventions, a failing backend costs its
cells only, and the CSV has one row per (domain, workload) with `-` for missing cells."""
from __future__ import annotations

import importlib.util
import json
from pathlib import Path
from types import SimpleNamespace

HARNESS = Path(__file__).resolve().parents[1] / "lumen-sosp26-ae_b200" / "harness"


def load():
    spec = importlib.util.spec_from_file_location("harness_table2", HARNESS / "table2.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_command_lines_follow_the_reference_grid():
    t2 = load()
    kw = dict(python="py", moe_input_dtype="fp8", warmup=10, repeat=100, graph_iters=1, check=False)
    g = t2.cli_command("gemm", "b200", t2.WORKLOADS, **kw)
    assert g[1].endswith("bench_gemm.py") and g[g.index("--matrix-sizes") + 1:][:5] == ["1024", "2048", "4096", "8192", "16384"]
    a = t2.cli_command("attention", "torch", [4096], **kw)
    for flag, val in (("--batch-size", "16"), ("--num-q-heads", "8"), ("--num-kv-heads", "1"), ("--head-dim", "128"),
                      ("--seq-lens", "4096"), ("--backend", "torch")):
        assert a[a.index(flag) + 1] == val
    m = t2.cli_command("moe", "b200", [1024], **dict(kw, check=True))
    for flag, val in (("--dim", "7168"), ("--inter-dim", "2048"), ("--experts", "32"), ("--topk", "4"),
                      ("--input-dtype", "fp8"), ("--repeat", "100")):
        assert m[m.index(flag) + 1] == val
    assert m[-1] == "--check-correctness"


def test_rates_use_the_reference_conventions():
    t2 = load()
    assert t2.tflops_of({"domain": "gemm", "m": 1000, "n": 1000, "k": 500, "mean_ms": 1.0}) == 1.0
    attn = {"domain": "attention", "batch_size": 16, "num_q_heads": 8, "seq_len": 1024, "head_dim": 128, "mean_ms": 1.0}
    full = t2.tflops_of(dict(attn, causal=False))
    assert abs(full - 8.0 * 16 * 8 * 1024 ** 2 * 128 / 1e9) < 1e-9
    assert t2.tflops_of(dict(attn, causal=True)) == full / 2
    moe = {"domain": "moe", "tokens": 1024, "topk": 4, "dim": 7168, "inter_dim": 2048, "mean_ms": 2.0}
    assert abs(t2.tflops_of(moe) - 6.0 * 1024 * 4 * 7168 * 2048 / 2e9) < 1e-9


def test_collect_keeps_records_of_a_failing_backend_and_render_marks_gaps(tmp_path):
    t2 = load()
    good = json.dumps({"domain": "gemm", "backend": "b200", "matrix_size": 1024, "m": 1024, "n": 1024, "k": 1024,
                       "mean_ms": 0.002})

    def fake_runner(cmd, **kw):
        if "torch" in cmd:
            return SimpleNamespace(stdout="noise\n{not json\n", stderr="boom", returncode=1)
        return SimpleNamespace(stdout=f"banner\n{good}\n", stderr="", returncode=0)

    sink = tmp_path / "gemm.jsonl"
    assert t2.collect(["py", "x", "--backend", "b200"], sink, timeout=1, runner=fake_runner) == 1
    assert t2.collect(["py", "x", "--backend", "torch"], sink, timeout=1, runner=fake_runner) == 0
    text = t2.render(t2.read_records(tmp_path), [1024, 2048], ["b200", "torch"])
    rows = text.strip().splitlines()
    assert rows[0] == "domain,workload,b200,torch"
    assert rows[1] == f"gemm,1024,{2.0 * 1024 ** 3 / 0.002e-3 / 1e12:.2f},-"
    assert rows[2] == "gemm,2048,-,-" and len(rows) == 1 + 3 * 2


def test_skip_run_renders_an_existing_workspace(tmp_path, capsys):
    t2 = load()
    (tmp_path / "moe.jsonl").write_text(json.dumps(
        {"domain": "moe", "backend": "b200", "tokens": 1024, "topk": 4, "dim": 7168, "inter_dim": 2048,
         "mean_ms": 1.0}) + "\n")
    assert t2.main(["--workspace-dir", str(tmp_path), "--skip-run", "--workloads", "1024"]) == 0
    out = capsys.readouterr().out
    assert "moe,1024,360.78,-" in out and (tmp_path / "table2.csv").read_text() == out
