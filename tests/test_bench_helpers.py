"""bench.py pieces that run without a GPU: the workload definition, the FLOP accounting and
the parsing of the nvidia-smi clock samples."""
from __future__ import annotations

import importlib.util
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def load_bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", REPO / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_sweep_is_the_20_shapes_of_the_configuration():
    b = load_bench()
    shapes = b.sweep_shapes()
    assert len(shapes) == 20 and len(set(shapes)) == 20
    assert {m for m, _, _ in shapes} == {1, 16, 128, 1024, 8192}
    assert {(n, k) for _, n, k in shapes} == {(4096, 4096), (14336, 4096), (4096, 14336), (6144, 4096)}
    assert b.flops([(2, 3, 5)]) == 60.0
    dense = [s for s in shapes if s[0] >= b.DENSE_M]
    assert len(dense) == 8 and b.flops(dense) / b.flops(shapes) > 0.98
    # both arms describe the same work: one config object, 20 shapes, the same FLOPs per step
    cfg = b.sweep_config(1)
    assert cfg["shapes"] == 20 and cfg["flop_per_step"] == b.flops(shapes) and cfg["workload"] == b.WORKLOAD
    assert b.sweep_config(8)["parallelism"].startswith("column-sharded over N x8")
    for world in (2, 4, 8):
        assert all(n % world == 0 for _, n, _ in shapes)


def test_peaks_come_from_the_measured_file_or_the_fallback(tmp_path, monkeypatch):
    b = load_bench()
    monkeypatch.setattr(b, "REPO", tmp_path)
    assert b.load_peaks() == {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0, "source": "fallback"}
    (tmp_path / "MEASURED_PEAKS.json").write_text('{"bf16_tflops": 1670.1, "hbm_gbs": 6559.7}')
    assert b.load_peaks() == {"bf16_tflops": 1670.1, "hbm_gbs": 6559.7, "source": "measured"}


def test_clock_samples_under_load_are_chosen_by_power():
    b = load_bench()
    s = b.ClockSampler(0)

    class Done:
        def terminate(self):
            pass

        def wait(self, timeout=None):
            return 0

    s.proc = Done()
    s.lines = [
        "0, 345, 1965, 140.0, Not Active, Not Active, Not Active, Not Active",
        "0, 1410, 1965, 980.5, Not Active, Not Active, Not Active, Active",
        "0, 1350, 1965, 1001.2, Not Active, Not Active, Not Active, Active",
        "0, 1965, 1965, 310.0, Not Active, Not Active, Not Active, Not Active",
        "garbage line",
    ]
    out = s.stop()
    assert out["sm_mhz"] == 1380.0 and out["sm_max_mhz"] == 1965.0
    assert out["samples"] == 4 and out["samples_under_load"] == 2
    assert out["reasons"] == ["sw_power_cap"] and out["power_w_max"] == 1001.2
    idle = b.ClockSampler(0)
    assert idle.stop()["reasons"] == ["nvidia-smi unavailable"]


def test_operator_records_follow_from_the_work_and_the_time():
    b = load_bench()
    peaks = {"bf16_tflops": 1000.0, "hbm_gbs": 5000.0, "source": "measured"}
    c = {"case": "gemm:1x2x3", "flop": 2.0e12, "bytes": 1.0e9, "launches": 1, "bound": "tensor", "kernel": "k"}
    rec = b.op_record(c, 4.0, 3.9, peaks, 5)
    assert rec["tflops"] == 500.0 and rec["roofline"]["frac"] == 0.5 and rec["roofline"]["unit"] == "TFLOP/s"
    c.update(bound="hbm", tokens=64, experts_touched=3)
    rec = b.op_record(c, 4.0, 3.9, peaks, 5)
    assert rec["gbs"] == 250.0 and rec["roofline"]["frac"] == 0.05 and rec["tokens_per_s"] == 16000.0
    assert set(b.OPS_CASES) <= set(b.CASE_PRESETS)
