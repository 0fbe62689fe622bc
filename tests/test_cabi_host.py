"""The C-ABI library builds, loads and exports every symbol include/lumen_b200.h
declares; the host wrappers validate like the reference's and never compute on the CPU."""
from __future__ import annotations

import ctypes
import re

import pytest
import torch

from conftest import REPO


def declared_symbols() -> list[str]:
    text = (REPO / "include" / "lumen_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lumen_b200_\w+)\s*\(", text)))


def test_header_declares_the_path():
    names = declared_symbols()
    for needed in ("lumen_b200_gemm_bf16_nt", "lumen_b200_fa_fwd_bf16", "lumen_b200_moe_route_topk",
                   "lumen_b200_moe_sort_routes", "lumen_b200_moe_grouped_gemm", "lumen_b200_moe_combine"):
        assert needed in names


def test_library_exports_every_declared_symbol(pkg):
    lib = ctypes.CDLL(str(pkg.LIB_PATH))
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} is declared in the header but not exported"


def test_binding_table_matches_header(pkg):
    assert sorted(pkg._cabi.SIGNATURES) == declared_symbols()


def test_version_string(pkg):
    assert b"sm_100a" in pkg._cabi.load().lumen_b200_version()


def test_missing_library_fails_loudly(pkg, tmp_path):
    with pytest.raises(RuntimeError, match="no CPU or PyTorch fallback"):
        pkg._cabi.load(tmp_path / "liblumen_b200.so")


def test_wrappers_raise_the_reference_exception_types(pkg):
    """What callers can rely on is the exception type per kind of mistake (ValueError for
    every bad GEMM argument; for attention TypeError on dtypes, ValueError otherwise) and that
    the message names the wrapper and the offending argument."""
    f = pkg.gemm_pipeline_transposed_b
    a = torch.zeros((4, 8), dtype=torch.bfloat16)
    for bad_call, word in ((lambda: f(a.float(), a), "A"), (lambda: f(a, a.float()), "B"),
                           (lambda: f(a[0], a), "A"), (lambda: f(a, a), "CPU")):
        with pytest.raises(ValueError, match=word) as err:
            bad_call()
        assert "gemm_pipeline_transposed_b" in str(err.value)
    q = torch.zeros((1, 4, 2, 128), dtype=torch.bfloat16)
    with pytest.raises(TypeError, match="q"):
        pkg.flash_attn(q.float(), q, q)
    with pytest.raises(ValueError, match="k"):
        pkg.flash_attn(q, q[0], q)
    with pytest.raises(ValueError, match="CPU"):
        pkg.flash_attn(q, q, q)
    p3 = torch.zeros((4, 2, 128), dtype=torch.bfloat16)
    with pytest.raises(TypeError, match="v"):
        pkg.flash_attn_packed(p3, p3, p3.half(), torch.tensor([0, 4]), 4)
    with pytest.raises(ValueError, match="flash_attn_packed"):
        pkg.flash_attn_packed(p3, p3, p3, torch.tensor([0, 4]), 4)  # CPU tensors


def test_shared_argument_checker():
    import importlib

    checks = importlib.import_module("lumen-sosp26-ae_b200._checks")
    t = torch.zeros((2, 3))
    with pytest.raises(ValueError, match="2 dimension"):
        checks.check_operands("op", [checks.Operand("x", t, "[a, b, c]")], dtype=torch.float32, dtype_error=TypeError)
    with pytest.raises(TypeError, match="float32"):
        checks.check_operands("op", [checks.Operand("x", t, "[a, b]")], dtype=torch.bfloat16, dtype_error=TypeError)
    with pytest.raises(ValueError, match="result buffer is"):
        checks.check_output("op", torch.zeros((2, 2)), (2, 3), t.device, dtype=torch.float32, dtype_error=TypeError)
    assert checks.check_output("op", None, (2, 3), t.device, dtype=torch.float32, dtype_error=TypeError).shape == (2, 3)
    with pytest.raises(TypeError, match="op: why"):
        checks.require(False, "op", "why", TypeError)


def test_moe_host_validation(pkg):
    with pytest.raises(ValueError, match="no CPU path"):
        pkg.moe.route_topk(torch.zeros((2, 8)), 2)
    assert pkg.moe.max_padded_routes(4096, 2, 8) == 4096 * 2 + 8 * 32 - 2


def test_null_arguments_are_refused_before_any_device_work(pkg):
    """Every entry point validates its arguments first: with null pointers it returns
    LUMEN_B200_EINVAL without touching a GPU (none exists where this test runs)."""
    lib = pkg._cabi.load()
    einval = pkg._cabi.EINVAL
    assert lib.lumen_b200_gemm_bf16_nt(None, None, None, 4, 4, 8, 8, 8, 4, None, 0, None) == einval
    assert lib.lumen_b200_gemm_bf16_nt_static(None, None, None, 4, 4, 8, 8, 8, 4, None) == einval
    assert lib.lumen_b200_fa_fwd_bf16(None, None, None, None, 1, 8, 1, 1, 128, 0.1, 1, None) == einval
    assert lib.lumen_b200_fa_fwd_varlen_bf16(None, None, None, None, None, 1, 8, 8, 1, 1, 128, 0.1, 1, None) == einval
    assert lib.lumen_b200_moe_route_topk(None, None, None, 4, 8, 2, None) == einval
    assert lib.lumen_b200_moe_router_logits(None, None, None, 4, 64, 8, None) == einval
    assert lib.lumen_b200_moe_sort_routes(None, None, None, None, None, None, None, None, None, None, 0,
                                          4, 8, 2, 32, None) == einval
    assert lib.lumen_b200_moe_permute_rows(None, None, None, None, 4, 64, 8, None) == einval
    assert lib.lumen_b200_moe_grouped_gemm(None, None, None, None, None, 8, 2, 64, 64, 0, 4, None) == einval
    assert lib.lumen_b200_moe_combine(None, None, None, None, 4, 64, 2, None) == einval
    assert lib.lumen_b200_moe_dequant_fp8(None, None, None, None, 4, 128, None) == einval
    assert lib.lumen_b200_moe_ep_plan(None, 2, 8, 0, None, None, None, None, None, None) == einval
    assert lib.lumen_b200_device_status(None) == einval
    assert lib.lumen_b200_moe_forward(None, None, None, None, None, None, None, None, 0, 4, 64, 64, 8, 2, None) == einval
    # the single-call forward wants exactly one of logits / (topk_ids, topk_weights), and a sane shape
    one = ctypes.c_void_p(256)  # never dereferenced: refused on the argument check
    assert lib.lumen_b200_moe_forward(one, one, one, one, one, one, one, one, 1 << 30, 4, 64, 64, 8, 2, None) == einval
    assert lib.lumen_b200_moe_forward(one, one, one, None, one, None, one, one, 1 << 30, 4, 64, 64, 8, 2, None) == einval
    assert lib.lumen_b200_moe_forward(one, one, one, one, None, None, one, one, 1 << 30, 4, 64, 64, 8, 9, None) == einval
    assert lib.lumen_b200_moe_forward(one, one, one, one, None, None, one, one, 1 << 30, 4, 60, 64, 8, 2, None) == einval
    assert lib.lumen_b200_moe_forward(one, one, one, one, None, None, one, one, 64, 4, 64, 64, 8, 2, None) == pkg._cabi.EWORKSPACE
    assert lib.lumen_b200_moe_forward_scratch_bytes(4, 60, 64, 8, 2) == 0
    small, large = (lib.lumen_b200_moe_forward_scratch_bytes(t, 64, 64, 8, 2) for t in (4, 400))
    rows = 4 * 2 + 8 * 32 - 2  # three [rows, 64] bf16 intermediates plus the route arrays
    assert 3 * rows * 64 * 2 < small < large
    assert lib.lumen_b200_moe_sort_scratch_bytes(1000, 8, 2) == 2 * 8 * 4
    assert lib.lumen_b200_gemm_static_scratch_limit() == 16 << 20
    err = pkg._cabi.LumenB200Error("f", pkg._cabi.EWORKSPACE)
    assert "EWORKSPACE" in str(err) and err.code == pkg._cabi.EWORKSPACE


def test_harness_loader_follows_the_reference_entry_point_order(pkg, tmp_path):
    import importlib.util

    spec = importlib.util.spec_from_file_location("harness_core_under_test", REPO / "lumen-sosp26-ae_b200" / "harness" / "core.py")
    core = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(core)
    src = tmp_path / "model.py"
    src.write_text("class Model:\n    tag = 'model'\nclass ModelNew:\n    tag = 'new'\ndef kernel_function():\n    return 'fn'\n")
    assert core.instantiate(core.import_by_path(src), device=torch.device("cpu")).tag == "new"
    src.write_text("class Model:\n    tag = 'model'\ndef kernel_function():\n    return 'fn'\n")
    assert core.instantiate(core.import_by_path(src), device=torch.device("cpu")).tag == "model"
    src.write_text("def kernel_function():\n    return 'fn'\n")
    assert core.instantiate(core.import_by_path(src), device=torch.device("cpu"))() == "fn"
    src.write_text("x = 1\n")
    with pytest.raises(RuntimeError, match="expected one of"):
        core.instantiate(core.import_by_path(src), device=torch.device("cpu"))
    assert core.default_model_path("gemm", "b200").exists()


def test_bench_reference_arm_runs_without_a_gpu():
    import json
    import subprocess
    import sys

    out = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0"],
                         capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference" and rec["unit"] == "TFLOP/s" and rec["value"] > 0
    assert rec["cpu_baseline"]["kind"] == "port" and rec["e2e"]["h2d_bytes_per_step"] == 0


def test_model_files_follow_the_task_contract(pkg):
    """get_inputs / get_init_inputs of every system (prompts/kernelbench/*.py contract) and the
    MoE system's EVAL_CONFIG override."""
    import importlib.util

    def load(op):
        path = REPO / "lumen-sosp26-ae_b200" / "datasets" / "inference" / op / "b200" / "model.py"
        spec = importlib.util.spec_from_file_location(f"b200_model_{op}", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return mod

    gemm = load("gemm")
    assert gemm.get_init_inputs() == [] and hasattr(gemm, "ModelNew") and callable(gemm.kernel_function)
    gemm.M, gemm.N, gemm.K = 8, 16, 32
    a, b = gemm.get_inputs()
    assert tuple(a.shape) == (8, 32) and tuple(b.shape) == (16, 32) and a.dtype == torch.bfloat16
    attn = load("attention")
    attn.batch_size, attn.sequence_length, attn.num_q_heads, attn.num_kv_heads = 1, 5, 4, 2
    q, k, v = attn.get_inputs()
    assert tuple(q.shape) == (1, 5, 4, 128) and tuple(k.shape) == (1, 5, 2, 128) and tuple(v.shape) == tuple(k.shape)
    assert attn.ModelNew().causal is True and attn.ModelNew(causal=False).causal is False
    moe = load("moe")
    moe.EVAL_CONFIG = {"tokens": 8, "dim": 128, "inter_dim": 128, "experts": 4, "topk": 9, "seed": "x"}
    xs = moe.get_inputs()
    assert [tuple(t.shape) for t in xs] == [(8, 128), (4, 256, 128), (4, 128, 128), (8, 4), (8, 4), (8, 1),
                                            (4, 2), (4, 1)]
    assert xs[4].dtype == torch.int32 and float(xs[3].sum(dim=1).min()) > 0.999
    with pytest.raises(ValueError, match="bf16 and fp8"):
        moe.Model(variant="b200").build_cases(seq_len=8, shared_input=None, shared_weights={}, dim=128,
                                              inter_dim=128, experts=4, topk=2, input_dtype="fp16")
