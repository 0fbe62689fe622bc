"""The KernelBench-style evaluator on the CPU (toy candidates) and, on a GPU, on the B200 GEMM system."""
from __future__ import annotations

import importlib
import os
import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
ORIGINAL = REPO / "tests" / "kernelbench" / "gemm_original.py"
B200_GEMM = REPO / "lumen-sosp26-ae_b200" / "datasets" / "inference" / "gemm" / "b200" / "model.py"


@pytest.fixture(scope="module")
def kb():
    if str(REPO) not in sys.path:
        sys.path.insert(0, str(REPO))
    return importlib.import_module("lumen-sosp26-ae_b200.harness.kernelbench_eval")


CPU = {"device": "cpu", "precision": "bf16", "num_trials": 3, "num_warmup": 1}

GOOD = """
import torch, torch.nn as nn
SEEN = []
class ModelNew(nn.Module):
    def forward(self, a, b):
        SEEN.append(float(a.float().sum()))
        return (b.float() @ a.float().T).T.to(a.dtype)
"""
WRONG = GOOD.replace(".T.to(a.dtype)", ".T.to(a.dtype) * 1.5")
BAD_SHAPE = GOOD.replace(".T.to(a.dtype)", ".T.to(a.dtype)[:, :-1]")
RAISES = GOOD.replace("SEEN.append", "raise RuntimeError('boom')  # ")


def candidate(tmp_path, text, name="cand.py"):
    path = tmp_path / name
    path.write_text(text)
    return path


def test_correct_candidate_passes_every_trial_and_is_timed(kb, tmp_path):
    res = kb.evaluate_generated_model(ORIGINAL, candidate(tmp_path, GOOD), dict(CPU, num_correct_trials=3))
    assert res.compiled and res.correctness, res.metadata
    assert res.metadata["correctness_trials"] == "(3 / 3)"
    assert res.runtime > 0 and res.ref_runtime > 0
    assert res.runtime_stats["num_trials"] == 3 and res.runtime_stats["timing_mode"] == "eager-wallclock"
    assert res.metadata["seed"] == 42 and res.metadata["num_correct_trials"] == 3


def test_trials_draw_different_inputs_and_repeat_for_the_same_seed(kb, tmp_path):
    """Each correctness trial reseeds the generator with its own seed; the same main seed gives the same trials."""
    torch.manual_seed(7)
    want_seeds = [int(torch.randint(0, 2 ** 32 - 1, (1,)).item()) for _ in range(2)]
    sums = []
    for s in want_seeds:
        torch.manual_seed(s)
        sums.append(float(torch.randn(512, 384, dtype=torch.bfloat16).float().sum()))
    assert sums[0] != sums[1]
    path = candidate(tmp_path, GOOD + "\nimport builtins\nbuiltins._kb_seen = SEEN\n")
    res = kb.evaluate_generated_model(ORIGINAL, path, dict(CPU, num_correct_trials=2, seed=7))
    import builtins
    assert res.correctness
    assert builtins._kb_seen[:2] == sums
    del builtins._kb_seen


def test_wrong_values_wrong_shape_and_runtime_errors_are_reported_not_raised(kb, tmp_path):
    res = kb.evaluate_generated_model(ORIGINAL, candidate(tmp_path, WRONG), CPU)
    assert res.compiled and not res.correctness and res.runtime == -1.0
    assert res.metadata["correctness_trials"] == "(0 / 1)" and float(res.metadata["max_difference"][0]) > 1.0
    res = kb.evaluate_generated_model(ORIGINAL, candidate(tmp_path, BAD_SHAPE), CPU)
    assert res.compiled and not res.correctness and "shape mismatch" in res.metadata["correctness_issue"]
    res = kb.evaluate_generated_model(ORIGINAL, candidate(tmp_path, RAISES), CPU)
    assert res.compiled and not res.correctness and res.metadata["runtime_error"] == "boom"


def test_files_that_do_not_load(kb, tmp_path):
    res = kb.evaluate_generated_model(ORIGINAL, tmp_path / "absent.py", CPU)
    assert not res.compiled and "Generated model file not found" in res.metadata["error"]
    res = kb.evaluate_generated_model(tmp_path / "absent.py", candidate(tmp_path, GOOD), CPU)
    assert not res.compiled and "Original model file not found" in res.metadata["error"]
    res = kb.evaluate_generated_model(ORIGINAL, candidate(tmp_path, "x = 1\n"), CPU)
    assert not res.compiled and res.metadata["compilation_error_name"] == "ModelNewNotFound"
    res = kb.evaluate_generated_model(ORIGINAL, candidate(tmp_path, "def broken(:\n"), CPU)
    assert not res.compiled and res.metadata["compilation_error_name"] == "SyntaxError"
    res = kb.evaluate_generated_model(candidate(tmp_path, "x = 1\n", "orig.py"), candidate(tmp_path, GOOD), CPU)
    assert not res.compiled and "must define Model" in res.metadata["error"]
    res = kb.evaluate_generated_model(ORIGINAL, candidate(tmp_path, GOOD), dict(CPU, num_trials=0))
    assert not res.compiled and "num_trials must be >= 1" in res.metadata["error"]


def test_reference_file_timing_and_the_cuda_requirement(kb, tmp_path):
    res = kb.evaluate_reference_file(ORIGINAL, {"device": "cpu", "num_trials": 2, "num_warmup": 1})
    assert res.compiled and res.correctness and res.runtime > 0 and res.metadata["precision"] == "torch.float32"
    if not torch.cuda.is_available():
        res = kb.evaluate_generated_model(ORIGINAL, candidate(tmp_path, GOOD), {})
        assert not res.compiled and res.metadata["error"] == "CUDA is not available, cannot run KernelBench eval"


def test_b200_model_files_load_from_source_text(kb):
    """The evaluator executes source text (no __file__): the systems find the package through
    LUMEN_B200_ROOT, and say how when they cannot."""
    for op in ("gemm", "attention", "moe"):
        path = B200_GEMM.parents[2] / op / "b200" / "model.py"
        new_cls, get_inputs = kb.load_source(path, ("ModelNew", "get_inputs"))
        assert new_cls is not None and callable(get_inputs)
    saved = os.environ.pop("LUMEN_B200_ROOT")
    try:
        with pytest.raises(ImportError, match="LUMEN_B200_ROOT"):
            kb.load_source(B200_GEMM, ("ModelNew",))
    finally:
        os.environ["LUMEN_B200_ROOT"] = saved


@pytest.mark.gpu
def test_b200_gemm_system_under_the_evaluator(kb):
    res = kb.evaluate_generated_model(ORIGINAL, B200_GEMM, {"precision": "bf16", "num_correct_trials": 3,
                                                           "num_trials": 10, "num_warmup": 2})
    assert res.compiled and res.correctness, res.metadata
    assert res.metadata["correctness_trials"] == "(3 / 3)"
    assert res.runtime_stats["timing_mode"] == "cudagraph" and 0 < res.runtime < 5.0 and res.ref_runtime > 0


@pytest.mark.gpu
@pytest.mark.parametrize("op", ["attention", "moe"])
def test_b200_attention_and_moe_systems_under_the_evaluator(kb, op):
    """ModelNew of the attention and MoE systems through randomised correctness trials and the
    evaluator's graph-captured timing: the captured call must not read anything back to the
    host, and new scale tensors in every trial must not meet stale folded weights."""
    original = REPO / "tests" / "kernelbench" / f"{op}_original.py"
    system = B200_GEMM.parents[2] / op / "b200" / "model.py"
    res = kb.evaluate_generated_model(original, system, {"precision": "bf16", "num_correct_trials": 3,
                                                         "num_trials": 5, "num_warmup": 2})
    assert res.compiled and res.correctness, res.metadata
    assert res.metadata["correctness_trials"] == "(3 / 3)"
    assert res.runtime_stats["timing_mode"] == "cudagraph" and res.runtime > 0
