"""The three b200/model.py files seen through the reference's OWN loader, unchanged.

scripts/benchmark/backends.py of the reference (load_module :18-31, entry-point resolution
through BACKEND_MAP :95-143) is imported from the reference checkout where one is present
(the build container); nothing of it is copied.  It must find ModelNew in each file, construct
it with no arguments, move it with .to(device, dtype), and the resulting objects must offer
the calls the per-operator drivers make next: build_call(a_mk=, b_nk=)
(backend_gemm.py:100-103), build_call(q_bshd=, k_bshd=, v_bshd=) (backend_attn.py:131-134)
and, for the MoE, a `Model` class with `build_cases` constructed as Model(variant=...)
(backend_moe.py:284-299, 406-409).  Skipped where the reference checkout is absent."""
from __future__ import annotations

import importlib.util
import inspect
import os
import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
REFERENCE = Path(os.environ.get("LUMEN_REFERENCE_ROOT", "/root/reference"))
BACKENDS_PY = REFERENCE / "scripts" / "benchmark" / "backends.py"
SYSTEMS = REPO / "lumen-sosp26-ae_b200" / "datasets" / "inference"

pytestmark = pytest.mark.skipif(not BACKENDS_PY.is_file(), reason="reference checkout not present on this machine")


@pytest.fixture(scope="module")
def ref_backends(pkg):
    spec = importlib.util.spec_from_file_location("reference_benchmark_backends", BACKENDS_PY)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # its dataclasses look the module up while they are built
    spec.loader.exec_module(mod)
    yield mod
    sys.modules.pop(spec.name, None)


@pytest.mark.parametrize("op", ["gemm", "attention", "moe"])
def test_reference_loader_resolves_and_builds_the_b200_systems(ref_backends, op):
    path = SYSTEMS / op / "b200" / "model.py"
    module = ref_backends.load_module(path)
    assert module.__name__.startswith("bench_dyn_model_") and module.__name__ in sys.modules
    # the search order ModelNew -> Model -> kernel_function picks ModelNew
    first = next(b for b in ref_backends.BACKEND_MAP.values() if b.supports(module))
    assert first.entrypoint == "ModelNew" and first.kind == "class"
    model = ref_backends.build_model_instance(module, device=torch.device("cpu"), dtype=torch.bfloat16)
    assert isinstance(model, module.ModelNew)
    fn = ref_backends.build_model_fn(module, device=torch.device("cpu"), dtype=torch.bfloat16)
    assert callable(fn)
    if op == "gemm":
        assert list(inspect.signature(model.build_call).parameters) == ["a_mk", "b_nk"]
        assert list(inspect.signature(model.forward).parameters) == ["a_mk", "b_nk"]
        assert callable(module.kernel_function)
    elif op == "attention":
        assert list(inspect.signature(model.build_call).parameters) == ["q_bshd", "k_bshd", "v_bshd"]
        assert list(inspect.signature(model.forward).parameters) == ["q_bshd", "k_bshd", "v_bshd"]
    else:
        case_model = module.Model(variant="lumen")  # how backend_moe.py constructs a case backend
        assert hasattr(module.Model, "build_cases") and hasattr(case_model, "_out_cache")
        want = {"seq_len", "shared_input", "shared_weights", "dim", "inter_dim", "experts", "topk", "input_dtype"}
        assert set(inspect.signature(case_model.build_cases).parameters) == want
        assert list(inspect.signature(model.forward).parameters) == [
            "input_q", "w1_q", "w2_q", "topk_weights", "topk_ids", "input_scale", "fc1_scale", "fc2_scale"]
    # no CPU path behind the contract: the call itself refuses host tensors
    if op == "gemm":
        a = torch.zeros((8, 16), dtype=torch.bfloat16)
        with pytest.raises(ValueError, match="CPU"):
            fn(a, a)
    assert not bool(getattr(module, "DIRECT_EXIT_AFTER_SUCCESS", False))
