"""Evaluator for KernelBench-style model files: correctness over randomised trials, then
CUDA-graph replay timing of the candidate (`ModelNew`) and of the original (`Model`).

The entry points, their configuration keys, their metadata and their failure behaviour follow
python/lumen/harness/datasets/kernelbench/evaluator.py:20-252 of the reference
(evaluate_reference_file, evaluate_generated_model; defaults seed 42, 5 warm-ups, 100 trials,
1 correctness trial; timing = one captured call replayed once per trial between events,
:340-377).  That file delegates to the third-party `kernelbench` package (ScalingIntelligence
KernelBench, installed un-pinned by the reference's docker/Dockerfile), which is not in this
repository's environment; the few functions of it that the evaluator uses are restated here
from their published behaviour:

* files are executed from their source text in a fresh namespace (no `__file__`);
* `set_seed` seeds torch's CPU and CUDA generators;
* inputs from `get_inputs()` / `get_init_inputs()`: tensors move to the device, floating-point
  tensors are cast to the evaluation precision, everything else passes through;
* correctness: trial seeds are drawn from a generator seeded with the main seed; per trial the
  seed is set before `get_inputs()` and before each model's call; outputs must have the same
  shape and satisfy `torch.allclose` with atol = rtol = 1e-4 (fp32) or 1e-2 (fp16 / bf16);
* timing statistics: mean, std, min, max, num_trials (+ hardware, device).

One extension: `eval_config["device"] = "cpu"` evaluates on the CPU with wall-clock timing
(`timing_mode` "eager-wallclock"), for machines without a GPU; the default needs CUDA, as in
the reference.
"""
from __future__ import annotations

import os
import statistics
import time
import traceback
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import torch

# model files of this package that are executed from source find the package through this variable
os.environ.setdefault("LUMEN_B200_ROOT", str(Path(__file__).resolve().parents[2]))

DEFAULT_SEED = 42
DEFAULT_NUM_WARMUP = 5
DEFAULT_NUM_TRIALS = 100
DEFAULT_BACKEND = "cuda"
PRECISIONS = {"fp32": torch.float32, "float32": torch.float32, "fp16": torch.float16,
              "float16": torch.float16, "bf16": torch.bfloat16, "bfloat16": torch.bfloat16}
TOLERANCE = {torch.float32: 1e-4, torch.float16: 1e-2, torch.bfloat16: 1e-2}


@dataclass
class KernelExecResult:
    """Field for field the result record of the KernelBench evaluators."""

    compiled: bool = False
    correctness: bool = False
    metadata: dict = field(default_factory=dict)
    runtime: float = -1.0  # mean milliseconds per call of the candidate
    runtime_stats: dict = field(default_factory=dict)
    ref_runtime: float = -1.0
    ref_runtime_stats: dict = field(default_factory=dict)


def set_seed(seed: int) -> None:
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed(seed)


def load_source(path: Path, names: tuple[str, ...]) -> list[Any]:
    """Execute a model file's source text in a fresh namespace; the named attributes (None if absent)."""
    namespace: dict[str, Any] = {"__name__": f"kernelbench_model_{path.stem}"}
    exec(compile(path.read_text(encoding="utf-8"), str(path), "exec"), namespace)  # noqa: S102
    return [namespace.get(n) for n in names]


def process_inputs(values, *, device: torch.device, precision: torch.dtype) -> list[Any]:
    out = []
    for v in values:
        if isinstance(v, torch.Tensor):
            v = v.to(device=device, dtype=precision) if v.is_floating_point() else v.to(device=device)
        out.append(v)
    return out


def _settings(config: dict) -> dict[str, int]:
    out = {}
    for key, default in (("seed", DEFAULT_SEED), ("num_correct_trials", 1), ("num_warmup", DEFAULT_NUM_WARMUP),
                         ("num_trials", DEFAULT_NUM_TRIALS)):
        value = int(config.get(key, default))
        if value < 1:
            raise ValueError(f"{key} must be >= 1, got {value}")
        out[key] = value
    return out


def _precision(config: dict) -> torch.dtype:
    p = config.get("precision", "fp32")
    if isinstance(p, torch.dtype):
        return p
    if str(p).lower() not in PRECISIONS:
        raise ValueError(f"unknown precision: {p}")
    return PRECISIONS[str(p).lower()]


def _device(config: dict, metadata: dict) -> torch.device | None:
    want = config.get("device")
    if want is not None and torch.device(want).type == "cpu":
        return torch.device("cpu")
    if not torch.cuda.is_available():
        metadata["error"] = "CUDA is not available, cannot run KernelBench eval"
        return None
    dev = torch.device(want) if want is not None else torch.device(f"cuda:{torch.cuda.current_device()}")
    torch.cuda.set_device(dev)
    metadata["hardware"] = torch.cuda.get_device_name(device=dev)
    return dev


def _sync(device: torch.device) -> None:
    if device.type == "cuda":
        torch.cuda.synchronize(device=device)


def _place(model, device: torch.device, precision: torch.dtype):
    if hasattr(model, "to"):
        model = model.to(device=device, dtype=precision)
    if hasattr(model, "eval"):
        model.eval()
    return model


def instantiate(cls, get_init_inputs, *, device, precision, seed):
    with torch.no_grad():
        set_seed(seed)
        init_inputs = process_inputs(get_init_inputs(), device=device, precision=precision)
        set_seed(seed)
        model = _place(cls(*init_inputs), device, precision)
        _sync(device)
    return model


def timing_stats(ms: list[float], device: torch.device) -> dict:
    stats = {"mean": float(statistics.fmean(ms)), "std": float(statistics.pstdev(ms)) if len(ms) > 1 else 0.0,
             "min": float(min(ms)), "max": float(max(ms)), "num_trials": len(ms), "device": str(device)}
    if device.type == "cuda":
        stats["hardware"] = torch.cuda.get_device_name(device=device)
    return stats


def measure(model, inputs, *, device: torch.device, num_warmup: int, num_trials: int) -> dict:
    """Milliseconds per call: one captured call replayed once per trial between two events."""
    times: list[float] = []
    with torch.no_grad():
        _sync(device)
        for _ in range(num_warmup):
            model(*inputs)
        _sync(device)
        if device.type != "cuda":
            for _ in range(num_trials):
                t0 = time.perf_counter()
                model(*inputs)
                times.append((time.perf_counter() - t0) * 1e3)
            stats = timing_stats(times, device)
            stats["timing_mode"] = "eager-wallclock"
            return stats
        with torch.cuda.device(device):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                keep = model(*inputs)  # noqa: F841  (keeps the captured output alive)
            torch.cuda.synchronize(device=device)
            for _ in range(num_trials):
                torch.cuda.synchronize(device=device)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                graph.replay()
                e1.record()
                torch.cuda.synchronize(device=device)
                times.append(float(e0.elapsed_time(e1)))
    stats = timing_stats(times, device)
    stats["timing_mode"] = "cudagraph"
    return stats


def check_correctness(original, candidate, get_inputs, *, metadata: dict, num_correct_trials: int, seed: int,
                      device: torch.device, precision: torch.dtype) -> KernelExecResult:
    tol = TOLERANCE[precision]
    torch.manual_seed(seed)
    trial_seeds = [int(torch.randint(0, 2 ** 32 - 1, (1,)).item()) for _ in range(num_correct_trials)]
    passed = 0
    with torch.no_grad():
        for trial_seed in trial_seeds:
            set_seed(trial_seed)
            inputs = process_inputs(get_inputs(), device=device, precision=precision)
            set_seed(trial_seed)
            want = original(*inputs)
            _sync(device)
            set_seed(trial_seed)
            try:
                got = candidate(*inputs)
                _sync(device)
            except Exception as exc:  # a candidate that fails at run time compiled but is wrong
                metadata["runtime_error"] = str(exc)
                metadata["runtime_error_name"] = type(exc).__name__
                return KernelExecResult(compiled=True, correctness=False, metadata=metadata)
            if tuple(want.shape) != tuple(got.shape):
                metadata["correctness_issue"] = f"Output shape mismatch: Expected {tuple(want.shape)}, got {tuple(got.shape)}"
                return KernelExecResult(compiled=True, correctness=False, metadata=metadata)
            if not torch.allclose(want.float(), got.float(), atol=tol, rtol=tol):
                diff = (want.float() - got.float()).abs()
                metadata.setdefault("max_difference", []).append(f"{float(diff.max()):.6f}")
                metadata.setdefault("avg_difference", []).append(f"{float(diff.mean()):.6f}")
                metadata["correctness_issue"] = "Output mismatch"
            else:
                passed += 1
    metadata["correctness_trials"] = f"({passed} / {num_correct_trials})"
    return KernelExecResult(compiled=True, correctness=passed == num_correct_trials, metadata=metadata)


def _missing(path: Path, label: str) -> str | None:
    return None if path.is_file() else f"{label} file not found: {path}"


def evaluate_reference_file(filename, eval_config: dict | None = None) -> KernelExecResult:
    """Time the `Model` of a KernelBench reference file (fp32, graph replay)."""
    path = Path(filename).expanduser()
    config = dict(eval_config or {})
    metadata: dict[str, Any] = {"filename": str(path)}
    err = _missing(path, "Reference")
    if err:
        metadata["error"] = err
        return KernelExecResult(metadata=metadata)
    device = _device(config, metadata)
    if device is None:
        return KernelExecResult(metadata=metadata)
    metadata["device"] = str(device)
    try:
        settings = _settings({k: v for k, v in config.items() if k in ("num_warmup", "num_trials")})
        precision = torch.float32
        cls, get_init_inputs, get_inputs = load_source(path, ("Model", "get_init_inputs", "get_inputs"))
        if cls is None or get_init_inputs is None or get_inputs is None:
            raise ValueError("Original model file must define Model, get_init_inputs, and get_inputs")
        model = instantiate(cls, get_init_inputs, device=device, precision=precision, seed=DEFAULT_SEED)
        inputs = process_inputs(get_inputs(), device=device, precision=precision)
        stats = measure(model, inputs, device=device, num_warmup=settings["num_warmup"],
                        num_trials=settings["num_trials"])
        metadata.update(precision=str(precision), backend=DEFAULT_BACKEND, seed=DEFAULT_SEED,
                        num_warmup=settings["num_warmup"], num_trials=settings["num_trials"],
                        cuda_graph=device.type == "cuda")
        return KernelExecResult(compiled=True, correctness=True, runtime=stats["mean"], runtime_stats=stats,
                                metadata=metadata)
    except Exception as exc:
        metadata.update(error=str(exc), error_name=type(exc).__name__, traceback=traceback.format_exc())
        return KernelExecResult(metadata=metadata)
    finally:
        if device.type == "cuda":
            torch.cuda.empty_cache()


def evaluate_generated_model(original_model_file, generated_model_file,
                             eval_config: dict | None = None) -> KernelExecResult:
    """Check `ModelNew` of the generated file against `Model` of the original file over
    `num_correct_trials` randomised trials, then time both.  Never raises: problems are reported
    in the result's metadata (`error`, `compilation_error`, `runtime_error`, `correctness_issue`)."""
    original_path = Path(original_model_file).expanduser()
    generated_path = Path(generated_model_file).expanduser()
    config = dict(eval_config or {})
    backend = str(config.get("backend", DEFAULT_BACKEND)).lower()
    metadata: dict[str, Any] = {"original_model_file": str(original_path),
                                "generated_model_file": str(generated_path), "backend": backend,
                                "eval_config": {k: str(v) if isinstance(v, torch.dtype) else v for k, v in config.items()}}
    if "gpu_arch" in config:
        metadata["gpu_arch"] = config["gpu_arch"]
    for path, label in ((original_path, "Original model"), (generated_path, "Generated model")):
        err = _missing(path, label)
        if err:
            metadata["error"] = err
            return KernelExecResult(metadata=metadata)
    device = _device(config, metadata)
    if device is None:
        return KernelExecResult(metadata=metadata)
    metadata["device"] = str(device)
    try:
        precision = _precision(config)
        s = _settings(config)
        metadata.update(precision=str(precision), seed=s["seed"], num_correct_trials=s["num_correct_trials"],
                        num_warmup=s["num_warmup"], num_trials=s["num_trials"], cuda_graph=device.type == "cuda")
        cls, get_init_inputs, get_inputs = load_source(original_path, ("Model", "get_init_inputs", "get_inputs"))
        if cls is None or get_init_inputs is None or get_inputs is None:
            raise ValueError("Original model file must define Model, get_init_inputs, and get_inputs")
        original = instantiate(cls, get_init_inputs, device=device, precision=precision, seed=s["seed"])
        try:
            (new_cls,) = load_source(generated_path, ("ModelNew",))
        except Exception as exc:
            metadata["compilation_error_name"] = type(exc).__name__
            metadata["compilation_error"] = str(exc)
            return KernelExecResult(metadata=metadata)
        if new_cls is None:
            metadata["compilation_error_name"] = "ModelNewNotFound"
            metadata["compilation_error"] = "Generated model must define ModelNew and compile successfully"
            return KernelExecResult(metadata=metadata)
        candidate = instantiate(new_cls, get_init_inputs, device=device, precision=precision, seed=s["seed"])
        result = check_correctness(original, candidate, get_inputs, metadata=metadata,
                                   num_correct_trials=s["num_correct_trials"], seed=s["seed"], device=device,
                                   precision=precision)
        if not result.correctness:
            return result
        set_seed(s["seed"])
        inputs = process_inputs(get_inputs(), device=device, precision=precision)
        stats = measure(candidate, inputs, device=device, num_warmup=s["num_warmup"], num_trials=s["num_trials"])
        ref_stats = measure(original, inputs, device=device, num_warmup=s["num_warmup"], num_trials=s["num_trials"])
        result.runtime, result.runtime_stats = stats["mean"], stats
        result.ref_runtime, result.ref_runtime_stats = ref_stats["mean"], ref_stats
        return result
    except Exception as exc:
        metadata.update(error=str(exc), error_name=type(exc).__name__, traceback=traceback.format_exc())
        return KernelExecResult(metadata=metadata)
    finally:
        if device.type == "cuda":
            torch.cuda.empty_cache()
