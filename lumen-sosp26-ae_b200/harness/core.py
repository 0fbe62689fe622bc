"""Shared pieces of the harness: module loading with the reference's entry-point order,
the CUDA-graph timer and the JSONL writer.

Behaviour follows scripts/benchmark/backends.py:95-143 (ModelNew, then Model, then
kernel_function; classes built without arguments and moved with .to(device, dtype)) and
scripts/benchmark/cudagraph_timer.py:15-62 (eager warm-up, capture `graph_iters` calls,
replay warm-up, `measure_trials` x `repeat` replays between events, best trial) of the
reference; the code is this repository's own.
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import sys
from pathlib import Path
from typing import Any, Callable

import torch

PKG_DIR = Path(__file__).resolve().parents[1]
DATASETS = PKG_DIR / "datasets" / "inference"
ENTRY_POINTS = (("ModelNew", True), ("Model", True), ("kernel_function", False))


def import_by_path(path: Path):
    path = Path(path).expanduser().resolve()
    tag = hashlib.sha1(str(path).encode()).hexdigest()[:12]
    name = f"b200_harness_{path.stem}_{tag}"
    spec = importlib.util.spec_from_file_location(name, path)
    if spec is None or spec.loader is None:
        raise RuntimeError(f"cannot import module: {path}")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    try:
        spec.loader.exec_module(mod)
    except Exception:
        sys.modules.pop(name, None)
        raise
    return mod


def instantiate(module, *, device: torch.device, dtype: torch.dtype | None = None, **kwargs):
    """First of ModelNew / Model / kernel_function that the module defines."""
    for attr, is_class in ENTRY_POINTS:
        target = getattr(module, attr, None)
        if target is None:
            continue
        if not is_class:
            if kwargs:
                raise RuntimeError(f"function backend {attr} does not accept model kwargs")
            return target
        obj = target(**kwargs)
        if hasattr(obj, "to"):
            obj = obj.to(device=device) if dtype is None else obj.to(device=device, dtype=dtype)
        return obj
    raise RuntimeError("expected one of: ModelNew, Model, kernel_function")


def default_model_path(op: str, backend: str) -> Path:
    return DATASETS / op / backend / "model.py"


def time_with_cudagraph(fn: Callable[[], Any], *, warmup: int = 10, repeat: int = 100,
                        graph_iters: int = 1, trials: int = 2) -> float:
    """Mean milliseconds per call, best of `trials`."""
    warmup, repeat, graph_iters = max(0, warmup), max(1, repeat), max(1, graph_iters)
    with torch.inference_mode():
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        keep = []
        with torch.cuda.graph(graph):
            for _ in range(graph_iters):
                keep.append(fn())
        torch.cuda.synchronize()
        for _ in range(max(1, min(5, warmup))):
            graph.replay()
        torch.cuda.synchronize()
        best = None
        for _ in range(max(1, trials)):
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
            for _ in range(repeat):
                graph.replay()
            t1.record()
            torch.cuda.synchronize()
            ms = float(t0.elapsed_time(t1))
            best = ms if best is None else min(best, ms)
    return best / float(repeat * graph_iters)


def emit(record: dict) -> None:
    print(json.dumps(record, separators=(",", ":")), flush=True)


def add_timer_flags(parser) -> None:
    parser.add_argument("--warmup", type=int, default=10)
    parser.add_argument("--repeat", type=int, default=100)
    parser.add_argument("--graph-iters", type=int, default=1)


def check_tensor(actual, expected: torch.Tensor, what: str, rtol: float, atol: float) -> None:
    if not isinstance(actual, torch.Tensor):
        raise AssertionError(f"{what}: backend returned {type(actual).__name__}, expected torch.Tensor")
    if tuple(actual.shape) != tuple(expected.shape):
        raise AssertionError(f"{what}: output shape {tuple(actual.shape)}, expected {tuple(expected.shape)}")
    if actual.dtype != expected.dtype:
        raise AssertionError(f"{what}: output dtype {actual.dtype}, expected {expected.dtype}")
    try:
        torch.testing.assert_close(actual, expected, rtol=rtol, atol=atol)
    except AssertionError as exc:
        raise AssertionError(f"{what} (rtol={rtol}, atol={atol}):\n{exc}") from exc
