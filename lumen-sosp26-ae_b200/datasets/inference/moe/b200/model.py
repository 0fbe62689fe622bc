"""B200 system for datasets/inference/moe: fused MoE forward in bf16.

    python scripts/benchmark/bench_moe.py --backend lumen --input-dtype bf16 \
        --model-path <this file> --check-correctness

`Model(variant=...).build_cases(...)` follows the case-backend contract
(scripts/benchmark/backend_moe.py:263-336): it receives the harness' precomputed routing
(topk_ids, topk_weights) and returns zero-argument callables.  `ModelNew.forward` follows
the python-backend contract (:339-403).

fp8 input (the harness default): codes and block scales go to the kernels as they are; both
expert GEMMs multiply fp8 on the tensor cores and apply the scales per 128-wide K block, the
intermediate is re-quantised per row like the reference kernel does
(datasets/inference/moe/lumen/fused_moe.py:400-443, 684-788).  Needs hidden and intermediate sizes
that are multiples of 128 (the harness requires that too).  By default this route serves the
token counts at which the expert GEMMs stream weights (up to 64 rows per expert); above that,
and always with LUMEN_B200_MOE_FP8=dequant, codes and scales are folded into bf16 copies of the
weights once, outside the timed call, the activations are dequantised in every call and the
GEMMs compute in bf16.  LUMEN_B200_MOE_FP8=mma forces the fp8 kernels at every size.

bf16 input: the expert GEMMs compute in bf16; non-unit block scales are folded into bf16 copies
of the weights once, outside the timed call, the way the reference's Lumen system pre-shuffles
its weights (datasets/inference/moe/lumen/model.py:184-199).
"""
from __future__ import annotations

import importlib.util
import os
from pathlib import Path
from typing import Any, Callable, List

import torch
import torch.nn as nn


def _find_loader() -> Path:
    """_loader.py sits two directories above this file.  An evaluator that executes this
    file's source text instead of importing it by path (no usable __file__, the
    KernelBench way: python/lumen/harness/datasets/kernelbench/evaluator.py:158-167) names
    the directory that contains the package in the environment variable LUMEN_B200_ROOT."""
    places = []
    here = globals().get("__file__")
    if here:
        places += [p / "_loader.py" for p in list(Path(here).resolve().parents)[2:3]]
    if os.environ.get("LUMEN_B200_ROOT"):
        places.append(Path(os.environ["LUMEN_B200_ROOT"]) / "lumen-sosp26-ae_b200" / "datasets" / "inference" / "_loader.py")
    for place in places:
        if place.is_file():
            return place
    raise ImportError("cannot locate the lumen-sosp26-ae_b200 package: import this file by its path "
                      "inside the package, or set LUMEN_B200_ROOT to the directory that contains the package")


_spec = importlib.util.spec_from_file_location("_b200_dataset_loader", _find_loader())
_loader = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(_loader)
_pkg = _loader.load_b200_package()
_moe = _pkg.moe

BLOCK = 128


FP8_KERNEL_ROWS = 64  # rows per expert up to which the fp8 kernels are the faster route


def _use_fp8_kernels(tokens: int, topk: int, experts: int) -> bool:
    """LUMEN_B200_MOE_FP8 = "mma": always the fp8 tensor-core kernels; "dequant": never; unset:
    the fp8 kernels while the expert GEMMs stream weights (few rows per expert, where half the
    bytes is close to half the time), the bf16 route above that (its 128 x 256 tiles have the
    higher tensor-core rate; the fp8 kernels promote partial sums on CUDA cores per K block)."""
    mode = os.environ.get("LUMEN_B200_MOE_FP8", "")
    if mode == "mma":
        return True
    if mode == "dequant":
        return False
    return tokens * topk <= FP8_KERNEL_ROWS * experts


def _tensor_key(t: torch.Tensor) -> tuple:
    """Identity of a tensor's present contents: same storage, same shape, no in-place write
    since (tensors made under torch.inference_mode keep no version counter)."""
    try:
        version = t._version
    except RuntimeError:
        version = -1
    return (t.data_ptr(), tuple(t.shape), t.dtype, version)


_unit_scale_seen: dict = {}


def _is_unit_scale(scale: torch.Tensor) -> bool:
    """Whether every scale equals 1.  Reading that back is a device-to-host synchronisation,
    so it happens once per scale tensor (keyed on its storage and version) and never again:
    later calls, including calls made while a CUDA graph is being captured, reuse the answer."""
    key = _tensor_key(scale)
    hit = _unit_scale_seen.get(key)
    if hit is None:
        if len(_unit_scale_seen) > 256:
            _unit_scale_seen.clear()
        hit = bool(torch.all(scale == 1.0))
        _unit_scale_seen[key] = hit
    return hit


def _fold_block_scale(w: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """w [E, rows, cols] (bf16 or fp8) times scale [E, (rows/128)*(cols/128)] -> bf16."""
    if w.dtype == torch.bfloat16 and _is_unit_scale(scale):
        return w
    E, rows, cols = w.shape
    out = torch.empty((E, rows, cols), dtype=torch.bfloat16, device=w.device)
    s = scale.to(torch.float32).view(E, rows // BLOCK, 1, cols // BLOCK, 1)
    for e in range(E):  # per expert: keeps the fp32 temporaries small
        wf = w[e].to(torch.float32).view(rows // BLOCK, BLOCK, cols // BLOCK, BLOCK) * s[e]
        out[e] = wf.view(rows, cols).to(torch.bfloat16)
    return out


def _fold_input_scale(x: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """bf16 activations times their per-128 scales, on the device, with no host read."""
    T, H = x.shape
    xf = x.to(torch.float32).view(T, H // BLOCK, BLOCK) * scale.to(torch.float32).unsqueeze(-1)
    return xf.view(T, H).to(torch.bfloat16)


class Model:
    def __init__(self, *, variant: str = "b200"):
        self.variant = variant
        self._out_cache: dict = {}
        self._ops: dict = {}
        self._weight_key = None
        self._weights = None

    def _prepare_weights(self, w: dict[str, torch.Tensor]):
        # the folded copies depend on the scales as much as on the codes
        key = tuple(_tensor_key(w[name]) for name in ("w1_q", "fc1_scale", "w2_q", "fc2_scale"))
        if self._weights is None or key != self._weight_key:
            self._weights = (_fold_block_scale(w["w1_q"], w["fc1_scale"]),
                             _fold_block_scale(w["w2_q"], w["fc2_scale"]))
            self._weight_key = key
        return self._weights

    def _fp8_case(self, x, w, seq_len, dim, inter_dim, experts, topk) -> Callable[[], torch.Tensor]:
        """fp8 codes and block scales straight into the fp8 kernels."""
        dev = x.input_q.device
        key = ("fp8", seq_len, dim, inter_dim, experts, topk, dev)
        op = self._ops.get(key)
        if op is None:
            op = _moe.FusedMoEFp8(tokens=seq_len, hidden=dim, inter=inter_dim, experts=experts, topk=topk, device=dev)
            self._ops[key] = op
        self._out_cache[key] = op.out
        xq, xscale = x.input_q.contiguous(), x.input_scale.to(torch.float32).contiguous()
        ids = x.topk_ids.to(torch.int32).contiguous()
        wts = x.topk_weights.to(torch.float32).contiguous()
        w1q, w2q = w["w1_q"].contiguous(), w["w2_q"].contiguous()
        s1, s2 = w["fc1_scale"].to(torch.float32).contiguous(), w["fc2_scale"].to(torch.float32).contiguous()

        def run_b200_fp8() -> torch.Tensor:
            return op.forward_routed(xq, xscale, ids, wts, w1q, s1, w2q, s2)

        return run_b200_fp8

    def build_cases(self, *, seq_len: int, shared_input: Any, shared_weights: dict[str, torch.Tensor],
                    dim: int, inter_dim: int, experts: int, topk: int,
                    input_dtype: str) -> List[Callable[[], torch.Tensor]]:
        if input_dtype not in ("bf16", "fp8"):
            raise ValueError("B200 MoE supports bf16 and fp8 input")
        x = shared_input
        for name in ("input_q", "topk_weights", "topk_ids", "input_scale"):
            if not hasattr(x, name):
                raise ValueError(f"shared_input missing field: {name}")
        if tuple(x.input_q.shape) != (seq_len, dim):
            raise ValueError(f"input_q shape mismatch: expected {(seq_len, dim)}, got {tuple(x.input_q.shape)}")
        if tuple(x.topk_ids.shape) != (seq_len, topk):
            raise ValueError(f"topk_ids shape mismatch: expected {(seq_len, topk)}, got {tuple(x.topk_ids.shape)}")
        if tuple(shared_weights["w1_q"].shape) != (experts, inter_dim * 2, dim):
            raise ValueError(f"w1_q shape mismatch: expected {(experts, inter_dim * 2, dim)}, "
                             f"got {tuple(shared_weights['w1_q'].shape)}")
        fp8_in = x.input_q.dtype != torch.bfloat16
        if fp8_in and shared_weights["w1_q"].dtype == x.input_q.dtype and dim % BLOCK == 0 \
                and inter_dim % BLOCK == 0 and _use_fp8_kernels(seq_len, topk, experts):
            return [self._fp8_case(x, shared_weights, seq_len, dim, inter_dim, experts, topk)]
        w13, w2 = self._prepare_weights(shared_weights)
        # fp8 activations are dequantised by a kernel inside the timed call (they arrive as
        # fp8); bf16 activations with non-unit scales are scaled inside the call as well
        # (device arithmetic only), so that the closure always reads the caller's tensor
        unit_in = fp8_in or _is_unit_scale(x.input_scale)
        dev = x.input_q.device
        key = (seq_len, dim, inter_dim, experts, topk, dev)
        op = self._ops.get(key)
        if op is None:
            op = _moe.FusedMoE(tokens=seq_len, hidden=dim, inter=inter_dim, experts=experts, topk=topk, device=dev)
            self._ops[key] = op
        self._out_cache[key] = op.out
        ids = x.topk_ids.to(torch.int32).contiguous()
        wts = x.topk_weights.to(torch.float32).contiguous()

        if fp8_in:
            xq, xscale = x.input_q.contiguous(), x.input_scale.to(torch.float32).contiguous()
            xbuf = torch.empty((seq_len, dim), dtype=torch.bfloat16, device=dev)

            def run_b200() -> torch.Tensor:
                _moe.dequant_fp8_rows(xq, xscale, out=xbuf)
                return op.forward_routed(xbuf, ids, wts, w13, w2)
        elif unit_in:
            xin = x.input_q.contiguous()

            def run_b200() -> torch.Tensor:
                return op.forward_routed(xin, ids, wts, w13, w2)
        else:
            xraw, xscale = x.input_q, x.input_scale

            def run_b200() -> torch.Tensor:
                return op.forward_routed(_fold_input_scale(xraw, xscale), ids, wts, w13, w2)

        return [run_b200]


class ModelNew(nn.Module):
    """forward(input_q, w1_q, w2_q, topk_weights, topk_ids, input_scale, fc1_scale, fc2_scale)."""

    def __init__(self):
        super().__init__()
        self._impl = Model(variant="b200")

    def forward(self, input_q, w1_q, w2_q, topk_weights, topk_ids, input_scale, fc1_scale, fc2_scale):
        class _In:
            pass

        s = _In()
        s.input_q, s.topk_weights, s.topk_ids, s.input_scale = input_q, topk_weights, topk_ids, input_scale
        T, H = input_q.shape
        E, two_i, _ = w1_q.shape
        weights = {"w1_q": w1_q, "w2_q": w2_q, "fc1_scale": fc1_scale, "fc2_scale": fc2_scale}
        return self._impl.build_cases(seq_len=T, shared_input=s, shared_weights=weights, dim=H,
                                      inter_dim=two_i // 2, experts=E, topk=topk_ids.shape[1],
                                      input_dtype="bf16" if input_q.dtype == torch.bfloat16 else "fp8")[0]()


# Defaults of get_inputs(): the Mixtral-like configuration.  An evaluator may override any
# of them by setting a module-global EVAL_CONFIG dict (keys tokens, dim, inter_dim, experts,
# topk, seed, device) before calling get_inputs(), the convention of the reference's
# KernelBench-style MoE system (datasets/inference/moe/kernelbench/model.py:347-441).
DEFAULTS = {"tokens": 4096, "dim": 4096, "inter_dim": 14336, "experts": 8, "topk": 2, "seed": 20260319,
            "device": "cpu"}


def _eval_config() -> dict:
    cfg = dict(DEFAULTS)
    raw = globals().get("EVAL_CONFIG", {})
    if isinstance(raw, dict):
        for key, default in DEFAULTS.items():
            if key not in raw:
                continue
            try:
                cfg[key] = type(default)(raw[key])
            except (TypeError, ValueError):
                pass
    cfg["topk"] = max(1, min(cfg["topk"], cfg["experts"]))
    return cfg


def get_inputs():
    """Stand-in inputs (x ~ N(0,1), weights ~ N(0,0.02), unit block scales) in the argument
    order of ModelNew.forward."""
    c = _eval_config()
    T, D, I, E, K = c["tokens"], c["dim"], c["inter_dim"], c["experts"], c["topk"]
    g = torch.Generator().manual_seed(c["seed"])
    x = torch.randn((T, D), generator=g, dtype=torch.float32).to(torch.bfloat16)
    scores = torch.randn((T, E), generator=g, dtype=torch.float32)
    tv, ti = torch.topk(scores, k=K, dim=-1, largest=True, sorted=True)
    gw = torch.Generator().manual_seed(c["seed"] + 17)
    w1 = torch.empty((E, 2 * I, D), dtype=torch.bfloat16)
    w2 = torch.empty((E, D, I), dtype=torch.bfloat16)
    for e in range(E):  # per expert: keeps the fp32 temporaries small
        w1[e] = (torch.randn((2 * I, D), generator=gw, dtype=torch.float32) * 0.02).to(torch.bfloat16)
    for e in range(E):
        w2[e] = (torch.randn((D, I), generator=gw, dtype=torch.float32) * 0.02).to(torch.bfloat16)
    ones = lambda *s: torch.ones(s, dtype=torch.float32)  # noqa: E731
    out = [x, w1, w2, torch.softmax(tv, dim=-1), ti.to(torch.int32), ones(T, D // BLOCK),
           ones(E, (2 * I // BLOCK) * (D // BLOCK)), ones(E, (D // BLOCK) * (I // BLOCK))]
    dev = torch.device(c["device"])
    return [t.to(dev) for t in out] if dev.type != "cpu" else out


def get_init_inputs():
    return []


__all__ = ["Model", "ModelNew", "get_inputs", "get_init_inputs"]
