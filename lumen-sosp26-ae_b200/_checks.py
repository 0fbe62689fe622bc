"""Argument checks shared by the three host wrappers.

One table-driven checker instead of a chain of `if` statements per wrapper: each wrapper
describes its tensors (name, rank, layout words) once and the checker reports the first
rule a tensor breaks.  The exception *types* follow the reference's wrappers, which is the
part of their behaviour callers can depend on: the GEMM wrapper raises ValueError for every
bad argument (datasets/inference/gemm/lumen/amdgpu_gemm.py:879-911); the attention wrapper
raises TypeError for a wrong dtype or a non-tensor and ValueError for everything else
(datasets/inference/attention/lumen/attn_06_inst_scheduling.py:108-165, 2152-2177).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Operand:
    name: str
    tensor: torch.Tensor
    layout: str              # e.g. "[M, K]": printed when the rank is wrong
    contiguous: bool = True  # False: only the innermost stride has to be 1


def check_operands(op: str, operands: list[Operand], *, dtype: torch.dtype, dtype_error: type) -> torch.device:
    """Every operand is a CUDA tensor of `dtype` with the rank its layout names, laid out as
    the kernels read it, and all of them live on the first operand's device."""
    first = operands[0]
    dev0 = first.tensor.device if isinstance(first.tensor, torch.Tensor) else None

    def rank_of(o: Operand) -> int:
        return o.layout.count(",") + 1

    # one rule at a time over all operands, so that the kind of mistake decides the error
    rules = (
        (lambda o: isinstance(o.tensor, torch.Tensor), TypeError,
         lambda o: f"argument {o.name} is a {type(o.tensor).__name__}, a torch.Tensor is needed"),
        (lambda o: o.tensor.dtype == dtype, dtype_error,
         lambda o: f"{o.name} holds {o.tensor.dtype}; this operator is {dtype} only"),
        (lambda o: o.tensor.ndim == rank_of(o), ValueError,
         lambda o: f"{o.name} has {o.tensor.ndim} dimension(s) {tuple(o.tensor.shape)}; its layout is {o.layout}"),
        (lambda o: o.tensor.is_cuda, ValueError,
         lambda o: f"{o.name} lives on {o.tensor.device}; the kernels run on CUDA devices and there is no CPU path"),
        (lambda o: o.tensor.device == dev0, ValueError,
         lambda o: f"{o.name} lives on {o.tensor.device} but {first.name} on {dev0}"),
        (lambda o: o.tensor.is_contiguous() if o.contiguous else o.tensor.stride(-1) == 1, ValueError,
         lambda o: f"{o.name} {o.layout} has to be " + ("dense (contiguous)" if o.contiguous else
                                                        "row-major (stride 1 along its last dimension)") +
                   f", strides are {o.tensor.stride()}"),
    )
    for holds, error, describe in rules:
        for o in operands:
            if not holds(o):
                raise error(f"{op}: {describe(o)}")
    return first.tensor.device


def check_output(op: str, out: torch.Tensor | None, like_shape: tuple, device: torch.device, *,
                 dtype: torch.dtype, dtype_error: type, contiguous: bool = True) -> torch.Tensor:
    """A caller-owned result buffer must be exactly what the wrapper would allocate."""
    if out is None:
        return torch.empty(like_shape, dtype=dtype, device=device)
    if tuple(out.shape) != tuple(like_shape):
        raise ValueError(f"{op}: result buffer is {tuple(out.shape)}, the result is {tuple(like_shape)}")
    if out.dtype != dtype:
        raise dtype_error(f"{op}: result buffer holds {out.dtype}, the result is {dtype}")
    if out.device != device:
        raise ValueError(f"{op}: result buffer lives on {out.device}, the inputs on {device}")
    if contiguous and not out.is_contiguous() or out.stride(-1) != 1:
        raise ValueError(f"{op}: result buffer has strides {out.stride()}; a dense row-major buffer is needed")
    return out


def require(cond: bool, op: str, what: str, error: type = ValueError) -> None:
    if not cond:
        raise error(f"{op}: {what}")
