"""ctypes binding of liblumen_b200.so (the C-ABI declared in include/lumen_b200.h).

There is no fallback: if the shared library is missing or does not export a
declared symbol, loading raises.
"""
from __future__ import annotations

import ctypes
from ctypes import c_char_p, c_float, c_int, c_size_t, c_void_p
from pathlib import Path

from ._build import LIB_PATH

OK = 0
EINVAL = -1
EWORKSPACE = -2
ECUDA = -3
EUNSUPPORTED = -4
EDEVICE = -5
ESCRATCH_LIMIT = -6

ERROR_NAMES = {
    EINVAL: "LUMEN_B200_EINVAL (bad pointer, size or pitch)",
    EWORKSPACE: "LUMEN_B200_EWORKSPACE (scratch buffer too small)",
    ECUDA: "LUMEN_B200_ECUDA (CUDA runtime/driver error)",
    EUNSUPPORTED: "LUMEN_B200_EUNSUPPORTED (shape not covered)",
    EDEVICE: "LUMEN_B200_EDEVICE (a kernel wait gave up)",
    ESCRATCH_LIMIT: "LUMEN_B200_ESCRATCH_LIMIT (shape exceeds the built-in scratch array)",
}

# name -> (restype, argtypes); mirrors include/lumen_b200.h
SIGNATURES = {
    "lumen_b200_version": (c_char_p, []),
    "lumen_b200_sm_count": (c_int, []),
    "lumen_b200_device_status": (c_int, [ctypes.POINTER(c_int)]),
    "lumen_b200_clear_status": (c_int, []),
    "lumen_b200_status_snapshot": (c_int, [c_void_p, c_void_p]),
    "lumen_b200_moe_ep_set_wait_limit_ns": (c_int, [ctypes.c_ulonglong]),
    "lumen_b200_gemm_bf16_nt": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_size_t,
         c_void_p],
    ),
    "lumen_b200_gemm_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "lumen_b200_gemm_bf16_nt_static": (
        c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "lumen_b200_gemm_static_scratch_limit": (c_size_t, []),
    "lumen_b200_fa_fwd_bf16": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_float, c_int,
         c_void_p],
    ),
    "lumen_b200_fa_fwd_varlen_bf16": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
         c_float, c_int, c_void_p],
    ),
    "lumen_b200_moe_router_logits": (
        c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "lumen_b200_moe_route_topk": (
        c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "lumen_b200_moe_sort_scratch_bytes": (c_size_t, [c_int, c_int, c_int]),
    "lumen_b200_moe_sort_routes": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_size_t, c_int, c_int, c_int, c_int, c_void_p],
    ),
    "lumen_b200_moe_permute_rows": (
        c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "lumen_b200_moe_grouped_gemm": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
         c_void_p],
    ),
    "lumen_b200_moe_ep_plan": (
        c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "lumen_b200_moe_ep_dispatch": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.POINTER(c_void_p), c_int,
         c_int, c_int, c_int, c_int, c_int, c_void_p],
    ),
    "lumen_b200_moe_ep_return": (
        c_int,
        [c_void_p, c_void_p, c_void_p, ctypes.POINTER(c_void_p), c_int, c_int, c_int, c_int, c_int,
         c_void_p],
    ),
    "lumen_b200_moe_grouped_gemm_to_rows": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
         c_void_p],
    ),
    "lumen_b200_moe_ep_row_ptrs": (
        c_int,
        [c_void_p, c_void_p, ctypes.POINTER(c_void_p), c_int, c_int, c_int, c_int, c_int, c_void_p,
         c_void_p],
    ),
    "lumen_b200_moe_dequant_fp8": (
        c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "lumen_b200_moe_gather_scales_t": (
        c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "lumen_b200_moe_grouped_gemm_fp8": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
         c_int, c_int, c_int, c_float, c_int, c_void_p],
    ),
    "lumen_b200_moe_ep_barrier": (
        c_int, [c_int, c_int, ctypes.POINTER(c_void_p), c_void_p, c_int, c_void_p]),
    "lumen_b200_moe_ep_exchange_counts": (
        c_int,
        [c_void_p, c_int, c_int, c_int, ctypes.POINTER(c_void_p), ctypes.POINTER(c_void_p), c_void_p,
         c_int, c_void_p],
    ),
    "lumen_b200_moe_combine": (
        c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "lumen_b200_moe_forward_scratch_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "lumen_b200_moe_forward": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
         c_int, c_int, c_int, c_int, c_int, c_void_p],
    ),
}

_lib = None


class LumenB200Error(RuntimeError):
    """A C-ABI call returned a negative code."""

    def __init__(self, fn: str, code: int):
        self.code = code
        super().__init__(f"{fn} failed: {ERROR_NAMES.get(code, code)}")


def load(path: Path | None = None) -> ctypes.CDLL:
    """Load the shared library and bind every declared symbol (raises if one is missing)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"{p} is missing: build it with `python __graft_entry__.py` "
            "(there is no CPU or PyTorch fallback for these operators)"
        )
    lib = ctypes.CDLL(str(p))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError if the symbol is not exported
        fn.restype = restype
        fn.argtypes = argtypes
    if path is None:
        _lib = lib
    return lib


def check(fn: str, code: int) -> None:
    if code != OK:
        raise LumenB200Error(fn, code)


class _NoSwitch:
    def __enter__(self):
        return None

    def __exit__(self, *exc):
        return False


_NO_SWITCH = _NoSwitch()


def on_device(device):
    """Context that makes `device` current for a C-ABI call; free when it already is."""
    import torch

    idx = device.index if device.index is not None else torch.cuda.current_device()
    if torch.cuda.current_device() == idx:
        return _NO_SWITCH
    return torch.cuda.device(idx)
