"""Host side of the BF16 GEMM  C[M,N] = A[M,K] * B[N,K]^T  (fp32 accumulation).

`gemm_pipeline_transposed_b` keeps the name, argument meaning and error behaviour of
the reference's host wrapper (datasets/inference/gemm/lumen/amdgpu_gemm.py:872-923):
bf16 2-D inputs, B stored [N,K], optional caller-owned `out`, ValueError on a bad
dtype / rank / shape.  The work is done by lumen_b200_gemm_bf16_nt in
liblumen_b200.so on the current CUDA stream; nothing here computes on the CPU.
"""
from __future__ import annotations

import torch

from . import _cabi
from ._checks import Operand, check_operands, check_output, require

_workspaces: dict[int, torch.Tensor] = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor | None:
    """Split-K scratch of `device`, zero-filled when created and grown on demand (never
    shrunk).  One buffer per device: GEMMs that use it (few activation rows, or a large
    problem whose last wave of tiles is split over K) must not overlap on the GPU (launch
    them on one stream, or pass explicit workspaces through the C-ABI).
    It is created by the first call that needs it, so make that call before capturing a
    CUDA graph; replays then reuse it without a fill."""
    if nbytes == 0:
        return None
    key = device.index if device.index is not None else torch.cuda.current_device()
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 32 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def gemm_workspace_bytes(m: int, n: int, k: int) -> int:
    return int(_cabi.load().lumen_b200_gemm_workspace_bytes(m, n, k))


def gemm_pipeline_transposed_b(
    A: torch.Tensor,
    B: torch.Tensor,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    op = "gemm_pipeline_transposed_b"
    dev = check_operands(op, [Operand("A", A, "[M, K]", contiguous=False),
                              Operand("B", B, "[N, K]", contiguous=False)],
                         dtype=torch.bfloat16, dtype_error=ValueError)
    m, k = A.shape
    n = B.shape[0]
    require(B.shape[1] == k, op, f"A is [{m}, {k}] and B is {tuple(B.shape)}: both need the same K (B is stored [N, K])")
    require(m > 0 and n > 0 and k > 0, op, f"nothing to multiply: M={m}, N={n}, K={k}")
    require(A.stride(0) % 8 == 0 and B.stride(0) % 8 == 0, op,
            f"rows of A and B must start on 16-byte boundaries (pitch a multiple of 8 elements); "
            f"pitches are {A.stride(0)} and {B.stride(0)}")
    out = check_output(op, out, (m, n), dev, dtype=torch.bfloat16, dtype_error=ValueError, contiguous=False)

    lib = _cabi.load()
    with _cabi.on_device(A.device):
        ws = _workspace(A.device, int(lib.lumen_b200_gemm_workspace_bytes(m, n, k)))
        stream = torch.cuda.current_stream(A.device).cuda_stream
        rc = lib.lumen_b200_gemm_bf16_nt(
            A.data_ptr(), B.data_ptr(), out.data_ptr(), m, n, k,
            A.stride(0), B.stride(0), out.stride(0),
            ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
            stream,
        )
    _cabi.check("lumen_b200_gemm_bf16_nt", rc)
    return out


def device_status() -> int:
    """Synchronise and return the device status word (0 = no kernel wait gave up)."""
    import ctypes

    st = ctypes.c_int(0)
    rc = _cabi.load().lumen_b200_device_status(ctypes.byref(st))
    if rc not in (_cabi.OK, _cabi.EDEVICE):
        _cabi.check("lumen_b200_device_status", rc)
    return int(st.value)


def clear_status() -> None:
    _cabi.check("lumen_b200_clear_status", _cabi.load().lumen_b200_clear_status())
