"""The allocation-free GEMM entry point against the ordinary one.

lumen_b200_gemm_bf16_nt_static is for callers that may not allocate device memory (code
inside a stream capture, plugins that own nothing but their inputs and outputs, processes
with a closed memory pool): its split-K scratch is an array built into the library.  This
test calls it through the C-ABI twice in a row, with different shapes, so that the second
call starts from whatever the first one left in the shared array, and compares each result
with lumen_b200_gemm_bf16_nt on the same operands.  It is collected last on purpose.
"""
from __future__ import annotations

import pytest
import torch

from conftest import ATOL, RTOL
from oracle import gemm_oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def both_entry_points(pkg, m, n, k, seed):
    lib = pkg._cabi.load()
    a, b = gemm_oracle.gemm_inputs(m, n, k, seed, b_std=0.02)
    a, b = a.to(DEV), b.to(DEV)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    # ordinary entry point, caller-owned workspace
    nbytes = int(lib.lumen_b200_gemm_workspace_bytes(m, n, k))
    ws = torch.zeros(max(nbytes, 16), dtype=torch.uint8, device=DEV)
    want = torch.empty((m, n), dtype=torch.bfloat16, device=DEV)
    rc = lib.lumen_b200_gemm_bf16_nt(a.data_ptr(), b.data_ptr(), want.data_ptr(), m, n, k, k, k, n,
                                      ws.data_ptr() if nbytes else None, nbytes, stream)
    assert rc == 0
    # allocation-free entry point: inputs and output only
    got = torch.empty((m, n), dtype=torch.bfloat16, device=DEV)
    rc = lib.lumen_b200_gemm_bf16_nt_static(a.data_ptr(), b.data_ptr(), got.data_ptr(), m, n, k, k, k, n, stream)
    assert rc == 0
    torch.cuda.synchronize()
    return got.cpu(), want.cpu(), nbytes


def test_static_scratch_gemm_matches_on_two_calls_in_a_row(cuda_pkg):
    lib = cuda_pkg._cabi.load()
    limit = int(lib.lumen_b200_gemm_static_scratch_limit())
    assert limit == 16 << 20
    # first call: 32 output tiles x 4 K slices of 128 rows; second call: a different tile
    # shape and slice count, so stale counters or partial sums of the first would show
    used = []
    for (m, n, k, seed) in ((128, 4096, 4096, 1), (16, 6144, 4096, 2)):
        got, want, nbytes = both_entry_points(cuda_pkg, m, n, k, seed)
        used.append(nbytes)
        torch.testing.assert_close(got.float(), want.float(), rtol=RTOL, atol=ATOL)
    assert all(0 < u <= limit for u in used), "both shapes must exercise the split-K scratch"
    assert cuda_pkg.device_status() == 0


def test_static_scratch_gemm_refuses_what_it_cannot_hold(cuda_pkg):
    lib = cuda_pkg._cabi.load()
    a = torch.zeros((128, 4096), dtype=torch.bfloat16, device=DEV)
    b = torch.zeros((1024, 4096), dtype=torch.bfloat16, device=DEV)
    c = torch.zeros((256, 1024), dtype=torch.bfloat16, device=DEV)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    # M > 128 has no scratch-using path
    rc = lib.lumen_b200_gemm_bf16_nt_static(a.data_ptr(), b.data_ptr(), c.data_ptr(), 256, 1024, 4096,
                                             4096, 4096, 1024, stream)
    assert rc == cuda_pkg._cabi.EUNSUPPORTED
    # a plan larger than the array: M = 128 with a long K is cut into many slices
    m, n, k = 128, 4096, 14336
    need = int(lib.lumen_b200_gemm_workspace_bytes(m, n, k))
    if need > int(lib.lumen_b200_gemm_static_scratch_limit()):
        a = torch.zeros((m, k), dtype=torch.bfloat16, device=DEV)
        b = torch.zeros((n, k), dtype=torch.bfloat16, device=DEV)
        c = torch.zeros((m, n), dtype=torch.bfloat16, device=DEV)
        rc = lib.lumen_b200_gemm_bf16_nt_static(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, k, k, n, stream)
        assert rc == cuda_pkg._cabi.ESCRATCH_LIMIT
    torch.cuda.synchronize()
