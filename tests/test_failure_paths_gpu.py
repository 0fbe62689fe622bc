"""The failure path of the device-side waits, exercised without faulting or hanging a GPU.

Every wait in the library is bounded: when it runs out, the kernel records a code in the
device status word and returns normally, so the context stays usable.  Here a barrier
between two "GPUs" is launched whose second peer is a piece of local memory that nothing
ever signals, with the wait limit set to a few milliseconds: the kernel must come back, the
status word must name the barrier slot and the silent peer, the expert-parallel data
kernels must refuse to move rows while the status is set, and after clear_status() the
next kernels must run clean.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from oracle import gemm_oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
BARRIER_GAVE_UP = 35


def _ptrs(tensors):
    return (ctypes.c_void_p * len(tensors))(*[t.data_ptr() for t in tensors])


def test_barrier_wait_runs_out_and_is_reported(cuda_pkg):
    pkg = cuda_pkg
    lib, check = pkg._cabi.load(), pkg._cabi.check
    stream = torch.cuda.current_stream(DEV).cuda_stream
    pkg.clear_status()
    mine = torch.zeros((64,), dtype=torch.int32, device=DEV)
    silent_peer = torch.zeros((64,), dtype=torch.int32, device=DEV)  # nobody announces anything here
    epochs = torch.zeros((4,), dtype=torch.int32, device=DEV)
    slot = 2
    check("limit", lib.lumen_b200_moe_ep_set_wait_limit_ns(5_000_000))  # 5 ms
    try:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        check("barrier", lib.lumen_b200_moe_ep_barrier(0, 2, _ptrs([mine, silent_peer]), epochs.data_ptr(),
                                                       slot, stream))
        t1.record()
        # the asynchronous status copy sees the code without a device-wide synchronisation
        snap = torch.zeros((1,), dtype=torch.int32).pin_memory()
        check("snapshot", lib.lumen_b200_status_snapshot(snap.data_ptr(), stream))
        torch.cuda.synchronize()
        assert t0.elapsed_time(t1) < 500.0  # returned after about the limit, not after seconds
        want = (BARRIER_GAVE_UP << 16) | (slot << 8) | 1
        assert int(snap.item()) == want
        assert pkg.device_status() == want
        # this GPU did announce its epoch to both arrays before it waited
        assert int(mine[slot * 16].item()) == 1 and int(silent_peer[slot * 16].item()) == 1

        # while the status word is set the exchange kernels move nothing
        H, T = 64, 4
        x = torch.ones((T, H), dtype=torch.bfloat16, device=DEV)
        buf = torch.zeros((T, H), dtype=torch.bfloat16, device=DEV)
        ids = torch.arange(T, dtype=torch.int32, device=DEV)
        zeros = torch.zeros((T,), dtype=torch.int32, device=DEV)
        offsets = torch.tensor([0, T], dtype=torch.int32, device=DEV)
        nvalid = torch.tensor([T, T], dtype=torch.int32, device=DEV)
        check("dispatch", lib.lumen_b200_moe_ep_dispatch(
            x.data_ptr(), ids.data_ptr(), zeros.data_ptr(), offsets.data_ptr(), zeros.data_ptr(),
            nvalid.data_ptr(), _ptrs([buf]), 1, T, H, 1, T, T, stream))
        torch.cuda.synchronize()
        assert float(buf.float().abs().sum()) == 0.0

        # reset: the same dispatch now copies, and a tensor-core GEMM runs clean
        pkg.clear_status()
        assert pkg.device_status() == 0
        check("dispatch", lib.lumen_b200_moe_ep_dispatch(
            x.data_ptr(), ids.data_ptr(), zeros.data_ptr(), offsets.data_ptr(), zeros.data_ptr(),
            nvalid.data_ptr(), _ptrs([buf]), 1, T, H, 1, T, T, stream))
        torch.cuda.synchronize()
        assert torch.equal(buf, x)
        a, b = gemm_oracle.gemm_inputs(256, 512, 256, seed=3)
        out = pkg.gemm_pipeline_transposed_b(a.to(DEV), b.to(DEV))
        torch.cuda.synchronize()
        torch.testing.assert_close(out.cpu().float(), gemm_oracle.gemm_reference(a, b).float(), rtol=2e-2, atol=2e-2)
        assert pkg.device_status() == 0
    finally:
        lib.lumen_b200_moe_ep_set_wait_limit_ns(0)  # back to the default
        pkg.clear_status()
