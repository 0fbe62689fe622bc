"""GPU parity of the BF16 GEMM (through the C-ABI) against the CPU oracle."""
from __future__ import annotations

import pytest
import torch

from conftest import ATOL, RTOL, load_golden
from oracle import gemm_oracle

pytestmark = pytest.mark.gpu


def run_gemm(pkg, a, b):
    dev = torch.device("cuda:0")
    out = pkg.gemm_pipeline_transposed_b(a.to(dev), b.to(dev))
    torch.cuda.synchronize()
    assert pkg.device_status() == 0
    return out.cpu()


@pytest.mark.parametrize("case", ["small", "ragged"])
def test_golden_fixture(cuda_pkg, case):
    g = load_golden("gemm")
    out = run_gemm(cuda_pkg, g[f"{case}_a"], g[f"{case}_b"])
    torch.testing.assert_close(out.float(), g[f"{case}_out"].float(), rtol=RTOL, atol=ATOL)


# edge cases the reference kernels reject (K % 64 != 0, partial tiles) and the M values of
# the shape sweep; sizes kept small enough for the fp32 CPU oracle
SHAPES = [
    (1, 128, 64), (1, 4096, 4096), (16, 256, 128), (16, 6144, 4096), (17, 200, 72),
    (33, 136, 264), (64, 128, 512), (100, 1000, 520), (128, 4096, 1024), (128, 128, 64),
    (129, 256, 64), (256, 256, 256), (300, 520, 136), (1024, 1024, 1024), (384, 2304, 1536),
]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_matches_oracle(cuda_pkg, m, n, k):
    a, b = gemm_oracle.gemm_inputs(m, n, k, seed=20260312 + m + n + k)
    out = run_gemm(cuda_pkg, a, b)
    want = gemm_oracle.gemm_reference(a, b)
    torch.testing.assert_close(out.float(), want.float(), rtol=RTOL, atol=ATOL)


def test_exact_on_integer_valued_inputs(cuda_pkg):
    """Small integers are exact in bf16 and their dot products exact in fp32: the GEMM
    must reproduce the oracle bit for bit (catches any operand/tile mix-up)."""
    g = torch.Generator().manual_seed(5)
    a = torch.randint(-3, 4, (260, 320), generator=g).to(torch.bfloat16)
    b = torch.randint(-3, 4, (520, 320), generator=g).to(torch.bfloat16)
    out = run_gemm(cuda_pkg, a, b)
    assert torch.equal(out, gemm_oracle.gemm_reference(a, b))
    out = run_gemm(cuda_pkg, a[:9], b)
    assert torch.equal(out, gemm_oracle.gemm_reference(a[:9], b))


# Shapes whose last round of 256 x 256 tiles fills at most half of the CTA pairs, so that its
# tiles are computed as K slices and summed through the workspace (ragged edges included), and
# one whose tile count divides evenly (no split).
TAIL_SHAPES = [(1000, 6000, 2048), (1024, 6144, 4096), (2048, 2560, 1024), (4096, 4096, 1536), (2048, 9472, 512)]


@pytest.mark.parametrize("m,n,k", TAIL_SHAPES)
def test_split_last_wave_matches_oracle_rows(cuda_pkg, m, n, k):
    dev = torch.device("cuda:0")
    a, b = gemm_oracle.gemm_inputs(m, n, k, seed=20260312 + m + n + k)
    ad, bd = a.to(dev), b.to(dev)
    out = cuda_pkg.gemm_pipeline_transposed_b(ad, bd)
    again = cuda_pkg.gemm_pipeline_transposed_b(ad, bd)
    torch.cuda.synchronize()
    assert cuda_pkg.device_status() == 0
    # the slices are added in slice order, whichever arrives last: bit-identical from run to run
    assert torch.equal(out, again)
    # every tile row and column band, the last (split) tiles included
    rows = torch.unique(torch.cat([torch.arange(0, m, 37), torch.arange(max(0, m - 300), m, 7)]))
    want = gemm_oracle.gemm_reference(a[rows], b)
    torch.testing.assert_close(out[rows.to(dev)].cpu().float(), want.float(), rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("m,n,k", [(128, 512, 4096), (16, 1792, 14336), (100, 1000, 4104)])
def test_split_k_slices_add_in_a_fixed_order(cuda_pkg, m, n, k):
    """Few rows, long K: up to 16 K slices per tile add their partial sums like a reduce-scatter.
    The order of the additions is fixed, so two runs agree bit for bit; rows against the oracle."""
    dev = torch.device("cuda:0")
    a, b = gemm_oracle.gemm_inputs(m, n, k, seed=7 + m + n + k)
    ad, bd = a.to(dev), b.to(dev)
    out = cuda_pkg.gemm_pipeline_transposed_b(ad, bd)
    again = cuda_pkg.gemm_pipeline_transposed_b(ad, bd)
    torch.cuda.synchronize()
    assert cuda_pkg.device_status() == 0
    assert torch.equal(out, again)
    torch.testing.assert_close(out.cpu().float(), gemm_oracle.gemm_reference(a, b).float(), rtol=RTOL, atol=ATOL)


def test_split_last_wave_is_exact_on_integers_and_optional(cuda_pkg):
    """Integer-valued operands: every partial sum is exact, so the split result equals the
    oracle bit for bit; the same call without a workspace (no split) must agree."""
    import ctypes

    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(11)
    m, n, k = 1024, 6144, 1024
    a = torch.randint(-3, 4, (m, k), generator=g).to(torch.bfloat16)
    b = torch.randint(-3, 4, (n, k), generator=g).to(torch.bfloat16)
    ad, bd = a.to(dev), b.to(dev)
    assert cuda_pkg.gemm_workspace_bytes(m, n, k) > 0  # this shape has a tail to split
    out = cuda_pkg.gemm_pipeline_transposed_b(ad, bd)
    plain = torch.empty_like(out)
    lib = cuda_pkg._cabi.load()
    rc = lib.lumen_b200_gemm_bf16_nt(ad.data_ptr(), bd.data_ptr(), plain.data_ptr(), m, n, k, k, k, n, None, 0,
                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert cuda_pkg.device_status() == 0
    want = gemm_oracle.gemm_reference(a[::5], b)
    assert torch.equal(out.cpu()[::5], want)
    assert torch.equal(out, plain)


@pytest.mark.parametrize("world", [4, 8])
def test_column_shards_of_the_sweep(cuda_pkg, world):
    """Every shape of the benchmark sweep at the width one rank of `world` GPUs computes (N / world
    columns): narrow problems take other tile plans (K slices, split last waves) than the full-width
    ones.  Checked on the device against an fp32 matmul of the same bf16 operands."""
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(20260312)
    for m in (1, 16, 128, 1024, 8192):
        for (n, k) in ((4096, 4096), (14336, 4096), (4096, 14336), (6144, 4096)):
            ns = n // world
            a = torch.randn((m, k), device=dev, dtype=torch.bfloat16, generator=g)
            b = (torch.randn((ns, k), device=dev, dtype=torch.float32, generator=g) * 0.02).to(torch.bfloat16)
            out = cuda_pkg.gemm_pipeline_transposed_b(a, b)
            want = a.float() @ b.float().T
            torch.testing.assert_close(out.float(), want, rtol=RTOL, atol=ATOL, msg=lambda s_: f"{m}x{ns}x{k}: {s_}")
    torch.cuda.synchronize()
    assert cuda_pkg.device_status() == 0


def test_caller_owned_output_and_pitch(cuda_pkg):
    dev = torch.device("cuda:0")
    a, b = gemm_oracle.gemm_inputs(200, 264, 128, seed=3)
    big = torch.full((200, 400), 7.0, dtype=torch.bfloat16, device=dev)
    view = big[:, :264]
    ret = cuda_pkg.gemm_pipeline_transposed_b(a.to(dev), b.to(dev), out=view)
    torch.cuda.synchronize()
    assert ret.data_ptr() == view.data_ptr()
    torch.testing.assert_close(view.cpu().float(), gemm_oracle.gemm_reference(a, b).float(), rtol=RTOL, atol=ATOL)
    assert torch.all(big[:, 264:] == 7.0)  # nothing written past N
    with pytest.raises(ValueError, match="result buffer"):
        cuda_pkg.gemm_pipeline_transposed_b(a.to(dev), b.to(dev), out=big)


def test_config1_full_size_rows_and_linearity(cuda_pkg):
    """C = A B^T at 4096^3 with the reference harness' distribution (A, B ~ N(0,1)).
    The oracle checks 96 sampled rows; linearity C(A1 + A2) = C(A1) + C(A2) holds for
    inputs whose products are exact, whatever the size."""
    dev = torch.device("cuda:0")
    a, b = gemm_oracle.gemm_inputs(4096, 4096, 4096, seed=20260312)
    out = run_gemm(cuda_pkg, a, b)
    rows = torch.randperm(4096, generator=torch.Generator().manual_seed(1))[:96]
    want = gemm_oracle.gemm_reference(a[rows], b)
    torch.testing.assert_close(out[rows].float(), want.float(), rtol=RTOL, atol=ATOL)
    g = torch.Generator().manual_seed(2)
    a1 = torch.randint(-2, 3, (4096, 4096), generator=g).to(torch.bfloat16)
    a2 = torch.randint(-2, 3, (4096, 4096), generator=g).to(torch.bfloat16)
    bi = torch.randint(-1, 2, (4096, 4096), generator=g).to(torch.bfloat16)
    c1 = run_gemm(cuda_pkg, a1, bi).float()
    c2 = run_gemm(cuda_pkg, a2, bi).float()
    c12 = run_gemm(cuda_pkg, (a1 + a2), bi).float()
    # |entries| <= 4 * 4096 * 1 is exact in bf16 only below 256 (257 already rounds); compare where exact
    exact = (c1.abs() < 256) & (c2.abs() < 256) & (c12.abs() < 256)
    assert exact.float().mean() > 0.5
    assert torch.equal((c1 + c2)[exact], c12[exact])


@pytest.mark.parametrize("m", [1, 16, 128, 1024, 8192])
@pytest.mark.parametrize("n,k", [(4096, 4096), (14336, 4096), (4096, 14336), (6144, 4096)])
def test_config2_sweep_sampled(cuda_pkg, m, n, k):
    """Shape sweep (A ~ N(0,1), B ~ N(0,0.02)); oracle on a sample of rows and columns."""
    a, b = gemm_oracle.gemm_inputs(m, n, k, seed=20260312, b_std=0.02)
    out = run_gemm(cuda_pkg, a, b)
    g = torch.Generator().manual_seed(m + n)
    rows = torch.randperm(m, generator=g)[: min(m, 24)]
    cols = torch.randperm(n, generator=g)[:512]
    want = gemm_oracle.gemm_reference(a[rows], b[cols])
    torch.testing.assert_close(out[rows][:, cols].float(), want.float(), rtol=RTOL, atol=ATOL)
