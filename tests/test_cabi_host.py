"""The C-ABI library builds, loads and exports every symbol include/lumen_b200.h
declares; the host wrappers validate like the reference's and never compute on the CPU."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from conftest import REPO


def declared_symbols() -> list[str]:
    text = (REPO / "include" / "lumen_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lumen_b200_\w+)\s*\(", text)))


def test_header_declares_the_path():
    names = declared_symbols()
    for needed in ("lumen_b200_gemm_bf16_nt", "lumen_b200_fa_fwd_bf16", "lumen_b200_moe_route_topk",
                   "lumen_b200_moe_sort_routes", "lumen_b200_moe_grouped_gemm", "lumen_b200_moe_combine"):
        assert needed in names


def test_library_exports_every_declared_symbol(pkg):
    lib = ctypes.CDLL(str(pkg.LIB_PATH))
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} is declared in the header but not exported"


def test_binding_table_matches_header(pkg):
    assert sorted(pkg._cabi.SIGNATURES) == declared_symbols()


def test_version_string(pkg):
    assert b"sm_100a" in pkg._cabi.load().lumen_b200_version()


def test_missing_library_fails_loudly(pkg, tmp_path):
    with pytest.raises(RuntimeError, match="no CPU or PyTorch fallback"):
        pkg._cabi.load(tmp_path / "liblumen_b200.so")


def test_gemm_validation_like_reference(pkg):
    f = pkg.gemm_pipeline_transposed_b
    a = torch.zeros((4, 8), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="A must have dtype torch.bfloat16"):
        f(a.float(), a)
    with pytest.raises(ValueError, match="B must have dtype torch.bfloat16"):
        f(a, a.float())
    with pytest.raises(ValueError, match="A must be 2D"):
        f(a[0], a)
    with pytest.raises(ValueError, match=r"B.shape\[1\] must equal K=8"):
        f(a, torch.zeros((4, 16), dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="no CPU path"):
        f(a, a)


def test_moe_host_validation(pkg):
    with pytest.raises(ValueError, match="no CPU path"):
        pkg.moe.route_topk(torch.zeros((2, 8)), 2)
    assert pkg.moe.max_padded_routes(4096, 2, 8) == 4096 * 2 + 8 * 32 - 2
