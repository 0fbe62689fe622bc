"""B200 (sm_100a) implementation of the inference-kernel path of lumen-sosp26-ae:
BF16 GEMM, flash-attention forward and fused MoE forward, behind a C-ABI shared
library (liblumen_b200.so) with thin PyTorch host wrappers.

The directory name is not a Python identifier; import it with
``importlib.import_module("lumen-sosp26-ae_b200")``.
"""
from . import _cabi  # noqa: F401
from ._build import LIB_PATH, build_library, library_is_current  # noqa: F401
from .gemm import clear_status, device_status, gemm_pipeline_transposed_b, gemm_workspace_bytes  # noqa: F401
from . import attention, moe, moe_ep, sharding  # noqa: F401
from .attention import flash_attn, flash_attn_packed  # noqa: F401
