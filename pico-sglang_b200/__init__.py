"""B200-native tensor-parallel linear path for pico-sglang.

Drop-in replacements for the reference's TP linear layers, fused
residual-add + RMSNorm and PyNCCL communicator, running hand-written
sm_100a kernels from libpgb.so (C ABI: include/pgb.h).

The directory name contains a hyphen, so import it with
``importlib.import_module("pico-sglang_b200")``.
"""

from . import _lib, ops
from ._lib import PGBError, PGBTimeout
from .ops import col_gemm, fused_add_rmsnorm, rmsnorm, row_gemm_allreduce_addnorm

__all__ = [
    "PGBError",
    "PGBTimeout",
    "_lib",
    "col_gemm",
    "fused_add_rmsnorm",
    "ops",
    "rmsnorm",
    "row_gemm_allreduce_addnorm",
]
