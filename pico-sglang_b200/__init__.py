"""B200-native tensor-parallel linear path for pico-sglang.

Drop-in replacements for the reference's TP linear layers, gated MLP
activation (fused into gate_up_proj), fused residual-add + RMSNorm and
PyNCCL communicator, running hand-written
sm_100a kernels from libpgb.so (C ABI: include/pgb.h).

The directory name contains a hyphen, so import it with
``importlib.import_module("pico-sglang_b200")``.
"""

from . import _lib, ops
from ._lib import PGBError, PGBTimeout
from .ops import col_gemm, fused_add_rmsnorm, gate_up_silu, rmsnorm, row_gemm_allreduce_addnorm, silu_and_mul

__all__ = [
    "PGBError",
    "PGBTimeout",
    "_lib",
    "col_gemm",
    "fused_add_rmsnorm",
    "gate_up_silu",
    "ops",
    "rmsnorm",
    "row_gemm_allreduce_addnorm",
    "silu_and_mul",
]
