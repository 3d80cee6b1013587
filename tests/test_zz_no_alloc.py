"""Allocation-free column GEMM (pgb_col_gemm_noalloc) against pgb_col_gemm.

The no-alloc entry point runs the same kernel on a fixed scratch array that
lives in the library's device image instead of a caller workspace. Through
the C ABI it must give the result of pgb_col_gemm, within the column-GEMM
tolerance (max |diff| <= max(2e-2 * RMS, 1 ulp)), on two calls in a row, and
refuse shapes whose scratch need is above the fixed maximum.

Named to be collected last, so it also runs after every other GPU test has
used the library in the same process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

PGB_ERR_INVALID = 1
PGB_BF16 = 1
SCRATCH_MAX = 16 * 1024 * 1024


def _check(y, ref, tol=2e-2):
    """|y - ref| <= max(tol * RMS(ref), 1 ulp of the output dtype at ref)."""
    mant = {torch.bfloat16: 7, torch.float16: 10}[y.dtype]
    ref = ref.float()
    rms = ref.pow(2).mean().sqrt().item()
    d = (y.float() - ref).abs()
    u = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(1e-30))) - mant)
    worst = (d / torch.maximum(torch.full_like(d, tol * rms), u)).max().item()
    assert worst <= 1.0, f"max|diff|={d.max().item():.4g} rms={rms:.4g} worst/bound={worst:.3g}"


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _with_workspace(lib, x, w, b, T, N, K):
    y = torch.empty(T, N, dtype=x.dtype, device=x.device)
    nbytes = lib.pgb_col_gemm_workspace_size(T, N, K)
    ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=x.device)
    rc = lib.pgb_col_gemm(_ptr(x), _ptr(w), _ptr(b), _ptr(y), T, N, K, PGB_BF16, _ptr(ws),
                          ctypes.c_size_t(ws.numel()), _stream())
    assert rc == 0, lib.pgb_last_error()
    return y


def _no_alloc(lib, x, w, b, T, N, K):
    y = torch.empty(T, N, dtype=x.dtype, device=x.device)
    rc = lib.pgb_col_gemm_noalloc(_ptr(x), _ptr(w), _ptr(b), _ptr(y), T, N, K, PGB_BF16, _stream())
    assert rc == 0, lib.pgb_last_error()
    return y


# Decode qkv/gate_up shapes (split tiles exchanging partials through the
# scratch, and a wave of whole tiles before them), a ragged shape with tails
# in N and K, and a prefill shape.
SHAPES = [(1, 6144, 4096), (32, 24576, 4096), (128, 6144, 4096), (200, 200, 136), (1000, 1024, 1000)]


@pytest.mark.parametrize("T,N,K", SHAPES)
def test_no_alloc_matches_col_gemm(pgb, cuda_device, T, N, K):
    lib = pgb._lib.load()
    g = torch.Generator(device=cuda_device).manual_seed(4242 + T + N + K)
    x = torch.randn(T, K, device=cuda_device, generator=g).bfloat16()
    w = (torch.randn(N, K, device=cuda_device, generator=g) * 0.02).bfloat16()
    b = torch.randn(N, device=cuda_device, generator=g).bfloat16() if T == 200 else None
    ref = _with_workspace(lib, x, w, b, T, N, K)
    y1 = _no_alloc(lib, x, w, b, T, N, K)
    y2 = _no_alloc(lib, x, w, b, T, N, K)
    torch.cuda.synchronize()
    _check(y1, ref)
    _check(y2, ref)


def test_no_alloc_refuses_oversize_scratch(pgb, cuda_device):
    lib = pgb._lib.load()
    T, N, K = 256, 6144, 4096
    assert lib.pgb_col_gemm_workspace_size(T, N, K) > SCRATCH_MAX
    x = torch.zeros(T, K, dtype=torch.bfloat16, device=cuda_device)
    w = torch.zeros(N, K, dtype=torch.bfloat16, device=cuda_device)
    y = torch.empty(T, N, dtype=torch.bfloat16, device=cuda_device)
    rc = lib.pgb_col_gemm_noalloc(_ptr(x), _ptr(w), None, _ptr(y), T, N, K, PGB_BF16, _stream())
    assert rc == PGB_ERR_INVALID
    assert b"scratch" in lib.pgb_last_error()
