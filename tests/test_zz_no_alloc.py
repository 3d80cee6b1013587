"""Allocation-free column GEMM (pgb_col_gemm_noalloc) through the C ABI.

Some callers cannot allocate device memory at the moment they run a GEMM: a
serving runtime that has handed nearly all of HBM to its KV-cache pool, an
allocator hook that must not re-enter the allocator, a latency path where
cudaMalloc would synchronise the device. The no-alloc entry point serves them
with the same kernel on a fixed scratch array in the library's device image
instead of a caller workspace. These tests check that it gives the result of
pgb_col_gemm and of a plain torch f32 restatement of F.linear, within the
column-GEMM tolerance (max |diff| <= max(2e-2 * RMS, 1 ulp)), on two calls in
a row and when calls of different shapes reuse the shared array on one
stream; that it refuses shapes whose scratch need is above the fixed maximum;
that f32 check mode needs no scratch; and that its sticky status word reads
clean after good calls.

Named to be collected last, so it also runs after every other GPU test has
used the library in the same process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

PGB_OK = 0
PGB_ERR_INVALID = 1
PGB_BF16 = 1
PGB_F32 = 2
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


def _f32_ref(x, w, b=None):
    """F.linear restated in f32 (python/picosgl/layers/linear.py:23-27)."""
    y = x.float() @ w.float().t()
    return y + b.float() if b is not None else y


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


def _no_alloc(lib, x, w, b, T, N, K, dtype=PGB_BF16):
    y = torch.empty(T, N, dtype=x.dtype, device=x.device)
    rc = lib.pgb_col_gemm_noalloc(_ptr(x), _ptr(w), _ptr(b), _ptr(y), T, N, K, dtype, _stream())
    assert rc == 0, lib.pgb_last_error()
    return y


def _status(lib, reset=0):
    st = ctypes.c_int(-1)
    rc = lib.pgb_col_gemm_noalloc_status(ctypes.byref(st), reset)
    assert rc == 0, lib.pgb_last_error()
    return st.value


def _inputs(dev, T, N, K, seed, bias=False):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(T, K, device=dev, generator=g).bfloat16()
    w = (torch.randn(N, K, device=dev, generator=g) * 0.02).bfloat16()
    b = torch.randn(N, device=dev, generator=g).bfloat16() if bias else None
    return x, w, b


# Decode qkv/gate_up shapes (split tiles exchanging partials through the
# scratch, and a wave of whole tiles before them), a ragged shape with tails
# in N and K, and a prefill shape.
SHAPES = [(1, 6144, 4096), (32, 24576, 4096), (128, 6144, 4096), (200, 200, 136), (1000, 1024, 1000)]


@pytest.mark.parametrize("T,N,K", SHAPES)
def test_no_alloc_matches_col_gemm(pgb, cuda_device, T, N, K):
    lib = pgb._lib.load()
    x, w, b = _inputs(cuda_device, T, N, K, 4242 + T + N + K, bias=(T == 200))
    ref = _with_workspace(lib, x, w, b, T, N, K)
    y1 = _no_alloc(lib, x, w, b, T, N, K)
    y2 = _no_alloc(lib, x, w, b, T, N, K)
    torch.cuda.synchronize()
    f32 = _f32_ref(x, w, b)
    for y in (y1, y2):
        _check(y, ref)
        _check(y, f32)
    assert _status(lib) == PGB_OK


def test_no_alloc_shapes_alternate_on_one_stream(pgb, cuda_device):
    """Calls of different shapes share the array back to back: a split-heavy
    decode shape, a one-token shape and a ragged one, twice round, every
    result checked only after all were enqueued."""
    lib = pgb._lib.load()
    shapes = [(32, 24576, 4096), (1, 6144, 4096), (200, 200, 136)]
    cases = [_inputs(cuda_device, T, N, K, 77 + i, bias=(T == 200)) + ((T, N, K),)
             for i, (T, N, K) in enumerate(shapes)]
    outs = []
    for _ in range(2):
        for x, w, b, (T, N, K) in cases:
            outs.append((_no_alloc(lib, x, w, b, T, N, K), _f32_ref(x, w, b)))
    torch.cuda.synchronize()
    for y, ref in outs:
        _check(y, ref)
    assert _status(lib, reset=1) == PGB_OK


def test_no_alloc_f32_check_mode_needs_no_scratch(pgb, cuda_device):
    """f32 runs the CUDA-core GEMM without scratch, even for shapes whose
    bf16 plan would not fit the fixed array."""
    lib = pgb._lib.load()
    T, N, K = 256, 6144, 4096
    assert lib.pgb_col_gemm_workspace_size(T, N, K) > SCRATCH_MAX
    g = torch.Generator(device=cuda_device).manual_seed(9)
    x = torch.randn(T, K, device=cuda_device, generator=g)
    w = torch.randn(N, K, device=cuda_device, generator=g) * 0.02
    y = _no_alloc(lib, x, w, None, T, N, K, dtype=PGB_F32)
    torch.cuda.synchronize()
    ref = x.double() @ w.double().t()
    rel = (y.double() - ref).abs().max().item() / ref.pow(2).mean().sqrt().item()
    assert rel <= 1e-5, rel


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
    # A misaligned output is refused before the shared array is touched.
    yb = torch.empty(T * N + 1, dtype=torch.bfloat16, device=cuda_device)[1:]
    rc = lib.pgb_col_gemm_noalloc(_ptr(x[:1]), _ptr(w), None, _ptr(yb), 1, N, K, PGB_BF16, _stream())
    assert rc == PGB_ERR_INVALID and b"aligned" in lib.pgb_last_error()
