"""Torch-level wrappers over the C ABI.

These functions take CUDA tensors, check them the way the reference's
TensorMatcher / runtime_assert checks do (csrc/include/picosgl/tensor.hpp,
csrc/src/pynccl.cu:95-100), and enqueue the sm_100a kernels on the current
torch stream. There is no CPU path: a missing library or a non-CUDA tensor
raises.
"""

from __future__ import annotations

import threading

import torch

from . import _lib

_DTYPES = {torch.float16: _lib.PGB_F16, torch.bfloat16: _lib.PGB_BF16, torch.float32: _lib.PGB_F32}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float16, bfloat16 or float32") from None


def _require_cuda(name: str, t: torch.Tensor) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (got {t.device})")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


class _Workspaces:
    """Per-device zero-initialised scratch: split-tile counters and the split-K exchange area.

    Grows outside CUDA-graph capture; inside a capture the size must already be
    sufficient (allocation during capture would not be replayed)."""

    def __init__(self) -> None:
        self._bufs: dict[int, torch.Tensor] = {}
        self._lock = threading.Lock()

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        with self._lock:
            buf = self._bufs.get(idx)
            if buf is None or buf.numel() < nbytes:
                if torch.cuda.is_current_stream_capturing():
                    raise RuntimeError(
                        f"split-K workspace of {nbytes} bytes needed during CUDA-graph capture; "
                        "run the same shapes once before capturing"
                    )
                size = max(nbytes, 1 << 20)
                buf = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", idx))
                self._bufs[idx] = buf
            return buf


WORKSPACES = _Workspaces()


def col_gemm(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x . w^T (+ bias) on the tcgen05 kernel; x [T, K], w [N, K]."""
    _require_cuda("x", x)
    _require_cuda("weight", w)
    if x.dim() != 2 or w.dim() != 2 or x.shape[1] != w.shape[1]:
        raise ValueError(f"shape mismatch: x {tuple(x.shape)} weight {tuple(w.shape)}")
    if x.dtype != w.dtype:
        raise TypeError(f"x {x.dtype} and weight {w.dtype} differ")
    T, K = x.shape
    N = w.shape[0]
    if bias is not None:
        _require_cuda("bias", bias)
        if bias.shape != (N,) or bias.dtype != x.dtype:
            raise ValueError("bias must be [N] with the input dtype")
    if out is None:
        out = torch.empty((T, N), dtype=x.dtype, device=x.device)
    else:
        _require_cuda("out", out)
        if out.shape != (T, N) or out.dtype != x.dtype:
            raise ValueError("out must be [T, N] with the input dtype")
    lib = _lib.load()
    need = lib.pgb_col_gemm_workspace_size(T, N, K)
    ws = WORKSPACES.get(x.device, need)
    _lib.call(
        "pgb_col_gemm",
        x.data_ptr(),
        w.data_ptr(),
        bias.data_ptr() if bias is not None else None,
        out.data_ptr(),
        T,
        N,
        K,
        dtype_code(x),
        ws.data_ptr(),
        ws.numel(),
        _stream(x),
    )
    return out


def gate_up_silu(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(x . Wg^T) * (x . Wu^T) in one kernel; x [T, K], w = [Wg; Wu] of [2I, K].

    GatedMLP.forward's gate_up_proj + silu_and_mul (python/picosgl/layers/mlp.py:43-46).
    """
    _require_cuda("x", x)
    _require_cuda("weight", w)
    if x.dim() != 2 or w.dim() != 2 or x.shape[1] != w.shape[1] or w.shape[0] % 2:
        raise ValueError(f"shape mismatch: x {tuple(x.shape)} merged gate/up weight {tuple(w.shape)}")
    if x.dtype != w.dtype:
        raise TypeError(f"x {x.dtype} and weight {w.dtype} differ")
    T, K = x.shape
    I = w.shape[0] // 2
    if bias is not None:
        _require_cuda("bias", bias)
        if bias.shape != (2 * I,) or bias.dtype != x.dtype:
            raise ValueError("bias must be [2I] with the input dtype")
    if out is None:
        out = torch.empty((T, I), dtype=x.dtype, device=x.device)
    else:
        _require_cuda("out", out)
        if out.shape != (T, I) or out.dtype != x.dtype:
            raise ValueError("out must be [T, I] with the input dtype")
    lib = _lib.load()
    need = lib.pgb_gate_up_silu_workspace_size(T, I, K, dtype_code(x))
    ws = WORKSPACES.get(x.device, need)
    _lib.call("pgb_gate_up_silu", x.data_ptr(), w.data_ptr(), bias.data_ptr() if bias is not None else None,
              out.data_ptr(), T, I, K, dtype_code(x), ws.data_ptr(), ws.numel(), _stream(x))
    return out


def silu_and_mul(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(x[..., :I]) * x[..., I:] (python/picosgl/layers/activation.py:9-12)."""
    _require_cuda("x", x)
    if x.shape[-1] % 2:
        raise ValueError(f"last dimension {x.shape[-1]} is not even")
    I = x.shape[-1] // 2
    T = x.numel() // max(x.shape[-1], 1)
    if out is None:
        out = torch.empty((*x.shape[:-1], I), dtype=x.dtype, device=x.device)
    else:
        _require_cuda("out", out)
        if out.shape != (*x.shape[:-1], I) or out.dtype != x.dtype:
            raise ValueError("out must be [..., I] with the input dtype")
    _lib.call("pgb_silu_and_mul", x.data_ptr(), out.data_ptr(), T, I, dtype_code(x), _stream(x))
    return out


_INDEX = {torch.int32: _lib.PGB_I32, torch.int64: _lib.PGB_I64}


def _rope_common(positions, out_loc, cos_sin_cache, k_cache, v_cache, T, nkv, hd):
    for name, t in (("positions", positions), ("out_loc", out_loc), ("cos_sin_cache", cos_sin_cache),
                    ("k_cache", k_cache), ("v_cache", v_cache)):
        _require_cuda(name, t)
    if positions.shape != (T,) or out_loc.shape != (T,):
        raise ValueError(f"positions and out_loc must be [{T}]")
    if positions.dtype not in _INDEX or out_loc.dtype != positions.dtype:
        raise TypeError("positions and out_loc must both be int32 or both int64")
    if cos_sin_cache.dtype != torch.float32 or cos_sin_cache.dim() != 2:
        raise TypeError("cos_sin_cache must be a [max_position, rotary_dim] float32 tensor")
    rows = k_cache.shape[0]
    for name, c in (("k_cache", k_cache), ("v_cache", v_cache)):
        if c.numel() != rows * nkv * hd or c.shape[0] != rows:
            raise ValueError(f"{name} must be [slots, {nkv}, {hd}] (one layer of the KV pool)")
    return rows


def qkv_rope_store(x: torch.Tensor, w: torch.Tensor, positions: torch.Tensor, out_loc: torch.Tensor,
                   cos_sin_cache: torch.Tensor, num_q_heads: int, num_kv_heads: int, head_dim: int,
                   k_cache: torch.Tensor, v_cache: torch.Tensor, bias: torch.Tensor | None = None,
                   q_out: torch.Tensor | None = None) -> torch.Tensor:
    """qkv_proj + RoPE + KV-cache store in one kernel; returns q [T, nq * hd].

    RotaryAttention.proj (python/picosgl/layers/attention.py:94-117) followed by
    store_kv (python/picosgl/cache/kv/mha_pool.py:45-56). k_cache / v_cache are
    one layer's [slots, nkv, hd] storage; out_loc[t] is token t's slot.
    """
    _require_cuda("x", x)
    _require_cuda("weight", w)
    nq, nkv, hd = num_q_heads, num_kv_heads, head_dim
    N = (nq + 2 * nkv) * hd
    if x.dim() != 2 or w.shape != (N, x.shape[1]):
        raise ValueError(f"shape mismatch: x {tuple(x.shape)} weight {tuple(w.shape)} (expected [{N}, K])")
    if x.dtype != w.dtype or k_cache.dtype != x.dtype or v_cache.dtype != x.dtype:
        raise TypeError("x, weight and the caches must share one dtype")
    T, K = x.shape
    rows = _rope_common(positions, out_loc, cos_sin_cache, k_cache, v_cache, T, nkv, hd)
    if bias is not None:
        _require_cuda("bias", bias)
        if bias.shape != (N,) or bias.dtype != x.dtype:
            raise ValueError("bias must be [N] with the input dtype")
    if q_out is None:
        q_out = torch.empty((T, nq * hd), dtype=x.dtype, device=x.device)
    else:
        _require_cuda("q_out", q_out)
        if q_out.numel() != T * nq * hd or q_out.dtype != x.dtype:
            raise ValueError("q_out must hold [T, nq * hd] of the input dtype")
    lib = _lib.load()
    need = lib.pgb_qkv_rope_store_workspace_size(T, nq, nkv, hd, K, dtype_code(x))
    ws = WORKSPACES.get(x.device, need)
    _lib.call("pgb_qkv_rope_store", x.data_ptr(), w.data_ptr(), bias.data_ptr() if bias is not None else None,
              T, K, nq, nkv, hd, cos_sin_cache.shape[1], positions.data_ptr(), out_loc.data_ptr(),
              _INDEX[positions.dtype], cos_sin_cache.data_ptr(), cos_sin_cache.shape[0], q_out.data_ptr(),
              k_cache.data_ptr(), v_cache.data_ptr(), rows, dtype_code(x), ws.data_ptr(), ws.numel(), _stream(x))
    return q_out


def rope_store(qkv: torch.Tensor, positions: torch.Tensor, out_loc: torch.Tensor, cos_sin_cache: torch.Tensor,
               num_q_heads: int, num_kv_heads: int, head_dim: int, k_cache: torch.Tensor,
               v_cache: torch.Tensor, q_out: torch.Tensor | None = None,
               status: torch.Tensor | None = None) -> torch.Tensor:
    """RoPE + KV-cache store from a materialised qkv [T, (nq + 2 nkv) hd]
    (flashinfer apply_rope_with_cos_sin_cache_inplace + store_cache); returns q."""
    # The kernel reads and writes every tensor in qkv's element type.
    for name, t in (("k_cache", k_cache), ("v_cache", v_cache), ("q_out", q_out)):
        if t is not None and t.dtype != qkv.dtype:
            raise TypeError(f"{name} dtype {t.dtype} differs from qkv {qkv.dtype}")
    if status is not None and (status.dtype != torch.int32 or status.numel() < 1):
        raise TypeError("status must be a CUDA int32 tensor of at least one element")
    _require_cuda("qkv", qkv)
    nq, nkv, hd = num_q_heads, num_kv_heads, head_dim
    T = qkv.shape[0]
    if qkv.dim() != 2 or qkv.shape[1] != (nq + 2 * nkv) * hd:
        raise ValueError(f"qkv must be [T, {(nq + 2 * nkv) * hd}]")
    rows = _rope_common(positions, out_loc, cos_sin_cache, k_cache, v_cache, T, nkv, hd)
    if q_out is None:
        q_out = torch.empty((T, nq * hd), dtype=qkv.dtype, device=qkv.device)
    else:
        _require_cuda("q_out", q_out)
        if q_out.numel() != T * nq * hd:
            raise ValueError("q_out must hold [T, nq * hd] elements")
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=qkv.device)
    else:
        _require_cuda("status", status)
    _lib.call("pgb_rope_store", qkv.data_ptr(), T, nq, nkv, hd, cos_sin_cache.shape[1], positions.data_ptr(),
              out_loc.data_ptr(), _INDEX[positions.dtype], cos_sin_cache.data_ptr(), cos_sin_cache.shape[0],
              q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), rows, dtype_code(qkv), status.data_ptr(),
              _stream(qkv))
    return q_out


def rope_index_error(device: torch.device, reset: bool = False) -> int:
    """Index-error word of the column-GEMM workspace on `device`: 5 once a
    qkv_rope_store call skipped a token whose position or cache slot was out
    of range, else 0. Synchronises."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = WORKSPACES._bufs.get(idx)
    if buf is None:
        return 0
    word = buf[4:8].view(torch.int32)
    val = int(word.item())
    if reset:
        word.zero_()
    return val


def row_gemm_allreduce_addnorm(comm, x_local: torch.Tensor, w_local: torch.Tensor,
                               residual: torch.Tensor | None, norm_w: torch.Tensor | None,
                               eps: float, out: torch.Tensor | None = None,
                               bias: torch.Tensor | None = None) -> torch.Tensor:
    """Fused row-parallel GEMM + all-reduce (+ residual-add + RMSNorm).

    With norm_w: residual <- y + residual (in place), returns rmsnorm(residual) * norm_w.
    Without: returns y = sum over ranks of x_local . w_local^T.
    """
    _require_cuda("x", x_local)
    _require_cuda("weight", w_local)
    if x_local.dim() != 2 or w_local.dim() != 2 or x_local.shape[1] != w_local.shape[1]:
        raise ValueError(f"shape mismatch: x {tuple(x_local.shape)} weight {tuple(w_local.shape)}")
    T, K = x_local.shape
    N = w_local.shape[0]
    for name, t in (("residual", residual), ("norm weight", norm_w), ("bias", bias)):
        if t is not None:
            _require_cuda(name, t)
            if t.dtype != x_local.dtype:
                raise TypeError(f"{name} dtype {t.dtype} differs from input {x_local.dtype}")
    if norm_w is not None:
        if residual is None or residual.shape != (T, N) or norm_w.shape != (N,):
            raise ValueError("residual must be [T, N] and norm weight [N]")
    if out is None:
        out = torch.empty((T, N), dtype=x_local.dtype, device=x_local.device)
    h = comm.handle if hasattr(comm, "handle") else comm
    _lib.call(
        "pgb_row_gemm_allreduce_addnorm",
        h,
        x_local.data_ptr(),
        w_local.data_ptr(),
        bias.data_ptr() if bias is not None else None,
        residual.data_ptr() if residual is not None else None,
        norm_w.data_ptr() if norm_w is not None else None,
        float(eps),
        out.data_ptr(),
        T,
        N,
        K,
        dtype_code(x_local),
        _stream(x_local),
    )
    return out


def fused_add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float) -> None:
    """In place: residual <- x + residual; x <- rmsnorm(residual) * weight."""
    for n, t in (("x", x), ("residual", residual), ("weight", weight)):
        _require_cuda(n, t)
    if x.shape != residual.shape or x.shape[-1] != weight.shape[-1]:
        raise ValueError("x / residual / weight shapes disagree")
    H = x.shape[-1]
    _lib.call("pgb_fused_add_rmsnorm", x.data_ptr(), residual.data_ptr(), weight.data_ptr(), float(eps),
              x.numel() // H, H, dtype_code(x), _stream(x))


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    _require_cuda("x", x)
    _require_cuda("weight", weight)
    H = x.shape[-1]
    if out is None:
        out = torch.empty_like(x)
    _lib.call("pgb_rmsnorm", x.data_ptr(), weight.data_ptr(), float(eps), out.data_ptr(), x.numel() // H, H,
              dtype_code(x), _stream(x))
    return out
