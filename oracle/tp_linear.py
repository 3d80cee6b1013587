"""numpy restatement of the reference's tensor-parallel linear path.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): the checker for the CUDA
library, never imported by it.

Arithmetic model. Values are carried as float32 arrays; `round_to` rounds
them to the representable values of the run's dtype (bf16 / f16 by
round-to-nearest-even, f32 unchanged). Products are accumulated in float64
and rounded once, which is the exact rounding of what cuBLAS approximates
with f32 accumulation.
"""

from __future__ import annotations

import numpy as np

# ----------------------------------------------------------------- dtypes --


def round_to(a, dtype: str) -> np.ndarray:
    """Round float values to `dtype` ("bf16", "f16" or "f32"), return float32.

    bf16: keep the upper 16 bits of the f32 pattern with round-to-nearest-even
    (the conversion torch and CUDA's __float2bfloat16_rn perform).
    """
    a = np.asarray(a, dtype=np.float32)
    if dtype == "f32":
        return a.copy()
    if dtype == "f16":
        return a.astype(np.float16).astype(np.float32)
    if dtype != "bf16":
        raise ValueError(f"unknown dtype {dtype!r}")
    u = a.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    out = u.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(a), a, out).astype(np.float32)


# ---------------------------------------------------------------- linears --


def linear(x, w, bias=None, dtype: str = "bf16", accum: str = "f64") -> np.ndarray:
    """y = x . w^T (+ bias), rounded to dtype.

    LinearTPImpl.forward = F.linear(x, self.weight, self.bias)
    (python/picosgl/layers/linear.py:23-27). accum="f64" (the default, used
    by the tests) accumulates exactly enough to round correctly; accum="f32"
    uses BLAS sgemm like the reference's CPU path (torch f32 matmul) and is
    what the CPU-baseline timing runs.
    """
    if accum == "f32":
        y = np.asarray(x, np.float32) @ np.asarray(w, np.float32).T
        if bias is not None:
            y = y + np.asarray(bias, np.float32)
        return round_to(y, dtype)
    y = np.asarray(x, np.float64) @ np.asarray(w, np.float64).T
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    return round_to(y, dtype)


def silu_and_mul(gate_up, dtype: str = "bf16") -> np.ndarray:
    """out = silu(g) * u for the halves g, u of gate_up's last dimension.

    silu_and_mul (python/picosgl/layers/activation.py:9-12) calls
    flashinfer.silu_and_mul (flashinfer 0.6.11, a third-party dependency not
    vendored in the reference), whose act_and_mul kernel reads both halves,
    computes g / (1 + exp(-g)) * u in float32 per element and casts the
    result to the tensor's dtype once. Same steps here in float32 numpy.
    """
    a = np.asarray(gate_up, np.float32)
    i = a.shape[-1] // 2
    g, u = a[..., :i], a[..., i:]
    with np.errstate(over="ignore"):
        s = g / (np.float32(1.0) + np.exp(-g))
    return round_to(s * u, dtype)


def gate_up_silu(x, w_gate_up, bias=None, dtype: str = "bf16", accum: str = "f64") -> np.ndarray:
    """GatedMLP.forward up to down_proj (python/picosgl/layers/mlp.py:43-46):
    gate_up = gate_up_proj.forward(x) (materialised in dtype), then
    silu_and_mul(gate_up)."""
    return silu_and_mul(linear(x, w_gate_up, bias, dtype, accum), dtype)


def apply_rope_neox(x, positions, cos_sin_cache, head_dim: int, dtype: str = "bf16") -> np.ndarray:
    """Rotate the heads of x [T, heads * head_dim] in place of the reference's
    RotaryEmbedding.forward (python/picosgl/layers/rotary.py:34-60), which calls
    flashinfer.apply_rope_with_cos_sin_cache_inplace with is_neox = True
    (flashinfer 0.6.11, a third-party dependency not vendored in the reference).
    Its kernel reads cos = table[pos][i], sin = table[pos][rd/2 + i] (float32)
    and, for head dim i < rd/2 and its partner i + rd/2, computes in float32
        x[i]        * cos - x[i + rd/2] * sin
        x[i + rd/2] * cos + x[i]        * sin
    rounded once to the tensor dtype; dims from rd on are unchanged.
    """
    a = np.asarray(x, np.float32)
    T = a.shape[0]
    h = a.reshape(T, -1, head_dim).copy()
    table = np.asarray(cos_sin_cache, np.float32)
    rd = table.shape[1]
    half = rd // 2
    rows = table[np.asarray(positions, np.int64)]
    c, s = rows[:, None, :half], rows[:, None, half:]
    x1, x2 = h[..., :half].copy(), h[..., half:rd].copy()
    h[..., :half] = x1 * c - x2 * s
    h[..., half:rd] = x2 * c + x1 * s
    return round_to(h.reshape(T, -1), dtype)


def store_kv(k_cache, v_cache, out_loc, k, v):
    """k_cache[out_loc[t]] = k[t], v_cache[out_loc[t]] = v[t] on copies of the
    caches ([slots, kv heads * head_dim] rows), as MHAKVCachePool.store_kv
    (python/picosgl/cache/kv/mha_pool.py:45-56) does through store_cache
    (python/picosgl/kernel/store.py:37-51, csrc/jit/store.cu:25-58: one warp
    copies one token's row to its slot)."""
    kc, vc = np.array(k_cache, copy=True), np.array(v_cache, copy=True)
    loc = np.asarray(out_loc, np.int64)
    kc.reshape(kc.shape[0], -1)[loc] = np.asarray(k).reshape(len(loc), -1)
    vc.reshape(vc.shape[0], -1)[loc] = np.asarray(v).reshape(len(loc), -1)
    return kc, vc


def qkv_rope_store(x, w_qkv, bias, positions, out_loc, cos_sin_cache, num_q_heads: int, num_kv_heads: int,
                   head_dim: int, k_cache, v_cache, dtype: str = "bf16", accum: str = "f64"):
    """RotaryAttention.proj (python/picosgl/layers/attention.py:94-117) and the
    backend's store_kv: qkv = qkv_proj(x) materialised in dtype, split into q,
    k, v heads, q and k rotated, k and v stored at out_loc. Returns
    (q [T, nq * hd], k_cache, v_cache)."""
    qkv = linear(x, w_qkv, bias, dtype, accum)
    qn, kvn = num_q_heads * head_dim, num_kv_heads * head_dim
    q, k, v = qkv[:, :qn], qkv[:, qn:qn + kvn], qkv[:, qn + kvn:qn + 2 * kvn]
    q = apply_rope_neox(q, positions, cos_sin_cache, head_dim, dtype)
    k = apply_rope_neox(k, positions, cos_sin_cache, head_dim, dtype)
    kc, vc = store_kv(k_cache, v_cache, out_loc, k, v)
    return q, kc, vc


def all_reduce_sum(partials, dtype: str = "bf16") -> np.ndarray:
    """Sum of the ranks' tensors, rounded to dtype once.

    NCCLWrapper::all_reduce -> ncclAllReduce(sum) (csrc/src/pynccl.cu:95-137),
    reached through DistributedCommunicator.all_reduce
    (python/picosgl/distributed/impl.py:53-58). NCCL's internal summation
    order and intermediate rounding are library-specific; this restatement
    sums exactly and rounds once, the limit that every NCCL algorithm
    approximates within the path's tolerance.
    """
    acc = np.zeros_like(np.asarray(partials[0], np.float64))
    for p in partials:
        acc = acc + np.asarray(p, np.float64)
    return round_to(acc, dtype)


def rmsnorm(x, w, eps: float, dtype: str = "bf16") -> np.ndarray:
    """out = x * rsqrt(mean(x^2) + eps) * w, computed in f32, rounded to dtype.

    RMSNormFused.forward with residual None -> flashinfer.rmsnorm
    (python/picosgl/layers/norm.py:71-72).
    """
    x32 = np.asarray(x, np.float32)
    ms = np.mean(x32.astype(np.float64) ** 2, axis=-1, keepdims=True)
    r = (1.0 / np.sqrt(ms + eps)).astype(np.float32)
    return round_to(x32 * r * np.asarray(w, np.float32), dtype)


def fused_add_rmsnorm(x, residual, w, eps: float, dtype: str = "bf16"):
    """Returns (x_out, residual_out) of flashinfer.fused_add_rmsnorm.

    Called in place by RMSNormFused.forward (python/picosgl/layers/norm.py:73-75).
    Algorithm of FlashInfer's FusedAddRMSNormKernel (third-party,
    flashinfer/data/include/flashinfer/norm.cuh:387-470): per row,
    s = f32(x) + f32(residual); residual <- dtype(s); sum of squares of the
    f32 s; x <- dtype(s * rsqrt(sum/d + eps) * f32(w)). The f32 sum is
    normalised, not its rounded copy.
    """
    s = np.asarray(x, np.float32) + np.asarray(residual, np.float32)
    res_out = round_to(s, dtype)
    ms = np.mean(s.astype(np.float64) ** 2, axis=-1, keepdims=True)
    r = (1.0 / np.sqrt(ms + eps)).astype(np.float32)
    out = round_to(s * r * np.asarray(w, np.float32), dtype)
    return out, res_out


# ----------------------------------------------------------- TP sharding --


def row_shard(w_full, x_full, rank: int, n: int):
    """Rank r's K-slices of a row-parallel layer.

    Weights: _shard_tensor splits o_proj / down_proj on dim 1 with
    value.chunk(n, dim=1)[r] (python/picosgl/models/weight.py:21,69-70);
    LinearRowParallel holds input_size / n columns (layers/linear.py:83-88),
    and the activations entering it are the rank's matching K-slice.
    """
    w = np.asarray(w_full)
    x = np.asarray(x_full)
    K = w.shape[1]
    if K % n:
        raise ValueError(f"K={K} not divisible by n={n} (div_even, utils/misc.py:20-26)")
    k = K // n
    return w[:, rank * k : (rank + 1) * k], x[:, rank * k : (rank + 1) * k]


def col_shard_merged(w_parts, rank: int, n: int) -> np.ndarray:
    """Rank r's weight of LinearColParallelMerged (gate_up_proj).

    Each part (gate, up) is split on dim 0 with chunk(n, 0)[r]
    (models/weight.py:62-68) and the slices are concatenated on dim 0 in
    slot order [gate; up] (models/weight.py:149-159, layers/linear.py:45-56).
    """
    out = []
    for p in w_parts:
        p = np.asarray(p)
        if p.shape[0] % n:
            raise ValueError("output size not divisible by tp size (div_even)")
        m = p.shape[0] // n
        out.append(p[rank * m : (rank + 1) * m])
    return np.concatenate(out, axis=0)


def col_shard_partitioned(wq, wk, wv, num_kv_heads: int, rank: int, n: int) -> np.ndarray:
    """Rank r's weight of LinearColParallelPartitioned (qkv_proj).

    q is split on dim 0; k and v are split on dim 0 too unless
    num_kv_heads < n, in which case rank r keeps kv head r*num_kv_heads//n
    (replication, models/weight.py:62-68). Concatenated [q; k; v]
    (weight.py:149-159), matching the local sizes of linear.py:59-73.
    """
    q = col_shard_merged([wq], rank, n)
    kv = []
    for w in (wk, wv):
        w = np.asarray(w)
        if num_kv_heads < n:
            hd = w.shape[0] // num_kv_heads
            h = rank * num_kv_heads // n
            kv.append(w[h * hd : (h + 1) * hd])
        else:
            kv.append(col_shard_merged([w], rank, n))
    return np.concatenate([q] + kv, axis=0)


# ------------------------------------------------------- fused row layer --


def row_parallel_addnorm(x_full, w_full, residual, norm_w, eps: float, n: int,
                         dtype: str = "bf16", bias=None, accum: str = "f64"):
    """The fused op the CUDA library implements, restated unfused.

    Per rank: p_r = dtype(x_r . W_r^T (+ bias)) (LinearRowParallel.forward,
    layers/linear.py:90-97; the bias is added on every rank before the
    reduce, as F.linear(x, W, b) there does), then y = all_reduce_sum(p),
    then (out, residual) = fused_add_rmsnorm(y, residual, w, eps)
    (layers/norm.py:73-75). With norm_w None the result is y alone.
    Returns (out, residual_out, y).
    """
    parts = []
    for r in range(n):
        w_r, x_r = row_shard(w_full, x_full, r, n)
        parts.append(linear(x_r, w_r, bias, dtype, accum))
    y = parts[0] if n == 1 else all_reduce_sum(parts, dtype)
    if norm_w is None:
        return y, None, y
    out, res = fused_add_rmsnorm(y, residual, norm_w, eps, dtype)
    return out, res, y


def tp_layer_step(h, a, m, residual, wts: dict, eps: float, n: int, rank: int = 0,
                  dtype: str = "bf16", accum: str = "f64"):
    """One pass of the linear path of a decoder layer at TP size n.

    The order of LlamaDecoderLayer.forward (python/picosgl/models/llama.py:77-86):
    qkv_proj (column) on the normed hidden state h; o_proj (row) + all-reduce
    + post_attention_layernorm on the attention output a; gate_up_proj
    (column) on that norm's output; down_proj (row) + all-reduce + the next
    layer's input_layernorm on the MLP activation m. Attention and
    silu_and_mul are outside the path, so a and m are given inputs.
    wts holds full (unsharded) weights: qkv, o, gate_up, down, ln1, ln2.
    Returns dict of the outputs on `rank`.
    """
    qkv = linear(h, col_shard_merged([wts["qkv"]], rank, n), None, dtype, accum)
    x1, r1, _ = row_parallel_addnorm(a, wts["o"], residual, wts["ln1"], eps, n, dtype, accum=accum)
    gu = linear(x1, col_shard_merged([wts["gate_up"]], rank, n), None, dtype, accum)
    x2, r2, _ = row_parallel_addnorm(m, wts["down"], r1, wts["ln2"], eps, n, dtype, accum=accum)
    return {"qkv": qkv, "x1": x1, "r1": r1, "gate_up": gu, "x2": x2, "r2": r2}
