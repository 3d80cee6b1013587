// qkv_rope.cu - qkv_proj GEMM with RoPE and the KV-cache store in its epilogue.
//
// The reference's RotaryAttention.proj (python/picosgl/layers/attention.py:94-117)
// runs qkv_proj (F.linear into [T, (nq + 2 nkv) hd]), splits q, k and v, and
// rotates q and k with flashinfer's apply_rope_with_cos_sin_cache_inplace
// (python/picosgl/layers/rotary.py:34-60). The attention backend then stores
// the k and v rows into the paged cache at out_loc before it reads the cache
// back (MHAKVCachePool.store_kv, python/picosgl/cache/kv/mha_pool.py:45-56 ->
// store_cache, csrc/jit/store.cu:25-58). k and v are not used otherwise.
//
// pgb_qkv_rope_store does all of it in the GEMM epilogue: q leaves rotated,
// k (rotated) and v go straight to their cache rows, and the
// [T, (nq + 2 nkv) hd] tensor is never stored.
//
// RoPE as flashinfer applies it with is_neox = true: within a head, dim
// d < rd/2 pairs with d + rd/2, and with c, s = cos_sin[pos][d mod rd/2],
// cos_sin[pos][rd/2 + d mod rd/2] (f32),
//   x'[d]        = x[d] * c - x[d + rd/2] * s
//   x'[d + rd/2] = x[d + rd/2] * c + x[d] * s
// in f32 on the values rounded to the model dtype (the reference
// materialises qkv), rounded once. Dims rd .. hd stay as they are.
//
// Shapes: head_dim 64, 128, 256 or 512 (the reference's RotaryEmbedding
// accepts these, python/picosgl/layers/rotary.py:49), rotary_dim a multiple of
// 64 up to head_dim (partner chunks of the prefill epilogue stay 32-column
// aligned). With head_dim 64 or 128 a 128-row decode tile holds whole heads,
// so every partner row is in the tile, and the rotation runs in the GEMM
// epilogue. Wider heads span several tiles: the GEMM then writes qkv into the
// workspace and the standalone RoPE + store kernel follows (two launches, the
// same arithmetic).
// An out-of-range position or cache slot skips that token and sets an
// index-error word (kDevBadIndex) instead of writing out of bounds. That word
// is not the workspace status word: the split-tile waits poll the status word
// and give up when it is set, which a bad index must not cause.
#include "col_kernel.cuh"
#include "gemm_f32.h"

namespace pgb {

// 8 consecutive values from 16-bit or f32 memory, as f32; and back.
template <typename E>
__device__ __forceinline__ void load8(const E* p, float* v) {
  if constexpr (std::is_same<E, float>::value) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  } else {
    unpack8<E>(*reinterpret_cast<const uint4*>(p), v);
  }
}
template <typename E>
__device__ __forceinline__ void store8(E* p, const float* v) {
  if constexpr (std::is_same<E, float>::value) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    *reinterpret_cast<uint4*>(p) = pack8<E>(v);
  }
}

// NeoX rotation of 8 consecutive dims [d0, d0 + 8) of a head, d0 < rd: x are
// those dims, p their partners (d0 + rd/2 when first, d0 - rd/2 otherwise),
// cs / sn the cos / sin at d0 mod rd/2.
// Written as one rounded product and one fused multiply-add, so the fused
// epilogue and the standalone kernel round identically.
__device__ __forceinline__ void rope8(float* x, const float* p, const float* cs, const float* sn, bool first) {
#pragma unroll
  for (int e = 0; e < 8; ++e) x[e] = fmaf(first ? -p[e] : p[e], sn[e], __fmul_rn(x[e], cs[e]));
}

// Where q, k and v go and how they rotate; shared by the fused epilogue and
// the standalone kernel.
template <typename IO>
struct RopeStore {
  IO* q;                 // [T, nq * hd]
  IO* k_cache;           // [cache_rows, nkv * hd] (the pool's [slots, kv heads, head dim])
  IO* v_cache;
  const void* positions; // [T] position ids, int32 or int64
  const void* out_loc;   // [T] cache slots, int32 or int64
  const float* cos_sin;  // [max_pos, rd]: cos in [0, rd/2), sin in [rd/2, rd)
  long long cache_rows;
  int max_pos;
  int idx64;             // index element type: 0 int32, 1 int64
  int nq, nkv, hd, rd;
  int* bad;              // index-error word (kDevBadIndex when a token was skipped)

  __device__ __forceinline__ long long index_at(const void* base, int t) const {
    return idx64 ? __ldg(static_cast<const long long*>(base) + t)
                 : static_cast<long long>(__ldg(static_cast<const int*>(base) + t));
  }
  // True if a token's position and cache slot are in range; otherwise the
  // index-error word is set and the token must not be written.
  __device__ __forceinline__ bool valid(long long pos, long long loc) const {
    if (pos < 0 || pos >= max_pos || loc < 0 || loc >= cache_rows) {
      record_error(bad, kDevBadIndex);
      return false;
    }
    return true;
  }
  // Position and cache slot of token t; false if either is out of range.
  __device__ __forceinline__ bool token(int t, long long& pos, long long& loc) const {
    pos = index_at(positions, t);
    loc = index_at(out_loc, t);
    return valid(pos, loc);
  }
  // Destination of features [f0, f0 + 8) of token t (q row t or cache row loc).
  __device__ __forceinline__ IO* dst(int t, long long loc, int f0) const {
    const int qn = nq * hd, kvn = nkv * hd;
    if (f0 < qn) return q + static_cast<size_t>(t) * qn + f0;
    if (f0 < qn + kvn) return k_cache + static_cast<size_t>(loc) * kvn + (f0 - qn);
    return v_cache + static_cast<size_t>(loc) * kvn + (f0 - qn - kvn);
  }
  // True if features [f0, f0 + 8) are rotated (q or k, head dim below rd).
  __device__ __forceinline__ bool rotated(int f0) const {
    return f0 < (nq + nkv) * hd && (f0 & (hd - 1)) < rd;
  }
  __device__ __forceinline__ void cos_sin8(long long pos, int ci, float* cs, float* sn) const {
    const float* base = cos_sin + pos * rd + ci;
    load8<float>(base, cs);
    load8<float>(base + (rd >> 1), sn);
  }
};

template <typename IO>
struct EpiRope {
  static constexpr bool kGlu = false;
  static constexpr int kSwapTokens = 256;  // the decode orientation serves T <= 256 tokens
  // Decode orientation: the tile's token positions and cache slots, staged
  // once (position -1: the token is skipped), [2][kSwapTokens] int.
  static constexpr int kSmemBytes = 2 * kSwapTokens * 4;
  RopeStore<IO> rs;
  const IO* bias;  // [(nq + 2 nkv) hd] or null

  // Decode orientation, while the main loop runs: stage every token's position
  // and slot (checked once here) in shared memory and bring its cos / sin row
  // into L2, so the epilogue's chunks wait on neither. Every CTA covers the
  // same tokens [0, T): in this orientation the token side is one tile.
  template <bool SWAP>
  __device__ __forceinline__ void prepare(const GemmShape& g, const GemmCtl& c) const {
    if constexpr (SWAP) {
      int* sp = reinterpret_cast<int*>(c.extra);
      int* sl = sp + kSwapTokens;
      const int n = g.T < kSwapTokens ? g.T : kSwapTokens;
      for (int t = epi_tid(); t < n; t += kEpiThreads) {
        const long long pos = rs.index_at(rs.positions, t), loc = rs.index_at(rs.out_loc, t);
        const bool ok = rs.valid(pos, loc);
        sp[t] = ok ? static_cast<int>(pos) : -1;
        sl[t] = ok ? static_cast<int>(loc) : 0;
        if (ok) {
          const float* row = rs.cos_sin + pos * rs.rd;
          for (int off = 0; off < rs.rd; off += 32) prefetch_l2(row + off);
        }
      }
      named_bar_sync(1, kEpiThreads);
    }
  }

  __device__ __forceinline__ float row_bias(const GemmShape& g, int p, int row) const {
    const int n = swap_weight_row<false>(g, p, row);
    return (bias != nullptr && n >= 0) ? io_to_f32<IO>(bias[n]) : 0.f;
  }
  // Swap orientation: a tile is 128 consecutive features, whole heads, so a
  // staged piece's partner (rd/2 rows away) is in the same staging tile. A
  // thread's 16-byte piece column is the same for the 4 tokens it serves
  // (t0 + jb + 8k); their positions and slots come from shared memory and
  // their cos / sin (L2-resident after prepare) are requested two tokens at
  // a time, ahead of the stores.
  __device__ __forceinline__ void swap_chunk(const GemmShape& g, const GemmCtl& c, const float* v, int p, int t0,
                                             int t_lo, int t_hi) const {
    swap_stage<IO>(c.epi, v);
    const int tid = epi_tid();
    const int jb = tid >> 4, row0 = (tid & 15) * 8;
    const int f0 = p * kTileP + row0;
    if (f0 >= g.N) return;
    const int half = rs.rd >> 1;
    const bool rot = rs.rotated(f0);
    const int d0 = f0 & (rs.hd - 1);
    const bool first = d0 < half;
    const int* sp = reinterpret_cast<const int*>(c.extra);  // staged by prepare()
    const int* sl = sp + kSwapTokens;
    int pos[4], loc[4];
    bool ok[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int t = t0 + jb + 8 * k;
      const bool in = t >= t_lo && t < t_hi;
      pos[k] = in ? sp[t] : -1;
      loc[k] = in ? sl[t] : 0;
      ok[k] = pos[k] >= 0;
    }
    const int ci = first ? d0 : d0 - half;
#pragma unroll
    for (int k0 = 0; k0 < 4; k0 += 2) {  // two tokens' cos / sin in flight at a time
      float cs[2][8], sn[2][8];
      if (rot) {
#pragma unroll
        for (int kk = 0; kk < 2; ++kk)
          if (ok[k0 + kk]) rs.cos_sin8(pos[k0 + kk], ci, cs[kk], sn[kk]);
      }
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const int k = k0 + kk;
        if (!ok[k]) continue;
        const uint16_t* src = c.epi + (jb + 8 * k) * kTileP + row0;
        uint4 out = *reinterpret_cast<const uint4*>(src);
        if (rot) {
          float x[8], pp[8];
          unpack8<IO>(out, x);
          unpack8<IO>(*reinterpret_cast<const uint4*>(src + (first ? half : -half)), pp);
          rope8(x, pp, cs[kk], sn[kk], first);
          out = pack8<IO>(x);
        }
        *reinterpret_cast<uint4*>(rs.dst(t0 + jb + 8 * k, loc[k], f0)) = out;
      }
    }
  }
  // Prefill orientation: lane = token, a tile is 256 consecutive features
  // (whole heads). A first-half chunk is loaded with its partner chunk rd/2
  // columns on and both are stored; the partner's own turn is skipped. (This
  // epilogue overlaps the next tile's main loop, so its loads are not batched.)
  template <int BN>
  __device__ __forceinline__ void nonswap_tile(const GemmShape& g, uint32_t tmem, int acc, int p, int q) const {
    const int t = p * kTileP + epi_row();
    const int half = rs.rd >> 1;
    long long pos = 0, loc = 0;
    if (t < g.T) {
      pos = rs.index_at(rs.positions, t);
      loc = rs.index_at(rs.out_loc, t);
    }
    const bool ok = t < g.T && rs.valid(pos, loc);
#pragma unroll 1
    for (int col = 0; col < BN; col += 32) {
      const int f0 = q * BN + col;
      if (f0 >= g.N) break;  // the same for every lane
      const bool rot = rs.rotated(f0);
      const int d0 = f0 & (rs.hd - 1);
      if (rot && d0 >= half) continue;  // stored with its first half
      float x[32], y[32];
      epi_load_chunk<BN>(tmem, acc, col, x);
      if (rot) epi_load_chunk<BN>(tmem, acc, col + half, y);
      if (!ok) continue;
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        if (bias != nullptr) x[jj] += io_to_f32<IO>(bias[f0 + jj]);
        x[jj] = io_to_f32<IO>(f32_to_io<IO>(x[jj]));
      }
      if (!rot) {
#pragma unroll
        for (int e = 0; e < 4; ++e) store8<IO>(rs.dst(t, loc, f0 + 8 * e), x + 8 * e);
        continue;
      }
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        if (bias != nullptr) y[jj] += io_to_f32<IO>(bias[f0 + half + jj]);
        y[jj] = io_to_f32<IO>(f32_to_io<IO>(y[jj]));
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float a[8], b[8], cs[8], sn[8];
        rs.cos_sin8(pos, d0 + 8 * e, cs, sn);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          a[i] = x[8 * e + i];
          b[i] = y[8 * e + i];
        }
        rope8(a, y + 8 * e, cs, sn, true);
        rope8(b, x + 8 * e, cs, sn, false);
        store8<IO>(rs.dst(t, loc, f0 + 8 * e), a);
        store8<IO>(rs.dst(t, loc, f0 + half + 8 * e), b);
      }
    }
  }
};

namespace {

// Standalone: RoPE + store from a materialised qkv [T, (nq + 2 nkv) hd]; one
// thread per 8 features of a token.
template <typename E>
__global__ void __launch_bounds__(256) rope_store_kernel(const E* __restrict__ qkv, int T, RopeStore<E> rs) {
  // The next kernel may become resident and prefetch its weights; it reads
  // this kernel's outputs only after its own wait.
  if (threadIdx.x == 0) pdl_launch_dependents();
  pdl_wait();
  const int N = (rs.nq + 2 * rs.nkv) * rs.hd;
  const int per_row = N / 8, half = rs.rd >> 1;
  const long long total = static_cast<long long>(T) * per_row;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / per_row), f0 = static_cast<int>(i - static_cast<long long>(t) * per_row) * 8;
    long long pos, loc;
    if (!rs.token(t, pos, loc)) continue;
    const E* src = qkv + static_cast<size_t>(t) * N + f0;
    float x[8];
    load8<E>(src, x);
    if (rs.rotated(f0)) {
      const int d0 = f0 & (rs.hd - 1);
      const bool first = d0 < half;
      float pp[8], cs[8], sn[8];
      load8<E>(src + (first ? half : -half), pp);
      rs.cos_sin8(pos, first ? d0 : d0 - half, cs, sn);
      rope8(x, pp, cs, sn, first);
    }
    store8<E>(rs.dst(t, loc, f0), x);
  }
}

template <typename E>
int launch_rope_store(const E* qkv, int T, const RopeStore<E>& rs, cudaStream_t stream) {
  if (T == 0) return PGB_OK;
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc) return rc;
  const long long pieces = static_cast<long long>(T) * ((rs.nq + 2 * rs.nkv) * rs.hd / 8);
  const long long want = (pieces + 255) / 256, cap = static_cast<long long>(dev.sm_count) * 8;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(want < cap ? want : cap));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  return launch_ex(cfg, /*cooperative=*/false, 1, rope_store_kernel<E>, qkv, T, rs);
}

// Checks shared by both entry points; fills rs except the output pointers.
int rope_args(int T, int nq, int nkv, int hd, int rd, const void* positions, const void* out_loc, int index_dtype,
              const float* cos_sin, int max_pos, const void* q, const void* kc, const void* vc, long long cache_rows,
              int elem_bytes, int& idx64) {
  if (T < 0 || nq <= 0 || nkv <= 0 || max_pos <= 0 || cache_rows < 0 || cache_rows > 0x7fffffffLL)
    return set_error(PGB_ERR_INVALID, "rope: bad sizes T=%d nq=%d nkv=%d max_pos=%d cache_rows=%lld", T, nq, nkv,
                     max_pos, cache_rows);
  if (hd != 64 && hd != 128 && hd != 256 && hd != 512)
    return set_error(PGB_ERR_UNSUPPORTED, "rope: head_dim %d (64, 128, 256 or 512 supported)", hd);
  if (rd <= 0 || rd > hd || rd % 64 != 0)
    return set_error(PGB_ERR_UNSUPPORTED, "rope: rotary_dim %d (a multiple of 64 up to head_dim)", rd);
  if (index_dtype != PGB_I32 && index_dtype != PGB_I64)
    return set_error(PGB_ERR_INVALID, "rope: index dtype %d (PGB_I32 or PGB_I64)", index_dtype);
  idx64 = index_dtype == PGB_I64 ? 1 : 0;
  if (T == 0) return PGB_OK;
  if (positions == nullptr || out_loc == nullptr || cos_sin == nullptr || q == nullptr || kc == nullptr ||
      vc == nullptr)
    return set_error(PGB_ERR_INVALID, "rope: null pointer argument");
  for (const void* ptr : {static_cast<const void*>(cos_sin), q, kc, vc})
    if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0u)
      return set_error(PGB_ERR_INVALID, "rope: q, caches and cos_sin_cache must be 16-byte aligned");
  (void)elem_bytes;
  return PGB_OK;
}

template <typename IO>
RopeStore<IO> make_rs(void* q, void* kc, void* vc, const void* positions, const void* out_loc, const float* cos_sin,
                      long long cache_rows, int max_pos, int idx64, int nq, int nkv, int hd, int rd, int* bad) {
  RopeStore<IO> rs{};
  rs.q = static_cast<IO*>(q);
  rs.k_cache = static_cast<IO*>(kc);
  rs.v_cache = static_cast<IO*>(vc);
  rs.positions = positions;
  rs.out_loc = out_loc;
  rs.cos_sin = cos_sin;
  rs.cache_rows = cache_rows;
  rs.max_pos = max_pos;
  rs.idx64 = idx64;
  rs.nq = nq;
  rs.nkv = nkv;
  rs.hd = hd;
  rs.rd = rd;
  rs.bad = bad;
  return rs;
}

size_t f32_qkv_bytes(int T, int N) { return static_cast<size_t>(T) * static_cast<size_t>(N) * 4u; }

// Heads too wide for the fused epilogue (see the file comment).
bool rope_in_epilogue(int hd) { return hd <= kTileP; }

// Wide heads: [column workspace | qkv T x N of the I/O type, 256-byte aligned].
size_t wide_qkv_offset(const GemmPlan& p) { return align_up(col_workspace_bytes(p), 256); }

int sm_count_or_148() {
  DeviceInfo d;
  if (current_device_info(&d) == PGB_OK) return d.sm_count;
  return 148;
}

}  // namespace
}  // namespace pgb

extern "C" size_t pgb_qkv_rope_store_workspace_size(int T, int num_q_heads, int num_kv_heads, int head_dim, int K,
                                                    int dtype) {
  using namespace pgb;
  const int N = (num_q_heads + 2 * num_kv_heads) * head_dim;
  if (T <= 0 || N <= 0 || K <= 0) return kWsHeaderBytes + kWsCounterBytes;
  if (dtype == PGB_F32) return kWsHeaderBytes + kWsCounterBytes + f32_qkv_bytes(T, N);
  const GemmPlan p = plan_gemm_col(T, N, K, sm_count_or_148(), SIZE_MAX);
  if (!rope_in_epilogue(head_dim)) return wide_qkv_offset(p) + f32_qkv_bytes(T, N) / 2;
  return col_workspace_bytes(p);
}

extern "C" int pgb_qkv_rope_store(const void* x, const void* w, const void* bias, int T, int K, int num_q_heads,
                                  int num_kv_heads, int head_dim, int rotary_dim, const void* positions,
                                  const void* out_loc, int index_dtype, const float* cos_sin_cache,
                                  int max_position, void* q_out, void* k_cache, void* v_cache,
                                  long long cache_rows, int dtype, void* workspace, size_t workspace_bytes,
                                  void* stream) {
  using namespace pgb;
  const int nq = num_q_heads, nkv = num_kv_heads, hd = head_dim, rd = rotary_dim;
  int idx64 = 0;
  int rc = rope_args(T, nq, nkv, hd, rd, positions, out_loc, index_dtype, cos_sin_cache, max_position, q_out,
                     k_cache, v_cache, cache_rows, dtype == PGB_F32 ? 4 : 2, idx64);
  if (rc || T == 0) return rc;
  if (K <= 0) return set_error(PGB_ERR_INVALID, "qkv_rope_store: bad K=%d", K);
  if (x == nullptr || w == nullptr || workspace == nullptr)
    return set_error(PGB_ERR_INVALID, "qkv_rope_store: null pointer argument");
  const int N = (nq + 2 * nkv) * hd;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (dtype == PGB_F32) {
    // f32 check mode: qkv into the workspace's exchange area, then the
    // standalone RoPE + store; index errors go to the workspace's index-error word.
    const size_t need = kWsHeaderBytes + kWsCounterBytes + f32_qkv_bytes(T, N);
    if (workspace_bytes < need)
      return set_error(PGB_ERR_INVALID, "qkv_rope_store: workspace of %zu bytes, %zu needed", workspace_bytes,
                       need);
    float* qkv = reinterpret_cast<float*>(ws + kWsHeaderBytes + kWsCounterBytes);
    rc = launch_gemm_f32(static_cast<const float*>(x), static_cast<const float*>(w),
                         static_cast<const float*>(bias), qkv, T, N, K, s);
    if (rc) return rc;
    return launch_rope_store<float>(qkv, T,
                                    make_rs<float>(q_out, k_cache, v_cache, positions, out_loc, cos_sin_cache,
                                                   cache_rows, max_position, idx64, nq, nkv, hd, rd,
                                                   reinterpret_cast<int*>(ws + kWsIndexErrorOffset)),
                                    s);
  }
  if (dtype != PGB_BF16 && dtype != PGB_F16)
    return set_error(PGB_ERR_UNSUPPORTED, "qkv_rope_store: dtype %d not supported", dtype);
  if (K % 8 != 0) return set_error(PGB_ERR_INVALID, "qkv_rope_store: K=%d must be a multiple of 8", K);
  DeviceInfo dev;
  rc = current_device_info(&dev);
  if (rc) return rc;
  const GemmPlan p = plan_gemm_col(T, N, K, dev.sm_count, SIZE_MAX);
  const bool fused = rope_in_epilogue(hd);
  const size_t need = fused ? col_workspace_bytes(p) : wide_qkv_offset(p) + f32_qkv_bytes(T, N) / 2;
  if (workspace_bytes < need)
    return set_error(PGB_ERR_INVALID, "qkv_rope_store: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  if (!fused) {
    // Wide heads: qkv into the workspace, then the standalone RoPE + store.
    void* qkv = ws + wide_qkv_offset(p);
    ColScratch sc = col_scratch(ws, col_workspace_bytes(p));
    int* bad = reinterpret_cast<int*>(ws + kWsIndexErrorOffset);
    if (dtype == PGB_BF16) {
      using B = __nv_bfloat16;
      rc = dispatch_col<B>(p, dev, x, w, T, N, K, sc, s, EpiPlain<B>{static_cast<B*>(qkv), static_cast<const B*>(bias)});
      if (rc) return rc;
      return launch_rope_store<B>(static_cast<const B*>(qkv), T,
                                  make_rs<B>(q_out, k_cache, v_cache, positions, out_loc, cos_sin_cache, cache_rows,
                                             max_position, idx64, nq, nkv, hd, rd, bad),
                                  s);
    }
    using F = __half;
    rc = dispatch_col<F>(p, dev, x, w, T, N, K, sc, s, EpiPlain<F>{static_cast<F*>(qkv), static_cast<const F*>(bias)});
    if (rc) return rc;
    return launch_rope_store<F>(static_cast<const F*>(qkv), T,
                                make_rs<F>(q_out, k_cache, v_cache, positions, out_loc, cos_sin_cache, cache_rows,
                                           max_position, idx64, nq, nkv, hd, rd, bad),
                                s);
  }
  if (dtype == PGB_BF16) {
    using B = __nv_bfloat16;
    const EpiRope<B> epi{make_rs<B>(q_out, k_cache, v_cache, positions, out_loc, cos_sin_cache, cache_rows,
                                    max_position, idx64, nq, nkv, hd, rd,
                                    reinterpret_cast<int*>(ws + kWsIndexErrorOffset)),
                         static_cast<const B*>(bias)};
    return dispatch_col<B>(p, dev, x, w, T, N, K, col_scratch(ws, workspace_bytes), s, epi);
  }
  const EpiRope<__half> epi{make_rs<__half>(q_out, k_cache, v_cache, positions, out_loc, cos_sin_cache, cache_rows,
                                            max_position, idx64, nq, nkv, hd, rd,
                                            reinterpret_cast<int*>(ws + kWsIndexErrorOffset)),
                            static_cast<const __half*>(bias)};
  return dispatch_col<__half>(p, dev, x, w, T, N, K, col_scratch(ws, workspace_bytes), s, epi);
}

extern "C" int pgb_rope_store(const void* qkv, int T, int num_q_heads, int num_kv_heads, int head_dim,
                              int rotary_dim, const void* positions, const void* out_loc, int index_dtype,
                              const float* cos_sin_cache, int max_position, void* q_out, void* k_cache,
                              void* v_cache, long long cache_rows, int dtype, int* status, void* stream) {
  using namespace pgb;
  const int nq = num_q_heads, nkv = num_kv_heads, hd = head_dim, rd = rotary_dim;
  int idx64 = 0;
  int rc = rope_args(T, nq, nkv, hd, rd, positions, out_loc, index_dtype, cos_sin_cache, max_position, q_out,
                     k_cache, v_cache, cache_rows, dtype == PGB_F32 ? 4 : 2, idx64);
  if (rc || T == 0) return rc;
  if (qkv == nullptr || status == nullptr) return set_error(PGB_ERR_INVALID, "rope_store: null pointer argument");
  if ((reinterpret_cast<uintptr_t>(qkv) & 15u) != 0u)
    return set_error(PGB_ERR_INVALID, "rope_store: qkv must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PGB_BF16:
      return launch_rope_store<__nv_bfloat16>(
          static_cast<const __nv_bfloat16*>(qkv), T,
          make_rs<__nv_bfloat16>(q_out, k_cache, v_cache, positions, out_loc, cos_sin_cache, cache_rows,
                                 max_position, idx64, nq, nkv, hd, rd, status),
          s);
    case PGB_F16:
      return launch_rope_store<__half>(static_cast<const __half*>(qkv), T,
                                       make_rs<__half>(q_out, k_cache, v_cache, positions, out_loc, cos_sin_cache,
                                                       cache_rows, max_position, idx64, nq, nkv, hd, rd, status),
                                       s);
    case PGB_F32:
      return launch_rope_store<float>(static_cast<const float*>(qkv), T,
                                      make_rs<float>(q_out, k_cache, v_cache, positions, out_loc, cos_sin_cache,
                                                     cache_rows, max_position, idx64, nq, nkv, hd, rd, status),
                                      s);
    default:
      return set_error(PGB_ERR_UNSUPPORTED, "rope_store: dtype %d not supported", dtype);
  }
}
