// reduce_phases.cuh - grid-wide cross-rank barrier and the reduce / add /
// RMSNorm / gather phases that follow the partial pushes.
//
// Kernels using these are launched cooperatively (all CTAs co-resident),
// because CTAs wait on the arrival of every other CTA of the grid.
#pragma once

#include <type_traits>

#include "comm.h"
#include "sm100.cuh"

namespace pgb {

constexpr int kBarPartials = 0;   // every rank pushed its partial rows
constexpr int kBarResults = 1;    // every row owner pushed its finished rows
constexpr int kBarFinish = 3;     // local only: last CTA publishes the new epoch

// Epoch of the call this kernel executes.
__device__ __forceinline__ uint32_t comm_begin(const CommDev& cm) {
  return ld_acquire_gpu(cm.epoch) + 1u;
}

// All CTAs of the grid arrive; the last one to arrive publishes this rank's
// arrival (epoch e) to every rank's flag `bar`; then every CTA waits until
// all ranks' flags reached e. The wait is bounded by cm.timeout_ns and ends
// early when another CTA already recorded an error. Every CTA must call this
// with the same `bar` sequence, errors or not, so counters stay balanced.
// sys_scope = false (one GPU) only synchronises the grid, at device scope.
__device__ __forceinline__ bool grid_cross_barrier(const CommDev& cm, int bar, uint32_t e,
                                                   bool sys_scope) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    // bar.sync above, then a gpu-scope release: the CTA's writes (local and
    // peer memory) are ordered before its arrival, and the last CTA acquires
    // them all before it publishes the flag (system scope across GPUs).
    const uint32_t old = atom_add_acqrel_gpu(&cm.arrive[bar], 1u);
    if (bar == 0) trace(1020);
    if (old == gridDim.x - 1) {
      cm.arrive[bar] = 0u;
      if (sys_scope) {
        // One acquire-release fence at system scope, then relaxed flag
        // stores (a release pattern for each of them): each st.release.sys
        // would repeat the fence, and a sequentially consistent fence is
        // not needed.
        fence_acq_rel_sys();
        if (bar == 0) trace(1021);
        for (int r = 0; r < cm.world; ++r) st_relaxed_sys(&cm.flags[r][bar * PGB_MAX_RANKS + cm.rank], e);
        if (bar == 0) trace(1022);
      } else {  // one GPU: its own flag, device scope
        st_release_gpu(&cm.flags[cm.rank][bar * PGB_MAX_RANKS + cm.rank], e);
      }
    }
    volatile int* st = cm.status;
    if (*st != 0) ok = 0;
    Deadline d(cm.timeout_ns);
    const uint32_t* mine = cm.flags[cm.rank] + bar * PGB_MAX_RANKS;
    const int nranks = sys_scope ? cm.world : 1;
    for (int r0 = 0; r0 < nranks && ok; ++r0) {
      const int r = sys_scope ? r0 : cm.rank;
      while (!epoch_reached(sys_scope ? ld_acquire_sys(mine + r) : ld_acquire_gpu(mine + r), e)) {
        if (d.expired()) {
          record_error(cm.status, kDevTimeoutPeer);
          ok = 0;
          break;
        }
        if ((d.n & 255u) == 0u && *st != 0) {
          ok = 0;
          break;
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// Last CTA to finish stores the epoch of this call.
__device__ __forceinline__ void comm_end(const CommDev& cm, uint32_t e) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t old = atom_add_acqrel_gpu(&cm.arrive[kBarFinish], 1u);
    if (old == gridDim.x - 1) {
      cm.arrive[kBarFinish] = 0u;
      st_release_gpu(cm.epoch, e);
    }
  }
}

// Row geometry of a reduction over `rows` rows of `width` elements.
struct RowSplit {
  int rows;
  int oneshot;     // 1: every rank reduces every row; 0: row owners (two-shot)
  int rows_per;    // two-shot ownership block
  int rows_cap;    // rows per source rank inside a slot region
  __device__ __forceinline__ int owner(int t) const { return oneshot ? -1 : t / rows_per; }
  __device__ __forceinline__ int first(int rank) const { return oneshot ? 0 : min(rows, rank * rows_per); }
  __device__ __forceinline__ int last(int rank) const {
    return oneshot ? rows : min(rows, (rank + 1) * rows_per);
  }
};

template <typename T>
struct Vec8;  // 8 elements in 16 (16-bit types) or 32 (f32) bytes

template <typename IO>
__device__ __forceinline__ void load8(const IO* p, float* v);
template <typename IO>
__device__ __forceinline__ void store8(IO* p, const float* v);

template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float* v) {
  const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[2 * j] = __uint_as_float(w[j] << 16);
    v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
  }
}
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float* v) {
  const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float* v) {
  const float4 a = __ldcg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldcg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float* v) {
  uint4 u;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
    w[j] = *reinterpret_cast<const uint32_t*>(&b);
  }
  *reinterpret_cast<uint4*>(p) = u;
}
template <>
__device__ __forceinline__ void store8<__half>(__half* p, const float* v) {
  uint4 u;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
    w[j] = *reinterpret_cast<const uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(p) = u;
}
template <>
__device__ __forceinline__ void store8<float>(float* p, const float* v) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// Round f32 values to the representable values of IO (the reduced output is
// materialised in IO precision in the reference before the norm reads it).
template <typename IO>
__device__ __forceinline__ float round_io(float v);
template <>
__device__ __forceinline__ float round_io<__nv_bfloat16>(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}
template <>
__device__ __forceinline__ float round_io<__half>(float v) {
  return __half2float(__float2half_rn(v));
}
template <>
__device__ __forceinline__ float round_io<float>(float v) {
  return v;
}

__device__ __forceinline__ float block_sum(float v, float* red /* >= 32 floats */) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = (blockDim.x + 31) >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

// Unpack 8 IO values held in 16 bytes.
template <typename IO>
__device__ __forceinline__ void unpack8_io(const uint4& u, float* v) {
  if constexpr (std::is_same<IO, __nv_bfloat16>::value) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = __uint_as_float(w[j] << 16);
      v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  } else {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
}

// Phase 2 for one row t. The row's sources are the world slot rows this rank
// received (one per source rank, already summed over k-ranges and rounded to
// IO); their sum is rounded to IO (the reference materialises the reduced
// tensor in that type) and then either written (do_norm == 0) or
// residual-added and RMS-normalised. Writes out[t] and residual[t] locally
// and, for two-shot, pushes both rows to every peer's result region.
//
// This code runs once per launch, after the weight stream has displaced it
// from the caches, so its instruction footprint costs more than its memory
// round trips: the loops stay rolled. Each step requests the source, residual
// and norm-weight vectors together; the f32 pre-norm row and the weights wait
// in shared memory `srow` (width f32 + width IO values) for the second pass,
// which only reads shared memory and stores. IO is 16-bit.
//
// reduce_row_src is the same for an explicit source: row t's nsrc partial rows
// start at slot0, src_stride elements apart; push sends the finished rows to
// every peer's result region (two-shot owners of row_fused.cu).
template <typename IO, int MAXV>
__device__ __forceinline__ void reduce_row_src(const CommDev& cm, uint32_t parity, const IO* slot0,
                                               size_t src_stride, int nsrc, bool push, int t, int width, IO* out,
                                               IO* residual, const IO* norm_w, float eps, int do_norm, float* red,
                                               float* srow) {
  static_assert(sizeof(IO) == 2, "16-bit I/O");
  const int nvec = width >> 3;
  uint4* wrow = reinterpret_cast<uint4*>(srow + width);
  const size_t row_off = static_cast<size_t>(t) * width;
  float ss = 0.f;
#pragma unroll 1
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    uint4 rr = make_uint4(0u, 0u, 0u, 0u), wv = rr;
    if (do_norm) {
      rr = __ldcg(reinterpret_cast<const uint4*>(residual + row_off) + v);
      wv = __ldg(reinterpret_cast<const uint4*>(norm_w) + v);
    }
    float s8[8], p[8];
    // Every rank's slot requested before the first add (one round trip, not
    // one per rank); the sum stays in rank order.
    uint4 sv[PGB_MAX_RANKS];
#pragma unroll
    for (int d = 0; d < PGB_MAX_RANKS; ++d)
      if (d < nsrc) sv[d] = __ldcg(reinterpret_cast<const uint4*>(slot0 + d * src_stride) + v);
    unpack8_io<IO>(sv[0], s8);
#pragma unroll
    for (int d = 1; d < PGB_MAX_RANKS; ++d) {
      if (d < nsrc) {
        unpack8_io<IO>(sv[d], p);
#pragma unroll
        for (int j = 0; j < 8; ++j) s8[j] += p[j];
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) s8[j] = round_io<IO>(s8[j]);
    if (do_norm) {
      unpack8_io<IO>(rr, p);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        s8[j] += p[j];
        ss += s8[j] * s8[j];
      }
      wrow[v] = wv;
    }
    float4* dst = reinterpret_cast<float4*>(srow) + 2 * v;
    dst[0] = make_float4(s8[0], s8[1], s8[2], s8[3]);
    dst[1] = make_float4(s8[4], s8[5], s8[6], s8[7]);
  }
  float rcp = 1.f;
  if (do_norm) rcp = rsqrtf(block_sum(ss, red) / static_cast<float>(width) + eps);
  else __syncthreads();
#pragma unroll 1
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    const float4 a = reinterpret_cast<const float4*>(srow)[2 * v];
    const float4 b = reinterpret_cast<const float4*>(srow)[2 * v + 1];
    float s8[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float o[8];
    if (do_norm) {
      float w[8];
      unpack8_io<IO>(wrow[v], w);
      store8<IO>(residual + row_off + v * 8, s8);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = s8[j] * rcp * w[j];
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = s8[j];
    }
    store8<IO>(out + row_off + v * 8, o);
    if (push) {
#pragma unroll 1
      for (int d = 0; d < cm.world; ++d) {
        if (d == cm.rank) continue;
        uint8_t* base = cm.results[d] + parity * cm.result_parity_bytes;
        store8<IO>(reinterpret_cast<IO*>(base) + row_off + v * 8, o);
        if (do_norm) store8<IO>(reinterpret_cast<IO*>(base + cm.result_parity_bytes / 2) + row_off + v * 8, s8);
      }
    }
  }
  // srow is reused by the next row of this CTA.
  __syncthreads();
}

template <typename IO, int MAXV>
__device__ __forceinline__ void reduce_row(const CommDev& cm, const RowSplit& rs, uint32_t parity, int t, int width,
                                        IO* out, IO* residual, const IO* norm_w, float eps, int do_norm, float* red,
                                        float* srow) {
  const int lr = rs.oneshot ? t : t - rs.first(cm.rank);
  const IO* slot0 = reinterpret_cast<const IO*>(cm.slots[cm.rank] + parity * cm.slot_parity_bytes) +
                    static_cast<size_t>(lr) * width;
  reduce_row_src<IO, MAXV>(cm, parity, slot0, static_cast<size_t>(rs.rows_cap) * width, cm.world,
                           !rs.oneshot && cm.world > 1, t, width, out, residual, norm_w, eps, do_norm, red, srow);
}

// Phase 2 with one warp per row, for launches with more rows than CTAs
// (prefill, and wide decode batches): every warp of the grid reduces its own
// rows, so rows proceed in parallel instead of one after another per CTA.
// Same arithmetic as reduce_row. Each lane requests the source and residual
// vectors of 8 vectors at a time; the warp's f32 pre-norm row waits in its
// slice of `stage` (width * 4 bytes per warp), the norm weights are staged
// once per CTA after those slices; the sum of squares is reduced with
// shuffles. Called by every thread of the CTA. IO is 16-bit.
//
// reduce_rows_warp_src takes the sources explicitly: src0(t) is row t of
// source 0, the nsrc sources src_stride elements apart; push as in
// reduce_row_src.
template <typename IO, typename Src0>
__device__ __forceinline__ void reduce_rows_warp_src(const CommDev& cm, uint32_t parity, Src0&& src0,
                                                     size_t src_stride, int nsrc, bool push, int r0, int r1,
                                                     int width, IO* out, IO* residual, const IO* norm_w, float eps,
                                                     int do_norm, uint8_t* stage) {
  static_assert(sizeof(IO) == 2, "16-bit I/O");
  constexpr int kBatch = 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int nvec = width >> 3;
  float* srow = reinterpret_cast<float*>(stage) + static_cast<size_t>(warp) * width;
  uint4* wrow = reinterpret_cast<uint4*>(reinterpret_cast<float*>(stage) + static_cast<size_t>(nwarps) * width);
  if (do_norm) {
#pragma unroll 1
    for (int v = threadIdx.x; v < nvec; v += blockDim.x) wrow[v] = __ldg(reinterpret_cast<const uint4*>(norm_w) + v);
  }
  __syncthreads();
#pragma unroll 1
  // Rows go to CTAs first, then to warps: the rows spread over every SM
  // instead of filling a few SMs six warps deep.
  for (int t = r0 + warp * static_cast<int>(gridDim.x) + static_cast<int>(blockIdx.x); t < r1;
       t += gridDim.x * nwarps) {
    const IO* slot0 = src0(t);
    const size_t row_off = static_cast<size_t>(t) * width;
    float ss = 0.f;
#pragma unroll 1
    for (int v0 = lane; v0 < nvec; v0 += 32 * kBatch) {
      uint4 sv[kBatch], rr[kBatch];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int v = min(v0 + 32 * b, nvec - 1);  // clamped: lanes past the row re-read its last vector
        sv[b] = __ldcg(reinterpret_cast<const uint4*>(slot0) + v);
        // residual is null without the norm.
        rr[b] = do_norm ? __ldcg(reinterpret_cast<const uint4*>(residual + row_off) + v) : make_uint4(0u, 0u, 0u, 0u);
      }
      float acc[kBatch][8];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) unpack8_io<IO>(sv[b], acc[b]);
#pragma unroll 1
      for (int d = 1; d < nsrc; ++d) {
#pragma unroll
        for (int b = 0; b < kBatch; ++b)
          sv[b] = __ldcg(reinterpret_cast<const uint4*>(slot0 + d * src_stride) + min(v0 + 32 * b, nvec - 1));
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
          float p[8];
          unpack8_io<IO>(sv[b], p);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[b][j] += p[j];
        }
      }
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int v = v0 + 32 * b;
        const bool in = v < nvec;
        float p[8];
        unpack8_io<IO>(rr[b], p);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          acc[b][j] = round_io<IO>(acc[b][j]);
          if (do_norm) acc[b][j] += p[j];
          if (do_norm && in) ss += acc[b][j] * acc[b][j];
        }
        if (in) {
          float4* dst = reinterpret_cast<float4*>(srow) + 2 * v;
          dst[0] = make_float4(acc[b][0], acc[b][1], acc[b][2], acc[b][3]);
          dst[1] = make_float4(acc[b][4], acc[b][5], acc[b][6], acc[b][7]);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rcp = do_norm ? rsqrtf(ss / static_cast<float>(width) + eps) : 1.f;
    __syncwarp();
#pragma unroll 1
    for (int v = lane; v < nvec; v += 32) {
      const float4 a = reinterpret_cast<const float4*>(srow)[2 * v];
      const float4 b = reinterpret_cast<const float4*>(srow)[2 * v + 1];
      float s8[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      float o[8];
      if (do_norm) {
        float w[8];
        unpack8_io<IO>(wrow[v], w);
        store8<IO>(residual + row_off + v * 8, s8);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = s8[j] * rcp * w[j];
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = s8[j];
      }
      store8<IO>(out + row_off + v * 8, o);
      if (push) {
#pragma unroll 1
        for (int d = 0; d < cm.world; ++d) {
          if (d == cm.rank) continue;
          uint8_t* base = cm.results[d] + parity * cm.result_parity_bytes;
          store8<IO>(reinterpret_cast<IO*>(base) + row_off + v * 8, o);
          if (do_norm) store8<IO>(reinterpret_cast<IO*>(base + cm.result_parity_bytes / 2) + row_off + v * 8, s8);
        }
      }
    }
    __syncwarp();  // srow is reused by this warp's next row
  }
}

template <typename IO>
__device__ __forceinline__ void reduce_rows_warp(const CommDev& cm, const RowSplit& rs, uint32_t parity, int r0,
                                                 int r1, int width, IO* out, IO* residual, const IO* norm_w,
                                                 float eps, int do_norm, uint8_t* stage) {
  const IO* slots = reinterpret_cast<const IO*>(cm.slots[cm.rank] + parity * cm.slot_parity_bytes);
  const int first = rs.first(cm.rank);
  const bool oneshot = rs.oneshot != 0;
  reduce_rows_warp_src<IO>(
      cm, parity,
      [&](int t) { return slots + static_cast<size_t>(oneshot ? t : t - first) * width; },
      static_cast<size_t>(rs.rows_cap) * width, cm.world, !rs.oneshot && cm.world > 1, r0, r1, width, out,
      residual, norm_w, eps, do_norm, stage);
}

// Phase 3 (two-shot): copy the rows owned by other ranks from this rank's
// result region into out / residual.
template <typename IO>
__device__ __forceinline__ void gather_rows(const CommDev& cm, const RowSplit& rs, uint32_t parity,
                                            int width, IO* out, IO* residual, int do_norm) {
  const uint8_t* base = cm.results[cm.rank] + parity * cm.result_parity_bytes;
  const uint4* out_plane = reinterpret_cast<const uint4*>(base);
  const uint4* res_plane = reinterpret_cast<const uint4*>(base + cm.result_parity_bytes / 2);
  // The rows owned by other ranks are two contiguous ranges, [0, r0) and
  // [r1, rows): copy them as 16-byte words, 4 per thread and step with the
  // loads issued before the stores.
  const size_t row_words = static_cast<size_t>(width) * sizeof(IO) / 16;
  const size_t r0 = static_cast<size_t>(rs.first(cm.rank)), r1 = static_cast<size_t>(rs.last(cm.rank));
  const size_t nthr = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t me = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  uint4* o4 = reinterpret_cast<uint4*>(out);
  uint4* r4 = reinterpret_cast<uint4*>(residual);
#pragma unroll 1
  for (int part = 0; part < 2; ++part) {
    const size_t w0 = part == 0 ? 0 : r1 * row_words;
    const size_t w1 = part == 0 ? r0 * row_words : static_cast<size_t>(rs.rows) * row_words;
#pragma unroll 1
    for (size_t i = w0 + me; i < w1; i += 4 * nthr) {
      uint4 ov[4], rv[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const size_t j = i + k * nthr;
        if (j < w1) {
          ov[k] = __ldcg(out_plane + j);
          if (do_norm) rv[k] = __ldcg(res_plane + j);
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const size_t j = i + k * nthr;
        if (j < w1) {
          o4[j] = ov[k];
          if (do_norm) r4[j] = rv[k];
        }
      }
    }
  }
}

}  // namespace pgb
