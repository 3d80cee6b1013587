// gemm_sm100.cuh - persistent, warp-specialised tcgen05 GEMM core.
//
// Computes the products of the tensor-parallel linear layers,
//   y[T, N] = x[T, K] . W[N, K]^T      (x, W row-major bf16/f16, f32 accumulate)
// which is what LinearTPImpl.forward (python/picosgl/layers/linear.py:23-27)
// obtains from F.linear / cuBLAS.
//
// Roles inside one 192-thread CTA (one CTA per SM, persistent over tiles):
//   warp 0, one lane : TMA producer. Streams A and B k-blocks (64 wide,
//                      128-byte swizzle) into a STAGES-deep shared ring.
//   warp 1, one lane : MMA issuer. tcgen05.mma (M=128, N=BN, K=16) into one of
//                      two TMEM accumulators, so the epilogue of tile i
//                      overlaps the main loop of tile i+1. Warp 1 also owns the
//                      TMEM allocation.
//   warps 2..5       : epilogue. TMEM -> registers (tcgen05.ld 32x32b), split-K
//                      combine, then the mode-specific store.
//
// Tile orientation. The MMA M side (128 rows, "P") and N side (BN rows, "Q")
// are assigned per problem shape:
//   SWAP = false : P = tokens, Q = output features  (prefill; T large)
//   SWAP = true  : P = output features, Q = tokens  (decode; T <= 256), so the
//                  128-row MMA side is always filled by weight rows and the
//                  token side is only as wide as the batch.
//
// Split-K. A (P, Q) tile may be cut into `splits` K ranges handled by
// different CTAs. Each writes its f32 partial into scratch, and the last CTA
// to arrive on the tile's counter adds the others' partials to its own TMEM
// accumulator and runs the epilogue. Counters are reset by that CTA, so the
// scratch needs zeroing only once, when it is created.
#pragma once

#include "sm100.cuh"

namespace pgb {

constexpr int kBlockK = 64;          // k-block: one 128-byte swizzle atom of 16-bit elements
constexpr int kTileP = 128;          // MMA M
constexpr int kGemmThreads = 192;    // 6 warps
constexpr int kEpiThreads = 128;     // warps 2..5
constexpr int kMaxRanks = 8;

// Everything the GEMM loop needs to know about the problem.
struct GemmShape {
  int T, N, K;
  int kblocks;   // ceil(K / 64)
  int splits;    // K splits per (P, Q) tile, 1 <= splits <= kblocks
  int p_tiles;   // tiles along the MMA M side
  int q_tiles;   // tiles along the MMA N side
  int num_units; // p_tiles * q_tiles * splits
  float* ws;                 // split-K partials [p_tiles*q_tiles][splits][128][BN] f32
  uint32_t* tile_counters;   // [p_tiles*q_tiles], zero at rest
  int* status;               // device status word (first error wins)
  uint64_t wait_ns;          // budget for every intra-kernel wait
};

struct TileCoord {
  int p, q, s, pq, kb0, kb1;
};

__device__ __forceinline__ TileCoord decode_unit(const GemmShape& g, int unit) {
  TileCoord c;
  c.s = unit % g.splits;
  c.pq = unit / g.splits;
  c.p = c.pq % g.p_tiles;
  c.q = c.pq / g.p_tiles;
  c.kb0 = static_cast<int>((static_cast<long long>(c.s) * g.kblocks) / g.splits);
  c.kb1 = static_cast<int>((static_cast<long long>(c.s + 1) * g.kblocks) / g.splits);
  return c;
}

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = kTileP * kBlockK * 2;  // 16 KB
  static constexpr int kBBytes = BN * kBlockK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;  // two accumulators
  // Layout (from a 1024-byte aligned base): A ring, B ring, barriers.
  static constexpr int kOffA = 0;
  static constexpr int kOffB = STAGES * kABytes;
  static constexpr int kOffEpi = kOffB + STAGES * kBBytes;
  static constexpr int kEpiBytes = 32 * kTileP * 2;  // 32 tokens x 128 features, 16-bit
  static constexpr int kOffBar = kOffEpi + kEpiBytes;
  static constexpr int kBarBytes = 8 * (2 * STAGES + 5) + 64;
  static constexpr int kBytes = kOffBar + kBarBytes + 1024;  // + alignment slack
};

// Pipeline depth that fills the shared-memory budget for a tile width.
template <int BN>
constexpr int gemm_stages() {
  constexpr int kBudget = 216 * 1024;  // leaves room for the epilogue tile and barriers
  constexpr int kStage = kTileP * kBlockK * 2 + BN * kBlockK * 2;
  return kBudget / kStage > 12 ? 12 : kBudget / kStage;
}

struct GemmCtl {
  uint64_t* full;       // [STAGES]
  uint64_t* empty;      // [STAGES]
  uint64_t* acc_full;   // [2]
  uint64_t* acc_empty;  // [2]
  uint64_t* drain;      // [1] used only when unwinding after a timeout
  uint32_t* tmem_base;
  int* abort;
  int* flag;
  uint8_t* a;
  uint8_t* b;
  uint16_t* epi;  // [32][128] staging tile of the swap-orientation epilogue
};

template <int BN, int STAGES>
__device__ __forceinline__ GemmCtl gemm_carve_smem(uint8_t* raw) {
  using L = GemmSmem<BN, STAGES>;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  GemmCtl c;
  c.a = base + L::kOffA;
  c.b = base + L::kOffB;
  c.epi = reinterpret_cast<uint16_t*>(base + L::kOffEpi);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + L::kOffBar);
  c.full = bars;
  c.empty = bars + STAGES;
  c.acc_full = bars + 2 * STAGES;
  c.acc_empty = bars + 2 * STAGES + 2;
  c.drain = bars + 2 * STAGES + 4;
  c.tmem_base = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  c.abort = reinterpret_cast<int*>(c.tmem_base + 1);
  c.flag = c.abort + 1;
  return c;
}

// Producer: one thread.
template <int BN, int STAGES>
__device__ __forceinline__ void gemm_producer(const GemmShape& g, const GemmCtl& c,
                                              const CUtensorMap* tm_a, const CUtensorMap* tm_b,
                                              uint64_t hint_a, uint64_t hint_b) {
  using L = GemmSmem<BN, STAGES>;
  int stage = 0;
  uint32_t phase = 0;
  int issued[STAGES];
#pragma unroll
  for (int i = 0; i < STAGES; ++i) issued[i] = -1;
  bool ok = true;
  for (int unit = blockIdx.x; unit < g.num_units && ok; unit += gridDim.x) {
    const TileCoord tc = decode_unit(g, unit);
    for (int kb = tc.kb0; kb < tc.kb1; ++kb) {
      if (!mbar_wait(&c.empty[stage], phase ^ 1u, g.wait_ns, c.abort)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx(&c.full[stage], L::kStageBytes);
      tma_load_2d(tm_a, &c.full[stage], c.a + stage * L::kABytes, kb * kBlockK, tc.p * kTileP,
                  hint_a);
      tma_load_2d(tm_b, &c.full[stage], c.b + stage * L::kBBytes, kb * kBlockK, tc.q * BN,
                  hint_b);
      issued[stage] = static_cast<int>(phase);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
  }
  if (!ok) {
    record_error(g.status, kDevTimeoutPipeline);
    *reinterpret_cast<volatile int*>(c.abort) = 1;
    // Let every load already in flight land before the CTA can retire.
    for (int i = 0; i < STAGES; ++i)
      if (issued[i] >= 0) (void)mbar_wait(&c.full[i], static_cast<uint32_t>(issued[i]), 10000000ull, nullptr);
  }
}

// MMA issuer: one thread.
template <int BN, int STAGES>
__device__ __forceinline__ void gemm_mma(const GemmShape& g, const GemmCtl& c, uint32_t idesc) {
  using L = GemmSmem<BN, STAGES>;
  int stage = 0;
  uint32_t phase = 0;
  int acc = 0;
  uint32_t acc_phase = 0;
  const uint32_t tmem = *c.tmem_base;
  bool ok = true;
  bool any_commit = false;
  for (int unit = blockIdx.x; unit < g.num_units && ok; unit += gridDim.x) {
    const TileCoord tc = decode_unit(g, unit);
    if (!mbar_wait(&c.acc_empty[acc], acc_phase ^ 1u, g.wait_ns, c.abort)) {
      ok = false;
      break;
    }
    tc_fence_after();
    const uint32_t d_tmem = tmem + static_cast<uint32_t>(acc * BN);
    for (int kb = tc.kb0; kb < tc.kb1; ++kb) {
      if (!mbar_wait(&c.full[stage], phase, g.wait_ns, c.abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint64_t da = umma_desc_sw128_kmajor(smem_u32(c.a + stage * L::kABytes));
      const uint64_t db = umma_desc_sw128_kmajor(smem_u32(c.b + stage * L::kBBytes));
#pragma unroll
      for (int k = 0; k < kBlockK / 16; ++k) {
        // Advancing K by 16 elements = 32 bytes = 2 units of the address field.
        umma_f16_ss(d_tmem, da + static_cast<uint64_t>(2 * k), db + static_cast<uint64_t>(2 * k),
                    idesc, (kb > tc.kb0 || k > 0) ? 1u : 0u);
      }
      umma_commit(&c.empty[stage]);
      any_commit = true;
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
    if (!ok) break;
    umma_commit(&c.acc_full[acc]);
    if (++acc == 2) {
      acc = 0;
      acc_phase ^= 1u;
    }
  }
  if (!ok) {
    record_error(g.status, kDevTimeoutPipeline);
    *reinterpret_cast<volatile int*>(c.abort) = 1;
    if (any_commit) {
      // No MMA may still read shared memory or write TMEM when the CTA
      // leaves: a commit tracks every earlier MMA of this thread.
      umma_commit(c.drain);
      (void)mbar_wait(c.drain, 0u, 10000000ull, nullptr);
    }
  }
}

// Epilogue helpers --------------------------------------------------------

// TMEM address of (lane quarter of this warp, column col) in accumulator acc.
__device__ __forceinline__ uint32_t epi_taddr(uint32_t tmem, int acc, int bn, int col) {
  const uint32_t quarter = static_cast<uint32_t>((threadIdx.x >> 5) & 3);
  return tmem + ((quarter * 32u) << 16) + static_cast<uint32_t>(acc * bn + col);
}

// Row of the 128-row tile owned by this epilogue thread (= its TMEM lane).
__device__ __forceinline__ int epi_row() {
  return static_cast<int>(((threadIdx.x >> 5) & 3) * 32 + (threadIdx.x & 31));
}

template <typename IO>
__device__ __forceinline__ IO f32_to_io(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 f32_to_io<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half f32_to_io<__half>(float v) {
  return __float2half_rn(v);
}
template <typename IO>
__device__ __forceinline__ float io_to_f32(IO v);
template <>
__device__ __forceinline__ float io_to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float io_to_f32<__half>(__half v) {
  return __half2float(v);
}

// Pack 8 f32 into 8 16-bit values (16 bytes).
template <typename IO>
__device__ __forceinline__ uint4 pack8(const float* v) {
  uint4 out;
  uint16_t h[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    IO t = f32_to_io<IO>(v[j]);
    h[j] = *reinterpret_cast<uint16_t*>(&t);
  }
  out.x = static_cast<uint32_t>(h[0]) | (static_cast<uint32_t>(h[1]) << 16);
  out.y = static_cast<uint32_t>(h[2]) | (static_cast<uint32_t>(h[3]) << 16);
  out.z = static_cast<uint32_t>(h[4]) | (static_cast<uint32_t>(h[5]) << 16);
  out.w = static_cast<uint32_t>(h[6]) | (static_cast<uint32_t>(h[7]) << 16);
  return out;
}

template <typename IO>
__device__ __forceinline__ void unpack8(uint4 u, float* v) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint16_t lo = static_cast<uint16_t>(w[j] & 0xFFFFu), hi = static_cast<uint16_t>(w[j] >> 16);
    v[2 * j] = io_to_f32<IO>(*reinterpret_cast<IO*>(&lo));
    v[2 * j + 1] = io_to_f32<IO>(*reinterpret_cast<IO*>(&hi));
  }
}

// Split-K partial of (tile pq, split s): BN/4 column groups x 128 rows of
// float4, so the 32 lanes of a warp (consecutive rows) store and load 512
// contiguous bytes per instruction.
template <int BN>
__device__ __forceinline__ float4* splitk_slab(const GemmShape& g, int pq, int s) {
  return reinterpret_cast<float4*>(g.ws) + (static_cast<size_t>(pq) * g.splits + s) * (BN / 4) * kTileP;
}

// Split-K combine. On entry every epilogue thread has waited for acc_full.
// Writes this unit's partial, arrives on the tile counter and returns true
// when this CTA is the last of the tile's splits (it then owns the epilogue
// and must add the other splits' partials, see splitk_add_others).
template <int BN>
__device__ __forceinline__ bool splitk_publish(const GemmShape& g, const GemmCtl& c,
                                               const TileCoord& tc, uint32_t tmem, int acc) {
  const int row = epi_row();
  float4* mine = splitk_slab<BN>(g, tc.pq, tc.s);
#pragma unroll 1
  for (int col = 0; col < BN; col += 32) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(epi_taddr(tmem, acc, BN, col), r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 8; ++j)
      __stcg(mine + (col / 4 + j) * kTileP + row,
             make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                         __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3])));
  }
  __threadfence();
  named_bar_sync(1, kEpiThreads);
  if (threadIdx.x == 64) {
    const uint32_t old = atom_add_acqrel_gpu(&g.tile_counters[tc.pq], 1u);
    const bool last = (old == static_cast<uint32_t>(g.splits - 1));
    if (last) g.tile_counters[tc.pq] = 0u;
    *c.flag = last ? 1 : 0;
  }
  named_bar_sync(1, kEpiThreads);
  const bool last = (*reinterpret_cast<volatile int*>(c.flag) != 0);
  if (last) __threadfence();
  named_bar_sync(1, kEpiThreads);  // flag may be rewritten by the next tile
  return last;
}

// Load 32 accumulator columns starting at col and, for split-K, add the
// partials of all splits in split order (the CTA's own partial taken from
// TMEM), so the result does not depend on which split finished last.
template <int BN>
__device__ __forceinline__ void epi_load_chunk(const GemmShape& g, const TileCoord& tc,
                                               uint32_t tmem, int acc, int col, float* v) {
  uint32_t r[32];
  tmem_ld_32x32b_x32(epi_taddr(tmem, acc, BN, col), r);
  tmem_ld_wait();
  if (g.splits == 1) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    return;
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = 0.f;
  const int row = epi_row();
  for (int s = 0; s < g.splits; ++s) {
    if (s == tc.s) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += __uint_as_float(r[j]);
      continue;
    }
    const float4* src = splitk_slab<BN>(g, tc.pq, s) + (col / 4) * kTileP + row;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 t = __ldcg(src + j * kTileP);
      v[4 * j] += t.x;
      v[4 * j + 1] += t.y;
      v[4 * j + 2] += t.z;
      v[4 * j + 3] += t.w;
    }
  }
}

// Swap orientation: this thread holds v[j] = out(feature p*128 + row,
// token t0 + j), j < 32. Stage the 32 x 128 block through shared memory so
// it leaves as 16-byte pieces of token rows. emit(t, n0, piece) receives
// 8 consecutive features [n0, n0 + 8) of token t. All 128 epilogue threads
// call this together.
template <typename IO, typename Emit>
__device__ __forceinline__ void swap_epilogue_store(uint16_t* epi, const float* v, int t0, int T,
                                                    int n_base, int N, Emit&& emit) {
  const int row = epi_row();
  named_bar_sync(1, kEpiThreads);  // previous chunk fully read
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    IO h = f32_to_io<IO>(v[j]);
    epi[j * kTileP + row] = *reinterpret_cast<uint16_t*>(&h);
  }
  named_bar_sync(1, kEpiThreads);
  const int tid = static_cast<int>(threadIdx.x) - (kGemmThreads - kEpiThreads);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int idx = tid + k * kEpiThreads;  // 512 pieces: 32 tokens x 16 pieces
    const int j = idx >> 4, piece = idx & 15;
    const int t = t0 + j, n0 = n_base + piece * 8;
    if (t < T && n0 < N) emit(t, n0, *reinterpret_cast<const uint4*>(epi + j * kTileP + piece * 8));
  }
}

}  // namespace pgb
