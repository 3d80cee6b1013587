// comm.cu - communicator lifetime, peer exchange, all_reduce and all_gather.
//
// Replaces the reference's NCCLWrapper (csrc/src/pynccl.cu:74-196): the
// same constructor arguments (rank, world size, max bytes, 128-byte uid) and
// the same three operations (all_reduce sum in place, all_gather, get_buffer).
// Instead of an NCCL communicator over a symmetric window, every rank opens
// its peers' buffers with CUDA IPC and the kernels move data with P2P stores
// over NVLink, synchronised by epoch flags (see comm.h).
#include <fcntl.h>
#include <unistd.h>

#include <chrono>
#include <cstring>
#include <algorithm>
#include <mutex>
#include <new>

#include "comm.h"
#include "host_common.h"
#include "reduce_phases.cuh"

namespace pgb {

size_t comm_user_offset() { return kHeaderBytes + kFlagBytes; }
size_t comm_slots_offset(const pgb_comm* c) { return comm_user_offset() + align_up(c->max_bytes, 4096); }
size_t comm_results_offset(const pgb_comm* c) {
  return comm_slots_offset(c) + 2 * c->slot_parity_bytes;
}

CommDev comm_dev(const pgb_comm* c) {
  CommDev d{};
  d.rank = c->rank;
  d.world = c->world;
  for (int r = 0; r < c->world; ++r) {
    uint8_t* b = c->peer[r];
    d.slots[r] = b + comm_slots_offset(c);
    d.results[r] = b + comm_results_offset(c);
    d.flags[r] = reinterpret_cast<uint32_t*>(b + kHeaderBytes);
  }
  d.slot_parity_bytes = c->slot_parity_bytes;
  d.result_parity_bytes = c->result_parity_bytes;
  d.epoch = reinterpret_cast<uint32_t*>(c->local + LocalLayout::kEpoch);
  d.arrive = reinterpret_cast<uint32_t*>(c->local + LocalLayout::kArrive);
  d.status = reinterpret_cast<int*>(c->local + LocalLayout::kStatus);
  d.timeout_ns = c->timeout_ns;
  return d;
}

namespace {

struct DeviceGuard {
  int prev = -1;
  bool ok = false;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) ok = true;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

int dtype_bytes(int dtype) { return dtype == PGB_F32 ? 4 : 2; }

// ------------------------------------------------------------- all_reduce --
// Flat payload of `count` elements. Ownership (two-shot): contiguous blocks of
// `per` elements (a multiple of 8). Slots hold [src][per] (two-shot) or
// [src][count] (one-shot) elements of IO.
template <typename IO>
__global__ void __launch_bounds__(256) allreduce_kernel(CommDev cm, IO* data, long long count,
                                                        long long per, int oneshot) {
  __shared__ uint32_t s_epoch;
  pdl_wait();
  if (threadIdx.x == 0) s_epoch = comm_begin(cm);
  __syncthreads();
  const uint32_t e = s_epoch;
  const uint32_t parity = e & 1u;
  const long long cap = oneshot ? count : per;
  const long long tid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long nthr = static_cast<long long>(gridDim.x) * blockDim.x;

  // Phase 1: push this rank's elements into the reducing ranks' slots.
  for (long long i = tid; i < count; i += nthr) {
    const IO v = data[i];
    if (oneshot) {
      for (int d = 0; d < cm.world; ++d) {
        IO* slot = reinterpret_cast<IO*>(cm.slots[d] + parity * cm.slot_parity_bytes);
        slot[cm.rank * cap + i] = v;
      }
    } else {
      const int o = static_cast<int>(i / per);
      IO* slot = reinterpret_cast<IO*>(cm.slots[o] + parity * cm.slot_parity_bytes);
      slot[cm.rank * cap + (i - o * per)] = v;
    }
  }
  const bool ok = grid_cross_barrier(cm, kBarPartials, e, true);
  // Phase 2: reduce the owned range in rank order; write locally and push.
  const long long lo = oneshot ? 0 : min(count, cm.rank * per);
  const long long hi = oneshot ? count : min(count, (cm.rank + 1) * per);
  if (ok) {
    const IO* slot = reinterpret_cast<const IO*>(cm.slots[cm.rank] + parity * cm.slot_parity_bytes);
    for (long long i = lo + tid; i < hi; i += nthr) {
      float acc = 0.f;
      for (int src = 0; src < cm.world; ++src) {
        IO v = slot[src * cap + (i - lo)];
        if constexpr (std::is_same<IO, float>::value)
          acc += v;
        else
          acc += static_cast<float>(v);
      }
      IO r = static_cast<IO>(acc);
      data[i] = r;
      if (!oneshot) {
        for (int d = 0; d < cm.world; ++d) {
          if (d == cm.rank) continue;
          IO* res = reinterpret_cast<IO*>(cm.results[d] + parity * cm.result_parity_bytes);
          res[i] = r;
        }
      }
    }
  }
  if (!oneshot) {
    const bool ok2 = grid_cross_barrier(cm, kBarResults, e, true);
    if (ok && ok2) {
      const IO* res = reinterpret_cast<const IO*>(cm.results[cm.rank] + parity * cm.result_parity_bytes);
      for (long long i = tid; i < count; i += nthr) {
        if (i >= lo && i < hi) continue;
        data[i] = __ldcg(res + i);
      }
    }
  }
  comm_end(cm, e);
}

// 16-byte vectors of IO summed element-wise in f32 (rank order) and rounded.
template <typename IO>
__device__ __forceinline__ void acc16(float* acc, uint4 v) {
  if constexpr (std::is_same<IO, float>::value) {
    acc[0] += __uint_as_float(v.x);
    acc[1] += __uint_as_float(v.y);
    acc[2] += __uint_as_float(v.z);
    acc[3] += __uint_as_float(v.w);
  } else {
    float f[8];
    unpack8_io<IO>(v, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] += f[j];
  }
}
template <typename IO>
__device__ __forceinline__ uint4 round16(const float* acc) {
  uint4 out;
  if constexpr (std::is_same<IO, float>::value) {
    out = make_uint4(__float_as_uint(acc[0]), __float_as_uint(acc[1]), __float_as_uint(acc[2]), __float_as_uint(acc[3]));
  } else {
    IO h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) h[j] = static_cast<IO>(acc[j]);
    out = *reinterpret_cast<const uint4*>(h);
  }
  return out;
}

// all_reduce on 16-byte vectors (count a multiple of 16 / sizeof(IO), data
// 16-byte aligned); same phases and slot layout as allreduce_kernel, in
// vectors: `nvec` vectors, two-shot owners hold `per` vectors each.
template <typename IO>
__global__ void __launch_bounds__(256) allreduce_vec_kernel(CommDev cm, uint4* data, long long nvec, long long per,
                                                            int oneshot) {
  constexpr int kVecElems = 16 / static_cast<int>(sizeof(IO));
  __shared__ uint32_t s_epoch;
  pdl_wait();
  if (threadIdx.x == 0) s_epoch = comm_begin(cm);
  __syncthreads();
  const uint32_t e = s_epoch;
  const uint32_t parity = e & 1u;
  const long long cap = oneshot ? nvec : per;
  const long long tid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long nthr = static_cast<long long>(gridDim.x) * blockDim.x;
  auto slot = [&](int d) { return reinterpret_cast<uint4*>(cm.slots[d] + parity * cm.slot_parity_bytes); };
  auto result = [&](int d) { return reinterpret_cast<uint4*>(cm.results[d] + parity * cm.result_parity_bytes); };

  // Every loop takes kLd independent iterations per pass, their loads issued
  // together: one 16-byte load in flight per thread held a 64 MiB payload to
  // about 600 GB/s per phase.
  constexpr int kLd = 4;
  // Phase 1: this rank's vectors into the reducing ranks' slots.
#pragma unroll 1
  for (long long i0 = tid; i0 < nvec; i0 += kLd * nthr) {
    uint4 v[kLd];
#pragma unroll
    for (int u = 0; u < kLd; ++u)
      if (i0 + u * nthr < nvec) v[u] = __ldcg(data + i0 + u * nthr);
#pragma unroll
    for (int u = 0; u < kLd; ++u) {
      const long long i = i0 + u * nthr;
      if (i >= nvec) break;
      if (oneshot) {
        for (int d = 0; d < cm.world; ++d) slot(d)[cm.rank * cap + i] = v[u];
      } else {
        const int o = static_cast<int>(i / per);
        slot(o)[cm.rank * cap + (i - o * per)] = v[u];
      }
    }
  }
  const bool ok = grid_cross_barrier(cm, kBarPartials, e, true);
  // Phase 2: reduce the owned range in rank order; write locally and push.
  const long long lo = oneshot ? 0 : min(nvec, cm.rank * per);
  const long long hi = oneshot ? nvec : min(nvec, (cm.rank + 1) * per);
  if (ok) {
    const uint4* mine = slot(cm.rank);
#pragma unroll 1
    for (long long i0 = lo + tid; i0 < hi; i0 += 2 * nthr) {
      uint4 sv[2][PGB_MAX_RANKS];
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int r = 0; r < PGB_MAX_RANKS; ++r)
          if (r < cm.world && i0 + u * nthr < hi) sv[u][r] = __ldcg(mine + r * cap + (i0 + u * nthr - lo));
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const long long i = i0 + u * nthr;
        if (i >= hi) break;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int r = 0; r < PGB_MAX_RANKS; ++r)
          if (r < cm.world) acc16<IO>(acc, sv[u][r]);
        const uint4 out = round16<IO>(acc);
        data[i] = out;
        if (!oneshot)
          for (int d = 0; d < cm.world; ++d)
            if (d != cm.rank) result(d)[i] = out;
      }
    }
  }
  if (!oneshot) {
    const bool ok2 = grid_cross_barrier(cm, kBarResults, e, true);
    if (ok && ok2) {
      const uint4* res = result(cm.rank);
#pragma unroll 1
      for (long long i0 = tid; i0 < nvec; i0 += kLd * nthr) {
        uint4 v[kLd];
#pragma unroll
        for (int u = 0; u < kLd; ++u) {
          const long long i = i0 + u * nthr;
          if (i < nvec && (i < lo || i >= hi)) v[u] = __ldcg(res + i);
        }
#pragma unroll
        for (int u = 0; u < kLd; ++u) {
          const long long i = i0 + u * nthr;
          if (i < nvec && (i < lo || i >= hi)) data[i] = v[u];
        }
      }
    }
  }
  comm_end(cm, e);
  (void)kVecElems;
}

// ------------------------------------------------------------- all_gather --
template <typename IO>
__global__ void __launch_bounds__(256) allgather_kernel(CommDev cm, IO* out, const IO* in,
                                                        long long count, long long out_stride,
                                                        long long out_offset) {
  __shared__ uint32_t s_epoch;
  pdl_wait();
  if (threadIdx.x == 0) s_epoch = comm_begin(cm);
  __syncthreads();
  const uint32_t e = s_epoch;
  const uint32_t parity = e & 1u;
  const long long tid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long nthr = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = tid; i < count; i += nthr) {
    const IO v = in[i];
    for (int d = 0; d < cm.world; ++d) {
      IO* res = reinterpret_cast<IO*>(cm.results[d] + parity * cm.result_parity_bytes);
      res[cm.rank * count + i] = v;
    }
  }
  const bool ok = grid_cross_barrier(cm, kBarPartials, e, true);
  if (ok) {
    const IO* res = reinterpret_cast<const IO*>(cm.results[cm.rank] + parity * cm.result_parity_bytes);
    const long long total = count * cm.world;
    for (long long i = tid; i < total; i += nthr) {
      const long long r = i / count, j = i % count;
      out[r * out_stride + out_offset + j] = __ldcg(res + i);
    }
  }
  comm_end(cm, e);
}

// all_gather on 16-byte vectors: in[count] of every rank to out, where a
// rank's block starts at out + r * out_stride + out_offset (all in vectors).
__global__ void __launch_bounds__(256) allgather_vec_kernel(CommDev cm, uint4* out, const uint4* in, long long nvec,
                                                            long long out_stride, long long out_offset) {
  __shared__ uint32_t s_epoch;
  pdl_wait();
  if (threadIdx.x == 0) s_epoch = comm_begin(cm);
  __syncthreads();
  const uint32_t e = s_epoch;
  const uint32_t parity = e & 1u;
  const long long tid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long nthr = static_cast<long long>(gridDim.x) * blockDim.x;
#pragma unroll 1
  for (long long i = tid; i < nvec; i += nthr) {
    const uint4 v = __ldcg(in + i);
    for (int d = 0; d < cm.world; ++d)
      reinterpret_cast<uint4*>(cm.results[d] + parity * cm.result_parity_bytes)[cm.rank * nvec + i] = v;
  }
  const bool ok = grid_cross_barrier(cm, kBarPartials, e, true);
  if (ok) {
    const uint4* res = reinterpret_cast<const uint4*>(cm.results[cm.rank] + parity * cm.result_parity_bytes);
    const long long total = nvec * cm.world;
#pragma unroll 1
    for (long long i = tid; i < total; i += nthr) {
      const long long r = i / nvec, j = i - r * nvec;
      out[r * out_stride + out_offset + j] = __ldcg(res + i);
    }
  }
  comm_end(cm, e);
}

template <typename K, typename... Args>
int launch_coop(K kern, int grid, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  return launch_ex(cfg, /*cooperative=*/true, 1, kern, args...);
}

int check_comm(const pgb_comm* c, const char* what) {
  if (c == nullptr) return set_error(PGB_ERR_INVALID, "%s: null communicator", what);
  if (c->world > 1 && !c->peers_open)
    return set_error(PGB_ERR_STATE, "%s: peers not opened (call pgb_comm_open_peers)", what);
  int cur = -1;
  PGB_CUDA_TRY(cudaGetDevice(&cur));
  if (cur != c->device)
    return set_error(PGB_ERR_INVALID, "%s: current device %d, communicator on %d", what, cur, c->device);
  return PGB_OK;
}

template <typename IO>
int all_reduce_typed(pgb_comm* c, IO* data, size_t count, cudaStream_t s) {
  const size_t elem = sizeof(IO);
  const int n = c->world;
  constexpr size_t kVec = 16 / sizeof(IO);
  if (count % kVec == 0 && (reinterpret_cast<uintptr_t>(data) & 15u) == 0u) {
    // 16-byte vectors: chunks whose two-shot slots [n][per] and result copy fit.
    size_t max_vec = std::min(c->slot_parity_bytes, c->result_parity_bytes) / 16;
    const size_t nvec_all = count / kVec;
    for (size_t off = 0; off < nvec_all; off += max_vec) {
      const size_t cnt = std::min(max_vec, nvec_all - off);
      const size_t per = (cnt + n - 1) / n;
      const double S = static_cast<double>(cnt) * 16.0;
      const int oneshot = (n * S <= static_cast<double>(c->slot_parity_bytes)) &&
                          ((n - 1) * S / 770e9 + n * S / 6.5e12 <= 2.0 * (n - 1) / n * S / 770e9 + S / 6.5e12 + 2e-6);
      if (!oneshot && static_cast<double>(n) * per * 16.0 > static_cast<double>(c->slot_parity_bytes))
        return set_error(PGB_ERR_INVALID, "all_reduce: chunk does not fit the slots");
      const long long work = static_cast<long long>(oneshot ? cnt : per);
      int grid = static_cast<int>(std::min<long long>(c->sm_count, (work + 255) / 256));
      if (grid < 1) grid = 1;
      int rc = launch_coop(allreduce_vec_kernel<IO>, grid, s, comm_dev(c), reinterpret_cast<uint4*>(data) + off,
                           static_cast<long long>(cnt), static_cast<long long>(per), oneshot);
      if (rc) return rc;
    }
    return PGB_OK;
  }
  // Largest chunk whose two-shot slots [n][per] and result copy fit.
  size_t max_chunk = std::min(c->slot_parity_bytes / elem, c->result_parity_bytes / elem);
  max_chunk = max_chunk / 8 * 8;
  for (size_t off = 0; off < count; off += max_chunk) {
    const size_t cnt = std::min(max_chunk, count - off);
    const size_t per = ((cnt + n - 1) / n + 7) / 8 * 8;
    const double S = static_cast<double>(cnt) * elem;
    int oneshot = (n * S <= static_cast<double>(c->slot_parity_bytes)) &&
                  ((n - 1) * S / 770e9 + n * S / 6.5e12 <=
                   2.0 * (n - 1) / n * S / 770e9 + S / 6.5e12 + 2e-6);
    if (!oneshot && static_cast<double>(n) * per * elem > static_cast<double>(c->slot_parity_bytes))
      return set_error(PGB_ERR_INVALID, "all_reduce: chunk does not fit the slots");
    const long long threads = static_cast<long long>(oneshot ? cnt : per);
    int grid = static_cast<int>(std::min<long long>(c->sm_count, (threads + 255) / 256));
    if (grid < 1) grid = 1;
    int rc = launch_coop(allreduce_kernel<IO>, grid, s, comm_dev(c), data + off,
                         static_cast<long long>(cnt), static_cast<long long>(per), oneshot);
    if (rc) return rc;
  }
  return PGB_OK;
}

template <typename IO>
int all_gather_typed(pgb_comm* c, IO* out, const IO* in, size_t count, cudaStream_t s) {
  const size_t elem = sizeof(IO);
  constexpr size_t kVec = 16 / sizeof(IO);
  if (count % kVec == 0 && ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(in)) & 15u) == 0u) {
    const size_t nvec_all = count / kVec;
    const size_t max_vec = c->result_parity_bytes / 16 / c->world;
    if (max_vec == 0) return set_error(PGB_ERR_INVALID, "all_gather: buffer too small");
    for (size_t off = 0; off < nvec_all; off += max_vec) {
      const size_t cnt = std::min(max_vec, nvec_all - off);
      int grid = static_cast<int>(std::min<long long>(c->sm_count, (static_cast<long long>(cnt) * c->world + 255) / 256));
      if (grid < 1) grid = 1;
      int rc = launch_coop(allgather_vec_kernel, grid, s, comm_dev(c), reinterpret_cast<uint4*>(out),
                           reinterpret_cast<const uint4*>(in) + off, static_cast<long long>(cnt),
                           static_cast<long long>(nvec_all), static_cast<long long>(off));
      if (rc) return rc;
    }
    return PGB_OK;
  }
  size_t max_chunk = c->result_parity_bytes / elem / c->world;
  if (max_chunk == 0) return set_error(PGB_ERR_INVALID, "all_gather: buffer too small");
  for (size_t off = 0; off < count; off += max_chunk) {
    const size_t cnt = std::min(max_chunk, count - off);
    int grid = static_cast<int>(std::min<long long>(c->sm_count, (static_cast<long long>(cnt) * c->world + 255) / 256));
    if (grid < 1) grid = 1;
    int rc = launch_coop(allgather_kernel<IO>, grid, s, comm_dev(c), out, in + off,
                         static_cast<long long>(cnt), static_cast<long long>(count),
                         static_cast<long long>(off));
    if (rc) return rc;
  }
  return PGB_OK;
}

}  // namespace
}  // namespace pgb

using namespace pgb;

extern "C" int pgb_create_uid(uint8_t* out) {
  if (out == nullptr) return set_error(PGB_ERR_INVALID, "create_uid: null output");
  // Random session id; peers must present the same bytes when they open
  // each other's buffers.
  int fd = open("/dev/urandom", O_RDONLY);
  size_t got = 0;
  if (fd >= 0) {
    while (got < PGB_UID_BYTES) {
      ssize_t r = read(fd, out + got, PGB_UID_BYTES - got);
      if (r <= 0) break;
      got += static_cast<size_t>(r);
    }
    close(fd);
  }
  if (got < PGB_UID_BYTES) {
    uint64_t x = static_cast<uint64_t>(std::chrono::high_resolution_clock::now().time_since_epoch().count()) ^
                 (static_cast<uint64_t>(getpid()) << 32);
    for (size_t i = got; i < PGB_UID_BYTES; ++i) {
      x ^= x << 13;
      x ^= x >> 7;
      x ^= x << 17;
      out[i] = static_cast<uint8_t>(x);
    }
  }
  return PGB_OK;
}

extern "C" int pgb_comm_handle_size(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

extern "C" int pgb_comm_create(int rank, int world_size, size_t max_bytes, const uint8_t* uid,
                               int device, pgb_comm** out) {
  if (out == nullptr || uid == nullptr) return set_error(PGB_ERR_INVALID, "comm_create: null argument");
  *out = nullptr;
  if (world_size < 1 || world_size > PGB_MAX_RANKS)
    return set_error(PGB_ERR_INVALID, "comm_create: world size %d outside [1, %d]", world_size,
                     PGB_MAX_RANKS);
  if (rank < 0 || rank >= world_size)
    return set_error(PGB_ERR_INVALID, "comm_create: rank %d outside [0, %d)", rank, world_size);
  DeviceGuard g(device);
  if (!g.ok) return set_error(PGB_ERR_CUDA, "comm_create: cannot select device %d", device);
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc) return rc;

  pgb_comm* c = new (std::nothrow) pgb_comm();
  if (c == nullptr) return set_error(PGB_ERR_INVALID, "comm_create: out of host memory");
  c->rank = rank;
  c->world = world_size;
  c->device = device;
  c->max_bytes = std::max<size_t>(max_bytes, 8u << 20);
  std::memcpy(c->uid, uid, PGB_UID_BYTES);
  c->slot_parity_bytes = align_up(c->max_bytes + static_cast<size_t>(world_size) * 65536u, 4096);
  c->result_parity_bytes = align_up(2 * c->max_bytes + 2 * 65536u, 4096);
  c->timeout_ns = 30ull * 1000000000ull;
  c->sm_count = dev.sm_count;
  c->buf_bytes = comm_results_offset(c) + 2 * c->result_parity_bytes;

  cudaError_t e = cudaMalloc(&c->buf, c->buf_bytes);
  if (e != cudaSuccess) {
    delete c;
    return cuda_error(e, "cudaMalloc(comm buffer)");
  }
  e = cudaMalloc(&c->local, LocalLayout::kBytes);
  if (e != cudaSuccess) {
    cudaFree(c->buf);
    delete c;
    return cuda_error(e, "cudaMalloc(comm state)");
  }
  CommHeader h{};
  h.magic = kCommMagic;
  std::memcpy(h.uid, uid, PGB_UID_BYTES);
  h.world = world_size;
  h.rank = rank;
  h.max_bytes = c->max_bytes;
  h.slot_parity_bytes = c->slot_parity_bytes;
  h.result_parity_bytes = c->result_parity_bytes;
  h.total_bytes = c->buf_bytes;
  if ((e = cudaMemset(c->buf, 0, c->buf_bytes)) != cudaSuccess ||
      (e = cudaMemset(c->local, 0, LocalLayout::kBytes)) != cudaSuccess ||
      (e = cudaMemcpy(c->buf, &h, sizeof(h), cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaDeviceSynchronize()) != cudaSuccess) {
    cudaFree(c->local);
    cudaFree(c->buf);
    delete c;
    return cuda_error(e, "comm_create: initialise buffers");
  }
  c->peer[rank] = c->buf;
  c->peers_open = (world_size == 1);
  *out = c;
  return PGB_OK;
}

extern "C" int pgb_comm_export_handle(pgb_comm* comm, const void* /*unused*/, uint8_t* out) {
  if (comm == nullptr || out == nullptr) return set_error(PGB_ERR_INVALID, "export_handle: null argument");
  DeviceGuard g(comm->device);
  cudaIpcMemHandle_t h;
  PGB_CUDA_TRY(cudaIpcGetMemHandle(&h, comm->buf));
  std::memcpy(out, &h, sizeof(h));
  return PGB_OK;
}

extern "C" int pgb_comm_open_peers(pgb_comm* comm, const uint8_t* handles) {
  if (comm == nullptr || handles == nullptr) return set_error(PGB_ERR_INVALID, "open_peers: null argument");
  if (comm->peers_open) return PGB_OK;
  DeviceGuard g(comm->device);
  const size_t hs = sizeof(cudaIpcMemHandle_t);
  for (int r = 0; r < comm->world; ++r) {
    if (r == comm->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles + r * hs, hs);
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (q != comm->rank && comm->peer[q] != nullptr) {
          cudaIpcCloseMemHandle(comm->peer[q]);
          comm->peer[q] = nullptr;
        }
      return set_error(PGB_ERR_CUDA, "open_peers: cudaIpcOpenMemHandle(rank %d): %s", r,
                       cudaGetErrorString(e));
    }
    comm->peer[r] = static_cast<uint8_t*>(p);
  }
  // Validate every peer's header: same session, world size and layout.
  for (int r = 0; r < comm->world; ++r) {
    CommHeader h{};
    PGB_CUDA_TRY(cudaMemcpy(&h, comm->peer[r], sizeof(h), cudaMemcpyDeviceToHost));
    const char* why = nullptr;
    if (h.magic != kCommMagic) why = "layout tag differs";
    else if (std::memcmp(h.uid, comm->uid, PGB_UID_BYTES) != 0) why = "uid differs";
    else if (h.world != comm->world) why = "world size differs";
    else if (h.rank != r) why = "rank order differs";
    else if (h.max_bytes != comm->max_bytes) why = "max_bytes differs";
    if (why != nullptr) {
      for (int q = 0; q < comm->world; ++q)
        if (q != comm->rank && comm->peer[q] != nullptr) {
          cudaIpcCloseMemHandle(comm->peer[q]);
          comm->peer[q] = nullptr;
        }
      return set_error(PGB_ERR_STATE, "open_peers: rank %d does not match this communicator (%s)", r, why);
    }
  }
  PGB_CUDA_TRY(cudaDeviceSynchronize());
  comm->peers_open = true;
  return PGB_OK;
}

// ------------------------------------------------------------------ NVLS --
// NVLink multicast objects through the driver API, resolved at run time
// (cudaGetDriverEntryPoint), so the library does not link libcuda.

namespace pgb {
namespace {

struct NvlsDriver {
  decltype(&cuMulticastCreate) mc_create = nullptr;
  decltype(&cuMulticastAddDevice) mc_add = nullptr;
  decltype(&cuMulticastBindMem) mc_bind = nullptr;
  decltype(&cuMulticastUnbind) mc_unbind = nullptr;
  decltype(&cuMulticastGetGranularity) mc_gran = nullptr;
  decltype(&cuMemCreate) mem_create = nullptr;
  decltype(&cuMemRelease) mem_release = nullptr;
  decltype(&cuMemExportToShareableHandle) mem_export = nullptr;
  decltype(&cuMemImportFromShareableHandle) mem_import = nullptr;
  decltype(&cuMemAddressReserve) va_reserve = nullptr;
  decltype(&cuMemAddressFree) va_free = nullptr;
  decltype(&cuMemMap) mem_map = nullptr;
  decltype(&cuMemUnmap) mem_unmap = nullptr;
  decltype(&cuMemSetAccess) mem_access = nullptr;
  decltype(&cuMemGetAllocationGranularity) mem_gran = nullptr;
  decltype(&cuDeviceGetAttribute) dev_attr = nullptr;
  bool ok = false;
};

template <typename F>
bool resolve(const char* name, F& out) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &fn, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess ||
      fn == nullptr)
    return false;
  out = reinterpret_cast<F>(fn);
  return true;
}

const NvlsDriver& nvls_driver() {
  static NvlsDriver d;
  static std::once_flag once;
  std::call_once(once, [] {
    d.ok = resolve("cuMulticastCreate", d.mc_create) && resolve("cuMulticastAddDevice", d.mc_add) &&
           resolve("cuMulticastBindMem", d.mc_bind) && resolve("cuMulticastUnbind", d.mc_unbind) &&
           resolve("cuMulticastGetGranularity", d.mc_gran) && resolve("cuMemCreate", d.mem_create) &&
           resolve("cuMemRelease", d.mem_release) && resolve("cuMemExportToShareableHandle", d.mem_export) &&
           resolve("cuMemImportFromShareableHandle", d.mem_import) && resolve("cuMemAddressReserve", d.va_reserve) &&
           resolve("cuMemAddressFree", d.va_free) && resolve("cuMemMap", d.mem_map) &&
           resolve("cuMemUnmap", d.mem_unmap) && resolve("cuMemSetAccess", d.mem_access) &&
           resolve("cuMemGetAllocationGranularity", d.mem_gran) && resolve("cuDeviceGetAttribute", d.dev_attr);
  });
  return d;
}

int cu_error(CUresult r, const char* what) {
  return set_error(PGB_ERR_CUDA, "%s failed (CUresult %d)", what, static_cast<int>(r));
}

#define PGB_CU_TRY(expr)                                  \
  do {                                                    \
    CUresult _r = (expr);                                 \
    if (_r != CUDA_SUCCESS) return ::pgb::cu_error(_r, #expr); \
  } while (0)

CUmulticastObjectProp nvls_prop(const pgb_comm* c) {
  CUmulticastObjectProp prop{};
  prop.numDevices = static_cast<unsigned int>(c->world);
  prop.size = c->nv_bytes;
  prop.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  prop.flags = 0;
  return prop;
}

// Size of the multicast region: two parities of [partials | reduced] of
// max_bytes each, rounded to the multicast and allocation granularities.
int nvls_size(pgb_comm* c) {
  const NvlsDriver& d = nvls_driver();
  c->nv_parity_bytes = 2 * align_up(c->max_bytes, 4096);
  CUmulticastObjectProp prop{};
  prop.numDevices = static_cast<unsigned int>(c->world);
  prop.size = 2 * c->nv_parity_bytes;
  prop.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  size_t mc_gran = 0, mem_gran = 0;
  PGB_CU_TRY(d.mc_gran(&mc_gran, &prop, CU_MULTICAST_GRANULARITY_MINIMUM));
  CUmemAllocationProp mp{};
  mp.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  mp.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  mp.location.id = c->device;
  mp.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  PGB_CU_TRY(d.mem_gran(&mem_gran, &mp, CU_MEM_ALLOC_GRANULARITY_MINIMUM));
  const size_t gran = std::max(mc_gran, mem_gran);
  c->nv_bytes = align_up(2 * c->nv_parity_bytes, gran);
  return PGB_OK;
}

void nvls_release(pgb_comm* c) {
  const NvlsDriver& d = nvls_driver();
  if (!d.ok) return;
  CUdevice dev = c->device;
  if (c->nv_mc != 0) {
    d.mem_unmap(c->nv_mc, c->nv_bytes);
    d.va_free(c->nv_mc, c->nv_bytes);
    c->nv_mc = 0;
  }
  if (c->nv_bound) {
    d.mc_unbind(static_cast<CUmemGenericAllocationHandle>(c->nv_mc_handle), dev, 0, c->nv_bytes);
    c->nv_bound = false;
  }
  if (c->nv_uc != 0) {
    d.mem_unmap(c->nv_uc, c->nv_bytes);
    d.va_free(c->nv_uc, c->nv_bytes);
    c->nv_uc = 0;
  }
  if (c->nv_mem_handle != 0) {
    d.mem_release(static_cast<CUmemGenericAllocationHandle>(c->nv_mem_handle));
    c->nv_mem_handle = 0;
  }
  if (c->nv_mc_handle != 0) {
    d.mem_release(static_cast<CUmemGenericAllocationHandle>(c->nv_mc_handle));
    c->nv_mc_handle = 0;
  }
  c->nvls = false;
  c->nv_added = false;
}

}  // namespace
}  // namespace pgb

extern "C" int pgb_comm_nvls_supported(pgb_comm* comm, int* out) {
  if (comm == nullptr || out == nullptr) return set_error(PGB_ERR_INVALID, "nvls_supported: null argument");
  *out = 0;
  const NvlsDriver& d = nvls_driver();
  if (!d.ok || comm->world < 2) return PGB_OK;
  int v = 0;
  if (d.dev_attr(&v, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, comm->device) == CUDA_SUCCESS) *out = v != 0;
  return PGB_OK;
}

extern "C" int pgb_comm_nvls_create(pgb_comm* comm, int* fd_out) {
  if (comm == nullptr || fd_out == nullptr) return set_error(PGB_ERR_INVALID, "nvls_create: null argument");
  if (comm->rank != 0) return set_error(PGB_ERR_INVALID, "nvls_create: rank 0 creates the multicast object");
  if (comm->nv_mc_handle != 0) return set_error(PGB_ERR_STATE, "nvls_create: already created");
  const NvlsDriver& d = nvls_driver();
  if (!d.ok) return set_error(PGB_ERR_UNSUPPORTED, "nvls_create: multicast driver API unavailable");
  DeviceGuard g(comm->device);
  int rc = nvls_size(comm);
  if (rc) return rc;
  CUmulticastObjectProp prop = nvls_prop(comm);
  CUmemGenericAllocationHandle h = 0;
  PGB_CU_TRY(d.mc_create(&h, &prop));
  comm->nv_mc_handle = h;
  int fd = -1;
  const CUresult r = d.mem_export(&fd, h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
  if (r != CUDA_SUCCESS) {
    nvls_release(comm);
    return cu_error(r, "cuMemExportToShareableHandle(multicast)");
  }
  *fd_out = fd;
  return PGB_OK;
}

extern "C" int pgb_comm_nvls_add(pgb_comm* comm, int fd) {
  if (comm == nullptr) return set_error(PGB_ERR_INVALID, "nvls_add: null communicator");
  if (comm->world > 1 && !comm->peers_open) return set_error(PGB_ERR_STATE, "nvls_add: peers not opened");
  const NvlsDriver& d = nvls_driver();
  if (!d.ok) return set_error(PGB_ERR_UNSUPPORTED, "nvls_add: multicast driver API unavailable");
  DeviceGuard g(comm->device);
  if (comm->rank != 0) {
    if (comm->nv_mc_handle != 0) return set_error(PGB_ERR_STATE, "nvls_add: already added");
    if (fd < 0) return set_error(PGB_ERR_INVALID, "nvls_add: no file descriptor");
    int rc = nvls_size(comm);
    if (rc) return rc;
    CUmemGenericAllocationHandle h = 0;
    PGB_CU_TRY(d.mem_import(&h, reinterpret_cast<void*>(static_cast<uintptr_t>(fd)),
                            CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR));
    comm->nv_mc_handle = h;
  } else if (comm->nv_mc_handle == 0) {
    return set_error(PGB_ERR_STATE, "nvls_add: rank 0 has not created the multicast object");
  }
  const CUresult r = d.mc_add(static_cast<CUmemGenericAllocationHandle>(comm->nv_mc_handle), comm->device);
  if (r != CUDA_SUCCESS) return cu_error(r, "cuMulticastAddDevice");
  comm->nv_added = true;
  return PGB_OK;
}

extern "C" int pgb_comm_nvls_bind(pgb_comm* comm) {
  if (comm == nullptr) return set_error(PGB_ERR_INVALID, "nvls_bind: null communicator");
  if (!comm->nv_added) return set_error(PGB_ERR_STATE, "nvls_bind: device not added (pgb_comm_nvls_add)");
  if (comm->nv_bound) return PGB_OK;
  const NvlsDriver& d = nvls_driver();
  DeviceGuard g(comm->device);
  const CUmemGenericAllocationHandle mc = static_cast<CUmemGenericAllocationHandle>(comm->nv_mc_handle);
  CUmemAllocationProp mp{};
  mp.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  mp.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  mp.location.id = comm->device;
  mp.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  CUmemGenericAllocationHandle mem = 0;
  PGB_CU_TRY(d.mem_create(&mem, comm->nv_bytes, &mp, 0));
  comm->nv_mem_handle = mem;
  CUmemAccessDesc acc{};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = comm->device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  CUdeviceptr uc = 0, mcp = 0;
  int rc = PGB_OK;
  CUresult r = d.va_reserve(&uc, comm->nv_bytes, 0, 0, 0);
  if (r == CUDA_SUCCESS) {
    comm->nv_uc = uc;  // released by nvls_release even if the map below fails
    r = d.mem_map(uc, comm->nv_bytes, 0, mem, 0);
    if (r == CUDA_SUCCESS) r = d.mem_access(uc, comm->nv_bytes, &acc, 1);
  }
  if (r == CUDA_SUCCESS) {
    r = d.mc_bind(mc, 0, mem, 0, comm->nv_bytes, 0);
    if (r == CUDA_SUCCESS) comm->nv_bound = true;
  }
  if (r == CUDA_SUCCESS) {
    r = d.va_reserve(&mcp, comm->nv_bytes, 0, 0, 0);
    if (r == CUDA_SUCCESS) {
      comm->nv_mc = mcp;
      r = d.mem_map(mcp, comm->nv_bytes, 0, mc, 0);
      if (r == CUDA_SUCCESS) r = d.mem_access(mcp, comm->nv_bytes, &acc, 1);
    }
  }
  if (r == CUDA_SUCCESS) {
    const cudaError_t e = cudaMemset(reinterpret_cast<void*>(uc), 0, comm->nv_bytes);
    if (e != cudaSuccess) rc = cuda_error(e, "cudaMemset(nvls region)");
    const cudaError_t e2 = cudaDeviceSynchronize();
    if (!rc && e2 != cudaSuccess) rc = cuda_error(e2, "nvls_bind: synchronise");
  } else {
    rc = cu_error(r, "nvls_bind: map / bind");
  }
  if (rc) return rc;  // partial state is released by pgb_comm_destroy
  comm->nvls = true;
  return PGB_OK;
}

extern "C" int pgb_comm_destroy(pgb_comm* comm) {
  if (comm == nullptr) return PGB_OK;
  DeviceGuard g(comm->device);
  cudaDeviceSynchronize();
  pgb::nvls_release(comm);
  for (int r = 0; r < comm->world; ++r)
    if (r != comm->rank && comm->peer[r] != nullptr) cudaIpcCloseMemHandle(comm->peer[r]);
  cudaFree(comm->local);
  cudaFree(comm->buf);
  delete comm;
  return PGB_OK;
}

extern "C" int pgb_comm_set_timeout_ns(pgb_comm* comm, uint64_t ns) {
  if (comm == nullptr) return set_error(PGB_ERR_INVALID, "set_timeout: null communicator");
  if (ns == 0) return set_error(PGB_ERR_INVALID, "set_timeout: zero budget");
  comm->timeout_ns = ns;
  return PGB_OK;
}

extern "C" int pgb_comm_set_one_rank_path(pgb_comm* comm, int fused) {
  if (comm == nullptr) return set_error(PGB_ERR_INVALID, "set_one_rank_path: null communicator");
  comm->one_rank_fused = fused != 0 ? 1 : 0;
  return PGB_OK;
}

extern "C" int pgb_comm_set_exchange_mode(pgb_comm* comm, int mode) {
  if (comm == nullptr) return set_error(PGB_ERR_INVALID, "set_exchange_mode: null communicator");
  if (mode < PGB_XCHG_AUTO || mode > PGB_XCHG_NVLS)
    return set_error(PGB_ERR_INVALID, "set_exchange_mode: unknown mode %d", mode);
  comm->exchange_mode = mode;
  return PGB_OK;
}

extern "C" int pgb_comm_get_status(pgb_comm* comm, int* out, int reset) {
  if (comm == nullptr || out == nullptr) return set_error(PGB_ERR_INVALID, "get_status: null argument");
  DeviceGuard g(comm->device);
  PGB_CUDA_TRY(cudaDeviceSynchronize());
  int v = 0;
  PGB_CUDA_TRY(cudaMemcpy(&v, comm->local + LocalLayout::kStatus, sizeof(int), cudaMemcpyDeviceToHost));
  // Device codes map to PGB_ERR_TIMEOUT (waits) or PGB_ERR_INVALID.
  *out = v == kDevOk ? PGB_OK : (v == kDevBadArgs ? PGB_ERR_INVALID : PGB_ERR_TIMEOUT);
  if (reset) PGB_CUDA_TRY(cudaMemset(comm->local + LocalLayout::kStatus, 0, sizeof(int)));
  return PGB_OK;
}

extern "C" int pgb_comm_get_buffer(pgb_comm* comm, void** out) {
  if (comm == nullptr || out == nullptr) return set_error(PGB_ERR_INVALID, "get_buffer: null argument");
  *out = comm->buf + comm_user_offset();
  return PGB_OK;
}

extern "C" int pgb_all_reduce(pgb_comm* comm, void* data, size_t count, int dtype, int op,
                              void* stream) {
  int rc = check_comm(comm, "all_reduce");
  if (rc) return rc;
  if (op != PGB_OP_SUM) return set_error(PGB_ERR_UNSUPPORTED, "all_reduce: only sum is implemented");
  if (count == 0 || comm->world == 1) return PGB_OK;
  if (data == nullptr) return set_error(PGB_ERR_INVALID, "all_reduce: null data");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PGB_BF16: return all_reduce_typed(comm, static_cast<__nv_bfloat16*>(data), count, s);
    case PGB_F16: return all_reduce_typed(comm, static_cast<__half*>(data), count, s);
    case PGB_F32: return all_reduce_typed(comm, static_cast<float*>(data), count, s);
    default: return set_error(PGB_ERR_INVALID, "all_reduce: unknown dtype %d", dtype);
  }
}

extern "C" int pgb_all_gather(pgb_comm* comm, void* out, const void* in, size_t count, int dtype,
                              void* stream) {
  int rc = check_comm(comm, "all_gather");
  if (rc) return rc;
  if (count == 0) return PGB_OK;
  if (out == nullptr || in == nullptr) return set_error(PGB_ERR_INVALID, "all_gather: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (comm->world == 1) {
    PGB_CUDA_TRY(cudaMemcpyAsync(out, in, count * dtype_bytes(dtype), cudaMemcpyDeviceToDevice, s));
    return PGB_OK;
  }
  switch (dtype) {
    case PGB_BF16:
      return all_gather_typed(comm, static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(in), count, s);
    case PGB_F16:
      return all_gather_typed(comm, static_cast<__half*>(out), static_cast<const __half*>(in), count, s);
    case PGB_F32:
      return all_gather_typed(comm, static_cast<float*>(out), static_cast<const float*>(in), count, s);
    default: return set_error(PGB_ERR_INVALID, "all_gather: unknown dtype %d", dtype);
  }
}
