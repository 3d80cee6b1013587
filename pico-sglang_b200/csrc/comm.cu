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

extern "C" int pgb_comm_destroy(pgb_comm* comm) {
  if (comm == nullptr) return PGB_OK;
  DeviceGuard g(comm->device);
  cudaDeviceSynchronize();
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
  if (mode < PGB_XCHG_AUTO || mode > PGB_XCHG_BARRIER)
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
