// comm.h - communicator state shared by the collective and fused kernels.
//
// Each rank owns one device allocation (the "shared buffer"), exported with
// CUDA IPC and opened by every peer, laid out identically on all ranks:
//
//   [header 4 KB]  magic, uid, world size, layout sizes (checked by peers)
//   [flags  4 KB]  flags[bar][src_rank]: epoch written by src when it passed
//                  cross-rank barrier `bar`
//   [user buffer]  max_bytes, returned by get_buffer
//   [slots  x 2]   two parities of partial rows pushed by the ranks:
//                  slot[src_rank][row][width]
//   [results x 2]  two parities of finished rows pushed by the row owners
//
// Plus one device-local allocation (not shared): status word, epoch
// counter, grid arrival counters, split-K tile counters and partials.
//
// Epochs. Every collective or fused call on a communicator increments a
// device-side epoch (read at kernel start, written back by the last CTA),
// so CUDA-graph replays need no host arguments. A flag reaching epoch e
// means "rank src passed this barrier in call e". Slot and result regions
// alternate by epoch parity; a rank can only start call e+2 after every
// rank finished reading call e's data (it waited for their call e+1
// arrivals), so a parity is never overwritten while still being read.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "../../include/pgb.h"

namespace pgb {

constexpr int kNumBars = 4;          // flags per rank: barrier ids 0..3
constexpr size_t kHeaderBytes = 4096;
constexpr size_t kFlagBytes = 4096;
constexpr uint64_t kCommMagic = 0x3230324247504255ull;  // layout tag
constexpr size_t kSplitScratchBytes = 32u << 20;        // split-tile exchange area per comm
constexpr size_t kTileCounterBytes = 64u << 10;

struct CommHeader {
  uint64_t magic;
  uint8_t uid[PGB_UID_BYTES];
  int32_t world;
  int32_t rank;
  uint64_t max_bytes;
  uint64_t slot_parity_bytes;
  uint64_t result_parity_bytes;
  uint64_t total_bytes;
};

// Device-local words (offsets inside the local allocation).
struct LocalLayout {
  static constexpr size_t kStatus = 0;      // int
  static constexpr size_t kEpoch = 64;      // uint32
  static constexpr size_t kArrive = 128;    // uint32[kNumBars]
  static constexpr size_t kCounters = 4096; // split-tile counters (zero at rest)
  static constexpr size_t kPartials = kCounters + kTileCounterBytes;
  static constexpr size_t kBytes = kPartials + kSplitScratchBytes;
};

// What a kernel needs to reach every rank's buffers; passed by value.
struct CommDev {
  int rank;
  int world;
  uint8_t* slots[PGB_MAX_RANKS];    // slot region base (parity 0) of each rank
  uint8_t* results[PGB_MAX_RANKS];  // result region base (parity 0) of each rank
  uint32_t* flags[PGB_MAX_RANKS];   // flag area of each rank
  uint64_t slot_parity_bytes;
  uint64_t result_parity_bytes;
  uint32_t* epoch;
  uint32_t* arrive;
  int* status;
  uint64_t timeout_ns;
};

}  // namespace pgb

struct pgb_comm {
  int rank;
  int world;
  int device;
  size_t max_bytes;
  uint8_t uid[PGB_UID_BYTES];
  uint8_t* buf;          // shared buffer (this rank)
  size_t buf_bytes;
  uint8_t* local;        // device-local state
  uint8_t* peer[PGB_MAX_RANKS];  // mapped shared buffer of every rank (peer[rank] == buf)
  bool peers_open;
  uint64_t slot_parity_bytes;
  uint64_t result_parity_bytes;
  uint64_t timeout_ns;
  int sm_count;
  int one_rank_fused = 0;  // world == 1: run the row op as the fused kernel (else GEMM + norm)
  int exchange_mode = PGB_XCHG_AUTO;  // multi-rank decode row ops, see pgb_comm_set_exchange_mode
  // NVLink multicast (NVLS) region, see pgb_comm_nvls_create: one physical
  // allocation on this device bound to a multicast object of the team,
  // mapped twice: nv_uc reaches this device's copy, nv_mc all copies at once.
  // Per parity: [partials max_bytes | reduced max_bytes].
  bool nvls = false;
  unsigned long long nv_mc_handle = 0;   // CUmemGenericAllocationHandle of the multicast object
  unsigned long long nv_mem_handle = 0;  // CUmemGenericAllocationHandle of this device's memory
  bool nv_added = false, nv_bound = false;
  unsigned long long nv_uc = 0, nv_mc = 0;  // CUdeviceptr of the two views (0: not mapped)
  size_t nv_bytes = 0;
  size_t nv_parity_bytes = 0;
};

namespace pgb {
// Build the kernel view of a communicator (peers must be open, or world == 1).
CommDev comm_dev(const pgb_comm* c);
size_t comm_user_offset();
size_t comm_slots_offset(const pgb_comm* c);
size_t comm_results_offset(const pgb_comm* c);
}  // namespace pgb
