/*
 * pgb.h - C ABI of the B200-native tensor-parallel linear path.
 *
 * One shared library (libpgb.so) exports every entry point below with plain
 * pointers, sizes and a CUDA stream handle (cudaStream_t passed as void*).
 * No torch or tvm-ffi types cross this boundary; the Python mirror of the
 * reference's layers (pico-sglang_b200/) binds it with ctypes.
 *
 * Reference interfaces each entry point replaces are cited as
 * <file>:<line> relative to the reference project root (dakingffo/pico-sglang).
 *
 * Errors. Every function returns PGB_OK (0) or a PGB_ERR_* code and records
 * a message retrievable with pgb_last_error() on the calling thread. This
 * replaces the reference's C++ PanicError / runtime_assert / NCCL_CHECK /
 * CUDA_CHECK exceptions (csrc/include/picosgl/utils.hpp:72-173); the Python
 * wrapper turns a non-zero code into an exception carrying that message.
 *
 * Streams. Work is enqueued on the given stream and never synchronises the
 * host, so calls can be captured into CUDA graphs (engine/graph.py:135-136),
 * except where a function says otherwise.
 */
#ifndef PGB_H_
#define PGB_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PGB_API __attribute__((visibility("default")))
#else
#define PGB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define PGB_OK 0
#define PGB_ERR_INVALID 1     /* bad argument: shape, dtype, alignment, pointer */
#define PGB_ERR_CUDA 2        /* a CUDA runtime or driver call failed */
#define PGB_ERR_TIMEOUT 3     /* a bounded device-side wait ran out (peer or pipeline) */
#define PGB_ERR_UNSUPPORTED 4 /* valid request this build does not implement */
#define PGB_ERR_STATE 5       /* object not ready, uid mismatch, peers not opened */

/* Element types (the three dtypes the reference communicator accepts,
 * csrc/src/pynccl.cu:60-65). */
#define PGB_F16 0
#define PGB_BF16 1
#define PGB_F32 2

/* Index element types (positions and KV-cache slots; the reference's engine
 * uses int32, engine/engine.py:138,383-395, its store kernel takes either,
 * csrc/jit/store.cu:25-28). */
#define PGB_I32 3
#define PGB_I64 4

/* Reduction ops (csrc/src/pynccl.cu:44-47). Only sum is on the hot path. */
#define PGB_OP_SUM 0

#define PGB_UID_BYTES 128     /* NCCL_UNIQUE_ID_BYTES, csrc/src/pynccl.cu:29-31 */
#define PGB_MAX_RANKS 8

/* Message of the last failed call on this thread ("" if none). */
PGB_API const char* pgb_last_error(void);

/* ABI version of this library (major * 100 + minor). */
PGB_API int pgb_version(void);

/* ------------------------------------------------------------------ comm --
 * Communicator: replaces NCCLWrapper (csrc/src/pynccl.cu:74-196) and the
 * PyNCCLCommunicator protocol (python/picosgl/distributed/pynccl.py:16-19).
 * Cross-GPU buffers are one device allocation per rank, exported with CUDA
 * IPC and opened by every peer; the fused kernels store into peers' buffers
 * over NVLink and synchronise with epoch flags and bounded waits.
 */
typedef struct pgb_comm pgb_comm;

/* Fill out[PGB_UID_BYTES] with a fresh session id. Replaces create_nccl_uid
 * (csrc/src/pynccl.cu:38-42,207). Rank 0 creates it; the host broadcasts it
 * over the CPU group as init_pynccl does (python/picosgl/distributed/pynccl.py:53-66). */
PGB_API int pgb_create_uid(uint8_t* out);

/* Create this rank's side of a communicator on CUDA device `device`.
 * max_bytes bounds one all_reduce payload served from the internal buffer,
 * as the reference's max_size_bytes (csrc/src/pynccl.cu:76-93,
 * engine/engine.py:225-227). world_size == 1 is valid (no peers to open).
 * Replaces NCCLWrapper::NCCLWrapper (csrc/src/pynccl.cu:76-93). */
PGB_API int pgb_comm_create(int rank, int world_size, size_t max_bytes, const uint8_t* uid, int device,
                    pgb_comm** out);

/* Bytes of one exported peer handle. */
PGB_API int pgb_comm_handle_size(void);

/* Export this rank's buffer handle into out[pgb_comm_handle_size()]. */
PGB_API int pgb_comm_export_handle(pgb_comm* comm, const void* unused, uint8_t* out);

/* Open every peer's buffer. handles holds world_size handles in rank order
 * (this rank's own entry is ignored). Checks that every peer was created
 * with the same uid, world size and layout; fails with PGB_ERR_STATE if not.
 * Synchronises the device. */
PGB_API int pgb_comm_open_peers(pgb_comm* comm, const uint8_t* handles);

/* Release peers, buffers and state. Synchronises the device. */
PGB_API int pgb_comm_destroy(pgb_comm* comm);

/* Budget of every device-side wait on a peer (default 30 s). */
PGB_API int pgb_comm_set_timeout_ns(pgb_comm* comm, uint64_t ns);

/* One-rank communicators only: 1 runs pgb_row_gemm_allreduce_addnorm as the
 * fused cooperative kernel; 0 (the default) runs the column GEMM followed by
 * pgb_fused_add_rmsnorm, two launches that are faster when there is no
 * all-reduce to overlap (the reference's own sequence at TP = 1,
 * python/picosgl/layers/linear.py:90-97 then norm.py:73-75). Results are the
 * same. No reference counterpart. */
PGB_API int pgb_comm_set_one_rank_path(pgb_comm* comm, int fused);

/* Multi-rank row ops (16-bit types): which exchange
 * pgb_row_gemm_allreduce_addnorm uses.
 *   PGB_XCHG_AUTO     the default: decode batches (T <= 256) on the
 *                     grid-barrier kernel (one-shot or two-shot rows by a
 *                     cost model); prefill batches (T > 256) as the column
 *                     GEMM on CTA pairs, pgb_all_reduce over its output and
 *                     pgb_fused_add_rmsnorm, measured faster there
 *   PGB_XCHG_ONESHOT  per-piece exchange kernel, every rank reduces every row
 *   PGB_XCHG_TWOSHOT  per-piece exchange kernel, reduce-scatter by feature
 *                     slices then all-gather of the reduced rows (needs
 *                     128 % world == 0 and N % 128 == 0, else one-shot)
 *   PGB_XCHG_BARRIER  the grid-barrier kernel at every T (prefill included)
 *   PGB_XCHG_NVLS     partials stay in this GPU's multicast-bound memory; the
 *                     owner of each slice sums it over every GPU with
 *                     multimem.ld_reduce and broadcasts it with multimem.st
 * Results are the same within the bf16 bar (NVLS sums in the switch with f32
 * accumulation). Tuning and diagnostics; no reference counterpart. */
#define PGB_XCHG_AUTO 0
#define PGB_XCHG_ONESHOT 1
#define PGB_XCHG_TWOSHOT 2
#define PGB_XCHG_BARRIER 3
#define PGB_XCHG_NVLS 4  /* NVLink multicast reduce (needs pgb_comm_nvls_bind; else auto) */
PGB_API int pgb_comm_set_exchange_mode(pgb_comm* comm, int mode);

/* NVLink multicast (NVLS) for the row op's reduction, set up after
 * pgb_comm_open_peers; no reference counterpart (the reference's NCCL may use
 * NVLS inside ncclAllReduce, csrc/src/pynccl.cu:84-92,127). Sequence, each
 * step on every rank before any rank starts the next (a host barrier):
 *   1. rank 0: pgb_comm_nvls_create(comm, &fd) creates the multicast object
 *      of the team and exports it as a POSIX file descriptor, which the host
 *      passes to the other ranks' processes (e.g. SCM_RIGHTS over a Unix
 *      socket);
 *   2. every rank: pgb_comm_nvls_add(comm, fd) imports it (ranks != 0; the
 *      caller closes its fd afterwards) and adds this device to the team;
 *   3. every rank: pgb_comm_nvls_bind(comm) binds and maps this device's
 *      memory (2 x 2 x max_bytes, rounded to the multicast granularity).
 * pgb_comm_nvls_supported reports whether the device can take part.
 * pgb_comm_destroy releases everything; call it on every rank after the last
 * kernel, never while another rank may still be inside a call. */
PGB_API int pgb_comm_nvls_supported(pgb_comm* comm, int* out);
PGB_API int pgb_comm_nvls_create(pgb_comm* comm, int* fd_out);
PGB_API int pgb_comm_nvls_add(pgb_comm* comm, int fd);
PGB_API int pgb_comm_nvls_bind(pgb_comm* comm);

/* Read the device status word (0 = ok, else PGB_ERR_TIMEOUT etc. as the
 * device recorded it); reset it to 0 when reset != 0. Synchronises the
 * device. */
PGB_API int pgb_comm_get_status(pgb_comm* comm, int* out, int reset);

/* This rank's internal buffer of max_bytes bytes (device pointer).
 * Replaces NCCLWrapper::get_buffer (csrc/src/pynccl.cu:181-183). */
PGB_API int pgb_comm_get_buffer(pgb_comm* comm, void** out);

/* In-place all-reduce of count elements at data (CUDA, contiguous).
 * Replaces NCCLWrapper::all_reduce (csrc/src/pynccl.cu:95-137). */
PGB_API int pgb_all_reduce(pgb_comm* comm, void* data, size_t count, int dtype, int op, void* stream);

/* out[world_size * count] = concatenation of every rank's in[count], rank 0
 * first. Replaces NCCLWrapper::all_gather (csrc/src/pynccl.cu:139-179). */
PGB_API int pgb_all_gather(pgb_comm* comm, void* out, const void* in, size_t count, int dtype,
                   void* stream);

/* --------------------------------------------------------------- linears --
 * Column-parallel GEMM: y[T, N] = x[T, K] . w[N, K]^T (+ bias[N]).
 * x, w, y row-major, element type dtype (PGB_BF16 or PGB_F16), f32
 * accumulation, K % 8 == 0, N % 8 == 0. workspace is split-K scratch of at
 * least pgb_col_gemm_workspace_size(T, N, K) bytes, zero-filled once when it
 * is allocated: its status word and split-tile counters sit in a fixed head
 * region that the kernels leave zeroed again, so calls of any shape may share
 * one workspace when they are ordered on one stream. Replaces
 * LinearTPImpl.forward = F.linear (python/picosgl/layers/linear.py:23-27) for
 * LinearColParallelMerged / LinearColParallelPartitioned (linear.py:45-73). */
PGB_API size_t pgb_col_gemm_workspace_size(int T, int N, int K);
PGB_API int pgb_col_gemm(const void* x, const void* w, const void* bias, void* y, int T, int N, int K,
                 int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* Size of the fixed per-device scratch used by pgb_col_gemm_noalloc. */
#define PGB_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)

/* pgb_col_gemm without a caller workspace and without any allocation. It has
 * no counterpart in the reference; it is for callers that cannot allocate
 * device memory when they run the GEMM (a runtime whose HBM is already given
 * to its KV-cache pool, an allocator hook, a latency path where cudaMalloc
 * would synchronise). The scratch is a fixed array of
 * PGB_NOALLOC_SCRATCH_BYTES in the library's device image, one per device:
 *  - shapes whose plan needs more scratch return PGB_ERR_INVALID;
 *  - all calls on a device share it, so calls whose GPU work overlaps
 *    (unordered streams) race and give wrong results;
 *  - the first call on each device looks up the scratch address, so make it
 *    before any stream capture; the address is kept for the life of the
 *    process, so do not use the library across a cudaDeviceReset;
 *  - PGB_F32 (check mode) uses no scratch and has no size limit;
 *  - a refused call (bad argument, size above the limit) does not touch the
 *    scratch.
 * Arguments and results are those of pgb_col_gemm. */
PGB_API int pgb_col_gemm_noalloc(const void* x, const void* w, const void* bias, void* y, int T, int N,
                                 int K, int dtype, void* stream);

/* Status word of pgb_col_gemm_noalloc on the current device: *out = PGB_OK,
 * or PGB_ERR_TIMEOUT when a bounded device-side wait of an earlier call ran
 * out (that call's output is then incomplete). The word is sticky across
 * calls; reset != 0 clears it. Synchronises the device. No reference
 * counterpart. */
PGB_API int pgb_col_gemm_noalloc_status(int* out, int reset);

/* gate_up_proj GEMM with silu_and_mul in its epilogue:
 *   gate_up  = x[T, K] . w[2I, K]^T (+ bias[2I]), rounded to dtype
 *   out[T, I] = silu(gate_up[:, :I]) * gate_up[:, I:]   (f32, rounded once)
 * w is the merged [gate; up] weight of LinearColParallelMerged
 * (python/picosgl/layers/linear.py:45-56) as the loader fills it. Replaces
 * GatedMLP.forward's gate_up_proj.forward + act_fn
 * (python/picosgl/layers/mlp.py:43-46) -> silu_and_mul
 * (python/picosgl/layers/activation.py:9-12); the [T, 2I] intermediate is
 * never stored. bf16 / f16: K % 8 == 0, I % 8 == 0, out 16-byte aligned.
 * f32 (check mode): the f32 GEMM into the workspace's exchange area, then
 * pgb_silu_and_mul. workspace: at least
 * pgb_gate_up_silu_workspace_size(T, I, K, dtype) bytes, zero-filled once
 * when allocated; it may be the one pgb_col_gemm uses on the same stream. */
PGB_API size_t pgb_gate_up_silu_workspace_size(int T, int I, int K, int dtype);
PGB_API int pgb_gate_up_silu(const void* x, const void* w, const void* bias, void* out, int T, int I,
                             int K, int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* out[T, I] = silu(x[:, :I]) * x[:, I:] for x [T, 2I] row-major, SiLU and
 * product in f32, rounded once to dtype (PGB_BF16, PGB_F16 or PGB_F32).
 * Replaces silu_and_mul (python/picosgl/layers/activation.py:9-12) on a
 * materialised gate_up tensor. */
PGB_API int pgb_silu_and_mul(const void* x, void* out, int T, int I, int dtype, void* stream);

/* qkv_proj GEMM with RoPE and the KV-cache store in its epilogue:
 *   qkv      = x[T, K] . w[N, K]^T (+ bias[N]), N = (nq + 2 nkv) hd, rounded to dtype
 *   q_out[t] = rope(q heads of qkv[t], positions[t])                  [T, nq hd]
 *   k_cache[out_loc[t]] = rope(k heads of qkv[t], positions[t])        rows of nkv hd
 *   v_cache[out_loc[t]] = v heads of qkv[t]
 * w is LinearColParallelPartitioned's local [q; k; v] weight
 * (python/picosgl/layers/linear.py:59-73). RoPE is flashinfer's
 * apply_rope_with_cos_sin_cache_inplace with is_neox = true as
 * RotaryEmbedding.forward calls it (python/picosgl/layers/rotary.py:34-60):
 * cos_sin_cache [max_position, rotary_dim] f32, cos in the first half; dims
 * d < rotary_dim/2 pair with d + rotary_dim/2, in f32, rounded once; dims from
 * rotary_dim on are not rotated. k_cache / v_cache are one layer's
 * [cache_rows, nkv, hd] storage of MHAKVCachePool
 * (python/picosgl/cache/kv/mha_pool.py:28-37). Replaces RotaryAttention.proj
 * (python/picosgl/layers/attention.py:94-117) followed by the backend's
 * store_kv (mha_pool.py:45-56 -> csrc/jit/store.cu:25-58). positions /
 * out_loc: [T] of index_dtype (PGB_I32 or PGB_I64). A token whose position or
 * slot is out of range is not written and sets the workspace's second int
 * (byte offset 4, the index-error word) to 5; the caller reads and clears it.
 * head_dim 64, 128, 256 or 512 (rotary.py:49; 64 and 128 rotate in the GEMM
 * epilogue, wider heads span several tiles and run the GEMM into the
 * workspace followed by pgb_rope_store's kernel); rotary_dim a multiple of 64
 * up to head_dim; K % 8 == 0; q_out, caches and cos_sin_cache 16-byte aligned.
 * dtype PGB_BF16 / PGB_F16, or PGB_F32 (check mode: f32 GEMM into the
 * workspace, then pgb_rope_store). workspace: at least
 * pgb_qkv_rope_store_workspace_size(...) bytes, zero-filled once; it may be
 * the column GEMM's workspace. */
PGB_API size_t pgb_qkv_rope_store_workspace_size(int T, int num_q_heads, int num_kv_heads, int head_dim,
                                                 int K, int dtype);
PGB_API int pgb_qkv_rope_store(const void* x, const void* w, const void* bias, int T, int K,
                               int num_q_heads, int num_kv_heads, int head_dim, int rotary_dim,
                               const void* positions, const void* out_loc, int index_dtype,
                               const float* cos_sin_cache, int max_position, void* q_out, void* k_cache,
                               void* v_cache, long long cache_rows, int dtype, void* workspace,
                               size_t workspace_bytes, void* stream);

/* RoPE + KV-cache store from a materialised qkv [T, (nq + 2 nkv) hd] (same
 * layout, arithmetic and limits as pgb_qkv_rope_store): flashinfer's
 * apply_rope_with_cos_sin_cache_inplace (python/picosgl/layers/rotary.py:53-59)
 * followed by store_cache (python/picosgl/kernel/store.py:37-51). qkv, q_out
 * and both caches are all of element type dtype. status is a
 * device int (the index-error word) set to 5 when a token is skipped for an
 * out-of-range index. */
PGB_API int pgb_rope_store(const void* qkv, int T, int num_q_heads, int num_kv_heads, int head_dim,
                           int rotary_dim, const void* positions, const void* out_loc, int index_dtype,
                           const float* cos_sin_cache, int max_position, void* q_out, void* k_cache,
                           void* v_cache, long long cache_rows, int dtype, int* status, void* stream);

/* Row-parallel GEMM fused with the all-reduce and the residual-add + RMSNorm
 * that consumes it:
 *   p_r      = x_local[T, K_local] . w_local[N, K_local]^T (+ bias) on rank r
 *   y        = sum_r p_r                         (over the communicator)
 *   s        = y + residual                      (f32)
 *   residual = s                                 (in place, dtype)
 *   out      = s * rsqrt(mean(s^2) + eps) * norm_w
 * Replaces LinearRowParallel.forward (python/picosgl/layers/linear.py:90-97)
 * -> NCCLWrapper::all_reduce (csrc/src/pynccl.cu:95-137) -> RMSNormFused.forward
 * with a residual (python/picosgl/layers/norm.py:56-75). With norm_w == NULL
 * the kernel stops after the reduction and writes y to out (residual unused),
 * which is LinearRowParallel.forward alone. out may alias nothing else.
 * On a one-rank communicator this is the column GEMM into out followed by
 * pgb_fused_add_rmsnorm (see pgb_comm_set_one_rank_path).
 * Payloads the communicator's buffer cannot hold run as the column GEMM into
 * out, the chunked pgb_all_reduce, then pgb_fused_add_rmsnorm (the reference
 * reduces them in place, csrc/src/pynccl.cu:127-135). */
PGB_API int pgb_row_gemm_allreduce_addnorm(pgb_comm* comm, const void* x_local, const void* w_local,
                                   const void* bias, void* residual, const void* norm_w,
                                   float eps, void* out, int T, int N, int K_local, int dtype,
                                   void* stream);

/* ----------------------------------------------------------------- norms --
 * In-place residual-add + RMSNorm: residual = x + residual; x = rmsnorm(residual) * w.
 * The FlashInfer fused_add_rmsnorm semantics used by RMSNormFused.forward
 * (python/picosgl/layers/norm.py:74): the sum is normalised in f32 and
 * stored into residual rounded to dtype. */
PGB_API int pgb_fused_add_rmsnorm(void* x, void* residual, const void* w, float eps, int T, int H,
                          int dtype, void* stream);

/* out = rmsnorm(x) * w (x unchanged); RMSNormFused.forward with residual None
 * (python/picosgl/layers/norm.py:71-72). */
PGB_API int pgb_rmsnorm(const void* x, const void* w, float eps, void* out, int T, int H, int dtype,
                void* stream);

/* ----------------------------------------------------------- diagnostics --
 * Replay on the host the work decomposition a GEMM of this shape would use
 * on `sms` SMs (all_streamk != 0: the row-parallel kernel's plan, whose
 * split-tile exchange area is the communicator's) with launch_grid CTAs (0:
 * the planned grid), and check that it covers every tile and k-block exactly
 * once, gives every split tile its CTAs with distinct k-ranges, cuts the
 * split tiles' tokens into contiguous runs, and fits the exchange area and
 * the pipeline ring. `clusters` is ignored (kept for ABI stability). Needs no
 * GPU. Internal consistency check, no reference counterpart. */
PGB_API int pgb_check_work_plan(int T, int N, int K, int sms, int all_streamk, int launch_grid,
                                int clusters);

/* Write a one-line description of the work decomposition plan_gemm picks
 * for this shape (fused_row != 0: the fused row-parallel kernel) into
 * out[out_bytes]. `clusters` is ignored (kept for ABI stability).
 * Diagnostic, no reference counterpart. */
PGB_API int pgb_describe_plan(int T, int N, int K, int sms, int fused_row, int clusters, char* out,
                              size_t out_bytes);

/* Launch features in effect for this process, as a bit mask: bit 0 set when
 * kernels are launched with programmatic dependent launch (environment
 * variable PGB_DISABLE_PDL=1 turns it off; it also turns itself off if the
 * driver refuses it). No reference counterpart. */
PGB_API int pgb_launch_features(void);

#ifdef __cplusplus
}
#endif

#endif /* PGB_H_ */
