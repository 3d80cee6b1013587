// stubs.cu - entry points declared in include/pgb.h whose kernels are not in
// this build yet. Each returns PGB_ERR_UNSUPPORTED with a message.
#include "host_common.h"

#define PGB_STUB(name, ...)                                                    \
  extern "C" int name(__VA_ARGS__) {                                           \
    return pgb::set_error(PGB_ERR_UNSUPPORTED, #name " is not built yet");     \
  }

PGB_STUB(pgb_create_uid, uint8_t*)
PGB_STUB(pgb_comm_create, int, int, size_t, const uint8_t*, int, pgb_comm**)
extern "C" int pgb_comm_handle_size(void) { return 0; }
PGB_STUB(pgb_comm_export_handle, pgb_comm*, const void*, uint8_t*)
PGB_STUB(pgb_comm_open_peers, pgb_comm*, const uint8_t*)
PGB_STUB(pgb_comm_destroy, pgb_comm*)
PGB_STUB(pgb_comm_set_timeout_ns, pgb_comm*, uint64_t)
PGB_STUB(pgb_comm_get_status, pgb_comm*, int*, int)
PGB_STUB(pgb_comm_get_buffer, pgb_comm*, void**)
PGB_STUB(pgb_all_reduce, pgb_comm*, void*, size_t, int, int, void*)
PGB_STUB(pgb_all_gather, pgb_comm*, void*, const void*, size_t, int, void*)
PGB_STUB(pgb_row_gemm_allreduce_addnorm, pgb_comm*, const void*, const void*, const void*, void*,
         const void*, float, void*, int, int, int, int, void*)
PGB_STUB(pgb_fused_add_rmsnorm, void*, void*, const void*, float, int, int, int, void*)
PGB_STUB(pgb_rmsnorm, const void*, const void*, float, void*, int, int, int, void*)
