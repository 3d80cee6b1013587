// capi.cu - C ABI entry points that are not kernels: errors and version.
#include "host_common.h"

namespace pgb {
const char* last_error_cstr();
}

extern "C" const char* pgb_last_error(void) { return pgb::last_error_cstr(); }

extern "C" int pgb_version(void) { return 100; }

extern "C" int pgb_launch_features(void) { return pgb::pdl_enabled() ? 1 : 0; }
