// Library-wide C-ABI pieces: the per-thread error message and the ABI version.
#include "capi_common.h"

namespace mad {

char* error_buffer() {
  static thread_local char buf[kErrorBufferSize] = {0};
  return buf;
}

}  // namespace mad

extern "C" const char* mad_last_error(void) { return mad::error_buffer(); }

extern "C" int32_t mad_abi_version(void) { return 4; }
