// Status word that a cross-GPU kernel writes when it gives up waiting.  Kept in
// host-mapped pinned memory so the host can read it without a device synchronisation.
// Plain C++ so that host-only translation units can include it.
#pragma once

#include <stdint.h>

namespace qfc {

struct KernelStatus {
  int32_t code;    // 0 = ok; otherwise an error code below (first error wins)
  int32_t phase;   // protocol phase that timed out
  int32_t block;   // CTA index
  int32_t peer;    // rank whose flag never arrived
  uint32_t want;   // epoch waited for
  uint32_t seen;   // last value observed
  int32_t pad[2];
};

enum : int32_t { QFC_OK = 0, QFC_ERR_TIMEOUT = 1, QFC_ERR_BAD_ARGS = 2 };

}  // namespace qfc
