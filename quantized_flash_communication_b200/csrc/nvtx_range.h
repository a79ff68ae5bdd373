// NVTX ranges around the extension's host entry points.
//
// When enabled (QFC_NVTX=1 in the environment at import, or set_nvtx(true) at run time)
// every CUDA op of the extension pushes an NVTX range named after the op while it
// enqueues its kernels, so that a timeline tool (nsys, or ncu --nvtx with
// --nvtx-include) groups each launch under the op that issued it.  Disabled, the cost is
// one relaxed atomic load per call.  nvtx3 is header-only: it loads the tool's injection
// library only when one is attached, and does nothing otherwise.
#pragma once
#include <nvtx3/nvToolsExt.h>

#include <atomic>
#include <cstdlib>
#include <utility>

namespace qfc {

inline std::atomic<bool>& nvtx_flag() {
  static std::atomic<bool> on{[] {
    const char* e = std::getenv("QFC_NVTX");
    return e != nullptr && e[0] == '1';
  }()};
  return on;
}

inline bool nvtx_enabled() { return nvtx_flag().load(std::memory_order_relaxed); }
inline void set_nvtx(bool on) { nvtx_flag().store(on, std::memory_order_relaxed); }

class NvtxRange {
 public:
  explicit NvtxRange(const char* name) : on_(nvtx_enabled()) {
    if (on_) nvtxRangePushA(name);
  }
  ~NvtxRange() {
    if (on_) nvtxRangePop();
  }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;

 private:
  bool on_;
};

// traced("name", &fn): a callable with fn's exact signature that runs fn inside an NVTX
// range called "name".  Parameters keep their reference types, so tensors bound by
// reference (outputs) are passed through unchanged.
template <typename R, typename... A>
auto traced(const char* name, R (*fn)(A...)) {
  return [name, fn](A... a) -> R {
    NvtxRange r(name);
    return fn(std::forward<A>(a)...);
  };
}

}  // namespace qfc
