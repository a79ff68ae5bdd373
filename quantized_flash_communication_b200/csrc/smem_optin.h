// Opting a kernel into more than 48 KB of dynamic shared memory, once per device.
//
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) applies to the current device's
// context only, so a process that launches on several GPUs must set it on each.  `done`
// holds one bit per device (devices 0..63; higher ordinals set the attribute every call).
#pragma once

#include <cuda_runtime.h>

#include <atomic>

namespace qfc {

template <typename Kern>
inline cudaError_t opt_in_smem_per_device(Kern kern, int bytes, std::atomic<unsigned long long>& done) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  const unsigned long long bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return err;
}

}  // namespace qfc
