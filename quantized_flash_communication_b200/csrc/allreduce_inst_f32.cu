// Explicit instantiations of the fused all-reduce kernels for f32 inputs.
#include "allreduce.cuh"

namespace qfc {
namespace ar {
template void dispatch_bits<float, float>(const ARParams&, const Plan&, bool, int64_t, int, int, cudaStream_t);
template void dispatch_bits<float, __half>(const ARParams&, const Plan&, bool, int64_t, int, int, cudaStream_t);
}  // namespace ar
}  // namespace qfc
