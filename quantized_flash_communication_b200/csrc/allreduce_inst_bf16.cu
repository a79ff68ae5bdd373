// Explicit instantiations of the fused all-reduce kernels for bf16 inputs.
#include "allreduce.cuh"

namespace qfc {
namespace ar {
template void dispatch_bits<__nv_bfloat16, __nv_bfloat16>(const ARParams&, const Plan&, bool, int64_t, int, int, cudaStream_t);
template void dispatch_bits<__nv_bfloat16, __half>(const ARParams&, const Plan&, bool, int64_t, int, int, cudaStream_t);
template void dispatch_gemm_reduce<__nv_bfloat16, __nv_bfloat16>(const ARParams&, const Plan&, int64_t, int,
                                                                 cudaStream_t);
}  // namespace ar
}  // namespace qfc
