// Weight-streaming form of the bf16 GEMM for a handful of tokens (M <= 8), opt-in.
//
// At decode with a small batch (the 70B configuration decodes 4 sequences per step) every
// linear layer is a matrix-vector product bound by reading the weights once, and the
// tcgen05 path's fixed costs (TMEM allocation, pipeline fill, split-K partials) dominate:
// a 64 x 4096 x 4096 o_proj measured 48 us against 5 us of weight streaming.  This kernel
// has no shared-memory pipeline and no waits: a CTA of 8 warps owns kRows output columns
// (2 x kRows weight rows for SwiGLU: the gate and the up row of each column); warp w
// takes the 256-element K segments w, w + 8, ...; a lane loads 16 bytes of each weight row
// per segment (a warp reads 512 contiguous bytes of a row) and the 16 bytes of every
// token's activation at the same K, and accumulates in fp32 registers.  The 8 warps'
// partial sums meet in shared memory and are added in warp order (deterministic), and
// the epilogue rounds exactly as the tensor-core kernel's: bf16(acc); bf16(bf16(acc) + r)
// for the residual; bf16(bf16(silu(bf16(g))) * bf16(u)) for SwiGLU.  The fp32 sums are
// accumulated in another order than the tensor cores', so outputs may differ from the
// tensor-core path in the last bit of the bf16 result.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>

#include <atomic>
#include <cstdlib>

#include "common.cuh"

namespace qfc {
namespace gemv {

constexpr int kWarps = 8;  // K slices per CTA
constexpr int kRows = 4;   // output columns per CTA
constexpr int kSeg = 256;  // K elements per warp step (32 lanes x 8)

enum Epi : int { STORE = 0, SWIGLU = 1, RESIDUAL = 2 };  // the GEMM's epilogue numbering

// 8 bf16 (one 16-byte word) -> fp32
QFC_DEV void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// out[m, n] for m < M, n in this CTA's kRows columns.  x [M, K] (row stride ldx), w [N or
// 2 I, K] (row stride ldw), out [M, N_out] (row stride ldo); swiglu: up rows at I + n.
template <int EPI, int MT>
__global__ void __launch_bounds__(kWarps * 32) gemv_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                          const __nv_bfloat16* __restrict__ w, int64_t ldw,
                                                          __nv_bfloat16* __restrict__ out, int64_t ldo,
                                                          const __nv_bfloat16* __restrict__ res, int64_t ldr, int M,
                                                          int N_out, int K, int I) {
  constexpr int RW = EPI == SWIGLU ? 2 * kRows : kRows;  // weight rows per CTA
  __shared__ float red[kWarps][RW][MT];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n0 = blockIdx.x * kRows;
  // weight row of slot r (columns past N_out read row 0 and are never stored)
  int64_t wrow[RW];
#pragma unroll
  for (int r = 0; r < RW; ++r) {
    const int col = n0 + (r % kRows);
    const int n = col < N_out ? col : 0;
    wrow[r] = (EPI == SWIGLU && r >= kRows) ? (int64_t)(I + n) : (int64_t)n;
  }
  float acc[RW][MT];
#pragma unroll
  for (int r = 0; r < RW; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[r][m] = 0.f;

  const int nseg = (K + kSeg - 1) / kSeg;
  for (int s = warp; s < nseg; s += kWarps) {
    const int k0 = s * kSeg + lane * 8;
    if (k0 >= K) continue;  // K % 8 == 0: a lane's 8 elements are all in range or all out
    uint4 wv[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) wv[r] = __ldg(reinterpret_cast<const uint4*>(w + wrow[r] * ldw + k0));
    float xf[MT][8];
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m < M) {
        bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(x + (int64_t)m * ldx + k0)), xf[m]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) xf[m][i] = 0.f;
      }
    }
#pragma unroll
    for (int r = 0; r < RW; ++r) {
      float wf[8];
      bf16x8_to_f32(wv[r], wf);
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[r][m] = fmaf(wf[i], xf[m][i], acc[r][m]);
    }
  }
  // warp sums, then the warps' sums in warp order
#pragma unroll
  for (int r = 0; r < RW; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      float v = acc[r][m];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) red[warp][r][m] = v;
    }
  __syncthreads();
  const int t = threadIdx.x;
  if (t < kRows * MT) {
    const int r = t / MT, m = t % MT;
    const int col = n0 + r;
    if (m < M && col < N_out) {
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int q = 0; q < kWarps; ++q) {
        s0 += red[q][r][m];
        if constexpr (EPI == SWIGLU) s1 += red[q][kRows + r][m];
      }
      float o;
      if constexpr (EPI == SWIGLU) {
        const float gb = to_f32(from_f32<__nv_bfloat16>(s0));
        const float ub = to_f32(from_f32<__nv_bfloat16>(s1));
        const float sb = to_f32(from_f32<__nv_bfloat16>(gb / (1.f + __expf(-gb))));
        o = sb * ub;
      } else if constexpr (EPI == RESIDUAL) {
        o = to_f32(from_f32<__nv_bfloat16>(s0)) + to_f32(res[(int64_t)m * ldr + col]);
      } else {
        o = s0;
      }
      out[(int64_t)m * ldo + col] = from_f32<__nv_bfloat16>(o);
    }
  }
}

std::atomic<bool>& enabled_flag() {
  static std::atomic<bool> on{[] {
    const char* e = std::getenv("QFC_GEMM_GEMV");
    return e != nullptr && e[0] == '1';
  }()};
  return on;
}

template <int EPI>
void launch_m(int MT, dim3 grid, cudaStream_t st, const __nv_bfloat16* x, int64_t ldx, const __nv_bfloat16* w,
              int64_t ldw, __nv_bfloat16* out, int64_t ldo, const __nv_bfloat16* res, int64_t ldr, int M, int N_out,
              int K, int I) {
  switch (MT) {
    case 1: gemv_kernel<EPI, 1><<<grid, kWarps * 32, 0, st>>>(x, ldx, w, ldw, out, ldo, res, ldr, M, N_out, K, I); break;
    case 2: gemv_kernel<EPI, 2><<<grid, kWarps * 32, 0, st>>>(x, ldx, w, ldw, out, ldo, res, ldr, M, N_out, K, I); break;
    case 4: gemv_kernel<EPI, 4><<<grid, kWarps * 32, 0, st>>>(x, ldx, w, ldw, out, ldo, res, ldr, M, N_out, K, I); break;
    default: gemv_kernel<EPI, 8><<<grid, kWarps * 32, 0, st>>>(x, ldx, w, ldw, out, ldo, res, ldr, M, N_out, K, I);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace gemv

bool set_gemv(bool on) { return gemv::enabled_flag().exchange(on); }

// out = a @ b^T (epi 0), silu(a @ gate^T) * (a @ up^T) (epi 1), a @ b^T + residual (epi
// 2) on the weight-streaming kernel.  Returns false (nothing launched) unless the kernel is
// switched on and the call fits it: M <= 8 rows, K a multiple of 8, rows 16-byte aligned.
// The caller has checked shapes, dtypes and the output / residual layout.
bool gemv_try(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, int64_t epi,
              const c10::optional<at::Tensor>& residual) {
  using namespace gemv;
  if (!enabled_flag().load(std::memory_order_relaxed)) return false;
  const int M = (int)a.size(0), K = (int)a.size(1);
  if (M < 1 || M > 8 || K % 8 != 0 || (epi != STORE && epi != SWIGLU && epi != RESIDUAL)) return false;
  if (out.stride(1) != 1 || (epi == RESIDUAL && residual->stride(1) != 1)) return false;
  const int N_out = (int)out.size(1);
  const int I = epi == SWIGLU ? N_out : 0;
  const int MT = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8;
  const dim3 grid((unsigned)((N_out + kRows - 1) / kRows));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const auto* x = reinterpret_cast<const __nv_bfloat16*>(a.data_ptr());
  const auto* w = reinterpret_cast<const __nv_bfloat16*>(b.data_ptr());
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  const __nv_bfloat16* r = epi == RESIDUAL ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr;
  const int64_t ldr = epi == RESIDUAL ? residual->stride(0) : 0;
  if (epi == SWIGLU)
    launch_m<SWIGLU>(MT, grid, st, x, a.stride(0), w, b.stride(0), o, out.stride(0), r, ldr, M, N_out, K, I);
  else if (epi == RESIDUAL)
    launch_m<RESIDUAL>(MT, grid, st, x, a.stride(0), w, b.stride(0), o, out.stride(0), r, ldr, M, N_out, K, I);
  else
    launch_m<STORE>(MT, grid, st, x, a.stride(0), w, b.stride(0), o, out.stride(0), r, ldr, M, N_out, K, I);
  return true;
}

}  // namespace qfc
