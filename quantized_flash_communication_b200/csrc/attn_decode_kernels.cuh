// Kernels of the paged split-KV decode attention (see attn_decode.cu for the design).
// Shared by the allocating entry point (attn_decode.cu) and the allocation-free one
// (attn_decode_noalloc.cu).
#pragma once

#include <cfloat>

#include "common.cuh"

namespace qfc {
namespace decode {

constexpr int kPart = 256;     // tokens per partition
constexpr int kWarps = 4;
constexpr int kMaxGroup = 8;   // query heads per kv head

// hd = 128: each lane holds 4 elements (8 bytes) of a 256-byte row.
template <typename T, int HD, int G>
__global__ void __launch_bounds__(kWarps * 32)
decode_partial_kernel(const T* __restrict__ q, const T* __restrict__ kc, const T* __restrict__ vc,
                      const int* __restrict__ block_table, const int* __restrict__ seq_lens, float* __restrict__ part_o,
                      float* __restrict__ part_ml, int nq, int nkv, int page, int max_pages, int n_parts, float scale) {
  constexpr int EPL = HD / 32;  // elements per lane
  const int b = blockIdx.z, kvh = blockIdx.y, part = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = seq_lens[b];
  const int t0 = part * kPart;
  const int t1 = min(L, t0 + kPart);
  __shared__ float s_m[kWarps][G], s_l[kWarps][G];
  __shared__ float s_acc[kWarps][G][HD];

  // query rows of this GQA group, pre-scaled
  float qv[G][EPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const T* qp = q + ((int64_t)b * nq + kvh * G + g) * HD + lane * EPL;
#pragma unroll
    for (int i = 0; i < EPL; ++i) qv[g][i] = to_f32(qp[i]) * scale;
  }
  float m[G], l[G], acc[G][EPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -FLT_MAX;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) acc[g][i] = 0.f;
  }
  const int* bt = block_table + (int64_t)b * max_pages;
  for (int t = t0 + warp; t < t1; t += kWarps) {
    const int pg = bt[t / page];
    const int64_t row = (((int64_t)pg * nkv + kvh) * page + (t % page)) * HD + lane * EPL;
    float kv[EPL], vv[EPL];
    if constexpr (EPL == 4) {
      const uint2 ku = *reinterpret_cast<const uint2*>(kc + row);
      const uint2 vu = *reinterpret_cast<const uint2*>(vc + row);
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        unpack_bf16x2(ku.x, kv[0], kv[1]); unpack_bf16x2(ku.y, kv[2], kv[3]);
        unpack_bf16x2(vu.x, vv[0], vv[1]); unpack_bf16x2(vu.y, vv[2], vv[3]);
      } else {
        unpack_f16x2(ku.x, kv[0], kv[1]); unpack_f16x2(ku.y, kv[2], kv[3]);
        unpack_f16x2(vu.x, vv[0], vv[1]); unpack_f16x2(vu.y, vv[2], vv[3]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        kv[i] = to_f32(kc[row + i]);
        vv[i] = to_f32(vc[row + i]);
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < EPL; ++i) s += qv[g][i] * kv[i];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(QFC_FULL_MASK, s, off);
      const float mn = fmaxf(m[g], s);
      const float corr = __expf(m[g] - mn);
      const float p = __expf(s - mn);
      l[g] = l[g] * corr + p;
#pragma unroll
      for (int i = 0; i < EPL; ++i) acc[g][i] = acc[g][i] * corr + p * vv[i];
      m[g] = mn;
    }
  }
  // merge the 4 warps
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      s_m[warp][g] = m[g];
      s_l[warp][g] = l[g];
    }
#pragma unroll
    for (int i = 0; i < EPL; ++i) s_acc[warp][g][lane * EPL + i] = acc[g][i];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * HD; idx += blockDim.x) {
    const int g = idx / HD, d = idx % HD;
    float M = -FLT_MAX;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, s_m[w][g]);
    float o = 0.f, Ls = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float c = (s_m[w][g] == -FLT_MAX) ? 0.f : __expf(s_m[w][g] - M);
      o += s_acc[w][g][d] * c;
      Ls += s_l[w][g] * c;
    }
    const int qh = kvh * G + g;
    const int64_t pi = ((int64_t)b * nq + qh) * n_parts + part;
    part_o[pi * HD + d] = o;
    if (d == 0) {
      part_ml[pi * 2] = M;
      part_ml[pi * 2 + 1] = Ls;
    }
  }
}

template <typename T, int HD>
__global__ void decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                      const int* __restrict__ seq_lens, T* __restrict__ out, int nq, int n_parts,
                                      int total_warps) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= total_warps) return;
  const int b = gw / nq, qh = gw % nq;
  const int L = seq_lens[b];
  const int np = min(n_parts, (L + kPart - 1) / kPart);
  const int64_t base = ((int64_t)b * nq + qh) * n_parts;
  float M = -FLT_MAX;
  for (int p = 0; p < np; ++p) M = fmaxf(M, part_ml[(base + p) * 2]);
  constexpr int EPL = HD / 32;
  float o[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) o[i] = 0.f;
  float Ls = 0.f;
  for (int p = 0; p < np; ++p) {
    const float mp = part_ml[(base + p) * 2];
    const float c = (mp == -FLT_MAX) ? 0.f : __expf(mp - M);
    Ls += part_ml[(base + p) * 2 + 1] * c;
#pragma unroll
    for (int i = 0; i < EPL; ++i) o[i] += part_o[(base + p) * HD + lane * EPL + i] * c;
  }
  const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
  T* op = out + ((int64_t)b * nq + qh) * HD + lane * EPL;
#pragma unroll
  for (int i = 0; i < EPL; ++i) op[i] = from_f32<T>(o[i] * inv);
}

}  // namespace decode
}  // namespace qfc
