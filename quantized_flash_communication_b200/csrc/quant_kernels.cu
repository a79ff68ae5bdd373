// Standalone blockwise quantize / dequantize and INT4 pack / unpack kernels for sm_100a.
//
// Capabilities of the reference's Triton kernels (kernels.py:8-131) and its JIT pack /
// unpack kernels (kernels_jit.py:18-98), redesigned:
//  * one warp handles 256 contiguous elements per step with 16-byte loads; a group of
//    gs <= 256 elements is gs/8 lanes and is reduced with xor-shuffles, a larger group
//    is one warp that makes a statistics pass and a quantize pass;
//  * INT8 and INT4, asymmetric and symmetric (including symmetric INT8, which the
//    reference's dispatcher leaves unlaunched, kernels.py:97-104), fp16 or fp32 scales;
//  * every launch goes on the caller's current CUDA stream.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAException.h>

#include "common.cuh"

namespace qfc {

namespace {

constexpr int kThreads = 256;

inline int grid_for_warps(int64_t warps_needed) {
  int64_t blocks = (warps_needed + (kThreads / 32) - 1) / (kThreads / 32);
  const int64_t cap = 148 * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

template <typename ST> QFC_DEV void store_scale(ST* p, float v);
template <> QFC_DEV void store_scale<float>(float* p, float v) { *p = v; }
template <> QFC_DEV void store_scale<__half>(__half* p, float v) { *p = __float2half_rn(v); }

template <typename T, int BITS, bool SYM, typename ST>
__global__ void __launch_bounds__(kThreads)
quantize_kernel(const T* __restrict__ x, uint8_t* __restrict__ q, ST* __restrict__ s_out,
                __half* __restrict__ z_out, int64_t n, int gs) {
  using QM = QMath<BITS, SYM>;
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  if (gs <= 256) {
    const int lpg = gs >> 3;  // lanes per group
    const int64_t n_units = (n + 255) / 256;
    constexpr int kUnroll = 4;  // independent loads in flight per lane
    for (int64_t ub = warp; ub < n_units; ub += kUnroll * nwarps) {
     Raw8<T> raws[kUnroll];
#pragma unroll
     for (int k = 0; k < kUnroll; ++k)
       if (ub + k * nwarps < n_units) raws[k] = load_raw8(x, (ub + k * nwarps) * 256 + lane * 8, n);
#pragma unroll
     for (int k = 0; k < kUnroll; ++k) {
      const int64_t u = ub + k * nwarps;
      if (u >= n_units) break;
      const int64_t idx = u * 256 + lane * 8;
      const Raw8<T>& raw = raws[k];
      float v[8];
      raw8_to_f32(raw, v);
      float mn, mx;
      if constexpr (sizeof(T) == 2) group_minmax16<T>(raw.a, lpg, mn, mx);
      else group_minmax_f32(v, lpg, mn, mx);
      float s, inv, z;
      QM::params(mn, mx, s, inv, z);
      uint32_t m[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) m[i] = QM::codebits(v[i], inv, z);
      const uint2 packed = codebits8_to_u2(m);
      if (idx + 8 <= n) {
        *reinterpret_cast<uint2*>(q + idx) = packed;
      } else {
        for (int i = 0; i < 8; ++i)
          if (idx + i < n) q[idx + i] = (uint8_t)(m[i] & 0xffu);
      }
      if ((lane & (lpg - 1)) == 0 && idx < n) {
        const int64_t g = idx >> (__ffs(gs) - 1);
        store_scale<ST>(s_out + g, s);
        z_out[g] = __float2half_rn(z);
      }
     }
    }
  } else {
    const int64_t n_groups = (n + gs - 1) / gs;
    for (int64_t g = warp; g < n_groups; g += nwarps) {
      const int64_t g0 = g * gs;
      float mn = 0.f, mx = 0.f;
      bool first = true;
      for (int off = lane * 8; off < gs; off += 256) {
        float v[8];
        load8_guard(x, g0 + off, n, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          mn = first ? v[i] : fminf(mn, v[i]);
          mx = first ? v[i] : fmaxf(mx, v[i]);
          first = false;
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(QFC_FULL_MASK, mn, off));
        mx = fmaxf(mx, __shfl_xor_sync(QFC_FULL_MASK, mx, off));
      }
      float s, inv, z;
      QM::params(mn, mx, s, inv, z);
      for (int off = lane * 8; off < gs; off += 256) {
        const int64_t idx = g0 + off;
        if (idx >= n) break;
        float v[8];
        load8_guard(x, idx, n, v);
        uint32_t c[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) c[i] = QM::code(v[i], inv, z);
        if (idx + 8 <= n) {
          *reinterpret_cast<uint2*>(q + idx) = codes8_to_u2(c);
        } else {
          for (int i = 0; i < 8; ++i)
            if (idx + i < n) q[idx + i] = (uint8_t)c[i];
        }
      }
      if (lane == 0) {
        store_scale<ST>(s_out + g, s);
        z_out[g] = __float2half_rn(z);
      }
    }
  }
}

// 16-bit inputs, group sizes 16..256: a warp unit is 512 elements, 16 per lane (two
// 16-byte loads, one 16-byte store of codes), so the per-lane address, guard and group-
// parameter work is spread over twice the elements of the 8-per-lane kernel; the lane's
// 16 values reduce their (-min, max) pair as packed 16-bit values before the shuffles.
// Same codes and parameters bit for bit.
template <typename T, int BITS, bool SYM, typename ST>
__global__ void __launch_bounds__(kThreads)
quantize16_kernel(const T* __restrict__ x, uint8_t* __restrict__ q, ST* __restrict__ s_out,
                  __half* __restrict__ z_out, int64_t n, int gs_shift) {
  using QM = QMath<BITS, SYM>;
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int lpg = 1 << (gs_shift - 4);  // lanes per group
  const bool leader = (lane & (lpg - 1)) == 0;
  const int64_t n_units = (n + kUnit16 - 1) / kUnit16;
  constexpr int kUnroll = 2;  // independent 32-byte loads in flight per lane
  for (int64_t ub = warp; ub < n_units; ub += kUnroll * nwarps) {
    Raw16 raws[kUnroll];
#pragma unroll
    for (int k = 0; k < kUnroll; ++k)
      if (ub + k * nwarps < n_units) raws[k] = load_raw16(x, (ub + k * nwarps) * kUnit16 + lane * kEPL, n);
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      const int64_t u = ub + k * nwarps;
      if (u >= n_units) break;
      const int64_t idx = u * kUnit16 + lane * kEPL;
      float mn, mx;
      group_minmax16x16<T>(raws[k], lpg, mn, mx);
      float v[16];
      raw16_to_f32<T>(raws[k], v);
      float s, inv, z;
      QM::params(mn, mx, s, inv, z);
      uint32_t m[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) m[i] = QM::codebits(v[i], inv, z);
      const uint32_t(&m_lo)[8] = *reinterpret_cast<const uint32_t(*)[8]>(&m[0]);
      const uint32_t(&m_hi)[8] = *reinterpret_cast<const uint32_t(*)[8]>(&m[8]);
      const uint2 a = codebits8_to_u2(m_lo), b = codebits8_to_u2(m_hi);
      if (idx + kEPL <= n) {
        *reinterpret_cast<uint4*>(q + idx) = make_uint4(a.x, a.y, b.x, b.y);
      } else {
        for (int i = 0; i < kEPL; ++i)
          if (idx + i < n) q[idx + i] = (uint8_t)(m[i] & 0xffu);
      }
      if (leader && idx < n) {
        const int64_t g = idx >> gs_shift;
        store_scale<ST>(s_out + g, s);
        z_out[g] = __float2half_rn(z);
      }
    }
  }
}

// Codes may arrive as bytes or as fp16 values (the unpacker's output, as in the reference
// where triton_dequantize consumes unpack_int4's fp16 codes, communication.py:55-59).
template <typename QT> struct CodeLoad;
template <> struct CodeLoad<uint8_t> {
  static QFC_DEV void load(const uint8_t* q, int64_t idx, int64_t n, uint32_t (&c)[8]) {
    if (idx + 8 <= n) {
      u2_to_codes8(*reinterpret_cast<const uint2*>(q + idx), c);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) c[i] = (idx + i < n) ? q[idx + i] : 0u;
    }
  }
};
template <> struct CodeLoad<__half> {
  static QFC_DEV void load(const __half* q, int64_t idx, int64_t n, uint32_t (&c)[8]) {
    float v[8];
    load8_guard(q, idx, n, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = (uint32_t)(uint8_t)(int)v[i];
  }
};

template <typename QT, typename ST, typename OT>
__global__ void __launch_bounds__(kThreads)
dequantize_kernel(const QT* __restrict__ q, const ST* __restrict__ s, const __half* __restrict__ z,
                  OT* __restrict__ out, int64_t n, int gs) {
  const int gsh = __ffs(gs) - 1;  // group sizes are powers of two
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * 8;
  for (int64_t idx = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8; idx < n; idx += stride) {
    const int64_t g = idx >> gsh;
    const float sc = to_f32(s[g]);
    const float zz = __half2float(z[g]);
    float v[8];
    if (std::is_same<QT, uint8_t>::value && idx + 8 <= n) {
      dq_u2(*reinterpret_cast<const uint2*>(reinterpret_cast<const uint8_t*>(q) + idx), zz, sc, v);
    } else {
      uint32_t c[8];
      CodeLoad<QT>::load(q, idx, n, c);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = dq(c[i], zz, sc);
    }
    store8_guard(out, idx, n, v);
  }
}

// 8 one-byte codes -> one int32 word in the interleaved nibble order; 4 words per thread.
__global__ void __launch_bounds__(kThreads)
pack_int4_kernel(const uint8_t* __restrict__ codes, uint32_t* __restrict__ words, int64_t n_codes,
                 int64_t n_words) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * 4;
  for (int64_t w0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; w0 < n_words; w0 += stride) {
    if ((w0 + 4) * 8 <= n_codes && w0 + 4 <= n_words) {
      const uint4 a = *reinterpret_cast<const uint4*>(codes + w0 * 8);
      const uint4 b = *reinterpret_cast<const uint4*>(codes + w0 * 8 + 16);
      const uint32_t m = 0x0f0f0f0fu;
      uint4 o;
      o.x = pack_nibbles(a.x & m, a.y & m);
      o.y = pack_nibbles(a.z & m, a.w & m);
      o.z = pack_nibbles(b.x & m, b.y & m);
      o.w = pack_nibbles(b.z & m, b.w & m);
      *reinterpret_cast<uint4*>(words + w0) = o;
    } else {
      for (int64_t w = w0; w < w0 + 4 && w < n_words; ++w) {
        uint32_t c[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int64_t k = w * 8 + i;
          c[i] = (k < n_codes) ? (codes[k] & 0xfu) : 0u;
        }
        words[w] = codes8_to_int4(c);
      }
    }
  }
}

// One int32 word -> 8 fp16 codes.  (0x6400 | nibble) is the fp16 number 1024 + nibble,
// so or-ing a nibble pair into 0x64006400 and subtracting 1024 from both halves yields
// the pair of codes as half2 without an integer-to-float conversion.
QFC_DEV uint32_t nibble_pair_to_half2(uint32_t w_shifted) {
  const uint32_t bits = (w_shifted & 0x000f000fu) | 0x64006400u;
  const uint32_t k1024 = 0x64006400u;
  __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&bits), *reinterpret_cast<const __half2*>(&k1024));
  return *reinterpret_cast<uint32_t*>(&r);
}

__global__ void __launch_bounds__(kThreads)
unpack_int4_kernel(const uint32_t* __restrict__ words, __half* __restrict__ out, int64_t n_words,
                   int64_t n_out) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < n_words; w += stride) {
    const uint32_t v = words[w];
    uint4 o;
    o.x = nibble_pair_to_half2(v);
    o.y = nibble_pair_to_half2(v >> 4);
    o.z = nibble_pair_to_half2(v >> 8);
    o.w = nibble_pair_to_half2(v >> 12);
    const int64_t e0 = w * 8;
    if (e0 + 8 <= n_out) {
      *reinterpret_cast<uint4*>(out + e0) = o;
    } else {
      const __half* h = reinterpret_cast<const __half*>(&o);
      for (int i = 0; i < 8; ++i)
        if (e0 + i < n_out) out[e0 + i] = h[i];
    }
  }
}

void check_group_size(int gs) {
  TORCH_CHECK(gs >= 8 && gs <= 65536 && (gs & (gs - 1)) == 0,
              "group_size must be a power of two in [8, 65536], got ", gs);
}

at::Tensor aligned_contig(const at::Tensor& t) {
  at::Tensor c = t.contiguous();
  if (reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 != 0) c = c.clone();
  return c;
}

template <typename T, typename ST>
void launch_quantize_t(const at::Tensor& x, at::Tensor& q, at::Tensor& s, at::Tensor& z, int bits,
                       bool sym, int gs, cudaStream_t st) {
  const int64_t n = x.numel();
  const T* xp = reinterpret_cast<const T*>(x.data_ptr());
  uint8_t* qp = reinterpret_cast<uint8_t*>(q.data_ptr());
  ST* sp = reinterpret_cast<ST*>(s.data_ptr());
  __half* zp = reinterpret_cast<__half*>(z.data_ptr());
  if constexpr (sizeof(T) == 2) {
    if (gs >= 16 && gs <= 256) {
      const int grid16 = grid_for_warps((n + kUnit16 - 1) / kUnit16);
      const int gsh = __builtin_ctz((unsigned)gs);
#define QFC_LAUNCH_Q16(B, S) quantize16_kernel<T, B, S, ST><<<grid16, kThreads, 0, st>>>(xp, qp, sp, zp, n, gsh)
      if (bits == 8 && !sym) QFC_LAUNCH_Q16(8, false);
      else if (bits == 8 && sym) QFC_LAUNCH_Q16(8, true);
      else if (bits == 4 && !sym) QFC_LAUNCH_Q16(4, false);
      else QFC_LAUNCH_Q16(4, true);
#undef QFC_LAUNCH_Q16
      C10_CUDA_KERNEL_LAUNCH_CHECK();
      return;
    }
  }
  const int64_t warps = gs <= 256 ? (n + 255) / 256 : (n + gs - 1) / gs;
  const int grid = grid_for_warps(warps);
#define QFC_LAUNCH_Q(B, S) quantize_kernel<T, B, S, ST><<<grid, kThreads, 0, st>>>(xp, qp, sp, zp, n, gs)
  if (bits == 8 && !sym) QFC_LAUNCH_Q(8, false);
  else if (bits == 8 && sym) QFC_LAUNCH_Q(8, true);
  else if (bits == 4 && !sym) QFC_LAUNCH_Q(4, false);
  else QFC_LAUNCH_Q(4, true);
#undef QFC_LAUNCH_Q
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace

// x: any float tensor.  Returns (q uint8 [n], s [G] fp16|fp32, z fp16 [G]).
std::vector<at::Tensor> quantize_cuda(const at::Tensor& x_in, int64_t bits, int64_t group_size,
                                      bool sym, bool scale_fp32) {
  TORCH_CHECK(x_in.is_cuda(), "quantize: expected a CUDA tensor");
  TORCH_CHECK(bits == 8 || bits == 4, "quantize: bits must be 8 or 4, got ", bits);
  const int gs = (int)group_size;
  check_group_size(gs);
  c10::cuda::CUDAGuard guard(x_in.device());
  at::Tensor x = aligned_contig(x_in);
  const int64_t n = x.numel();
  const int64_t G = (n + gs - 1) / gs;
  auto opts = x.options();
  at::Tensor q = at::empty({n}, opts.dtype(at::kByte));
  at::Tensor s = at::empty({G}, opts.dtype(scale_fp32 ? at::kFloat : at::kHalf));
  at::Tensor z = at::empty({G}, opts.dtype(at::kHalf));
  if (n == 0) return {q, s, z};
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
#define QFC_DISPATCH_ST(T)                                                   \
  if (scale_fp32) launch_quantize_t<T, float>(x, q, s, z, (int)bits, sym, gs, st); \
  else launch_quantize_t<T, __half>(x, q, s, z, (int)bits, sym, gs, st);
  switch (x.scalar_type()) {
    case at::kBFloat16: { QFC_DISPATCH_ST(__nv_bfloat16); break; }
    case at::kHalf: { QFC_DISPATCH_ST(__half); break; }
    case at::kFloat: { QFC_DISPATCH_ST(float); break; }
    default: TORCH_CHECK(false, "quantize: unsupported dtype ", x.scalar_type());
  }
#undef QFC_DISPATCH_ST
  return {q, s, z};
}

// q: uint8/int8 codes or fp16 codes [n].  Returns out [n] in out_dtype.
at::Tensor dequantize_cuda(const at::Tensor& q_in, const at::Tensor& s_in, const at::Tensor& z_in,
                           int64_t group_size, at::ScalarType out_dtype) {
  TORCH_CHECK(q_in.is_cuda() && s_in.is_cuda() && z_in.is_cuda(), "dequantize: expected CUDA tensors");
  const int gs = (int)group_size;
  check_group_size(gs);
  c10::cuda::CUDAGuard guard(q_in.device());
  at::Tensor q = aligned_contig(q_in);
  at::Tensor s = s_in.contiguous();
  at::Tensor z = z_in.contiguous().to(at::kHalf);
  const int64_t n = q.numel();
  TORCH_CHECK(s.numel() >= (n + gs - 1) / gs && z.numel() >= (n + gs - 1) / gs,
              "dequantize: too few scales / zero points for ", n, " codes");
  at::Tensor out = at::empty({n}, q.options().dtype(out_dtype));
  if (n == 0) return out;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int64_t threads_needed = (n + 7) / 8;
  int grid = (int)std::min<int64_t>((threads_needed + kThreads - 1) / kThreads, 148 * 16);
  const __half* zp = reinterpret_cast<const __half*>(z.data_ptr());
  auto launch = [&](auto qtag, auto stag, auto otag) {
    using QT = decltype(qtag);
    using ST = decltype(stag);
    using OT = decltype(otag);
    dequantize_kernel<QT, ST, OT><<<grid, kThreads, 0, st>>>(
        reinterpret_cast<const QT*>(q.data_ptr()), reinterpret_cast<const ST*>(s.data_ptr()), zp,
        reinterpret_cast<OT*>(out.data_ptr()), n, gs);
  };
  auto with_out = [&](auto qtag, auto stag) {
    switch (out_dtype) {
      case at::kHalf: launch(qtag, stag, __half()); break;
      case at::kBFloat16: launch(qtag, stag, __nv_bfloat16()); break;
      case at::kFloat: launch(qtag, stag, float()); break;
      default: TORCH_CHECK(false, "dequantize: unsupported out dtype");
    }
  };
  auto with_scale = [&](auto qtag) {
    if (s.scalar_type() == at::kFloat) with_out(qtag, float());
    else if (s.scalar_type() == at::kHalf) with_out(qtag, __half());
    else TORCH_CHECK(false, "dequantize: scales must be fp16 or fp32");
  };
  if (q.scalar_type() == at::kByte || q.scalar_type() == at::kChar) with_scale(uint8_t());
  else if (q.scalar_type() == at::kHalf) with_scale(__half());
  else TORCH_CHECK(false, "dequantize: codes must be uint8/int8 or fp16");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

at::Tensor pack_int4_cuda(const at::Tensor& codes_in) {
  TORCH_CHECK(codes_in.is_cuda(), "pack_int4: expected a CUDA tensor");
  TORCH_CHECK(codes_in.element_size() == 1, "pack_int4: codes must be one byte each");
  c10::cuda::CUDAGuard guard(codes_in.device());
  at::Tensor codes = aligned_contig(codes_in);
  const int64_t n = codes.numel();
  const int64_t n_words = (n + 7) / 8;
  at::Tensor words = at::empty({n_words}, codes.options().dtype(at::kInt));
  if (n_words == 0) return words;
  const int64_t threads_needed = (n_words + 3) / 4;
  int grid = (int)std::min<int64_t>((threads_needed + kThreads - 1) / kThreads, 148 * 16);
  pack_int4_kernel<<<grid, kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint8_t*>(codes.data_ptr()), reinterpret_cast<uint32_t*>(words.data_ptr()),
      n, n_words);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return words;
}

at::Tensor unpack_int4_cuda(const at::Tensor& words_in, int64_t numel) {
  TORCH_CHECK(words_in.is_cuda(), "unpack_int4: expected a CUDA tensor");
  TORCH_CHECK(words_in.element_size() == 4, "unpack_int4: expected int32 words");
  c10::cuda::CUDAGuard guard(words_in.device());
  at::Tensor words = words_in.contiguous();
  const int64_t n_words = words.numel();
  TORCH_CHECK(numel <= n_words * 8, "unpack_int4: numel exceeds 8 * words");
  at::Tensor out = at::empty({numel}, words.options().dtype(at::kHalf));
  if (numel == 0) return out;
  int grid = (int)std::min<int64_t>((n_words + kThreads - 1) / kThreads, 148 * 16);
  unpack_int4_kernel<<<grid, kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint32_t*>(words.data_ptr()), reinterpret_cast<__half*>(out.data_ptr()),
      n_words, numel);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

}  // namespace qfc
