// Shared device helpers: dtype conversion, 8-element vector I/O, the quantizer's
// per-group arithmetic, INT4 nibble packing, and the memory-ordering / bounded-wait
// primitives used by every cross-GPU kernel.
//
// The quantizer arithmetic here is the device restatement of the torch specification in
// quantization.py (quantize_groups / dequantize_groups); tests compare both bit-for-bit.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "status.h"

#define QFC_DEV __device__ __forceinline__
#define QFC_FULL_MASK 0xffffffffu

namespace qfc {

// ------------------------------------------------------------------------------------
// Scalar conversions
// ------------------------------------------------------------------------------------
template <typename T> QFC_DEV float to_f32(T v);
template <> QFC_DEV float to_f32<float>(float v) { return v; }
template <> QFC_DEV float to_f32<__half>(__half v) { return __half2float(v); }
template <> QFC_DEV float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> QFC_DEV T from_f32(float v);
template <> QFC_DEV float from_f32<float>(float v) { return v; }
template <> QFC_DEV __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> QFC_DEV __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// ------------------------------------------------------------------------------------
// 8 consecutive elements <-> float[8].  16-bit types move as one 16-byte access, fp32
// as two.  The caller guarantees 16-byte alignment of p for the unguarded forms.
// ------------------------------------------------------------------------------------
QFC_DEV void unpack_bf16x2(uint32_t u, float& a, float& b) {
  a = __uint_as_float(u << 16);
  b = __uint_as_float(u & 0xffff0000u);
}
QFC_DEV void unpack_f16x2(uint32_t u, float& a, float& b) {
  __half2 h = *reinterpret_cast<__half2*>(&u);
  float2 f = __half22float2(h);
  a = f.x;
  b = f.y;
}
QFC_DEV uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
QFC_DEV uint32_t pack_f16x2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <typename T> struct Vec8IO;

template <> struct Vec8IO<__nv_bfloat16> {
  static QFC_DEV void load(const __nv_bfloat16* p, float (&v)[8]) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    unpack_bf16x2(u.x, v[0], v[1]);
    unpack_bf16x2(u.y, v[2], v[3]);
    unpack_bf16x2(u.z, v[4], v[5]);
    unpack_bf16x2(u.w, v[6], v[7]);
  }
  static QFC_DEV void load_cg(const __nv_bfloat16* p, float (&v)[8]) {
    uint4 u = __ldcg(reinterpret_cast<const uint4*>(p));
    unpack_bf16x2(u.x, v[0], v[1]);
    unpack_bf16x2(u.y, v[2], v[3]);
    unpack_bf16x2(u.z, v[4], v[5]);
    unpack_bf16x2(u.w, v[6], v[7]);
  }
  static QFC_DEV uint4 pack(const float (&v)[8]) {
    return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                      pack_bf16x2(v[6], v[7]));
  }
  static QFC_DEV void store(__nv_bfloat16* p, const float (&v)[8]) {
    *reinterpret_cast<uint4*>(p) = pack(v);
  }
};

template <> struct Vec8IO<__half> {
  static QFC_DEV void load(const __half* p, float (&v)[8]) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    unpack_f16x2(u.x, v[0], v[1]);
    unpack_f16x2(u.y, v[2], v[3]);
    unpack_f16x2(u.z, v[4], v[5]);
    unpack_f16x2(u.w, v[6], v[7]);
  }
  static QFC_DEV void load_cg(const __half* p, float (&v)[8]) {
    uint4 u = __ldcg(reinterpret_cast<const uint4*>(p));
    unpack_f16x2(u.x, v[0], v[1]);
    unpack_f16x2(u.y, v[2], v[3]);
    unpack_f16x2(u.z, v[4], v[5]);
    unpack_f16x2(u.w, v[6], v[7]);
  }
  static QFC_DEV uint4 pack(const float (&v)[8]) {
    return make_uint4(pack_f16x2(v[0], v[1]), pack_f16x2(v[2], v[3]), pack_f16x2(v[4], v[5]),
                      pack_f16x2(v[6], v[7]));
  }
  static QFC_DEV void store(__half* p, const float (&v)[8]) { *reinterpret_cast<uint4*>(p) = pack(v); }
};

template <> struct Vec8IO<float> {
  static QFC_DEV void load(const float* p, float (&v)[8]) {
    float4 a = reinterpret_cast<const float4*>(p)[0];
    float4 b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  static QFC_DEV void load_cg(const float* p, float (&v)[8]) {
    float4 a = __ldcg(reinterpret_cast<const float4*>(p));
    float4 b = __ldcg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  static QFC_DEV void store(float* p, const float (&v)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
};

// Elements at or beyond n read as 0.0 (the zero padding of a partial last group).
template <typename T>
QFC_DEV void load8_guard(const T* base, int64_t idx, int64_t n, float (&v)[8]) {
  if (idx + 8 <= n) {
    Vec8IO<T>::load(base + idx, v);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = (idx + i < n) ? to_f32(base[idx + i]) : 0.f;
  }
}

template <typename T>
QFC_DEV void store8_guard(T* base, int64_t idx, int64_t n, const float (&v)[8]) {
  if (idx + 8 <= n) {
    Vec8IO<T>::store(base + idx, v);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (idx + i < n) base[idx + i] = from_f32<T>(v[i]);
  }
}

// ------------------------------------------------------------------------------------
// Quantizer arithmetic (must stay identical to quantization.quantize_groups)
// ------------------------------------------------------------------------------------
// Round half away from zero.
QFC_DEV float rhaz(float v) { return roundf(v); }

template <int BITS, bool SYM>
struct QMath {
  static constexpr float QMAX = float((1 << BITS) - 1);
  // Group statistics -> (scale, 1/scale, zero point), all fp32.
  static QFC_DEV void params(float mn, float mx, float& s, float& inv, float& z) {
    if (SYM) {
      const float a = fmaxf(-mn, mx);  // == max |x| over the group
      s = a / (QMAX * 0.5f);
      if (s < 1e-9f) s = 1.f;
      inv = 1.f / s;
      z = (QMAX + 1.f) * 0.5f;
    } else {
      s = (mx - mn) / QMAX;
      if (s < 1e-9f) s = 1.f;
      inv = 1.f / s;
      z = fminf(fmaxf(rhaz(-mn * inv), 0.f), QMAX);
    }
  }
  static QFC_DEV uint32_t code(float x, float inv, float z) {
    return (uint32_t)fminf(fmaxf(rhaz(x * inv) + z, 0.f), QMAX);
  }
};

// Dequantize one code.  __fmul_rn keeps the product from being fused into a following
// add, so that sums match the oracle's separately rounded (q - z) * s terms.
QFC_DEV float dq(uint32_t c, float z, float s) { return __fmul_rn((float)c - z, s); }

// 8 byte codes (element order) <-> uint2
QFC_DEV uint2 codes8_to_u2(const uint32_t (&c)[8]) {
  return make_uint2(c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24),
                    c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24));
}
QFC_DEV void u2_to_codes8(uint2 u, uint32_t (&c)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    c[i] = (u.x >> (8 * i)) & 0xffu;
    c[4 + i] = (u.y >> (8 * i)) & 0xffu;
  }
}

// INT4: 8 codes -> one word; nibble k (from the LSB) holds element {0,2,4,6,1,3,5,7}[k].
QFC_DEV uint32_t pack_nibbles(uint32_t lo, uint32_t hi) {
  // lo holds codes 0..3 as bytes, hi codes 4..7; each byte <= 15.
  uint32_t e = __byte_perm(lo, hi, 0x6420);  // bytes: c0 c2 c4 c6
  uint32_t o = __byte_perm(lo, hi, 0x7531);  // bytes: c1 c3 c5 c7
  e |= e >> 4;                               // byte0 = c0|c2<<4, byte2 = c4|c6<<4
  o |= o >> 4;
  return __byte_perm(e, o, 0x6420);
}
QFC_DEV uint32_t codes8_to_int4(const uint32_t (&c)[8]) {
  uint2 u = codes8_to_u2(c);
  return pack_nibbles(u.x & 0x0f0f0f0fu, u.y & 0x0f0f0f0fu);
}
QFC_DEV void int4_to_codes8(uint32_t w, uint32_t (&c)[8]) {
  const uint32_t a = w & 0x0f0f0f0fu;          // bytes: c0 c4 c1 c5
  const uint32_t b = (w >> 4) & 0x0f0f0f0fu;   // bytes: c2 c6 c3 c7
  uint2 u = make_uint2(__byte_perm(a, b, 0x6420), __byte_perm(a, b, 0x7531));
  u2_to_codes8(u, c);
}

// ------------------------------------------------------------------------------------
// Cross-GPU memory ordering and bounded waits
// ------------------------------------------------------------------------------------
QFC_DEV uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
QFC_DEV void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
QFC_DEV void red_release_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
QFC_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

QFC_DEV void report_timeout(KernelStatus* st, int phase, int block, int peer, uint32_t want,
                            uint32_t seen) {
  if (st == nullptr) return;
  if (atomicCAS(&st->code, 0, QFC_ERR_TIMEOUT) == 0) {
    st->phase = phase;
    st->block = block;
    st->peer = peer;
    st->want = want;
    st->seen = seen;
    __threadfence_system();
  }
}

// Spin until *flag >= want (wrap-around aware) or the deadline passes.  Two bounds: the
// %globaltimer deadline, and an iteration cap in case the timer does not advance.
// Returns true when the flag arrived.
QFC_DEV bool wait_flag_geq(const uint32_t* flag, uint32_t want, uint64_t deadline_ns,
                           uint32_t& seen) {
  constexpr uint32_t kMaxPolls = 1u << 30;
  for (uint32_t it = 0; it < kMaxPolls; ++it) {
    seen = ld_acquire_sys(flag);
    if ((int32_t)(seen - want) >= 0) return true;
    if ((it & 31u) == 31u) {
      if (globaltimer_ns() > deadline_ns) return false;
      if (it > 4096u) __nanosleep(64);
    }
  }
  return false;
}

}  // namespace qfc
