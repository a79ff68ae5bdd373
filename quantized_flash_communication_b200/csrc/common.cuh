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

#include <type_traits>

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
// Round half away from zero, exactly, without the libm routine: for any finite v,
// trunc(|v| + 0.49999997f) == floor(|v| + 0.5).  0.49999997f is the largest float below
// 0.5.  Proof sketch: if frac(|v|) >= 0.5 the true sum is >= k + 0.99999997 and rounds to
// >= k + 1 in the result's binade (half an ulp there is >= 2^-25); if frac(|v|) < 0.5 the
// true sum is <= k + 1 - ulp(v) - 2^-25, which rounds to below k + 1.  (With 0.5 itself,
// v = 0.49999997 would round up to 1.)  Tested exhaustively on ties and their
// neighbours against the oracle.
QFC_DEV float rhaz(float v) { return copysignf(truncf(fabsf(v) + 0.49999997f), v); }

constexpr float kMagic = 8388608.f;  // 2^23: (2^23 + c) holds the integer c in its low mantissa bits

template <int BITS, bool SYM>
struct QMath {
  static constexpr float QMAX = float((1 << BITS) - 1);
  // Group statistics -> (scale, 1/scale, zero point), all fp32, IEEE-rounded.
  static QFC_DEV void params(float mn, float mx, float& s, float& inv, float& z) {
    if (SYM) {
      const float a = fmaxf(-mn, mx);  // == max |x| over the group
      s = __fdiv_rn(a, QMAX * 0.5f);
      if (s < 1e-9f) s = 1.f;
      inv = __frcp_rn(s);
      z = (QMAX + 1.f) * 0.5f;
    } else {
      s = __fdiv_rn(mx - mn, QMAX);
      if (s < 1e-9f) s = 1.f;
      inv = __frcp_rn(s);
      z = fminf(fmaxf(rhaz(-mn * inv), 0.f), QMAX);
    }
  }
  // The code of x as the bit pattern of the float 2^23 + code (code in the low byte).
  // rhaz(x * inv) + (2^23 + z) is exact while the code is in range; the clamp to
  // [0, QMAX] then runs on the bit pattern as a signed integer: any result below 2^23
  // (a negative code, or a negative float) sorts below 0x4B000000, any result above
  // 2^23 + QMAX sorts above 0x4B000000 + QMAX, since positive floats order like their
  // bits.  Identical to clamp(rhaz(x * inv) + z, 0, QMAX) + 2^23 for every non-NaN x.
  static QFC_DEV uint32_t codebits(float x, float inv, float z) {
    const int b = __float_as_int(rhaz(x * inv) + (z + kMagic));
    return (uint32_t)min(max(b, 0x4b000000), 0x4b000000 + (int)QMAX);
  }
  static QFC_DEV uint32_t code(float x, float inv, float z) { return codebits(x, inv, z) & 0xffu; }
};

// Dequantize one code: (c - z) * s.  Both subtractions below are exact (integers < 2^24),
// so this equals the oracle's (float(c) - z) * s; __fmul_rn keeps the product from being
// fused into a following add.
QFC_DEV float dq(uint32_t c, float z, float s) {
  return __fmul_rn(__uint_as_float(0x4b000000u | c) - (kMagic + z), s);
}
// Same, with zb = 2^23 + z precomputed and the code already in magic-float form.
QFC_DEV float dq_bits(uint32_t cbits, float zb, float s) { return __fmul_rn(__uint_as_float(cbits) - zb, s); }

// Byte i of w as the magic float bits 0x4B0000cc.
template <int I>
QFC_DEV uint32_t byte_magic(uint32_t w) {
  return __byte_perm(w, 0x4b000000u, 0x7440 | I);
}

// 8 byte codes <-> uint2 (element order)
QFC_DEV uint2 codes8_to_u2(const uint32_t (&c)[8]) {
  return make_uint2(c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24),
                    c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24));
}
// From magic-float code bits (code in byte 0 of each word).
QFC_DEV uint2 codebits8_to_u2(const uint32_t (&m)[8]) {
  const uint32_t a = __byte_perm(m[0], m[1], 0x0040), b = __byte_perm(m[2], m[3], 0x0040);
  const uint32_t c = __byte_perm(m[4], m[5], 0x0040), d = __byte_perm(m[6], m[7], 0x0040);
  return make_uint2(__byte_perm(a, b, 0x5410), __byte_perm(c, d, 0x5410));
}
QFC_DEV void u2_to_codes8(uint2 u, uint32_t (&c)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    c[i] = (u.x >> (8 * i)) & 0xffu;
    c[4 + i] = (u.y >> (8 * i)) & 0xffu;
  }
}
// uint2 of byte codes -> 8 dequantized values.
QFC_DEV void dq_u2(uint2 u, float z, float s, float (&d)[8]) {
  const float zb = kMagic + z;
  d[0] = dq_bits(byte_magic<0>(u.x), zb, s);
  d[1] = dq_bits(byte_magic<1>(u.x), zb, s);
  d[2] = dq_bits(byte_magic<2>(u.x), zb, s);
  d[3] = dq_bits(byte_magic<3>(u.x), zb, s);
  d[4] = dq_bits(byte_magic<0>(u.y), zb, s);
  d[5] = dq_bits(byte_magic<1>(u.y), zb, s);
  d[6] = dq_bits(byte_magic<2>(u.y), zb, s);
  d[7] = dq_bits(byte_magic<3>(u.y), zb, s);
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
// INT4 word -> uint2 of byte codes in element order.
QFC_DEV uint2 int4_to_u2(uint32_t w) {
  const uint32_t a = w & 0x0f0f0f0fu, b = (w >> 4) & 0x0f0f0f0fu;
  return make_uint2(__byte_perm(a, b, 0x6420), __byte_perm(a, b, 0x7531));
}
// 8 magic-float code words (codes <= 15) -> INT4 word.
QFC_DEV uint32_t codebits8_to_int4(const uint32_t (&m)[8]) {
  const uint2 u = codebits8_to_u2(m);
  return pack_nibbles(u.x, u.y);
}

// ------------------------------------------------------------------------------------
// Raw 8-element vectors and group statistics
// ------------------------------------------------------------------------------------
// Raw 8 elements: one 16-byte vector for 16-bit types, two for fp32.  Elements at or
// beyond n read as zero.
template <typename T>
struct Raw8 {
  uint4 a, b;
};
template <typename T>
QFC_DEV Raw8<T> load_raw8(const T* base, int64_t idx, int64_t n) {
  Raw8<T> r;
  r.a = make_uint4(0, 0, 0, 0);
  r.b = make_uint4(0, 0, 0, 0);
  if (idx + 8 <= n) {
    r.a = *reinterpret_cast<const uint4*>(base + idx);
    if constexpr (sizeof(T) == 4) r.b = *(reinterpret_cast<const uint4*>(base + idx) + 1);
  } else {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = (idx + i < n) ? to_f32(base[idx + i]) : 0.f;
    if constexpr (sizeof(T) == 4) {
      r.a = make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]), __float_as_uint(v[3]));
      r.b = make_uint4(__float_as_uint(v[4]), __float_as_uint(v[5]), __float_as_uint(v[6]), __float_as_uint(v[7]));
    } else {
      r.a = Vec8IO<T>::pack(v);
    }
  }
  return r;
}
template <typename T>
QFC_DEV void raw8_to_f32(const Raw8<T>& r, float (&v)[8]) {
  if constexpr (sizeof(T) == 4) {
    v[0] = __uint_as_float(r.a.x); v[1] = __uint_as_float(r.a.y);
    v[2] = __uint_as_float(r.a.z); v[3] = __uint_as_float(r.a.w);
    v[4] = __uint_as_float(r.b.x); v[5] = __uint_as_float(r.b.y);
    v[6] = __uint_as_float(r.b.z); v[7] = __uint_as_float(r.b.w);
  } else {
    const uint32_t w[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (std::is_same<T, __nv_bfloat16>::value) unpack_bf16x2(w[i], v[2 * i], v[2 * i + 1]);
      else unpack_f16x2(w[i], v[2 * i], v[2 * i + 1]);
    }
  }
}

// Min and max of a group spread over lpg consecutive lanes (8 fp32 values per lane).
QFC_DEV void group_minmax_f32(const float (&v)[8], int lpg, float& mn, float& mx) {
  mn = fminf(fminf(fminf(v[0], v[1]), fminf(v[2], v[3])), fminf(fminf(v[4], v[5]), fminf(v[6], v[7])));
  mx = fmaxf(fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3])), fmaxf(fmaxf(v[4], v[5]), fmaxf(v[6], v[7])));
  for (int off = lpg >> 1; off > 0; off >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(QFC_FULL_MASK, mn, off));
    mx = fmaxf(mx, __shfl_xor_sync(QFC_FULL_MASK, mx, off));
  }
}

// Same for 16-bit inputs, on the packed values: the pair (-min, max) travels as one
// bf16x2 / half2 word, so each reduction level is one shuffle and one packed max.
// Negation and min / max are exact, so the result equals the fp32 computation.
template <typename T>
QFC_DEV void group_minmax16(const uint4& r, int lpg, float& mn, float& mx) {
  using T2 = typename std::conditional<std::is_same<T, __nv_bfloat16>::value, __nv_bfloat162, __half2>::type;
  auto as2 = [](uint32_t u) { return *reinterpret_cast<T2*>(&u); };
  auto bits = [](T2 x) { return *reinterpret_cast<uint32_t*>(&x); };
  const T2 hi = __hmax2(__hmax2(as2(r.x), as2(r.y)), __hmax2(as2(r.z), as2(r.w)));
  const T2 lo = __hmin2(__hmin2(as2(r.x), as2(r.y)), __hmin2(as2(r.z), as2(r.w)));
  const uint32_t nlo = bits(lo) ^ 0x80008000u;              // (-min_even, -min_odd)
  const uint32_t q1 = __byte_perm(nlo, bits(hi), 0x7610);   // (-min_even, max_odd)
  const uint32_t q2 = __byte_perm(nlo, bits(hi), 0x5432);   // (-min_odd,  max_even)
  uint32_t p = bits(__hmax2(as2(q1), as2(q2)));             // (-min, max)
  for (int off = lpg >> 1; off > 0; off >>= 1)
    p = bits(__hmax2(as2(p), as2(__shfl_xor_sync(QFC_FULL_MASK, p, off))));
  float a, b;
  if constexpr (std::is_same<T, __nv_bfloat16>::value) unpack_bf16x2(p, a, b);
  else unpack_f16x2(p, a, b);
  mn = -a;
  mx = b;
}

// ------------------------------------------------------------------------------------
// 16 elements per lane (a 512-element warp unit): vector I/O and group statistics
// ------------------------------------------------------------------------------------
constexpr int kEPL = 16;
constexpr int kUnit16 = 32 * kEPL;  // elements per warp unit

// 16 consecutive 16-bit elements as two 16-byte vectors; elements at or beyond n read 0.
struct Raw16 {
  uint4 a, b;
};
template <typename T>
QFC_DEV Raw16 load_raw16(const T* base, int64_t idx, int64_t n) {
  Raw16 r;
  if (idx + kEPL <= n) {
    const uint4* p = reinterpret_cast<const uint4*>(base + idx);
    r.a = p[0];
    r.b = p[1];
  } else {
    const uint16_t* h = reinterpret_cast<const uint16_t*>(base);
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t lo = (idx + 2 * i < n) ? h[idx + 2 * i] : 0u;
      const uint32_t hi = (idx + 2 * i + 1 < n) ? h[idx + 2 * i + 1] : 0u;
      w[i] = lo | (hi << 16);
    }
    r.a = make_uint4(w[0], w[1], w[2], w[3]);
    r.b = make_uint4(w[4], w[5], w[6], w[7]);
  }
  return r;
}
template <typename T>
QFC_DEV void raw16_to_f32(const Raw16& r, float (&v)[16]) {
  const uint32_t w[8] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) unpack_bf16x2(w[i], v[2 * i], v[2 * i + 1]);
    else unpack_f16x2(w[i], v[2 * i], v[2 * i + 1]);
  }
}
template <typename T>
QFC_DEV void store16_guard(T* base, int64_t idx, int64_t n, const float (&v)[16]) {
  if (idx + kEPL <= n) {
    uint4* d = reinterpret_cast<uint4*>(base + idx);
    const float(&lo)[8] = *reinterpret_cast<const float(*)[8]>(&v[0]);
    const float(&hi)[8] = *reinterpret_cast<const float(*)[8]>(&v[8]);
    d[0] = Vec8IO<T>::pack(lo);
    d[1] = Vec8IO<T>::pack(hi);
  } else {
#pragma unroll
    for (int i = 0; i < kEPL; ++i)
      if (idx + i < n) base[idx + i] = from_f32<T>(v[i]);
  }
}

// Group (min, max) of 16-bit inputs: the lane's 16 values reduce as packed pairs, then
// the (-min, max) pair crosses lpg lanes as one word per shuffle level.  Exact.
template <typename T>
QFC_DEV void group_minmax16x16(const Raw16& r, int lpg, float& mn, float& mx) {
  using T2 = typename std::conditional<std::is_same<T, __nv_bfloat16>::value, __nv_bfloat162, __half2>::type;
  auto as2 = [](uint32_t u) { return *reinterpret_cast<T2*>(&u); };
  auto bits = [](T2 x) { return *reinterpret_cast<uint32_t*>(&x); };
  const T2 hi = __hmax2(__hmax2(__hmax2(as2(r.a.x), as2(r.a.y)), __hmax2(as2(r.a.z), as2(r.a.w))),
                        __hmax2(__hmax2(as2(r.b.x), as2(r.b.y)), __hmax2(as2(r.b.z), as2(r.b.w))));
  const T2 lo = __hmin2(__hmin2(__hmin2(as2(r.a.x), as2(r.a.y)), __hmin2(as2(r.a.z), as2(r.a.w))),
                        __hmin2(__hmin2(as2(r.b.x), as2(r.b.y)), __hmin2(as2(r.b.z), as2(r.b.w))));
  const uint32_t nlo = bits(lo) ^ 0x80008000u;             // (-min_even, -min_odd)
  const uint32_t q1 = __byte_perm(nlo, bits(hi), 0x7610);  // (-min_even, max_odd)
  const uint32_t q2 = __byte_perm(nlo, bits(hi), 0x5432);  // (-min_odd,  max_even)
  uint32_t p = bits(__hmax2(as2(q1), as2(q2)));            // (-min, max)
  for (int off = lpg >> 1; off > 0; off >>= 1) p = bits(__hmax2(as2(p), as2(__shfl_xor_sync(QFC_FULL_MASK, p, off))));
  float a, b;
  if constexpr (std::is_same<T, __nv_bfloat16>::value) unpack_bf16x2(p, a, b);
  else unpack_f16x2(p, a, b);
  mn = -a;
  mx = b;
}
// Same for fp32 values (the reduced sum in phase 2).
QFC_DEV void group_minmax_f32x16(const float (&v)[16], int lpg, float& mn, float& mx) {
  float a[4], b[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    a[q] = fminf(fminf(v[q], v[q + 4]), fminf(v[q + 8], v[q + 12]));
    b[q] = fmaxf(fmaxf(v[q], v[q + 4]), fmaxf(v[q + 8], v[q + 12]));
  }
  mn = fminf(fminf(a[0], a[1]), fminf(a[2], a[3]));
  mx = fmaxf(fmaxf(b[0], b[1]), fmaxf(b[2], b[3]));
  for (int off = lpg >> 1; off > 0; off >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(QFC_FULL_MASK, mn, off));
    mx = fmaxf(mx, __shfl_xor_sync(QFC_FULL_MASK, mx, off));
  }
}

// ------------------------------------------------------------------------------------
// Rotary embedding of one (x1, x2) pair (elements i and i + hd/2 of a head) with the
// position's (cos, sin): the rounding is spelled out so that the standalone RoPE kernel
// and the GEMM epilogue that fuses it give identical bits.
// ------------------------------------------------------------------------------------
QFC_DEV void rope_pair(float x1, float x2, float c, float s, float& y1, float& y2) {
  y1 = __fmaf_rn(x1, c, -__fmul_rn(x2, s));
  y2 = __fmaf_rn(x2, c, __fmul_rn(x1, s));
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
