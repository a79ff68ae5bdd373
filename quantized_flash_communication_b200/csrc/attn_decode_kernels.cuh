// Kernels of the paged split-KV decode attention (see attn_decode.cu for the design).
// Shared by the allocating entry point (attn_decode.cu) and the allocation-free one
// (attn_decode_noalloc.cu).
#pragma once

#include <atomic>

#include <cfloat>
#include <type_traits>

#include "common.cuh"
#include "smem_optin.h"

namespace qfc {
namespace decode {

constexpr int kPart = 256;     // smallest partition (tokens); the host may pick 2^k * kPart
constexpr int kMaxPart = 4096;
constexpr int kWarps = 4;
constexpr int kMaxGroup = 8;   // query heads per kv head

// Lanes per token: the head dim of a token is split over LPT lanes so that each lane keeps
// the query slices of all G heads of the GQA group and their accumulators in registers
// (G * HD / LPT of each) while a warp still covers 32 / LPT tokens per step; a token's
// scores need log2(LPT) shuffles per head.  A lane owns the 16-byte chunks
// sub, sub + LPT, sub + 2 LPT, ... of a row (sub = lane % LPT), so the LPT lanes of a token
// read consecutive 16-byte chunks of shared memory.
template <int HD, int G>
struct DecodeShape {
  static constexpr int LPT_RAW = (2 * G < 4) ? 4 : 2 * G;
  static constexpr int LPT = LPT_RAW > HD / 8 ? HD / 8 : LPT_RAW;
  static constexpr int EPL = HD / LPT;   // head-dim elements per lane (>= 8)
  static constexpr int NCH = EPL / 8;    // 16-byte chunks per lane
  static constexpr int TPW = 32 / LPT;   // tokens per warp step
  static constexpr int NCR = HD / 8;     // 16-byte chunks per row
  // rows that share a quarter-warp (8 lanes x 16 bytes = one 128-byte wavefront); chunk
  // indices are XOR-swizzled by (row % QW_ROWS) * LPT so those rows hit distinct banks
  static constexpr int QW_ROWS = LPT >= 8 ? 1 : 8 / LPT;
};

// K/V staging: kStageTok tokens per stage, kStages stages in flight (cp.async groups).
constexpr int kStageTok = 32;
constexpr int kStages = 4;
static_assert(kPart % kStageTok == 0 && kStageTok % kWarps == 0, "stage tiling");

template <int HD>
constexpr int decode_smem_bytes() { return kStages * 2 * kStageTok * HD * 2; }

template <int HD, int G>
QFC_DEV int swz_chunk(int row, int c) {
  using Sh = DecodeShape<HD, G>;
  return c ^ ((row % Sh::QW_ROWS) * Sh::LPT);
}

QFC_DEV float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Blackwell packed fp32 FMA: (a.x*b.x + c.x, a.y*b.y + c.y), round-to-nearest each.
QFC_DEV float2 ffma2(float2 a, float2 b, float2 c) {
  uint64_t ua, ub, uc, d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(ua) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(ub) : "f"(b.x), "f"(b.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(uc) : "f"(c.x), "f"(c.y));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(ua), "l"(ub), "l"(uc));
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(d));
  return r;
}

template <typename T>
QFC_DEV void unpack8(const uint4& u, float2 (&v)[4]) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    unpack_bf16x2(u.x, v[0].x, v[0].y);
    unpack_bf16x2(u.y, v[1].x, v[1].y);
    unpack_bf16x2(u.z, v[2].x, v[2].y);
    unpack_bf16x2(u.w, v[3].x, v[3].y);
  } else {
    unpack_f16x2(u.x, v[0].x, v[0].y);
    unpack_f16x2(u.y, v[1].x, v[1].y);
    unpack_f16x2(u.z, v[2].x, v[2].y);
    unpack_f16x2(u.w, v[3].x, v[3].y);
  }
}

QFC_DEV void cp_async16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(pred ? 16 : 0) : "memory");
}
QFC_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
QFC_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Pass 1.  CTA = (partition, kv head, sequence), 4 warps.  The partition's K and V rows
// stream through a kStages-deep shared-memory ring filled with 16-byte cp.async copies
// (rows past the sequence end are zero-filled), so the loads of the next stages are in
// flight while the warps compute on the current one.  Each warp takes kStageTok / kWarps
// tokens of a stage; scores and the softmax run in the log2 domain (q pre-scaled by
// scale * log2(e)); the running max is only rescaled when a score exceeds it.
// Three CTAs per SM (the ring is 64 KiB for head_dim 128) need <= 168 registers a thread.
template <int G>
constexpr int decode_min_ctas() { return G >= 8 ? 2 : 3; }

template <typename T, int HD, int G>
__global__ void __launch_bounds__(kWarps * 32, decode_min_ctas<G>())
decode_partial_kernel(const T* __restrict__ q, const T* __restrict__ kc, const T* __restrict__ vc,
                      const int* __restrict__ block_table, const int* __restrict__ seq_lens, float* __restrict__ part_o,
                      float* __restrict__ part_ml, int nq, int nkv, int page_shift, int max_pages, int n_parts,
                      int part_tok, float scale, int64_t q_stride) {
  using Sh = DecodeShape<HD, G>;
  constexpr int LPT = Sh::LPT, EPL = Sh::EPL, NCH = Sh::NCH, TPW = Sh::TPW, NCR = Sh::NCR;
  static_assert(kStageTok % (kWarps * 32 / NCR) == 0, "loader tiling");
  constexpr int TW = kStageTok / kWarps;  // tokens per warp per stage
  static_assert(TW % TPW == 0, "warp step tiling");
  constexpr int ROWB = HD * 2;
  constexpr int STAGE_B = 2 * kStageTok * ROWB;
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ float s_m[kWarps][G], s_l[kWarps][G];

  const int b = blockIdx.z, kvh = blockIdx.y, part = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sub = lane % LPT, tg = lane / LPT;
  const int L = min(seq_lens[b], max_pages << page_shift);  // never past the block table
  const int t0 = part * part_tok;
  const int t1 = min(L, t0 + part_tok);
  const int n_st = t1 > t0 ? (t1 - t0 + kStageTok - 1) / kStageTok : 0;
  const int* bt = block_table + (int64_t)b * max_pages;
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(dsm);
  // loader mapping: thread -> chunk c of rows r0, r0 + RSTEP, ... (K and V alike)
  constexpr int RSTEP = kWarps * 32 / NCR;
  constexpr int RPT = kStageTok / RSTEP;
  const int lc = tid % NCR, lr0 = tid / NCR;
  const int64_t page_stride = (int64_t)nkv * HD << page_shift;  // elements per page
  const int64_t head_off = (int64_t)kvh * HD << page_shift;
  const int page_mask = (1 << page_shift) - 1;

  auto issue = [&](int st) {
    if (st < n_st) {
      const uint32_t dst0 = sbase + (st % kStages) * STAGE_B;
#pragma unroll
      for (int j = 0; j < RPT; ++j) {
        const int r = lr0 + j * RSTEP;
        const int t = t0 + st * kStageTok + r;
        const bool ok = t < t1;
        const int64_t off = ok ? (int64_t)bt[t >> page_shift] * page_stride + head_off + (t & page_mask) * HD + lc * 8 : 0;
        const uint32_t dst = dst0 + r * ROWB + swz_chunk<HD, G>(r, lc) * 16;
        cp_async16(dst, kc + off, ok);
        cp_async16(dst + kStageTok * ROWB, vc + off, ok);
      }
    }
    cp_async_commit();  // empty groups keep the group count uniform
  };
#pragma unroll
  for (int st = 0; st < kStages - 1; ++st) issue(st);

  // this lane's chunks of the group's query rows, scaled to the log2 domain
  const float sl2 = scale * 1.4426950408889634f;
  float2 qv[G][EPL / 2];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const T* qp = q + (int64_t)b * q_stride + (int64_t)(kvh * G + g) * HD;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      float2 v[4];
      unpack8<T>(*reinterpret_cast<const uint4*>(qp + (sub + j * LPT) * 8), v);
#pragma unroll
      for (int i = 0; i < 4; ++i) qv[g][j * 4 + i] = make_float2(v[i].x * sl2, v[i].y * sl2);
    }
  }
  float m[G], l[G];
  float2 acc[G][EPL / 2];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) acc[g][i] = make_float2(0.f, 0.f);
  }

  for (int st = 0; st < n_st; ++st) {
    cp_async_wait<kStages - 2>();
    __syncthreads();  // stage st visible to all; everyone is done with stage st - 1
    issue(st + kStages - 1);
    const unsigned char* ks = dsm + (st % kStages) * STAGE_B;
    const unsigned char* vs = ks + kStageTok * ROWB;
#pragma unroll
    for (int step = 0; step < TW / TPW; ++step) {
      const int r = warp * TW + step * TPW + tg;
      const bool valid = t0 + st * kStageTok + r < t1;
      float2 kf[EPL / 2];
#pragma unroll
      for (int j = 0; j < NCH; ++j) {
        float2 v[4];
        unpack8<T>(*reinterpret_cast<const uint4*>(ks + r * ROWB + swz_chunk<HD, G>(r, sub + j * LPT) * 16), v);
#pragma unroll
        for (int i = 0; i < 4; ++i) kf[j * 4 + i] = v[i];
      }
      float s[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float2 a = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < EPL / 2; ++i) a = ffma2(qv[g][i], kf[i], a);
        s[g] = a.x + a.y;
      }
#pragma unroll
      for (int off = LPT >> 1; off > 0; off >>= 1) {
#pragma unroll
        for (int g = 0; g < G; ++g) s[g] += __shfl_xor_sync(QFC_FULL_MASK, s[g], off);
      }
      float2 vf[EPL / 2];
#pragma unroll
      for (int j = 0; j < NCH; ++j) {
        float2 v[4];
        unpack8<T>(*reinterpret_cast<const uint4*>(vs + r * ROWB + swz_chunk<HD, G>(r, sub + j * LPT) * 16), v);
#pragma unroll
        for (int i = 0; i < 4; ++i) vf[j * 4 + i] = v[i];
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float sg = valid ? s[g] : -INFINITY;
        if (sg > m[g]) {  // rare after the first tokens: rescale once per new maximum
          const float corr = ex2f(m[g] - sg);
          l[g] *= corr;
#pragma unroll
          for (int i = 0; i < EPL / 2; ++i) acc[g][i] = make_float2(acc[g][i].x * corr, acc[g][i].y * corr);
          m[g] = sg;
        }
        const float p = valid ? ex2f(sg - m[g]) : 0.f;
        l[g] += p;
        const float2 pp = make_float2(p, p);
#pragma unroll
        for (int i = 0; i < EPL / 2; ++i) acc[g][i] = ffma2(pp, vf[i], acc[g][i]);
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // the ring is reused below for the per-warp accumulators

  float* s_acc = reinterpret_cast<float*>(dsm);  // [kWarps][G][HD]
  // merge the token slots of this warp (lanes with the same sub)
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int off = LPT; off < 32; off <<= 1) {
      const float mo = __shfl_xor_sync(QFC_FULL_MASK, m[g], off);
      const float lo = __shfl_xor_sync(QFC_FULL_MASK, l[g], off);
      const float mn = fmaxf(m[g], mo);
      const float mu = (mn == -INFINITY) ? 0.f : mn;
      const float c0 = ex2f(m[g] - mu), c1 = ex2f(mo - mu);
      l[g] = l[g] * c0 + lo * c1;
#pragma unroll
      for (int i = 0; i < EPL / 2; ++i) {
        const float ax = __shfl_xor_sync(QFC_FULL_MASK, acc[g][i].x, off);
        const float ay = __shfl_xor_sync(QFC_FULL_MASK, acc[g][i].y, off);
        acc[g][i] = make_float2(acc[g][i].x * c0 + ax * c1, acc[g][i].y * c0 + ay * c1);
      }
      m[g] = mn;
    }
    if (lane == 0) {
      s_m[warp][g] = m[g];
      s_l[warp][g] = l[g];
    }
    if (tg == 0) {
#pragma unroll
      for (int j = 0; j < NCH; ++j) {
        float* dst = s_acc + (warp * G + g) * HD + (sub + j * LPT) * 8;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          dst[2 * i] = acc[g][j * 4 + i].x;
          dst[2 * i + 1] = acc[g][j * 4 + i].y;
        }
      }
    }
  }
  __syncthreads();
  // merge the warps (values are in the log2 domain)
  for (int idx = tid; idx < G * HD; idx += kWarps * 32) {
    const int g = idx / HD, d = idx % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, s_m[w][g]);
    const float Mu = (M == -INFINITY) ? 0.f : M;
    float o = 0.f, Ls = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float c = ex2f(s_m[w][g] - Mu);
      o += s_acc[(w * G + g) * HD + d] * c;
      Ls += s_l[w][g] * c;
    }
    const int qh = kvh * G + g;
    const int64_t pi = ((int64_t)b * nq + qh) * n_parts + part;
    part_o[pi * HD + d] = o;
    if (d == 0) {
      part_ml[pi * 2] = M;  // -inf for a partition with no tokens
      part_ml[pi * 2 + 1] = Ls;
    }
  }
}

// ---------------------------------------------------------------- tensor-core variant
// For GQA groups of 2..8 query heads the per-token work is a [G x HD] x [HD x tokens]
// product and a [G x tokens] x [tokens x HD] product, so it runs on the tensor cores with
// mma.sync m16n8k16 (bf16/fp16 in, fp32 accumulate): the group's query rows are the A
// operand (rows >= G are zero), K tiles are B operands read straight from shared memory by
// ldmatrix, the probabilities stay in registers (the S accumulator layout of two 8-token
// tiles is the A-operand layout of the next product) and V tiles come from ldmatrix.trans.
// Nothing is unpacked or multiplied on the CUDA cores except the softmax.  K/V stream
// through a 3-stage ring of 64-token stages; warp w owns tokens [16 w, 16 w + 16) of every
// stage.  Rows of the ring are XOR-swizzled (16-byte chunk c of row r lives at c ^ (r & 7))
// so that the eight rows an ldmatrix reads hit distinct banks.
constexpr int kMmaStageTok = 64;
constexpr int kMmaStages = 3;

template <int HD>
constexpr int decode_mma_smem_bytes() { return kMmaStages * 2 * kMmaStageTok * HD * 2; }

QFC_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
QFC_DEV void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A(16x16, rows g / g+8 in a0,a2 / a1,a3) * B(16x8) + D; the padded rows 8..15 of A are
// zero here, so a1 = a3 = 0.
template <typename T>
QFC_DEV void mma16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
  }
}

template <typename T>
QFC_DEV uint32_t pack2(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return pack_bf16x2(lo, hi);
  else return pack_f16x2(lo, hi);
}

template <typename T, int HD, int G>
__global__ void __launch_bounds__(kWarps * 32, 2)
decode_partial_mma_kernel(const T* __restrict__ q, const T* __restrict__ kc, const T* __restrict__ vc,
                          const int* __restrict__ block_table, const int* __restrict__ seq_lens,
                          float* __restrict__ part_o, float* __restrict__ part_ml, int nq, int nkv, int page_shift,
                          int max_pages, int n_parts, int part_tok, float scale, int64_t q_stride) {
  static_assert(G >= 2 && G <= 8, "mma decode: 2..8 query heads per kv head");
  constexpr int NCR = HD / 8;             // 16-byte chunks per row
  constexpr int KSTEPS = HD / 16;         // k16 steps of q . k
  constexpr int NT = HD / 8;              // n8 tiles of the output
  constexpr int ROWB = HD * 2;
  constexpr int STAGE_B = 2 * kMmaStageTok * ROWB;
  constexpr int RSTEP = kWarps * 32 / NCR;
  constexpr int RPT = kMmaStageTok / RSTEP;
  static_assert(kMmaStageTok == kWarps * 16, "one 16-token block per warp per stage");
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ float s_m[kWarps][8], s_l[kWarps][8];

  const int b = blockIdx.z, kvh = blockIdx.y, part = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;  // mma group row / thread-in-group
  const int L = min(seq_lens[b], max_pages << page_shift);  // never past the block table
  const int t0 = part * part_tok;
  const int t1 = min(L, t0 + part_tok);
  const int n_st = t1 > t0 ? (t1 - t0 + kMmaStageTok - 1) / kMmaStageTok : 0;
  const int* bt = block_table + (int64_t)b * max_pages;
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(dsm);
  const int lc = tid % NCR, lr0 = tid / NCR;
  const int64_t page_stride = (int64_t)nkv * HD << page_shift;
  const int64_t head_off = (int64_t)kvh * HD << page_shift;
  const int page_mask = (1 << page_shift) - 1;

  auto issue = [&](int st) {
    if (st < n_st) {
      const uint32_t dst0 = sbase + (st % kMmaStages) * STAGE_B;
#pragma unroll
      for (int j = 0; j < RPT; ++j) {
        const int r = lr0 + j * RSTEP;
        const int t = t0 + st * kMmaStageTok + r;
        const bool ok = t < t1;
        const int64_t off = ok ? (int64_t)bt[t >> page_shift] * page_stride + head_off + (t & page_mask) * HD + lc * 8 : 0;
        const uint32_t dst = dst0 + r * ROWB + ((lc ^ (r & 7)) << 4);
        cp_async16(dst, kc + off, ok);
        cp_async16(dst + kMmaStageTok * ROWB, vc + off, ok);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int st = 0; st < kMmaStages - 1; ++st) issue(st);

  // A fragments of the query rows: row gq (a head of the group, zero beyond G), columns
  // 16 kk + 2 tq (+1) and 16 kk + 8 + 2 tq (+1).
  uint32_t qa0[KSTEPS], qa2[KSTEPS];
  {
    const bool hv = gq < G;
    const T* qp = q + (int64_t)b * q_stride + (int64_t)(kvh * G + (hv ? gq : 0)) * HD;
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      qa0[kk] = hv ? *reinterpret_cast<const uint32_t*>(qp + 16 * kk + 2 * tq) : 0u;
      qa2[kk] = hv ? *reinterpret_cast<const uint32_t*>(qp + 16 * kk + 8 + 2 * tq) : 0u;
    }
  }
  const float sl2 = scale * 1.4426950408889634f;
  float m = -INFINITY, l = 0.f;  // of head row gq (shared by the 4 lanes of the group)
  float o[NT][4];
#pragma unroll
  for (int d = 0; d < NT; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;

  // ldmatrix lane roles: matrix mi = lane / 8, row lane % 8
  const int mi = lane >> 3, mr = lane & 7;
  for (int st = 0; st < n_st; ++st) {
    cp_async_wait<kMmaStages - 2>();
    __syncthreads();
    issue(st + kMmaStages - 1);
    const uint32_t ks = sbase + (st % kMmaStages) * STAGE_B;
    const uint32_t vs = ks + kMmaStageTok * ROWB;
    const int rb = warp * 16;  // this warp's first row in the stage
    // S = q . K^T for two 8-token tiles
    float sc[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
      const int r = rb + 8 * j + mr;
#pragma unroll
      for (int kk = 0; kk < KSTEPS; kk += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(ks + r * ROWB + (((2 * kk + mi) ^ (r & 7)) << 4), b0, b1, b2, b3);
        mma16816<T>(sc[j], qa0[kk], qa2[kk], b0, b1);
        mma16816<T>(sc[j], qa0[kk + 1], qa2[kk + 1], b2, b3);
      }
    }
    // online softmax over the 16 tokens of row gq (lane holds tokens 2tq, 2tq+1 of each tile)
    const int tb = t0 + st * kMmaStageTok + rb;
    float sv[4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = tb + 8 * j + 2 * tq + e;
        sv[2 * j + e] = t < t1 ? sc[j][e] * sl2 : -INFINITY;
      }
    }
    float mx = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
    mx = fmaxf(mx, __shfl_xor_sync(QFC_FULL_MASK, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(QFC_FULL_MASK, mx, 2));
    if (mx > m) {  // rare after the first tokens
      const float corr = ex2f(m - mx);
      l *= corr;
#pragma unroll
      for (int d = 0; d < NT; ++d) {
        o[d][0] *= corr;
        o[d][1] *= corr;
      }
      m = mx;
    }
    const float mu = (m == -INFINITY) ? 0.f : m;
    float p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      p[i] = ex2f(sv[i] - mu);
      l += p[i];
    }
    const uint32_t pa0 = pack2<T>(p[0], p[1]), pa2 = pack2<T>(p[2], p[3]);
    // O += P . V: B fragments of V tiles [16 tokens x 8 dims] by ldmatrix.trans
    const int vr = rb + (mi & 1) * 8 + mr;
#pragma unroll
    for (int d = 0; d < NT; d += 2) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(vs + vr * ROWB + (((d + (mi >> 1)) ^ (vr & 7)) << 4), b0, b1, b2, b3);
      mma16816<T>(o[d], pa0, pa2, b0, b1);
      mma16816<T>(o[d + 1], pa0, pa2, b2, b3);
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // the ring is reused below

  // row sums of the group, then per-warp results to shared memory
  l += __shfl_xor_sync(QFC_FULL_MASK, l, 1);
  l += __shfl_xor_sync(QFC_FULL_MASK, l, 2);
  float* s_acc = reinterpret_cast<float*>(dsm);  // [kWarps][G][HD]
  if (gq < G) {
    if (tq == 0) {
      s_m[warp][gq] = m;
      s_l[warp][gq] = l;
    }
#pragma unroll
    for (int d = 0; d < NT; ++d) {
      float* dst = s_acc + (warp * G + gq) * HD + 8 * d + 2 * tq;
      dst[0] = o[d][0];
      dst[1] = o[d][1];
    }
  }
  __syncthreads();
  for (int idx = tid; idx < G * HD; idx += kWarps * 32) {
    const int g = idx / HD, dd = idx % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, s_m[w][g]);
    const float Mu = (M == -INFINITY) ? 0.f : M;
    float ov = 0.f, Ls = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float c = ex2f(s_m[w][g] - Mu);
      ov += s_acc[(w * G + g) * HD + dd] * c;
      Ls += s_l[w][g] * c;
    }
    const int64_t pi = ((int64_t)b * nq + kvh * G + g) * n_parts + part;
    part_o[pi * HD + dd] = ov;
    if (dd == 0) {
      part_ml[pi * 2] = M;
      part_ml[pi * 2 + 1] = Ls;
    }
  }
}

template <typename T, int HD, int G>
inline cudaError_t decode_mma_prepare() {
  static std::atomic<unsigned long long> done{0};
  return opt_in_smem_per_device(decode_partial_mma_kernel<T, HD, G>, decode_mma_smem_bytes<HD>(), done);
}

// Opts the partial kernel into its dynamic shared memory (once per instantiation and device).
template <typename T, int HD, int G>
inline cudaError_t decode_prepare() {
  static std::atomic<unsigned long long> done{0};
  return opt_in_smem_per_device(decode_partial_kernel<T, HD, G>, decode_smem_bytes<HD>(), done);
}

// Pass 2.  One warp per (sequence, query head): lane p reads partition p's (max, sum),
// the warp reduces them, then every lane accumulates its HD / 32 output elements over the
// partitions (one coalesced row of partials per partition).
template <typename T, int HD>
__global__ void decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                      const int* __restrict__ seq_lens, T* __restrict__ out, int nq, int n_parts,
                                      int part_tok, int total_warps) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= total_warps) return;
  const int b = gw / nq, qh = gw % nq;
  const int L = seq_lens[b];
  const int np = min(n_parts, (L + part_tok - 1) / part_tok);
  const int64_t base = ((int64_t)b * nq + qh) * n_parts;
  float M = -INFINITY;
  for (int p = lane; p < np; p += 32) M = fmaxf(M, part_ml[(base + p) * 2]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(QFC_FULL_MASK, M, off));
  const float Mu = (M == -INFINITY) ? 0.f : M;
  constexpr int EPL = HD / 32;
  float o[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) o[i] = 0.f;
  float Ls = 0.f;
  for (int p0 = 0; p0 < np; p0 += 32) {
    float myc = 0.f;
    if (p0 + lane < np) {
      const float mp = part_ml[(base + p0 + lane) * 2];
      myc = (mp == -INFINITY) ? 0.f : ex2f(mp - Mu);
      Ls += part_ml[(base + p0 + lane) * 2 + 1] * myc;
    }
    const int cnt = min(32, np - p0);
#pragma unroll 4
    for (int j = 0; j < cnt; ++j) {
      const float c = __shfl_sync(QFC_FULL_MASK, myc, j);
      const float* src = part_o + (base + p0 + j) * HD + lane * EPL;
      float v[EPL];
      if constexpr (EPL == 4) {
        const float4 x = *reinterpret_cast<const float4*>(src);
        v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
      } else {
#pragma unroll
        for (int i = 0; i < EPL; ++i) v[i] = src[i];
      }
#pragma unroll
      for (int i = 0; i < EPL; ++i) o[i] = fmaf(v[i], c, o[i]);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) Ls += __shfl_xor_sync(QFC_FULL_MASK, Ls, off);
  const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
  T* op = out + ((int64_t)b * nq + qh) * HD + lane * EPL;
#pragma unroll
  for (int i = 0; i < EPL; ++i) op[i] = from_f32<T>(o[i] * inv);
}

// Both passes on stream st: the tensor-core partial kernel for GQA groups of 2..8 heads,
// the CUDA-core one for multi-head attention (G = 1), then the merge.  Sequence b's query
// heads start at q + b * q_stride (nq * HD for a packed q; a row of the fused qkv
// activation is read in place).
template <typename T, int HD, int G>
inline cudaError_t decode_launch(const T* q, const T* kc, const T* vc, const int* bt, const int* sl, T* out,
                                 float* part_o, float* part_ml, int B, int nq, int nkv, int page_shift, int max_pages,
                                 int n_parts, int part_tok, float scale, cudaStream_t st, int64_t q_stride) {
  const dim3 grid(n_parts, nkv, B);
  cudaError_t err;
  if constexpr (G >= 2) {
    if ((err = decode_mma_prepare<T, HD, G>()) != cudaSuccess) return err;
    decode_partial_mma_kernel<T, HD, G><<<grid, kWarps * 32, decode_mma_smem_bytes<HD>(), st>>>(
        q, kc, vc, bt, sl, part_o, part_ml, nq, nkv, page_shift, max_pages, n_parts, part_tok, scale, q_stride);
  } else {
    if ((err = decode_prepare<T, HD, G>()) != cudaSuccess) return err;
    decode_partial_kernel<T, HD, G><<<grid, kWarps * 32, decode_smem_bytes<HD>(), st>>>(
        q, kc, vc, bt, sl, part_o, part_ml, nq, nkv, page_shift, max_pages, n_parts, part_tok, scale, q_stride);
  }
  if ((err = cudaGetLastError()) != cudaSuccess) return err;
  const int warps = B * nq;
  decode_combine_kernel<T, HD><<<(warps * 32 + 255) / 256, 256, 0, st>>>(part_o, part_ml, sl, out, nq, n_parts,
                                                                           part_tok, warps);
  return cudaGetLastError();
}

// Partition length chosen on the host: the longest power-of-two multiple of kPart that
// still gives the partial kernel at least four waves of three CTAs per SM (longer
// partitions amortise the pipeline fill and the per-CTA merge).
inline int decode_part_tokens(int B, int nkv, int max_ctx, int sms) {
  int part = kPart;
  while (part < kMaxPart) {
    const long long ctas = (long long)B * nkv * ((max_ctx + 2 * part - 1) / (2 * part));
    if (ctas < 12LL * sms) break;
    part *= 2;
  }
  return part;
}

inline int ilog2_exact(int v) {
  int s = 0;
  while ((1 << s) < v) ++s;
  return (1 << s) == v ? s : -1;
}

}  // namespace decode
}  // namespace qfc
