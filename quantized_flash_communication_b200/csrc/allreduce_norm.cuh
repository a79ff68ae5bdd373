#pragma once
// Sequence-parallel variant of the fused two-shot all-reduce: the reduce-scatter is
// followed by the residual add and RMSNorm on the rows each rank owns, and the all-gather
// carries the normalised activations instead of the sum.
//
// A row-parallel layer (o_proj, down_proj) produces a partial [M, H] on every rank whose
// sum S is needed only as  h <- h + S  and  x = rmsnorm(h) * w  (the residual stream and
// the next layer's input).  With rank r owning rows [r*R, (r+1)*R) (R = ceil(M/W)):
//
//   phase 1  every CTA quantizes its rows of every rank's row block and stores them into
//            the owner's reduce-scatter slot (or the row-parallel GEMM's epilogue did);
//   phase 2  the owner dequant-sums the W contributions of each own row in fp32,
//            h_row = bf16(bf16(sum) + h_row) (the residual shard, updated in place),
//            x_row = bf16(bf16(h_row * rsqrt(mean(h_row^2) + eps)) * w) (rounding as the
//            RMSNorm kernel and Hugging Face's module), quantizes x_row, pushes it into
//            every peer's all-gather slot and writes its dequantized value to its own x;
//   phase 3  after the all-gather flags, it dequantizes the other ranks' rows into x.
//
// Compared with all-reduce -> replicated residual add + RMSNorm, every rank normalises
// only M/W rows, the residual stream is never all-gathered, and the sum enters the
// residual unquantized (its all-gather quantization moves to x).  The flag / epoch /
// timeout protocol is the two-shot kernel's (allreduce.cuh): CTA b of every rank handles
// the same rows, waits only for CTA b of its peers, and every wait is bounded.
//
// A warp owns whole rows (H / 256 units of 8 elements per lane); group size 128.
#include "allreduce.cuh"

namespace qfc {

struct ARNormParams {
  ARParams p;                 // in = partial [M, H] (unfused), out = x [M, H], chunk = R * H
  void* h[kMaxRanks];         // residual shard of each rank: [R, H]
  const __nv_bfloat16* w;     // RMSNorm weight [H]
  float eps;
  int M, H, R;                // rows, hidden size, rows per rank
};

namespace ar {

// Rows of CTA b, warp w: rr = b + G * (w + wpb * i) < R.
template <typename InT, int P1, int P2, int WC, bool FROM_GEMM>
__global__ void __launch_bounds__(512) two_shot_norm_kernel(const __grid_constant__ ARNormParams np) {
  using T = __nv_bfloat16;
  const ARParams& p = np.p;
  const int rank = gridDim.y > 1 ? (int)blockIdx.y : p.rank;
  const int W = WC > 0 ? WC : p.world;
  const int b = blockIdx.x, G = gridDim.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, wpb = blockDim.x >> 5;
  constexpr int lpg = 16;  // lanes per 128-element group
  const bool leader = (lane & (lpg - 1)) == 0;
  const int H = np.H, R = np.R, M = np.M;
  const int upr = H >> 8;  // 256-element units per row
  const InT* in = static_cast<const InT*>(p.in[rank]);
  T* x = static_cast<T*>(p.out[rank]);
  T* h = static_cast<T*>(np.h[rank]);
  char* my = p.base[rank];
  uint32_t* ep = p.epochs[rank] + ALG_TWO_SHOT * kMaxBlocks + b;
  __shared__ uint32_t s_e;
  __shared__ int s_abort;
  if (threadIdx.x == 0) {
    s_e = *ep + 1u;
    s_abort = 0;
  }
  __syncthreads();
  const uint32_t e = s_e;
  const int64_t lane_off = lane * 8;
  const int row_step = G * wpb;
  const int row0 = b + G * warp;

  // ---------------------------------------------------------------- phase 1
  if constexpr (FROM_GEMM) {
    const uint32_t eg = *p.gemm_epoch;
    if (!wait_sources(p, my, PH_GEMM, 0, rank, W, eg, false, &s_abort)) return;
  } else {
    for (int rr = row0; rr < R; rr += row_step) {
      for (int jj = 0; jj < W; ++jj) {
        const int j = (rank + 1 + jj) % W;  // peers staggered, own block last
        const int g = j * R + rr;
        if (g >= M) continue;
        char* slot = p.base[j] + p.rs_off + (int64_t)rank * p.slot1;
        for (int u0 = 0; u0 < upr; u0 += kBatch) {
          Raw8<InT> raw[kBatch];
#pragma unroll
          for (int k = 0; k < kBatch; ++k)
            if (u0 + k < upr) raw[k] = load_raw8(in, (int64_t)g * H + ((u0 + k) << 8) + lane_off, (int64_t)M * H);
#pragma unroll
          for (int k = 0; k < kBatch; ++k) {
            if (u0 + k < upr) {
              float v[8];
              const Enc8 en = encode_raw<P1, InT>(raw[k], lpg, p.sym, v);
              store8<P1, InT>(slot, slot + p.pay1, (int64_t)rr * H + ((u0 + k) << 8) + lane_off, en, leader, 7,
                              p.meta_fp32);
            }
          }
        }
      }
    }
    __syncthreads();
    if ((int)threadIdx.x < W) st_release_sys(flag_at(p.base[threadIdx.x], PH_RS, b, rank), e);
    if (!wait_sources(p, my, PH_RS, b, rank, W, e, false, &s_abort)) return;
  }

  // ---------------------------------------------------------------- phase 2
  {
    constexpr int NW = WC > 0 ? WC : kMaxRanks;
    for (int rr = row0; rr < R; rr += row_step) {
      const int g = rank * R + rr;
      if (g >= M) continue;
      T* hrow = h + (int64_t)rr * H;
      float ss = 0.f;
      // NU units per batch so that NU * W slot loads (and NU residual loads) are in flight
      constexpr int NU = (WC > 0 && kBatch / NW > 1) ? kBatch / NW : 1;
      for (int u0 = 0; u0 < upr; u0 += NU) {
        Wire8 wv[NU][NW];
        float hv[NU][8];
#pragma unroll
        for (int a = 0; a < NU; ++a) {
          if (u0 + a < upr) {
            const int64_t loc = (int64_t)rr * H + ((u0 + a) << 8) + lane_off;
#pragma unroll
            for (int s = 0; s < NW; ++s) {
              if (s < W && !(s == rank && !p.quantize_local)) {
                const char* slot = my + p.rs_off + (int64_t)s * p.slot1;
                wv[a][s] = load_wire<P1, InT>(slot, slot + p.pay1, loc, 7, p.meta_fp32);
              }
            }
            Vec8IO<T>::load(hrow + ((u0 + a) << 8) + lane_off, hv[a]);
          }
        }
#pragma unroll
        for (int a = 0; a < NU; ++a) {
          if (u0 + a < upr) {
            const int u = u0 + a;
            float acc[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
            for (int s = 0; s < NW; ++s) {
              if (s < W) {
                float d[8];
                if (s == rank && !p.quantize_local)
                  load8_guard(in, (int64_t)g * H + (u << 8) + lane_off, (int64_t)M * H, d);
                else
                  decode_wire<P1, InT>(wv[a][s], p.meta_fp32, d);
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], d[i]);
              }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              hv[a][i] = to_f32(from_f32<T>(to_f32(from_f32<T>(acc[i])) + hv[a][i]));
              ss += hv[a][i] * hv[a][i];
            }
            Vec8IO<T>::store(hrow + (u << 8) + lane_off, hv[a]);
          }
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(QFC_FULL_MASK, ss, off);
      const float rstd = rsqrtf(ss / (float)H + np.eps);
      for (int u = 0; u < upr; ++u) {
        const int64_t loc = (int64_t)rr * H + (u << 8) + lane_off;
        float hv[8], wv8[8], y[8];
        Vec8IO<T>::load(hrow + (u << 8) + lane_off, hv);
        Vec8IO<T>::load(np.w + (u << 8) + lane_off, wv8);
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = to_f32(from_f32<T>(to_f32(from_f32<T>(hv[i] * rstd)) * wv8[i]));
        const Enc8 en = encode8<P2, T>(y, lpg, p.sym);
#pragma unroll
        for (int jj = 1; jj < NW; ++jj) {
          if (jj < W) {
            const int j = (rank + jj) % W;
            char* slot = p.base[j] + p.ag_off + (int64_t)rank * p.slot2;
            store8<P2, T>(slot, slot + p.pay2, loc, en, leader, 7, p.meta_fp32);
          }
        }
        float o[8];
        decode8<P2, T>(en, p.meta_fp32, o);
        Vec8IO<T>::store(x + (int64_t)g * H + (u << 8) + lane_off, o);
      }
    }
  }
  __syncthreads();
  if ((int)threadIdx.x < W && (int)threadIdx.x != rank) st_release_sys(flag_at(p.base[threadIdx.x], PH_AG, b, rank), e);
  if (!wait_sources(p, my, PH_AG, b, rank, W, e, true, &s_abort)) return;

  // ---------------------------------------------------------------- phase 3
  for (int jj = 1; jj < W; ++jj) {
    const int j = (rank + jj) % W;
    const char* slot = my + p.ag_off + (int64_t)j * p.slot2;
    for (int rr = row0; rr < R; rr += row_step) {
      const int g = j * R + rr;
      if (g >= M) continue;
      for (int u0 = 0; u0 < upr; u0 += kBatch) {
        Wire8 wv[kBatch];
#pragma unroll
        for (int k = 0; k < kBatch; ++k)
          if (u0 + k < upr)
            wv[k] = load_wire<P2, T>(slot, slot + p.pay2, (int64_t)rr * H + ((u0 + k) << 8) + lane_off, 7, p.meta_fp32);
#pragma unroll
        for (int k = 0; k < kBatch; ++k) {
          if (u0 + k < upr) {
            float d[8];
            decode_wire<P2, T>(wv[k], p.meta_fp32, d);
            Vec8IO<T>::store(x + (int64_t)g * H + ((u0 + k) << 8) + lane_off, d);
          }
        }
      }
    }
  }
  if (threadIdx.x == 0) *ep = e;
}

// The same kernel with 16 elements per lane (512-element units; H % 512 == 0): 16-byte
// code stores, metadata as 16-byte vectors, 80 registers so that three 256-thread CTAs
// share an SM.  Bit-identical to two_shot_norm_kernel.
template <typename InT, int P1, int P2, int WC, bool FROM_GEMM>
__global__ void __launch_bounds__(kWarps16 * 32, 3) two_shot_norm16_kernel(const __grid_constant__ ARNormParams np) {
  using T = __nv_bfloat16;
  const ARParams& p = np.p;
  const int rank = gridDim.y > 1 ? (int)blockIdx.y : p.rank;
  const int W = WC > 0 ? WC : p.world;
  const int b = blockIdx.x, G = gridDim.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, wpb = blockDim.x >> 5;
  constexpr int lpg = 8;  // lanes per 128-element group
  const int H = np.H, R = np.R, M = np.M;
  const int upr = H / kUnit16;  // 512-element units per row
  const InT* in = static_cast<const InT*>(p.in[rank]);
  T* x = static_cast<T*>(p.out[rank]);
  T* h = static_cast<T*>(np.h[rank]);
  char* my = p.base[rank];
  uint32_t* ep = p.epochs[rank] + ALG_TWO_SHOT * kMaxBlocks + b;
  __shared__ uint32_t s_e;
  __shared__ int s_abort;
  if (threadIdx.x == 0) {
    s_e = *ep + 1u;
    s_abort = 0;
  }
  __syncthreads();
  const uint32_t e = s_e;
  const int64_t lane_off = lane * kEPL;
  const int row_step = G * wpb;
  const int row0 = b + G * warp;

  // ---------------------------------------------------------------- phase 1
  if constexpr (FROM_GEMM) {
    const uint32_t eg = *p.gemm_epoch;
    if (!wait_sources(p, my, PH_GEMM, 0, rank, W, eg, false, &s_abort)) return;
  } else {
    constexpr int KB = 4;
    for (int rr = row0; rr < R; rr += row_step) {
      for (int jj = 0; jj < W; ++jj) {
        const int j = (rank + 1 + jj) % W;  // peers staggered, own block last
        const int g = j * R + rr;
        if (g >= M) continue;
        char* slot = p.base[j] + p.rs_off + (int64_t)rank * p.slot1;
        for (int u0 = 0; u0 < upr; u0 += KB) {
          Raw16 raw[KB];
#pragma unroll
          for (int k = 0; k < KB; ++k)
            if (u0 + k < upr) raw[k] = load_raw16(in, (int64_t)g * H + (u0 + k) * kUnit16 + lane_off, (int64_t)M * H);
#pragma unroll
          for (int k = 0; k < KB; ++k) {
            if (u0 + k < upr) {
              const int64_t unit = (int64_t)rr * upr + u0 + k;
              const Enc16 en = encode_raw16<P1, InT>(raw[k], lpg, p.sym, p.meta_fp32);
              store_payload16<P1>(slot, unit * kUnit16 + lane_off, en);
              if constexpr (P1 != 16) store_meta16(slot + p.pay1, unit, en, lane, 7, p.meta_fp32);
            }
          }
        }
      }
    }
    __syncthreads();
    if ((int)threadIdx.x < W) st_release_sys(flag_at(p.base[threadIdx.x], PH_RS, b, rank), e);
    if (!wait_sources(p, my, PH_RS, b, rank, W, e, false, &s_abort)) return;
  }

  // ---------------------------------------------------------------- phase 2
  {
    constexpr int NW = WC > 0 ? WC : kMaxRanks;
    constexpr int SBMAX = P1 == 16 ? 2 : 4;
    constexpr int SB = NW < SBMAX ? NW : SBMAX;
    for (int rr = row0; rr < R; rr += row_step) {
      const int g = rank * R + rr;
      if (g >= M) continue;
      T* hrow = h + (int64_t)rr * H;
      float ss = 0.f;
      for (int u = 0; u < upr; ++u) {
        const int64_t loc = (int64_t)rr * H + u * kUnit16 + lane_off;
        const Raw16 hraw = load_raw16(hrow, u * kUnit16 + lane_off, (int64_t)H);
        float acc[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = 0.f;
#pragma unroll
        for (int s0 = 0; s0 < NW; s0 += SB) {
          Wire16 wv[SB];
#pragma unroll
          for (int t = 0; t < SB; ++t) {
            const int s = s0 + t;
            if (s < W && !(s == rank && !p.quantize_local)) {
              const char* slot = my + p.rs_off + (int64_t)s * p.slot1;
              wv[t] = load_wire16<P1>(slot, slot + p.pay1, loc, 7, p.meta_fp32);
            }
          }
#pragma unroll
          for (int t = 0; t < SB; ++t) {
            const int s = s0 + t;
            if (s < W) {
              float d[16];
              if (s == rank && !p.quantize_local)
                raw16_to_f32<InT>(load_raw16(in, (int64_t)g * H + u * kUnit16 + lane_off, (int64_t)M * H), d);
              else
                decode_wire16<P1, InT>(wv[t], p.meta_fp32, d);
#pragma unroll
              for (int i = 0; i < 16; ++i) acc[i] = __fadd_rn(acc[i], d[i]);
            }
          }
        }
        float hv[16];
        raw16_to_f32<T>(hraw, hv);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          hv[i] = to_f32(from_f32<T>(to_f32(from_f32<T>(acc[i])) + hv[i]));
          ss += hv[i] * hv[i];
        }
        store16_guard(hrow, u * kUnit16 + lane_off, (int64_t)H, hv);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(QFC_FULL_MASK, ss, off);
      const float rstd = rsqrtf(ss / (float)H + np.eps);
      for (int u = 0; u < upr; ++u) {
        const int64_t unit = (int64_t)rr * upr + u;
        const int64_t loc = unit * kUnit16 + lane_off;
        float hv[16], wv16[16], y[16];
        raw16_to_f32<T>(load_raw16(hrow, u * kUnit16 + lane_off, (int64_t)H), hv);
        raw16_to_f32<T>(load_raw16(np.w, u * kUnit16 + lane_off, (int64_t)H), wv16);
#pragma unroll
        for (int i = 0; i < 16; ++i) y[i] = to_f32(from_f32<T>(to_f32(from_f32<T>(hv[i] * rstd)) * wv16[i]));
        const Enc16 en = encode_f32x16<P2, T>(y, lpg, p.sym, p.meta_fp32);
#pragma unroll
        for (int jj = 1; jj < NW; ++jj) {
          if (jj < W) {
            const int j = (rank + jj) % W;
            char* slot = p.base[j] + p.ag_off + (int64_t)rank * p.slot2;
            store_payload16<P2>(slot, loc, en);
            if constexpr (P2 != 16) store_meta16(slot + p.pay2, unit, en, lane, 7, p.meta_fp32);
          }
        }
        float o[16];
        decode_enc16<P2, T>(en, o);
        store16_guard(x + (int64_t)g * H, u * kUnit16 + lane_off, (int64_t)H, o);
      }
    }
  }
  __syncthreads();
  if ((int)threadIdx.x < W && (int)threadIdx.x != rank) st_release_sys(flag_at(p.base[threadIdx.x], PH_AG, b, rank), e);
  if (!wait_sources(p, my, PH_AG, b, rank, W, e, true, &s_abort)) return;

  // ---------------------------------------------------------------- phase 3
  constexpr int KB3 = 4;
  for (int jj = 1; jj < W; ++jj) {
    const int j = (rank + jj) % W;
    const char* slot = my + p.ag_off + (int64_t)j * p.slot2;
    for (int rr = row0; rr < R; rr += row_step) {
      const int g = j * R + rr;
      if (g >= M) continue;
      for (int u0 = 0; u0 < upr; u0 += KB3) {
        Wire16 wv[KB3];
#pragma unroll
        for (int k = 0; k < KB3; ++k)
          if (u0 + k < upr)
            wv[k] = load_wire16<P2>(slot, slot + p.pay2, ((int64_t)rr * upr + u0 + k) * kUnit16 + lane_off, 7,
                                    p.meta_fp32);
#pragma unroll
        for (int k = 0; k < KB3; ++k) {
          if (u0 + k < upr) {
            float d[16];
            decode_wire16<P2, T>(wv[k], p.meta_fp32, d);
            store16_guard(x + (int64_t)g * H, (u0 + k) * kUnit16 + lane_off, (int64_t)H, d);
          }
        }
      }
    }
  }
  if (threadIdx.x == 0) *ep = e;
}

// The 16-per-lane kernel with WPR warps per row.  With one warp per row the grid has
// ceil(R / 8) CTAs: at 8 ranks and 8192 x 4096 that is 128 CTAs of 8 warps, one per SM on
// 128 of the 148 SMs, a third of the warps the SM could hold, so the kernel waits on
// memory latency.  Here the warps of a row group (WPR consecutive warps) split the row's
// 512-element units (warp q takes units q, q + WPR, ...), which multiplies the grid by
// WPR.  Phase 2 needs the whole row's sum of squares: each warp reduces its units' part,
// the WPR parts meet in shared memory behind a named barrier of the row group, and every
// warp adds them in the same order.  The residual shard and every wire byte are those of
// two_shot_norm16_kernel; x may differ from it in the last bit of rstd (the sum of squares
// is added in another order).  Selected with set_norm_warps_per_row (default 1: the
// one-warp kernel above).
template <typename InT, int P1, int P2, int WC, bool FROM_GEMM, int WPR>
__global__ void __launch_bounds__(kWarps16 * 32, 3) two_shot_norm16mw_kernel(const __grid_constant__ ARNormParams np) {
  static_assert(WPR == 2 || WPR == 4 || WPR == 8, "warps per row: 2, 4 or 8");
  using T = __nv_bfloat16;
  constexpr int RG = kWarps16 / WPR;  // row groups per CTA
  const ARParams& p = np.p;
  const int rank = gridDim.y > 1 ? (int)blockIdx.y : p.rank;
  const int W = WC > 0 ? WC : p.world;
  const int b = blockIdx.x, G = gridDim.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rg = warp / WPR, q = warp % WPR;
  constexpr int lpg = 8;  // lanes per 128-element group
  const int H = np.H, R = np.R, M = np.M;
  const int upr = H / kUnit16;  // 512-element units per row
  const InT* in = static_cast<const InT*>(p.in[rank]);
  T* x = static_cast<T*>(p.out[rank]);
  T* h = static_cast<T*>(np.h[rank]);
  char* my = p.base[rank];
  uint32_t* ep = p.epochs[rank] + ALG_TWO_SHOT * kMaxBlocks + b;
  __shared__ uint32_t s_e;
  __shared__ int s_abort;
  __shared__ float s_ss[RG][WPR];
  if (threadIdx.x == 0) {
    s_e = *ep + 1u;
    s_abort = 0;
  }
  __syncthreads();
  const uint32_t e = s_e;
  const int64_t lane_off = lane * kEPL;
  const int row_step = G * RG;
  const int row0 = b + G * rg;
  // all warps of a row group walk the same rows, so they meet at every group barrier
  auto group_sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(1 + rg), "r"(WPR * 32) : "memory"); };

  // ---------------------------------------------------------------- phase 1
  if constexpr (FROM_GEMM) {
    const uint32_t eg = *p.gemm_epoch;
    if (!wait_sources(p, my, PH_GEMM, 0, rank, W, eg, false, &s_abort)) return;
  } else {
    constexpr int KB = 4;
    for (int rr = row0; rr < R; rr += row_step) {
      for (int jj = 0; jj < W; ++jj) {
        const int j = (rank + 1 + jj) % W;  // peers staggered, own block last
        const int g = j * R + rr;
        if (g >= M) continue;
        char* slot = p.base[j] + p.rs_off + (int64_t)rank * p.slot1;
        for (int u0 = q; u0 < upr; u0 += KB * WPR) {
          Raw16 raw[KB];
#pragma unroll
          for (int k = 0; k < KB; ++k) {
            const int u = u0 + k * WPR;
            if (u < upr) raw[k] = load_raw16(in, (int64_t)g * H + u * kUnit16 + lane_off, (int64_t)M * H);
          }
#pragma unroll
          for (int k = 0; k < KB; ++k) {
            const int u = u0 + k * WPR;
            if (u < upr) {
              const int64_t unit = (int64_t)rr * upr + u;
              const Enc16 en = encode_raw16<P1, InT>(raw[k], lpg, p.sym, p.meta_fp32);
              store_payload16<P1>(slot, unit * kUnit16 + lane_off, en);
              if constexpr (P1 != 16) store_meta16(slot + p.pay1, unit, en, lane, 7, p.meta_fp32);
            }
          }
        }
      }
    }
    __syncthreads();
    if ((int)threadIdx.x < W) st_release_sys(flag_at(p.base[threadIdx.x], PH_RS, b, rank), e);
    if (!wait_sources(p, my, PH_RS, b, rank, W, e, false, &s_abort)) return;
  }

  // ---------------------------------------------------------------- phase 2
  {
    constexpr int NW = WC > 0 ? WC : kMaxRanks;
    constexpr int SBMAX = P1 == 16 ? 2 : 4;
    constexpr int SB = NW < SBMAX ? NW : SBMAX;
    for (int rr = row0; rr < R; rr += row_step) {
      const int g = rank * R + rr;
      if (g >= M) continue;
      T* hrow = h + (int64_t)rr * H;
      float ss = 0.f;
      for (int u = q; u < upr; u += WPR) {
        const int64_t loc = (int64_t)rr * H + u * kUnit16 + lane_off;
        const Raw16 hraw = load_raw16(hrow, u * kUnit16 + lane_off, (int64_t)H);
        float acc[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = 0.f;
#pragma unroll
        for (int s0 = 0; s0 < NW; s0 += SB) {
          Wire16 wv[SB];
#pragma unroll
          for (int t = 0; t < SB; ++t) {
            const int s = s0 + t;
            if (s < W && !(s == rank && !p.quantize_local)) {
              const char* slot = my + p.rs_off + (int64_t)s * p.slot1;
              wv[t] = load_wire16<P1>(slot, slot + p.pay1, loc, 7, p.meta_fp32);
            }
          }
#pragma unroll
          for (int t = 0; t < SB; ++t) {
            const int s = s0 + t;
            if (s < W) {
              float d[16];
              if (s == rank && !p.quantize_local)
                raw16_to_f32<InT>(load_raw16(in, (int64_t)g * H + u * kUnit16 + lane_off, (int64_t)M * H), d);
              else
                decode_wire16<P1, InT>(wv[t], p.meta_fp32, d);
#pragma unroll
              for (int i = 0; i < 16; ++i) acc[i] = __fadd_rn(acc[i], d[i]);
            }
          }
        }
        float hv[16];
        raw16_to_f32<T>(hraw, hv);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          hv[i] = to_f32(from_f32<T>(to_f32(from_f32<T>(acc[i])) + hv[i]));
          ss += hv[i] * hv[i];
        }
        store16_guard(hrow, u * kUnit16 + lane_off, (int64_t)H, hv);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(QFC_FULL_MASK, ss, off);
      if (lane == 0) s_ss[rg][q] = ss;
      group_sync();
      float tot = 0.f;
#pragma unroll
      for (int t = 0; t < WPR; ++t) tot += s_ss[rg][t];
      group_sync();  // every warp of the group has read s_ss before the next row writes it
      const float rstd = rsqrtf(tot / (float)H + np.eps);
      for (int u = q; u < upr; u += WPR) {
        const int64_t unit = (int64_t)rr * upr + u;
        const int64_t loc = unit * kUnit16 + lane_off;
        float hv[16], wv16[16], y[16];
        raw16_to_f32<T>(load_raw16(hrow, u * kUnit16 + lane_off, (int64_t)H), hv);
        raw16_to_f32<T>(load_raw16(np.w, u * kUnit16 + lane_off, (int64_t)H), wv16);
#pragma unroll
        for (int i = 0; i < 16; ++i) y[i] = to_f32(from_f32<T>(to_f32(from_f32<T>(hv[i] * rstd)) * wv16[i]));
        const Enc16 en = encode_f32x16<P2, T>(y, lpg, p.sym, p.meta_fp32);
#pragma unroll
        for (int jj = 1; jj < NW; ++jj) {
          if (jj < W) {
            const int j = (rank + jj) % W;
            char* slot = p.base[j] + p.ag_off + (int64_t)rank * p.slot2;
            store_payload16<P2>(slot, loc, en);
            if constexpr (P2 != 16) store_meta16(slot + p.pay2, unit, en, lane, 7, p.meta_fp32);
          }
        }
        float o[16];
        decode_enc16<P2, T>(en, o);
        store16_guard(x + (int64_t)g * H, u * kUnit16 + lane_off, (int64_t)H, o);
      }
    }
  }
  __syncthreads();
  if ((int)threadIdx.x < W && (int)threadIdx.x != rank) st_release_sys(flag_at(p.base[threadIdx.x], PH_AG, b, rank), e);
  if (!wait_sources(p, my, PH_AG, b, rank, W, e, true, &s_abort)) return;

  // ---------------------------------------------------------------- phase 3
  constexpr int KB3 = 4;
  for (int jj = 1; jj < W; ++jj) {
    const int j = (rank + jj) % W;
    const char* slot = my + p.ag_off + (int64_t)j * p.slot2;
    for (int rr = row0; rr < R; rr += row_step) {
      const int g = j * R + rr;
      if (g >= M) continue;
      for (int u0 = q; u0 < upr; u0 += KB3 * WPR) {
        Wire16 wv[KB3];
#pragma unroll
        for (int k = 0; k < KB3; ++k) {
          const int u = u0 + k * WPR;
          if (u < upr)
            wv[k] = load_wire16<P2>(slot, slot + p.pay2, ((int64_t)rr * upr + u) * kUnit16 + lane_off, 7,
                                    p.meta_fp32);
        }
#pragma unroll
        for (int k = 0; k < KB3; ++k) {
          const int u = u0 + k * WPR;
          if (u < upr) {
            float d[16];
            decode_wire16<P2, T>(wv[k], p.meta_fp32, d);
            store16_guard(x + (int64_t)g * H, u * kUnit16 + lane_off, (int64_t)H, d);
          }
        }
      }
    }
  }
  if (threadIdx.x == 0) *ep = e;
}

// Rows per rank and the slot sizes of a row-blocked two-shot call.
inline Plan make_plan_rows(int64_t M, int64_t H, int W, int bits, bool fp32) {
  Plan pl;
  phase_bits(bits, pl.p1, pl.p2);
  const int64_t R = (M + W - 1) / W;
  pl.chunk = R * H;
  pl.pay1 = align_up(payload_bytes(pl.chunk, pl.p1, 2), 256);
  pl.slot1 = pl.pay1 + align_up(meta_bytes(pl.chunk, pl.p1, 128, fp32), 256);
  pl.pay2 = align_up(payload_bytes(pl.chunk, pl.p2, 2), 256);
  pl.slot2 = pl.pay2 + align_up(meta_bytes(pl.chunk, pl.p2, 128, fp32), 256);
  pl.need_rs = (int64_t)W * pl.slot1;
  pl.need_ag = (int64_t)W * pl.slot2;
  pl.need_os = 0;
  return pl;
}

// multi: the kernel is built for several CTAs per SM and the grid may use them all (every
// CTA must be resident at once: CTA b waits for CTA b of the other ranks).
template <typename Kern>
void launch_norm(Kern kern, const ARNormParams& np, int W_emul, int dev, cudaStream_t st, bool multi = false) {
  const int sms = num_sms(dev);
  const int wpb = 8;  // 256 threads; a warp per row
  int occ = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, wpb * 32, 0);
  if (occ < 1) occ = 1;
  int64_t cap = (int64_t)occ * sms / std::max(1, W_emul);
  cap = std::min<int64_t>(cap, multi ? (int64_t)kStageBlockOff : std::min<int64_t>(sms, kStageBlockOff));
  TORCH_CHECK(cap >= 1, "all_reduce_norm: no co-resident CTA budget (emulated world too large)");
  const int64_t G = std::max<int64_t>(1, std::min<int64_t>((np.R + wpb - 1) / wpb, cap));
  dim3 grid((unsigned)G, (unsigned)std::max(1, W_emul));
  kern<<<grid, wpb * 32, 0, st>>>(np);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Warps per row of the 16-per-lane norm kernel (1: two_shot_norm16_kernel; 2, 4, 8:
// two_shot_norm16mw_kernel).  Process-wide; QFC_NORM_WARPS_PER_ROW sets the initial value.
int& norm_warps_per_row();

// rows_per_cta: rows a CTA covers in one pass (warps per CTA / warps per row).
template <typename Kern>
void launch_norm_rows(Kern kern, const ARNormParams& np, int W_emul, int dev, cudaStream_t st, int rows_per_cta) {
  const int sms = num_sms(dev);
  const int threads = kWarps16 * 32;
  int occ = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, 0);
  if (occ < 1) occ = 1;
  // every CTA must be resident at once (CTA b waits for CTA b of the other ranks)
  int64_t cap = (int64_t)occ * sms / std::max(1, W_emul);
  cap = std::min<int64_t>(cap, (int64_t)kStageBlockOff);  // the two-shot family stays below the staged flags
  TORCH_CHECK(cap >= 1, "all_reduce_norm: no co-resident CTA budget (emulated world too large)");
  const int64_t G = std::max<int64_t>(1, std::min<int64_t>((np.R + rows_per_cta - 1) / rows_per_cta, cap));
  dim3 grid((unsigned)G, (unsigned)std::max(1, W_emul));
  kern<<<grid, threads, 0, st>>>(np);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <typename InT, int P1, int P2, int WC, bool FROM_GEMM>
void launch_norm16_mw(const ARNormParams& np, int W_emul, int dev, cudaStream_t st, int wpr) {
  if (wpr == 2)
    launch_norm_rows(two_shot_norm16mw_kernel<InT, P1, P2, WC, FROM_GEMM, 2>, np, W_emul, dev, st, kWarps16 / 2);
  else if (wpr == 4)
    launch_norm_rows(two_shot_norm16mw_kernel<InT, P1, P2, WC, FROM_GEMM, 4>, np, W_emul, dev, st, kWarps16 / 4);
  else
    launch_norm_rows(two_shot_norm16mw_kernel<InT, P1, P2, WC, FROM_GEMM, 8>, np, W_emul, dev, st, kWarps16 / 8);
}

template <typename InT, int WC, bool FROM_GEMM>
void dispatch_norm_w(const ARNormParams& np, const Plan& pl, int W_emul, int dev, cudaStream_t st) {
  const int wpr = norm_warps_per_row();
  if (np.H % kUnit16 == 0 && wpr > 1) {
    if (pl.p1 == 16) launch_norm16_mw<InT, 16, 16, WC, FROM_GEMM>(np, W_emul, dev, st, wpr);
    else if (pl.p1 == 8) launch_norm16_mw<InT, 8, 8, WC, FROM_GEMM>(np, W_emul, dev, st, wpr);
    else if (pl.p2 == 8) launch_norm16_mw<InT, 4, 8, WC, FROM_GEMM>(np, W_emul, dev, st, wpr);
    else launch_norm16_mw<InT, 4, 4, WC, FROM_GEMM>(np, W_emul, dev, st, wpr);
    return;
  }
  if (np.H % kUnit16 == 0) {
    if (pl.p1 == 16) launch_norm(two_shot_norm16_kernel<InT, 16, 16, WC, FROM_GEMM>, np, W_emul, dev, st, true);
    else if (pl.p1 == 8) launch_norm(two_shot_norm16_kernel<InT, 8, 8, WC, FROM_GEMM>, np, W_emul, dev, st, true);
    else if (pl.p2 == 8) launch_norm(two_shot_norm16_kernel<InT, 4, 8, WC, FROM_GEMM>, np, W_emul, dev, st, true);
    else launch_norm(two_shot_norm16_kernel<InT, 4, 4, WC, FROM_GEMM>, np, W_emul, dev, st, true);
    return;
  }
  if (pl.p1 == 16) launch_norm(two_shot_norm_kernel<InT, 16, 16, WC, FROM_GEMM>, np, W_emul, dev, st);
  else if (pl.p1 == 8) launch_norm(two_shot_norm_kernel<InT, 8, 8, WC, FROM_GEMM>, np, W_emul, dev, st);
  else if (pl.p2 == 8) launch_norm(two_shot_norm_kernel<InT, 4, 8, WC, FROM_GEMM>, np, W_emul, dev, st);
  else launch_norm(two_shot_norm_kernel<InT, 4, 4, WC, FROM_GEMM>, np, W_emul, dev, st);
}

template <bool FROM_GEMM>
void dispatch_norm(const ARNormParams& np, const Plan& pl, int W_emul, int dev, cudaStream_t st) {
  using B = __nv_bfloat16;
  switch (np.p.world) {
    case 2: dispatch_norm_w<B, 2, FROM_GEMM>(np, pl, W_emul, dev, st); break;
    case 4: dispatch_norm_w<B, 4, FROM_GEMM>(np, pl, W_emul, dev, st); break;
    case 8: dispatch_norm_w<B, 8, FROM_GEMM>(np, pl, W_emul, dev, st); break;
    default: dispatch_norm_w<B, 0, FROM_GEMM>(np, pl, W_emul, dev, st); break;
  }
}

}  // namespace ar
}  // namespace qfc
