#pragma once
// Two-shot all-reduce, 16 elements per lane, in two stages per CTA (opt-in).
//
// two_shot16_kernel runs its three phases back to back in every CTA: all of phase 1 (the
// NVLink scatter), a wait for the peers' reduce-scatter flags, all of phase 2 (reduce,
// requantize, the NVLink all-gather), a wait for the all-gather flags, all of phase 3
// (local dequantization).  Each wait exposes the slowest peer's skew and the flag round
// trip, and phase 3 moves nothing over NVLink.  Here each warp's units are split into two
// halves (stage 0 and stage 1) with their own flags, and the CTA runs
//
//   P1(s0)  release RS(s0)   P1(s1)  release RS(s1)
//   wait RS(s0)  P2(s0)  release AG(s0)   wait RS(s1)  P2(s1)  release AG(s1)
//   wait AG(s0)  P3(s0)   wait AG(s1)  P3(s1)
//
// so that every wait finds its flags already set by the time the other stage's work is
// done, and the stores of one stage drain over NVLink while the next runs.  Stage 1's
// flags are the stage-0 flag words at block index b + kStageBlockOff (the two-shot grids
// stay below that offset), published with the same per-block epoch; the protocol model
// (tests/protocol_model.py, "two_shot_staged") checks this schedule for races and
// deadlocks.  Slot layout, unit ownership and arithmetic are two_shot16_kernel's, so the
// result is bit-identical to it.  Selected with set_two_shot_stages(2) (default 1).
#include "allreduce.cuh"

namespace qfc {
namespace ar {

template <typename InT, typename OutT, int P1, int P2, int WC>
__global__ void __launch_bounds__(kWarps16 * 32, 3) two_shot16s_kernel(const __grid_constant__ ARParams p) {
  static_assert(sizeof(InT) == 2, "two_shot16s_kernel takes 16-bit inputs");
  const int rank = gridDim.y > 1 ? (int)blockIdx.y : p.rank;
  const int W = WC > 0 ? WC : p.world;
  const int b = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, wpb = blockDim.x >> 5;
  const int lpg = p.gs >> 4;
  const InT* in = static_cast<const InT*>(p.in[rank]);
  OutT* out = static_cast<OutT*>(p.out[rank]);
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
  const int64_t C = p.chunk;
  const int64_t units = C / kUnit16;
  const int64_t ustride = (int64_t)gridDim.x * wpb;
  const int64_t u0 = (int64_t)b * wpb + warp;
  const int64_t my_units = (u0 < units) ? (units - 1 - u0) / ustride + 1 : 0;
  const int64_t half = (my_units + 1) / 2;  // stage 0: units [0, half), stage 1: [half, my_units)
  const int64_t lane_off = lane * kEPL;
  const int fb[2] = {b, b + kStageBlockOff};  // flag block of each stage

  // ---------------------------------------------------------------- phase 1, both stages
#pragma unroll 1
  for (int s = 0; s < 2; ++s) {
    const int64_t i_lo = s == 0 ? 0 : half, i_hi = s == 0 ? half : my_units;
    constexpr int KB = 4;
    const int64_t items = (i_hi - i_lo) * W;
    for (int64_t it = 0; it < items; it += KB) {
      Raw16 raw[KB];
#pragma unroll
      for (int k = 0; k < KB; ++k) {
        if (it + k < items) {
          int64_t i;
          int jj;
          split_item<WC>(it + k, W, i, jj);
          const int j = (rank + 1 + jj) % W;  // peers staggered, own chunk last
          raw[k] = load_raw16(in, (int64_t)j * C + (u0 + (i_lo + i) * ustride) * kUnit16 + lane_off, p.n);
        }
      }
#pragma unroll
      for (int k = 0; k < KB; ++k) {
        if (it + k < items) {
          int64_t i;
          int jj;
          split_item<WC>(it + k, W, i, jj);
          const int j = (rank + 1 + jj) % W;
          if (j == rank && !p.quantize_local) continue;
          const int64_t unit = u0 + (i_lo + i) * ustride;
          const Enc16 en = encode_raw16<P1, InT>(raw[k], lpg, p.sym, p.meta_fp32);
          char* slot = p.base[j] + p.rs_off + (int64_t)rank * p.slot1;
          store_payload16<P1>(slot, unit * kUnit16 + lane_off, en);
          if constexpr (P1 != 16) store_meta16(slot + p.pay1, unit, en, lane, p.gs_shift, p.meta_fp32);
        }
      }
    }
    __syncthreads();
    if ((int)threadIdx.x < W) st_release_sys(flag_at(p.base[threadIdx.x], PH_RS, fb[s], rank), e);
  }

  // ---------------------------------------------------------------- phase 2, both stages
#pragma unroll 1
  for (int s = 0; s < 2; ++s) {
    if (!wait_sources(p, my, PH_RS, fb[s], rank, W, e, false, &s_abort)) return;
    const int64_t i_lo = s == 0 ? 0 : half, i_hi = s == 0 ? half : my_units;
    constexpr int NW = WC > 0 ? WC : kMaxRanks;
    constexpr int SBMAX = P1 == 16 ? 2 : 4;
    constexpr int SB = NW < SBMAX ? NW : SBMAX;
    for (int64_t i0 = i_lo; i0 < i_hi; ++i0) {
      const int64_t unit = u0 + i0 * ustride;
      const int64_t loc = unit * kUnit16 + lane_off;
      float acc[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] = 0.f;
#pragma unroll
      for (int s0 = 0; s0 < NW; s0 += SB) {
        Wire16 wv[SB];
#pragma unroll
        for (int t = 0; t < SB; ++t) {
          const int src = s0 + t;
          if (src < W && !(src == rank && !p.quantize_local)) {
            const char* slot = my + p.rs_off + (int64_t)src * p.slot1;
            wv[t] = load_wire16<P1>(slot, slot + p.pay1, loc, p.gs_shift, p.meta_fp32);
          }
        }
#pragma unroll
        for (int t = 0; t < SB; ++t) {
          const int src = s0 + t;
          if (src < W) {
            float d[16];
            if (src == rank && !p.quantize_local) raw16_to_f32<InT>(load_raw16(in, (int64_t)rank * C + loc, p.n), d);
            else decode_wire16<P1, InT>(wv[t], p.meta_fp32, d);
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = __fadd_rn(acc[i], d[i]);
          }
        }
      }
      const Enc16 en = encode_f32x16<P2, InT>(acc, lpg, p.sym, p.meta_fp32);
#pragma unroll
      for (int jj = 1; jj < NW; ++jj) {
        if (jj < W) {
          const int j = (rank + jj) % W;
          char* slot = p.base[j] + p.ag_off + (int64_t)rank * p.slot2;
          store_payload16<P2>(slot, loc, en);
          if constexpr (P2 != 16) store_meta16(slot + p.pay2, unit, en, lane, p.gs_shift, p.meta_fp32);
        }
      }
      float o[16];
      decode_enc16<P2, InT>(en, o);
      store16_guard(out, (int64_t)rank * C + loc, p.n, o);
    }
    __syncthreads();
    if ((int)threadIdx.x < W && (int)threadIdx.x != rank)
      st_release_sys(flag_at(p.base[threadIdx.x], PH_AG, fb[s], rank), e);
  }

  // ---------------------------------------------------------------- phase 3, both stages
#pragma unroll 1
  for (int s = 0; s < 2; ++s) {
    if (!wait_sources(p, my, PH_AG, fb[s], rank, W, e, true, &s_abort)) return;
    if (W == 1) continue;
    const int64_t i_lo = s == 0 ? 0 : half, i_hi = s == 0 ? half : my_units;
    constexpr int KB = 4;
    const int64_t items = (i_hi - i_lo) * (W - 1);
    for (int64_t it = 0; it < items; it += KB) {
      Wire16 wv[KB];
#pragma unroll
      for (int k = 0; k < KB; ++k) {
        if (it + k < items) {
          int64_t i;
          int jj;
          split_item<(WC > 1 ? WC - 1 : 0)>(it + k, W - 1, i, jj);
          const int j = (rank + 1 + jj) % W;
          const int64_t loc = (u0 + (i_lo + i) * ustride) * kUnit16 + lane_off;
          const char* slot = my + p.ag_off + (int64_t)j * p.slot2;
          wv[k] = load_wire16<P2>(slot, slot + p.pay2, loc, p.gs_shift, p.meta_fp32);
        }
      }
#pragma unroll
      for (int k = 0; k < KB; ++k) {
        if (it + k < items) {
          int64_t i;
          int jj;
          split_item<(WC > 1 ? WC - 1 : 0)>(it + k, W - 1, i, jj);
          const int j = (rank + 1 + jj) % W;
          const int64_t loc = (u0 + (i_lo + i) * ustride) * kUnit16 + lane_off;
          float d[16];
          decode_wire16<P2, InT>(wv[k], p.meta_fp32, d);
          store16_guard(out, (int64_t)j * C + loc, p.n, d);
        }
      }
    }
  }
  if (threadIdx.x == 0) *ep = e;
}

}  // namespace ar
}  // namespace qfc
