#pragma once
// Fused quantized all-reduce over peer memory (NVLink 5 / NVSwitch): one kernel per call.
//
// Capability of the reference's flash_all_reduce (communication.py:7-97): the two-step
// Flash-Communication all-reduce (quantize -> reduce-scatter -> dequant-sum -> requantize
// -> all-gather -> dequantize) with INT8 / INT6 (INT4 + INT8) / INT4 / 16-bit payloads,
// asymmetric or symmetric groups.  The reference runs it as ~7W+10 kernel launches, six
// NCCL collectives and two host synchronisations per call; here it is a single launch:
//
//   phase 1  every CTA quantizes its warp units of every chunk in registers and
//            stores the packed codes + per-group metadata straight into the chunk owner's
//            reduce-scatter slot (plain st.global to the peer's mapped buffer), then
//            publishes a per-(block, source) flag with a release store;
//   phase 2  the owner CTA waits for the W flags of its block, dequant-sums the W
//            contributions in fp32, requantizes, pushes the result into every peer's
//            all-gather slot and writes its own chunk of the output;
//   phase 3  after the all-gather flags, it dequantizes the other chunks into the output.
//
// CTA b of every rank handles the same unit indices, so each CTA only ever waits for
// CTA b of the other ranks: no grid-wide barrier, and the grid is capped at the number
// of co-resident CTAs so that every waited-for CTA is running.  Each wait is bounded by
// %globaltimer; on expiry the CTA records the failure in a host-mapped status word and
// returns.  A one-shot variant (every rank gathers every rank's quantized tensor and
// sums locally, one round trip, one quantization) serves small, latency-bound messages.
//
// Epochs live in device memory (one counter per algorithm and block, advanced by the
// kernel itself), so the launch is safe to capture in a CUDA graph and replay.
//
// Single-GPU emulation: with gridDim.y == W, block row y plays rank y, and every "peer"
// buffer is a separate local allocation.  All W ranks then run inside one launch, which
// lets the multi-rank protocol be exercised on one GPU.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAException.h>

#include <atomic>
#include <memory>

#include "common.cuh"
#include "workspace.h"

namespace qfc {

struct ARParams {
  const void* in[kMaxRanks];
  void* out[kMaxRanks];
  char* base[kMaxRanks];
  uint32_t* epochs[kMaxRanks];
  KernelStatus* status;
  uint32_t* gemm_epoch;  // FROM_GEMM: this rank's fused-GEMM epoch counter (device)
  int64_t n;       // elements
  int64_t chunk;   // two-shot: elements per chunk (a multiple of 512); one-shot: n rounded up to 256
  int64_t rs_off, ag_off, os_off, os_bytes;
  int64_t slot1, slot2;  // slot strides in bytes (one-shot uses slot1)
  int64_t pay1, pay2;    // payload bytes at the head of a slot; metadata follows
  uint64_t timeout_ns;
  int world, rank, gs, gs_shift, meta_fp32, sym, quantize_local;
};

namespace ar {

QFC_DEV uint32_t* flag_at(char* base, int phase, int block, int src) {
  return reinterpret_cast<uint32_t*>(base) + ((int64_t)(phase * kMaxBlocks + block) * kMaxRanks + src);
}

// One lane's 8 elements in wire form, plus its group's parameters.
struct Enc8 {
  uint4 a, b;
  float s, z;
};

// Quantize 8 values given their group's (min, max).
template <int P>
QFC_DEV Enc8 encode_stats(const float (&v)[8], float mn, float mx, bool sym) {
  Enc8 e;
  e.a = make_uint4(0, 0, 0, 0);
  e.b = make_uint4(0, 0, 0, 0);
  float inv;
  if (sym) QMath<P, true>::params(mn, mx, e.s, inv, e.z);
  else QMath<P, false>::params(mn, mx, e.s, inv, e.z);
  uint32_t m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = QMath<P, false>::codebits(v[i], inv, e.z);
  if constexpr (P == 8) {
    const uint2 u = codebits8_to_u2(m);
    e.a.x = u.x;
    e.a.y = u.y;
  } else {
    e.a.x = codebits8_to_int4(m);
  }
  return e;
}

// Wire form of 8 fp32 values (group statistics from the values themselves).
template <int P, typename WT>
QFC_DEV Enc8 encode8(const float (&v)[8], int lpg, bool sym) {
  if constexpr (P == 16) {
    Enc8 e;
    e.b = make_uint4(0, 0, 0, 0);
    e.s = 1.f;
    e.z = 0.f;
    if constexpr (sizeof(WT) == 2) {
      e.a = Vec8IO<WT>::pack(v);
    } else {
      e.a = make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]), __float_as_uint(v[3]));
      e.b = make_uint4(__float_as_uint(v[4]), __float_as_uint(v[5]), __float_as_uint(v[6]), __float_as_uint(v[7]));
    }
    return e;
  } else {
    float mn, mx;
    group_minmax_f32(v, lpg, mn, mx);
    return encode_stats<P>(v, mn, mx, sym);
  }
}

// Wire form of 8 raw input elements; 16-bit inputs reduce their group statistics on the
// packed values.  v receives the fp32 values.
template <int P, typename WT>
QFC_DEV Enc8 encode_raw(const Raw8<WT>& r, int lpg, bool sym, float (&v)[8]) {
  raw8_to_f32(r, v);
  if constexpr (P == 16) {
    Enc8 e;
    e.a = r.a;
    e.b = r.b;
    e.s = 1.f;
    e.z = 0.f;
    return e;
  } else if constexpr (sizeof(WT) == 2) {
    float mn, mx;
    group_minmax16<WT>(r.a, lpg, mn, mx);
    return encode_stats<P>(v, mn, mx, sym);
  } else {
    return encode8<P, WT>(v, lpg, sym);
  }
}

template <int P, typename WT>
QFC_DEV void store8(char* slot, char* meta, int64_t loc, const Enc8& e, bool leader, int gs_shift, int meta_fp32) {
  if constexpr (P == 16) {
    if constexpr (sizeof(WT) == 2) {
      *reinterpret_cast<uint4*>(slot + loc * 2) = e.a;
    } else {
      uint4* d = reinterpret_cast<uint4*>(slot + loc * 4);
      d[0] = e.a;
      d[1] = e.b;
    }
  } else {
    if constexpr (P == 8) *reinterpret_cast<uint2*>(slot + loc) = make_uint2(e.a.x, e.a.y);
    else *reinterpret_cast<uint32_t*>(slot + (loc >> 1)) = e.a.x;
    if (leader) {
      const int64_t g = loc >> gs_shift;
      if (meta_fp32) *reinterpret_cast<float2*>(meta + g * 8) = make_float2(e.s, e.z);
      else *reinterpret_cast<uint32_t*>(meta + g * 4) = pack_f16x2(e.s, e.z);
    }
  }
}

// Values a receiver reconstructs from an Enc8 (uses the scale as stored on the wire).
template <int P, typename WT>
QFC_DEV void decode8(const Enc8& e, int meta_fp32, float (&d)[8]) {
  if constexpr (P == 16) {
    if constexpr (sizeof(WT) == 2) {
      const uint32_t w[4] = {e.a.x, e.a.y, e.a.z, e.a.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if constexpr (std::is_same<WT, __nv_bfloat16>::value) unpack_bf16x2(w[i], d[2 * i], d[2 * i + 1]);
        else unpack_f16x2(w[i], d[2 * i], d[2 * i + 1]);
      }
    } else {
      d[0] = __uint_as_float(e.a.x); d[1] = __uint_as_float(e.a.y);
      d[2] = __uint_as_float(e.a.z); d[3] = __uint_as_float(e.a.w);
      d[4] = __uint_as_float(e.b.x); d[5] = __uint_as_float(e.b.y);
      d[6] = __uint_as_float(e.b.z); d[7] = __uint_as_float(e.b.w);
    }
  } else {
    const float ss = meta_fp32 ? e.s : __half2float(__float2half_rn(e.s));
    if constexpr (P == 8) dq_u2(make_uint2(e.a.x, e.a.y), e.z, ss, d);
    else dq_u2(int4_to_u2(e.a.x), e.z, ss, d);
  }
}

// One lane's 8 elements as they sit in a slot: payload words + the group's metadata.
struct Wire8 {
  uint4 a, b;
  float s, z;
};

// Read a lane's wire data from a slot in local memory (L2, bypassing L1: the bytes were
// written by another GPU).  Separate from decoding so that a warp can put the loads of
// all W slots in flight before it uses any of them.
template <int P, typename WT>
QFC_DEV Wire8 load_wire(const char* slot, const char* meta, int64_t loc, int gs_shift, int meta_fp32) {
  Wire8 w;
  w.b = make_uint4(0, 0, 0, 0);
  w.s = 1.f;
  w.z = 0.f;
  if constexpr (P == 16) {
    const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const WT*>(slot) + loc);
    w.a = __ldcg(p);
    if constexpr (sizeof(WT) == 4) w.b = __ldcg(p + 1);
  } else {
    const int64_t g = loc >> gs_shift;
    if (meta_fp32) {
      const float2 m = __ldcg(reinterpret_cast<const float2*>(meta + g * 8));
      w.s = m.x;
      w.z = m.y;
    } else {
      const uint32_t m = __ldcg(reinterpret_cast<const unsigned int*>(meta + g * 4));
      w.s = __uint_as_float(m);  // unpacked in decode_wire
    }
    if constexpr (P == 8) {
      const uint2 u = __ldcg(reinterpret_cast<const uint2*>(slot + loc));
      w.a = make_uint4(u.x, u.y, 0, 0);
    } else {
      w.a = make_uint4(__ldcg(reinterpret_cast<const unsigned int*>(slot + (loc >> 1))), 0, 0, 0);
    }
  }
  return w;
}

template <int P, typename WT>
QFC_DEV void decode_wire(const Wire8& w, int meta_fp32, float (&d)[8]) {
  if constexpr (P == 16) {
    Raw8<WT> r;
    r.a = w.a;
    r.b = w.b;
    raw8_to_f32<WT>(r, d);
  } else {
    float s = w.s, z = w.z;
    if (!meta_fp32) unpack_f16x2(__float_as_uint(w.s), s, z);
    if constexpr (P == 8) dq_u2(make_uint2(w.a.x, w.a.y), z, s, d);
    else dq_u2(int4_to_u2(w.a.x), z, s, d);
  }
}

// Threads 0..W-1 each wait for one source's flag; returns false (for the whole CTA)
// if any wait ran out.  skip_self: the own flag is not waited for.
QFC_DEV bool wait_sources(const ARParams& p, char* my, int phase, int b, int rank, int W, uint32_t e,
                          bool skip_self, int* s_abort) {
  if ((int)threadIdx.x < W && !(skip_self && (int)threadIdx.x == rank)) {
    uint32_t seen = 0;
    const uint64_t deadline = globaltimer_ns() + p.timeout_ns;
    if (!wait_flag_geq(flag_at(my, phase, b, threadIdx.x), e, deadline, seen)) {
      report_timeout(p.status, phase, b, threadIdx.x, e, seen);
      *s_abort = 1;
    }
  }
  __syncthreads();
  return *s_abort == 0;
}

// Independent 16-byte loads a lane keeps in flight per batch.  The kernels are bound by
// memory-level parallelism, not arithmetic: with ~80 registers only 16 warps fit on an
// SM, so each warp must overlap several loads.
constexpr int kBatch = 8;

// Item i of this warp's list -> (unit, chunk offset jj).  WC = compile-time world (0 = runtime).
template <int WC>
QFC_DEV void split_item(int64_t item, int W, int64_t& i, int& jj) {
  if constexpr (WC > 0) {
    i = item / WC;
    jj = (int)(item % WC);
  } else {
    i = item / W;
    jj = (int)(item - i * W);
  }
}

// FROM_GEMM: phase 1 was done by the row-parallel GEMM's epilogue (gemm.cu, EPI_QS*), which
// stored every tile straight into its owner's reduce-scatter slot; this kernel waits for
// the per-rank epoch flag each rank's GEMM published, then runs phases 2 and 3.
template <typename InT, typename OutT, int P1, int P2, int WC, bool FROM_GEMM = false>
__global__ void __launch_bounds__(512) two_shot_kernel(const __grid_constant__ ARParams p) {
  const int rank = gridDim.y > 1 ? (int)blockIdx.y : p.rank;
  const int W = WC > 0 ? WC : p.world;
  const int b = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, wpb = blockDim.x >> 5;
  const int lpg = p.gs >> 3;
  const bool leader = (lane & (lpg - 1)) == 0;
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
  const int64_t units = C >> 8;
  const int64_t ustride = (int64_t)gridDim.x * wpb;
  const int64_t u0 = (int64_t)b * wpb + warp;
  // Units of this warp: u0, u0 + ustride, ...  (the same set on every rank and phase)
  const int64_t my_units = (u0 < units) ? (units - 1 - u0) / ustride + 1 : 0;
  const int64_t lane_off = lane * 8;

  // Phase 1: quantize every chunk's units of this warp, push them to the chunk's owner.
  // Items (unit i, chunk jj), kBatch loads issued before the first is used.
  if constexpr (FROM_GEMM) {
    const uint32_t eg = *p.gemm_epoch;  // advanced by this rank's GEMM, which ran before
    if (!wait_sources(p, my, PH_GEMM, 0, rank, W, eg, false, &s_abort)) return;
  } else {
    const int64_t items = my_units * W;
    for (int64_t it = 0; it < items; it += kBatch) {
      Raw8<InT> raw[kBatch];
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        if (it + k < items) {
          int64_t i;
          int jj;
          split_item<WC>(it + k, W, i, jj);
          const int j = (rank + 1 + jj) % W;  // peers staggered, own chunk last
          raw[k] = load_raw8(in, (int64_t)j * C + ((u0 + i * ustride) << 8) + lane_off, p.n);
        }
      }
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        if (it + k < items) {
          int64_t i;
          int jj;
          split_item<WC>(it + k, W, i, jj);
          const int j = (rank + 1 + jj) % W;
          if (j == rank && !p.quantize_local) continue;
          const int64_t loc = ((u0 + i * ustride) << 8) + lane_off;
          float v[8];
          const Enc8 en = encode_raw<P1, InT>(raw[k], lpg, p.sym, v);
          char* slot = p.base[j] + p.rs_off + (int64_t)rank * p.slot1;
          store8<P1, InT>(slot, slot + p.pay1, loc, en, leader, p.gs_shift, p.meta_fp32);
        }
      }
    }
  }
  if constexpr (!FROM_GEMM) {
    __syncthreads();
    if ((int)threadIdx.x < W) st_release_sys(flag_at(p.base[threadIdx.x], PH_RS, b, rank), e);
    if (!wait_sources(p, my, PH_RS, b, rank, W, e, false, &s_abort)) return;
  }

  // Phase 2: reduce the own chunk, requantize, push to every peer, write own output.
  // NU units per batch so that NU * W slot loads are in flight.
  {
    constexpr int NW = WC > 0 ? WC : kMaxRanks;
    constexpr int NU = (WC > 0 && kBatch / NW > 1) ? kBatch / NW : 1;
    for (int64_t i0 = 0; i0 < my_units; i0 += NU) {
      Wire8 wv[NU][NW];
#pragma unroll
      for (int a = 0; a < NU; ++a) {
        if (i0 + a < my_units) {
          const int64_t loc = ((u0 + (i0 + a) * ustride) << 8) + lane_off;
#pragma unroll
          for (int s = 0; s < NW; ++s) {
            if (s < W && !(s == rank && !p.quantize_local)) {
              const char* slot = my + p.rs_off + (int64_t)s * p.slot1;
              wv[a][s] = load_wire<P1, InT>(slot, slot + p.pay1, loc, p.gs_shift, p.meta_fp32);
            }
          }
        }
      }
#pragma unroll
      for (int a = 0; a < NU; ++a) {
        if (i0 + a < my_units) {
          const int64_t loc = ((u0 + (i0 + a) * ustride) << 8) + lane_off;
          float acc[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
          for (int s = 0; s < NW; ++s) {
            if (s < W) {
              float d[8];
              if (s == rank && !p.quantize_local) load8_guard(in, (int64_t)rank * C + loc, p.n, d);
              else decode_wire<P1, InT>(wv[a][s], p.meta_fp32, d);
#pragma unroll
              for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], d[i]);
            }
          }
          const Enc8 en = encode8<P2, InT>(acc, lpg, p.sym);
#pragma unroll
          for (int jj = 1; jj < NW; ++jj) {
            if (jj < W) {
              const int j = (rank + jj) % W;
              char* slot = p.base[j] + p.ag_off + (int64_t)rank * p.slot2;
              store8<P2, InT>(slot, slot + p.pay2, loc, en, leader, p.gs_shift, p.meta_fp32);
            }
          }
          float o[8];
          decode8<P2, InT>(en, p.meta_fp32, o);
          store8_guard(out, (int64_t)rank * C + loc, p.n, o);
        }
      }
    }
  }
  __syncthreads();
  if ((int)threadIdx.x < W && (int)threadIdx.x != rank)
    st_release_sys(flag_at(p.base[threadIdx.x], PH_AG, b, rank), e);
  if (!wait_sources(p, my, PH_AG, b, rank, W, e, true, &s_abort)) return;

  // Phase 3: dequantize the gathered chunks of the other ranks.  Items (unit, peer).
  if (W > 1) {
    const int64_t items = my_units * (W - 1);
    for (int64_t it = 0; it < items; it += kBatch) {
      Wire8 wv[kBatch];
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        if (it + k < items) {
          int64_t i;
          int jj;
          split_item<(WC > 1 ? WC - 1 : 0)>(it + k, W - 1, i, jj);
          const int j = (rank + 1 + jj) % W;
          const int64_t loc = ((u0 + i * ustride) << 8) + lane_off;
          const char* slot = my + p.ag_off + (int64_t)j * p.slot2;
          wv[k] = load_wire<P2, InT>(slot, slot + p.pay2, loc, p.gs_shift, p.meta_fp32);
        }
      }
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        if (it + k < items) {
          int64_t i;
          int jj;
          split_item<(WC > 1 ? WC - 1 : 0)>(it + k, W - 1, i, jj);
          const int j = (rank + 1 + jj) % W;
          const int64_t loc = ((u0 + i * ustride) << 8) + lane_off;
          float d[8];
          decode_wire<P2, InT>(wv[k], p.meta_fp32, d);
          store8_guard(out, (int64_t)j * C + loc, p.n, d);
        }
      }
    }
  }
  if (threadIdx.x == 0) *ep = e;
}

template <typename InT, typename OutT, int P, int WC>
__global__ void __launch_bounds__(512) one_shot_kernel(const __grid_constant__ ARParams p) {
  const int rank = gridDim.y > 1 ? (int)blockIdx.y : p.rank;
  const int W = WC > 0 ? WC : p.world;
  const int b = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, wpb = blockDim.x >> 5;
  const int lpg = p.gs >> 3;
  const bool leader = (lane & (lpg - 1)) == 0;
  const InT* in = static_cast<const InT*>(p.in[rank]);
  OutT* out = static_cast<OutT*>(p.out[rank]);
  char* my = p.base[rank];
  uint32_t* ep = p.epochs[rank] + ALG_ONE_SHOT * kMaxBlocks + b;
  uint32_t* calls = p.epochs[rank] + ALG_ONE_SHOT * kMaxBlocks + kOneShotCallsWord;
  uint32_t* done = p.epochs[rank] + ALG_ONE_SHOT * kMaxBlocks + kOneShotDoneWord;
  __shared__ uint32_t s_e, s_par;
  __shared__ int s_abort;
  if (threadIdx.x == 0) {
    s_e = *ep + 1u;
    s_par = *calls & 1u;
    s_abort = 0;
  }
  __syncthreads();
  const uint32_t e = s_e;
  // Double-buffered: a peer may start call k+1 while this rank still reads call k's
  // slots.  The region is chosen by the parity of the rank's one-shot call count, the
  // same for every block of a call.  (A block's own epoch would not do: when the grid
  // changes between calls, a unit moves to a block whose epoch has another parity, and a
  // fast rank's call k+1 could then overwrite call k's slots while they are read.)
  const int64_t region = p.os_off + (int64_t)s_par * p.os_bytes;
  // The last CTA of this rank to finish (also after a timed-out wait) advances the call
  // count; every CTA has read it by then, and the next call is a later kernel.
  auto finish = [&]() {
    if (threadIdx.x == 0 && atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0u;
      *calls = *calls + 1u;
    }
  };
  const int64_t units = p.chunk >> 8;
  const int64_t ustride = (int64_t)gridDim.x * wpb;
  const int64_t u0 = (int64_t)b * wpb + warp;
  const int64_t my_units = (u0 < units) ? (units - 1 - u0) / ustride + 1 : 0;
  const int64_t lane_off = lane * 8;

  for (int64_t i0 = 0; i0 < my_units; i0 += kBatch) {
    Raw8<InT> raw[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k)
      if (i0 + k < my_units) raw[k] = load_raw8(in, ((u0 + (i0 + k) * ustride) << 8) + lane_off, p.n);
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      if (i0 + k < my_units) {
        const int64_t loc = ((u0 + (i0 + k) * ustride) << 8) + lane_off;
        float v[8];
        const Enc8 en = encode_raw<P, InT>(raw[k], lpg, p.sym, v);
#pragma unroll
        for (int jj = 1; jj < kMaxRanks; ++jj) {
          if (jj < W) {
            const int j = (rank + jj) % W;
            char* slot = p.base[j] + region + (int64_t)rank * p.slot1;
            store8<P, InT>(slot, slot + p.pay1, loc, en, leader, p.gs_shift, p.meta_fp32);
          }
        }
      }
    }
  }
  __syncthreads();
  if ((int)threadIdx.x < W && (int)threadIdx.x != rank)
    st_release_sys(flag_at(p.base[threadIdx.x], PH_OS, b, rank), e);
  if (!wait_sources(p, my, PH_OS, b, rank, W, e, true, &s_abort)) {
    finish();
    return;
  }

  constexpr int NW = WC > 0 ? WC : kMaxRanks;
  constexpr int NU = (WC > 0 && kBatch / NW > 1) ? kBatch / NW : 1;
  for (int64_t i0 = 0; i0 < my_units; i0 += NU) {
    Wire8 wv[NU][NW];
    Raw8<InT> own_raw[NU];
#pragma unroll
    for (int a = 0; a < NU; ++a) {
      if (i0 + a < my_units) {
        const int64_t loc = ((u0 + (i0 + a) * ustride) << 8) + lane_off;
        own_raw[a] = load_raw8(in, loc, p.n);
#pragma unroll
        for (int s = 0; s < NW; ++s) {
          if (s < W && s != rank) {
            const char* slot = my + region + (int64_t)s * p.slot1;
            wv[a][s] = load_wire<P, InT>(slot, slot + p.pay1, loc, p.gs_shift, p.meta_fp32);
          }
        }
      }
    }
#pragma unroll
    for (int a = 0; a < NU; ++a) {
      if (i0 + a < my_units) {
        const int64_t loc = ((u0 + (i0 + a) * ustride) << 8) + lane_off;
        float own[8];
        const Enc8 en_own = encode_raw<P, InT>(own_raw[a], lpg, p.sym, own);
        if (p.quantize_local) decode8<P, InT>(en_own, p.meta_fp32, own);
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
        for (int s = 0; s < NW; ++s) {
          if (s < W) {
            float d[8];
            if (s == rank) {
#pragma unroll
              for (int i = 0; i < 8; ++i) d[i] = own[i];
            } else {
              decode_wire<P, InT>(wv[a][s], p.meta_fp32, d);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], d[i]);
          }
        }
        store8_guard(out, loc, p.n, acc);
      }
    }
  }
  if (threadIdx.x == 0) *ep = e;
  finish();
}

// ---------------------------------------------------------------------------------------
// Two-shot kernel with 16 elements per lane (16-bit inputs, group sizes 16..256)
// ---------------------------------------------------------------------------------------
// The same protocol, slot layout and arithmetic as two_shot_kernel, restructured for
// throughput: a warp unit is 512 elements (16 per lane), so an INT8 lane stores its codes
// as one 16-byte vector, the per-lane address / guard / group-parameter work is spread
// over twice the elements, and the metadata of a unit's groups leaves as whole 16-byte
// vectors gathered by shuffles instead of one 4-byte store per group.  The (-min, max)
// statistics of a lane's 16 values are reduced on packed 16-bit pairs before the
// cross-lane levels.  Results are bit-identical to two_shot_kernel.
constexpr int kWarps16 = 8;         // warps per CTA: 256 threads, three CTAs per SM (80 registers)

// A lane's 16 values in wire form: payload (P = 8: one uint4 of codes; P = 4: uint2 in .a.x,
// .a.y; P = 16: the raw 16-bit values in .a, .b) and its group's metadata words
// (fp16 pair in m0, or fp32 scale / zero in m0 / m1).
struct Enc16 {
  uint4 a, b;
  uint32_t m0, m1;
  float s, z;  // the scale as used for decoding (fp16-rounded unless fp32 metadata)
};

template <int P>
QFC_DEV Enc16 encode16_stats(const float (&v)[16], float mn, float mx, bool sym, int meta_fp32) {
  Enc16 e;
  e.b = make_uint4(0, 0, 0, 0);
  float s, inv, z;
  if (sym) QMath<P, true>::params(mn, mx, s, inv, z);
  else QMath<P, false>::params(mn, mx, s, inv, z);
  uint32_t m[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) m[i] = QMath<P, false>::codebits(v[i], inv, z);
  const uint32_t(&m_lo)[8] = *reinterpret_cast<const uint32_t(*)[8]>(&m[0]);
  const uint32_t(&m_hi)[8] = *reinterpret_cast<const uint32_t(*)[8]>(&m[8]);
  if constexpr (P == 8) {
    const uint2 u0 = codebits8_to_u2(m_lo), u1 = codebits8_to_u2(m_hi);
    e.a = make_uint4(u0.x, u0.y, u1.x, u1.y);
  } else {
    e.a = make_uint4(codebits8_to_int4(m_lo), codebits8_to_int4(m_hi), 0, 0);
  }
  if (meta_fp32) {
    e.m0 = __float_as_uint(s);
    e.m1 = __float_as_uint(z);
    e.s = s;
  } else {
    e.m0 = pack_f16x2(s, z);
    e.m1 = 0;
    e.s = __half2float(__float2half_rn(s));
  }
  e.z = z;
  return e;
}

// Payload of a lane's 16 elements into a slot (codes at slot + loc * P / 8).
template <int P>
QFC_DEV void store_payload16(char* slot, int64_t loc, const Enc16& e) {
  if constexpr (P == 16) {
    uint4* d = reinterpret_cast<uint4*>(slot + loc * 2);
    d[0] = e.a;
    d[1] = e.b;
  } else if constexpr (P == 8) {
    *reinterpret_cast<uint4*>(slot + loc) = e.a;
  } else {
    *reinterpret_cast<uint2*>(slot + (loc >> 1)) = make_uint2(e.a.x, e.a.y);
  }
}

// Metadata of the unit's groups as 16-byte vectors: lane v gathers groups 4v..4v+3
// (fp16 pairs) or 2v..2v+1 (fp32 pairs) from their lanes and stores them.  gs = 256
// (two groups per unit, fp16) stores one 8-byte vector.
QFC_DEV void store_meta16(char* meta, int64_t unit, const Enc16& e, int lane, int gs_shift, int meta_fp32) {
  const int lpg = 1 << (gs_shift - 4);                 // lanes per group
  const int gpu = kUnit16 >> gs_shift;                 // groups per unit
  const int64_t g0 = unit * gpu;                       // the unit's first group
  if (!meta_fp32) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) w[j] = __shfl_sync(QFC_FULL_MASK, e.m0, ((lane * 4 + j) * lpg) & 31);
    if (gpu >= 4) {
      if (lane < (gpu >> 2)) *reinterpret_cast<uint4*>(meta + (g0 + 4 * lane) * 4) = make_uint4(w[0], w[1], w[2], w[3]);
    } else if (lane == 0) {
      *reinterpret_cast<uint2*>(meta + g0 * 4) = make_uint2(w[0], w[1]);
    }
  } else {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      w[2 * j] = __shfl_sync(QFC_FULL_MASK, e.m0, ((lane * 2 + j) * lpg) & 31);
      w[2 * j + 1] = __shfl_sync(QFC_FULL_MASK, e.m1, ((lane * 2 + j) * lpg) & 31);
    }
    if (lane < (gpu >> 1)) *reinterpret_cast<uint4*>(meta + (g0 + 2 * lane) * 8) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// A lane's 16 elements as read from a slot (local memory written by peers: L2, no L1).
struct Wire16 {
  uint4 a, b;
  uint32_t m0, m1;
};
template <int P>
QFC_DEV Wire16 load_wire16(const char* slot, const char* meta, int64_t loc, int gs_shift, int meta_fp32) {
  Wire16 w;
  w.b = make_uint4(0, 0, 0, 0);
  w.m0 = w.m1 = 0;
  if constexpr (P == 16) {
    const uint4* p = reinterpret_cast<const uint4*>(slot + loc * 2);
    w.a = __ldcg(p);
    w.b = __ldcg(p + 1);
  } else {
    const int64_t g = loc >> gs_shift;
    if (meta_fp32) {
      const uint2 m = __ldcg(reinterpret_cast<const uint2*>(meta + g * 8));
      w.m0 = m.x;
      w.m1 = m.y;
    } else {
      w.m0 = __ldcg(reinterpret_cast<const unsigned int*>(meta + g * 4));
    }
    if constexpr (P == 8) {
      w.a = __ldcg(reinterpret_cast<const uint4*>(slot + loc));
    } else {
      const uint2 u = __ldcg(reinterpret_cast<const uint2*>(slot + (loc >> 1)));
      w.a = make_uint4(u.x, u.y, 0, 0);
    }
  }
  return w;
}
template <int P, typename T>
QFC_DEV void decode_wire16(const Wire16& w, int meta_fp32, float (&d)[16]) {
  if constexpr (P == 16) {
    Raw16 r;
    r.a = w.a;
    r.b = w.b;
    raw16_to_f32<T>(r, d);
  } else {
    float s, z;
    if (meta_fp32) {
      s = __uint_as_float(w.m0);
      z = __uint_as_float(w.m1);
    } else {
      unpack_f16x2(w.m0, s, z);
    }
    float(&lo)[8] = *reinterpret_cast<float(*)[8]>(&d[0]);
    float(&hi)[8] = *reinterpret_cast<float(*)[8]>(&d[8]);
    if constexpr (P == 8) {
      dq_u2(make_uint2(w.a.x, w.a.y), z, s, lo);
      dq_u2(make_uint2(w.a.z, w.a.w), z, s, hi);
    } else {
      dq_u2(int4_to_u2(w.a.x), z, s, lo);
      dq_u2(int4_to_u2(w.a.y), z, s, hi);
    }
  }
}
// Values a receiver reconstructs from an Enc16 (the own chunk's output).
template <int P, typename T>
QFC_DEV void decode_enc16(const Enc16& e, float (&d)[16]) {
  if constexpr (P == 16) {
    Raw16 r;
    r.a = e.a;
    r.b = e.b;
    raw16_to_f32<T>(r, d);
  } else {
    float(&lo)[8] = *reinterpret_cast<float(*)[8]>(&d[0]);
    float(&hi)[8] = *reinterpret_cast<float(*)[8]>(&d[8]);
    if constexpr (P == 8) {
      dq_u2(make_uint2(e.a.x, e.a.y), e.z, e.s, lo);
      dq_u2(make_uint2(e.a.z, e.a.w), e.z, e.s, hi);
    } else {
      dq_u2(int4_to_u2(e.a.x), e.z, e.s, lo);
      dq_u2(int4_to_u2(e.a.y), e.z, e.s, hi);
    }
  }
}
// Wire form of a lane's 16 raw 16-bit inputs.
template <int P, typename T>
QFC_DEV Enc16 encode_raw16(const Raw16& r, int lpg, bool sym, int meta_fp32) {
  if constexpr (P == 16) {
    Enc16 e;
    e.a = r.a;
    e.b = r.b;
    e.m0 = e.m1 = 0;
    e.s = 1.f;
    e.z = 0.f;
    return e;
  } else {
    float mn, mx;
    group_minmax16x16<T>(r, lpg, mn, mx);
    float v[16];
    raw16_to_f32<T>(r, v);
    return encode16_stats<P>(v, mn, mx, sym, meta_fp32);
  }
}
// Wire form of 16 fp32 values (the reduced sum); P = 16 rounds to the input type T.
template <int P, typename T>
QFC_DEV Enc16 encode_f32x16(const float (&v)[16], int lpg, bool sym, int meta_fp32) {
  if constexpr (P == 16) {
    Enc16 e;
    const float(&lo)[8] = *reinterpret_cast<const float(*)[8]>(&v[0]);
    const float(&hi)[8] = *reinterpret_cast<const float(*)[8]>(&v[8]);
    e.a = Vec8IO<T>::pack(lo);
    e.b = Vec8IO<T>::pack(hi);
    e.m0 = e.m1 = 0;
    e.s = 1.f;
    e.z = 0.f;
    return e;
  } else {
    float mn, mx;
    group_minmax_f32x16(v, lpg, mn, mx);
    return encode16_stats<P>(v, mn, mx, sym, meta_fp32);
  }
}

// Two-shot all-reduce, 16 elements per lane.  InT: bf16 / fp16.  Group size 16..256.
template <typename InT, typename OutT, int P1, int P2, int WC, bool FROM_GEMM = false>
__global__ void __launch_bounds__(kWarps16 * 32, 3) two_shot16_kernel(const __grid_constant__ ARParams p) {
  static_assert(sizeof(InT) == 2, "two_shot16_kernel takes 16-bit inputs");
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
  const int64_t lane_off = lane * kEPL;

  // Phase 1: quantize this warp's units of every chunk and push them to the chunk owners.
  if constexpr (FROM_GEMM) {
    const uint32_t eg = *p.gemm_epoch;  // advanced by this rank's GEMM, which ran before
    if (!wait_sources(p, my, PH_GEMM, 0, rank, W, eg, false, &s_abort)) return;
  } else {
    constexpr int KB = 4;
    const int64_t items = my_units * W;
    for (int64_t it = 0; it < items; it += KB) {
      Raw16 raw[KB];
#pragma unroll
      for (int k = 0; k < KB; ++k) {
        if (it + k < items) {
          int64_t i;
          int jj;
          split_item<WC>(it + k, W, i, jj);
          const int j = (rank + 1 + jj) % W;  // peers staggered, own chunk last
          raw[k] = load_raw16(in, (int64_t)j * C + (u0 + i * ustride) * kUnit16 + lane_off, p.n);
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
          const int64_t unit = u0 + i * ustride;
          const Enc16 en = encode_raw16<P1, InT>(raw[k], lpg, p.sym, p.meta_fp32);
          char* slot = p.base[j] + p.rs_off + (int64_t)rank * p.slot1;
          store_payload16<P1>(slot, unit * kUnit16 + lane_off, en);
          if constexpr (P1 != 16) store_meta16(slot + p.pay1, unit, en, lane, p.gs_shift, p.meta_fp32);
        }
      }
    }
    __syncthreads();
    if ((int)threadIdx.x < W) st_release_sys(flag_at(p.base[threadIdx.x], PH_RS, b, rank), e);
    if (!wait_sources(p, my, PH_RS, b, rank, W, e, false, &s_abort)) return;
  }

  // Phase 2: reduce the own chunk's units, requantize, push to every peer, write own output.
  // Sources are summed in rank order (as the oracle does), SB slot loads in flight at a
  // time, so that a warp's registers stay within the 3-CTA-per-SM budget at W = 8.
  {
    constexpr int NW = WC > 0 ? WC : kMaxRanks;
    constexpr int SBMAX = P1 == 16 ? 2 : 4;  // 16-bit payloads hold twice the registers
    constexpr int SB = NW < SBMAX ? NW : SBMAX;
    constexpr int NU = 1;
    for (int64_t i0 = 0; i0 < my_units; i0 += NU) {
      float acc[NU][16];
#pragma unroll
      for (int a = 0; a < NU; ++a)
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[a][i] = 0.f;
#pragma unroll
      for (int s0 = 0; s0 < NW; s0 += SB) {
        Wire16 wv[NU][SB];
#pragma unroll
        for (int a = 0; a < NU; ++a) {
          if (i0 + a < my_units) {
            const int64_t loc = (u0 + (i0 + a) * ustride) * kUnit16 + lane_off;
#pragma unroll
            for (int t = 0; t < SB; ++t) {
              const int s = s0 + t;
              if (s < W && !(s == rank && !p.quantize_local)) {
                const char* slot = my + p.rs_off + (int64_t)s * p.slot1;
                wv[a][t] = load_wire16<P1>(slot, slot + p.pay1, loc, p.gs_shift, p.meta_fp32);
              }
            }
          }
        }
#pragma unroll
        for (int a = 0; a < NU; ++a) {
          if (i0 + a < my_units) {
            const int64_t loc = (u0 + (i0 + a) * ustride) * kUnit16 + lane_off;
#pragma unroll
            for (int t = 0; t < SB; ++t) {
              const int s = s0 + t;
              if (s < W) {
                float d[16];
                if (s == rank && !p.quantize_local) raw16_to_f32<InT>(load_raw16(in, (int64_t)rank * C + loc, p.n), d);
                else decode_wire16<P1, InT>(wv[a][t], p.meta_fp32, d);
#pragma unroll
                for (int i = 0; i < 16; ++i) acc[a][i] = __fadd_rn(acc[a][i], d[i]);
              }
            }
          }
        }
      }
#pragma unroll
      for (int a = 0; a < NU; ++a) {
        if (i0 + a < my_units) {
          const int64_t unit = u0 + (i0 + a) * ustride;
          const int64_t loc = unit * kUnit16 + lane_off;
          const Enc16 en = encode_f32x16<P2, InT>(acc[a], lpg, p.sym, p.meta_fp32);
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
      }
    }
  }
  __syncthreads();
  if ((int)threadIdx.x < W && (int)threadIdx.x != rank) st_release_sys(flag_at(p.base[threadIdx.x], PH_AG, b, rank), e);
  if (!wait_sources(p, my, PH_AG, b, rank, W, e, true, &s_abort)) return;

  // Phase 3: dequantize the gathered chunks of the other ranks.  Items (unit, peer).
  if (W > 1) {
    constexpr int KB = 4;
    const int64_t items = my_units * (W - 1);
    for (int64_t it = 0; it < items; it += KB) {
      Wire16 wv[KB];
#pragma unroll
      for (int k = 0; k < KB; ++k) {
        if (it + k < items) {
          int64_t i;
          int jj;
          split_item<(WC > 1 ? WC - 1 : 0)>(it + k, W - 1, i, jj);
          const int j = (rank + 1 + jj) % W;
          const int64_t loc = (u0 + i * ustride) * kUnit16 + lane_off;
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
          const int64_t loc = (u0 + i * ustride) * kUnit16 + lane_off;
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

#include "allreduce_staged.cuh"

namespace qfc {
namespace ar {

// ---------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------
struct Plan {
  int p1, p2;
  int64_t chunk, slot1, slot2, pay1, pay2;
  int64_t need_rs, need_ag, need_os;
};

inline int64_t payload_bytes(int64_t elems, int P, int in_elem) {
  if (P == 16) return elems * in_elem;
  return P == 8 ? elems : elems / 2;
}
inline int64_t meta_bytes(int64_t elems, int P, int gs, bool fp32) {
  if (P == 16) return 0;
  return (elems / gs) * (fp32 ? 8 : 4);
}

inline void phase_bits(int bits, int& p1, int& p2) {
  switch (bits) {
    case 16: p1 = 16; p2 = 16; break;
    case 8: p1 = 8; p2 = 8; break;
    case 6: p1 = 4; p2 = 8; break;
    case 4: p1 = 4; p2 = 4; break;
    default: TORCH_CHECK(false, "quant_all_reduce: bits must be 16, 8, 6 or 4; got ", bits);
  }
}

inline Plan make_plan(int64_t n, int W, int bits, int gs, bool fp32, int in_elem, bool one_shot) {
  Plan pl;
  phase_bits(bits, pl.p1, pl.p2);
  if (one_shot) {
    // A single quantization step; INT6 uses its wider (INT8) half.
    const int P = (bits == 6) ? 8 : pl.p1;
    pl.p1 = pl.p2 = P;
    pl.chunk = align_up(std::max<int64_t>(n, 1), 256);
    pl.pay1 = align_up(payload_bytes(pl.chunk, P, in_elem), 256);
    pl.slot1 = pl.pay1 + align_up(meta_bytes(pl.chunk, P, gs, fp32), 256);
    pl.pay2 = pl.pay1;
    pl.slot2 = pl.slot1;
    pl.need_rs = pl.need_ag = 0;
    pl.need_os = (int64_t)W * pl.slot1;
  } else {
    // 512: a whole warp unit of the 16-element-per-lane kernel (and two of the 8-element one)
    pl.chunk = align_up((std::max<int64_t>(n, 1) + W - 1) / W, 512);
    pl.pay1 = align_up(payload_bytes(pl.chunk, pl.p1, in_elem), 256);
    pl.slot1 = pl.pay1 + align_up(meta_bytes(pl.chunk, pl.p1, gs, fp32), 256);
    pl.pay2 = align_up(payload_bytes(pl.chunk, pl.p2, in_elem), 256);
    pl.slot2 = pl.pay2 + align_up(meta_bytes(pl.chunk, pl.p2, gs, fp32), 256);
    pl.need_rs = (int64_t)W * pl.slot1;
    pl.need_ag = (int64_t)W * pl.slot2;
    pl.need_os = 0;
  }
  return pl;
}

inline int num_sms(int dev) {
  static std::atomic<int> cached[64] = {};  // threads may race to fill an entry: same value
  if (dev >= 0 && dev < 64) {
    const int c = cached[dev].load(std::memory_order_relaxed);
    if (c) return c;
  }
  int v = 0;
  cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
  if (dev >= 0 && dev < 64) cached[dev].store(v, std::memory_order_relaxed);
  return v;
}

// max_wpb: warps per CTA the kernel was compiled for (its __launch_bounds__); with
// max_wpb < 16 the kernel is built for several CTAs per SM and the grid may use them all,
// otherwise the grid stays at one CTA per SM.
template <typename Kern>
void launch_ar(Kern kern, const ARParams& prm, int64_t units, int W_emul, int dev, cudaStream_t st,
               int max_wpb = 16) {
  const int sms = num_sms(dev);
  int wpb = (int)std::min<int64_t>(max_wpb, std::max<int64_t>(2, (units + sms - 1) / sms));
  const int threads = wpb * 32;
  int occ = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, 0);
  if (occ < 1) occ = 1;
  // every CTA must be resident at once (CTA b waits for CTA b of the other ranks)
  int64_t cap = (int64_t)occ * sms / std::max(1, W_emul);
  // two-shot grids stay below kStageBlockOff (the staged kernel's second flag set); the
  // one-shot row keeps its last two words
  cap = std::min<int64_t>(cap, max_wpb < 16 ? (int64_t)kStageBlockOff : std::min<int64_t>(sms, kStageBlockOff));
  TORCH_CHECK(cap >= 1, "quant_all_reduce: no co-resident CTA budget (emulated world too large)");
  const int64_t G = std::max<int64_t>(1, std::min<int64_t>((units + wpb - 1) / wpb, cap));
  dim3 grid((unsigned)G, (unsigned)std::max(1, W_emul));
  kern<<<grid, threads, 0, st>>>(prm);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Stages of the 16-per-lane two-shot kernel: 1 (two_shot16_kernel) or 2
// (two_shot16s_kernel).  Process-wide; QFC_AR_STAGES sets the initial value.
int& two_shot_stages();

template <typename InT, typename OutT, int WC>
void dispatch_bits_w(const ARParams& prm, const Plan& pl, bool one_shot, int64_t units, int W_emul, int dev,
                     cudaStream_t st) {
  if (one_shot) {
    switch (pl.p1) {
      case 16: launch_ar(one_shot_kernel<InT, OutT, 16, WC>, prm, units, W_emul, dev, st); break;
      case 8: launch_ar(one_shot_kernel<InT, OutT, 8, WC>, prm, units, W_emul, dev, st); break;
      default: launch_ar(one_shot_kernel<InT, OutT, 4, WC>, prm, units, W_emul, dev, st); break;
    }
    return;
  }
  if constexpr (sizeof(InT) == 2) {
    if (prm.gs >= 16 && two_shot_stages() == 2) {  // 16 per lane, two stages per CTA
      const int64_t u16 = prm.chunk / kUnit16;
      if (pl.p1 == 16) launch_ar(two_shot16s_kernel<InT, OutT, 16, 16, WC>, prm, u16, W_emul, dev, st, kWarps16);
      else if (pl.p1 == 8) launch_ar(two_shot16s_kernel<InT, OutT, 8, 8, WC>, prm, u16, W_emul, dev, st, kWarps16);
      else if (pl.p2 == 8) launch_ar(two_shot16s_kernel<InT, OutT, 4, 8, WC>, prm, u16, W_emul, dev, st, kWarps16);
      else launch_ar(two_shot16s_kernel<InT, OutT, 4, 4, WC>, prm, u16, W_emul, dev, st, kWarps16);
      return;
    }
    if (prm.gs >= 16) {  // 16 elements per lane: 512-element units
      const int64_t u16 = prm.chunk / kUnit16;
      if (pl.p1 == 16) launch_ar(two_shot16_kernel<InT, OutT, 16, 16, WC>, prm, u16, W_emul, dev, st, kWarps16);
      else if (pl.p1 == 8) launch_ar(two_shot16_kernel<InT, OutT, 8, 8, WC>, prm, u16, W_emul, dev, st, kWarps16);
      else if (pl.p2 == 8) launch_ar(two_shot16_kernel<InT, OutT, 4, 8, WC>, prm, u16, W_emul, dev, st, kWarps16);
      else launch_ar(two_shot16_kernel<InT, OutT, 4, 4, WC>, prm, u16, W_emul, dev, st, kWarps16);
      return;
    }
  }
  if (pl.p1 == 16) launch_ar(two_shot_kernel<InT, OutT, 16, 16, WC>, prm, units, W_emul, dev, st);
  else if (pl.p1 == 8) launch_ar(two_shot_kernel<InT, OutT, 8, 8, WC>, prm, units, W_emul, dev, st);
  else if (pl.p2 == 8) launch_ar(two_shot_kernel<InT, OutT, 4, 8, WC>, prm, units, W_emul, dev, st);
  else launch_ar(two_shot_kernel<InT, OutT, 4, 4, WC>, prm, units, W_emul, dev, st);
}

template <typename InT, typename OutT, int WC>
void dispatch_gemm_reduce_w(const ARParams& prm, const Plan& pl, int64_t units, int dev, cudaStream_t st) {
  (void)units;
  const int64_t u16 = prm.chunk / kUnit16;
  if (pl.p1 == 16) launch_ar(two_shot16_kernel<InT, OutT, 16, 16, WC, true>, prm, u16, 1, dev, st, kWarps16);
  else if (pl.p1 == 8) launch_ar(two_shot16_kernel<InT, OutT, 8, 8, WC, true>, prm, u16, 1, dev, st, kWarps16);
  else if (pl.p2 == 8) launch_ar(two_shot16_kernel<InT, OutT, 4, 8, WC, true>, prm, u16, 1, dev, st, kWarps16);
  else launch_ar(two_shot16_kernel<InT, OutT, 4, 4, WC, true>, prm, u16, 1, dev, st, kWarps16);
}

// Phases 2-3 after a fused quantize-and-scatter GEMM.
template <typename InT, typename OutT>
void dispatch_gemm_reduce(const ARParams& prm, const Plan& pl, int64_t units, int dev, cudaStream_t st) {
  switch (prm.world) {
    case 2: dispatch_gemm_reduce_w<InT, OutT, 2>(prm, pl, units, dev, st); break;
    case 4: dispatch_gemm_reduce_w<InT, OutT, 4>(prm, pl, units, dev, st); break;
    case 8: dispatch_gemm_reduce_w<InT, OutT, 8>(prm, pl, units, dev, st); break;
    default: dispatch_gemm_reduce_w<InT, OutT, 0>(prm, pl, units, dev, st); break;
  }
}

// World sizes 2, 4 and 8 get specialised kernels (static indices, batched reduce);
// any other size runs the generic one.
template <typename InT, typename OutT>
void dispatch_bits(const ARParams& prm, const Plan& pl, bool one_shot, int64_t units, int W_emul, int dev,
                   cudaStream_t st) {
  switch (prm.world) {
    case 2: dispatch_bits_w<InT, OutT, 2>(prm, pl, one_shot, units, W_emul, dev, st); break;
    case 4: dispatch_bits_w<InT, OutT, 4>(prm, pl, one_shot, units, W_emul, dev, st); break;
    case 8: dispatch_bits_w<InT, OutT, 8>(prm, pl, one_shot, units, W_emul, dev, st); break;
    default: dispatch_bits_w<InT, OutT, 0>(prm, pl, one_shot, units, W_emul, dev, st); break;
  }
}

}  // namespace ar
}  // namespace qfc
