// Persistent tcgen05 / TMEM GEMM for sm_100a:  D[M, N] = A[M, K] * B[N, K]^T  (bf16 in,
// fp32 accumulate), the layout of nn.Linear (activations x weights^T).
//
// Replaces the cuBLAS GEMMs behind the reference's nn.Linear layers (model.py:32-35 and
// the HF attention projections).  One CTA per SM, 6 warps:
//   warp 0      TMA producer: 128x64 A tile + two 128x64 B half-tiles per stage, 128-byte
//               swizzle, 4-stage ring of full / empty mbarriers (plain loads, no multicast);
//   warp 1      TMEM allocator and MMA issuer: one elected thread issues
//               tcgen05.mma.cta_group::1.kind::f16 (M=128, N=256, K=16) x4 per stage and
//               commits each stage back to its empty barrier;
//   warps 2-5   epilogue: tcgen05.ld of the fp32 accumulator (each warp its 32-lane TMEM
//               quarter), fused epilogue, 16-byte global stores.
// The accumulator is double-buffered in TMEM (2 x 256 of the 512 columns), so the
// epilogue of tile t overlaps the main loop of tile t+1.  Fused epilogues:
//   EPI_STORE     bf16 D
//   EPI_SWIGLU    B = [gate; up] (2I rows); each N tile holds 128 gate + 128 up columns
//                 and writes silu(gate) * up (the reference's act_fn(gate) * up,
//                 model.py:32-34) as bf16 [M, I]
//   EPI_RESIDUAL  D = acc + R (bf16), for the residual stream when no all-reduce follows
//   EPI_ROPE      the qkv projection of a decoder layer: D = acc (bf16) with the rotary
//                 embedding applied to the q and k heads of each row at its position, and
//                 the (rotated) k and v heads also written to the paged KV cache (the
//                 standalone rope_kv kernel's work, done while the next tile's MMAs run)
//   EPI_QS*       quantize every 128-column group of the bf16-rounded tile and store codes +
//                 (scale, zero) into the owning rank's reduce-scatter slot over NVLink: the
//                 first phase of the two-shot all-reduce, overlapped with the GEMM.  The
//                 last CTA publishes a per-rank epoch flag to every peer.
// Every mbarrier wait is bounded (%globaltimer); on expiry the CTA records an error code,
// drains its in-flight copies and MMAs (bounded), frees TMEM and returns.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "scatter.h"
#include "smem_optin.h"
#include "tcgen05.cuh"

namespace qfc {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int A_BYTES = BM * BK * 2;        // 16 KiB
constexpr int B_HALF_BYTES = 128 * BK * 2;  // 16 KiB
constexpr int B_BYTES = 2 * B_HALF_BYTES;   // 32 KiB
constexpr int NUM_THREADS = 192;
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 16;

// Single CTA: a 128 x 256 tile per CTA, 4 stages of A + both B halves (48 KiB).
// CTA pair (cta_group::2): a 256 x 256 tile per pair; each CTA loads its 128 rows of A and
// one 128-row half of B per stage (32 KiB, 6 stages), the even CTA issues M=256 MMAs that
// read both CTAs' shared memory, and each CTA's TMEM holds its 128 rows of the tile.  Per
// FLOP a CTA loads a third less than alone.
template <bool PAIR>
struct Cfg {
  static constexpr int STAGES = PAIR ? 6 : 4;
  static constexpr int B_LOAD = PAIR ? B_HALF_BYTES : B_BYTES;  // B bytes this CTA loads per stage
  static constexpr int STAGE_BYTES = A_BYTES + B_LOAD;
  static constexpr int TILE_M = PAIR ? 2 * BM : BM;
  static constexpr uint32_t IDESC = tc::idesc_f16(TILE_M, BN, true);
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};
// EPI_QS*: per epilogue warp, 32 staged rows of one quantized 128-column group.
constexpr int QS_STAGE_BYTES = 4 * 32 * 256;

// EPI_QS8 / EPI_QS4 / EPI_QS16: quantize each 128-column group of the (bf16-rounded) tile
// to INT8 / INT4 / raw bf16 and store it into the owner rank's reduce-scatter slot.
enum Epi : int { EPI_STORE = 0, EPI_SWIGLU = 1, EPI_RESIDUAL = 2, EPI_QS8 = 3, EPI_QS4 = 4, EPI_QS16 = 5,
                 EPI_ROPE = 6 };

// EPI_ROPE: head_dim 128, so a 256-column tile holds two whole heads.
struct RopeArgs {
  const int64_t* pos;       // [M] position of each row
  const float2* cs;         // [max_position, 64] (cos, sin)
  __nv_bfloat16* kc;        // [pages, nkv, page, 128] or nullptr (no cache)
  __nv_bfloat16* vc;
  const int64_t* slots;     // [M] cache slot page * page_size + offset; < 0 = not cached
  int nq, nkv, page, page_shift;
};

constexpr bool is_qs(int epi) { return epi == EPI_QS8 || epi == EPI_QS4 || epi == EPI_QS16; }

enum : int { GEMM_ERR_PRODUCER = 0x100, GEMM_ERR_MMA = 0x200, GEMM_ERR_EPI = 0x300 };

struct GemmArgs {
  int M, N, K;       // D[M, N]; for EPI_SWIGLU N is the output width I and B has 2I rows
  int n_tiles;       // tiles along N
  int n_tile_cols;   // output columns per N tile (256, or 128 for EPI_SWIGLU)
  int b_second;      // row offset of the second 128-row half of a B tile
  int b_first_step;  // rows of B advanced per N tile
  __nv_bfloat16* D;
  int ldd;
  const __nv_bfloat16* R;
  int ldr;
  int* status;
  uint64_t timeout_ns;
  ScatterArgs sc;    // EPI_QS*
  RopeArgs rope;     // EPI_ROPE
  // split-K (single CTAs, small M): work unit = (tile, split); each unit writes its fp32
  // partial tile, the last unit of a tile (device counter) sums them in split order into
  // TMEM and runs the epilogue.
  int splits;        // 1 = no split
  int kb_split;      // k-blocks per split
  float* part;       // [tiles][splits][BM][BN] fp32
  int* counters;     // [tiles], zero between launches (the last unit resets its entry)
};

// Payload bytes of one 128-value group: INT8 codes, packed INT4 codes or raw bf16.
template <int P>
constexpr int qs_group_bytes() { return P == 8 ? 128 : (P == 4 ? 64 : 256); }

// Staging row of one thread: its group's payload, 16-byte chunk c at c ^ (row & 7) (mask
// 3 for the 4-chunk INT4 rows) so that a warp's rows spread over the banks.
template <int P>
QFC_DEV int qs_swz(int row, int c) { return c ^ (row & (P == 4 ? 3 : 7)); }

// Quantize 128 consecutive values of one row (held by this thread): the codes go to the
// warp's staging row `stage` (shared memory), the group's (scale, zero) straight to meta.
// P = 8, 4 or 16 (raw bf16).
template <int P>
QFC_DEV void qs_encode_group(const float (&v)[128], uint8_t* stage, int srow, char* meta, int64_t local,
                             const ScatterArgs& sc) {
  uint4* st = reinterpret_cast<uint4*>(stage);
  if constexpr (P == 16) {
#pragma unroll
    for (int k = 0; k < 16; ++k)
      st[qs_swz<P>(srow, k)] = make_uint4(pack_bf16x2(v[8 * k], v[8 * k + 1]), pack_bf16x2(v[8 * k + 2], v[8 * k + 3]),
                                          pack_bf16x2(v[8 * k + 4], v[8 * k + 5]), pack_bf16x2(v[8 * k + 6], v[8 * k + 7]));
  } else {
    float mn4[4] = {v[0], v[1], v[2], v[3]}, mx4[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
    for (int i = 4; i < 128; i += 4)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        mn4[q] = fminf(mn4[q], v[i + q]);
        mx4[q] = fmaxf(mx4[q], v[i + q]);
      }
    const float mn = fminf(fminf(mn4[0], mn4[1]), fminf(mn4[2], mn4[3]));
    const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
    float s, inv, z;
    if (sc.sym) QMath<P, true>::params(mn, mx, s, inv, z);
    else QMath<P, false>::params(mn, mx, s, inv, z);
    if constexpr (P == 8) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {  // 16 codes per 16-byte chunk
        uint32_t m0[8], m1[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          m0[i] = QMath<P, false>::codebits(v[16 * k + i], inv, z);
          m1[i] = QMath<P, false>::codebits(v[16 * k + 8 + i], inv, z);
        }
        const uint2 a = codebits8_to_u2(m0), b = codebits8_to_u2(m1);
        st[qs_swz<P>(srow, k)] = make_uint4(a.x, a.y, b.x, b.y);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) {  // 32 codes per 16-byte chunk
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t m[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) m[i] = QMath<P, false>::codebits(v[32 * k + 8 * q + i], inv, z);
          w[q] = codebits8_to_int4(m);
        }
        st[qs_swz<P>(srow, k)] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    const int64_t g = local >> sc.gs_shift;
    if (sc.meta_fp32) *reinterpret_cast<float2*>(meta + g * 8) = make_float2(s, z);
    else *reinterpret_cast<uint32_t*>(meta + g * 4) = pack_f16x2(s, z);
  }
}

// The warp's 32 staged rows go out row-contiguous: LPR lanes per row, 16 bytes each, so a
// store instruction writes 512 bytes as a few whole 64- to 256-byte row segments (over
// NVLink when the owner is a peer) instead of 32 scattered 16-byte pieces.  dst = the
// row's payload destination (nullptr: row outside the output).
template <int P>
QFC_DEV void qs_flush_rows(const uint8_t* stage_warp, char* dst, int lane) {
  constexpr int PB = qs_group_bytes<P>();
  constexpr int LPR = PB / 16;
  constexpr int RPI = 32 / LPR;
  __syncwarp();
#pragma unroll 4
  for (int it = 0; it < 32 / RPI; ++it) {
    const int rr = it * RPI + lane / LPR, c = lane % LPR;
    const unsigned long long d =
        __shfl_sync(QFC_FULL_MASK, (unsigned long long)reinterpret_cast<uintptr_t>(dst), rr);
    if (d) {
      const uint4 x = *reinterpret_cast<const uint4*>(stage_warp + rr * PB + (qs_swz<P>(rr, c) << 4));
      *reinterpret_cast<uint4*>(reinterpret_cast<char*>(d) + c * 16) = x;
    }
  }
  __syncwarp();  // the staging rows are rewritten by the next group
}

QFC_DEV void tile_coords(int tile, int m_tiles, int n_tiles, int& mb, int& nb) {
  const int group = GROUP_M * n_tiles;
  const int g = tile / group;
  const int first_m = g * GROUP_M;
  const int gm = min(m_tiles - first_m, GROUP_M);
  const int r = tile % group;
  mb = first_m + r % gm;
  nb = r / gm;
}

QFC_DEV void fail(const GemmArgs& a, volatile int* s_abort, int code) {
  *s_abort = 1;
  if (a.status) atomicCAS(a.status, 0, code);
}

QFC_DEV uint32_t pack_bf16(float lo, float hi) { return pack_bf16x2(lo, hi); }

template <int EPI, bool PAIR>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const GemmArgs args) {
  using C = Cfg<PAIR>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * C::B_LOAD);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = bars + 2 * STAGES + 2;
  uint64_t* drain = bars + 2 * STAGES + 4;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_holder + 1);
  uint8_t* qs_stage = reinterpret_cast<uint8_t*>(bars) + 256;  // EPI_QS* only (QS_STAGE_BYTES)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // scheduling unit: a CTA, or a CTA pair (cluster of 2; rank 0 issues the MMAs)
  const uint32_t crank = PAIR ? tc::cluster_ctarank() : 0u;
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int n_units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int m_tiles = (args.M + C::TILE_M - 1) / C::TILE_M;
  const int tiles = m_tiles * args.n_tiles;
  const int works = tiles * args.splits;
  const int kbs = (args.K + BK - 1) / BK;
  __shared__ int s_split_last;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(tc::smem_u32(&full[s]), 1);
      tc::mbar_init(tc::smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(tc::smem_u32(&tfull[b]), 1);
      tc::mbar_init(tc::smem_u32(&tempty[b]), PAIR ? 256 : 128);  // epilogue threads (of both CTAs)
    }
    tc::mbar_init(tc::smem_u32(drain), 1);
    *s_abort = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tc::tma_prefetch_desc(&tmA);
    tc::tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tc::tmem_alloc_pair(tc::smem_u32(tmem_holder), TMEM_COLS);
      tc::tmem_relinquish_pair();
    } else {
      tc::tmem_alloc(tc::smem_u32(tmem_holder), TMEM_COLS);
      tc::tmem_relinquish();
    }
  }
  tc::tc_fence_before();
  if constexpr (PAIR) tc::cluster_sync();  // the peer's barriers are initialised before any remote signal
  else __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      int last_issue[STAGES];
      for (int s = 0; s < STAGES; ++s) last_issue[s] = -1;
      bool ok = true;
      for (int w = unit; w < works && ok; w += n_units) {
        const int tile = w / args.splits, sp = w - tile * args.splits;
        const int kb0 = sp * args.kb_split, kb1 = min(kbs, kb0 + args.kb_split);
        int mb, nb;
        tile_coords(tile, m_tiles, args.n_tiles, mb, nb);
        const int yb = nb * args.b_first_step;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!tc::mbar_wait(tc::smem_u32(&empty[s]), ph ^ 1, globaltimer_ns() + args.timeout_ns, s_abort)) {
            fail(args, s_abort, GEMM_ERR_PRODUCER | 1);
            ok = false;
            break;
          }
          const uint32_t fb = tc::smem_u32(&full[s]);
          if constexpr (PAIR) {
            // both CTAs' copies complete on the even CTA's barrier, which expects both
            const uint32_t fb0 = tc::mapa_shared(fb, 0);
            if (crank == 0) tc::mbar_arrive_expect_tx(fb, 2 * C::STAGE_BYTES);
            tc::tma_load_2d_pair(tc::smem_u32(sA + s * A_BYTES), &tmA, fb0, kb * BK, mb * C::TILE_M + (int)crank * BM);
            tc::tma_load_2d_pair(tc::smem_u32(sB + s * C::B_LOAD), &tmB, fb0, kb * BK,
                                 crank ? yb + args.b_second : yb);
          } else {
            tc::mbar_arrive_expect_tx(fb, C::STAGE_BYTES);
            tc::tma_load_2d(tc::smem_u32(sA + s * A_BYTES), &tmA, fb, kb * BK, mb * BM);
            tc::tma_load_2d(tc::smem_u32(sB + s * C::B_LOAD), &tmB, fb, kb * BK, yb);
            tc::tma_load_2d(tc::smem_u32(sB + s * C::B_LOAD + B_HALF_BYTES), &tmB, fb, kb * BK, yb + args.b_second);
          }
          last_issue[s] = it;
        }
      }
      if ((!ok || *s_abort) && crank == 0) {
        // Let every issued copy land before the CTA (and its shared memory) goes away.
        for (int s = 0; s < STAGES; ++s) {
          if (last_issue[s] < 0) continue;
          const uint32_t ph = (last_issue[s] / STAGES) & 1;
          int never = 0;
          tc::mbar_wait(tc::smem_u32(&full[s]), ph, globaltimer_ns() + 50000000ull, &never);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && crank == 0) {
      int it = 0, t = 0;
      bool ok = true;
      bool issued = false;
      for (int w = unit; w < works && ok; w += n_units, ++t) {
        const int kb0 = (w % args.splits) * args.kb_split, kb1 = min(kbs, kb0 + args.kb_split);
        const int buf = t & 1;
        if (!tc::mbar_wait(tc::smem_u32(&tempty[buf]), ((t >> 1) & 1) ^ 1, globaltimer_ns() + args.timeout_ns,
                           s_abort)) {
          fail(args, s_abort, GEMM_ERR_MMA | 1);
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t tmem_d = tmem_base + (uint32_t)(buf * BN);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!tc::mbar_wait(tc::smem_u32(&full[s]), ph, globaltimer_ns() + args.timeout_ns, s_abort)) {
            fail(args, s_abort, GEMM_ERR_MMA | 2);
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t a0 = tc::smem_u32(sA + s * A_BYTES);
          const uint32_t b0 = tc::smem_u32(sB + s * C::B_LOAD);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            if constexpr (PAIR)
              tc::umma_f16_pair(tmem_d, tc::sw128_kmajor_desc(a0 + k * 32), tc::sw128_kmajor_desc(b0 + k * 32),
                                C::IDESC, (kb != kb0) || (k != 0));
            else
              tc::umma_f16(tmem_d, tc::sw128_kmajor_desc(a0 + k * 32), tc::sw128_kmajor_desc(b0 + k * 32), C::IDESC,
                           (kb != kb0) || (k != 0));
          }
          issued = true;
          if constexpr (PAIR) tc::umma_commit_pair(tc::smem_u32(&empty[s]), 0x3);
          else tc::umma_commit(tc::smem_u32(&empty[s]));
        }
        if (!ok) break;
        if constexpr (PAIR) tc::umma_commit_pair(tc::smem_u32(&tfull[buf]), 0x3);
        else tc::umma_commit(tc::smem_u32(&tfull[buf]));
      }
      if ((!ok || *s_abort) && issued) {
        // Wait for the MMAs already issued before TMEM is released.
        if constexpr (PAIR) tc::umma_commit_pair(tc::smem_u32(drain), 0x1);
        else tc::umma_commit(tc::smem_u32(drain));
        int never = 0;
        tc::mbar_wait(tc::smem_u32(drain), 0, globaltimer_ns() + 50000000ull, &never);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;  // the TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    int t = 0;
    for (int w = unit; w < works; w += n_units, ++t) {
      const int tile = w / args.splits;
      int mb, nb;
      tile_coords(tile, m_tiles, args.n_tiles, mb, nb);
      const int buf = t & 1;
      if (!tc::mbar_wait(tc::smem_u32(&tfull[buf]), (t >> 1) & 1, globaltimer_ns() + args.timeout_ns, s_abort)) {
        fail(args, s_abort, GEMM_ERR_EPI | 1);
        break;
      }
      tc::tc_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t)(buf * BN) + ((uint32_t)(q * 32) << 16);
      const int row = mb * C::TILE_M + (int)crank * BM + row_in_tile;
      const int col0 = nb * args.n_tile_cols;
      if constexpr (!PAIR && !is_qs(EPI)) {
        if (args.splits > 1) {
          // this unit's fp32 partial out of TMEM
          const int S = args.splits, sp = w - tile * S;
          float* mine = args.part + (((int64_t)tile * S + sp) * BM + row_in_tile) * BN;
#pragma unroll 1
          for (int c = 0; c < BN; c += 32) {
            uint32_t r[32];
            tc::tmem_ld_32x32b_x32(taddr + c, r);
            tc::tmem_wait_ld();
            tc::tmem_reg_fence(r);
            if (row < args.M) {
#pragma unroll
              for (int j = 0; j < 8; ++j)
                reinterpret_cast<uint4*>(mine + c)[j] = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
            }
          }
          __threadfence();
          asm volatile("bar.sync 1, 128;" ::: "memory");  // the 4 epilogue warps
          if (threadIdx.x == 64) {
            const int prev = atomicAdd(args.counters + tile, 1);
            s_split_last = (prev == S - 1);
            if (prev == S - 1) args.counters[tile] = 0;  // every unit of the tile has arrived
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (!s_split_last) {
            tc::tc_fence_before();
            tc::mbar_arrive(tc::smem_u32(&tempty[buf]));
            continue;
          }
          __threadfence();
          // the sum of all splits, in split order, back into this TMEM buffer
          const float* p0 = args.part + ((int64_t)tile * S * BM + row_in_tile) * BN;
#pragma unroll 1
          for (int c = 0; c < BN; c += 32) {
            float acc[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = 0.f;
            if (row < args.M) {
              for (int s2 = 0; s2 < S; ++s2) {
                const float4* src = reinterpret_cast<const float4*>(p0 + (int64_t)s2 * BM * BN + c);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const float4 x = __ldcg(src + j);
                  acc[4 * j] += x.x;
                  acc[4 * j + 1] += x.y;
                  acc[4 * j + 2] += x.z;
                  acc[4 * j + 3] += x.w;
                }
              }
            }
            uint32_t r[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(acc[j]);
            tc::tmem_st_32x32b_x32(taddr + c, r);
          }
          tc::tmem_wait_st();
        }
      }
      if constexpr (is_qs(EPI)) {
        constexpr int P = EPI == EPI_QS8 ? 8 : (EPI == EPI_QS4 ? 4 : 16);
#pragma unroll 1
        for (int g0 = 0; g0 < BN; g0 += 128) {  // two 128-column groups per tile
          uint32_t r[4][32];
#pragma unroll
          for (int c = 0; c < 4; ++c) tc::tmem_ld_32x32b_x32(taddr + g0 + c * 32, r[c]);
          tc::tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 4; ++c) tc::tmem_reg_fence(r[c]);
          const int col = col0 + g0;
          uint8_t* stage_warp = qs_stage + q * 32 * qs_group_bytes<P>();
          char* dst = nullptr;
          if (row < args.M && col < args.N) {
            float v[128];
#pragma unroll
            for (int c = 0; c < 4; ++c)
#pragma unroll
              for (int j = 0; j < 32; ++j)  // the bf16 value the unfused GEMM would have stored
                v[c * 32 + j] = to_f32(from_f32<__nv_bfloat16>(__uint_as_float(r[c][j])));
            const int64_t e = (int64_t)row * args.N + col;
            const int owner = (int)(e / args.sc.chunk);
            const int64_t local = e - (int64_t)owner * args.sc.chunk;
            char* slot = args.sc.base[owner] + args.sc.rs_off + (int64_t)args.sc.rank * args.sc.slot1;
            qs_encode_group<P>(v, stage_warp + lane * qs_group_bytes<P>(), lane, slot + args.sc.pay1, local, args.sc);
            dst = slot + (P == 8 ? local : (P == 4 ? (local >> 1) : local * 2));
          }
          qs_flush_rows<P>(stage_warp, dst, lane);
        }
      } else if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          uint32_t g[32], u[32];
          tc::tmem_ld_32x32b_x32(taddr + c, g);
          tc::tmem_ld_32x32b_x32(taddr + 128 + c, u);
          tc::tmem_wait_ld();
          tc::tmem_reg_fence(g);
          tc::tmem_reg_fence(u);
          const int col = col0 + c;
          if (row < args.M && col < args.N) {
            uint32_t o[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float v[2];
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const float gb = to_f32(from_f32<__nv_bfloat16>(__uint_as_float(g[2 * j + h])));
                const float ub = to_f32(from_f32<__nv_bfloat16>(__uint_as_float(u[2 * j + h])));
                const float sb = to_f32(from_f32<__nv_bfloat16>(gb / (1.f + __expf(-gb))));
                v[h] = sb * ub;
              }
              o[j] = pack_bf16(v[0], v[1]);
            }
            __nv_bfloat16* dst = args.D + (int64_t)row * args.ldd + col;
            if (col + 32 <= args.N) {
#pragma unroll
              for (int j = 0; j < 4; ++j)
                reinterpret_cast<uint4*>(dst)[j] = make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
            } else {
              const __nv_bfloat16* ob = reinterpret_cast<const __nv_bfloat16*>(o);
              for (int j = 0; j < 32 && col + j < args.N; ++j) dst[j] = ob[j];
            }
          }
        }
      } else if constexpr (EPI == EPI_ROPE) {
        const RopeArgs& ra = args.rope;
        const int hq = ra.nq, hk = ra.nq + ra.nkv;
#pragma unroll 1
        for (int hl = 0; hl < 2; ++hl) {  // the tile's two heads
          const int hcol = col0 + hl * 128;
          const int head = hcol >> 7;
          const bool live = row < args.M && hcol < args.N;
          const bool rot = head < hk;  // q and k heads rotate, v heads pass through
          int64_t p_row = 0, slot = -1;
          if (live) {
            p_row = ra.pos[row];
            if (ra.slots != nullptr && head >= hq) slot = ra.slots[row];
          }
          __nv_bfloat16* dst = args.D + (int64_t)row * args.ldd + hcol;
          __nv_bfloat16* cdst = nullptr;
          if (slot >= 0) {
            const int64_t pg = ra.page_shift >= 0 ? slot >> ra.page_shift : slot / ra.page;
            const int64_t off = ra.page_shift >= 0 ? (slot & (ra.page - 1)) : slot % ra.page;
            const int kvh = head < hk ? head - hq : head - hk;
            cdst = (head < hk ? ra.kc : ra.vc) + ((pg * ra.nkv + kvh) * (int64_t)ra.page + off) * 128;
          }
#pragma unroll 1
          for (int c = 0; c < 64; c += 32) {  // element i pairs with i + 64
            uint32_t r1[32], r2[32];
            tc::tmem_ld_32x32b_x32(taddr + hl * 128 + c, r1);
            tc::tmem_ld_32x32b_x32(taddr + hl * 128 + 64 + c, r2);
            tc::tmem_wait_ld();
            tc::tmem_reg_fence(r1);
            tc::tmem_reg_fence(r2);
            if (!live) continue;
            float x1[32], x2[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {  // the bf16 values the unfused GEMM would store
              x1[j] = to_f32(from_f32<__nv_bfloat16>(__uint_as_float(r1[j])));
              x2[j] = to_f32(from_f32<__nv_bfloat16>(__uint_as_float(r2[j])));
            }
            if (rot) {
              const float4* csp = reinterpret_cast<const float4*>(ra.cs + p_row * 64 + c);
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float4 a = __ldg(csp + j);  // (cos, sin) of elements 2j and 2j + 1
                rope_pair(x1[2 * j], x2[2 * j], a.x, a.y, x1[2 * j], x2[2 * j]);
                rope_pair(x1[2 * j + 1], x2[2 * j + 1], a.z, a.w, x1[2 * j + 1], x2[2 * j + 1]);
              }
            }
            uint4 o1[4], o2[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              o1[j] = make_uint4(pack_bf16(x1[8 * j], x1[8 * j + 1]), pack_bf16(x1[8 * j + 2], x1[8 * j + 3]),
                                 pack_bf16(x1[8 * j + 4], x1[8 * j + 5]), pack_bf16(x1[8 * j + 6], x1[8 * j + 7]));
              o2[j] = make_uint4(pack_bf16(x2[8 * j], x2[8 * j + 1]), pack_bf16(x2[8 * j + 2], x2[8 * j + 3]),
                                 pack_bf16(x2[8 * j + 4], x2[8 * j + 5]), pack_bf16(x2[8 * j + 6], x2[8 * j + 7]));
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              reinterpret_cast<uint4*>(dst + c)[j] = o1[j];
              reinterpret_cast<uint4*>(dst + 64 + c)[j] = o2[j];
            }
            if (cdst != nullptr) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                reinterpret_cast<uint4*>(cdst + c)[j] = o1[j];
                reinterpret_cast<uint4*>(cdst + 64 + c)[j] = o2[j];
              }
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tc::tmem_ld_32x32b_x32(taddr + c, r);
          tc::tmem_wait_ld();
          tc::tmem_reg_fence(r);
          const int col = col0 + c;
          if (row < args.M && col < args.N) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
            if constexpr (EPI == EPI_RESIDUAL) {
              const __nv_bfloat16* rp = args.R + (int64_t)row * args.ldr + col;
              if (col + 32 <= args.N) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  float rv[8];
                  Vec8IO<__nv_bfloat16>::load(rp + 8 * j, rv);
#pragma unroll
                  for (int i = 0; i < 8; ++i) v[8 * j + i] = to_f32(from_f32<__nv_bfloat16>(v[8 * j + i])) + rv[i];
                }
              } else {
                for (int j = 0; j < 32 && col + j < args.N; ++j)
                  v[j] = to_f32(from_f32<__nv_bfloat16>(v[j])) + to_f32(rp[j]);
              }
            }
            __nv_bfloat16* dst = args.D + (int64_t)row * args.ldd + col;
            if (col + 32 <= args.N) {
#pragma unroll
              for (int j = 0; j < 4; ++j)
                reinterpret_cast<uint4*>(dst)[j] =
                    make_uint4(pack_bf16(v[8 * j], v[8 * j + 1]), pack_bf16(v[8 * j + 2], v[8 * j + 3]),
                               pack_bf16(v[8 * j + 4], v[8 * j + 5]), pack_bf16(v[8 * j + 6], v[8 * j + 7]));
            } else {
              for (int j = 0; j < 32 && col + j < args.N; ++j) dst[j] = from_f32<__nv_bfloat16>(v[j]);
            }
          }
        }
      }
      tc::tc_fence_before();
      if constexpr (PAIR) tc::mbar_arrive_cluster(tc::mapa_shared(tc::smem_u32(&tempty[buf]), 0));
      else tc::mbar_arrive(tc::smem_u32(&tempty[buf]));
    }
    // Peer stores of this thread are visible system-wide before the CTA reports done.
    if constexpr (is_qs(EPI)) __threadfence_system();
  }
  __syncthreads();
  if constexpr (is_qs(EPI)) {
    // The last CTA to finish advances this rank's fused-GEMM epoch and publishes it to
    // every rank: the reduce-scatter slots of all of this rank's tiles are filled.
    if (threadIdx.x == 0) {
      __threadfence_system();
      const uint32_t prev = atomicAdd(args.sc.done_ctas, 1u);
      if (prev == gridDim.x - 1) {
        *args.sc.done_ctas = 0u;
        const uint32_t e = *args.sc.epoch + 1u;
        *args.sc.epoch = e;
        __threadfence_system();
        for (int j = 0; j < args.sc.world; ++j) {
          uint32_t* flag = reinterpret_cast<uint32_t*>(args.sc.base[j]) +
                           ((int64_t)(PH_GEMM * kMaxBlocks + 0) * kMaxRanks + args.sc.rank);
          st_release_sys(flag, e);
        }
      }
    }
  }
  // No CTA of a pair leaves (or frees TMEM) while its peer may still signal its barriers.
  if constexpr (PAIR) tc::cluster_sync();
  if (warp == 1) {
    tc::tc_fence_after();
    if constexpr (PAIR) tc::tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else tc::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p != nullptr,
                "gemm: cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix (row stride ld elements),
// box = box_rows x 64 columns, 128-byte swizzle, out-of-range elements read as zero.
CUtensorMap make_tmap(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "gemm: cuTensorMapEncodeTiled failed (", (int)r, ")");
  return m;
}

int* status_word() {
  static int* p = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = nullptr;
    TORCH_CHECK(cudaHostAlloc(&h, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable) == cudaSuccess,
                "gemm: cudaHostAlloc(status) failed");
    *reinterpret_cast<volatile int*>(h) = 0;
    p = reinterpret_cast<int*>(h);
  });
  return p;
}

// Split-K for small M is on unless QFC_GEMM_SPLITK=0 (kept for A/B measurements).
bool split_k_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("QFC_GEMM_SPLITK");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Per-device arrival counters of split-K tiles, zeroed once; each launch leaves them zero.
// One set per device: split-K GEMMs that run at the same time on two streams of one
// device would share them, so such GEMMs must be ordered (the models launch everything
// on one stream).
int* split_counters(int dev, int tiles) {
  constexpr int kMaxTiles = 1 << 14;
  static int* buf[64] = {nullptr};
  static std::mutex mu;
  TORCH_CHECK(tiles <= kMaxTiles, "gemm: too many split-K tiles");
  std::lock_guard<std::mutex> lock(mu);
  if (buf[dev] == nullptr) {
    void* p = nullptr;
    C10_CUDA_CHECK(cudaMalloc(&p, kMaxTiles * sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(p, 0, kMaxTiles * sizeof(int)));
    buf[dev] = static_cast<int*>(p);
  }
  return buf[dev];
}

// CTA-pair GEMMs are on unless QFC_GEMM_PAIR=0 (kept for A/B measurements).
bool pair_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("QFC_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}

int sm_count(int dev) {
  static std::atomic<int> cached[64] = {};  // threads may race to fill an entry: same value
  int v = cached[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cached[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

template <int EPI, bool PAIR>
void launch_cfg(const CUtensorMap& tA, const CUtensorMap& tB, const GemmArgs& a, int M, int dev, int max_ctas) {
  using C = Cfg<PAIR>;
  constexpr int smem = C::SMEM_BYTES + (is_qs(EPI) ? QS_STAGE_BYTES : 0);
  static_assert(smem <= 232448, "GEMM shared memory exceeds 227 KiB");
  static std::atomic<unsigned long long> smem_set{0};
  auto kern = gemm_bf16_kernel<EPI, PAIR>;
  C10_CUDA_CHECK(opt_in_smem_per_device(kern, smem, smem_set));
  const int tiles = ((M + C::TILE_M - 1) / C::TILE_M) * a.n_tiles;
  const int per_unit = PAIR ? 2 : 1;
  GemmArgs args = a;
  args.splits = 1;
  args.kb_split = (a.K + BK - 1) / BK;
  args.part = nullptr;
  args.counters = nullptr;
  at::Tensor part;
  const int kbs = (a.K + BK - 1) / BK;
  if (!PAIR && !is_qs(EPI) && split_k_enabled() && 2 * tiles <= sm_count(dev) && kbs >= 8 && max_ctas <= 0) {
    // small M: too few tiles to stream the weights from every SM; split K so that about
    // one unit per SM runs, each with at least 4 k-blocks
    int S = std::min(sm_count(dev) / tiles, kbs / 4);
    if (S > 1) {
      args.kb_split = (kbs + S - 1) / S;
      args.splits = (kbs + args.kb_split - 1) / args.kb_split;
      part = at::empty({(int64_t)tiles * args.splits * BM * BN},
                       at::TensorOptions().dtype(at::kFloat).device(at::kCUDA, dev));
      args.part = part.data_ptr<float>();
      args.counters = split_counters(dev, tiles);
    }
  }
  const int works = tiles * args.splits;
  int units = std::min(works, sm_count(dev) / per_unit);
  if (max_ctas > 0) units = std::min(units, std::max(1, max_ctas / per_unit));
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(units * per_unit);
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = per_unit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = PAIR ? 1 : 0;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, tA, tB, args));
}

// CTA pairs serve M >= 256 (a 256-row tile per pair); smaller M runs one CTA per tile.
template <int EPI>
void launch(const at::Tensor& A, const at::Tensor& B, at::Tensor* D, const at::Tensor* R, int M, int N, int K,
            double timeout_ms, int max_ctas, const ScatterArgs* sc = nullptr, const RopeArgs* rope = nullptr) {
  const int dev = A.get_device();
  GemmArgs a;
  a.M = M;
  a.N = N;
  a.K = K;
  if (EPI == EPI_SWIGLU) {
    a.n_tile_cols = 128;
    a.b_first_step = 128;
    a.b_second = N;  // up rows start at I
  } else {
    a.n_tile_cols = BN;
    a.b_first_step = BN;
    a.b_second = 128;
  }
  a.n_tiles = (N + a.n_tile_cols - 1) / a.n_tile_cols;
  a.D = D ? reinterpret_cast<__nv_bfloat16*>(D->data_ptr()) : nullptr;
  a.ldd = D ? (int)D->stride(0) : 0;
  std::memset(&a.sc, 0, sizeof(a.sc));
  if (sc) a.sc = *sc;
  std::memset(&a.rope, 0, sizeof(a.rope));
  if (rope) a.rope = *rope;
  a.R = R ? reinterpret_cast<const __nv_bfloat16*>(R->data_ptr()) : nullptr;
  a.ldr = R ? (int)R->stride(0) : 0;
  a.status = status_word();
  a.timeout_ns = (uint64_t)(timeout_ms * 1e6);
  a.splits = 1;
  a.kb_split = (K + BK - 1) / BK;
  a.part = nullptr;
  a.counters = nullptr;
  const CUtensorMap tA = make_tmap(A.data_ptr(), M, K, A.stride(0), BM);
  const CUtensorMap tB = make_tmap(B.data_ptr(), B.size(0), K, B.stride(0), 128);
  const bool pair = M >= 2 * BM && pair_enabled() && (max_ctas <= 0 || max_ctas >= 2);
  if (pair) launch_cfg<EPI, true>(tA, tB, a, M, dev, max_ctas);
  else launch_cfg<EPI, false>(tA, tB, a, M, dev, max_ctas);
}

void check_operand(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2, "gemm: ", name,
              " must be a 2-D bf16 CUDA tensor");
  TORCH_CHECK(t.stride(1) == 1 && (t.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              "gemm: ", name, " must be row-major with 16-byte aligned rows");
}


// ---------------------------------------------------------------------------------------
// Small M (decode): swapped operands.  D^T[N, M] = W[N, K] . X[M, K]^T with the weight
// rows as the MMA's M = 128 and up to 64 tokens as its N: a tile is 128 weight rows, a
// stage is 16 KiB of weights + 8 KiB of activations (8 stages in flight), and the tiles
// are twice as many as with 256-row weight tiles.  Each epilogue thread owns one output
// column (TMEM lane) for every token, so a warp's stores run along an output row.  Split-K
// as in the main kernel (fp32 partials, the last unit of a tile sums them in split order
// into TMEM).  EPI_STORE and EPI_RESIDUAL.
// ---------------------------------------------------------------------------------------
namespace small {

constexpr int BW = 128;       // weight rows per tile (MMA M)
constexpr int TN = 64;        // tokens (MMA N)
constexpr int STAGES = 8;
constexpr int W_BYTES = BW * BK * 2;   // 16 KiB
constexpr int X_BYTES = TN * BK * 2;   // 8 KiB
constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
constexpr int TMEM_COLS_S = 128;       // 2 accumulator buffers x 64 columns
constexpr uint32_t IDESC_S = tc::idesc_f16(BW, TN, true);
constexpr int SMEM_BYTES_S = STAGES * STAGE_BYTES + 1024 + 256;

struct SArgs {
  int M, N, K;
  int n_tiles, splits, kb_split;
  __nv_bfloat16* D;
  int ldd;
  const __nv_bfloat16* R;  // nullptr: plain store
  int ldr;
  float* part;             // [tiles][splits][BW][TN]
  int* counters;
  int* status;
  uint64_t timeout_ns;
};

QFC_DEV void sfail(const SArgs& a, volatile int* ab, int code) {
  *ab = 1;
  if (a.status) atomicCAS(a.status, 0, code);
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_small_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, const SArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sX = smem + STAGES * W_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sX + STAGES * X_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = bars + 2 * STAGES + 2;
  uint64_t* drain = bars + 2 * STAGES + 4;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_holder + 1);
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int works = args.n_tiles * args.splits;
  const int kbs = (args.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(tc::smem_u32(&full[s]), 1);
      tc::mbar_init(tc::smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(tc::smem_u32(&tfull[b]), 1);
      tc::mbar_init(tc::smem_u32(&tempty[b]), 128);
    }
    tc::mbar_init(tc::smem_u32(drain), 1);
    *s_abort = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tc::tma_prefetch_desc(&tmW);
    tc::tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tc::tmem_alloc(tc::smem_u32(tmem_holder), TMEM_COLS_S);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      int last_issue[STAGES];
      for (int s = 0; s < STAGES; ++s) last_issue[s] = -1;
      bool ok = true;
      for (int w = blockIdx.x; w < works && ok; w += gridDim.x) {
        const int tile = w / args.splits, sp = w - tile * args.splits;
        const int kb0 = sp * args.kb_split, kb1 = min(kbs, kb0 + args.kb_split);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!tc::mbar_wait(tc::smem_u32(&empty[s]), ph ^ 1, globaltimer_ns() + args.timeout_ns, s_abort)) {
            sfail(args, s_abort, GEMM_ERR_PRODUCER | 0x10);
            ok = false;
            break;
          }
          const uint32_t fb = tc::smem_u32(&full[s]);
          tc::mbar_arrive_expect_tx(fb, STAGE_BYTES);
          tc::tma_load_2d(tc::smem_u32(sW + s * W_BYTES), &tmW, fb, kb * BK, tile * BW);
          tc::tma_load_2d(tc::smem_u32(sX + s * X_BYTES), &tmX, fb, kb * BK, 0);
          last_issue[s] = it;
        }
      }
      if (!ok || *s_abort) {
        for (int s = 0; s < STAGES; ++s) {
          if (last_issue[s] < 0) continue;
          int never = 0;
          tc::mbar_wait(tc::smem_u32(&full[s]), (last_issue[s] / STAGES) & 1, globaltimer_ns() + 50000000ull, &never);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, t = 0;
      bool ok = true, issued = false;
      for (int w = blockIdx.x; w < works && ok; w += gridDim.x, ++t) {
        const int kb0 = (w % args.splits) * args.kb_split, kb1 = min(kbs, kb0 + args.kb_split);
        const int buf = t & 1;
        if (!tc::mbar_wait(tc::smem_u32(&tempty[buf]), ((t >> 1) & 1) ^ 1, globaltimer_ns() + args.timeout_ns,
                           s_abort)) {
          sfail(args, s_abort, GEMM_ERR_MMA | 0x10);
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t tmem_d = tmem_base + (uint32_t)(buf * TN);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!tc::mbar_wait(tc::smem_u32(&full[s]), ph, globaltimer_ns() + args.timeout_ns, s_abort)) {
            sfail(args, s_abort, GEMM_ERR_MMA | 0x11);
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t a0 = tc::smem_u32(sW + s * W_BYTES), b0 = tc::smem_u32(sX + s * X_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            tc::umma_f16(tmem_d, tc::sw128_kmajor_desc(a0 + k * 32), tc::sw128_kmajor_desc(b0 + k * 32), IDESC_S,
                         (kb != kb0) || (k != 0));
          issued = true;
          tc::umma_commit(tc::smem_u32(&empty[s]));
        }
        if (!ok) break;
        tc::umma_commit(tc::smem_u32(&tfull[buf]));
      }
      if ((!ok || *s_abort) && issued) {
        tc::umma_commit(tc::smem_u32(drain));
        int never = 0;
        tc::mbar_wait(tc::smem_u32(drain), 0, globaltimer_ns() + 50000000ull, &never);
      }
    }
  } else {
    const int q = warp & 3;
    const int nl = q * 32 + lane;  // weight row in the tile = TMEM lane = output column
    int t = 0;
    for (int w = blockIdx.x; w < works; w += gridDim.x, ++t) {
      const int tile = w / args.splits;
      const int buf = t & 1;
      if (!tc::mbar_wait(tc::smem_u32(&tfull[buf]), (t >> 1) & 1, globaltimer_ns() + args.timeout_ns, s_abort)) {
        sfail(args, s_abort, GEMM_ERR_EPI | 0x10);
        break;
      }
      tc::tc_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t)(buf * TN) + ((uint32_t)(q * 32) << 16);
      const int n = tile * BW + nl;
      if (args.splits > 1) {
        const int S = args.splits, sp = w - tile * S;
        float* mine = args.part + (((int64_t)tile * S + sp) * BW + nl) * TN;
#pragma unroll 1
        for (int c = 0; c < TN; c += 32) {
          uint32_t r[32];
          tc::tmem_ld_32x32b_x32(taddr + c, r);
          tc::tmem_wait_ld();
          tc::tmem_reg_fence(r);
          if (n < args.N) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              reinterpret_cast<uint4*>(mine + c)[j] = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
          }
        }
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (threadIdx.x == 64) {
          const int prev = atomicAdd(args.counters + tile, 1);
          s_last = (prev == S - 1);
          if (prev == S - 1) args.counters[tile] = 0;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (!s_last) {
          tc::tc_fence_before();
          tc::mbar_arrive(tc::smem_u32(&tempty[buf]));
          continue;
        }
        __threadfence();
        const float* p0 = args.part + ((int64_t)tile * S * BW + nl) * TN;
#pragma unroll 1
        for (int c = 0; c < TN; c += 32) {
          float acc[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[j] = 0.f;
          if (n < args.N) {
            for (int s2 = 0; s2 < S; ++s2) {
              const float4* src = reinterpret_cast<const float4*>(p0 + (int64_t)s2 * BW * TN + c);
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float4 x = __ldcg(src + j);
                acc[4 * j] += x.x;
                acc[4 * j + 1] += x.y;
                acc[4 * j + 2] += x.z;
                acc[4 * j + 3] += x.w;
              }
            }
          }
          uint32_t r[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(acc[j]);
          tc::tmem_st_32x32b_x32(taddr + c, r);
        }
        tc::tmem_wait_st();
      }
      // epilogue: column n of D for every token m
#pragma unroll 1
      for (int c = 0; c < TN; c += 32) {
        uint32_t r[32];
        tc::tmem_ld_32x32b_x32(taddr + c, r);
        tc::tmem_wait_ld();
        tc::tmem_reg_fence(r);
        if (n < args.N) {
#pragma unroll 4
          for (int j = 0; j < 32; ++j) {
            const int m = c + j;
            if (m < args.M) {
              float v = __uint_as_float(r[j]);
              if (args.R != nullptr) v = to_f32(from_f32<__nv_bfloat16>(v)) + to_f32(args.R[(int64_t)m * args.ldr + n]);
              args.D[(int64_t)m * args.ldd + n] = from_f32<__nv_bfloat16>(v);
            }
          }
        }
      }
      tc::tc_fence_before();
      tc::mbar_arrive(tc::smem_u32(&tempty[buf]));
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, TMEM_COLS_S);
  }
}

// Swapped-operand kernel for M <= 64 unless QFC_GEMM_SMALL=0.
bool small_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("QFC_GEMM_SMALL");
    return !(e && e[0] == '0');
  }();
  return on;
}

int* small_counters(int dev, int tiles) {
  constexpr int kMaxTiles = 1 << 14;
  static int* buf[64] = {nullptr};
  static std::mutex mu;
  TORCH_CHECK(tiles <= kMaxTiles, "gemm_small: too many tiles");
  std::lock_guard<std::mutex> lock(mu);
  if (buf[dev] == nullptr) {
    void* p = nullptr;
    C10_CUDA_CHECK(cudaMalloc(&p, kMaxTiles * sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(p, 0, kMaxTiles * sizeof(int)));
    buf[dev] = static_cast<int*>(p);
  }
  return buf[dev];
}

// out[M, N] = a[M, K] @ b[N, K]^T (+ residual), M <= 64.
void launch_small(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, const at::Tensor* R, double timeout_ms) {
  const int M = (int)a.size(0), K = (int)a.size(1), N = (int)b.size(0);
  const int dev = a.get_device();
  static std::atomic<unsigned long long> smem_set{0};
  C10_CUDA_CHECK(opt_in_smem_per_device(gemm_small_kernel, SMEM_BYTES_S, smem_set));
  SArgs s;
  std::memset(&s, 0, sizeof(s));
  s.M = M;
  s.N = N;
  s.K = K;
  s.n_tiles = (N + BW - 1) / BW;
  const int kbs = (K + BK - 1) / BK;
  const int sms = sm_count(dev);
  s.splits = 1;
  s.kb_split = kbs;
  at::Tensor part;
  if (s.n_tiles < sms && kbs >= 8) {
    const int S = std::min(sms / s.n_tiles, kbs / 4);
    if (S > 1) {
      s.kb_split = (kbs + S - 1) / S;
      s.splits = (kbs + s.kb_split - 1) / s.kb_split;
      part = at::empty({(int64_t)s.n_tiles * s.splits * BW * TN},
                       at::TensorOptions().dtype(at::kFloat).device(at::kCUDA, dev));
      s.part = part.data_ptr<float>();
      s.counters = small_counters(dev, s.n_tiles);
    }
  }
  s.D = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  s.ldd = (int)out.stride(0);
  s.R = R ? reinterpret_cast<const __nv_bfloat16*>(R->data_ptr()) : nullptr;
  s.ldr = R ? (int)R->stride(0) : 0;
  s.status = status_word();
  s.timeout_ns = (uint64_t)(timeout_ms * 1e6);
  const CUtensorMap tW = make_tmap(b.data_ptr(), N, K, b.stride(0), BW);
  const CUtensorMap tX = make_tmap(a.data_ptr(), M, K, a.stride(0), TN);
  const int grid = std::min(s.n_tiles * s.splits, sms);
  gemm_small_kernel<<<grid, NUM_THREADS, SMEM_BYTES_S, at::cuda::getCurrentCUDAStream()>>>(tW, tX, s);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace small
}  // namespace gemm

// gemv.cu: the weight-streaming kernel for M <= 8 (opt-in); false when it does not apply.
bool gemv_try(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, int64_t epi,
              const c10::optional<at::Tensor>& residual);

// out = a @ b^T (epi 0), silu(a @ gate^T) * (a @ up^T) with b = [gate; up] (epi 1),
// a @ b^T + residual (epi 2).
at::Tensor gemm_bf16(const at::Tensor& a, const at::Tensor& b, const c10::optional<at::Tensor>& out_opt, int64_t epi,
                     const c10::optional<at::Tensor>& residual, double timeout_ms, int64_t max_ctas) {
  using namespace gemm;
  check_operand(a, "a");
  check_operand(b, "b");
  TORCH_CHECK(a.size(1) == b.size(1), "gemm: K mismatch");
  const int M = (int)a.size(0), K = (int)a.size(1);
  int N = (int)b.size(0);
  if (epi == EPI_SWIGLU) {
    TORCH_CHECK(N % 2 == 0, "gemm(swiglu): b must stack gate and up rows");
    N /= 2;
  }
  c10::cuda::CUDAGuard guard(a.device());
  at::Tensor out = out_opt.has_value() ? *out_opt : at::empty({M, N}, a.options());
  check_operand(out, "out");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm: bad output shape");
  if (M == 0 || N == 0) return out;
  if (epi == EPI_RESIDUAL) {
    TORCH_CHECK(residual.has_value(), "gemm(residual): residual tensor required");
    check_operand(*residual, "residual");
    TORCH_CHECK(residual->size(0) == M && residual->size(1) == N, "gemm: bad residual shape");
  }
  if (max_ctas <= 0 && gemv_try(a, b, out, epi, residual)) return out;
  if (M <= small::TN && max_ctas <= 0 && (epi == EPI_STORE || epi == EPI_RESIDUAL) && small::small_enabled()) {
    small::launch_small(a, b, out, epi == EPI_RESIDUAL ? &*residual : nullptr, timeout_ms);
    return out;
  }
  switch (epi) {
    case EPI_STORE: launch<EPI_STORE>(a, b, &out, nullptr, M, N, K, timeout_ms, (int)max_ctas); break;
    case EPI_SWIGLU: launch<EPI_SWIGLU>(a, b, &out, nullptr, M, N, K, timeout_ms, (int)max_ctas); break;
    case EPI_RESIDUAL: launch<EPI_RESIDUAL>(a, b, &out, &*residual, M, N, K, timeout_ms, (int)max_ctas); break;
    default: TORCH_CHECK(false, "gemm: unknown epilogue ", epi);
  }
  return out;
}

// qkv = a @ w^T for a decoder layer's fused q/k/v projection (head_dim 128), with the
// rotary embedding of the q and k heads at positions pos [M] (int64) applied in the
// epilogue, and the k, v heads written to the paged caches at slots [M] (int64, < 0 = not
// cached) when k_cache / v_cache / slots are given.  Identical to gemm_bf16 + rope_kv.
void gemm_qkv_rope(const at::Tensor& a, const at::Tensor& w, at::Tensor& out, const at::Tensor& pos,
                   const at::Tensor& cos_sin, const c10::optional<at::Tensor>& k_cache,
                   const c10::optional<at::Tensor>& v_cache, const c10::optional<at::Tensor>& slots, int64_t nq,
                   int64_t nkv, double timeout_ms) {
  using namespace gemm;
  check_operand(a, "a");
  check_operand(w, "w");
  check_operand(out, "out");
  const int M = (int)a.size(0), K = (int)a.size(1), N = (int)w.size(0);
  TORCH_CHECK(w.size(1) == K && out.size(0) == M && out.size(1) == N, "gemm_qkv_rope: shape mismatch");
  TORCH_CHECK(N == (nq + 2 * nkv) * 128, "gemm_qkv_rope: head_dim 128 and w = [q; k; v] rows required");
  TORCH_CHECK(pos.scalar_type() == at::kLong && pos.numel() == M && pos.is_contiguous(), "gemm_qkv_rope: int64 pos [M]");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous() && cos_sin.dim() == 3 &&
                  cos_sin.size(1) == 64 && cos_sin.size(2) == 2,
              "gemm_qkv_rope: fp32 cos/sin table [max_position, 64, 2]");
  RopeArgs r;
  std::memset(&r, 0, sizeof(r));
  r.pos = pos.data_ptr<int64_t>();
  r.cs = reinterpret_cast<const float2*>(cos_sin.data_ptr());
  r.nq = (int)nq;
  r.nkv = (int)nkv;
  r.page = 1;
  r.page_shift = -1;
  const bool cache = slots.has_value() && slots->defined();
  if (cache) {
    TORCH_CHECK(k_cache.has_value() && v_cache.has_value(), "gemm_qkv_rope: caches required with slots");
    TORCH_CHECK(k_cache->dim() == 4 && k_cache->size(1) == nkv && k_cache->size(3) == 128 &&
                    k_cache->scalar_type() == at::kBFloat16 && k_cache->is_contiguous() &&
                    v_cache->sizes() == k_cache->sizes() && v_cache->is_contiguous(),
                "gemm_qkv_rope: bf16 caches [pages, nkv, page, 128]");
    TORCH_CHECK(slots->scalar_type() == at::kLong && slots->numel() == M && slots->is_contiguous(),
                "gemm_qkv_rope: int64 slots [M]");
    r.kc = reinterpret_cast<__nv_bfloat16*>(k_cache->data_ptr());
    r.vc = reinterpret_cast<__nv_bfloat16*>(v_cache->data_ptr());
    r.slots = slots->data_ptr<int64_t>();
    r.page = (int)k_cache->size(2);
    for (int sh = 0; sh < 31; ++sh)
      if ((1 << sh) == r.page) r.page_shift = sh;
  }
  c10::cuda::CUDAGuard guard(a.device());
  if (M == 0) return;
  launch<EPI_ROPE>(a, w, &out, nullptr, M, N, K, timeout_ms, 0, nullptr, &r);
}

// a @ b^T whose epilogue quantizes every 128-column group (p_bits 8 / 4, or 16 = raw
// bf16) and stores it into the owner rank's reduce-scatter slot described by sc.
void gemm_qscatter(const at::Tensor& a, const at::Tensor& b, const ScatterArgs& sc, int p_bits, double timeout_ms) {
  using namespace gemm;
  check_operand(a, "a");
  check_operand(b, "b");
  TORCH_CHECK(a.size(1) == b.size(1), "gemm: K mismatch");
  const int M = (int)a.size(0), K = (int)a.size(1), N = (int)b.size(0);
  TORCH_CHECK(N % 128 == 0 && sc.gs_shift == 7, "gemm_qscatter: group size 128 and N % 128 == 0 required");
  TORCH_CHECK(sc.chunk % 256 == 0, "gemm_qscatter: chunk must be a multiple of 256");
  c10::cuda::CUDAGuard guard(a.device());
  if (M == 0) return;
  switch (p_bits) {
    case 8: launch<EPI_QS8>(a, b, nullptr, nullptr, M, N, K, timeout_ms, 0, &sc); break;
    case 4: launch<EPI_QS4>(a, b, nullptr, nullptr, M, N, K, timeout_ms, 0, &sc); break;
    case 16: launch<EPI_QS16>(a, b, nullptr, nullptr, M, N, K, timeout_ms, 0, &sc); break;
    default: TORCH_CHECK(false, "gemm_qscatter: bits must be 8, 4 or 16");
  }
}

// Error word of the GEMM kernels (0 = ok); clear = reset it to 0.
int64_t gemm_status(bool clear) {
  volatile int* p = gemm::status_word();
  const int v = *p;
  if (clear) *p = 0;
  return v;
}

}  // namespace qfc
