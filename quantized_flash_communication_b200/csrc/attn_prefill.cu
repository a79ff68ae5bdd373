// Causal flash attention for prefill on sm_100a tensor cores (tcgen05 / TMEM / TMA).
//
// Replaces the attention of the reference's Hugging Face model (replicated on every rank,
// main.py:194).  Inputs come straight from the fused qkv activation [B*S, (nq + 2 nkv) hd]
// (after RoPE).  Q and K tiles are K-major operands (head dim contiguous); V tiles, loaded
// the same way, are the MN-major B operand of P V, so nothing is transposed.
//
// Persistent: one CTA per SM walks work items (a pair of adjacent 128-query tiles A and B
// of one head of one sequence), heaviest first.  Both tiles share every K / V tile load.
// 10 warps:
//   warp 0      TMA: Q_A and Q_B once per item, then K_j and V_j into 2-stage rings;
//   warp 1      TMEM allocation and MMA issue.  Per KV tile j the order is
//                 PV_A(j), S_A(j+1), PV_B(j), S_B(j+1)
//               with S = Q K_j^T (M = N = 128, K = hd) and O += P V_j (M = 128, N = hd,
//               K = 128) accumulated in TMEM, P read from TMEM as the A operand, so tile
//               A's softmax of j + 1 overlaps the tensor core's work on B and the other way
//               round (ping-pong);
//   warps 2-5   softmax of tile A, warps 6-9 softmax of tile B: thread = query row.  It
//               reads its S row from TMEM, masks (causal, sequence end), keeps the row's
//               reference maximum and sum, and writes P (bf16 pairs) back over the first 64
//               columns of its S row.
//               The reference maximum moves only when a new maximum exceeds it by more
//               than 2^8 (log2 domain); only then is the O row in TMEM rescaled, by the
//               same thread, before P is released.  After the last tile the thread reads
//               its O row, divides by the sum and stores bf16.
// TMEM (512 columns): S_A (then P_A) | S_B (then P_B) | O_A | O_B.  Shared memory: Q_A,
// Q_B, K[2], V[2] (6 x 32 KiB).  The tensor pipe runs one thread's MMAs in order, so S_t of
// tile j + 1 (issued after PV_t of tile j) never overwrites P_t before it is read, and the
// completion of S_t(j + 1) implies that of PV_t(j).  K / V tiles above the diagonal are
// skipped; tile A has one tile fewer than B.  Every mbarrier wait is bounded; on expiry the
// CTA records an error, drains its copies and MMAs and frees TMEM.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cfloat>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "smem_optin.h"
#include "tcgen05.cuh"

namespace qfc {
namespace attn {

constexpr int HD = 128;
constexpr int BQ = 128, BKV = 128;
constexpr int TILE_BYTES = 128 * 128 * 2;  // one 128 x 128 bf16 operand (two 64-column swizzle tiles)
constexpr int HALF_BYTES = TILE_BYTES / 2;
constexpr int NUM_THREADS = 320;
constexpr uint32_t IDESC = tc::idesc_f16(128, 128, true);           // S = Q K^T, both K-major
constexpr uint32_t IDESC_PV = tc::idesc_f16(128, 128, true, true);  // O = P V, V MN-major
// smem: Q[2] | K[2] | V[2] | barriers
constexpr int SMEM_BYTES = 6 * TILE_BYTES + 1024 + 2048;
// log2-domain growth of the row maximum tolerated before O is rescaled (P <= 2^8)
constexpr float kRescaleLog2 = 8.f;
// Every kPolyEvery-th pair of exponentials is evaluated on the FMA pipe (0: none), which
// balances the MUFU unit against the FMA pipe's other softmax work.
constexpr int kPolyEvery = 4;

struct Args {
  int B, S, nq, nkv, group;
  int q_tiles, q_pairs;
  float scale_log2;
  __nv_bfloat16* out;  // [B*S, nq*HD]
  int* status;
  uint64_t timeout_ns;
};

QFC_DEV void fail(const Args& a, volatile int* ab, int code) {
  *ab = 1;
  if (a.status) atomicCAS(a.status, 0, code);
}

QFC_DEV float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for x <= 0 on the FMA pipe, to share the softmax's exponentials with the MUFU unit.
// Range reduction to x = i + f with i = round(x), f in [-1/2, 1/2]: adding 1.5 * 2^23
// leaves i in the low mantissa bits of r (round to nearest), then 2^f is a cubic whose
// coefficients were fitted for this library to minimise the maximum relative error on
// [-1/2, 1/2] (Lawson's iteratively reweighted least squares, a standard route to the
// minimax polynomial); that error is 7.5e-5, far below the 2^-9 half-ulp of the bf16 P it
// feeds.  2^i enters by adding i to the exponent field.  x is clamped at -125, so masked
// scores (-inf) give 2^-125 instead of 0, which no bf16 sum can see.
constexpr float kEx2C0 = 0.99992812f, kEx2C1 = 0.69326097f, kEx2C2 = 0.24261054f, kEx2C3 = 0.05517132f;
QFC_DEV float ex2_poly(float x) {
  x = fmaxf(x, -125.f);
  const float r = x + 12582912.f;  // 1.5 * 2^23
  const float f = x - (r - 12582912.f);
  const float p = fmaf(fmaf(fmaf(kEx2C3, f, kEx2C2), f, kEx2C1), f, kEx2C0);
  return __int_as_float(__float_as_int(p) + (__float_as_int(r) << 23));
}

// ex2_poly on a pair, with the packed fp32 FMA / add of sm_100 (two lanes per instruction).
// Every lane performs the same roundings as ex2_poly: x - (r - M) is one fma(r', -1, x) of
// the exact r' = r - M, and the cubic is the same chain of fused multiply-adds.
QFC_DEV float2 ex2_poly2(float2 x) {
  x.x = fmaxf(x.x, -125.f);
  x.y = fmaxf(x.y, -125.f);
  const float2 r = __fadd2_rn(x, make_float2(12582912.f, 12582912.f));
  const float2 t = __fadd2_rn(r, make_float2(-12582912.f, -12582912.f));
  const float2 f = __ffma2_rn(t, make_float2(-1.f, -1.f), x);
  float2 p = __ffma2_rn(make_float2(kEx2C3, kEx2C3), f, make_float2(kEx2C2, kEx2C2));
  p = __ffma2_rn(p, f, make_float2(kEx2C1, kEx2C1));
  p = __ffma2_rn(p, f, make_float2(kEx2C0, kEx2C0));
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(r.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(r.y) << 23)));
}

__global__ void exp2_poly_kernel(const float* x, float* y, int64_t n, bool pairs) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (!pairs) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) y[i] = ex2_poly(x[i]);
    return;
  }
  // elements 2k and 2k + 1 as the two lanes of ex2_poly2
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; 2 * k < n; k += stride) {
    const bool two = 2 * k + 1 < n;
    const float2 r = ex2_poly2(make_float2(x[2 * k], two ? x[2 * k + 1] : 0.f));
    y[2 * k] = r.x;
    if (two) y[2 * k + 1] = r.y;
  }
}

// Work item i -> (query tile pair, head, sequence); heaviest (last) pairs first.
QFC_DEV void item_coords(int i, const Args& a, int& pr, int& h, int& b) {
  const int per_pair = a.nq * a.B;
  pr = a.q_pairs - 1 - i / per_pair;
  const int r = i % per_pair;
  h = r % a.nq;
  b = r / a.nq;
}

// KV tiles of the pair's two query tiles (A = 2 pr, B = 2 pr + 1; B is empty past S).
QFC_DEV void item_tiles(int pr, const Args& a, int kv_tiles, int& na, int& nb) {
  const int qa = 2 * pr, qb = 2 * pr + 1;
  na = min(qa + 1, kv_tiles);
  nb = (qb < a.q_tiles) ? min(qb + 1, kv_tiles) : 0;
}

// PACKED: the softmax's scale-and-subtract, row sums and FMA-pipe exponentials use the
// packed two-lane fp32 instructions (half the issue slots for that arithmetic); P is
// bit-identical, the row sum l is added in another order.
template <bool PACKED>
__global__ void __launch_bounds__(NUM_THREADS, 1)
attn_prefill_kernel(const __grid_constant__ CUtensorMap tmQKV, const Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                    // [2]: A, B
  uint8_t* sK = smem + 2 * TILE_BYTES;   // [2] ring
  uint8_t* sV = smem + 4 * TILE_BYTES;   // [2] ring
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * TILE_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;    // [2]
  uint64_t* k_empty = bars + 4;   // [2]
  uint64_t* v_full = bars + 6;    // [2]
  uint64_t* v_empty = bars + 8;   // [2]
  uint64_t* s_full = bars + 10;   // [2] per query tile
  uint64_t* p_full = bars + 12;   // [2]
  uint64_t* o_done = bars + 14;   // [2] the last issued PV of the tile is complete
  uint64_t* o_empty = bars + 16;  // [2] the final O of the item has been read
  uint64_t* drain = bars + 18;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 19);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = args.q_pairs * args.nq * args.B;
  const int kv_tiles = (args.S + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    tc::mbar_init(tc::smem_u32(q_full), 1);
    tc::mbar_init(tc::smem_u32(q_empty), 1);
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(tc::smem_u32(&k_full[i]), 1);
      tc::mbar_init(tc::smem_u32(&k_empty[i]), 1);
      tc::mbar_init(tc::smem_u32(&v_full[i]), 1);
      tc::mbar_init(tc::smem_u32(&v_empty[i]), 1);
      tc::mbar_init(tc::smem_u32(&s_full[i]), 1);
      tc::mbar_init(tc::smem_u32(&p_full[i]), 128);
      tc::mbar_init(tc::smem_u32(&o_done[i]), 1);
      tc::mbar_init(tc::smem_u32(&o_empty[i]), 128);
    }
    tc::mbar_init(tc::smem_u32(drain), 1);
    *s_abort = 0;
    tc::fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tc::smem_u32(tmem_holder), 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_holder;  // S_A = +0, S_B = +128, O_A = +256, O_B = +384
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    return tc::mbar_wait(tc::smem_u32(bar), parity, globaltimer_ns() + args.timeout_ns, s_abort);
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tc::tma_prefetch_desc(&tmQKV);
      int tk = 0, k = 0;  // KV tiles loaded (all items), items started
      int k_issued[2] = {-1, -1}, v_issued[2] = {-1, -1}, q_issued = -1;
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++k) {
        int pr, h, b, na, nb;
        item_coords(item, args, pr, h, b);
        item_tiles(pr, args, kv_tiles, na, nb);
        const int n_kv = max(na, nb);
        const int kvh = h / args.group;
        const int row_base = b * args.S;
        if (!wait(q_empty, (k & 1) ^ 1)) {
          fail(args, s_abort, 0x1001);
          break;
        }
        const uint32_t qb = tc::smem_u32(q_full);
        tc::mbar_arrive_expect_tx(qb, 2 * TILE_BYTES);
        for (int t = 0; t < 2; ++t) {  // rows past the batch's end read as zero; unused rows are masked
          const int qrow = row_base + (2 * pr + t) * BQ;
          tc::tma_load_2d(tc::smem_u32(sQ + t * TILE_BYTES), &tmQKV, qb, h * HD, qrow);
          tc::tma_load_2d(tc::smem_u32(sQ + t * TILE_BYTES + HALF_BYTES), &tmQKV, qb, h * HD + 64, qrow);
        }
        q_issued = k;
        const int kcol = (args.nq + kvh) * HD, vcol = (args.nq + args.nkv + kvh) * HD;
        for (int j = 0; j < n_kv; ++j, ++tk) {
          const int st = tk & 1;
          if (!wait(&k_empty[st], ((tk >> 1) & 1) ^ 1)) {
            fail(args, s_abort, 0x1002);
            ok = false;
            break;
          }
          const uint32_t fb = tc::smem_u32(&k_full[st]);
          tc::mbar_arrive_expect_tx(fb, TILE_BYTES);
          tc::tma_load_2d(tc::smem_u32(sK + st * TILE_BYTES), &tmQKV, fb, kcol, row_base + j * BKV);
          tc::tma_load_2d(tc::smem_u32(sK + st * TILE_BYTES + HALF_BYTES), &tmQKV, fb, kcol + 64, row_base + j * BKV);
          k_issued[st] = tk;
          if (!wait(&v_empty[st], ((tk >> 1) & 1) ^ 1)) {
            fail(args, s_abort, 0x1003);
            ok = false;
            break;
          }
          const uint32_t vb = tc::smem_u32(&v_full[st]);
          tc::mbar_arrive_expect_tx(vb, TILE_BYTES);
          tc::tma_load_2d(tc::smem_u32(sV + st * TILE_BYTES), &tmQKV, vb, vcol, row_base + j * BKV);
          tc::tma_load_2d(tc::smem_u32(sV + st * TILE_BYTES + HALF_BYTES), &tmQKV, vb, vcol + 64, row_base + j * BKV);
          v_issued[st] = tk;
        }
      }
      if (*s_abort) {  // let issued copies land before shared memory goes away
        int never = 0;
        if (q_issued >= 0) tc::mbar_wait(tc::smem_u32(q_full), q_issued & 1, globaltimer_ns() + 50000000ull, &never);
        for (int st = 0; st < 2; ++st) {
          if (k_issued[st] >= 0)
            tc::mbar_wait(tc::smem_u32(&k_full[st]), (k_issued[st] >> 1) & 1, globaltimer_ns() + 50000000ull, &never);
          if (v_issued[st] >= 0)
            tc::mbar_wait(tc::smem_u32(&v_full[st]), (v_issued[st] >> 1) & 1, globaltimer_ns() + 50000000ull, &never);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      bool ok = true, issued_any = false;
      int tk = 0, k = 0;
      int ns[2] = {0, 0};  // S MMAs issued per query tile (all items)
      int np[2] = {0, 0};  // PV MMAs issued per query tile
      int ni[2] = {0, 0};  // items started per query tile
      // S_t = Q_t K^T for the KV tile with counter j_tk.  Its columns held P_t of the previous
      // tile, whose PV was issued before: the in-order tensor pipe reads P first.
      auto issue_s = [&](int t, int j_tk) -> bool {
        tc::tc_fence_after();
        const uint32_t a0 = tc::smem_u32(sQ + t * TILE_BYTES), b0 = tc::smem_u32(sK + (j_tk & 1) * TILE_BYTES);
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc::umma_f16(tmem + t * 128, tc::sw128_kmajor_desc(a0 + s * HALF_BYTES + kk * 32),
                         tc::sw128_kmajor_desc(b0 + s * HALF_BYTES + kk * 32), IDESC, (s | kk) != 0);
        tc::umma_commit(tc::smem_u32(&s_full[t]));
        ++ns[t];
        issued_any = true;
        return true;
      };
      auto issue_pv = [&](int t, bool first, int v_tk) -> bool {  // O_t (+)= P_t V
        if (!wait(&p_full[t], np[t] & 1)) return false;
        if (first && !wait(&o_empty[t], (ni[t] & 1) ^ 1)) return false;
        tc::tc_fence_after();
        const uint32_t b0 = tc::smem_u32(sV + (v_tk & 1) * TILE_BYTES);
        // P: TMEM columns t*128 + 8 i hold keys 16 i .. 16 i + 15.  V: MN-major as loaded
        // (rows = keys, 64 head dims per 128-byte row, the second 64 dims HALF_BYTES later);
        // 16 keys = 2048 bytes per MMA.
#pragma unroll
        for (int i = 0; i < 8; ++i)
          tc::umma_f16_ts(tmem + 256 + t * 128, tmem + t * 128 + i * 8,
                          tc::sw128_mnmajor_desc(b0 + i * 2048, HALF_BYTES), IDESC_PV, !first || i != 0);
        tc::umma_commit(tc::smem_u32(&o_done[t]));
        ++np[t];
        if (first) ++ni[t];
        issued_any = true;
        return true;
      };
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++k) {
        int pr, h, b, na, nb;
        item_coords(item, args, pr, h, b);
        item_tiles(pr, args, kv_tiles, na, nb);
        const int n_kv = max(na, nb);
        const int nt[2] = {na, nb};
        if (!wait(q_full, k & 1) || !wait(&k_full[tk & 1], (tk >> 1) & 1)) {
          ok = false;
          break;
        }
        // prologue: S of KV tile 0 for both query tiles
        for (int t = 0; t < 2 && ok; ++t)
          if (nt[t] > 0 && !issue_s(t, tk)) ok = false;
        if (!ok) break;
        tc::umma_commit(tc::smem_u32(&k_empty[tk & 1]));
        if (n_kv == 1) tc::umma_commit(tc::smem_u32(q_empty));
        for (int j = 0; j < n_kv && ok; ++j) {
          const int cur = tk + j;
          const bool more = j + 1 < n_kv;
          if (!wait(&v_full[cur & 1], (cur >> 1) & 1)) {
            ok = false;
            break;
          }
          bool k_ready = false;  // K_{j+1} is waited for only right before its first use
          for (int t = 0; t < 2 && ok; ++t) {
            if (j < nt[t] && !issue_pv(t, j == 0, cur)) ok = false;
            if (ok && more && j + 1 < nt[t]) {
              if (!k_ready && !wait(&k_full[(cur + 1) & 1], ((cur + 1) >> 1) & 1)) ok = false;
              k_ready = true;
              if (ok && !issue_s(t, cur + 1)) ok = false;
            }
          }
          if (!ok) break;
          tc::umma_commit(tc::smem_u32(&v_empty[cur & 1]));  // V free once both PV MMAs are done
          if (more) {
            tc::umma_commit(tc::smem_u32(&k_empty[(cur + 1) & 1]));
            if (j + 2 == n_kv) tc::umma_commit(tc::smem_u32(q_empty));  // the item's last S MMAs
          }
        }
        tk += n_kv;
      }
      if (!ok) fail(args, s_abort, 0x2001);
      if ((!ok || *s_abort) && issued_any) {
        tc::umma_commit(tc::smem_u32(drain));
        int never = 0;
        tc::mbar_wait(tc::smem_u32(drain), 0, globaltimer_ns() + 50000000ull, &never);
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax (tile A or B)
    const int t = (warp - 2) >> 2;             // 0: query tile A (warps 2-5), 1: B (warps 6-9)
    const int r = (warp & 3) * 32 + lane;      // query row in the tile (= TMEM lane)
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t s_col = tmem + lane_off + t * 128, o_col = tmem + lane_off + 256 + t * 128;
    int n = 0;  // tiles processed by this query tile (all items)
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      int pr, h, b, na, nb;
      item_coords(item, args, pr, h, b);
      item_tiles(pr, args, kv_tiles, na, nb);
      const int my_n = t == 0 ? na : nb;
      if (my_n == 0) continue;
      const int qpos = (2 * pr + t) * BQ + r;
      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j < my_n; ++j, ++n) {
        if (!wait(&s_full[t], n & 1)) {
          fail(args, s_abort, 0x3001);
          ok = false;
          break;
        }
        tc::tc_fence_after();
        float sv[128];
        {
          uint32_t u[4][32];
#pragma unroll
          for (int c = 0; c < 4; ++c) tc::tmem_ld_32x32b_x32(s_col + c * 32, u[c]);
          tc::tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            tc::tmem_reg_fence(u[c]);
#pragma unroll
            for (int i = 0; i < 32; ++i) sv[c * 32 + i] = __uint_as_float(u[c][i]);
          }
        }
        // columns past kmax are masked: keys above the diagonal or past the sequence end
        const int kmax = min(qpos, args.S - 1) - j * BKV;
        if (kmax < BKV - 1) {
#pragma unroll
          for (int i = 0; i < 128; ++i) sv[i] = (i <= kmax) ? sv[i] : -INFINITY;
        }
        float mx4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
        for (int i = 4; i < 128; i += 4) {
#pragma unroll
          for (int q = 0; q < 4; ++q) mx4[q] = fmaxf(mx4[q], sv[i + q]);
        }
        const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * args.scale_log2;
        // S of this tile completed after the previous PV of this tile (in-order tensor pipe),
        // so O holds every earlier tile and may be rescaled here.
        float alpha = 1.f;
        const bool move = j == 0 || mx > m_ref + kRescaleLog2;
        if (move) {
          const float m_new = fmaxf(m_ref, mx);
          const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
          if (j > 0) alpha = ex2(m_ref - m_use);
          m_ref = m_use;
        }
        // O rows *= alpha, in TMEM.  tcgen05.ld / st are warp-collective, so the whole warp
        // rescales when any of its rows moved its maximum (the others multiply by 1).
        if (j > 0 && __any_sync(QFC_FULL_MASK, move)) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t u[32];
            tc::tmem_ld_32x32b_x32(o_col + c * 32, u);
            tc::tmem_wait_ld();
            tc::tmem_reg_fence(u);
#pragma unroll
            for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * alpha);
            tc::tmem_st_32x32b_x32(o_col + c * 32, u);
          }
          tc::tmem_wait_st();
        }
        float sum4[4] = {0.f, 0.f, 0.f, 0.f};
        float2 sum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        const float2 sc2 = make_float2(args.scale_log2, args.scale_log2);
        const float2 nm2 = make_float2(-m_ref, -m_ref);
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // 4 chunks of 32 keys -> 16 TMEM columns of bf16 pairs
          uint32_t w[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            // one pair in kPolyEvery on the FMA pipe, the rest on MUFU
            const bool poly = kPolyEvery > 0 && (q % kPolyEvery) == kPolyEvery - 1;
            float p0, p1;
            if constexpr (PACKED) {
              const float2 a = __ffma2_rn(make_float2(sv[c * 32 + 2 * q], sv[c * 32 + 2 * q + 1]), sc2, nm2);
              const float2 pp = poly ? ex2_poly2(a) : make_float2(ex2(a.x), ex2(a.y));
              sum2[q & 1] = __fadd2_rn(sum2[q & 1], pp);
              p0 = pp.x;
              p1 = pp.y;
            } else {
              const float a0 = fmaf(sv[c * 32 + 2 * q], args.scale_log2, -m_ref);
              const float a1 = fmaf(sv[c * 32 + 2 * q + 1], args.scale_log2, -m_ref);
              p0 = poly ? ex2_poly(a0) : ex2(a0);
              p1 = poly ? ex2_poly(a1) : ex2(a1);
              sum4[q & 3] += p0 + p1;
            }
            w[q] = pack_bf16x2(p0, p1);  // key 2q in the low half
          }
          tc::tmem_st_32x32b_x16(s_col + c * 16, w);
        }
        tc::tmem_wait_st();
        tc::tc_fence_before();
        if constexpr (PACKED) l = l * alpha + ((sum2[0].x + sum2[1].x) + (sum2[0].y + sum2[1].y));
        else l = l * alpha + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
        tc::mbar_arrive(tc::smem_u32(&p_full[t]));
      }
      if (!ok) break;
      // the item's last PV is done: O / l to global memory, then O's columns are free
      if (!wait(&o_done[t], (n - 1) & 1)) {
        fail(args, s_abort, 0x3003);
        break;
      }
      tc::tc_fence_after();
      uint32_t u[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tc::tmem_ld_32x32b_x32(o_col + c * 32, u[c]);
      tc::tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 4; ++c) tc::tmem_reg_fence(u[c]);
      tc::tc_fence_before();
      tc::mbar_arrive(tc::smem_u32(&o_empty[t]));
      if (qpos < args.S) {
        const float inv = 1.f / l;
        __nv_bfloat16* dst = args.out + (int64_t)(b * args.S + qpos) * (args.nq * HD) + h * HD;
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t* x = &u[c][8 * q];
            const uint4 v = make_uint4(pack_bf16x2(__uint_as_float(x[0]) * inv, __uint_as_float(x[1]) * inv),
                                       pack_bf16x2(__uint_as_float(x[2]) * inv, __uint_as_float(x[3]) * inv),
                                       pack_bf16x2(__uint_as_float(x[4]) * inv, __uint_as_float(x[5]) * inv),
                                       pack_bf16x2(__uint_as_float(x[6]) * inv, __uint_as_float(x[7]) * inv));
            reinterpret_cast<uint4*>(dst)[c * 4 + q] = v;
          }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p != nullptr,
                "attn: cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

CUtensorMap make_map(const void* ptr, int64_t rows, int64_t cols, int64_t ld) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "attn: cuTensorMapEncodeTiled failed (", (int)r, ")");
  return m;
}

int* status_word() {
  static int* p = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* hptr = nullptr;
    TORCH_CHECK(cudaHostAlloc(&hptr, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable) == cudaSuccess,
                "attn: cudaHostAlloc(status) failed");
    *reinterpret_cast<volatile int*>(hptr) = 0;
    p = reinterpret_cast<int*>(hptr);
  });
  return p;
}

// The packed-arithmetic softmax (attn_prefill_kernel<true>) is off unless QFC_ATTN_PACKED=1
// or set_attn_packed(true): it has to win a measurement before it becomes the default.
std::atomic<bool>& packed_flag() {
  static std::atomic<bool> on{[] {
    const char* e = std::getenv("QFC_ATTN_PACKED");
    return e != nullptr && e[0] == '1';
  }()};
  return on;
}

}  // namespace attn

bool set_attn_packed(bool on) { return attn::packed_flag().exchange(on); }

// qkv [B*S, (nq + 2 nkv) * 128] bf16 (RoPE applied) -> out [B*S, nq * 128] bf16, causal.
void attn_prefill_cuda(const at::Tensor& qkv, at::Tensor& out, int64_t B, int64_t S, int64_t nq, int64_t nkv,
                       int64_t hd, double scale) {
  using namespace attn;
  TORCH_CHECK(hd == HD, "attn_prefill: head_dim must be 128");
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16, "attn_prefill: bf16 only");
  TORCH_CHECK(qkv.is_contiguous() && out.is_contiguous(), "attn_prefill: contiguous tensors");
  TORCH_CHECK(nq % nkv == 0, "attn_prefill: nq must be a multiple of nkv");
  TORCH_CHECK(qkv.size(0) == B * S && qkv.size(1) == (nq + 2 * nkv) * HD, "attn_prefill: bad qkv shape");
  if (B == 0 || S == 0) return;
  c10::cuda::CUDAGuard guard(qkv.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  static std::atomic<unsigned long long> smem_set{0}, smem_set_packed{0};
  const int dev = qkv.get_device();
  const bool packed = packed_flag().load(std::memory_order_relaxed);
  if (packed) C10_CUDA_CHECK(opt_in_smem_per_device(attn_prefill_kernel<true>, SMEM_BYTES, smem_set_packed));
  else C10_CUDA_CHECK(opt_in_smem_per_device(attn_prefill_kernel<false>, SMEM_BYTES, smem_set));
  const CUtensorMap tq = make_map(qkv.data_ptr(), B * S, (nq + 2 * nkv) * HD, (nq + 2 * nkv) * HD);
  Args a;
  a.B = (int)B;
  a.S = (int)S;
  a.nq = (int)nq;
  a.nkv = (int)nkv;
  a.group = (int)(nq / nkv);
  a.q_tiles = (int)((S + BQ - 1) / BQ);
  a.q_pairs = (a.q_tiles + 1) / 2;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.status = status_word();
  a.timeout_ns = 10000000000ull;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t items = (int64_t)a.q_pairs * nq * B;
  const int grid = (int)std::min<int64_t>(items, sms);
  if (packed) attn_prefill_kernel<true><<<grid, NUM_THREADS, SMEM_BYTES, st>>>(tq, a);
  else attn_prefill_kernel<false><<<grid, NUM_THREADS, SMEM_BYTES, st>>>(tq, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// y = 2^x through the softmax's FMA-pipe exponential (for tests against exp2f); pairs: the
// packed two-lane form used by the packed softmax.
void attn_exp2_poly(const at::Tensor& x, at::Tensor& y, bool pairs) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.is_contiguous() && y.sizes() == x.sizes() &&
                  y.scalar_type() == at::kFloat && y.is_contiguous(), "attn_exp2_poly: fp32 CUDA tensors");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t n = x.numel();
  if (n == 0) return;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
  attn::exp2_poly_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(x.data_ptr<float>(),
                                                                               y.data_ptr<float>(), n, pairs);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t attn_status(bool clear) {
  volatile int* p = attn::status_word();
  const int v = *p;
  if (clear) *p = 0;
  return v;
}

}  // namespace qfc
