// Causal flash attention for prefill on sm_100a tensor cores (tcgen05 / TMEM / TMA).
//
// Replaces the attention of the reference's Hugging Face model (replicated on every rank,
// main.py:194).  Inputs come straight from the fused qkv activation [B*S, (nq + 2 nkv) hd]
// (after RoPE).  Q and K tiles are K-major operands (head dim contiguous); V tiles, loaded
// the same way, are the MN-major B operand of P V, so nothing is transposed.
//
// Persistent: one CTA per SM walks (128-query tile, query head, sequence) work items,
// heaviest first; 10 warps:
//   warp 0      TMA: Q once, then K_j and V^T_j into a 2-stage ring;
//   warp 1      TMEM allocation and MMA issue: S_j = Q K_j^T (M=N=128, K=hd) into one of two
//               TMEM S buffers, then O_j = P_j V_j (M=128, N=hd, K=128) into one of two
//               TMEM O buffers (fresh accumulation per tile);
//   warps 2-5   softmax: thread = query row; reads its S row from TMEM, applies the causal
//               and sequence-end masks, keeps the running max / sum, writes P_j (bf16) into
//               swizzled shared memory for the next MMA and the rescale factor alpha_j;
//   warps 6-9   correction: thread = query row; O += alpha_j * O + O_j in registers, and the
//               final O / l to global memory.
// K/V tiles above the diagonal are skipped.  Every mbarrier wait is bounded.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>

#include <cfloat>
#include <mutex>

#include "common.cuh"
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
// smem: Q | K[2] | Vt[2] | P[2] | barriers + alpha/l
constexpr int SMEM_BYTES = 7 * TILE_BYTES + 1024 + 2048;

struct Args {
  int B, S, nq, nkv, group;
  int q_tiles;
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

QFC_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Byte offset of the 16-byte chunk `c` (0..7) of row `r` inside a 128-byte-swizzled
// K-major tile of 64 bf16 columns: rows are 128 bytes, chunk index XOR (row mod 8).
QFC_DEV uint32_t sw128_off(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// Work item i -> (query tile, head, sequence); heaviest (last) query tiles first.
QFC_DEV void item_coords(int i, const Args& a, int& qt, int& h, int& b) {
  const int per_tile = a.nq * a.B;
  qt = a.q_tiles - 1 - i / per_tile;
  const int r = i % per_tile;
  h = r % a.nq;
  b = r / a.nq;
}

// Persistent: each CTA walks work items blockIdx.x, +gridDim.x, ...  Every role walks
// the same items, and a global tile counter t (over all items of this CTA) selects the
// ring slot (t & 1) and mbarrier phase ((t >> 1) & 1) of every double buffer.
__global__ void __launch_bounds__(NUM_THREADS, 1)
attn_prefill_kernel(const __grid_constant__ CUtensorMap tmQKV, const Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + TILE_BYTES;          // 2 stages
  uint8_t* sV = smem + 3 * TILE_BYTES;      // 2 stages
  uint8_t* sP = smem + 5 * TILE_BYTES;      // 2 buffers
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 7 * TILE_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_empty = bars + 7;   // [2]
  uint64_t* p_full = bars + 9;    // [2]
  uint64_t* p_empty = bars + 11;  // [2]
  uint64_t* o_full = bars + 13;   // [2]
  uint64_t* o_empty = bars + 15;  // [2]
  uint64_t* drain = bars + 17;
  uint64_t* a_empty = bars + 18;  // [2] correction has read alpha / l of this buffer
  uint64_t* q_empty = bars + 20;  // all QK MMAs of the current item are done with Q
  uint64_t* v_full = bars + 21;   // [2] V^T tile landed (kv_full / kv_empty track K)
  uint64_t* v_empty = bars + 23;  // [2] PV MMA done with V^T
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 25);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* s_alpha = reinterpret_cast<float*>(tmem_holder + 4);  // [2][128]
  float* s_l = s_alpha + 256;                                   // [2][128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = args.q_tiles * args.nq * args.B;
  const int kv_tiles = (args.S + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    tc::mbar_init(tc::smem_u32(q_full), 1);
    tc::mbar_init(tc::smem_u32(q_empty), 1);
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(tc::smem_u32(&kv_full[i]), 1);
      tc::mbar_init(tc::smem_u32(&kv_empty[i]), 1);
      tc::mbar_init(tc::smem_u32(&s_full[i]), 1);
      tc::mbar_init(tc::smem_u32(&s_empty[i]), 128);
      tc::mbar_init(tc::smem_u32(&p_full[i]), 128);
      tc::mbar_init(tc::smem_u32(&p_empty[i]), 1);
      tc::mbar_init(tc::smem_u32(&o_full[i]), 1);
      tc::mbar_init(tc::smem_u32(&o_empty[i]), 128);
      tc::mbar_init(tc::smem_u32(&a_empty[i]), 128);
      tc::mbar_init(tc::smem_u32(&v_full[i]), 1);
      tc::mbar_init(tc::smem_u32(&v_empty[i]), 1);
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
  const uint32_t tmem = *tmem_holder;  // S[0]=+0, S[1]=+128, O[0]=+256, O[1]=+384
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    return tc::mbar_wait(tc::smem_u32(bar), parity, globaltimer_ns() + args.timeout_ns, s_abort);
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tc::tma_prefetch_desc(&tmQKV);
      int t = 0, k = 0;
      int issued[2] = {-1, -1}, v_issued[2] = {-1, -1}, q_issued = -1;
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++k) {
        int qt, h, b;
        item_coords(item, args, qt, h, b);
        const int kvh = h / args.group;
        const int row_base = b * args.S;
        const int n_kv = min(qt + 1, kv_tiles);
        if (!wait(q_empty, (k & 1) ^ 1)) {
          fail(args, s_abort, 0x1002);
          break;
        }
        const uint32_t qb = tc::smem_u32(q_full);
        tc::mbar_arrive_expect_tx(qb, TILE_BYTES);
        tc::tma_load_2d(tc::smem_u32(sQ), &tmQKV, qb, h * HD, row_base + qt * BQ);
        tc::tma_load_2d(tc::smem_u32(sQ + HALF_BYTES), &tmQKV, qb, h * HD + 64, row_base + qt * BQ);
        q_issued = k;
        for (int j = 0; j < n_kv; ++j, ++t) {
          const int st = t & 1;
          if (!wait(&kv_empty[st], ((t >> 1) & 1) ^ 1)) {
            fail(args, s_abort, 0x1001);
            ok = false;
            break;
          }
          const uint32_t fb = tc::smem_u32(&kv_full[st]);
          tc::mbar_arrive_expect_tx(fb, TILE_BYTES);
          const int kcol = (args.nq + kvh) * HD;
          tc::tma_load_2d(tc::smem_u32(sK + st * TILE_BYTES), &tmQKV, fb, kcol, row_base + j * BKV);
          tc::tma_load_2d(tc::smem_u32(sK + st * TILE_BYTES + HALF_BYTES), &tmQKV, fb, kcol + 64, row_base + j * BKV);
          issued[st] = t;
          // V^T of this tile: its slot frees later (after PV), so it is loaded second
          if (!wait(&v_empty[st], ((t >> 1) & 1) ^ 1)) {
            fail(args, s_abort, 0x1003);
            ok = false;
            break;
          }
          const uint32_t vb = tc::smem_u32(&v_full[st]);
          tc::mbar_arrive_expect_tx(vb, TILE_BYTES);
          const int vcol = (args.nq + args.nkv + kvh) * HD;
          tc::tma_load_2d(tc::smem_u32(sV + st * TILE_BYTES), &tmQKV, vb, vcol, row_base + j * BKV);
          tc::tma_load_2d(tc::smem_u32(sV + st * TILE_BYTES + HALF_BYTES), &tmQKV, vb, vcol + 64, row_base + j * BKV);
          v_issued[st] = t;
        }
      }
      if (*s_abort) {  // let issued copies land before shared memory goes away
        int never = 0;
        if (q_issued >= 0) tc::mbar_wait(tc::smem_u32(q_full), q_issued & 1, globaltimer_ns() + 50000000ull, &never);
        for (int st = 0; st < 2; ++st) {
          if (issued[st] >= 0)
            tc::mbar_wait(tc::smem_u32(&kv_full[st]), (issued[st] >> 1) & 1, globaltimer_ns() + 50000000ull, &never);
          if (v_issued[st] >= 0)
            tc::mbar_wait(tc::smem_u32(&v_full[st]), (v_issued[st] >> 1) & 1, globaltimer_ns() + 50000000ull, &never);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      bool ok = true, issued_any = false;
      int t = 0, k = 0;
      auto issue_qk = [&](int tt) -> bool {
        const int st = tt & 1;
        if (!wait(&kv_full[st], (tt >> 1) & 1) || !wait(&s_empty[st], ((tt >> 1) & 1) ^ 1)) return false;
        tc::tc_fence_after();
        const uint32_t a0 = tc::smem_u32(sQ), b0 = tc::smem_u32(sK + st * TILE_BYTES);
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc::umma_f16(tmem + st * 128, tc::sw128_kmajor_desc(a0 + s * HALF_BYTES + kk * 32),
                         tc::sw128_kmajor_desc(b0 + s * HALF_BYTES + kk * 32), IDESC, (s | kk) != 0);
        tc::umma_commit(tc::smem_u32(&s_full[st]));
        tc::umma_commit(tc::smem_u32(&kv_empty[st]));  // K slot free once this QK is done
        issued_any = true;
        return true;
      };
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++k) {
        int qt, h, b;
        item_coords(item, args, qt, h, b);
        const int n_kv = min(qt + 1, kv_tiles);
        if (!wait(q_full, k & 1) || !issue_qk(t)) {
          ok = false;
          break;
        }
        for (int j = 0; j < n_kv; ++j, ++t) {
          const int st = t & 1;
          if (j + 1 < n_kv) {
            if (!issue_qk(t + 1)) {
              ok = false;
              break;
            }
          } else {
            tc::umma_commit(tc::smem_u32(q_empty));  // Q free once this item's QK MMAs are done
          }
          if (!wait(&p_full[st], (t >> 1) & 1) || !wait(&o_empty[st], ((t >> 1) & 1) ^ 1) ||
              !wait(&v_full[st], (t >> 1) & 1)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t a0 = tc::smem_u32(sP + st * TILE_BYTES), b0 = tc::smem_u32(sV + st * TILE_BYTES);
          // P: K-major, keys split in two 64-key swizzle tiles.  V: MN-major as loaded
          // (rows = keys, 64 head dims per 128-byte row, second 64 dims HALF_BYTES later);
          // 16 keys = 2048 bytes per MMA.
#pragma unroll
          for (int s = 0; s < 2; ++s)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc::umma_f16(tmem + 256 + st * 128, tc::sw128_kmajor_desc(a0 + s * HALF_BYTES + kk * 32),
                           tc::sw128_mnmajor_desc(b0 + (s * 4 + kk) * 2048, HALF_BYTES), IDESC_PV, (s | kk) != 0);
          tc::umma_commit(tc::smem_u32(&o_full[st]));
          tc::umma_commit(tc::smem_u32(&p_empty[st]));
          tc::umma_commit(tc::smem_u32(&v_empty[st]));
        }
      }
      if (!ok) fail(args, s_abort, 0x2001);
      if ((!ok || *s_abort) && issued_any) {
        tc::umma_commit(tc::smem_u32(drain));
        int never = 0;
        tc::mbar_wait(tc::smem_u32(drain), 0, globaltimer_ns() + 50000000ull, &never);
      }
    }
  } else if (warp < 6) {
    // ---------------------------------------------------------------- softmax
    const int r = (warp & 3) * 32 + lane;  // query row in the tile (= TMEM lane)
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    int t = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      int qt, h, b;
      item_coords(item, args, qt, h, b);
      const int n_kv = min(qt + 1, kv_tiles);
      const int qpos = qt * BQ + r;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < n_kv; ++j, ++t) {
        const int st = t & 1;
        if (!wait(&s_full[st], (t >> 1) & 1)) {
          fail(args, s_abort, 0x3001);
          ok = false;
          break;
        }
        tc::tc_fence_after();
        float sv[128];
        {
          uint32_t u[4][32];
#pragma unroll
          for (int c = 0; c < 4; ++c) tc::tmem_ld_32x32b_x32(tmem + st * 128 + lane_off + c * 32, u[c]);
          tc::tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            tc::tmem_reg_fence(u[c]);
#pragma unroll
            for (int i = 0; i < 32; ++i) sv[c * 32 + i] = __uint_as_float(u[c][i]);
          }
        }
        tc::tc_fence_before();
        tc::mbar_arrive(tc::smem_u32(&s_empty[st]));
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
        const float m_new = fmaxf(m, mx);
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        const float alpha = ex2(m - m_use);
        // P buffer st is free once PV(t-2) finished reading it
        if (!wait(&p_empty[st], ((t >> 1) & 1) ^ 1)) {
          fail(args, s_abort, 0x3002);
          ok = false;
          break;
        }
        float sum4[4] = {0.f, 0.f, 0.f, 0.f};
        uint8_t* pbase = sP + st * TILE_BYTES;
#pragma unroll
        for (int c = 0; c < 16; ++c) {  // 16 chunks of 8 keys
          uint32_t w[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float p0 = ex2(fmaf(sv[c * 8 + 2 * q], args.scale_log2, -m_use));
            const float p1 = ex2(fmaf(sv[c * 8 + 2 * q + 1], args.scale_log2, -m_use));
            sum4[q] += p0 + p1;
            w[q] = pack_bf16x2(p0, p1);
          }
          uint8_t* dst = pbase + (c >> 3) * HALF_BYTES + sw128_off(r, c & 7);
          *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        fence_async_smem();
        // alpha / l buffer st is free once the correction thread has read tile t-2's
        if (!wait(&a_empty[st], ((t >> 1) & 1) ^ 1)) {
          fail(args, s_abort, 0x3003);
          ok = false;
          break;
        }
        l = l * alpha + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
        m = m_new;
        s_alpha[st * 128 + r] = alpha;
        s_l[st * 128 + r] = l;
        tc::mbar_arrive(tc::smem_u32(&p_full[st]));
      }
    }
  } else {
    // ---------------------------------------------------------------- correction / output
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    int t = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      int qt, h, b;
      item_coords(item, args, qt, h, b);
      const int n_kv = min(qt + 1, kv_tiles);
      float o[HD];
#pragma unroll
      for (int i = 0; i < HD; ++i) o[i] = 0.f;
      float l_final = 1.f;
      for (int j = 0; j < n_kv; ++j, ++t) {
        const int st = t & 1;
        if (!wait(&p_full[st], (t >> 1) & 1) || !wait(&o_full[st], (t >> 1) & 1)) {
          fail(args, s_abort, 0x4001);
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const float alpha = s_alpha[st * 128 + r];
        l_final = s_l[st * 128 + r];
        tc::mbar_arrive(tc::smem_u32(&a_empty[st]));
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t u[32];
          tc::tmem_ld_32x32b_x32(tmem + 256 + st * 128 + lane_off + c * 32, u);
          tc::tmem_wait_ld();
          tc::tmem_reg_fence(u);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[c * 32 + i] = fmaf(o[c * 32 + i], alpha, __uint_as_float(u[i]));
        }
        tc::tc_fence_before();
        tc::mbar_arrive(tc::smem_u32(&o_empty[st]));
      }
      // l_final was written by this row's softmax thread before its last p_full arrival
      if (!ok || *s_abort) break;
      const int qpos = qt * BQ + r;
      if (qpos < args.S) {
        const float inv = 1.f / l_final;
        __nv_bfloat16* dst = args.out + (int64_t)(b * args.S + qpos) * (args.nq * HD) + h * HD;
#pragma unroll
        for (int c = 0; c < HD / 8; ++c) {
          const uint4 v = make_uint4(pack_bf16x2(o[8 * c] * inv, o[8 * c + 1] * inv),
                                     pack_bf16x2(o[8 * c + 2] * inv, o[8 * c + 3] * inv),
                                     pack_bf16x2(o[8 * c + 4] * inv, o[8 * c + 5] * inv),
                                     pack_bf16x2(o[8 * c + 6] * inv, o[8 * c + 7] * inv));
          reinterpret_cast<uint4*>(dst)[c] = v;
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

}  // namespace attn

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
  static bool attr_set[64] = {false};
  const int dev = qkv.get_device();
  if (!attr_set[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    attr_set[dev] = true;
  }
  const CUtensorMap tq = make_map(qkv.data_ptr(), B * S, (nq + 2 * nkv) * HD, (nq + 2 * nkv) * HD);
  Args a;
  a.B = (int)B;
  a.S = (int)S;
  a.nq = (int)nq;
  a.nkv = (int)nkv;
  a.group = (int)(nq / nkv);
  a.q_tiles = (int)((S + BQ - 1) / BQ);
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.status = status_word();
  a.timeout_ns = 10000000000ull;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t items = (int64_t)a.q_tiles * nq * B;
  const int grid = (int)std::min<int64_t>(items, sms);
  attn_prefill_kernel<<<grid, NUM_THREADS, SMEM_BYTES, st>>>(tq, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t attn_status(bool clear) {
  volatile int* p = attn::status_word();
  const int v = *p;
  if (clear) *p = 0;
  return v;
}

}  // namespace qfc
