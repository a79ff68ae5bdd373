// Causal flash attention for prefill on sm_100a tensor cores (tcgen05 / TMEM / TMA).
//
// Replaces the attention of the reference's Hugging Face model (replicated on every rank,
// main.py:194).  Inputs come straight from the fused qkv activation [B*S, (nq + 2 nkv) hd]
// (after RoPE); V is first transposed into vt [B * nkv * hd, S_pad] so that both matrix
// products read K-major operands with the same 128-byte-swizzled TMA layout as the GEMM.
//
// One CTA per (128-query tile, query head, sequence), 10 warps:
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
constexpr uint32_t IDESC = tc::idesc_f16(128, 128, true);
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

__global__ void __launch_bounds__(NUM_THREADS, 1)
attn_prefill_kernel(const __grid_constant__ CUtensorMap tmQKV, const __grid_constant__ CUtensorMap tmVT,
                    const Args args) {
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
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 20);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* s_alpha = reinterpret_cast<float*>(tmem_holder + 4);  // [2][128]
  float* s_l = s_alpha + 256;                                   // [2][128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Heaviest (last) query tiles first.
  const int qt = args.q_tiles - 1 - (int)blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / args.group;
  const int q0 = qt * BQ;
  const int n_kv = min(qt + 1, (args.S + BKV - 1) / BKV);  // causal: tiles 0..qt
  const int row_base = b * args.S;

  if (threadIdx.x == 0) {
    tc::mbar_init(tc::smem_u32(q_full), 1);
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

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tc::tma_prefetch_desc(&tmQKV);
      tc::tma_prefetch_desc(&tmVT);
      const uint32_t qb = tc::smem_u32(q_full);
      tc::mbar_arrive_expect_tx(qb, TILE_BYTES);
      tc::tma_load_2d(tc::smem_u32(sQ), &tmQKV, qb, h * HD, row_base + q0);
      tc::tma_load_2d(tc::smem_u32(sQ + HALF_BYTES), &tmQKV, qb, h * HD + 64, row_base + q0);
      int issued[2] = {-1, -1};
      for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        if (!tc::mbar_wait(tc::smem_u32(&kv_empty[st]), ((j >> 1) & 1) ^ 1, globaltimer_ns() + args.timeout_ns,
                           s_abort)) {
          fail(args, s_abort, 0x1001);
          break;
        }
        const uint32_t fb = tc::smem_u32(&kv_full[st]);
        tc::mbar_arrive_expect_tx(fb, 2 * TILE_BYTES);
        const int kcol = (args.nq + kvh) * HD;
        tc::tma_load_2d(tc::smem_u32(sK + st * TILE_BYTES), &tmQKV, fb, kcol, row_base + j * BKV);
        tc::tma_load_2d(tc::smem_u32(sK + st * TILE_BYTES + HALF_BYTES), &tmQKV, fb, kcol + 64, row_base + j * BKV);
        const int vrow = (b * args.nkv + kvh) * HD;
        tc::tma_load_2d(tc::smem_u32(sV + st * TILE_BYTES), &tmVT, fb, j * BKV, vrow);
        tc::tma_load_2d(tc::smem_u32(sV + st * TILE_BYTES + HALF_BYTES), &tmVT, fb, j * BKV + 64, vrow);
        issued[st] = j;
      }
      if (*s_abort) {  // let issued copies land before shared memory goes away
        int never = 0;
        tc::mbar_wait(qb, 0, globaltimer_ns() + 50000000ull, &never);
        for (int st = 0; st < 2; ++st)
          if (issued[st] >= 0)
            tc::mbar_wait(tc::smem_u32(&kv_full[st]), (issued[st] >> 1) & 1, globaltimer_ns() + 50000000ull, &never);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      bool ok = tc::mbar_wait(tc::smem_u32(q_full), 0, globaltimer_ns() + args.timeout_ns, s_abort);
      bool issued_any = false;
      auto issue_qk = [&](int j) -> bool {
        const int st = j & 1;
        if (!tc::mbar_wait(tc::smem_u32(&kv_full[st]), (j >> 1) & 1, globaltimer_ns() + args.timeout_ns, s_abort))
          return false;
        if (!tc::mbar_wait(tc::smem_u32(&s_empty[st]), ((j >> 1) & 1) ^ 1, globaltimer_ns() + args.timeout_ns, s_abort))
          return false;
        tc::tc_fence_after();
        const uint32_t a0 = tc::smem_u32(sQ), b0 = tc::smem_u32(sK + st * TILE_BYTES);
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc::umma_f16(tmem + st * 128, tc::sw128_kmajor_desc(a0 + s * HALF_BYTES + k * 32),
                         tc::sw128_kmajor_desc(b0 + s * HALF_BYTES + k * 32), IDESC, (s | k) != 0);
        tc::umma_commit(tc::smem_u32(&s_full[st]));
        issued_any = true;
        return true;
      };
      if (ok) ok = issue_qk(0);
      for (int j = 0; ok && j < n_kv; ++j) {
        const int st = j & 1;
        if (j + 1 < n_kv && !issue_qk(j + 1)) {
          ok = false;
          break;
        }
        if (!tc::mbar_wait(tc::smem_u32(&p_full[st]), (j >> 1) & 1, globaltimer_ns() + args.timeout_ns, s_abort) ||
            !tc::mbar_wait(tc::smem_u32(&o_empty[st]), ((j >> 1) & 1) ^ 1, globaltimer_ns() + args.timeout_ns,
                           s_abort)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t a0 = tc::smem_u32(sP + st * TILE_BYTES), b0 = tc::smem_u32(sV + st * TILE_BYTES);
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc::umma_f16(tmem + 256 + st * 128, tc::sw128_kmajor_desc(a0 + s * HALF_BYTES + k * 32),
                         tc::sw128_kmajor_desc(b0 + s * HALF_BYTES + k * 32), IDESC, (s | k) != 0);
        tc::umma_commit(tc::smem_u32(&o_full[st]));
        tc::umma_commit(tc::smem_u32(&p_empty[st]));
        tc::umma_commit(tc::smem_u32(&kv_empty[st]));
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
    const int qpos = q0 + r;
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j < n_kv; ++j) {
      const int st = j & 1;
      if (!tc::mbar_wait(tc::smem_u32(&s_full[st]), (j >> 1) & 1, globaltimer_ns() + args.timeout_ns, s_abort)) {
        fail(args, s_abort, 0x3001);
        break;
      }
      tc::tc_fence_after();
      float sv[128];
      const uint32_t ta = tmem + st * 128 + ((uint32_t)((warp & 3) * 32) << 16);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t u[32];
        tc::tmem_ld_32x32b_x32(ta + c * 32, u);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[c * 32 + i] = __uint_as_float(u[i]);
      }
      tc::tc_fence_before();
      tc::mbar_arrive(tc::smem_u32(&s_empty[st]));
      // masks: keys above the diagonal and keys past the end of the sequence
      const int k0 = j * BKV;
      const int kmax = min(qpos, args.S - 1) - k0;  // last visible column (may be < 0 or >= 127)
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        sv[i] = (i <= kmax) ? sv[i] * args.scale_log2 : -INFINITY;
        mx = fmaxf(mx, sv[i]);
      }
      const float m_new = fmaxf(m, mx);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = ex2(m - m_use);
      // P buffer st is free once PV(j-2) finished reading it
      if (!tc::mbar_wait(tc::smem_u32(&p_empty[st]), ((j >> 1) & 1) ^ 1, globaltimer_ns() + args.timeout_ns,
                         s_abort)) {
        fail(args, s_abort, 0x3002);
        break;
      }
      float sum = 0.f;
      uint8_t* pbase = sP + st * TILE_BYTES;
#pragma unroll
      for (int c = 0; c < 16; ++c) {  // 16 chunks of 8 keys
        uint32_t w[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float p0 = ex2(sv[c * 8 + 2 * t] - m_use);
          const float p1 = ex2(sv[c * 8 + 2 * t + 1] - m_use);
          sum += p0 + p1;
          w[t] = pack_bf16x2(p0, p1);
        }
        uint8_t* dst = pbase + (c >> 3) * HALF_BYTES + sw128_off(r, c & 7);
        *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_async_smem();
      // alpha / l buffer st is free once the correction thread has read tile j-2's
      if (!tc::mbar_wait(tc::smem_u32(&a_empty[st]), ((j >> 1) & 1) ^ 1, globaltimer_ns() + args.timeout_ns,
                         s_abort)) {
        fail(args, s_abort, 0x3003);
        break;
      }
      l = l * alpha + sum;
      m = m_new;
      s_alpha[st * 128 + r] = alpha;
      s_l[st * 128 + r] = l;
      tc::mbar_arrive(tc::smem_u32(&p_full[st]));
    }
  } else {
    // ---------------------------------------------------------------- correction / output
    const int r = (warp & 3) * 32 + lane;
    float o[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) o[i] = 0.f;
    bool ok = true;
    float l_final = 1.f;
    for (int j = 0; j < n_kv; ++j) {
      const int st = j & 1;
      if (!tc::mbar_wait(tc::smem_u32(&p_full[st]), (j >> 1) & 1, globaltimer_ns() + args.timeout_ns, s_abort) ||
          !tc::mbar_wait(tc::smem_u32(&o_full[st]), (j >> 1) & 1, globaltimer_ns() + args.timeout_ns, s_abort)) {
        fail(args, s_abort, 0x4001);
        ok = false;
        break;
      }
      tc::tc_fence_after();
      const float alpha = s_alpha[st * 128 + r];
      l_final = s_l[st * 128 + r];
      tc::mbar_arrive(tc::smem_u32(&a_empty[st]));
      const uint32_t ta = tmem + 256 + st * 128 + ((uint32_t)((warp & 3) * 32) << 16);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t u[32];
        tc::tmem_ld_32x32b_x32(ta + c * 32, u);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[c * 32 + i] = o[c * 32 + i] * alpha + __uint_as_float(u[i]);
      }
      tc::tc_fence_before();
      tc::mbar_arrive(tc::smem_u32(&o_empty[st]));
    }
    // l_final was written by this row's softmax thread before its last p_full arrival
    if (ok && !*s_abort) {
      const int qpos = q0 + r;
      if (qpos < args.S) {
        const float inv = 1.f / l_final;
        __nv_bfloat16* dst = args.out + (int64_t)(row_base + qpos) * (args.nq * HD) + h * HD;
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

// vt[(b*nkv + kvh)*HD + d][s] = v[b*S + s][kvh*HD + d]  (32x32 tiles through shared memory)
__global__ void transpose_v_kernel(const __nv_bfloat16* __restrict__ qkv, __nv_bfloat16* __restrict__ vt, int B, int S,
                                   int S_pad, int nq, int nkv) {
  __shared__ __nv_bfloat16 tile[32][33];
  const int ld = (nq + 2 * nkv) * HD;
  const int bk = blockIdx.z;  // b * nkv + kvh
  const int b = bk / nkv, kvh = bk % nkv;
  const int s0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int s = s0 + i, d = d0 + threadIdx.x;
    tile[i][threadIdx.x] = (s < S) ? qkv[(int64_t)(b * S + s) * ld + (nq + nkv + kvh) * HD + d] : __float2bfloat16(0.f);
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int d = d0 + i, s = s0 + threadIdx.x;
    if (s < S_pad) vt[((int64_t)bk * HD + d) * S_pad + s] = tile[threadIdx.x][i];
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
  const int64_t S_pad = (S + 7) / 8 * 8;
  at::Tensor vt = at::empty({B * nkv * HD, S_pad}, qkv.options());
  dim3 tgrid((unsigned)((S_pad + 31) / 32), HD / 32, (unsigned)(B * nkv));
  transpose_v_kernel<<<tgrid, dim3(32, 8), 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
                                                    reinterpret_cast<__nv_bfloat16*>(vt.data_ptr()), (int)B, (int)S,
                                                    (int)S_pad, (int)nq, (int)nkv);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  static bool attr_set[64] = {false};
  const int dev = qkv.get_device();
  if (!attr_set[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    attr_set[dev] = true;
  }
  const CUtensorMap tq = make_map(qkv.data_ptr(), B * S, (nq + 2 * nkv) * HD, (nq + 2 * nkv) * HD);
  const CUtensorMap tv = make_map(vt.data_ptr(), B * nkv * HD, S, S_pad);
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
  dim3 grid((unsigned)a.q_tiles, (unsigned)nq, (unsigned)B);
  attn_prefill_kernel<<<grid, NUM_THREADS, SMEM_BYTES, st>>>(tq, tv, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t attn_status(bool clear) {
  volatile int* p = attn::status_word();
  const int v = *p;
  if (clear) *p = 0;
  return v;
}

}  // namespace qfc
