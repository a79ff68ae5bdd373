// Llama layer kernels for sm_100a: RMSNorm (with fused residual add), rotary embedding
// with the paged KV-cache write, SwiGLU, token embedding and greedy argmax.
//
// In the reference these come from Hugging Face modules (LlamaRMSNorm, rotary embedding,
// nn.SiLU in model.py:27 and the elementwise multiply at model.py:34); here each is one
// memory-bound kernel with 16-byte accesses, launched on the caller's stream.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>

#include <cfloat>

#include "common.cuh"

namespace qfc {

namespace {

template <int NT>
QFC_DEV float block_sum(float v, float* smem) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(QFC_FULL_MASK, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) smem[warp] = v;
  __syncthreads();
  float t = (lane < NT / 32) ? smem[lane] : 0.f;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) t += __shfl_xor_sync(QFC_FULL_MASK, t, off);
  return t;
}

// y = rmsnorm(x + residual) * w;  when residual is given, x + residual is also written to
// residual_out (the new residual stream).  One CTA per row, up to 8 x 8 elements/thread
// held in registers.  Rounding follows the HF module: normalise in fp32, round to the
// activation dtype, then multiply by the weight and round again.
template <typename T, int NT, int VPT>
__global__ void __launch_bounds__(NT)
rmsnorm_kernel(const T* __restrict__ x, const T* __restrict__ residual, T* __restrict__ residual_out,
               const T* __restrict__ w, T* __restrict__ y, int H, float eps) {
  __shared__ float smem[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * H;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = (k * NT + threadIdx.x) * 8;
    if (c < H) {
      Vec8IO<T>::load(xr + c, v[k]);
      if (residual != nullptr) {
        float r[8];
        Vec8IO<T>::load(residual + row * H + c, r);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[k][i] = to_f32(from_f32<T>(v[k][i] + r[i]));
        Vec8IO<T>::store(residual_out + row * H + c, v[k]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[k][i] * v[k][i];
    }
  }
  const float tot = block_sum<NT>(ss, smem);
  const float r = rsqrtf(tot / (float)H + eps);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = (k * NT + threadIdx.x) * 8;
    if (c < H) {
      float wv[8];
      Vec8IO<T>::load(w + c, wv);
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = to_f32(from_f32<T>(v[k][i] * r)) * wv[i];
      Vec8IO<T>::store(y + row * H + c, o);
    }
  }
}

// Rotary embedding (rotate-half convention) applied in place to q and k of the fused
// qkv activation [M, (nq + 2*nkv) * hd], and k / v copied into the paged cache
// k_cache / v_cache [num_pages, nkv, page, hd] at slot_mapping[m] (page * page_size +
// offset; negative = do not cache).  One thread per (token, head, 8-element slice j of
// the first half): it loads the 16-byte slices j of both halves, rotates them with the
// (cos, sin) pairs of positions j*8 .. j*8+7 and stores both back (q, k) and into the
// cache (k, v).  Every access is a 16-byte vector; hd = 64 or 128.
//
// Decode form (seq_lens != nullptr, one token per sequence, m = sequence): the position is
// seq_lens[m] - 1 (the count already includes the new token) and the cache slot comes
// from the block table in the kernel, so a decode step needs no position / slot tensors;
// positions at or past max_pages * page are not cached.
template <typename T, int HD>
__global__ void rope_kv_kernel(T* __restrict__ qkv, const int64_t* __restrict__ pos, const float2* __restrict__ cs,
                               T* __restrict__ k_cache, T* __restrict__ v_cache,
                               const int64_t* __restrict__ slot_mapping, int64_t M, int nq, int nkv, int page,
                               int page_shift, const int* __restrict__ seq_lens, const int* __restrict__ block_table,
                               int max_pages) {
  constexpr int HALF = HD / 2, HJ = HALF / 8;
  const uint32_t heads = (uint32_t)(nq + 2 * nkv);
  const int64_t total = M * heads * HJ;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(t % HJ);
    const uint64_t hh = (uint64_t)(t / HJ);
    const uint32_t h = (uint32_t)(hh % heads);
    const int64_t m = (int64_t)(hh / heads);
    const int64_t pm = seq_lens != nullptr ? (int64_t)seq_lens[m] - 1 : pos[m];
    T* row = qkv + (m * heads + h) * HD;
    float x1[8], x2[8];
    Vec8IO<T>::load(row + j * 8, x1);
    Vec8IO<T>::load(row + HALF + j * 8, x2);
    if (h < (uint32_t)(nq + nkv)) {
      const float4* c = reinterpret_cast<const float4*>(cs + pm * HALF + j * 8);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 a = c[i];  // (cos, sin) of elements 2i and 2i+1
        rope_pair(x1[2 * i], x2[2 * i], a.x, a.y, x1[2 * i], x2[2 * i]);
        rope_pair(x1[2 * i + 1], x2[2 * i + 1], a.z, a.w, x1[2 * i + 1], x2[2 * i + 1]);
      }
      Vec8IO<T>::store(row + j * 8, x1);
      Vec8IO<T>::store(row + HALF + j * 8, x2);
    }
    if (h >= (uint32_t)nq && (slot_mapping != nullptr || seq_lens != nullptr)) {
      int64_t slot;
      if (seq_lens != nullptr) {
        slot = (pm >= 0 && pm < (int64_t)max_pages * page)
                   ? (int64_t)block_table[m * max_pages + (pm / page)] * page + pm % page
                   : -1;
      } else {
        slot = slot_mapping[m];
      }
      if (slot >= 0) {
        const int64_t pg = page_shift >= 0 ? slot >> page_shift : slot / page;
        const int64_t off = page_shift >= 0 ? slot & (page - 1) : slot % page;
        const bool is_k = h < (uint32_t)(nq + nkv);
        const int kvh = is_k ? (int)h - nq : (int)h - nq - nkv;
        T* dst = (is_k ? k_cache : v_cache) + ((pg * nkv + kvh) * (int64_t)page + off) * HD;
        // the stored k is the bf16/fp16 value written back to qkv above
        Vec8IO<T>::store(dst + j * 8, x1);
        Vec8IO<T>::store(dst + HALF + j * 8, x2);
      }
    }
  }
}

// out[m, j] = silu(gu[m, j]) * gu[m, I + j] for the fused gate|up activation [M, 2I].
template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ gu, T* __restrict__ out, int64_t M, int I) {
  const int64_t per_row = I / 8;
  const int64_t total = M * per_row;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = t / per_row;
    const int64_t j = (t % per_row) * 8;
    float g[8], u[8], o[8];
    Vec8IO<T>::load(gu + m * 2 * I + j, g);
    Vec8IO<T>::load(gu + m * 2 * I + I + j, u);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // HF order: act_fn(gate) is rounded to the activation dtype before the multiply.
      const float s = to_f32(from_f32<T>(g[i] / (1.f + __expf(-g[i]))));
      o[i] = s * u[i];
    }
    Vec8IO<T>::store(out + m * I + j, o);
  }
}

template <typename T>
__global__ void embedding_kernel(const int64_t* __restrict__ ids, const T* __restrict__ table, T* __restrict__ out,
                                 int64_t M, int H, int64_t vocab_start, int64_t vocab_end) {
  const int64_t per_row = H / 8;
  const int64_t total = M * per_row;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = t / per_row;
    const int64_t j = (t % per_row) * 8;
    const int64_t id = ids[m];
    uint4 v = make_uint4(0, 0, 0, 0);
    if (id >= vocab_start && id < vocab_end)
      v = *reinterpret_cast<const uint4*>(table + (id - vocab_start) * H + j);
    *reinterpret_cast<uint4*>(out + m * H + j) = v;
  }
}

// Counter-based random bits for sampling: the SplitMix64 output function (Steele, Lea and
// Flood, "Fast splittable pseudorandom number generators", OOPSLA 2014) applied to a key
// built from (seed, step, row, vocabulary index).  The same key gives the same bits on
// every rank and at every tensor-parallel degree, so ranks that sample their own slice of
// the vocabulary agree on the token without exchanging random state.
QFC_DEV uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// Standard Gumbel noise -log(-log(u)) with u in (0, 1) from 24 random bits.
QFC_DEV float gumbel_noise(uint64_t seed, uint64_t step, int64_t row, int64_t idx) {
  const uint64_t h = mix64(mix64(mix64(seed ^ (step * 0xd1b54a32d192ed03ull)) ^ (uint64_t)row) ^ (uint64_t)idx);
  const float u = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
  return -logf(-logf(u));
}

// Row-wise (max score, argmax) over logits [M, V] (row stride V; only the first V_valid
// columns count; the first index wins ties).  Greedy: score = logit.  SAMPLE: score =
// logit * inv_temp + Gumbel noise keyed by (rng[0] = seed, rng[1] = step, row, global
// index), whose argmax is an exact draw from softmax(logit * inv_temp) (the Gumbel-max
// trick); the last CTA to finish then advances rng[1], so a captured decode step samples
// afresh on every replay.
template <typename T, bool SAMPLE>
__global__ void __launch_bounds__(1024) argmax_kernel(const T* __restrict__ logits, float* __restrict__ best_val, int64_t* __restrict__ best_idx,
                              int64_t V, int64_t V_valid, int64_t idx_offset, int64_t* __restrict__ rng,
                              float inv_temp, unsigned int* __restrict__ done) {
  const int64_t row = blockIdx.x;
  const T* r = logits + row * V;
  float bv = -FLT_MAX;
  int64_t bi = INT64_MAX;
  uint64_t seed = 0, step = 0;
  if constexpr (SAMPLE) {
    seed = (uint64_t)rng[0];
    step = (uint64_t)rng[1];
  }
  auto score = [&](float v, int64_t i) -> float {
    if constexpr (SAMPLE) return v * inv_temp + gumbel_noise(seed, step, row, i + idx_offset);
    else return v;
  };
  if (sizeof(T) == 2 && (V & 7) == 0 && (reinterpret_cast<uintptr_t>(r) & 15) == 0) {
    // 16-byte loads, 4 in flight per thread; a thread's elements rise in index, so the
    // strict comparison keeps the first maximum
    const int64_t nv = (V_valid + 7) >> 3;
    for (int64_t c0 = threadIdx.x; c0 < nv; c0 += 4 * (int64_t)blockDim.x) {
      float v[4][8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int64_t c = c0 + k * (int64_t)blockDim.x;
        if (c < nv) Vec8IO<T>::load(r + c * 8, v[k]);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int64_t c = c0 + k * (int64_t)blockDim.x;
        if (c < nv) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int64_t i = c * 8 + j;
            if (i < V_valid) {
              const float sc = score(v[k][j], i);
              if (sc > bv) {
                bv = sc;
                bi = i;
              }
            }
          }
        }
      }
    }
  } else {
    for (int64_t i = threadIdx.x; i < V_valid; i += blockDim.x) {
      const float v = score(to_f32(r[i]), i);
      if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
      }
    }
  }
  __shared__ float sv[32];
  __shared__ int64_t si[32];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(QFC_FULL_MASK, bv, off);
    const int64_t oi = __shfl_xor_sync(QFC_FULL_MASK, bi, off);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    bv = lane < nw ? sv[lane] : -FLT_MAX;
    bi = lane < nw ? si[lane] : INT64_MAX;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(QFC_FULL_MASK, bv, off);
      const int64_t oi = __shfl_xor_sync(QFC_FULL_MASK, bi, off);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      best_val[row] = bv;
      best_idx[row] = (bi == INT64_MAX) ? -1 : bi + idx_offset;
      if constexpr (SAMPLE) {
        // every CTA read rng[1] before it arrives here; the last arrival advances it
        __threadfence();
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
          rng[1] = (int64_t)(step + 1);
          *done = 0u;
          __threadfence();
        }
      }
    }
  }
}

#define QFC_DISPATCH_16(dt, ...)                                          \
  do {                                                                    \
    if ((dt) == at::kBFloat16) {                                          \
      using scalar_t = __nv_bfloat16;                                     \
      __VA_ARGS__();                                                      \
    } else if ((dt) == at::kHalf) {                                       \
      using scalar_t = __half;                                            \
      __VA_ARGS__();                                                      \
    } else {                                                              \
      TORCH_CHECK(false, "expected a bf16 or fp16 tensor, got ", (dt));   \
    }                                                                     \
  } while (0)

}  // namespace

// y = rmsnorm(x [+ residual]) * w; when residual is given, residual is updated in place
// to x + residual.
void rmsnorm_cuda(const at::Tensor& x, const c10::optional<at::Tensor>& residual, const at::Tensor& w, at::Tensor& y,
                  double eps) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && y.is_contiguous() && w.is_contiguous(), "rmsnorm: contiguous CUDA tensors");
  const int H = (int)x.size(-1);
  const int64_t M = x.numel() / H;
  TORCH_CHECK(H % 8 == 0 && H <= 8 * 8 * 1024, "rmsnorm: hidden size must be a multiple of 8, <= 65536");
  if (M == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const bool has_res = residual.has_value() && residual->defined();
  QFC_DISPATCH_16(x.scalar_type(), [&] {
    const scalar_t* rp = has_res ? reinterpret_cast<const scalar_t*>(residual->data_ptr()) : nullptr;
    scalar_t* ro = has_res ? reinterpret_cast<scalar_t*>(residual->data_ptr()) : nullptr;
    auto xp = reinterpret_cast<const scalar_t*>(x.data_ptr());
    auto wp = reinterpret_cast<const scalar_t*>(w.data_ptr());
    auto yp = reinterpret_cast<scalar_t*>(y.data_ptr());
    const int vec = H / 8;
    if (vec <= 512) {
      constexpr int NT = 512;
      rmsnorm_kernel<scalar_t, NT, 1><<<M, NT, 0, st>>>(xp, rp, ro, wp, yp, H, (float)eps);
    } else if (vec <= 1024) {
      constexpr int NT = 512;
      rmsnorm_kernel<scalar_t, NT, 2><<<M, NT, 0, st>>>(xp, rp, ro, wp, yp, H, (float)eps);
    } else {
      constexpr int NT = 1024;
      rmsnorm_kernel<scalar_t, NT, 8><<<M, NT, 0, st>>>(xp, rp, ro, wp, yp, H, (float)eps);
    }
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rope_kv_cuda(at::Tensor& qkv, const at::Tensor& pos, const at::Tensor& cos_sin, const c10::optional<at::Tensor>& k_cache,
                  const c10::optional<at::Tensor>& v_cache, const c10::optional<at::Tensor>& slot_mapping, int64_t nq,
                  int64_t nkv, int64_t hd) {
  TORCH_CHECK(qkv.is_cuda() && qkv.is_contiguous(), "rope_kv: contiguous CUDA qkv");
  TORCH_CHECK(pos.scalar_type() == at::kLong && cos_sin.scalar_type() == at::kFloat, "rope_kv: int64 positions, fp32 cos/sin");
  const int64_t M = qkv.numel() / ((nq + 2 * nkv) * hd);
  if (M == 0) return;
  c10::cuda::CUDAGuard guard(qkv.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const bool cache = slot_mapping.has_value() && slot_mapping->defined();
  int page = 1;
  if (cache) {
    TORCH_CHECK(k_cache->dim() == 4, "rope_kv: cache must be [pages, nkv, page, hd]");
    page = (int)k_cache->size(2);
  }
  TORCH_CHECK(hd == 64 || hd == 128, "rope_kv: head_dim must be 64 or 128");
  int page_shift = -1;
  for (int sh = 0; sh < 31; ++sh)
    if ((1 << sh) == page) page_shift = sh;
  const int64_t total = M * (nq + 2 * nkv) * (hd / 16);
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((total + threads - 1) / threads, 148 * 8);
  QFC_DISPATCH_16(qkv.scalar_type(), [&] {
    auto* q = reinterpret_cast<scalar_t*>(qkv.data_ptr());
    auto* csp = reinterpret_cast<const float2*>(cos_sin.data_ptr());
    auto* kcp = cache ? reinterpret_cast<scalar_t*>(k_cache->data_ptr()) : nullptr;
    auto* vcp = cache ? reinterpret_cast<scalar_t*>(v_cache->data_ptr()) : nullptr;
    const int64_t* sm = cache ? slot_mapping->data_ptr<int64_t>() : nullptr;
    if (hd == 128)
      rope_kv_kernel<scalar_t, 128><<<blocks, threads, 0, st>>>(q, pos.data_ptr<int64_t>(), csp, kcp, vcp, sm, M,
                                                                 (int)nq, (int)nkv, page, page_shift, nullptr,
                                                                 nullptr, 0);
    else
      rope_kv_kernel<scalar_t, 64><<<blocks, threads, 0, st>>>(q, pos.data_ptr<int64_t>(), csp, kcp, vcp, sm, M,
                                                                (int)nq, (int)nkv, page, page_shift, nullptr,
                                                                nullptr, 0);
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Decode step: qkv [B, (nq+2nkv)*hd], one token per sequence at position seq_lens[b] - 1,
// written to the paged cache through block_table [B, max_pages] (int32).
void rope_kv_decode_cuda(at::Tensor& qkv, const at::Tensor& cos_sin, at::Tensor& k_cache, at::Tensor& v_cache,
                         const at::Tensor& block_table, const at::Tensor& seq_lens, int64_t nq, int64_t nkv,
                         int64_t hd) {
  TORCH_CHECK(qkv.is_cuda() && qkv.is_contiguous(), "rope_kv_decode: contiguous CUDA qkv");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat, "rope_kv_decode: fp32 cos/sin");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt &&
                  block_table.is_contiguous() && seq_lens.is_contiguous(),
              "rope_kv_decode: int32 contiguous block table and sequence lengths");
  TORCH_CHECK(k_cache.dim() == 4 && v_cache.dim() == 4, "rope_kv_decode: cache must be [pages, nkv, page, hd]");
  TORCH_CHECK(hd == 64 || hd == 128, "rope_kv_decode: head_dim must be 64 or 128");
  const int64_t M = qkv.numel() / ((nq + 2 * nkv) * hd);
  TORCH_CHECK(seq_lens.numel() == M && block_table.size(0) == M, "rope_kv_decode: one row per sequence");
  if (M == 0) return;
  c10::cuda::CUDAGuard guard(qkv.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int page = (int)k_cache.size(2);
  int page_shift = -1;
  for (int sh = 0; sh < 31; ++sh)
    if ((1 << sh) == page) page_shift = sh;
  const int max_pages = (int)block_table.size(1);
  const int64_t total = M * (nq + 2 * nkv) * (hd / 16);
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((total + threads - 1) / threads, 148 * 8);
  QFC_DISPATCH_16(qkv.scalar_type(), [&] {
    auto* q = reinterpret_cast<scalar_t*>(qkv.data_ptr());
    auto* csp = reinterpret_cast<const float2*>(cos_sin.data_ptr());
    auto* kcp = reinterpret_cast<scalar_t*>(k_cache.data_ptr());
    auto* vcp = reinterpret_cast<scalar_t*>(v_cache.data_ptr());
    if (hd == 128)
      rope_kv_kernel<scalar_t, 128><<<blocks, threads, 0, st>>>(q, nullptr, csp, kcp, vcp, nullptr, M, (int)nq,
                                                                 (int)nkv, page, page_shift, seq_lens.data_ptr<int>(),
                                                                 block_table.data_ptr<int>(), max_pages);
    else
      rope_kv_kernel<scalar_t, 64><<<blocks, threads, 0, st>>>(q, nullptr, csp, kcp, vcp, nullptr, M, (int)nq,
                                                                (int)nkv, page, page_shift, seq_lens.data_ptr<int>(),
                                                                block_table.data_ptr<int>(), max_pages);
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void silu_mul_cuda(const at::Tensor& gu, at::Tensor& out) {
  TORCH_CHECK(gu.is_contiguous() && out.is_contiguous(), "silu_mul: contiguous tensors");
  const int I = (int)out.size(-1);
  const int64_t M = out.numel() / I;
  TORCH_CHECK(gu.size(-1) == 2 * I && I % 8 == 0, "silu_mul: gu must be [M, 2I], I % 8 == 0");
  if (M == 0) return;
  c10::cuda::CUDAGuard guard(gu.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int64_t total = M * (I / 8);
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  QFC_DISPATCH_16(gu.scalar_type(), [&] {
    silu_mul_kernel<scalar_t><<<blocks, 256, 0, st>>>(reinterpret_cast<const scalar_t*>(gu.data_ptr()),
                                                       reinterpret_cast<scalar_t*>(out.data_ptr()), M, I);
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embedding_cuda(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out, int64_t vocab_start) {
  TORCH_CHECK(ids.scalar_type() == at::kLong && table.is_contiguous() && out.is_contiguous(), "embedding: bad args");
  const int H = (int)table.size(1);
  const int64_t M = ids.numel();
  TORCH_CHECK(H % 8 == 0, "embedding: hidden size must be a multiple of 8");
  if (M == 0) return;
  c10::cuda::CUDAGuard guard(table.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int64_t total = M * (H / 8);
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  QFC_DISPATCH_16(table.scalar_type(), [&] {
    embedding_kernel<scalar_t><<<blocks, 256, 0, st>>>(ids.data_ptr<int64_t>(), reinterpret_cast<const scalar_t*>(table.data_ptr()),
                                                        reinterpret_cast<scalar_t*>(out.data_ptr()), M, H, vocab_start,
                                                        vocab_start + table.size(0));
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void argmax_cuda(const at::Tensor& logits, at::Tensor& best_val, at::Tensor& best_idx, int64_t idx_offset,
                 int64_t valid, const c10::optional<at::Tensor>& rng, double inv_temp,
                 const c10::optional<at::Tensor>& done) {
  TORCH_CHECK(logits.is_contiguous() && logits.dim() == 2, "argmax: contiguous [M, V] logits");
  const int64_t M = logits.size(0), V = logits.size(1);
  const int64_t V_valid = valid < 0 ? V : std::min<int64_t>(valid, V);
  if (M == 0) return;
  const bool sample = rng.has_value();
  if (sample) {
    TORCH_CHECK(rng->scalar_type() == at::kLong && rng->numel() >= 2 && rng->is_cuda(),
                "argmax: rng must be an int64 CUDA tensor [seed, step]");
    TORCH_CHECK(done.has_value() && done->scalar_type() == at::kInt && done->is_cuda(),
                "argmax: sampling needs an int32 CUDA arrival counter (zero before the first call)");
  }
  c10::cuda::CUDAGuard guard(logits.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  int64_t* rp = sample ? rng->data_ptr<int64_t>() : nullptr;
  unsigned int* dp = sample ? reinterpret_cast<unsigned int*>(done->data_ptr<int>()) : nullptr;
  auto launch = [&](auto tag) {
    using T = decltype(tag);
    const T* lp = reinterpret_cast<const T*>(logits.data_ptr());
    if (sample)
      argmax_kernel<T, true><<<M, 1024, 0, st>>>(lp, best_val.data_ptr<float>(), best_idx.data_ptr<int64_t>(), V,
                                                 V_valid, idx_offset, rp, (float)inv_temp, dp);
    else
      argmax_kernel<T, false><<<M, 1024, 0, st>>>(lp, best_val.data_ptr<float>(), best_idx.data_ptr<int64_t>(), V,
                                                  V_valid, idx_offset, nullptr, 1.f, nullptr);
  };
  if (logits.scalar_type() == at::kBFloat16) launch(__nv_bfloat16());
  else if (logits.scalar_type() == at::kHalf) launch(__half());
  else if (logits.scalar_type() == at::kFloat) launch(float());
  else TORCH_CHECK(false, "argmax: unsupported dtype");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace qfc
