// Paged decode attention for sm_100a (one query token per sequence, GQA).
//
// The reference decodes through Hugging Face's generate() and its KV cache
// (inference.py:29); here the cache is paged per rank ([pages, kv_heads, page, head_dim])
// and attention is split along the context ("flash-decoding"):
//   pass 1: one CTA per (sequence, kv head, partition of 256..4096 tokens, chosen so the
//           grid still fills the GPU); the partition's K and V rows stream through a
//           shared-memory ring (cp.async).  GQA groups of 2..8 heads run both products on
//           the tensor cores (mma.sync m16n8k16, K/V fragments by ldmatrix); multi-head
//           attention splits each row over 4 lanes on the CUDA cores.  An online softmax
//           keeps (max, sum, acc) per head; the CTA writes fp32 partials;
//   pass 2: one warp per (sequence, query head) merges the partitions' partials.
// The partials are scratch memory passed in by the caller.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>

#include <cfloat>

#include "common.cuh"

#include "attn_decode_kernels.cuh"

namespace qfc {

namespace {

using namespace decode;

template <typename T, int HD, int G>
void launch_decode(const at::Tensor& q, const at::Tensor& kc, const at::Tensor& vc, const at::Tensor& bt,
                   const at::Tensor& sl, at::Tensor& out, at::Tensor& part_o, at::Tensor& part_ml, int B, int nq,
                   int nkv, int page_shift, int n_parts, int part_tok, float scale, cudaStream_t st) {
  C10_CUDA_CHECK((decode_launch<T, HD, G>(
      reinterpret_cast<const T*>(q.data_ptr()), reinterpret_cast<const T*>(kc.data_ptr()),
      reinterpret_cast<const T*>(vc.data_ptr()), bt.data_ptr<int>(), sl.data_ptr<int>(),
      reinterpret_cast<T*>(out.data_ptr()), part_o.data_ptr<float>(), part_ml.data_ptr<float>(), B, nq, nkv,
      page_shift, (int)bt.size(1), n_parts, part_tok, scale, st, q.stride(0))));
}

}  // namespace

// q [B, nq*hd] (rows may be strided: a view of the fused qkv activation works in place);
// caches [pages, nkv, page, hd]; block_table [B, max_pages] int32; seq_lens [B] int32;
// out [B, nq*hd].  Context length is bounded by max_pages * page.
void attn_decode_cuda(const at::Tensor& q, const at::Tensor& kc, const at::Tensor& vc, const at::Tensor& bt,
                      const at::Tensor& sl, at::Tensor& out, int64_t nq, int64_t nkv, int64_t hd, double scale) {
  TORCH_CHECK(kc.is_contiguous() && vc.is_contiguous() && out.is_contiguous(),
              "attn_decode: contiguous caches and output required");
  TORCH_CHECK(q.dim() == 2 && q.size(1) == nq * hd && q.stride(1) == 1 && q.stride(0) % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0,
              "attn_decode: q must be [B, nq*hd] with unit column stride and 16-byte aligned rows");
  TORCH_CHECK(bt.scalar_type() == at::kInt && sl.scalar_type() == at::kInt, "attn_decode: int32 block table / lens");
  TORCH_CHECK(nq % nkv == 0 && nq / nkv <= kMaxGroup, "attn_decode: GQA group must be <= 8");
  TORCH_CHECK(hd == 128 || hd == 64, "attn_decode: head_dim must be 64 or 128");
  const int B = (int)q.size(0);
  if (B == 0) return;
  c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int page = (int)kc.size(2);
  const int page_shift = ilog2_exact(page);
  TORCH_CHECK(page_shift >= 0, "attn_decode: page size must be a power of two");
  const int max_ctx = (int)bt.size(1) * page;
  const int part_tok = decode_part_tokens(B, (int)nkv, max_ctx, at::cuda::getCurrentDeviceProperties()->multiProcessorCount);
  const int n_parts = (max_ctx + part_tok - 1) / part_tok;
  at::Tensor part_o = at::empty({(int64_t)B * nq * n_parts * hd}, q.options().dtype(at::kFloat));
  at::Tensor part_ml = at::empty({(int64_t)B * nq * n_parts * 2}, q.options().dtype(at::kFloat));
  const int G = (int)(nq / nkv);
  auto go = [&](auto tag) {
    using T = decltype(tag);
#define QFC_DEC(HD_, G_) launch_decode<T, HD_, G_>(q, kc, vc, bt, sl, out, part_o, part_ml, B, (int)nq, (int)nkv, page_shift, n_parts, part_tok, (float)scale, st)
    if (hd == 128) {
      switch (G) {
        case 1: QFC_DEC(128, 1); break;
        case 2: QFC_DEC(128, 2); break;
        case 4: QFC_DEC(128, 4); break;
        case 8: QFC_DEC(128, 8); break;
        default: TORCH_CHECK(false, "attn_decode: unsupported GQA group ", G);
      }
    } else {
      switch (G) {
        case 1: QFC_DEC(64, 1); break;
        case 2: QFC_DEC(64, 2); break;
        case 4: QFC_DEC(64, 4); break;
        case 8: QFC_DEC(64, 8); break;
        default: TORCH_CHECK(false, "attn_decode: unsupported GQA group ", G);
      }
    }
#undef QFC_DEC
  };
  if (q.scalar_type() == at::kBFloat16) go(__nv_bfloat16());
  else if (q.scalar_type() == at::kHalf) go(__half());
  else TORCH_CHECK(false, "attn_decode: bf16 or fp16 required");
}

}  // namespace qfc
