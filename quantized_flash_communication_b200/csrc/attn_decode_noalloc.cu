// Allocation-free entry point of the paged decode attention (declared in qfc_noalloc.h).
//
// No counterpart in the reference.  It runs the same two kernels as attn_decode.cu (split-KV
// partials, then their merge) but takes the fp32 partials from a fixed array compiled
// into the library, so a caller that may not allocate device memory (a runtime with its
// own memory pool, a plugin inside one, C code without PyTorch's allocator) can use it.
// The array's size limits batch x heads x context; larger calls are refused.
#include <cuda_runtime.h>

#include <mutex>

#include "attn_decode_kernels.cuh"
#include "qfc_noalloc.h"

namespace {

using namespace qfc::decode;

// The scratch shared by every call on a device: fp32 partial outputs then (max, sum) pairs.
static __device__ __align__(256) float qfc_noalloc_scratch[QFC_NOALLOC_SCRATCH_BYTES / sizeof(float)];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_scratch[kMaxDevices] = {nullptr};  // guarded by g_mu
int g_sms[kMaxDevices] = {0};               // guarded by g_mu

// Device address of the scratch array on the current device and that device's SM count,
// both looked up once per device under g_mu.  In host code the array's name is only a
// host-side stand-in; passing it to a kernel would be wrong, so the address always comes
// from cudaGetSymbolAddress.
int scratch_for_current_device(float** out, int* sms) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return QFC_NOALLOC_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, qfc_noalloc_scratch) != cudaSuccess || p == nullptr) return QFC_NOALLOC_ERR_CUDA;
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      return QFC_NOALLOC_ERR_CUDA;
    g_sms[dev] = n;
    g_scratch[dev] = static_cast<float*>(p);
  }
  *out = g_scratch[dev];
  *sms = g_sms[dev];
  return QFC_NOALLOC_OK;
}

unsigned long long needed_bytes(int batch, int nq, int hd, int page, int max_pages) {
  const unsigned long long parts = ((unsigned long long)max_pages * page + kPart - 1) / kPart;
  return (unsigned long long)batch * nq * parts * (hd + 2) * sizeof(float);
}

template <typename T, int HD, int G>
int launch(const void* q, const void* kc, const void* vc, const int* bt, const int* sl, void* out, int B, int nq,
           int nkv, int page, int max_pages, float scale, float* scratch, int sms, cudaStream_t st) {
  const int page_shift = ilog2_exact(page);
  if (page_shift < 0) return QFC_NOALLOC_ERR_BAD_ARGS;
  const int max_ctx = max_pages * page;
  const int part_tok = decode_part_tokens(B, nkv, max_ctx, sms);
  const int n_parts = (max_ctx + part_tok - 1) / part_tok;
  float* part_o = scratch;
  float* part_ml = scratch + (size_t)B * nq * n_parts * HD;
  const cudaError_t err = decode_launch<T, HD, G>(static_cast<const T*>(q), static_cast<const T*>(kc),
                                                  static_cast<const T*>(vc), bt, sl, static_cast<T*>(out), part_o,
                                                  part_ml, B, nq, nkv, page_shift, max_pages, n_parts, part_tok, scale,
                                                  st, (int64_t)nq * HD);
  return err == cudaSuccess ? QFC_NOALLOC_OK : QFC_NOALLOC_ERR_CUDA;
}

template <typename T>
int dispatch(int hd, int G, const void* q, const void* kc, const void* vc, const int* bt, const int* sl, void* out,
             int B, int nq, int nkv, int page, int max_pages, float scale, float* scratch, int sms, cudaStream_t st) {
#define QFC_NA(HD_, G_) \
  return launch<T, HD_, G_>(q, kc, vc, bt, sl, out, B, nq, nkv, page, max_pages, scale, scratch, sms, st)
  if (hd == 128) {
    switch (G) {
      case 1: QFC_NA(128, 1);
      case 2: QFC_NA(128, 2);
      case 4: QFC_NA(128, 4);
      case 8: QFC_NA(128, 8);
    }
  } else if (hd == 64) {
    switch (G) {
      case 1: QFC_NA(64, 1);
      case 2: QFC_NA(64, 2);
      case 4: QFC_NA(64, 4);
      case 8: QFC_NA(64, 8);
    }
  }
#undef QFC_NA
  return QFC_NOALLOC_ERR_BAD_ARGS;
}

}  // namespace

extern "C" {

unsigned long long qfc_attn_decode_noalloc_scratch_bytes(int batch, int num_q_heads, int head_dim, int page_size,
                                                         int max_pages_per_seq) {
  return needed_bytes(batch, num_q_heads, head_dim, page_size, max_pages_per_seq);
}

int qfc_attn_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, const int* block_table,
                            const int* seq_lens, void* out, int batch, int num_q_heads, int num_kv_heads, int head_dim,
                            int page_size, int max_pages_per_seq, float scale, int dtype, cudaStream_t stream) {
  if (!q || !k_cache || !v_cache || !block_table || !seq_lens || !out) return QFC_NOALLOC_ERR_BAD_ARGS;
  if (batch <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0 || page_size <= 0 || max_pages_per_seq <= 0)
    return QFC_NOALLOC_ERR_BAD_ARGS;
  if (needed_bytes(batch, num_q_heads, head_dim, page_size, max_pages_per_seq) > QFC_NOALLOC_SCRATCH_BYTES)
    return QFC_NOALLOC_ERR_TOO_LARGE;
  float* scratch = nullptr;
  int sms = 0;
  const int rc = scratch_for_current_device(&scratch, &sms);
  if (rc != QFC_NOALLOC_OK) return rc;
  const int G = num_q_heads / num_kv_heads;
  if (dtype == 0)
    return dispatch<__nv_bfloat16>(head_dim, G, q, k_cache, v_cache, block_table, seq_lens, out, batch, num_q_heads,
                                   num_kv_heads, page_size, max_pages_per_seq, scale, scratch, sms, stream);
  if (dtype == 1)
    return dispatch<__half>(head_dim, G, q, k_cache, v_cache, block_table, seq_lens, out, batch, num_q_heads,
                            num_kv_heads, page_size, max_pages_per_seq, scale, scratch, sms, stream);
  return QFC_NOALLOC_ERR_BAD_ARGS;
}

const char* qfc_noalloc_error_string(int code) {
  switch (code) {
    case QFC_NOALLOC_OK: return "ok";
    case QFC_NOALLOC_ERR_TOO_LARGE:
      return "call needs more scratch than the 16 MiB compiled into the library "
             "(batch * q_heads * ceil(max_pages * page / 256) * (head_dim + 2) * 4 bytes)";
    case QFC_NOALLOC_ERR_BAD_ARGS:
      return "bad arguments (null pointer, head_dim not 64/128, GQA group not 1/2/4/8, page size not a power of two, "
             "dtype)";
    case QFC_NOALLOC_ERR_CUDA: return "a CUDA runtime call failed";
    default: return "unknown error code";
  }
}

}  // extern "C"
