// Host side of the sequence-parallel all-reduce + residual + RMSNorm (allreduce_norm.cuh):
// argument checks, planning and dispatch, unfused (partial tensor in) and fused with the
// row-parallel GEMM's quantize-and-scatter epilogue.
#include <cstdlib>

#include "allreduce_norm.cuh"
#include "scatter.h"

namespace qfc {

// gemm.cu
void gemm_qscatter(const at::Tensor& a, const at::Tensor& b, const ScatterArgs& sc, int p_bits, double timeout_ms);

using namespace ar;
using WsPtr = std::shared_ptr<Workspace>;

// (chunk, need_rs, need_ag, need_os) of a row-blocked call: rank r owns rows
// [r*R, (r+1)*R), R = ceil(M / world).
std::vector<int64_t> ar_plan_rows(int64_t M, int64_t H, int64_t world, int64_t bits, bool scale_fp32) {
  const Plan pl = make_plan_rows(M, H, (int)world, (int)bits, scale_fp32);
  return {pl.chunk, pl.need_rs, pl.need_ag, pl.need_os};
}

namespace ar {
int& norm_warps_per_row() {
  static int wpr = [] {
    const char* e = std::getenv("QFC_NORM_WARPS_PER_ROW");
    const int v = e ? std::atoi(e) : 1;
    return (v == 2 || v == 4 || v == 8) ? v : 1;
  }();
  return wpr;
}
}  // namespace ar

// Warps per row of the sequence-parallel norm kernel (1, 2, 4 or 8); returns the previous value.
int64_t set_norm_warps_per_row(int64_t wpr) {
  TORCH_CHECK(wpr == 1 || wpr == 2 || wpr == 4 || wpr == 8, "set_norm_warps_per_row: 1, 2, 4 or 8");
  const int prev = norm_warps_per_row();
  norm_warps_per_row() = (int)wpr;
  return prev;
}

namespace {

void check_bf16(const at::Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous(), "all_reduce_norm: ", what,
              " must be a contiguous bf16 CUDA tensor");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, "all_reduce_norm: ", what, " must be 16-byte aligned");
}

ARNormParams base_params(const Workspace& w0, const Plan& pl, int64_t M, int64_t H, int W, bool sym, bool scale_fp32,
                         double eps, double timeout_ms) {
  ARNormParams np;
  std::memset(&np, 0, sizeof(np));
  ARParams& prm = np.p;
  prm.status = w0.status_dev();
  prm.n = M * H;
  prm.chunk = pl.chunk;
  prm.rs_off = w0.rs_off();
  prm.ag_off = w0.ag_off();
  prm.os_off = w0.os_off();
  prm.os_bytes = w0.os_bytes();
  prm.slot1 = pl.slot1;
  prm.slot2 = pl.slot2;
  prm.pay1 = pl.pay1;
  prm.pay2 = pl.pay2;
  prm.timeout_ns = (uint64_t)(timeout_ms * 1e6);
  prm.world = W;
  prm.gs = 128;
  prm.gs_shift = 7;
  prm.meta_fp32 = scale_fp32 ? 1 : 0;
  prm.sym = sym ? 1 : 0;
  np.eps = (float)eps;
  np.M = (int)M;
  np.H = (int)H;
  np.R = (int)((M + W - 1) / W);
  return np;
}

}  // namespace

// x = all_gather(rmsnorm(h_shard + reduce_scatter(partial)) * weight), h_shard updated in
// place.  wss / partials / hs / xs: one entry (this rank) or W entries (single-GPU
// emulation).  partial [M, H], h [ceil(M/W), H], x [M, H], weight [H]; bf16, group 128.
void quant_all_reduce_norm(const std::vector<WsPtr>& wss, const std::vector<at::Tensor>& partials,
                           const std::vector<at::Tensor>& hs, const at::Tensor& weight,
                           const std::vector<at::Tensor>& xs, int64_t bits, bool sym, bool scale_fp32,
                           bool quantize_local, double eps, double timeout_ms) {
  TORCH_CHECK(!wss.empty() && wss.size() == partials.size() && partials.size() == hs.size() && hs.size() == xs.size(),
              "all_reduce_norm: need one partial, residual shard and output per workspace");
  const int W = (int)wss[0]->world();
  const bool emulate = wss.size() > 1;
  TORCH_CHECK(!emulate || (int)wss.size() == W, "all_reduce_norm: emulation needs W workspaces");
  TORCH_CHECK(partials[0].dim() == 2, "all_reduce_norm: partial must be [M, H]");
  const int64_t M = partials[0].size(0), H = partials[0].size(1);
  TORCH_CHECK(H % 256 == 0, "all_reduce_norm: H must be a multiple of 256");
  const int64_t R = (M + W - 1) / W;
  check_bf16(weight, "weight");
  TORCH_CHECK(weight.numel() == H, "all_reduce_norm: weight must have H elements");
  for (size_t i = 0; i < partials.size(); ++i) {
    check_bf16(partials[i], "partial");
    check_bf16(hs[i], "residual shard");
    check_bf16(xs[i], "output");
    TORCH_CHECK(partials[i].numel() == M * H && xs[i].numel() == M * H, "all_reduce_norm: size mismatch");
    TORCH_CHECK(hs[i].numel() == R * H, "all_reduce_norm: residual shard must be [ceil(M/W), H]");
    TORCH_CHECK(wss[i]->peers_ready(), "all_reduce_norm: workspace peers not mapped");
  }
  if (M == 0) return;
  c10::cuda::CUDAGuard guard(partials[0].device());
  const int dev = partials[0].get_device();
  const Plan pl = make_plan_rows(M, H, W, (int)bits, scale_fp32);
  const Workspace& w0 = *wss[0];
  TORCH_CHECK(pl.need_rs <= w0.rs_bytes() && pl.need_ag <= w0.ag_bytes(),
              "all_reduce_norm: workspace too small for this message (grow it first)");
  ARNormParams np = base_params(w0, pl, M, H, W, sym, scale_fp32, eps, timeout_ms);
  ARParams& prm = np.p;
  for (int r = 0; r < W; ++r) {
    if (emulate) {
      prm.in[r] = partials[r].data_ptr();
      prm.out[r] = xs[r].data_ptr();
      np.h[r] = hs[r].data_ptr();
      prm.base[r] = wss[r]->base();
      prm.epochs[r] = wss[r]->epochs();
    } else {
      prm.base[r] = w0.peer_base(r);
    }
  }
  if (!emulate) {
    const int rk = (int)w0.rank();
    prm.in[rk] = partials[0].data_ptr();
    prm.out[rk] = xs[0].data_ptr();
    np.h[rk] = hs[0].data_ptr();
    prm.epochs[rk] = w0.epochs();
  }
  prm.rank = emulate ? 0 : (int)w0.rank();
  prm.quantize_local = quantize_local ? 1 : 0;
  np.w = reinterpret_cast<const __nv_bfloat16*>(weight.data_ptr());
  dispatch_norm<false>(np, pl, emulate ? W : 1, dev, at::cuda::getCurrentCUDAStream());
}

// The same with the reduce-scatter fused into the row-parallel GEMM a @ w^T: its epilogue
// quantizes every 128-column group of the output tile into the owner's slot.
void gemm_all_reduce_norm(const WsPtr& ws, const at::Tensor& a, const at::Tensor& w, const at::Tensor& h,
                          const at::Tensor& weight, at::Tensor& x, int64_t bits, bool sym, bool scale_fp32, double eps,
                          double timeout_ms) {
  TORCH_CHECK(ws->peers_ready(), "gemm_all_reduce_norm: workspace peers not mapped");
  const int64_t M = a.size(0), H = w.size(0);
  TORCH_CHECK(H % 256 == 0, "gemm_all_reduce_norm: H must be a multiple of 256");
  const int W = (int)ws->world();
  const int64_t R = (M + W - 1) / W;
  check_bf16(h, "residual shard");
  check_bf16(x, "output");
  check_bf16(weight, "weight");
  TORCH_CHECK(h.numel() == R * H && x.numel() == M * H && weight.numel() == H, "gemm_all_reduce_norm: bad sizes");
  if (M == 0) return;
  c10::cuda::CUDAGuard guard(a.device());
  const int dev = a.get_device();
  const Plan pl = make_plan_rows(M, H, W, (int)bits, scale_fp32);
  TORCH_CHECK(pl.need_rs <= ws->rs_bytes() && pl.need_ag <= ws->ag_bytes(),
              "gemm_all_reduce_norm: workspace too small for this message (grow it first)");
  ScatterArgs sc;
  std::memset(&sc, 0, sizeof(sc));
  for (int r = 0; r < W; ++r) sc.base[r] = ws->peer_base(r);
  sc.rs_off = ws->rs_off();
  sc.slot1 = pl.slot1;
  sc.pay1 = pl.pay1;
  sc.chunk = pl.chunk;  // R * H: owner = row / R
  sc.rank = (int)ws->rank();
  sc.world = W;
  sc.gs_shift = 7;
  sc.sym = sym ? 1 : 0;
  sc.meta_fp32 = scale_fp32 ? 1 : 0;
  sc.epoch = ws->epochs() + ALG_GEMM_RS * kMaxBlocks + 0;
  sc.done_ctas = ws->epochs() + ALG_GEMM_RS * kMaxBlocks + 1;
  gemm_qscatter(a, w, sc, pl.p1, timeout_ms);
  ARNormParams np = base_params(*ws, pl, M, H, W, sym, scale_fp32, eps, timeout_ms);
  ARParams& prm = np.p;
  for (int r = 0; r < W; ++r) prm.base[r] = ws->peer_base(r);
  const int rk = (int)ws->rank();
  prm.out[rk] = x.data_ptr();
  np.h[rk] = h.data_ptr();
  prm.epochs[rk] = ws->epochs();
  prm.gemm_epoch = sc.epoch;
  prm.rank = rk;
  prm.quantize_local = 1;
  np.w = reinterpret_cast<const __nv_bfloat16*>(weight.data_ptr());
  dispatch_norm<true>(np, pl, 1, dev, at::cuda::getCurrentCUDAStream());
}

}  // namespace qfc
