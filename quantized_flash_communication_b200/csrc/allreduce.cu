// Host side of the fused quantized all-reduce: planning, argument checks, dispatch.
// The kernels are in allreduce.cuh and are instantiated per input dtype in
// allreduce_inst_*.cu (compiled in parallel).
#include <cfloat>
#include <cstdlib>

#include "allreduce.cuh"
#include "scatter.h"

namespace qfc {
namespace ar {
#define QFC_AR_DECL(I, O)                                                                                  \
  extern template void dispatch_bits<I, O>(const ARParams&, const Plan&, bool, int64_t, int, int, cudaStream_t);
QFC_AR_DECL(__nv_bfloat16, __nv_bfloat16)
QFC_AR_DECL(__nv_bfloat16, __half)
QFC_AR_DECL(__half, __half)
QFC_AR_DECL(float, float)
QFC_AR_DECL(float, __half)
#undef QFC_AR_DECL
extern template void dispatch_gemm_reduce<__nv_bfloat16, __nv_bfloat16>(const ARParams&, const Plan&, int64_t, int,
                                                                        cudaStream_t);
}  // namespace ar

// gemm.cu
void gemm_qscatter(const at::Tensor& a, const at::Tensor& b, const ScatterArgs& sc, int p_bits, double timeout_ms);

using namespace ar;

using WsPtr = std::shared_ptr<Workspace>;

namespace ar {
int& two_shot_stages() {
  static int stages = [] {
    const char* e = std::getenv("QFC_AR_STAGES");
    return (e && e[0] == '2') ? 2 : 1;
  }();
  return stages;
}
}  // namespace ar

// Stages of the 16-per-lane two-shot all-reduce (1 or 2); returns the previous value.
int64_t set_two_shot_stages(int64_t stages) {
  TORCH_CHECK(stages == 1 || stages == 2, "set_two_shot_stages: 1 or 2");
  const int prev = two_shot_stages();
  two_shot_stages() = (int)stages;
  return prev;
}

// Region sizes a call needs: (chunk, need_rs, need_ag, need_os) for the given algorithm.
std::vector<int64_t> ar_plan(int64_t n, int64_t world, int64_t bits, int64_t gs, bool scale_fp32,
                             int64_t in_elem_size, bool one_shot) {
  const Plan pl = make_plan(n, (int)world, (int)bits, (int)gs, scale_fp32, (int)in_elem_size, one_shot);
  return {pl.chunk, pl.need_rs, pl.need_ag, pl.need_os};
}

// wss: one workspace (normal, this rank) or W workspaces (single-GPU emulation, one per
// emulated rank, all on the current device).  ins / outs: one tensor per entry of wss.
void quant_all_reduce(const std::vector<WsPtr>& wss, const std::vector<at::Tensor>& ins,
                      const std::vector<at::Tensor>& outs, int64_t bits, int64_t gs, bool sym,
                      bool scale_fp32, bool one_shot, bool quantize_local, double timeout_ms) {
  TORCH_CHECK(!wss.empty() && wss.size() == ins.size() && ins.size() == outs.size(),
              "quant_all_reduce: need one input and one output per workspace");
  const int W = (int)wss[0]->world();
  const bool emulate = wss.size() > 1;
  TORCH_CHECK(!emulate || (int)wss.size() == W, "quant_all_reduce: emulation needs W workspaces");
  TORCH_CHECK(gs >= 8 && gs <= 256 && (gs & (gs - 1)) == 0,
              "quant_all_reduce: fused kernel supports power-of-two group sizes 8..256, got ", gs);
  const int64_t n = ins[0].numel();
  const auto in_dt = ins[0].scalar_type();
  const auto out_dt = outs[0].scalar_type();
  for (size_t i = 0; i < ins.size(); ++i) {
    TORCH_CHECK(ins[i].is_cuda() && outs[i].is_cuda(), "quant_all_reduce: CUDA tensors required");
    TORCH_CHECK(ins[i].numel() == n && outs[i].numel() == n, "quant_all_reduce: size mismatch");
    TORCH_CHECK(ins[i].is_contiguous() && outs[i].is_contiguous(), "quant_all_reduce: contiguous tensors required");
    TORCH_CHECK(ins[i].scalar_type() == in_dt && outs[i].scalar_type() == out_dt, "quant_all_reduce: dtype mismatch");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(ins[i].data_ptr()) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(outs[i].data_ptr()) % 16 == 0,
                "quant_all_reduce: tensors must be 16-byte aligned");
    TORCH_CHECK(wss[i]->peers_ready(), "quant_all_reduce: workspace peers not mapped");
  }
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(ins[0].device());
  const int dev = ins[0].get_device();
  const int in_elem = (int)ins[0].element_size();
  const Plan pl = make_plan(n, W, (int)bits, (int)gs, scale_fp32, in_elem, one_shot);
  const Workspace& w0 = *wss[0];
  TORCH_CHECK(pl.need_rs <= w0.rs_bytes() && pl.need_ag <= w0.ag_bytes() && pl.need_os <= w0.os_bytes(),
              "quant_all_reduce: workspace too small for this message (grow it first)");
  ARParams prm;
  std::memset(&prm, 0, sizeof(prm));
  for (int r = 0; r < W; ++r) {
    if (emulate) {
      prm.in[r] = ins[r].data_ptr();
      prm.out[r] = outs[r].data_ptr();
      prm.base[r] = wss[r]->base();
      prm.epochs[r] = wss[r]->epochs();
    } else {
      prm.base[r] = w0.peer_base(r);
    }
  }
  if (!emulate) {
    const int rk = (int)w0.rank();
    prm.in[rk] = ins[0].data_ptr();
    prm.out[rk] = outs[0].data_ptr();
    prm.epochs[rk] = w0.epochs();
  }
  prm.status = w0.status_dev();
  prm.n = n;
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
  prm.rank = emulate ? 0 : (int)w0.rank();
  prm.gs = (int)gs;
  prm.gs_shift = __builtin_ctz((unsigned)gs);
  prm.meta_fp32 = scale_fp32 ? 1 : 0;
  prm.sym = sym ? 1 : 0;
  prm.quantize_local = quantize_local ? 1 : 0;
  const int64_t units = pl.chunk >> 8;
  const int W_emul = emulate ? W : 1;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto go = [&](auto in_tag, auto out_tag) {
    dispatch_bits<decltype(in_tag), decltype(out_tag)>(prm, pl, one_shot, units, W_emul, dev, st);
  };
  if (in_dt == at::kBFloat16 && out_dt == at::kBFloat16) go(__nv_bfloat16(), __nv_bfloat16());
  else if (in_dt == at::kBFloat16 && out_dt == at::kHalf) go(__nv_bfloat16(), __half());
  else if (in_dt == at::kHalf && out_dt == at::kHalf) go(__half(), __half());
  else if (in_dt == at::kFloat && out_dt == at::kFloat) go(float(), float());
  else if (in_dt == at::kFloat && out_dt == at::kHalf) go(float(), __half());
  else TORCH_CHECK(false, "quant_all_reduce: unsupported (input, output) dtype pair ", in_dt, ", ", out_dt);
}

// out = all_reduce(a @ w^T) over the workspace's ranks, with the quantize-and-scatter of the
// two-shot all-reduce fused into the GEMM epilogue (one GEMM launch + one reduce-gather
// launch).  a [M, K], w [N, K] bf16; out [M, N] bf16.  Group size 128, bits 16/8/6/4.
void gemm_all_reduce(const WsPtr& ws, const at::Tensor& a, const at::Tensor& w, at::Tensor& out, int64_t bits,
                     int64_t gs, bool sym, bool scale_fp32, double timeout_ms) {
  TORCH_CHECK(gs == 128, "gemm_all_reduce: group size 128 only");
  TORCH_CHECK(ws->peers_ready(), "gemm_all_reduce: workspace peers not mapped");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.is_contiguous(), "gemm_all_reduce: bf16 out");
  const int64_t M = a.size(0), N = w.size(0);
  TORCH_CHECK(out.numel() == M * N, "gemm_all_reduce: bad output size");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "gemm_all_reduce: out must be 16-byte aligned");
  const int64_t n = M * N;
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(a.device());
  const int dev = a.get_device();
  const int W = (int)ws->world();
  const Plan pl = make_plan(n, W, (int)bits, (int)gs, scale_fp32, 2, false);
  TORCH_CHECK(pl.need_rs <= ws->rs_bytes() && pl.need_ag <= ws->ag_bytes(),
              "gemm_all_reduce: workspace too small for this message (grow it first)");
  ScatterArgs sc;
  std::memset(&sc, 0, sizeof(sc));
  for (int r = 0; r < W; ++r) sc.base[r] = ws->peer_base(r);
  sc.rs_off = ws->rs_off();
  sc.slot1 = pl.slot1;
  sc.pay1 = pl.pay1;
  sc.chunk = pl.chunk;
  sc.rank = (int)ws->rank();
  sc.world = W;
  sc.gs_shift = 7;
  sc.sym = sym ? 1 : 0;
  sc.meta_fp32 = scale_fp32 ? 1 : 0;
  sc.epoch = ws->epochs() + ALG_GEMM_RS * kMaxBlocks + 0;
  sc.done_ctas = ws->epochs() + ALG_GEMM_RS * kMaxBlocks + 1;
  gemm_qscatter(a, w, sc, pl.p1, timeout_ms);
  ARParams prm;
  std::memset(&prm, 0, sizeof(prm));
  for (int r = 0; r < W; ++r) prm.base[r] = ws->peer_base(r);
  const int rk = (int)ws->rank();
  prm.out[rk] = out.data_ptr();
  prm.epochs[rk] = ws->epochs();
  prm.gemm_epoch = sc.epoch;
  prm.status = ws->status_dev();
  prm.n = n;
  prm.chunk = pl.chunk;
  prm.rs_off = ws->rs_off();
  prm.ag_off = ws->ag_off();
  prm.os_off = ws->os_off();
  prm.os_bytes = ws->os_bytes();
  prm.slot1 = pl.slot1;
  prm.slot2 = pl.slot2;
  prm.pay1 = pl.pay1;
  prm.pay2 = pl.pay2;
  prm.timeout_ns = (uint64_t)(timeout_ms * 1e6);
  prm.world = W;
  prm.rank = rk;
  prm.gs = (int)gs;
  prm.gs_shift = 7;
  prm.meta_fp32 = scale_fp32 ? 1 : 0;
  prm.sym = sym ? 1 : 0;
  prm.quantize_local = 1;
  dispatch_gemm_reduce<__nv_bfloat16, __nv_bfloat16>(prm, pl, pl.chunk >> 8, dev, at::cuda::getCurrentCUDAStream());
}


// ---------------------------------------------------------------------------------------
// Cross-rank argmax of a vocabulary-parallel head (one kernel)
// ---------------------------------------------------------------------------------------
// Every rank holds, per row, the (score, global index) of its best vocabulary entry
// (greedy logit or sampled Gumbel score).  Thread t pushes row t's pair into every peer's
// argmax slot, the CTA publishes one flag per peer, waits (bounded) for the W - 1 peers'
// flags and writes the winner: the highest score, ties to the lower rank, i.e. to the
// lower vocabulary index.  Slots are double-buffered by epoch parity: a rank can only
// start call k + 1 after every peer has started call k, so no peer is still reading the
// buffer it writes.  Replaces the reference's full-vocabulary head on every rank
// (Hugging Face lm_head in main.py:190-194) with one small exchange.
namespace {
__global__ void __launch_bounds__(512) argmax_gather_kernel(const __grid_constant__ ARParams p, const float* val,
                                                            const int64_t* idx, int64_t* out, int rows,
                                                            int64_t argmax_off) {
  const int rank = p.rank, W = p.world;
  const int t = threadIdx.x;
  char* my = p.base[rank];
  uint32_t* ep = p.epochs[rank] + ALG_ARGMAX * kMaxBlocks;
  __shared__ uint32_t s_e;
  __shared__ int s_abort;
  if (t == 0) {
    s_e = *ep + 1u;
    s_abort = 0;
  }
  __syncthreads();
  const uint32_t e = s_e;
  const int64_t region = argmax_off + (int64_t)(e & 1u) * (kArgmaxBytes / 2);
  float v = -FLT_MAX;
  int32_t ix = -1;
  if (t < rows) {
    v = val[t];
    ix = (int32_t)idx[t];
    const uint2 pair = make_uint2(__float_as_uint(v), (uint32_t)ix);
    for (int j = 0; j < W; ++j) {
      if (j == rank) continue;
      *reinterpret_cast<uint2*>(p.base[j] + region + ((int64_t)rank * kArgmaxRows + t) * 8) = pair;
    }
  }
  __syncthreads();
  if (t < W && t != rank) st_release_sys(flag_at(p.base[t], PH_ARGMAX, 0, rank), e);
  if (!wait_sources(p, my, PH_ARGMAX, 0, rank, W, e, true, &s_abort)) return;
  if (t < rows) {
    float best = -FLT_MAX;
    int32_t bi = -1;
    for (int r = 0; r < W; ++r) {  // rank order = vocabulary order: the first maximum wins
      float rv;
      int32_t ri;
      if (r == rank) {
        rv = v;
        ri = ix;
      } else {
        const uint2 pr = __ldcg(reinterpret_cast<const uint2*>(my + region + ((int64_t)r * kArgmaxRows + t) * 8));
        rv = __uint_as_float(pr.x);
        ri = (int32_t)pr.y;
      }
      if (ri >= 0 && (bi < 0 || rv > best)) {
        best = rv;
        bi = ri;
      }
    }
    out[t] = bi;
  }
  if (t == 0) *ep = e;
}
}  // namespace

// out[t] = the global argmax of row t over every rank's (val[t], idx[t]).  rows <= 512.
void argmax_gather(const WsPtr& ws, const at::Tensor& val, const at::Tensor& idx, at::Tensor& out,
                   double timeout_ms) {
  TORCH_CHECK(ws->peers_ready(), "argmax_gather: workspace peers not mapped");
  TORCH_CHECK(val.is_cuda() && val.scalar_type() == at::kFloat && val.is_contiguous(), "argmax_gather: fp32 val");
  TORCH_CHECK(idx.scalar_type() == at::kLong && idx.is_contiguous() && out.scalar_type() == at::kLong &&
                  out.is_contiguous(), "argmax_gather: int64 idx / out");
  const int64_t rows = val.numel();
  TORCH_CHECK(idx.numel() == rows && out.numel() == rows, "argmax_gather: size mismatch");
  TORCH_CHECK(rows <= kArgmaxRows, "argmax_gather: at most ", kArgmaxRows, " rows");
  if (rows == 0) return;
  c10::cuda::CUDAGuard guard(val.device());
  ARParams prm;
  std::memset(&prm, 0, sizeof(prm));
  const int W = (int)ws->world();
  for (int r = 0; r < W; ++r) prm.base[r] = ws->peer_base(r);
  prm.rank = (int)ws->rank();
  prm.world = W;
  prm.epochs[prm.rank] = ws->epochs();
  prm.status = ws->status_dev();
  prm.timeout_ns = (uint64_t)(timeout_ms * 1e6);
  const int threads = std::max(32, (int)((rows + 31) / 32 * 32));
  argmax_gather_kernel<<<1, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      prm, val.data_ptr<float>(), idx.data_ptr<int64_t>(), out.data_ptr<int64_t>(), (int)rows, ws->argmax_off());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace qfc
