// Python bindings of the native extension (quantized_flash_communication_b200._C).
#include <pybind11/stl.h>
#include <torch/extension.h>

#include <memory>

#include "nvtx_range.h"
#include "workspace.h"

namespace qfc {
// quant_kernels.cu
std::vector<at::Tensor> quantize_cuda(const at::Tensor& x, int64_t bits, int64_t group_size, bool sym,
                                      bool scale_fp32);
at::Tensor dequantize_cuda(const at::Tensor& q, const at::Tensor& s, const at::Tensor& z, int64_t group_size,
                           at::ScalarType out_dtype);
at::Tensor pack_int4_cuda(const at::Tensor& codes);
at::Tensor unpack_int4_cuda(const at::Tensor& words, int64_t numel);
// quant_cpu.cpp
std::vector<at::Tensor> quantize_cpu(const at::Tensor& x, int64_t bits, int64_t group_size, bool sym,
                                     bool scale_fp32);
at::Tensor dequantize_cpu(const at::Tensor& q, const at::Tensor& s, const at::Tensor& z, int64_t group_size,
                          at::ScalarType out_dtype);
at::Tensor pack_int4_cpu(const at::Tensor& codes);
at::Tensor unpack_int4_cpu(const at::Tensor& words, int64_t numel);
// allreduce.cu
std::vector<int64_t> ar_plan(int64_t n, int64_t world, int64_t bits, int64_t gs, bool scale_fp32,
                             int64_t in_elem_size, bool one_shot);
void quant_all_reduce(const std::vector<std::shared_ptr<Workspace>>& wss, const std::vector<at::Tensor>& ins,
                      const std::vector<at::Tensor>& outs, int64_t bits, int64_t gs, bool sym, bool scale_fp32,
                      bool one_shot, bool quantize_local, double timeout_ms);
void gemm_all_reduce(const std::shared_ptr<Workspace>& ws, const at::Tensor& a, const at::Tensor& w, at::Tensor& out,
                     int64_t bits, int64_t gs, bool sym, bool scale_fp32, double timeout_ms);
void argmax_gather(const std::shared_ptr<Workspace>& ws, const at::Tensor& val, const at::Tensor& idx, at::Tensor& out,
                   double timeout_ms);
// allreduce_norm.cu
std::vector<int64_t> ar_plan_rows(int64_t M, int64_t H, int64_t world, int64_t bits, bool scale_fp32);
void quant_all_reduce_norm(const std::vector<std::shared_ptr<Workspace>>& wss, const std::vector<at::Tensor>& partials,
                           const std::vector<at::Tensor>& hs, const at::Tensor& weight,
                           const std::vector<at::Tensor>& xs, int64_t bits, bool sym, bool scale_fp32,
                           bool quantize_local, double eps, double timeout_ms);
int64_t set_norm_warps_per_row(int64_t wpr);
int64_t set_two_shot_stages(int64_t stages);
void gemm_all_reduce_norm(const std::shared_ptr<Workspace>& ws, const at::Tensor& a, const at::Tensor& w,
                          const at::Tensor& h, const at::Tensor& weight, at::Tensor& x, int64_t bits, bool sym,
                          bool scale_fp32, double eps, double timeout_ms);
// gemm.cu
at::Tensor gemm_bf16(const at::Tensor& a, const at::Tensor& b, const c10::optional<at::Tensor>& out, int64_t epi,
                     const c10::optional<at::Tensor>& residual, double timeout_ms, int64_t max_ctas);
void gemm_qkv_rope(const at::Tensor& a, const at::Tensor& w, at::Tensor& out, const at::Tensor& pos,
                   const at::Tensor& cos_sin, const c10::optional<at::Tensor>& k_cache,
                   const c10::optional<at::Tensor>& v_cache, const c10::optional<at::Tensor>& slots, int64_t nq,
                   int64_t nkv, double timeout_ms);
int64_t gemm_status(bool clear);
bool set_gemv(bool on);
// layers.cu
void rmsnorm_cuda(const at::Tensor& x, const c10::optional<at::Tensor>& residual, const at::Tensor& w, at::Tensor& y,
                  double eps);
void rope_kv_cuda(at::Tensor& qkv, const at::Tensor& pos, const at::Tensor& cos_sin,
                  const c10::optional<at::Tensor>& k_cache, const c10::optional<at::Tensor>& v_cache,
                  const c10::optional<at::Tensor>& slot_mapping, int64_t nq, int64_t nkv, int64_t hd);
void rope_kv_decode_cuda(at::Tensor& qkv, const at::Tensor& cos_sin, at::Tensor& k_cache, at::Tensor& v_cache,
                         const at::Tensor& block_table, const at::Tensor& seq_lens, int64_t nq, int64_t nkv,
                         int64_t hd);
void silu_mul_cuda(const at::Tensor& gu, at::Tensor& out);
void embedding_cuda(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out, int64_t vocab_start);
void argmax_cuda(const at::Tensor& logits, at::Tensor& best_val, at::Tensor& best_idx, int64_t idx_offset,
                 int64_t valid, const c10::optional<at::Tensor>& rng, double inv_temp,
                 const c10::optional<at::Tensor>& done);
// attn_decode.cu
void attn_decode_cuda(const at::Tensor& q, const at::Tensor& kc, const at::Tensor& vc, const at::Tensor& bt,
                      const at::Tensor& sl, at::Tensor& out, int64_t nq, int64_t nkv, int64_t hd, double scale);
// attn_prefill.cu
void attn_prefill_cuda(const at::Tensor& qkv, at::Tensor& out, int64_t B, int64_t S, int64_t nq, int64_t nkv,
                       int64_t hd, double scale);
int64_t attn_status(bool clear);
bool set_attn_packed(bool on);
void attn_exp2_poly(const at::Tensor& x, at::Tensor& y, bool pairs);
}  // namespace qfc

namespace py = pybind11;

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "B200-native kernels for quantized tensor-parallel communication";
  m.def("set_nvtx", &qfc::set_nvtx, "turn the NVTX range around every CUDA op on or off", py::arg("on"));
  m.def("nvtx_enabled", &qfc::nvtx_enabled);

  m.def("quantize", qfc::traced("quantize", &qfc::quantize_cuda), "blockwise quantize (CUDA)", py::arg("x"), py::arg("bits"),
        py::arg("group_size"), py::arg("sym"), py::arg("scale_fp32"));
  m.def("dequantize", qfc::traced("dequantize", &qfc::dequantize_cuda), "blockwise dequantize (CUDA)", py::arg("q"), py::arg("s"),
        py::arg("z"), py::arg("group_size"), py::arg("out_dtype"));
  m.def("pack_int4", qfc::traced("pack_int4", &qfc::pack_int4_cuda), "pack 4-bit codes into int32 words (CUDA)");
  m.def("unpack_int4", qfc::traced("unpack_int4", &qfc::unpack_int4_cuda), "unpack int32 words into fp16 codes (CUDA)");

  m.def("quantize_cpu", &qfc::quantize_cpu, "blockwise quantize (C++ CPU oracle)");
  m.def("dequantize_cpu", &qfc::dequantize_cpu, "blockwise dequantize (C++ CPU oracle)");
  m.def("pack_int4_cpu", &qfc::pack_int4_cpu, "pack 4-bit codes (C++ CPU oracle)");
  m.def("unpack_int4_cpu", &qfc::unpack_int4_cpu, "unpack 4-bit codes to uint8 (C++ CPU oracle)");

  py::class_<qfc::Workspace, std::shared_ptr<qfc::Workspace>>(m, "Workspace")
      .def(py::init<int64_t, int64_t, int64_t, int64_t, int64_t, int64_t>(), py::arg("device"),
           py::arg("rank"), py::arg("world"), py::arg("rs_bytes"), py::arg("ag_bytes"), py::arg("os_bytes"))
      .def("ipc_handle", [](const qfc::Workspace& w) { return py::bytes(w.ipc_handle()); })
      .def("open_peers", &qfc::Workspace::open_peers)
      .def("set_peer_ptrs", &qfc::Workspace::set_peer_ptrs)
      .def("status", &qfc::Workspace::status)
      .def("clear_status", &qfc::Workspace::clear_status)
      .def_property_readonly("local_ptr", &qfc::Workspace::local_ptr)
      .def_property_readonly("device", &qfc::Workspace::device)
      .def_property_readonly("rank", &qfc::Workspace::rank)
      .def_property_readonly("world", &qfc::Workspace::world)
      .def_property_readonly("rs_bytes", &qfc::Workspace::rs_bytes)
      .def_property_readonly("ag_bytes", &qfc::Workspace::ag_bytes)
      .def_property_readonly("os_bytes", &qfc::Workspace::os_bytes)
      .def_property_readonly("peers_ready", &qfc::Workspace::peers_ready);

  m.def("gemm_qkv_rope", qfc::traced("gemm_qkv_rope", &qfc::gemm_qkv_rope), "qkv GEMM with RoPE and the KV-cache write in its epilogue",
        py::arg("a"), py::arg("w"), py::arg("out"), py::arg("pos"), py::arg("cos_sin"), py::arg("k_cache") = py::none(),
        py::arg("v_cache") = py::none(), py::arg("slots") = py::none(), py::arg("nq"), py::arg("nkv"),
        py::arg("timeout_ms") = 10000.0);
  m.def("gemm_bf16", qfc::traced("gemm_bf16", &qfc::gemm_bf16), "tcgen05 GEMM a @ b^T with fused epilogue (0 store, 1 swiglu, 2 residual)",
        py::arg("a"), py::arg("b"), py::arg("out") = py::none(), py::arg("epi") = 0,
        py::arg("residual") = py::none(), py::arg("timeout_ms") = 10000.0, py::arg("max_ctas") = 0);
  m.def("gemm_status", &qfc::gemm_status, py::arg("clear") = false);
  m.def("set_gemv", &qfc::set_gemv,
        "weight-streaming kernel for GEMMs of at most 8 rows (off by default); returns the previous value",
        py::arg("on"));
  m.def("rmsnorm", qfc::traced("rmsnorm", &qfc::rmsnorm_cuda), py::arg("x"), py::arg("residual"), py::arg("w"), py::arg("y"), py::arg("eps"));
  m.def("rope_kv_decode", qfc::traced("rope_kv_decode", &qfc::rope_kv_decode_cuda), "RoPE + paged KV write of one decode token per sequence");
  m.def("rope_kv", qfc::traced("rope_kv", &qfc::rope_kv_cuda), py::arg("qkv"), py::arg("pos"), py::arg("cos_sin"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("slot_mapping"), py::arg("nq"), py::arg("nkv"), py::arg("hd"));
  m.def("silu_mul", qfc::traced("silu_mul", &qfc::silu_mul_cuda));
  m.def("embedding", qfc::traced("embedding", &qfc::embedding_cuda));
  m.def("argmax", qfc::traced("argmax", &qfc::argmax_cuda), py::arg("logits"), py::arg("best_val"), py::arg("best_idx"),
        py::arg("idx_offset") = 0, py::arg("valid") = -1, py::arg("rng") = py::none(), py::arg("inv_temp") = 1.0,
        py::arg("done") = py::none());
  m.def("attn_decode", qfc::traced("attn_decode", &qfc::attn_decode_cuda), "paged split-KV decode attention");
  m.def("attn_prefill", qfc::traced("attn_prefill", &qfc::attn_prefill_cuda), "causal flash prefill attention (tcgen05)");
  m.def("attn_exp2_poly", qfc::traced("attn_exp2_poly", &qfc::attn_exp2_poly),
        "2^x as the prefill softmax evaluates it on the FMA pipe", py::arg("x"), py::arg("y"),
        py::arg("pairs") = false);
  m.def("attn_status", &qfc::attn_status, py::arg("clear") = false);
  m.def("set_attn_packed", &qfc::set_attn_packed,
        "prefill attention softmax with packed two-lane fp32 arithmetic (off by default); returns the previous value",
        py::arg("on"));

  m.def("ar_plan", &qfc::ar_plan, "region sizes a quantized all-reduce call needs");
  m.def("quant_all_reduce", qfc::traced("quant_all_reduce", &qfc::quant_all_reduce), "fused quantized all-reduce over peer memory",
        py::arg("workspaces"), py::arg("ins"), py::arg("outs"), py::arg("bits"), py::arg("group_size"),
        py::arg("sym"), py::arg("scale_fp32"), py::arg("one_shot"), py::arg("quantize_local"),
        py::arg("timeout_ms"));
  m.def("argmax_gather", qfc::traced("argmax_gather", &qfc::argmax_gather), "cross-rank argmax of (score, index) pairs (one kernel)");
  m.def("gemm_all_reduce", qfc::traced("gemm_all_reduce", &qfc::gemm_all_reduce),
        "all_reduce(a @ w^T) with the quantize-and-scatter fused into the GEMM epilogue", py::arg("workspace"),
        py::arg("a"), py::arg("w"), py::arg("out"), py::arg("bits"), py::arg("group_size"), py::arg("sym"),
        py::arg("scale_fp32"), py::arg("timeout_ms"));
  m.def("set_two_shot_stages", &qfc::set_two_shot_stages,
        "stages per CTA of the 16-per-lane two-shot all-reduce (1 or 2); returns the previous value",
        py::arg("stages"));
  m.def("set_norm_warps_per_row", &qfc::set_norm_warps_per_row,
        "warps per row of the sequence-parallel all-reduce + norm kernel (1, 2, 4 or 8); returns the previous value",
        py::arg("wpr"));
  m.def("ar_plan_rows", &qfc::ar_plan_rows, "region sizes of a row-blocked (sequence-parallel) all-reduce + norm");
  m.def("quant_all_reduce_norm", qfc::traced("quant_all_reduce_norm", &qfc::quant_all_reduce_norm),
        "x = all_gather(rmsnorm(h_shard += reduce_scatter(partial)) * w), one kernel over peer memory",
        py::arg("workspaces"), py::arg("partials"), py::arg("residual_shards"), py::arg("weight"), py::arg("outs"),
        py::arg("bits"), py::arg("sym"), py::arg("scale_fp32"), py::arg("quantize_local"), py::arg("eps"),
        py::arg("timeout_ms"));
  m.def("gemm_all_reduce_norm", qfc::traced("gemm_all_reduce_norm", &qfc::gemm_all_reduce_norm),
        "the same with the reduce-scatter fused into the row-parallel GEMM's epilogue", py::arg("workspace"),
        py::arg("a"), py::arg("w"), py::arg("residual_shard"), py::arg("weight"), py::arg("out"), py::arg("bits"),
        py::arg("sym"), py::arg("scale_fp32"), py::arg("eps"), py::arg("timeout_ms"));
}
