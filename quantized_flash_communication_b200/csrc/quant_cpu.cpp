// C++ CPU oracle of the blockwise quantizer and the INT4 nibble packer.
//
// A host restatement of the arithmetic in common.cuh (QMath, dq, pack_nibbles) and of
// the torch specification in quantization.py.  It serves two purposes: a native
// reference that the CUDA kernels are compared against bit-for-bit on small cases, and
// a CPU implementation of the reference's quantizer API for CPU tensors (the reference
// itself only runs on CUDA, kernels.py / kernels_jit.py).  Built with
// -ffp-contract=off so that no multiply-add is fused.
#include <ATen/ATen.h>

#include <cmath>
#include <cstdint>
#include <vector>

namespace qfc {

namespace {

struct GroupParams {
  float s, inv, z;
};

GroupParams group_params(float mn, float mx, int bits, bool sym) {
  const float qmax = float((1 << bits) - 1);
  GroupParams p;
  if (sym) {
    const float a = std::fmax(-mn, mx);
    p.s = a / (qmax * 0.5f);
    if (p.s < 1e-9f) p.s = 1.f;
    p.inv = 1.f / p.s;
    p.z = (qmax + 1.f) * 0.5f;
  } else {
    p.s = (mx - mn) / qmax;
    if (p.s < 1e-9f) p.s = 1.f;
    p.inv = 1.f / p.s;
    p.z = std::fmin(std::fmax(std::round(-mn * p.inv), 0.f), qmax);
  }
  return p;
}

constexpr int kNibbleOrder[8] = {0, 2, 4, 6, 1, 3, 5, 7};

}  // namespace

std::vector<at::Tensor> quantize_cpu(const at::Tensor& x_in, int64_t bits, int64_t group_size, bool sym,
                                     bool scale_fp32) {
  TORCH_CHECK(bits == 8 || bits == 4, "quantize_cpu: bits must be 8 or 4");
  TORCH_CHECK(group_size >= 1, "quantize_cpu: bad group size");
  at::Tensor x = x_in.reshape({-1}).to(at::kFloat).contiguous().cpu();
  const int64_t n = x.numel();
  const int64_t gs = group_size;
  const int64_t G = (n + gs - 1) / gs;
  const float qmax = float((1 << bits) - 1);
  at::Tensor q = at::empty({n}, at::kByte);
  at::Tensor s = at::empty({G}, at::kFloat);
  at::Tensor z = at::empty({G}, at::kFloat);
  const float* xp = x.data_ptr<float>();
  uint8_t* qp = q.data_ptr<uint8_t>();
  float* sp = s.data_ptr<float>();
  float* zp = z.data_ptr<float>();
  for (int64_t g = 0; g < G; ++g) {
    const int64_t b = g * gs;
    float mn = 0.f, mx = 0.f;
    for (int64_t i = 0; i < gs; ++i) {
      const float v = (b + i < n) ? xp[b + i] : 0.f;  // zero padding of the tail group
      if (i == 0) {
        mn = v;
        mx = v;
      } else {
        mn = std::fmin(mn, v);
        mx = std::fmax(mx, v);
      }
    }
    const GroupParams p = group_params(mn, mx, (int)bits, sym);
    for (int64_t i = 0; i < gs && b + i < n; ++i) {
      const float c = std::fmin(std::fmax(std::round(xp[b + i] * p.inv) + p.z, 0.f), qmax);
      qp[b + i] = (uint8_t)c;
    }
    sp[g] = p.s;
    zp[g] = p.z;
  }
  at::Tensor s_out = scale_fp32 ? s : s.to(at::kHalf);
  return {q, s_out, z.to(at::kHalf)};
}

at::Tensor dequantize_cpu(const at::Tensor& q_in, const at::Tensor& s_in, const at::Tensor& z_in,
                          int64_t group_size, at::ScalarType out_dtype) {
  at::Tensor q = q_in.reshape({-1}).contiguous().cpu();
  if (q.scalar_type() == at::kChar) q = q.view(at::kByte);
  at::Tensor qf = q.to(at::kFloat);
  at::Tensor s = s_in.reshape({-1}).to(at::kFloat).contiguous().cpu();
  at::Tensor z = z_in.reshape({-1}).to(at::kFloat).contiguous().cpu();
  const int64_t n = qf.numel();
  at::Tensor out = at::empty({n}, at::kFloat);
  const float* qp = qf.data_ptr<float>();
  const float* sp = s.data_ptr<float>();
  const float* zp = z.data_ptr<float>();
  float* op = out.data_ptr<float>();
  for (int64_t i = 0; i < n; ++i) {
    const int64_t g = i / group_size;
    const float d = qp[i] - zp[g];
    op[i] = d * sp[g];
  }
  return out.to(out_dtype);
}

at::Tensor pack_int4_cpu(const at::Tensor& codes_in) {
  at::Tensor c = codes_in.reshape({-1}).contiguous().cpu();
  TORCH_CHECK(c.element_size() == 1, "pack_int4_cpu: codes must be one byte each");
  const int64_t n = c.numel();
  const int64_t nw = (n + 7) / 8;
  at::Tensor w = at::empty({nw}, at::kInt);
  const uint8_t* cp = reinterpret_cast<const uint8_t*>(c.data_ptr());
  uint32_t* wp = reinterpret_cast<uint32_t*>(w.data_ptr());
  for (int64_t k = 0; k < nw; ++k) {
    uint32_t word = 0;
    for (int nib = 0; nib < 8; ++nib) {
      const int64_t e = k * 8 + kNibbleOrder[nib];
      const uint32_t v = (e < n) ? (cp[e] & 0xfu) : 0u;
      word |= v << (4 * nib);
    }
    wp[k] = word;
  }
  return w;
}

at::Tensor unpack_int4_cpu(const at::Tensor& words_in, int64_t numel) {
  at::Tensor w = words_in.reshape({-1}).contiguous().cpu();
  TORCH_CHECK(w.element_size() == 4, "unpack_int4_cpu: expected int32 words");
  TORCH_CHECK(numel <= w.numel() * 8, "unpack_int4_cpu: numel exceeds 8 * words");
  at::Tensor out = at::empty({numel}, at::kByte);
  const uint32_t* wp = reinterpret_cast<const uint32_t*>(w.data_ptr());
  uint8_t* op = out.data_ptr<uint8_t>();
  for (int64_t k = 0; k * 8 < numel; ++k) {
    for (int nib = 0; nib < 8; ++nib) {
      const int64_t e = k * 8 + kNibbleOrder[nib];
      if (e < numel) op[e] = (uint8_t)((wp[k] >> (4 * nib)) & 0xfu);
    }
  }
  return out;
}

}  // namespace qfc
