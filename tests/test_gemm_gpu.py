"""tcgen05 GEMM vs an fp32 torch reference.

Every check is an element-wise bound against the fp32 product of the same bf16 operands:
``|y - ref| <= rel * |ref| + extra + 1e-3 * sigma``.  ``rel`` covers the final rounding to
bf16 (half an ulp is at most 2^-8 of the value); ``sigma = sqrt(K) * std(a) * std(b)`` is
the typical size of an output element, so the absolute term is a thousandth of it.
``extra`` covers epilogues that round an intermediate to bf16 as the unfused ops would
(the residual and SwiGLU epilogues): a different fp32 summation order may land that
rounding one bf16 ulp (2^-7 of the value) away.  Dropping, repeating or mis-swizzling one
64-deep k-block moves an element by about ``sqrt(64) * std(a) * std(b) = sigma * 8 /
sqrt(K)``, far above the bound for every K here.
"""
import math

import pytest
import torch

from quantized_flash_communication_b200.ops import gemm as G

pytestmark = pytest.mark.gpu


def _ref(a, b):
    return a.float() @ b.float().T


def _sigma(a, b):
    return math.sqrt(a.shape[-1]) * a.float().std().item() * b.float().std().item()


def _bf16(x):
    return x.to(torch.bfloat16).float()


def _check(y, ref, sigma, rel=2.0 ** -8, what="", extra=0.0):
    err = (y.float() - ref).abs()
    bound = rel * ref.abs() + extra + 1e-3 * sigma
    worst = (err - bound).max().item()
    assert worst <= 0, f"{what}: max |err| {err.max().item():.3e} exceeds the bound (sigma {sigma:.3e})"


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (1, 256, 64), (100, 312, 136),
                                   (1000, 1536, 4096), (8192, 4096, 512), (513, 2752, 1376), (64, 4096, 4096)])
def test_gemm_store(cuda_device, M, N, K):
    torch.manual_seed(M + N + K)
    a = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=cuda_device, dtype=torch.bfloat16) * 0.05
    y = G.linear(a, b)
    torch.cuda.synchronize()
    assert G.gemm_status() == 0
    _check(y, _ref(a, b), _sigma(a, b), what=f"{M}x{N}x{K}")


@pytest.mark.parametrize("M,I,K", [(128, 128, 64), (300, 1376, 4096), (64, 2048, 1024)])
def test_gemm_swiglu(cuda_device, M, I, K):
    torch.manual_seed(I)
    a = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(2 * I, K, device=cuda_device, dtype=torch.bfloat16) * 0.03
    y = G.linear_swiglu(a, w)
    torch.cuda.synchronize()
    g = _bf16(_ref(a, w[:I]))   # fp32 products of the bf16 operands, stored as bf16
    u = _bf16(_ref(a, w[I:]))
    ref = _bf16(torch.nn.functional.silu(g)) * u
    s = _sigma(a, w)
    extra = 2.0 ** -6 * (g.abs() + 1.0) * u.abs()  # one-ulp flips of g, u or silu(g)
    _check(y, ref, s * s, rel=2.0 ** -7, what=f"swiglu {M}x{I}x{K}", extra=extra)


def test_gemm_residual_in_place(cuda_device):
    M, N, K = 777, 4096, 512
    a = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=cuda_device, dtype=torch.bfloat16) * 0.05
    r = torch.randn(M, N, device=cuda_device, dtype=torch.bfloat16)
    ab = _ref(a, w)
    ref = _bf16(ab) + r.float()  # the product is rounded to bf16 before the add
    s = _sigma(a, w)
    G.linear_residual(a, w, r, out=r)
    torch.cuda.synchronize()
    _check(r, ref, s, what="residual", extra=2.0 ** -7 * ab.abs())


@pytest.mark.parametrize("M,N,K", [(50, 1024, 2048), (128, 512, 4096), (7, 4096, 14336)])
def test_gemm_split_k_small_m(cuda_device, M, N, K):
    """Few tiles and a long K: the GEMM splits K; plain and residual epilogues, run twice
    (the arrival counters must be back to zero after a launch)."""
    a = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=cuda_device, dtype=torch.bfloat16) * 0.02
    r = torch.randn(M, N, device=cuda_device, dtype=torch.bfloat16)
    ref = _ref(a, w)
    s = _sigma(a, w)
    for _ in range(2):
        y = G.linear(a, w)
        torch.cuda.synchronize()
        assert G.gemm_status() == 0
        _check(y, ref, s, what=f"split-k {M}x{N}x{K}")
        out = r.clone()
        G.linear_residual(a, w, out, out=out)
        _check(out, _bf16(ref) + r.float(), s, what=f"split-k residual {M}x{N}x{K}", extra=2.0 ** -7 * ref.abs())
    y2 = G.linear(a, w)
    assert torch.equal(y, y2)  # the split order is fixed: deterministic


def test_gemm_persistent_small_grid(cuda_device):
    from quantized_flash_communication_b200._ext import ext
    a = torch.randn(1024, 1024, device=cuda_device, dtype=torch.bfloat16)
    b = torch.randn(1024, 1024, device=cuda_device, dtype=torch.bfloat16) * 0.05
    y = ext().gemm_bf16(a, b, None, 0, None, 10000.0, 3)  # 3 CTAs loop over 32 tiles
    _check(y, _ref(a, b), _sigma(a, b), what="3-CTA persistent")

