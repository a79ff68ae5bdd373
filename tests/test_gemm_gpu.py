"""tcgen05 GEMM vs an fp32 torch reference."""
import pytest
import torch

from quantized_flash_communication_b200.ops import gemm as G

pytestmark = pytest.mark.gpu


def _ref(a, b):
    return a.float() @ b.float().T


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (1, 256, 64), (100, 312, 136),
                                   (1000, 1536, 4096), (8192, 4096, 512), (513, 2752, 1376), (64, 4096, 4096)])
def test_gemm_store(cuda_device, M, N, K):
    torch.manual_seed(M + N + K)
    a = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=cuda_device, dtype=torch.bfloat16) * 0.05
    y = G.linear(a, b)
    torch.cuda.synchronize()
    assert G.gemm_status() == 0
    ref = _ref(a, b)
    err = (y.float() - ref).abs().max().item()
    assert err <= 0.02 * ref.abs().max().item() + 1e-2, err
    assert torch.allclose(y.float(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("M,I,K", [(128, 128, 64), (300, 1376, 4096), (64, 2048, 1024)])
def test_gemm_swiglu(cuda_device, M, I, K):
    torch.manual_seed(I)
    a = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(2 * I, K, device=cuda_device, dtype=torch.bfloat16) * 0.03
    y = G.linear_swiglu(a, w)
    torch.cuda.synchronize()
    g = (a @ w[:I].T)
    u = (a @ w[I:].T)
    ref = (torch.nn.functional.silu(g) * u).float()
    assert torch.allclose(y.float(), ref, rtol=3e-2, atol=3e-2)


def test_gemm_residual_in_place(cuda_device):
    M, N, K = 777, 4096, 512
    a = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=cuda_device, dtype=torch.bfloat16) * 0.05
    r = torch.randn(M, N, device=cuda_device, dtype=torch.bfloat16)
    ref = _ref(a, w) + r.float()
    G.linear_residual(a, w, r, out=r)
    torch.cuda.synchronize()
    assert torch.allclose(r.float(), ref, rtol=2e-2, atol=3e-2)


@pytest.mark.parametrize("M,N,K", [(50, 1024, 2048), (128, 512, 4096), (7, 4096, 14336)])
def test_gemm_split_k_small_m(cuda_device, M, N, K):
    """Few tiles and a long K: the GEMM splits K; plain and residual epilogues, run twice
    (the arrival counters must be back to zero after a launch)."""
    a = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=cuda_device, dtype=torch.bfloat16) * 0.02
    r = torch.randn(M, N, device=cuda_device, dtype=torch.bfloat16)
    ref = _ref(a, w)
    for _ in range(2):
        y = G.linear(a, w)
        torch.cuda.synchronize()
        assert G.gemm_status() == 0
        assert torch.allclose(y.float(), ref, rtol=2e-2, atol=2e-2)
        out = r.clone()
        G.linear_residual(a, w, out, out=out)
        assert torch.allclose(out.float(), ref + r.float(), rtol=2e-2, atol=3e-2)
    y2 = G.linear(a, w)
    assert torch.equal(y, y2)  # the split order is fixed: deterministic


def test_gemm_persistent_small_grid(cuda_device):
    from quantized_flash_communication_b200._ext import ext
    a = torch.randn(1024, 1024, device=cuda_device, dtype=torch.bfloat16)
    b = torch.randn(1024, 1024, device=cuda_device, dtype=torch.bfloat16) * 0.05
    y = ext().gemm_bf16(a, b, None, 0, None, 10000.0, 3)  # 3 CTAs loop over 32 tiles
    assert torch.allclose(y.float(), _ref(a, b), rtol=2e-2, atol=2e-2)
