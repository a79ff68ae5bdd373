"""tcgen05 flash prefill attention vs an fp32 torch reference."""
import pytest
import torch

from quantized_flash_communication_b200.ops.attention import attn_status, prefill_attention
from quantized_flash_communication_b200.quantization import rel_l2

pytestmark = pytest.mark.gpu


def _ref(qkv, B, S, nq, nkv, hd):
    x = qkv.float().view(B, S, nq + 2 * nkv, hd)
    q = x[:, :, :nq].transpose(1, 2)
    k = x[:, :, nq:nq + nkv].transpose(1, 2).repeat_interleave(nq // nkv, 1)
    v = x[:, :, nq + nkv:].transpose(1, 2).repeat_interleave(nq // nkv, 1)
    s = (q @ k.transpose(-1, -2)) / hd ** 0.5
    mask = torch.ones(S, S, dtype=torch.bool, device=qkv.device).triu(1)
    s = s.masked_fill(mask, float("-inf"))
    return (torch.softmax(s, -1) @ v).transpose(1, 2).reshape(B * S, nq * hd)


@pytest.mark.parametrize("B,S,nq,nkv", [(1, 128, 1, 1), (2, 100, 4, 4), (2, 300, 8, 2), (1, 1024, 4, 1), (3, 100, 8, 4),
                                         (3, 257, 2, 2), (8, 1024, 4, 4)])
def test_prefill_attention_matches_reference(cuda_device, B, S, nq, nkv):
    hd = 128
    torch.manual_seed(B * S + nq)
    qkv = torch.randn(B * S, (nq + 2 * nkv) * hd, device=cuda_device, dtype=torch.bfloat16)
    o = prefill_attention(qkv, B, S, nq, nkv, hd)
    torch.cuda.synchronize()
    assert attn_status(clear=True) == 0
    ref = _ref(qkv, B, S, nq, nkv, hd)
    assert rel_l2(o.float(), ref) < 1e-2
    assert torch.isfinite(o.float()).all()


def test_fma_pipe_exp2_against_exp2f(cuda_device):
    """The softmax's polynomial 2^x (FMA pipe) vs CUDA's exp2f (torch.exp2) on x <= 0."""
    from quantized_flash_communication_b200._ext import ext
    x = torch.cat([torch.linspace(-125.0, 0.0, 1 << 20, device=cuda_device),
                   -torch.rand(1 << 20, device=cuda_device) * 30,
                   torch.tensor([0.0, -0.5, -1.0, -1.5, -2.5, -124.5], device=cuda_device)])
    y = torch.empty_like(x)
    ext().attn_exp2_poly(x, y)
    ref = torch.exp2(x)
    rel = ((y - ref).abs() / ref).max().item()
    assert rel < 1e-4, rel  # fitted bound 7.5e-5; bf16 P needs 2^-9
    y2 = torch.empty(1, device=cuda_device)
    ext().attn_exp2_poly(torch.tensor([float("-inf")], device=cuda_device), y2)
    assert 0 <= y2.item() < 1e-37


@pytest.mark.parametrize("B,S,nq,nkv", [(2, 1024, 4, 4), (1, 2048, 8, 2)])
def test_prefill_attention_row_maxima_that_grow(cuda_device, B, S, nq, nkv):
    """Keys whose scale grows along the sequence make the running maximum of some rows (not
    all) jump by more than 2^8 between tiles: the lazy O rescale runs for part of a warp."""
    hd = 128
    g = torch.Generator(device="cpu").manual_seed(S + nq)
    x = torch.randn(B * S, nq + 2 * nkv, hd, generator=g)
    ramp = 1.0 + 6.0 * torch.arange(S).float().repeat(B) / S          # later keys score higher
    x[:, nq:nq + nkv] *= ramp[:, None, None]
    x[:, :nq] *= (0.5 + torch.rand(B * S, nq, 1, generator=g) * 2.5)   # rows differ in sharpness
    qkv = x.reshape(B * S, -1).to(cuda_device, torch.bfloat16)
    o = prefill_attention(qkv, B, S, nq, nkv, hd)
    torch.cuda.synchronize()
    assert attn_status(clear=True) == 0
    ref = _ref(qkv, B, S, nq, nkv, hd)
    assert rel_l2(o.float(), ref) < 1e-2
