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
