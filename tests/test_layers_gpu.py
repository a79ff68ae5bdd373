"""Layer kernels (RMSNorm, RoPE + KV cache, SwiGLU, embedding, argmax) vs torch."""
import pytest
import torch

from quantized_flash_communication_b200.ops import layers as L

pytestmark = pytest.mark.gpu


def _rms_ref(x, w, eps):
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return w * y.to(x.dtype)


@pytest.mark.parametrize("H", [4096, 8192, 3072, 5120])
def test_rmsnorm(cuda_device, H):
    x = torch.randn(37, H, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(H, device=cuda_device, dtype=torch.bfloat16)
    y = L.rmsnorm(x, w, 1e-5)
    assert torch.allclose(y.float(), _rms_ref(x, w, 1e-5).float(), rtol=2e-2, atol=2e-2)
    r = torch.randn_like(x)
    h = x + r
    r2 = r.clone()
    y2 = L.rmsnorm(x, w, 1e-5, residual=r2)
    assert torch.equal(r2, h)
    assert torch.allclose(y2.float(), _rms_ref(h, w, 1e-5).float(), rtol=2e-2, atol=2e-2)


def _rope_ref(x, pos, cs):
    # x [M, heads, hd]
    hd = x.shape[-1]
    c = cs[pos, :, 0].unsqueeze(1)
    s = cs[pos, :, 1].unsqueeze(1)
    x1, x2 = x[..., : hd // 2].float(), x[..., hd // 2:].float()
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


@pytest.mark.parametrize("hd,page", [(128, 16), (64, 16), (128, 24)])
def test_rope_and_cache(cuda_device, hd, page):
    nq, nkv, M = 8, 2, 50
    cs = L.rope_cos_sin(4096, hd, 10000.0, cuda_device)
    qkv = torch.randn(M, (nq + 2 * nkv) * hd, device=cuda_device, dtype=torch.bfloat16)
    pos = torch.randint(0, 4096, (M,), device=cuda_device)
    orig = qkv.clone().view(M, nq + 2 * nkv, hd)
    kc = torch.zeros(8, nkv, page, hd, device=cuda_device, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(8 * page, device=cuda_device)[:M]
    slots[::7] = -1  # not cached
    L.rope_kv(qkv, pos, cs, nq, nkv, hd, kc, vc, slots)
    out = qkv.view(M, nq + 2 * nkv, hd)
    ref_q = _rope_ref(orig[:, :nq], pos, cs)
    ref_k = _rope_ref(orig[:, nq:nq + nkv], pos, cs)
    assert torch.allclose(out[:, :nq].float(), ref_q, atol=2e-2, rtol=2e-2)
    assert torch.allclose(out[:, nq:nq + nkv].float(), ref_k, atol=2e-2, rtol=2e-2)
    assert torch.equal(out[:, nq + nkv:], orig[:, nq + nkv:])
    keep = slots >= 0
    pg, off = slots[keep] // page, slots[keep] % page
    assert torch.equal(kc[pg, :, off], out[keep, nq:nq + nkv])
    assert torch.equal(vc[pg, :, off], out[keep, nq + nkv:])
    written = (kc.abs().sum(-1) > 0).sum().item()
    assert written == int(keep.sum()) * nkv


def test_silu_mul(cuda_device):
    gu = torch.randn(33, 2 * 1376, device=cuda_device, dtype=torch.bfloat16)
    y = L.silu_mul(gu)
    ref = torch.nn.functional.silu(gu[:, :1376]) * gu[:, 1376:]
    assert torch.allclose(y.float(), ref.float(), rtol=2e-2, atol=2e-2)


def test_embedding_and_argmax(cuda_device):
    table = torch.randn(1000, 256, device=cuda_device, dtype=torch.bfloat16)
    ids = torch.randint(0, 2000, (64,), device=cuda_device)
    y = L.embedding(ids, table, vocab_start=500)
    for i, t in enumerate(ids.tolist()):
        if 500 <= t < 1500:
            assert torch.equal(y[i], table[t - 500])
        else:
            assert bool((y[i] == 0).all())
    logits = torch.randn(7, 32000, device=cuda_device, dtype=torch.bfloat16)
    bv, bi = L.argmax(logits, idx_offset=100)
    assert torch.equal(bi - 100, logits.float().argmax(-1))


@pytest.mark.parametrize("V,dtype", [(128256, torch.bfloat16), (1001, torch.bfloat16), (4096, torch.float32),
                                     (8, torch.float16)])
def test_argmax_first_maximum(cuda_device, V, dtype):
    logits = torch.randn(64, V, device=cuda_device).to(dtype)
    # ties: the same maximum at two positions of every row; the first must win
    hi = logits.float().max().item() + 1.0
    cols = torch.randint(0, V, (64, 2), device=cuda_device).sort(-1).values
    logits[torch.arange(64), cols[:, 0]] = hi
    logits[torch.arange(64), cols[:, 1]] = hi
    bv, bi = L.argmax(logits)
    assert torch.equal(bi, cols[:, 0])
    assert torch.equal(bv.float(), torch.full_like(bv.float(), float(torch.tensor(hi).to(dtype))))


@pytest.mark.parametrize("M,nq,nkv,page", [(100, 8, 2, 16), (513, 4, 4, 64), (2048, 32, 8, 64)])
def test_qkv_gemm_with_fused_rope_matches_unfused(cuda_device, M, nq, nkv, page):
    """The qkv GEMM's RoPE + KV-cache epilogue equals the GEMM followed by rope_kv, bit for bit."""
    from quantized_flash_communication_b200.ops import gemm as G
    hd, K = 128, 1024
    g = torch.Generator(device="cpu").manual_seed(M)
    x = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    w = (torch.randn((nq + 2 * nkv) * hd, K, generator=g) * 0.03).to(cuda_device, torch.bfloat16)
    cs = L.rope_cos_sin(8192, hd, 500000.0, cuda_device)
    pos = torch.randint(0, 8192, (M,), generator=g).to(cuda_device)
    pages = (M + page - 1) // page + 2
    slots = torch.randperm(pages * page, generator=g)[:M].to(cuda_device)
    slots[::11] = -1
    kc1 = torch.zeros(pages, nkv, page, hd, device=cuda_device, dtype=torch.bfloat16)
    vc1 = torch.zeros_like(kc1)
    kc2, vc2 = kc1.clone(), vc1.clone()
    ref = G.linear(x, w)
    L.rope_kv(ref, pos, cs, nq, nkv, hd, kc1, vc1, slots)
    got = G.linear_qkv_rope(x, w, pos, cs, nq, nkv, kc2, vc2, slots)
    torch.cuda.synchronize()
    assert G.gemm_status() == 0
    assert torch.equal(got, ref)
    assert torch.equal(kc2, kc1) and torch.equal(vc2, vc1)
    got2 = G.linear_qkv_rope(x, w, pos, cs, nq, nkv)  # no cache
    assert torch.equal(got2, ref)
