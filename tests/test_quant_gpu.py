"""sm_100a quantize / dequantize / pack / unpack kernels vs the torch specification."""
import pytest
import torch

from quantized_flash_communication_b200 import quantization as spec
from quantized_flash_communication_b200.ops import quant as Q

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("mode", ["asym", "sym"])
@pytest.mark.parametrize("gs", [8, 16, 32, 64, 128, 256, 1024, 8192])
def test_quantize_bit_exact(cuda_device, dtype, bits, mode, gs):
    torch.manual_seed(gs + bits)
    for n in (1, 9, 255, 4096, 100003):
        x = (torch.randn(n, device=cuda_device) * 3).to(dtype)
        x[::97] *= 50
        for sd in (torch.float16, torch.float32):
            q, s, z = Q.quantize(x, bits, gs, mode, sd)
            q2, s2, z2 = spec.quantize_groups(x.cpu(), bits, gs, mode, sd)
            assert torch.equal(q.cpu(), q2), (n, sd)
            assert torch.equal(s.cpu(), s2), (n, sd)
            assert torch.equal(z.cpu(), z2), (n, sd)
            for od in (torch.float16, torch.bfloat16, torch.float32):
                d = Q.dequantize(q, s, z, gs, od)
                assert torch.equal(d.cpu(), spec.dequantize_groups(q2, s2, z2, gs, od)), (n, od)


def test_dequantize_fp16_codes(cuda_device):
    x = torch.randn(5000, device=cuda_device, dtype=torch.float16)
    q, s, z = Q.quantize(x, 4, 128, "asym")
    d1 = Q.dequantize(q, s, z, 128, torch.float16)
    d2 = Q.dequantize(q.to(torch.float16), s, z, 128, torch.float16)
    assert torch.equal(d1, d2)


@pytest.mark.parametrize("n", [8, 64, 1000, 1003, 1 << 20])
def test_pack_unpack(cuda_device, n):
    c = torch.randint(0, 16, (n,), dtype=torch.uint8, device=cuda_device)
    w = Q.pack_int4(c)
    assert torch.equal(w.cpu(), spec.pack_int4_ref(c.cpu()))
    u = Q.unpack_int4(w, n)
    assert u.dtype == torch.float16
    assert torch.equal(u.to(torch.uint8).cpu(), c.cpu())


def test_reference_pack_self_test(cuda_device):
    # The reference's only test (kernels_jit.py:130-163): int8 codes [128, 64] -> pack -> unpack.
    from quantized_flash_communication_b200.kernels_jit import pack_int4, unpack_int4
    x = torch.randint(0, 16, (128, 64), dtype=torch.int8, device=cuda_device)
    u = unpack_int4(pack_int4(x), x.shape)
    assert u.shape == x.shape and torch.equal(u.to(torch.int8), x)


def test_launches_on_current_stream(cuda_device):
    s = torch.cuda.Stream()
    x = torch.randn(1 << 20, device=cuda_device)
    with torch.cuda.stream(s):
        q, sc, z = Q.quantize(x, 8, 128)
        d = Q.dequantize(q, sc, z, 128, torch.float32)
    s.synchronize()
    assert (d - x).abs().max().item() < 0.1


def test_rounding_ties_bit_exact(cuda_device):
    """Codes of exact .5 ties and their neighbours (fp32 input, scale 1, zero point 0)."""
    import numpy as np
    vals = []
    for k in range(0, 255):
        t = np.float32(k + 0.5)
        vals += [t, np.nextafter(t, np.float32(0)), np.nextafter(t, np.float32(1e9))]
    vals += [np.float32(0.49999997)]
    vals = [v for v in vals if 0 <= v <= 255]
    groups = []
    for i in range(0, len(vals), 126):
        chunk = vals[i:i + 126]
        chunk = chunk + [np.float32(1.0)] * (126 - len(chunk))
        groups.append([np.float32(0.0), np.float32(255.0)] + chunk)
    x = torch.tensor(np.array(groups, dtype=np.float32).reshape(-1), device=cuda_device)
    q, s, z = Q.quantize(x, 8, 128, "asym", torch.float32)
    q2, s2, z2 = spec.quantize_groups(x.cpu(), 8, 128, "asym", torch.float32)
    assert bool((s2 == 1.0).all()) and bool((z2 == 0).all())
    assert torch.equal(q.cpu(), q2)
