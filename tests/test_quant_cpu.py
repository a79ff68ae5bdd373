"""CPU checks of the quantization specification, the C++ oracle and the compat API."""
import pytest
import torch

from quantized_flash_communication_b200 import quantization as spec
from quantized_flash_communication_b200._ext import ext, has_ext
from quantized_flash_communication_b200.ops import quant as Q


def test_rhaz_is_half_away_from_zero():
    v = torch.tensor([0.5, -0.5, 1.5, -1.5, 2.5, 0.49999997, -0.49999997, 3.0, -2.7])
    assert spec.rhaz(v).tolist() == [1.0, -1.0, 2.0, -2.0, 3.0, 0.0, -0.0, 3.0, -3.0]


def test_nibble_layout_matches_reference_word():
    # Reference kernels_jit.py:18-30: codes 0..7 pack to 0x75316420.
    w = spec.pack_int4_ref(torch.arange(8, dtype=torch.uint8))
    assert (int(w.item()) & 0xFFFFFFFF) == 0x75316420
    assert spec.INT4_NIBBLE_ORDER == (0, 2, 4, 6, 1, 3, 5, 7)


def test_pack_unpack_roundtrip_with_padding():
    c = torch.randint(0, 16, (1003,), dtype=torch.uint8)
    w = spec.pack_int4_ref(c)
    assert w.numel() == 126
    assert torch.equal(spec.unpack_int4_ref(w, 1003), c)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("mode", ["asym", "sym"])
def test_quantize_properties(bits, mode):
    torch.manual_seed(0)
    x = torch.randn(4096) * 2
    q, s, z = spec.quantize_groups(x, bits, 128, mode, torch.float32)
    qmax = (1 << bits) - 1
    assert int(q.max()) <= qmax
    d = spec.dequantize_groups(q, s, z, 128, torch.float32)
    g = x.view(-1, 128)
    # error bounded by one quantization step (plus the symmetric top-code clamp)
    step = s.view(-1, 1)
    err = (d.view(-1, 128) - g).abs()
    assert bool((err <= step * (1.0 if mode == "sym" else 0.5) + 1e-6).all())
    if mode == "sym":
        assert bool((z == (qmax + 1) // 2).all())


def test_scale_floor_and_constant_groups():
    x = torch.zeros(256)
    q, s, z = spec.quantize_groups(x, 8, 128, "asym", torch.float32)
    assert bool((s == 1.0).all()) and bool((z == 0).all()) and bool((q == 0).all())


def test_partial_group_counts_padding_as_zero():
    x = torch.full((130,), 5.0)  # last group: 2 real values + 126 zero pads
    q, s, z = spec.quantize_groups(x, 8, 128, "asym", torch.float32)
    assert float(s[1]) == pytest.approx(5.0 / 255.0)


@pytest.mark.skipif(not has_ext(), reason="extension not built")
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("mode", ["asym", "sym"])
@pytest.mark.parametrize("gs", [8, 32, 128, 256, 2048])
@pytest.mark.parametrize("sd", [torch.float16, torch.float32])
def test_cpp_oracle_matches_torch_spec(bits, mode, gs, sd):
    torch.manual_seed(bits * 7 + gs)
    for n in (1, 9, 1000, 4101):
        x = torch.randn(n) * 3
        x[::13] *= 40
        q1, s1, z1 = ext().quantize_cpu(x, bits, gs, mode == "sym", sd == torch.float32)
        q2, s2, z2 = spec.quantize_groups(x, bits, gs, mode, sd)
        assert torch.equal(q1, q2) and torch.equal(s1, s2) and torch.equal(z1, z2)
        d1 = ext().dequantize_cpu(q1, s1, z1, gs, torch.float32)
        assert torch.equal(d1, spec.dequantize_groups(q2, s2, z2, gs, torch.float32))


@pytest.mark.skipif(not has_ext(), reason="extension not built")
def test_cpp_pack_matches_spec():
    c = torch.randint(0, 16, (777,), dtype=torch.uint8)
    assert torch.equal(ext().pack_int4_cpu(c), spec.pack_int4_ref(c))
    assert torch.equal(ext().unpack_int4_cpu(spec.pack_int4_ref(c), 777), c)


def test_compat_api_shapes_cpu():
    from quantized_flash_communication_b200 import kernels, kernels_jit, quantization
    x = torch.randn(3, 100)
    q, s, z = kernels.triton_quantize(x, bits=8, block_size=128, mode="asym")
    assert q.dtype == torch.int8 and s.dtype == torch.float16 and z.dtype == torch.float16
    assert q.numel() == 300 and s.numel() == 3
    d = kernels.triton_dequantize(q, s, z, x.shape, 128)
    assert d.shape == x.shape and d.dtype == torch.float16
    assert (d.float() - x).abs().max() < 0.05
    q4, s4, z4 = kernels.triton_quantize(x, bits=4, block_size=128, mode="sym")
    w = kernels_jit.pack_int4(q4)
    assert w.dtype == torch.int32 and w.numel() == 38
    u = kernels_jit.unpack_int4(w, torch.Size([304]))
    assert torch.equal(u[:300].to(torch.uint8), q4.view(torch.uint8))
    qb, sb, zb, shape, pad = quantization.quantize_blockwise(x, bits=8, group_size=128)
    assert qb.shape == (3, 128) and pad == 84 and shape == x.shape
    xr = quantization.dequantize_blockwise(qb, sb, zb, shape, pad)
    assert xr.shape == x.shape and (xr - x).abs().max() < 0.05


def test_fast_round_half_away_identity():
    """trunc(|v| + 0.49999997f) == floor(|v| + 0.5) for every float of interest (fp32 math).

    The CUDA kernels round with this identity; check it on all .5 ties up to 2^23, their
    float neighbours, and a dense sweep of [0, 4).
    """
    import numpy as np
    c = np.float32(0.49999997)
    assert c == np.nextafter(np.float32(0.5), np.float32(0))
    k = np.arange(0, 1 << 23, dtype=np.float64)
    ties = (k + 0.5).astype(np.float32)
    ties = ties[(ties.astype(np.float64) == k + 0.5)]  # exactly representable ties
    cand = np.concatenate([ties, np.nextafter(ties, np.float32(0)), np.nextafter(ties, np.float32(np.inf)),
                           np.linspace(0, 4, 1 << 22, dtype=np.float32), np.float32([0.49999997, 0.5, 0.0])])
    got = np.trunc(np.abs(cand) + c)  # fp32 add, fp32 trunc
    want = np.floor(np.abs(cand).astype(np.float64) + 0.5)
    assert got.dtype == np.float32
    bad = np.nonzero(got.astype(np.float64) != want)[0]
    assert bad.size == 0, cand[bad[:5]]
