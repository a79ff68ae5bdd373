"""The allocation-free decode-attention entry point, called through its exported C symbol.

Callers such as a serving runtime that owns all device memory through its own pool (or a
plugin running inside one, or plain C code without PyTorch's allocator) must not allocate
on their hot path.  ``qfc_attn_decode_noalloc`` serves them: it keeps its scratch in a
fixed array inside the library.  This test loads the symbol with ctypes from the in-tree
extension, checks two consecutive calls against the regular (allocating) entry point for
every dispatch branch (tensor-core GQA and CUDA-core multi-head partial kernels, head_dim
64 and 128, bf16 and fp16, and a call that nearly fills the array), and checks that an
oversized call is refused.  The file name makes pytest collect it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 16 * 2 ** 20


def _lib():
    from quantized_flash_communication_b200._ext import ext
    lib = ctypes.CDLL(ext().__file__)
    f = lib.qfc_attn_decode_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 6 + [ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
    lib.qfc_noalloc_error_string.restype = ctypes.c_char_p
    lib.qfc_noalloc_error_string.argtypes = [ctypes.c_int]
    lib.qfc_attn_decode_noalloc_scratch_bytes.restype = ctypes.c_ulonglong
    lib.qfc_attn_decode_noalloc_scratch_bytes.argtypes = [ctypes.c_int] * 5
    return lib


def _case(dev, B=6, nq=16, nkv=4, hd=128, page=64, pps=20, dtype=torch.bfloat16, lens=None):
    g = torch.Generator(device="cpu").manual_seed(5)
    kc = torch.randn(B * pps, nkv, page, hd, generator=g).to(dev, dtype)
    vc = torch.randn(B * pps, nkv, page, hd, generator=g).to(dev, dtype)
    bt = torch.randperm(B * pps, generator=g).to(torch.int32).view(B, pps).to(dev).contiguous()
    if lens is None:
        lens = [1, 65, 300, 640, 1000, 1280][:B]
    lens = torch.tensor(lens, dtype=torch.int32, device=dev)
    q = torch.randn(B, nq * hd, generator=g).to(dev, dtype)
    return q, kc, vc, bt, lens


def _call(lib, q, kc, vc, bt, lens, out, nq, nkv, hd, B=None):
    B = q.shape[0] if B is None else B
    dt = {torch.bfloat16: 0, torch.float16: 1}[q.dtype]
    stream = torch.cuda.current_stream().cuda_stream
    return lib.qfc_attn_decode_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), lens.data_ptr(),
                                       out.data_ptr(), B, nq, nkv, hd, kc.shape[2], bt.shape[1], 1.0 / hd ** 0.5, dt,
                                       stream)


def _check_twice(lib, dev, nq, nkv, hd, dtype, **kw):
    from quantized_flash_communication_b200.ops.attention import decode_attention
    from quantized_flash_communication_b200.quantization import rel_l2
    q, kc, vc, bt, lens = _case(dev, nq=nq, nkv=nkv, hd=hd, dtype=dtype, **kw)
    ref = decode_attention(q, kc, vc, bt, lens, nq, nkv, hd)
    for call in range(2):
        out = torch.full_like(q, float("nan"))
        rc = _call(lib, q, kc, vc, bt, lens, out, nq, nkv, hd)
        assert rc == 0, lib.qfc_noalloc_error_string(rc)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert rel_l2(out.float(), ref.float()) < 1e-3, call


@pytest.mark.parametrize("nq,nkv,hd,dtype", [
    (16, 4, 128, torch.bfloat16),   # GQA group 4: tensor-core partial kernel
    (8, 8, 128, torch.bfloat16),    # group 1: CUDA-core partial kernel
    (16, 2, 64, torch.bfloat16),    # head_dim 64, group 8
    (8, 8, 64, torch.float16),      # fp16, head_dim 64, group 1
    (16, 4, 128, torch.float16),    # fp16, tensor-core path
])
def test_noalloc_matches_allocating_entry_point_twice(cuda_device, nq, nkv, hd, dtype):
    _check_twice(_lib(), cuda_device, nq, nkv, hd, dtype)


def test_noalloc_call_that_nearly_fills_the_scratch(cuda_device):
    lib = _lib()
    B, nq, nkv, hd, page, pps = 63, 32, 8, 128, 64, 64  # 63 x 32 x 16 partitions x 130 x 4 bytes
    need = lib.qfc_attn_decode_noalloc_scratch_bytes(B, nq, hd, page, pps)
    assert 0.99 * SCRATCH_BYTES < need <= SCRATCH_BYTES
    g = torch.Generator().manual_seed(11)
    lens = torch.randint(1, page * pps + 1, (B,), generator=g).tolist()
    lens[0] = page * pps
    _check_twice(lib, cuda_device, nq, nkv, hd, torch.bfloat16, B=B, page=page, pps=pps, lens=lens)


def test_noalloc_refuses_calls_beyond_its_scratch(cuda_device):
    lib = _lib()
    nq, nkv, hd = 32, 8, 128
    q, kc, vc, bt, lens = _case(cuda_device, B=1, nq=nq, nkv=nkv, hd=hd, pps=2)
    big_batch = 4096  # needs 4096 * 32 * 1 * 130 * 4 bytes > 16 MiB
    assert lib.qfc_attn_decode_noalloc_scratch_bytes(big_batch, nq, hd, 64, 2) > SCRATCH_BYTES
    out = torch.empty_like(q)
    rc = _call(lib, q, kc, vc, bt, lens, out, nq, nkv, hd, B=big_batch)
    assert rc == 1
    assert b"16 MiB" in lib.qfc_noalloc_error_string(rc)
