"""Kernels that are built but switched off until a measurement decides for them.

* the two-stage two-shot all-reduce (``set_two_shot_stages(2)``),
* the sequence-parallel norm kernel with 2 or 4 warps per row (``set_norm_warps_per_row``),
* the prefill-attention softmax on packed two-lane fp32 instructions (``set_attn_packed``),
* the weight-streaming GEMM for at most 8 rows (``set_gemv``).

Each is held to the same checks as the default kernel it would replace (bit-exact with
the oracle where the default is, the same error bounds otherwise).  The file name makes
pytest collect it last, so that a failure here cannot stop the default kernels' tests
under ``-x``.
"""
import os
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import free_port
from quantized_flash_communication_b200 import quantization as spec
from quantized_flash_communication_b200._ext import ext
from quantized_flash_communication_b200.ops import gemm as G
from quantized_flash_communication_b200.ops.attention import attn_status, prefill_attention
from quantized_flash_communication_b200.parallel import EmulatedQuantAllReduce
from quantized_flash_communication_b200.parallel.quant_allreduce import set_norm_warps_per_row, set_two_shot_stages
from quantized_flash_communication_b200.quantization import rel_l2
from test_allreduce_gpu import CASES, _inputs
from test_attention_gpu import _ref as attn_ref
from test_gemm_gpu import _bf16, _check, _ref, _sigma

pytestmark = pytest.mark.gpu


# ------------------------------------------------------------------ two-stage two-shot
@pytest.fixture
def two_stages():
    prev = set_two_shot_stages(2)
    yield
    set_two_shot_stages(prev)


@pytest.mark.parametrize("W,bits,gs,mode,shape,algo", [c for c in CASES if c[5] == "two_shot"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_two_stage_two_shot_matches_oracle(cuda_device, two_stages, W, bits, gs, mode, shape, algo, dtype):
    ar = EmulatedQuantAllReduce(W, cuda_device, bits=bits, group_size=gs, quant_type=mode, algo=algo,
                                timeout_ms=5000)
    xs = _inputs(W, shape, dtype, cuda_device, seed=W * 100 + bits)
    for it in range(3):  # repeated calls: epochs and both flag sets are reused
        outs = ar(xs)
        ar.check()
        ref = spec.two_step_all_reduce_ref([x.cpu() for x in xs], bits, gs, mode, torch.float16, dtype)
        for r in range(W):
            assert torch.equal(outs[r].cpu(), ref), (it, r)
        xs = [x.roll(1) for x in xs]


def test_two_stage_and_one_stage_calls_interleaved(cuda_device):
    """Both kernels on one workspace (they share the stage-0 flags and the epochs)."""
    W = 4
    ar = EmulatedQuantAllReduce(W, cuda_device, bits=8, group_size=128, algo="two_shot", timeout_ms=5000)
    for it, shape in enumerate([(300, 4096), (64, 4096), (1000, 4096), (7, 8192), (300, 4096), (2048, 4096)]):
        prev = set_two_shot_stages(1 + it % 2)
        try:
            xs = _inputs(W, shape, torch.bfloat16, cuda_device, seed=it)
            outs = ar(xs)
            ar.check()
        finally:
            set_two_shot_stages(prev)
        ref = spec.two_step_all_reduce_ref([x.cpu() for x in xs], 8, 128, "asym", torch.float16, torch.bfloat16)
        for r in range(W):
            assert torch.equal(outs[r].cpu(), ref), (it, shape, r)


# ------------------------------------------------------------------ norm kernel, warps per row
@pytest.fixture(params=[2, 4], ids=["wpr2", "wpr4"])
def norm_wpr(request):
    prev = set_norm_warps_per_row(request.param)
    yield request.param
    set_norm_warps_per_row(prev)


@pytest.mark.parametrize("W,M,H,bits,mode", [(2, 256, 1024, 8, "asym"), (4, 1000, 4096, 8, "asym"),
                                               (8, 300, 2048, 4, "sym"), (3, 77, 512, 6, "asym"),
                                               (1, 130, 1024, 8, "asym"), (8, 1024, 8192, 8, "asym")])
def test_norm_warps_per_row_matches_oracle(cuda_device, norm_wpr, W, M, H, bits, mode):
    """Residual shards bit-exact with the oracle, x identical on every rank and equal to the
    oracle up to rsqrt rounding (the row's sum of squares is added in another order)."""
    torch.manual_seed(M + H + bits)
    ar = EmulatedQuantAllReduce(W, cuda_device, bits=bits, group_size=128, quant_type=mode, algo="two_shot")
    R = (M + W - 1) // W
    ps = [torch.randn(M, H, device=cuda_device).to(torch.bfloat16) for _ in range(W)]
    hs = [torch.randn(R, H, device=cuda_device).to(torch.bfloat16) for _ in range(W)]
    w = (torch.rand(H, device=cuda_device) + 0.5).to(torch.bfloat16)
    hs_in = [h.cpu().clone() for h in hs]
    for rep in range(2):
        xs = ar.all_reduce_norm(ps, hs, w, 1e-5)
        ar.check()
        x_ref, h_ref = spec.two_step_all_reduce_norm_ref([p.cpu() for p in ps], hs_in, w.cpu(), 1e-5, bits, 128, mode)
        for r in range(W):
            n = max(0, min(M, (r + 1) * R) - r * R)
            assert torch.equal(hs[r].cpu()[:n], h_ref[r][:n]), (rep, r)
            assert torch.equal(xs[r], xs[0]), (rep, r)
        x0 = xs[0].cpu()
        assert (x0 != x_ref).float().mean().item() < 0.01
        assert spec.rel_l2(x0.float(), x_ref.float()) < (2e-3 if bits >= 8 else 2e-2)
        hs_in = h_ref


def test_norm_warps_per_row_after_fused_gemm(cuda_device, norm_wpr):
    """GEMM with the scatter epilogue + the multi-warp norm kernel == GEMM, then the same."""
    from quantized_flash_communication_b200.parallel import QuantAllReduce
    ar = QuantAllReduce(None, cuda_device, bits=8, group_size=128, quant_type="asym", algo="two_shot")
    for M, K, H in [(256, 512, 1024), (1000, 1376, 4096)]:
        a = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
        wt = torch.randn(H, K, device=cuda_device, dtype=torch.bfloat16) * 0.05
        nw = (torch.rand(H, device=cuda_device) + 0.5).to(torch.bfloat16)
        h0 = torch.randn(M, H, device=cuda_device, dtype=torch.bfloat16)
        h1, h2 = h0.clone(), h0.clone()
        x1 = ar.gemm_all_reduce_norm(a, wt, h1, nw, 1e-5)
        ar.check()
        x2 = ar.all_reduce_norm(G.linear(a, wt), h2, nw, 1e-5)
        ar.check()
        assert torch.equal(h1, h2) and torch.equal(x1, x2), (M, K, H)


# ------------------------------------------------------------------ packed softmax
@pytest.fixture
def packed_softmax():
    prev = ext().set_attn_packed(True)
    yield
    ext().set_attn_packed(prev)


def test_packed_exp2_rounds_like_the_scalar_one(cuda_device):
    x = torch.cat([torch.linspace(-125.0, 0.0, 1 << 20, device=cuda_device),
                   -torch.rand(1 << 20, device=cuda_device) * 30,
                   torch.tensor([0.0, -0.5, -1.0, -1.5, -2.5, -124.5, float("-inf")], device=cuda_device)])
    y, yp = torch.empty_like(x), torch.empty_like(x)
    ext().attn_exp2_poly(x, y)
    ext().attn_exp2_poly(x, yp, pairs=True)
    assert torch.equal(yp.view(torch.int32), y.view(torch.int32))


@pytest.mark.parametrize("B,S,nq,nkv", [(1, 128, 1, 1), (2, 300, 8, 2), (3, 257, 2, 2), (8, 1024, 4, 4)])
def test_packed_softmax_attention_matches_reference(cuda_device, packed_softmax, B, S, nq, nkv):
    hd = 128
    torch.manual_seed(B * S + nq)
    qkv = torch.randn(B * S, (nq + 2 * nkv) * hd, device=cuda_device, dtype=torch.bfloat16)
    o = prefill_attention(qkv, B, S, nq, nkv, hd)
    torch.cuda.synchronize()
    assert attn_status(clear=True) == 0
    assert rel_l2(o.float(), attn_ref(qkv, B, S, nq, nkv, hd)) < 1e-2
    assert torch.isfinite(o.float()).all()


def test_packed_softmax_with_growing_row_maxima(cuda_device, packed_softmax):
    B, S, nq, nkv, hd = 2, 1024, 4, 4, 128
    g = torch.Generator(device="cpu").manual_seed(S + nq)
    x = torch.randn(B * S, nq + 2 * nkv, hd, generator=g)
    x[:, nq:nq + nkv] *= (1.0 + 6.0 * torch.arange(S).float().repeat(B) / S)[:, None, None]
    x[:, :nq] *= (0.5 + torch.rand(B * S, nq, 1, generator=g) * 2.5)
    qkv = x.reshape(B * S, -1).to(cuda_device, torch.bfloat16)
    o = prefill_attention(qkv, B, S, nq, nkv, hd)
    torch.cuda.synchronize()
    assert attn_status(clear=True) == 0
    assert rel_l2(o.float(), attn_ref(qkv, B, S, nq, nkv, hd)) < 1e-2


# ------------------------------------------------------------------ weight-streaming GEMM
@pytest.fixture
def gemv_on():
    prev = ext().set_gemv(True)
    yield
    ext().set_gemv(prev)


@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (3, 300, 1000), (4, 1280, 8192), (8, 4096, 4096), (5, 9, 2056)])
def test_gemv_store_and_residual(cuda_device, gemv_on, M, N, K):
    torch.manual_seed(M * N + K)
    a = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=cuda_device, dtype=torch.bfloat16) * 0.05
    s = _sigma(a, b)
    ab = _ref(a, b)
    _check(G.linear(a, b), ab, s, what=f"gemv {M}x{N}x{K}")
    r = torch.randn(M, N, device=cuda_device, dtype=torch.bfloat16)
    ref = _bf16(ab) + r.float()
    G.linear_residual(a, b, r, out=r)
    torch.cuda.synchronize()
    _check(r, ref, s, what=f"gemv residual {M}x{N}x{K}", extra=2.0 ** -7 * ab.abs())


@pytest.mark.parametrize("M,I,K", [(1, 128, 64), (4, 3584, 8192), (7, 1376, 4096)])
def test_gemv_swiglu(cuda_device, gemv_on, M, I, K):
    torch.manual_seed(I + M)
    a = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(2 * I, K, device=cuda_device, dtype=torch.bfloat16) * 0.03
    y = G.linear_swiglu(a, w)
    torch.cuda.synchronize()
    g = _bf16(_ref(a, w[:I]))
    u = _bf16(_ref(a, w[I:]))
    ref = _bf16(torch.nn.functional.silu(g)) * u
    s = _sigma(a, w)
    _check(y, ref, s * s, rel=2.0 ** -7, what=f"gemv swiglu {M}x{I}x{K}", extra=2.0 ** -6 * (g.abs() + 1.0) * u.abs())


def test_gemv_declines_more_than_eight_rows(cuda_device, gemv_on):
    a = torch.randn(9, 512, device=cuda_device, dtype=torch.bfloat16)
    b = torch.randn(256, 512, device=cuda_device, dtype=torch.bfloat16) * 0.05
    _check(G.linear(a, b), _ref(a, b), _sigma(a, b), what="9 rows")


# ------------------------------------------------------------------ two-stage kernel on real ranks
WORLD = (min(torch.cuda.device_count(), int(os.environ.get("QFC_TEST_WORLD", "4")))
         if torch.cuda.is_available() else 0)


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from quantized_flash_communication_b200.communication import reset_communicators
        from quantized_flash_communication_b200.parallel import QuantAllReduce
        dev = torch.device("cuda", rank)
        ar = QuantAllReduce(None, dev, bits=8, group_size=128, quant_type="asym", timeout_ms=5000)
        prev = set_two_shot_stages(2)
        ok = True
        for it, shape in enumerate([(300, 4096), (1000, 4096), (4096, 4096)]):
            xs = []
            for r in range(world):
                g = torch.Generator().manual_seed(2000 + it + r)
                xs.append(torch.randn(*shape, generator=g).to(torch.bfloat16))
            y = ar(xs[rank].to(dev), algo="two_shot")
            ar.check()
            ok = ok and torch.equal(y.cpu(), spec.two_step_all_reduce_ref(xs, 8, 128, "asym", torch.float16,
                                                                          torch.bfloat16))
        set_two_shot_stages(prev)
        results[rank] = ok
        reset_communicators()
    finally:
        dist.destroy_process_group()


@pytest.mark.multigpu
@pytest.mark.skipif(WORLD < 2, reason="needs >= 2 GPUs")
def test_two_stage_two_shot_on_real_ranks():
    mgr = mp.Manager()
    results = mgr.dict()
    mp.spawn(_worker, args=(WORLD, free_port(), results), nprocs=WORLD, join=True)
    assert all(results[r] for r in range(WORLD)), dict(results)
