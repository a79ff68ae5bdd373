"""Fused quantized all-reduce kernel on ONE GPU, with W ranks emulated in one launch.

Each emulated rank has its own workspace; block row y of the launch plays rank y and
stores into the other ranks' buffers, so the flag protocol, slot layout and numerics of
the multi-GPU kernel run unchanged.  Results must equal the oracle bit for bit and be
identical on every rank.
"""
import pytest
import torch

from quantized_flash_communication_b200 import quantization as spec
from quantized_flash_communication_b200._ext import ext
from quantized_flash_communication_b200.parallel import EmulatedQuantAllReduce

pytestmark = pytest.mark.gpu


def _inputs(W, shape, dtype, device, seed=0):
    xs = []
    for r in range(W):
        g = torch.Generator(device="cpu").manual_seed(seed + r)
        x = torch.randn(*shape, generator=g)
        x.view(-1)[::1000] *= 50  # 0.1% outliers
        xs.append(x.to(dtype).to(device))
    return xs


CASES = [
    # (W, bits, gs, mode, shape, algo)
    (2, 8, 128, "asym", (8, 4096), "two_shot"),
    (8, 8, 128, "asym", (128, 4096), "two_shot"),
    (8, 6, 128, "asym", (16, 8192), "two_shot"),
    (8, 4, 128, "sym", (16, 4096), "two_shot"),
    (4, 8, 32, "sym", (3, 1000), "two_shot"),
    (4, 4, 64, "asym", (1, 4096), "two_shot"),
    (8, 16, 128, "asym", (1024, 4096), "two_shot"),
    (1, 8, 128, "asym", (5, 4096), "two_shot"),
    (3, 8, 128, "asym", (37, 4096), "two_shot"),   # generic (runtime world size) kernels
    (5, 6, 64, "sym", (9, 1000), "two_shot"),
    (4, 8, 16, "asym", (6, 4096), "two_shot"),     # one lane per group
    (2, 4, 256, "sym", (10, 4096), "two_shot"),    # two groups per 512-element unit
    (3, 8, 8, "asym", (5, 1000), "two_shot"),      # 8-element groups: 8-per-lane kernel
    (8, 6, 32, "asym", (33, 8192), "two_shot"),
    (3, 4, 128, "asym", (5, 4096), "one_shot"),
    (2, 8, 128, "asym", (1, 4096), "one_shot"),
    (8, 8, 128, "asym", (64, 4096), "one_shot"),
    (8, 4, 128, "sym", (7, 999), "one_shot"),
    (8, 6, 256, "asym", (4, 4096), "one_shot"),
    (4, 16, 128, "asym", (16, 4096), "one_shot"),
]


@pytest.mark.parametrize("W,bits,gs,mode,shape,algo", CASES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_emulated_matches_oracle(cuda_device, W, bits, gs, mode, shape, algo, dtype):
    ar = EmulatedQuantAllReduce(W, cuda_device, bits=bits, group_size=gs, quant_type=mode, algo=algo,
                                timeout_ms=5000)
    xs = _inputs(W, shape, dtype, cuda_device, seed=W * 100 + bits)
    for it in range(3):  # repeated calls exercise epochs and slot reuse
        outs = ar(xs)
        ar.check()
        cpu = [x.cpu() for x in xs]
        if algo == "two_shot":
            ref = spec.two_step_all_reduce_ref(cpu, bits, gs, mode, torch.float16, dtype)
        else:
            ref = spec.one_shot_all_reduce_ref(cpu, bits, gs, mode, torch.float16, dtype)
        for r in range(W):
            assert torch.equal(outs[r].cpu(), ref), (it, r)
        xs = [x.roll(1) for x in xs]


def test_sizes_change_between_calls(cuda_device):
    """One workspace, back-to-back calls whose sizes (and so grids) change, one-shot and
    two-shot interleaved: the one-shot slot region follows the rank's call count, the
    same in every block, so every call must still match the oracle on every rank."""
    W = 4
    ar = EmulatedQuantAllReduce(W, cuda_device, bits=8, group_size=128, quant_type="asym", algo="auto",
                                timeout_ms=5000)
    shapes = [(1, 4096), (64, 4096), (5, 1000), (16, 8192), (64, 4096), (1, 4096), (300, 4096), (7, 4096)]
    for it, shape in enumerate(shapes):
        xs = _inputs(W, shape, torch.bfloat16, cuda_device, seed=it)
        one = xs[0].numel() * 2 <= ar.one_shot_max_bytes
        outs = ar(xs)
        ar.check()
        cpu = [x.cpu() for x in xs]
        if one:
            ref = spec.one_shot_all_reduce_ref(cpu, 8, 128, "asym", torch.float16, torch.bfloat16)
        else:
            ref = spec.two_step_all_reduce_ref(cpu, 8, 128, "asym", torch.float16, torch.bfloat16)
        for r in range(W):
            assert torch.equal(outs[r].cpu(), ref), (it, shape, r)


@pytest.mark.parametrize("scale_dtype", [torch.float32])
def test_fp32_scales_and_fp16_output(cuda_device, scale_dtype):
    W = 4
    ar = EmulatedQuantAllReduce(W, cuda_device, bits=8, group_size=128, quant_type="sym", scale_dtype=scale_dtype,
                                algo="two_shot")
    xs = _inputs(W, (32, 4096), torch.bfloat16, cuda_device)
    outs = ar(xs, out_dtype=torch.float16)
    ar.check()
    ref = spec.two_step_all_reduce_ref([x.cpu() for x in xs], 8, 128, "sym", scale_dtype, torch.float16)
    for r in range(W):
        assert torch.equal(outs[r].cpu(), ref)


def test_exact_local_contribution(cuda_device):
    W = 2
    xs = _inputs(W, (4, 4096), torch.float32, cuda_device)
    exact = (xs[0] + xs[1]).cpu()
    errs = {}
    for ql in (True, False):
        ar = EmulatedQuantAllReduce(W, cuda_device, bits=8, group_size=128, algo="two_shot", quantize_local=ql)
        outs = ar(xs)
        ar.check()
        assert torch.equal(outs[0].cpu(), outs[1].cpu())
        errs[ql] = spec.rel_l2(outs[0].cpu(), exact)
    assert errs[False] < errs[True] < 0.05, errs


def test_in_place(cuda_device):
    W = 4
    ar = EmulatedQuantAllReduce(W, cuda_device, bits=8, group_size=128, algo="two_shot")
    xs = _inputs(W, (16, 4096), torch.bfloat16, cuda_device)
    ref = spec.two_step_all_reduce_ref([x.cpu() for x in xs], 8, 128, "asym", torch.float16, torch.bfloat16)
    ar(xs, outs=xs)
    ar.check()
    for r in range(W):
        assert torch.equal(xs[r].cpu(), ref)


def test_cuda_graph_replay(cuda_device):
    W = 4
    ar = EmulatedQuantAllReduce(W, cuda_device, bits=8, group_size=128, algo="auto")
    xs = _inputs(W, (64, 4096), torch.bfloat16, cuda_device)
    outs = [torch.empty_like(x) for x in xs]
    ar(xs, outs)  # warm-up sizes the workspaces
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ar(xs, outs)
    for it in range(4):
        for x in xs:
            x.copy_(torch.randn_like(x))
        g.replay()
        ar.check()
        ref = spec.one_shot_all_reduce_ref([x.cpu() for x in xs], 8, 128, "asym", torch.float16, torch.bfloat16)
        for r in range(W):
            assert torch.equal(outs[r].cpu(), ref), it


@pytest.mark.parametrize("bits,mode", [(8, "asym"), (4, "sym"), (6, "asym"), (16, "asym")])
def test_gemm_fused_scatter_single_rank(cuda_device, bits, mode):
    """GEMM with the quantize-and-scatter epilogue + reduce-gather == GEMM then all-reduce."""
    from quantized_flash_communication_b200.ops import gemm as G
    from quantized_flash_communication_b200.parallel import QuantAllReduce
    ar = QuantAllReduce(None, cuda_device, bits=bits, group_size=128, quant_type=mode, algo="two_shot")
    for M, K, N in [(256, 512, 1024), (1000, 1376, 4096), (130, 256, 384)]:
        a = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
        w = torch.randn(N, K, device=cuda_device, dtype=torch.bfloat16) * 0.05
        for _ in range(2):
            fused = ar.gemm_all_reduce(a, w)
            ar.check()
            plain = ar(G.linear(a, w))
            ar.check()
            assert torch.equal(fused, plain), (M, K, N)
        ref = spec.two_step_all_reduce_ref([G.linear(a, w).cpu()], bits, 128, mode, torch.float16, torch.bfloat16)
        assert torch.equal(fused.cpu(), ref)


@pytest.mark.parametrize("W,M,H,bits,mode", [(2, 256, 1024, 8, "asym"), (4, 1000, 4096, 8, "asym"),
                                               (8, 300, 2048, 4, "sym"), (3, 77, 512, 6, "asym"),
                                               (2, 64, 256, 16, "asym"), (1, 130, 1024, 8, "asym")])
def test_emulated_all_reduce_norm(cuda_device, W, M, H, bits, mode):
    """Sequence-parallel all-reduce + residual + RMSNorm: residual shards bit-exact with the
    oracle, x identical on every rank and equal to the oracle up to rsqrt rounding."""
    from quantized_flash_communication_b200.parallel import EmulatedQuantAllReduce
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
        hs_in = h_ref  # the second call continues from the updated shards


def test_gemm_fused_all_reduce_norm_single_rank(cuda_device):
    """GEMM with the scatter epilogue + norm kernel == GEMM, then the norm all-reduce."""
    from quantized_flash_communication_b200.ops import gemm as G
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


def test_timeout_reports_status_and_context_survives(cuda_device):
    """Rank 0 of a 2-rank workspace whose peer never runs: every wait must expire."""
    C = ext()
    ws0 = C.Workspace(0, 0, 2, 1 << 22, 1 << 22, 1 << 22)
    ws1 = C.Workspace(0, 1, 2, 1 << 22, 1 << 22, 1 << 22)  # "peer" memory nobody signals
    ws0.set_peer_ptrs([ws0.local_ptr, ws1.local_ptr])
    x = torch.randn(8, 4096, device=cuda_device, dtype=torch.bfloat16)
    out = torch.empty_like(x)
    C.quant_all_reduce([ws0], [x], [out], 8, 128, False, False, False, True, 50.0)
    torch.cuda.synchronize()
    code, phase, block, peer, want, seen = ws0.status()
    assert code == 1 and phase == 0 and peer == 1 and want == 1 and seen == 0
    ws0.clear_status()
    assert ws0.status()[0] == 0
    # the context is still usable
    y = (x.float() * 2).sum()
    torch.cuda.synchronize()
    assert torch.isfinite(y)
