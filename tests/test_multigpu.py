"""Multi-GPU checks (one process per GPU, NCCL process group, CUDA-IPC peer workspaces).

Skipped unless at least two GPUs are visible.  Every spin-wait in the kernels is bounded,
and the failure test only makes a wait run out (a peer that never joins); it faults,
traps or hangs no GPU.  NVLS is disabled for these child processes.
"""
import os
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import free_port

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

# QFC_TEST_WORLD raises the rank count (default: up to 4 of the visible GPUs).
WORLD = (min(torch.cuda.device_count(), int(os.environ.get("QFC_TEST_WORLD", "4")))
         if torch.cuda.is_available() else 0)
need2 = pytest.mark.skipif(WORLD < 2, reason="needs >= 2 GPUs")


def _inputs(world, shape, dtype, seed):
    xs = []
    for r in range(world):
        g = torch.Generator().manual_seed(seed + r)
        x = torch.randn(*shape, generator=g)
        x.view(-1)[::1000] *= 50
        xs.append(x.to(dtype))
    return xs


def _case_allreduce(rank, world):
    from quantized_flash_communication_b200 import quantization as spec
    from quantized_flash_communication_b200.communication import flash_all_reduce
    from quantized_flash_communication_b200.parallel import QuantAllReduce
    dev = torch.device("cuda", rank)
    res = {}
    cases = [(8, 128, "asym", (64, 4096), "two_shot"), (6, 128, "asym", (33, 4096), "two_shot"),
             (4, 64, "sym", (16, 8192), "two_shot"), (16, 128, "asym", (128, 4096), "two_shot"),
             (8, 128, "asym", (4, 4096), "one_shot"), (4, 128, "asym", (7, 999), "one_shot"),
             (8, 32, "sym", (1000, 4096), "auto")]
    for bits, gs, mode, shape, algo in cases:
        ar = QuantAllReduce(None, dev, bits=bits, group_size=gs, quant_type=mode, algo=algo, timeout_ms=5000)
        ok = True
        for it in range(3):
            xs = _inputs(world, shape, torch.bfloat16, 100 * it + bits)
            y = ar(xs[rank].to(dev))
            ar.check()
            one = algo == "one_shot" or (algo == "auto" and xs[0].numel() * 2 <= 512 * 1024)
            fn = spec.one_shot_all_reduce_ref if one else spec.two_step_all_reduce_ref
            ref = fn(xs, bits, gs, mode, torch.float16, torch.bfloat16)
            ok = ok and torch.equal(y.cpu(), ref)
        res[(bits, gs, mode, shape, algo)] = ok
    # one workspace, sizes (and so grids) changing between back-to-back calls, one rank
    # lagging: the one-shot slot region must follow the call count, not a block's epoch
    ar = QuantAllReduce(None, dev, bits=8, group_size=128, quant_type="asym", algo="auto", timeout_ms=5000)
    ok = True
    for it, shape in enumerate([(1, 4096), (64, 4096), (5, 1000), (16, 8192), (300, 4096), (7, 4096)] * 2):
        xs = _inputs(world, shape, torch.bfloat16, 1000 + it)
        if rank == it % world:
            torch.cuda._sleep(100_000)  # this rank starts late; the others run ahead
        y = ar(xs[rank].to(dev))
        ar.check()
        one = xs[0].numel() * 2 <= 512 * 1024
        fn = spec.one_shot_all_reduce_ref if one else spec.two_step_all_reduce_ref
        ok = ok and torch.equal(y.cpu(), fn(xs, 8, 128, "asym", torch.float16, torch.bfloat16))
    res["sizes_change_between_calls"] = ok
    # reference-compatible API: fp16 output, host-timed latency
    xs = _inputs(world, (8, 4096), torch.float16, 7)
    y, ms = flash_all_reduce(xs[rank].to(dev), group_size=128, bits=8, quant_type="asym")
    ref = spec.two_step_all_reduce_ref(xs, 8, 128, "asym", torch.float16, torch.float16)
    res["flash_all_reduce"] = bool(torch.equal(y.cpu(), ref)) and y.dtype == torch.float16 and ms > 0
    return res


def _case_gemm_fused(rank, world):
    from quantized_flash_communication_b200 import quantization as spec
    from quantized_flash_communication_b200.ops import gemm as G
    from quantized_flash_communication_b200.parallel import QuantAllReduce
    dev = torch.device("cuda", rank)
    res = {}
    for bits in (8, 6, 16):
        ar = QuantAllReduce(None, dev, bits=bits, group_size=128, algo="two_shot", timeout_ms=5000)
        for M, K, N in [(512, 512, 4096), (300, 1376, 1024)]:
            outs = []
            for r in range(world):
                g = torch.Generator().manual_seed(10 * r + M)
                a = torch.randn(M, K, generator=g).to(torch.bfloat16).to(dev)
                w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16).to(dev)
                outs.append((a, w))
            parts = [G.linear(a, w).cpu() for a, w in outs]  # every rank's partial, computed here
            ref = spec.two_step_all_reduce_ref(parts, bits, 128, "asym", torch.float16, torch.bfloat16)
            ok = True
            for _ in range(2):
                y = ar.gemm_all_reduce(*outs[rank])
                ar.check()
                ok = ok and torch.equal(y.cpu(), ref)
            res[(bits, M, K, N)] = ok
    return res


def _case_model(rank, world):
    from quantized_flash_communication_b200.models.config import get_config
    from quantized_flash_communication_b200.models.llama import LlamaTP, TPContext
    from quantized_flash_communication_b200.quantization import rel_l2
    dev = torch.device("cuda", rank)
    cfg = get_config("tiny-mha")
    ids = torch.randint(0, cfg.vocab_size, (4, 96), generator=torch.Generator().manual_seed(3)).to(dev)
    out = {}
    ref = LlamaTP(cfg, TPContext(device=dev, world=1), dev, init="full", seed=9)
    _, h1 = ref.prefill(ids, return_last_hidden=True)
    for bits, sp in ((16, False), (8, False), (16, True), (8, True)):
        tp = TPContext(None, dev, ar_backend="qfc", bits=bits, group_size=128, seq_parallel=sp)
        m = LlamaTP(cfg, tp, dev, init="full", seed=9)
        cache = m.new_cache(4, 100)
        tok, h = m.prefill(ids, cache, return_last_hidden=True)
        tok2 = m.decode_step(tok, cache)
        gathered = [torch.empty_like(h) for _ in range(world)]
        dist.all_gather(gathered, h)
        out[(bits, sp)] = dict(err=rel_l2(h.float(), h1.float()), same=all(torch.equal(g, h) for g in gathered),
                               tok2_shape=tuple(tok2.shape), sp_used=tp.sp_active(ids.numel(), cfg.hidden_size))
        tp.ar.check()
    return out


def _case_sampling(rank, world):
    """Every rank must draw the same sampled tokens (temperature and top-p paths)."""
    from quantized_flash_communication_b200.models.config import get_config
    from quantized_flash_communication_b200.models.llama import LlamaTP, TPContext
    dev = torch.device("cuda", rank)
    cfg = get_config("tiny-mha")
    ids = torch.randint(0, cfg.vocab_size, (3, 20), generator=torch.Generator().manual_seed(8)).to(dev)
    m = LlamaTP(cfg, TPContext(None, dev, ar_backend="qfc", bits=8), dev, init="full", seed=4)
    out = {}
    for top_p in (1.0, 0.9):
        toks = m.generate(ids, 10, do_sample=True, temperature=0.7, top_p=top_p)  # seed from rank 0
        gathered = [torch.empty_like(toks) for _ in range(world)]
        dist.all_gather(gathered, toks)
        out[top_p] = all(torch.equal(g, toks) for g in gathered)
    m.tp.ar.check()
    return out


def _case_peer_never_joins(rank, world):
    """Rank 1 skips an all-reduce: rank 0's kernel must time out and report it."""
    from quantized_flash_communication_b200.parallel import CommTimeoutError, QuantAllReduce
    dev = torch.device("cuda", rank)
    ar = QuantAllReduce(None, dev, bits=8, algo="two_shot", timeout_ms=200)
    x = torch.randn(16, 4096, device=dev, dtype=torch.bfloat16)
    ar(x)
    ar.check()  # one good call first
    dist.barrier()
    raised = None
    if rank == 0:
        ar(x)
        try:
            ar.check()
        except CommTimeoutError as e:
            raised = str(e)
    torch.cuda.synchronize()
    dist.barrier()
    return raised


def _worker(rank, world, port, case, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        results[rank] = globals()[case](rank, world)
    finally:
        from quantized_flash_communication_b200.communication import reset_communicators
        reset_communicators()
        dist.destroy_process_group()


def _run(case, world=WORLD):
    mgr = mp.Manager()
    results = mgr.dict()
    mp.spawn(_worker, args=(world, free_port(), case, results), nprocs=world, join=True)
    return dict(results)


@need2
def test_fused_allreduce_matches_oracle_on_every_rank():
    res = _run("_case_allreduce")
    for rank, r in res.items():
        for k, ok in r.items():
            assert ok, (rank, k)


@need2
def test_gemm_fused_scatter_matches_oracle_on_every_rank():
    res = _run("_case_gemm_fused")
    for rank, r in res.items():
        for k, ok in r.items():
            assert ok, (rank, k)


@need2
def test_tp_model_matches_tp1():
    res = _run("_case_model")
    for rank, r in res.items():
        for sp in (False, True):  # plain all-reduce, and the sequence-parallel residual
            assert r[(16, sp)]["err"] < 0.02, r
            assert r[(8, sp)]["err"] < 0.08, r
            assert r[(16, sp)]["same"] and r[(8, sp)]["same"]
            assert r[(8, sp)]["sp_used"] == sp


@need2
def test_sampled_generation_is_identical_on_every_rank():
    res = _run("_case_sampling")
    for rank, r in res.items():
        assert r[1.0] and r[0.9], (rank, r)


@need2
def test_peer_that_never_joins_times_out_cleanly():
    res = _run("_case_peer_never_joins", world=2)
    assert res[0] is not None and "timed out" in res[0]
    assert res[1] is None
