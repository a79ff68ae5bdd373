"""Two-step quantized all-reduce on CPU / gloo ranks (no GPU).

The gloo configuration: world_size 2, each rank holds fp32 [8, 4096] drawn N(0,1) from
seed+rank; symmetric groups of 128 with fp32 absmax scales; INT8 and INT4 (nibble
packed); checked against the exact fp32 sum by relative L2 and bit-for-bit against the
single-process oracle.
"""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import free_port


def _worker(rank, world, port, cases, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from quantized_flash_communication_b200 import quantization as spec
        from quantized_flash_communication_b200.communication import flash_all_reduce
        from quantized_flash_communication_b200.parallel.staged import staged_all_reduce
        out = {}
        for (bits, gs, mode, sd, shape) in cases:
            xs = []
            for r in range(world):
                g = torch.Generator().manual_seed(1234 + r)
                xs.append(torch.randn(*shape, generator=g))
            y = staged_all_reduce(xs[rank], bits, gs, mode, sd, None, torch.float32)
            ref = spec.two_step_all_reduce_ref(xs, bits, gs, mode, sd, torch.float32)
            exact = sum(x.double() for x in xs)
            y2, ms = flash_all_reduce(xs[rank].clone(), group_size=gs, bits=bits, quant_type=mode,
                                      out_dtype=torch.float32, scale_dtype=sd)
            gathered = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(gathered, y)
            out[(bits, gs, mode, str(sd), shape)] = dict(
                exact_match=bool(torch.equal(y, ref)),
                compat_match=bool(torch.equal(y2, ref)),
                ranks_agree=all(torch.equal(g_, gathered[0]) for g_ in gathered),
                rel_l2=spec.rel_l2(y, exact.float()),
                ms=ms)
        results[rank] = out
    finally:
        dist.destroy_process_group()


def _run(world, cases):
    port = free_port()
    mgr = mp.Manager()
    results = mgr.dict()
    mp.spawn(_worker, args=(world, port, cases, results), nprocs=world, join=True)
    return dict(results)


def test_baseline_config1_gloo_w2():
    cases = [(8, 128, "sym", torch.float32, (8, 4096)), (4, 128, "sym", torch.float32, (8, 4096))]
    res = _run(2, cases)
    for rank in range(2):
        for key, r in res[rank].items():
            assert r["exact_match"], (rank, key)
            assert r["compat_match"], (rank, key)
            assert r["ranks_agree"], (rank, key)
    r8 = res[0][(8, 128, "sym", str(torch.float32), (8, 4096))]["rel_l2"]
    r4 = res[0][(4, 128, "sym", str(torch.float32), (8, 4096))]["rel_l2"]
    # INT8 ~ 0.6%, INT4 ~ 12% relative L2 for Gaussian inputs at group 128
    assert r8 < 0.02, r8
    assert r4 < 0.25, r4


def test_gloo_modes_w3_odd_sizes():
    cases = [(6, 64, "asym", torch.float16, (5, 999)), (16, 32, "asym", torch.float16, (7, 33)),
             (4, 256, "asym", torch.float16, (3, 1000)), (8, 1024, "sym", torch.float16, (2, 3000))]
    res = _run(3, cases)
    for rank in range(3):
        for key, r in res[rank].items():
            assert r["exact_match"] and r["compat_match"] and r["ranks_agree"], (rank, key, r)
