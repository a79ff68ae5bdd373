"""Failure detection on CPU ranks (gloo): the failure is made on the host, no GPU involved.

A rank that never joins an all-reduce, and a rank that raises before it, must end the
other rank's call with an error within the process group's timeout instead of leaving it
waiting.  The ranks run the package's staged two-step all-reduce (the gloo path of
``flash_all_reduce``), with the process group created through ``init_distributed`` and a
short timeout.
"""
import os
import time

import pytest
import torch.multiprocessing as mp

from conftest import free_port

TIMEOUT_S = 3.0


def _worker(rank, world, port, behaviour, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch
    import torch.distributed as dist
    from quantized_flash_communication_b200.parallel.staged import staged_all_reduce
    from quantized_flash_communication_b200.utils.dist import init_distributed
    init_distributed(backend="gloo", timeout_s=TIMEOUT_S)
    x = torch.randn(8, 4096, generator=torch.Generator().manual_seed(rank))
    # one call that every rank takes, so that the group is known to work
    staged_all_reduce(x, 8, 128, "asym", torch.float16, None, torch.float32)
    if rank == 1 and behaviour == "never_joins":
        time.sleep(3 * TIMEOUT_S)  # skips the next call; leaves without destroying the group
        results[rank] = "left"
        os._exit(0)
    if rank == 1 and behaviour == "raises":
        results[rank] = "raised"
        raise RuntimeError("injected failure on rank 1")
    t0 = time.time()
    try:
        staged_all_reduce(x, 8, 128, "asym", torch.float16, None, torch.float32)
        results[rank] = ("completed", time.time() - t0)
    except Exception as e:  # the failure must surface as an exception
        results[rank] = ("error", time.time() - t0, type(e).__name__, str(e)[:200])
    os._exit(0)  # the group is broken: do not wait in its destructor


def _run(behaviour):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, behaviour, results)) for r in range(2)]
    for p in procs:
        p.start()
    deadline = time.time() + 120
    for p in procs:
        p.join(max(1.0, deadline - time.time()))
    alive = [p for p in procs if p.is_alive()]
    for p in alive:  # only our own child processes, by handle
        p.kill()
        p.join(5)
    assert not alive, f"ranks still running after 120 s ({behaviour})"
    return dict(results)


@pytest.mark.parametrize("behaviour", ["never_joins", "raises"])
def test_peer_failure_ends_the_call_with_an_error(behaviour):
    res = _run(behaviour)
    assert res[1] in ("left", "raised"), res
    status = res[0]
    assert status[0] == "error", status
    assert status[1] < 10 * TIMEOUT_S, status  # bounded by the group's timeout, not hung
