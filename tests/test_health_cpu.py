"""Host-side liveness of the ranks (utils/health.py), with processes and a TCP store on
the CPU: a rank that stops its heartbeat or announces its exit is reported by the others'
``check()`` within the staleness window; live ranks are not."""
import time

import pytest
import torch.multiprocessing as mp

from conftest import free_port


def _worker(rank, world, port, behaviour, results):
    from datetime import timedelta

    import torch.distributed as dist

    from quantized_flash_communication_b200.utils.health import PeerLostError, PeerMonitor
    # rank 0 hosts the store; every monitor opens its own client connection to it
    store = dist.TCPStore("127.0.0.1", port, world_size=world, is_master=(rank == 0),
                          timeout=timedelta(seconds=30), wait_for_workers=False)
    mon = PeerMonitor(rank, world, host="127.0.0.1", port=port, interval_s=0.2, stale_s=1.0).start()
    mon.wait_for_peers(timeout_s=30)
    time.sleep(0.6)
    try:
        mon.check()  # everyone alive
        first = "ok"
    except PeerLostError as e:
        first = f"false alarm: {e}"
    store.set(f"checked/{rank}", "1")
    store.wait([f"checked/{r}" for r in range(world)])
    if rank == 1:
        mon.stop(announce_exit=(behaviour == "exits"))  # "stalls": the heartbeat just stops
        results[rank] = first
        time.sleep(2.5)  # stay alive while rank 0 checks
        return
    t0 = time.time()
    seen = None
    while time.time() - t0 < 10:
        try:
            mon.check()
        except PeerLostError as e:
            seen = (str(e), time.time() - t0, e.peers)
            break
        time.sleep(0.1)
    results[rank] = (first, seen)
    mon.stop()
    time.sleep(3.0)  # keep the store up until rank 1 has finished


@pytest.mark.parametrize("behaviour", ["exits", "stalls"])
def test_lost_peer_is_reported(behaviour):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, behaviour, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    for p in procs:
        if p.is_alive():  # our own children only
            p.kill()
            p.join(5)
    assert results[1] == "ok", dict(results)
    first, seen = results[0]
    assert first == "ok", first
    assert seen is not None and seen[2] == [1], seen
    assert ("left" in seen[0]) if behaviour == "exits" else ("heartbeat" in seen[0])
    assert seen[1] < (1.0 if behaviour == "exits" else 3.0), seen


def test_bad_windows_are_refused():
    from quantized_flash_communication_b200.utils.health import PeerMonitor
    with pytest.raises(ValueError):
        PeerMonitor(0, 2, store=object(), interval_s=1.0, stale_s=1.5)
