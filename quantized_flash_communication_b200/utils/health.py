"""Host-side liveness of the ranks of a tensor-parallel group.

The fused collectives wait for their peers on the device, with a bounded wait that ends
in ``CommTimeoutError`` (``parallel/symm_mem.py``).  A rank that has died is better
noticed on the host before the next launch: the launch would otherwise spend the whole
device timeout waiting for a peer that will never arrive.  ``PeerMonitor`` keeps a
heartbeat per rank in a ``torch.distributed`` key-value store (its own TCP client, so it
never shares a connection with collectives in flight): a background thread writes this
rank's wall-clock time every ``interval_s``; ``check()`` reads the peers' entries and
raises ``PeerLostError`` for a peer whose heartbeat is older than ``stale_s`` or that
announced its exit.  Call ``check()`` between steps (``LlamaTP.generate`` takes a
``monitor`` for that), never while a step's kernels are in flight.

All ranks run on one node, so their wall clocks agree.
"""
from __future__ import annotations

import os
import threading
import time
from datetime import timedelta
from typing import List, Optional

import torch.distributed as dist

__all__ = ["PeerMonitor", "PeerLostError"]

_EXIT = "exit"


class PeerLostError(RuntimeError):
    """A rank of the group stopped its heartbeat or left."""

    def __init__(self, rank: int, peers: List[int], reason: str):
        super().__init__(f"rank {rank}: peer rank(s) {peers} {reason}; the tensor-parallel group is no longer "
                         "usable")
        self.peers = peers


class PeerMonitor:
    def __init__(self, rank: int, world: int, store: Optional[dist.Store] = None, interval_s: float = 0.5,
                 stale_s: float = 5.0, prefix: str = "qfc_heartbeat", host: Optional[str] = None,
                 port: Optional[int] = None):
        """``store``: an existing store; by default a new TCP client of the rendezvous store at
        ``host``:``port`` (MASTER_ADDR / MASTER_PORT)."""
        if stale_s <= 2 * interval_s:
            raise ValueError("stale_s must exceed two heartbeat intervals")
        self.rank, self.world = rank, world
        self.interval_s, self.stale_s, self.prefix = interval_s, stale_s, prefix
        if store is None:
            host = host or os.environ.get("MASTER_ADDR", "127.0.0.1")
            port = int(port or os.environ["MASTER_PORT"])
            store = dist.TCPStore(host, port, is_master=False, timeout=timedelta(seconds=30))
        self.store = store
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def _beat(self):
        self.store.set(self._key(self.rank), repr(time.time()))

    def start(self) -> "PeerMonitor":
        self._beat()

        def loop():
            while not self._stop.wait(self.interval_s):
                try:
                    self._beat()
                except Exception:  # the store went away: the peers will see this rank go stale
                    return
        self._thread = threading.Thread(target=loop, name="qfc-heartbeat", daemon=True)
        self._thread.start()
        return self

    def wait_for_peers(self, timeout_s: float = 60.0):
        """Block until every rank has written a first heartbeat."""
        keys = [self._key(r) for r in range(self.world)]
        deadline = time.time() + timeout_s
        while not self.store.check(keys):
            if time.time() > deadline:
                missing = [r for r in range(self.world) if not self.store.check([self._key(r)])]
                raise PeerLostError(self.rank, missing, f"never joined within {timeout_s} s")
            time.sleep(min(self.interval_s, 0.1))

    def check(self):
        """Raise ``PeerLostError`` if a peer's heartbeat is stale or the peer has exited."""
        now = time.time()
        stale, left = [], []
        for r in range(self.world):
            if r == self.rank:
                continue
            key = self._key(r)
            if not self.store.check([key]):
                stale.append(r)
                continue
            v = self.store.get(key).decode()
            if v == _EXIT:
                left.append(r)
            elif now - float(v) > self.stale_s:
                stale.append(r)
        if left:
            raise PeerLostError(self.rank, left, "left the group")
        if stale:
            raise PeerLostError(self.rank, stale, f"sent no heartbeat for more than {self.stale_s} s")

    def stop(self, announce_exit: bool = True):
        """Stop the heartbeat; ``announce_exit`` tells the peers at once that this rank left."""
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2 * self.interval_s + 1.0)
        if announce_exit:
            try:
                self.store.set(self._key(self.rank), _EXIT)
            except Exception:
                pass
