"""Peer-mapped symmetric workspaces for the fused cross-GPU kernels.

A :class:`SymmetricWorkspace` wraps the native ``_C.Workspace`` (``csrc/workspace.cu``):
one device buffer per rank, mapped into every other rank's address space with CUDA IPC.
The 64-byte IPC handles travel once over ``torch.distributed`` (``all_gather_object``),
after which kernels store straight into peers' memory over NVLink / NVSwitch.

:class:`EmulatedWorkspaces` builds W workspaces on ONE GPU whose "peer" pointers are the
other local buffers; a kernel launched with ``gridDim.y == W`` then runs all W ranks of
the protocol in one launch (used to test the multi-rank protocol on a single GPU).

The reference has no counterpart (it uses NCCL collectives only, communication.py:48-81).
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist

from .._ext import ext

__all__ = ["SymmetricWorkspace", "EmulatedWorkspaces", "CommTimeoutError", "default_timeout_ms"]


class CommTimeoutError(RuntimeError):
    """A fused cross-GPU kernel gave up waiting for a peer's flag."""


_PHASES = {0: "reduce-scatter", 1: "all-gather", 2: "one-shot", 3: "gemm-scatter", 4: "argmax"}


def default_timeout_ms() -> float:
    return float(os.environ.get("QFC_COMM_TIMEOUT_MS", "10000"))


@dataclass
class Capacity:
    rs_bytes: int
    ag_bytes: int
    os_bytes: int


def _round_cap(v: int) -> int:
    # round up to a multiple of 2 MiB so that small growth steps do not thrash
    q = 2 << 20
    return max(q, (int(v) + q - 1) // q * q)


class SymmetricWorkspace:
    """One rank's peer-mapped workspace for a process group.

    Every rank of ``group`` must construct it (collectively) and must later make the same
    sequence of calls that may grow it.
    """

    def __init__(self, group: Optional[dist.ProcessGroup] = None, device: Optional[torch.device] = None,
                 rs_bytes: int = 8 << 20, ag_bytes: int = 8 << 20, os_bytes: int = 4 << 20):
        self.group = group
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        if dist.is_available() and dist.is_initialized():
            self.world = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        self._ws = None
        self._alloc(Capacity(_round_cap(rs_bytes), _round_cap(ag_bytes), _round_cap(os_bytes)))

    # -- allocation / rendezvous ------------------------------------------------------
    def _alloc(self, cap: Capacity):
        C = ext()
        self._ws = C.Workspace(self.device.index, self.rank, self.world, cap.rs_bytes, cap.ag_bytes,
                               cap.os_bytes)
        if self.world > 1:
            handles: List[bytes] = [b""] * self.world
            dist.all_gather_object(handles, self._ws.ipc_handle(), group=self.group)
            self._ws.open_peers(handles)
        self.capacity = cap

    def ensure(self, need_rs: int, need_ag: int, need_os: int) -> bool:
        """Grow (collectively) if a call needs more room; returns True if it grew."""
        cap = self.capacity
        if need_rs <= cap.rs_bytes and need_ag <= cap.ag_bytes and need_os <= cap.os_bytes:
            return False
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("SymmetricWorkspace must be sized before CUDA graph capture "
                               "(call reserve() with the largest message first)")
        new = Capacity(_round_cap(max(need_rs, cap.rs_bytes)), _round_cap(max(need_ag, cap.ag_bytes)),
                       _round_cap(max(need_os, cap.os_bytes)))
        # No kernel of any rank may still touch the old buffers.
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        self._ws = None
        self._alloc(new)
        return True

    @property
    def native(self):
        return self._ws

    # -- failure detection --------------------------------------------------------------
    def status(self):
        code, phase, block, peer, want, seen = self._ws.status()
        return dict(code=code, phase=phase, block=block, peer=peer, want=want, seen=seen)

    def check(self, synchronize: bool = True):
        """Raise :class:`CommTimeoutError` if a kernel recorded a failed wait."""
        if synchronize:
            torch.cuda.synchronize(self.device)
        st = self.status()
        if st["code"] != 0:
            raise CommTimeoutError(
                f"rank {self.rank}: fused collective timed out in the "
                f"{_PHASES.get(st['phase'], st['phase'])} phase (block {st['block']}) waiting for "
                f"rank {st['peer']} (wanted epoch {st['want']}, saw {st['seen']}); the communicator "
                "is no longer usable")

    def clear_status(self):
        self._ws.clear_status()


class EmulatedWorkspaces:
    """W workspaces on one GPU that play W ranks inside single kernel launches."""

    def __init__(self, world: int, device: Optional[torch.device] = None, rs_bytes: int = 8 << 20,
                 ag_bytes: int = 8 << 20, os_bytes: int = 4 << 20):
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        self.world = world
        self.rank = 0
        self._alloc(Capacity(_round_cap(rs_bytes), _round_cap(ag_bytes), _round_cap(os_bytes)))

    def _alloc(self, cap: Capacity):
        C = ext()
        self.all = [C.Workspace(self.device.index, r, self.world, cap.rs_bytes, cap.ag_bytes, cap.os_bytes)
                    for r in range(self.world)]
        ptrs = [w.local_ptr for w in self.all]
        for w in self.all:
            w.set_peer_ptrs(ptrs)
        self.capacity = cap

    def ensure(self, need_rs: int, need_ag: int, need_os: int) -> bool:
        cap = self.capacity
        if need_rs <= cap.rs_bytes and need_ag <= cap.ag_bytes and need_os <= cap.os_bytes:
            return False
        torch.cuda.synchronize(self.device)
        self.all = None
        self._alloc(Capacity(_round_cap(max(need_rs, cap.rs_bytes)), _round_cap(max(need_ag, cap.ag_bytes)),
                             _round_cap(max(need_os, cap.os_bytes))))
        return True

    def status(self):
        code, phase, block, peer, want, seen = self.all[0].status()
        return dict(code=code, phase=phase, block=block, peer=peer, want=want, seen=seen)

    def check(self, synchronize: bool = True):
        if synchronize:
            torch.cuda.synchronize(self.device)
        st = self.status()
        if st["code"] != 0:
            raise CommTimeoutError(f"emulated collective timed out: {st}")

    def clear_status(self):
        self.all[0].clear_status()
