"""torch.distributed lifecycle for one process per GPU (single node, torchrun env://)."""
from __future__ import annotations

import os
import random
from datetime import timedelta
from typing import Optional, Tuple

import numpy as np
import torch
import torch.distributed as dist

__all__ = ["setup_ddp", "cleanup_ddp", "set_seed", "init_distributed", "get_rank", "get_world_size", "barrier",
           "is_distributed"]


def is_distributed() -> bool:
    return dist.is_available() and dist.is_initialized()


def get_rank(group=None) -> int:
    return dist.get_rank(group) if is_distributed() else 0


def get_world_size(group=None) -> int:
    return dist.get_world_size(group) if is_distributed() else 1


def barrier(group=None):
    if is_distributed():
        dist.barrier(group=group)


def init_distributed(backend: Optional[str] = None, timeout_s: float = 600.0) -> Tuple[int, int, torch.device]:
    """Initialise the default process group from torchrun's environment, if present.

    Returns ``(rank, world_size, device)``.  Without RANK / WORLD_SIZE in the environment
    it is a no-op for a single process.  The device is ``cuda:LOCAL_RANK`` when CUDA is
    available (one process per GPU), else CPU with the gloo backend.
    """
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if torch.cuda.is_available():
        device = torch.device("cuda", local % torch.cuda.device_count())
        torch.cuda.set_device(device)
    else:
        device = torch.device("cpu")
    if world > 1 and not is_distributed():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        backend = backend or ("nccl" if device.type == "cuda" else "gloo")
        kw = dict(backend=backend, rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))
        if backend == "nccl":
            kw["device_id"] = device
        dist.init_process_group(**kw)
    return rank, world, device


def setup_ddp(backend: Optional[str] = None, timeout_s: float = 1800.0):
    """Reference-compatible name: initialise the process group; returns (rank, world, device)."""
    return init_distributed(backend, timeout_s)


def cleanup_ddp():
    """Reference-compatible name: drop communicators, then destroy the process group."""
    try:
        from ..communication import reset_communicators
        reset_communicators()
    except Exception:
        pass
    if is_distributed():
        dist.destroy_process_group()


def set_seed(seed: int = 42):
    random.seed(seed)
    np.random.seed(seed % (2 ** 32))
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)
