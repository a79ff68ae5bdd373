"""Process-group lifecycle, seeding, clocks sampling and logging helpers.

``setup_ddp``, ``cleanup_ddp`` and ``set_seed`` are the helpers the reference imports from
a ``utils`` module it does not ship (main.py:17, 185).
"""
from .dist import (setup_ddp, cleanup_ddp, set_seed, init_distributed, get_rank, get_world_size,  # noqa: F401
                   barrier, is_distributed)
