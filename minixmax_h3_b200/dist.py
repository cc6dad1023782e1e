"""Process-group state for sequence parallelism (one process per GPU).

Mirrors the contract of the reference's runtime/dist.py:18-38 (``DistState``,
``state()``, ``is_distributed()``) that its Ulysses helpers read; the
transport is torch.distributed over NCCL (gloo for CPU tests) instead of HCCL.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta
from typing import Optional

import torch
import torch.distributed as tdist


@dataclass
class DistState:
    rank: int = 0
    local_rank: int = 0
    world_size: int = 1
    group: Optional[object] = None
    backend: str = "none"


_STATE = DistState()


def state() -> DistState:
    return _STATE


def is_distributed() -> bool:
    return _STATE.world_size > 1


def set_state(rank: int, world_size: int, *, local_rank: Optional[int] = None, group=None,
              backend: str = "external") -> DistState:
    """Adopts a process group created elsewhere (e.g. by a launcher or a test)."""
    global _STATE
    _STATE = DistState(rank=rank, local_rank=rank if local_rank is None else local_rank, world_size=world_size,
                       group=group, backend=backend)
    return _STATE


def init(backend: Optional[str] = None, timeout_s: float = 120.0) -> DistState:
    """Initialises torch.distributed from RANK/WORLD_SIZE/LOCAL_RANK/MASTER_*.

    NCCL ranks bind cuda:LOCAL_RANK.  A short timeout makes ranks that wait on
    a dead peer fail with an error instead of hanging.
    """
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if world > 1 and not tdist.is_initialized():
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        tdist.init_process_group(backend=backend, timeout=timedelta(seconds=timeout_s), **kw)
    elif backend == "nccl" and torch.cuda.is_available():
        torch.cuda.set_device(local)
    return set_state(rank, world, local_rank=local, group=tdist.group.WORLD if world > 1 else None,
                     backend=backend if world > 1 else "none")


def destroy() -> None:
    global _STATE
    from .ulysses import release_peer_buffers  # P2P mappings go before the group

    release_peer_buffers()
    if tdist.is_initialized():
        tdist.destroy_process_group()
    _STATE = DistState()
