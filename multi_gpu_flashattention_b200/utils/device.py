"""Bind this process to its local CUDA device (one process per GPU)."""
from __future__ import annotations

import os
from typing import Optional, Tuple

from .._ext import sched as _sched


def local_rank() -> Tuple[int, str]:
    """(local rank, variable it came from) or (-1, "") when no launcher set one."""
    return tuple(_sched().local_rank_from_env())


def choose_device(device_count: int, fallback_local_rank: int = 0):
    """(device, local_rank, source, error) with the reference's precedence rules."""
    return tuple(_sched().choose_device(device_count, fallback_local_rank))


def select_local_device(fallback_local_rank: Optional[int] = None) -> int:
    """Pick and set this rank's device; raise RuntimeError like the reference aborts."""
    import torch
    if fallback_local_rank is None:
        fallback_local_rank = int(os.environ.get("RANK", "0")) % max(1, torch.cuda.device_count())
    dev, lr, src, err = choose_device(torch.cuda.device_count(), fallback_local_rank)
    if err:
        raise RuntimeError(err)
    torch.cuda.set_device(dev)
    return dev
