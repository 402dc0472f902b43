"""Process-group plumbing: one process per GPU, NCCL over NVLink/NVSwitch.

Ranks find each other through the torchrun environment (MASTER_ADDR/PORT, RANK,
WORLD_SIZE).  The group gets a short timeout so that ranks waiting on a dead peer fail
with an error instead of hanging (reference: DistComm status-tagged responses that
unblock every rank on error, internal/model/dist_collective.go:59-62).
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist

_GROUP = None


def init(world: int, rank: int, local_rank: int, timeout_s: float | None = None, backend: str | None = None):
    global _GROUP
    if dist.is_initialized():
        _GROUP = dist.group.WORLD
        return _GROUP
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29511")
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    timeout = datetime.timedelta(seconds=timeout_s or float(os.environ.get("FAK_PG_TIMEOUT_S", "120")))
    kw = {}
    if backend == "nccl":
        kw["device_id"] = torch.device("cuda", local_rank)
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=timeout, **kw)
    _GROUP = dist.group.WORLD
    return _GROUP


def group():
    return _GROUP


def shutdown() -> None:
    global _GROUP
    if dist.is_initialized():
        try:
            dist.barrier()
        except Exception:
            pass
        dist.destroy_process_group()
    _GROUP = None
