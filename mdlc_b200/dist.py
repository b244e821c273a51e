"""Process-group plumbing for one-process-per-GPU runs.

Images are independent, so multi-GPU inference is batch sharding with no
collective on the hot path: every rank compiles the graph for its own shard on
its own GPU (``compile(devices=[local_rank])``). ``torch.distributed`` is used
only around the measured region -- a barrier before and after, and the maximum
of the per-rank device times -- over NCCL on GPU boxes and gloo on CPU (tests).

Launch with ``torchrun`` (``--master-addr 127.0.0.1``); ranks read ``RANK``,
``LOCAL_RANK`` and ``WORLD_SIZE`` from the environment.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass


def shard(total: int, world: int, rank: int) -> tuple:
    """Contiguous slice ``[lo, hi)`` of ``total`` items owned by ``rank`` (the
    same split ``compile(devices=G)`` uses across the GPUs of one process)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if total % world:
        raise ValueError(f"{total} items do not split evenly over {world} ranks")
    per = total // world
    return rank * per, (rank + 1) * per


@dataclass
class Dist:
    rank: int
    world: int
    local_rank: int
    backend: str
    _pg: object = None

    def _tensor(self, value):
        import torch
        dev = torch.device("cuda", torch.cuda.current_device()) if self.backend == "nccl" else torch.device("cpu")
        return torch.tensor([float(value)], dtype=torch.float64, device=dev)

    def barrier(self) -> None:
        if self.world > 1:
            import torch
            import torch.distributed as td
            if self.backend == "nccl":
                torch.cuda.synchronize()
            td.barrier()

    def max(self, value: float) -> float:
        """Maximum of ``value`` over all ranks (every rank gets it)."""
        if self.world == 1:
            return float(value)
        import torch.distributed as td
        t = self._tensor(value)
        td.all_reduce(t, op=td.ReduceOp.MAX)
        return float(t.item())

    def sum(self, value: float) -> float:
        if self.world == 1:
            return float(value)
        import torch.distributed as td
        t = self._tensor(value)
        td.all_reduce(t, op=td.ReduceOp.SUM)
        return float(t.item())

    def gather(self, arr):
        """Concatenate every rank's ``arr`` (same shape and dtype on each) along
        axis 0, in rank order, on every rank: the final output gather of a
        batch-sharded run (one all-gather; through device memory on NCCL)."""
        import numpy as np
        arr = np.ascontiguousarray(arr)
        if self.world == 1:
            return arr.copy()
        import torch
        import torch.distributed as td
        dev = torch.device("cuda", torch.cuda.current_device()) if self.backend == "nccl" else torch.device("cpu")
        t = torch.from_numpy(arr).to(dev)
        parts = [torch.empty_like(t) for _ in range(self.world)]
        td.all_gather(parts, t)
        return torch.cat(parts, 0).cpu().numpy()

    def close(self) -> None:
        if self.world > 1:
            import torch.distributed as td
            if td.is_initialized():
                td.destroy_process_group()


def from_env(backend: str | None = None, timeout_s: int = 120) -> Dist:
    """Join the process group described by the torchrun environment (a world
    of one needs no group). ``backend`` defaults to NCCL when CUDA is
    available, else gloo; a short timeout makes a rank that never arrives end
    the others' collective with an error instead of a hang."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if backend is None:
        import torch
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    d = Dist(rank, world, local, backend)
    if world > 1:
        import torch
        import torch.distributed as td
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        td.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return d
