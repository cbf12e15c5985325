"""Multi-GPU window scheduler: independent audio windows sharded over devices.

The reference processes 45 s / 30 s windows one after another on one GPU
(``parakeet_cuda/__main__.py:101-116``, ``recording.py:23-47``); the windows are
independent until their words are merged on the host. Here one process per
GPU (``torchrun``) takes a contiguous block of windows, the Q8_0 weights are
replicated on every device, and nothing crosses devices on the data path:
results come back to host memory per process and are gathered on rank 0 over
a CPU (gloo) group. Timing across ranks is the maximum over ranks.
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def shard(n_items: int, world: int, rank: int) -> range:
    """Contiguous, balanced block of ``range(n_items)`` for ``rank`` (first ranks take the remainder)."""
    if world < 1 or not 0 <= rank < world or n_items < 0:
        raise ValueError(f'bad shard request n={n_items} world={world} rank={rank}')
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


class WindowScheduler:
    """Rank/world bookkeeping, window assignment and host-side result gathering."""

    def __init__(self, backend: str | None = None, timeout_s: float = 120.0):
        self.owns_group = False
        if 'WORLD_SIZE' in os.environ and int(os.environ['WORLD_SIZE']) > 1 and not dist.is_initialized():
            backend = backend or ('nccl' if torch.cuda.is_available() else 'gloo')
            if backend == 'nccl':
                torch.cuda.set_device(int(os.environ.get('LOCAL_RANK', 0)))
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
            self.owns_group = True
        self.distributed = dist.is_initialized()
        self.rank = dist.get_rank() if self.distributed else 0
        self.world = dist.get_world_size() if self.distributed else 1
        self.local_rank = int(os.environ.get('LOCAL_RANK', self.rank))
        self.cpu_group = None
        if self.distributed:
            self.cpu_group = (dist.group.WORLD if dist.get_backend() == 'gloo'
                              else dist.new_group(backend='gloo', timeout=datetime.timedelta(seconds=timeout_s)))

    def assign(self, windows):
        """This rank's share of ``windows`` (a sequence), in order."""
        r = shard(len(windows), self.world, self.rank)
        return [windows[i] for i in r]

    def gather(self, local_results):
        """Concatenate every rank's result list on rank 0 in window order (None elsewhere)."""
        if not self.distributed:
            return list(local_results)
        out = [None] * self.world if self.rank == 0 else None
        dist.gather_object(list(local_results), out, dst=0, group=self.cpu_group)
        if self.rank != 0:
            return None
        return [item for part in out for item in part]

    def max_over_ranks(self, value: float) -> float:
        if not self.distributed:
            return float(value)
        t = torch.tensor([float(value)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.cpu_group)
        return float(t.item())

    def barrier(self):
        if self.distributed:
            dist.barrier(group=self.cpu_group)

    def close(self):
        if self.owns_group and dist.is_initialized():
            dist.destroy_process_group()
