"""Data-parallel plumbing for the RMSNorm weight gradients.

Token rows shard across ranks with no communication for RMSNorm, SwiGLU or RoPE. The
only exchange is the RMSNorm weight gradient: each rank reduces its per-CTA partials to
one fp32 vector per norm layer directly into a slot of one packed buffer
(``DWeightBucket``), and one all-reduce of that buffer per step averages the gradients
over ranks, which is what the reference's DistributedDataParallel does for these
parameters (src/picotron/parallel/ddp.py:72-91). With NCCL the all-reduce uses
``ReduceOp.AVG``; backends without AVG (gloo) sum and divide by the world size.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor


class DWeightBucket:
    """One contiguous fp32 buffer holding the weight gradient of several norm layers."""

    def __init__(self, sizes: list[int], device: torch.device | str) -> None:
        if not sizes or any(int(s) <= 0 for s in sizes):
            raise ValueError("DWeightBucket needs positive slot sizes")
        self.sizes = [int(s) for s in sizes]
        self.offsets = [0]
        for s in self.sizes:
            # Keep every slot 16-byte aligned (4 floats) so kernels can use vector stores.
            self.offsets.append(self.offsets[-1] + (s + 3) // 4 * 4)
        self.buffer = torch.zeros(self.offsets[-1], dtype=torch.float32, device=device)

    def __len__(self) -> int:
        return len(self.sizes)

    def slot(self, index: int) -> Tensor:
        start = self.offsets[index]
        return self.buffer[start : start + self.sizes[index]]

    def zero_(self) -> None:
        self.buffer.zero_()

    def all_reduce(self, group: dist.ProcessGroup | None = None, average: bool = True) -> None:
        """Sum (or average) the buffer over the ranks of ``group`` in place."""

        if not dist.is_available() or not dist.is_initialized():
            return
        world = dist.get_world_size(group)
        if world == 1:
            return
        if average and dist.get_backend(group) == "nccl":
            dist.all_reduce(self.buffer, op=dist.ReduceOp.AVG, group=group)
            return
        dist.all_reduce(self.buffer, op=dist.ReduceOp.SUM, group=group)
        if average:
            self.buffer.div_(world)
