"""Data-parallel plumbing for the RMSNorm weight gradients.

Token rows shard across ranks with no communication for RMSNorm, SwiGLU or RoPE. The
only exchange is the RMSNorm weight gradient: each rank reduces its per-CTA partials to
one fp32 vector per norm layer directly into a slot of one packed buffer
(``DWeightBucket``), and all-reduces of that buffer average the gradients over ranks,
which is what the reference's DistributedDataParallel does for these parameters
(src/picotron/parallel/ddp.py:72-91, gradient buckets reduced as they fill). Either the
whole buffer at once (``all_reduce``) or a range of slots as soon as the backward has
produced them (``all_reduce_async``: the collective runs on the process group's own
stream while the backward of earlier layers continues). With NCCL the all-reduce uses
``ReduceOp.AVG``; backends without AVG (gloo) sum and divide by the world size.
"""

from __future__ import annotations

import datetime

import torch
import torch.distributed as dist
from torch import Tensor


def nccl_options():
    """Options for a NCCL process group whose collectives overlap the hot-path kernels: its
    stream has high priority. Every kernel of the backward fills the GPU (persistent grids
    sized to the SMs), so on a normal-priority stream NCCL's all-reduce kernels wait for free
    SMs behind the compute stream's queued kernels and run only after the backward's last
    kernel; with high priority their CTAs are dispatched first as SMs free up.
    Pass as ``dist.init_process_group("nccl", pg_options=nccl_options(), ...)``. For these
    small (32-256 KB), latency-bound all-reduces also set ``NCCL_NVLS_ENABLE=0`` before NCCL
    loads: on B200 with NVLink SHARP enabled about one two-GPU run in three left 1.6-2.4 ms
    of all-reduce exposed at the end of every step, without it none of four did."""

    return dist.ProcessGroupNCCL.Options(is_high_priority_stream=True)


class PendingAllReduce:
    """An all-reduce issued by ``DWeightBucket.all_reduce_async``; ``wait`` completes it.

    With NCCL, ``wait`` only makes the current CUDA stream wait for the collective (the
    host does not block); with gloo it blocks and then applies the average."""

    def __init__(self, work, view: Tensor | None, divide_by: int) -> None:
        self._work, self._view, self._divide_by = work, view, divide_by

    def wait(self, timeout: datetime.timedelta | None = None) -> None:
        """Completes the all-reduce. A peer that never issues the matching all-reduce makes
        this raise (RuntimeError / DistBackendError) once ``timeout``, or else the process
        group's timeout, has passed, instead of waiting for ever."""

        if self._work is not None:
            if timeout is None:
                self._work.wait()
            else:
                self._work.wait(timeout)
            self._work = None
        if self._view is not None and self._divide_by > 1:
            self._view.div_(self._divide_by)
        self._view = None


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

    def all_reduce_async(self, first: int, stop: int, group: dist.ProcessGroup | None = None,
                         average: bool = True) -> PendingAllReduce:
        """Start the sum (or average) of slots ``[first, stop)`` over the ranks of ``group``.

        Every rank must issue the same ranges in the same order. Returns a handle whose
        ``wait`` must be called before the slots are read."""

        if not 0 <= first < stop <= len(self.sizes):
            raise ValueError(f"slot range [{first}, {stop}) is outside [0, {len(self.sizes)})")
        if not dist.is_available() or not dist.is_initialized():
            return PendingAllReduce(None, None, 1)
        world = dist.get_world_size(group)
        if world == 1:
            return PendingAllReduce(None, None, 1)
        view = self.buffer[self.offsets[first] : self.offsets[stop]]
        if average and dist.get_backend(group) == "nccl":
            work = dist.all_reduce(view, op=dist.ReduceOp.AVG, group=group, async_op=True)
            return PendingAllReduce(work, None, 1)
        work = dist.all_reduce(view, op=dist.ReduceOp.SUM, group=group, async_op=True)
        return PendingAllReduce(work, view, world if average else 1)
