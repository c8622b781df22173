"""Fused AdamW step with the reference's names and contract.

The reference reserves ``triton_adamw_step(optimizer)`` and ``AdamWStepWithFallback``
(src/picotron/nn/triton_kernels/adamw.py:14-45) and always falls back to
``optimizer.step()`` of the torch.optim.AdamW its training loop builds (train_loop.py:302-325),
because "a fused AdamW update can silently alter optimizer math". This implementation does not
alter it: one sm_100a kernel performs the same fp32 operations with the same roundings as
torch.optim.AdamW's CUDA multi-tensor path (checked bit for bit on the GPU), reading and
writing each of param, grad, exp_avg, exp_avg_sq once instead of eight elementwise passes.
Optimizer state keeps torch's format (``step`` as a float32 CPU tensor, ``exp_avg`` and
``exp_avg_sq`` like the parameter), so fused and PyTorch steps can be mixed and checkpoints
are unchanged.
"""

from __future__ import annotations

import warnings
from collections import defaultdict

import torch
from torch.optim import Optimizer

from picotron_b200 import _capi, ops
from picotron_b200.errors import TritonAdamWUnavailable


def _plan(optimizer: Optimizer):
    """Validate the optimizer and list (param, grad, state, lr, wd) per device; raises
    TritonAdamWUnavailable for anything the fused step does not cover."""

    if not isinstance(optimizer, torch.optim.AdamW):
        raise TritonAdamWUnavailable(
            f"the fused step covers torch.optim.AdamW, not {type(optimizer).__name__}")
    per_device = defaultdict(list)
    settings = None
    for group in optimizer.param_groups:
        if group.get("amsgrad") or group.get("capturable") or group.get("differentiable"):
            raise TritonAdamWUnavailable("amsgrad, capturable and differentiable are not fused")
        if group.get("fused"):
            raise TritonAdamWUnavailable("the optimizer already uses PyTorch's fused kernel")
        lr, (b1, b2), eps = group["lr"], group["betas"], group["eps"]
        if any(isinstance(v, torch.Tensor) for v in (lr, b1, b2, eps)):
            raise TritonAdamWUnavailable("tensor-valued lr / betas / eps are not fused")
        key = (float(b1), float(b2), float(eps), bool(group.get("maximize", False)))
        if settings is not None and key != settings:
            raise TritonAdamWUnavailable("parameter groups with different betas/eps/maximize")
        settings = key
        for p in group["params"]:
            if p.grad is None:
                continue
            g = p.grad
            if g.is_sparse or not p.is_cuda or p.dtype != torch.float32 or g.dtype != torch.float32:
                raise TritonAdamWUnavailable("the fused step takes dense fp32 CUDA parameters")
            if not (p.is_contiguous() and g.is_contiguous()) or g.device != p.device:
                raise TritonAdamWUnavailable("parameters and gradients must be contiguous")
            per_device[p.device].append((p, g, group))
    return per_device, settings


def triton_adamw_step(optimizer: Optimizer) -> None:
    """One AdamW step of ``optimizer`` on the fused sm_100a kernel.

    Raises :class:`TritonAdamWUnavailable` (before changing anything) when the optimizer or
    its parameters are outside what the kernel covers: a torch.optim.AdamW without amsgrad,
    capturable or differentiable, fp32 dense contiguous CUDA parameters and gradients.
    """

    per_device, settings = _plan(optimizer)
    if settings is None:
        return
    beta1, beta2, eps, maximize = settings
    for device, items in per_device.items():
        ops.check_device(device, TritonAdamWUnavailable)
        for p, _, _ in items:
            state = optimizer.state[p]
            if len(state) == 0:  # lazy state, as torch.optim.AdamW creates it
                state["step"] = torch.tensor(0.0, dtype=torch.float32)
                state["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            for name in ("exp_avg", "exp_avg_sq"):
                if not state[name].is_contiguous() or state[name].shape != p.shape:
                    raise TritonAdamWUnavailable("optimizer state must match the parameter")
        # The reference increments its step tensors first; here they are advanced once the
        # kernel has been queued, so a refused call leaves the optimizer untouched.
        steps = [int(optimizer.state[p]["step"].item()) + 1 for p, _, _ in items]
        with ops._OnDevice(device):
            _capi.adamw_step(
                [p.data_ptr() for p, _, _ in items], [g.data_ptr() for _, g, _ in items],
                [optimizer.state[p]["exp_avg"].data_ptr() for p, _, _ in items],
                [optimizer.state[p]["exp_avg_sq"].data_ptr() for p, _, _ in items],
                [p.numel() for p, _, _ in items], steps,
                [float(grp["lr"]) for _, _, grp in items],
                [float(grp["weight_decay"]) for _, _, grp in items],
                beta1, beta2, eps, maximize, torch.cuda.current_stream(device).cuda_stream,
                TritonAdamWUnavailable,
            )
        for p, _, _ in items:
            optimizer.state[p]["step"].add_(1)


class AdamWStepWithFallback:
    """The training loop's optimizer-step object (reference adamw.py:27-45).

    With ``use_triton`` the fused step runs; an optimizer it does not cover (see
    :func:`triton_adamw_step`) warns once with the reference's message and takes
    ``optimizer.step()``, as the reference does. A missing library raises.
    """

    def __init__(self, *, use_triton: bool = False) -> None:
        self.use_triton = use_triton
        self._fallback_warned = False

    def step(self, optimizer: Optimizer) -> None:
        if self.use_triton:
            try:
                triton_adamw_step(optimizer)
                return
            except TritonAdamWUnavailable as error:
                if not self._fallback_warned:
                    warnings.warn(
                        f"Triton AdamW unavailable; using PyTorch fallback: {error}",
                        RuntimeWarning,
                        stacklevel=2,
                    )
                    self._fallback_warned = True
        optimizer.step()
