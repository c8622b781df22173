"""RMSNorm entry points with the reference's names and contract.

``triton_rms_norm`` keeps the signature and error type of the reference
(src/picotron/nn/triton_kernels/rmsnorm.py:152-160) and runs the sm_100a forward and
backward kernels through ``torch.ops.picotron_b200.rms_norm`` (autograd included). Unlike
the reference it accepts non-contiguous inputs and any hidden size, and its backward is a
fused kernel instead of eager PyTorch.
"""

from __future__ import annotations

import torch
from torch import Tensor

from picotron_b200 import ops
from picotron_b200.errors import TritonRMSNormUnavailable


def _validate(hidden_states: Tensor, weight: Tensor) -> None:
    """Reject inputs the kernel cannot take (reference rmsnorm.py:137-149)."""

    if not isinstance(hidden_states, Tensor) or not isinstance(weight, Tensor):
        raise TritonRMSNormUnavailable("RMSNorm expects tensors.")
    if not hidden_states.is_cuda or not weight.is_cuda:
        raise TritonRMSNormUnavailable("sm_100a RMSNorm requires CUDA tensors.")
    ops.check_device(hidden_states.device, TritonRMSNormUnavailable)
    if hidden_states.ndim < 1 or hidden_states.size(-1) != weight.numel():
        raise TritonRMSNormUnavailable("RMSNorm hidden size must match the weight size.")


def triton_rms_norm(hidden_states: Tensor, weight: Tensor, eps: float) -> Tensor:
    """``y = x * rsqrt(mean(x^2) + eps) * weight`` on the sm_100a kernels, with autograd.

    Output dtype = input dtype (the reference's fused-forward semantics, rmsnorm.py:72).
    Raises :class:`TritonRMSNormUnavailable` when the inputs cannot run on this path.
    """

    _validate(hidden_states, weight)
    return torch.ops.picotron_b200.rms_norm(hidden_states, weight, float(eps))


class _EagerRMSNorm(torch.autograd.Function):
    """Eager PyTorch forward and the reference's explicit backward formula.

    Same arithmetic as the reference's ``_RMSNormAutogradFunction`` with its PyTorch
    forward (rmsnorm.py:49-60, 109-134): fp32 math, outputs cast back to the input and
    weight dtypes.
    """

    @staticmethod
    def forward(ctx, hidden_states: Tensor, weight: Tensor, eps: float) -> Tensor:
        values = hidden_states.float()
        inverse_rms = torch.rsqrt(values.square().mean(dim=-1, keepdim=True) + eps)
        ctx.save_for_backward(hidden_states, weight, inverse_rms)
        return (values * inverse_rms * weight.float()).to(dtype=hidden_states.dtype)

    @staticmethod
    def backward(ctx, grad_output: Tensor):
        hidden_states, weight, inverse_rms = ctx.saved_tensors
        x = hidden_states.float()
        g = grad_output.float() * weight.float()
        dot_mean = (g * x).mean(dim=-1, keepdim=True)
        grad_x = inverse_rms * (g - x * inverse_rms.square() * dot_mean)
        grad_w = (grad_output.float() * x * inverse_rms).reshape(-1, weight.numel()).sum(dim=0)
        return grad_x.to(hidden_states.dtype), grad_w.to(weight.dtype), None


def rms_norm_with_pytorch_forward(hidden_states: Tensor, weight: Tensor, eps: float) -> Tensor:
    """Device-agnostic eager RMSNorm with the explicit backward formula.

    Kept for API compatibility with the reference's CPU verification entry point
    (rmsnorm.py:163-171). It never launches the sm_100a kernels.
    """

    return _EagerRMSNorm.apply(hidden_states, weight, eps)


def fused_add_rms_norm(residual: Tensor, branch: Tensor, weight: Tensor,
                       eps: float) -> tuple[Tensor, Tensor]:
    """``h = residual + branch`` and ``y = RMSNorm(h) * weight`` in one sm_100a kernel.

    Replaces the residual add followed by the next norm in the reference decoder block
    (src/picotron/models/picotron_decoder.py:116-123): returns ``(h, y)`` with the values
    ``h = residual + branch; y = RMSNorm(h)`` would give (h rounded to the input dtype, as
    PyTorch stores it), with autograd. residual and branch must share shape and dtype.
    Raises :class:`TritonRMSNormUnavailable` when the inputs cannot run on this path.
    """

    _validate(residual, weight)
    if not isinstance(branch, Tensor) or not branch.is_cuda:
        raise TritonRMSNormUnavailable("sm_100a fused add + RMSNorm requires CUDA tensors.")
    return torch.ops.picotron_b200.add_rms_norm(residual, branch, weight, float(eps))
