"""SwiGLU activation entry points with the reference's names and contract.

``triton_swiglu`` keeps the signature and error type of the reference
(src/picotron/nn/triton_kernels/swiglu.py:97-101) and runs the sm_100a forward and
backward kernels through ``torch.ops.picotron_b200.swiglu`` (autograd included).
"""

from __future__ import annotations

import torch
from torch import Tensor
from torch.nn import functional as F

from picotron_b200 import ops
from picotron_b200.errors import TritonSwiGLUUnavailable


def _validate(gate: Tensor, up: Tensor) -> None:
    """Reject inputs the kernel cannot take (reference swiglu.py:84-94)."""

    if not isinstance(gate, Tensor) or not isinstance(up, Tensor):
        raise TritonSwiGLUUnavailable("SwiGLU expects tensors.")
    if not gate.is_cuda or not up.is_cuda:
        raise TritonSwiGLUUnavailable("sm_100a SwiGLU requires CUDA tensors.")
    ops.check_device(gate.device, TritonSwiGLUUnavailable)
    if gate.shape != up.shape:
        raise TritonSwiGLUUnavailable("SwiGLU requires gate and up of the same shape.")


def triton_swiglu(gate: Tensor, up: Tensor) -> Tensor:
    """``silu(gate) * up`` on the sm_100a kernels (fp32 math, one rounding), with autograd."""

    _validate(gate, up)
    return torch.ops.picotron_b200.swiglu(gate, up)


class _EagerSwiGLU(torch.autograd.Function):
    """Eager forward ``F.silu(gate) * up`` and the reference's explicit backward formula
    (swiglu.py:56-81), evaluated in the input dtype."""

    @staticmethod
    def forward(ctx, gate: Tensor, up: Tensor) -> Tensor:
        ctx.save_for_backward(gate, up)
        return F.silu(gate) * up

    @staticmethod
    def backward(ctx, grad_output: Tensor):
        gate, up = ctx.saved_tensors
        sigmoid_gate = torch.sigmoid(gate)
        silu_gate = gate * sigmoid_gate
        silu_derivative = sigmoid_gate * (1 + gate * (1 - sigmoid_gate))
        return grad_output * up * silu_derivative, grad_output * silu_gate


def swiglu_with_pytorch_forward(gate: Tensor, up: Tensor) -> Tensor:
    """Device-agnostic eager SwiGLU with the explicit backward formula.

    Kept for API compatibility with the reference's CPU verification entry point
    (swiglu.py:104-107). It never launches the sm_100a kernels.
    """

    return _EagerSwiGLU.apply(gate, up)


def swiglu_gate_up(hidden_states: Tensor, w_gate: Tensor, w_up: Tensor) -> Tensor:
    """``silu(hidden_states @ w_gate^T) * (hidden_states @ w_up^T)`` as one tensor-core GEMM.

    The gate and up projections of the reference's SwiGLU.forward
    (src/picotron/nn/feedforward.py:27-42) and the activation, fused: a tcgen05 GEMM whose
    epilogue applies the activation to the fp32 accumulators (rounded to the input dtype
    first, as the unfused path stores gate and up). Weights in another dtype are cast to the
    input's (what autocast does for the reference's nn.Linear). Autograd: the activation
    backward runs on the sm_100a kernel and the projections' backward on library GEMMs.
    Raises :class:`TritonSwiGLUUnavailable` when the inputs cannot run on this path.
    """

    if not hidden_states.is_cuda or not w_gate.is_cuda or not w_up.is_cuda:
        raise TritonSwiGLUUnavailable("the fused gate/up GEMM requires CUDA tensors.")
    ops.check_device(hidden_states.device, TritonSwiGLUUnavailable)
    if w_gate.dtype != hidden_states.dtype:
        w_gate = w_gate.to(hidden_states.dtype)
    if w_up.dtype != hidden_states.dtype:
        w_up = w_up.to(hidden_states.dtype)
    act, _, _ = torch.ops.picotron_b200.swiglu_gate_up(hidden_states, w_gate, w_up)
    return act
