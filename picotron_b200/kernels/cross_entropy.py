"""Cross-entropy entry points with the reference's names and contract.

``triton_cross_entropy`` keeps the signature and error type of the reference's
(src/picotron/nn/triton_kernels/cross_entropy.py:50-87: mean cross-entropy of [rows, vocab]
logits) and ``CrossEntropyWithFallback`` its call-site wrapper (:90-112, used by the training
loop at src/picotron/training/train_loop.py:95-97,141-145). Both run the sm_100a kernels
through ``torch.ops.picotron_b200.cross_entropy``. Unlike the reference's forward-only
kernel they have a backward (the training path), accept the training call's strided
``logits[:, :-1, :].transpose(1, 2)`` view without a copy, any vocabulary size, and
``ignore_index`` (-100, as F.cross_entropy).
"""

from __future__ import annotations

import warnings

import torch
from torch import Tensor
from torch.nn import functional as F

from picotron_b200 import ops
from picotron_b200.errors import TritonCrossEntropyUnavailable


def _loss_dtype(logits: Tensor) -> torch.dtype:
    # F.cross_entropy returns the input dtype, or fp32 under CUDA autocast (cross_entropy is
    # on autocast's fp32 list).
    if logits.is_cuda and torch.is_autocast_enabled("cuda"):
        return torch.float32
    return logits.dtype


def cross_entropy(logits: Tensor, targets: Tensor, ignore_index: int = -100) -> Tensor:
    """Mean cross-entropy, ``F.cross_entropy(logits, targets, ignore_index=...)`` semantics
    (class dimension 1: logits [N, V] with targets [N], or [B, V, S] with targets [B, S]),
    fp32 math, with autograd. Raises :class:`TritonCrossEntropyUnavailable` when the inputs
    cannot run on this path."""

    if not isinstance(logits, Tensor) or not isinstance(targets, Tensor):
        raise TritonCrossEntropyUnavailable("cross-entropy expects tensors.")
    if not logits.is_cuda or not targets.is_cuda:
        raise TritonCrossEntropyUnavailable("sm_100a cross-entropy requires CUDA tensors.")
    loss, _, _ = torch.ops.picotron_b200.cross_entropy(logits, targets, int(ignore_index))
    return loss.to(_loss_dtype(logits))


def triton_cross_entropy(logits: Tensor, targets: Tensor) -> Tensor:
    """Mean cross-entropy of ``logits`` [rows, vocab] (reference cross_entropy.py:50-87).

    The reference's version is inference-only and limited to contiguous 2-D logits with a
    vocabulary of at most 65536; this one takes any vocabulary, the 3-D layout of
    F.cross_entropy and gradients. Targets outside [0, vocab) give a NaN loss and set the
    library's device error word (a kernel cannot raise the reference's exception).
    """

    return cross_entropy(logits, targets)


class CrossEntropyWithFallback:
    """The training loop's loss object (reference cross_entropy.py:90-112).

    With ``use_triton`` and CUDA tensors the sm_100a kernels run (failures raise). With
    ``use_triton`` and non-CUDA tensors it warns once with the reference's message and uses
    F.cross_entropy, as the reference does when its kernel cannot run.
    """

    def __init__(self, *, use_triton: bool = False) -> None:
        self.use_triton = use_triton
        self._fallback_warned = False

    def __call__(self, logits: Tensor, targets: Tensor) -> Tensor:
        if self.use_triton:
            if logits.is_cuda:
                ops.check_device(logits.device, TritonCrossEntropyUnavailable)
                return cross_entropy(logits, targets)
            if not self._fallback_warned:
                warnings.warn(
                    "Triton cross-entropy unavailable; using PyTorch fallback: "
                    "sm_100a cross-entropy requires CUDA tensors.",
                    RuntimeWarning,
                    stacklevel=2,
                )
                self._fallback_warned = True
        return F.cross_entropy(logits, targets)
