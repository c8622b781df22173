"""RoPE entry point with the reference's name and contract.

``triton_apply_rotary_embedding`` keeps the signature and error type of the reference
(src/picotron/nn/triton_kernels/rope.py:52-91) but, unlike the reference's
inference-only kernel, supports autograd (the backward is the inverse rotation on the
same kernel) and reads strided [B, H, S, D] views in place without ``.contiguous()``.
"""

from __future__ import annotations

import torch
from torch import Tensor

from picotron_b200 import ops
from picotron_b200.errors import TritonRoPEUnavailable


def _validate(states: Tensor, cosine: Tensor, sine: Tensor) -> None:
    """Reject inputs the kernel cannot take (reference triton_kernels/rope.py:56-74)."""

    for t in (states, cosine, sine):
        if not isinstance(t, Tensor):
            raise TritonRoPEUnavailable("RoPE expects tensors.")
    if not states.is_cuda or not cosine.is_cuda or not sine.is_cuda:
        raise TritonRoPEUnavailable("sm_100a RoPE requires CUDA tensors.")
    ops.check_device(states.device, TritonRoPEUnavailable)
    if (
        states.ndim != 4
        or states.size(-1) != cosine.size(-1) * 2
        or cosine.shape != sine.shape
        or cosine.size(0) != states.size(-2)
    ):
        raise TritonRoPEUnavailable("sm_100a RoPE requires compatible [B,H,S,D] / [S,D/2] tensors.")


def triton_apply_rotary_embedding(
    states: Tensor, cosine: Tensor, sine: Tensor, *, layout: str = "interleaved"
) -> Tensor:
    """Rotate ``(batch, heads, sequence, head_dim)`` states by the RoPE tables.

    ``layout="interleaved"`` (default) rotates pairs (x[2i], x[2i+1]) exactly like the
    reference; ``layout="rotate_half"`` rotates (x[i], x[i + D/2]).
    """

    _validate(states, cosine, sine)
    if layout not in ops.LAYOUTS:
        raise TritonRoPEUnavailable(f"unknown RoPE layout {layout!r}")
    return torch.ops.picotron_b200.rope(states, cosine, sine, ops.LAYOUTS[layout])

