"""Exception types of the drop-in kernel layer.

The names and the RuntimeError base match the reference's
``picotron.nn.triton_kernels`` exceptions (rmsnorm.py:19, swiglu.py:20,
triton_kernels/rope.py:19), so callers that catch them keep working. Here they are
raised when the sm_100a library cannot run a call: missing library, non-CUDA tensors,
wrong device, unsupported shape or dtype, or a non-zero status from the C ABI.
"""

from __future__ import annotations


class TritonRMSNormUnavailable(RuntimeError):
    """The sm_100a RMSNorm path cannot run these inputs."""


class TritonSwiGLUUnavailable(RuntimeError):
    """The sm_100a SwiGLU path cannot run these inputs."""


class TritonRoPEUnavailable(RuntimeError):
    """The sm_100a RoPE path cannot run these inputs."""


class TritonCrossEntropyUnavailable(RuntimeError):
    """The sm_100a cross-entropy path cannot run these inputs (reference
    triton_kernels/cross_entropy.py:22)."""


class TritonAdamWUnavailable(RuntimeError):
    """The fused AdamW step cannot run this optimizer (reference triton_kernels/adamw.py:10)."""
