"""Drop-in replacement of ``picotron.nn.triton_kernels`` for the hot path.

Same public names as the reference package (src/picotron/nn/triton_kernels/__init__.py)
for RMSNorm, SwiGLU and RoPE, backed by the sm_100a CUDA library instead of Triton, plus
``fused_add_rms_norm`` (the decoder block's residual add fused into the following norm) and
``swiglu_gate_up`` (the MLP's gate/up projections with the activation as one tcgen05 GEMM),
the loss: ``triton_cross_entropy`` / ``CrossEntropyWithFallback`` (forward and backward), and
the optimizer step: ``triton_adamw_step`` / ``AdamWStepWithFallback``.
"""

from picotron_b200.errors import (
    TritonAdamWUnavailable,
    TritonCrossEntropyUnavailable,
    TritonRMSNormUnavailable,
    TritonRoPEUnavailable,
    TritonSwiGLUUnavailable,
)
from picotron_b200.kernels.adamw import AdamWStepWithFallback, triton_adamw_step
from picotron_b200.kernels.cross_entropy import (
    CrossEntropyWithFallback,
    cross_entropy,
    triton_cross_entropy,
)
from picotron_b200.kernels.rmsnorm import (
    fused_add_rms_norm,
    rms_norm_with_pytorch_forward,
    triton_rms_norm,
)
from picotron_b200.kernels.rope import triton_apply_rotary_embedding
from picotron_b200.kernels.swiglu import (
    swiglu_gate_up,
    swiglu_with_pytorch_forward,
    triton_swiglu,
)

__all__ = [
    "AdamWStepWithFallback",
    "TritonAdamWUnavailable",
    "triton_adamw_step",
    "CrossEntropyWithFallback",
    "TritonCrossEntropyUnavailable",
    "cross_entropy",
    "triton_cross_entropy",
    "TritonRMSNormUnavailable",
    "fused_add_rms_norm",
    "swiglu_gate_up",
    "TritonRoPEUnavailable",
    "TritonSwiGLUUnavailable",
    "triton_apply_rotary_embedding",
    "triton_rms_norm",
    "triton_swiglu",
    "swiglu_with_pytorch_forward",
    "rms_norm_with_pytorch_forward",
]
