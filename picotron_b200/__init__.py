"""picotron_b200: sm_100a (B200) kernels for picotron's RMSNorm / SwiGLU / RoPE hot path.

Public surface:

* ``picotron_b200.kernels`` -- drop-in for ``picotron.nn.triton_kernels``
  (``triton_rms_norm``, ``triton_swiglu``, ``triton_apply_rotary_embedding`` and the
  ``Triton*Unavailable`` exceptions);
* ``picotron_b200.modules`` -- ``RMSNorm``, ``SwiGLU``, ``RotaryEmbedding`` with the
  reference's constructors and parameter names;
* ``picotron_b200.ops`` -- the ``torch.ops.picotron_b200.*`` custom ops (with autograd);
* ``picotron_b200.config`` -- ``TritonKernelsConfig`` (the ``model.triton_kernels`` keys);
* ``picotron_b200.hardware`` -- ``detect_triton_support`` and ``probe_hot_path``;
* ``picotron_b200.dist`` -- the packed weight-gradient all-reduce for data parallelism;
* ``picotron_b200._capi`` -- the ctypes binding of the C ABI (include/picotron_b200.h).
"""

from picotron_b200 import ops  # registers torch.ops.picotron_b200.*
from picotron_b200.config import TritonKernelsConfig
from picotron_b200.errors import (
    TritonRMSNormUnavailable,
    TritonRoPEUnavailable,
    TritonSwiGLUUnavailable,
)
from picotron_b200.hardware import TritonReport, detect_triton_support, probe_hot_path
from picotron_b200.kernels import (
    fused_add_rms_norm,
    rms_norm_with_pytorch_forward,
    swiglu_with_pytorch_forward,
    triton_apply_rotary_embedding,
    triton_rms_norm,
    triton_swiglu,
)
from picotron_b200.modules import (
    RMSNorm,
    RotaryEmbedding,
    SwiGLU,
    apply_rotary_embedding,
    rotary_cos_sin,
)

__all__ = [
    "ops",
    "fused_add_rms_norm",
    "RMSNorm",
    "RotaryEmbedding",
    "SwiGLU",
    "TritonKernelsConfig",
    "TritonRMSNormUnavailable",
    "TritonRoPEUnavailable",
    "TritonReport",
    "TritonSwiGLUUnavailable",
    "apply_rotary_embedding",
    "detect_triton_support",
    "probe_hot_path",
    "rms_norm_with_pytorch_forward",
    "rotary_cos_sin",
    "swiglu_with_pytorch_forward",
    "triton_apply_rotary_embedding",
    "triton_rms_norm",
    "triton_swiglu",
]
