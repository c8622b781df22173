"""Drop-in ``RMSNorm``, ``SwiGLU`` and ``RotaryEmbedding`` modules.

Constructors, parameter names (and therefore checkpoint keys) and the
``_triton_fallback_warned`` attribute match the reference:

* ``RMSNorm(hidden_size, eps=1e-6, *, use_triton_rmsnorm=False)``
  (src/picotron/models/picotron_decoder.py:20-46), parameter ``weight [H]``;
* ``SwiGLU(hidden_size, intermediate_size, *, use_triton_swiglu=False)``
  (src/picotron/nn/feedforward.py:13-43), parameters
  ``{gate,up,down}_projection.weight``;
* ``RotaryEmbedding(head_dim, theta=1e4, *, use_triton_rope=False)``
  (src/picotron/nn/rope.py:54-107), no parameters.

With the ``use_triton_*`` switch on and CUDA inputs, the sm_100a kernels run and any
failure raises (there is no silent fallback on a GPU). With the switch on and non-CUDA
inputs, the modules keep the reference's documented behaviour: warn once with the
reference's message ("Triton X unavailable; using PyTorch fallback: ...") and evaluate
the module's eager PyTorch formula, the same formula they use with the switch off.
"""

from __future__ import annotations

import warnings

import torch
from torch import Tensor, nn
from torch.nn import functional as F

from picotron_b200 import ops


def _warn_once(module: nn.Module, what: str, error: Exception) -> None:
    if not module._triton_fallback_warned:
        warnings.warn(
            f"Triton {what} unavailable; using PyTorch fallback: {error}",
            RuntimeWarning,
            stacklevel=3,
        )
        module._triton_fallback_warned = True


class RMSNorm(nn.Module):
    """Root mean square normalization with a learned scale."""

    def __init__(
        self, hidden_size: int, eps: float = 1e-6, *, use_triton_rmsnorm: bool = False
    ) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.eps = eps
        self.use_triton_rmsnorm = use_triton_rmsnorm
        self._triton_fallback_warned = False

    def forward(self, hidden_states: Tensor) -> Tensor:
        if self.use_triton_rmsnorm:
            if hidden_states.is_cuda:
                return torch.ops.picotron_b200.rms_norm(hidden_states, self.weight, float(self.eps))
            _warn_once(self, "RMSNorm", RuntimeError("sm_100a RMSNorm requires CUDA tensors."))
        # Eager formula of the reference module (picotron_decoder.py:44-46).
        variance = hidden_states.pow(2).mean(dim=-1, keepdim=True)
        normalized = hidden_states * torch.rsqrt(variance + self.eps)
        return normalized * self.weight

    def forward_with_residual(self, residual: Tensor, branch: Tensor) -> tuple[Tensor, Tensor]:
        """``h = residual + branch`` and ``self(h)``, returned as ``(h, self(h))``.

        The decoder block's residual add followed by this norm
        (picotron_decoder.py:116-123) as one fused kernel when the kernel path is enabled,
        the inputs are CUDA tensors and residual and branch share dtype; otherwise the two
        eager steps.
        """

        if (self.use_triton_rmsnorm and residual.is_cuda and branch.is_cuda
                and residual.dtype == branch.dtype and residual.shape == branch.shape):
            return torch.ops.picotron_b200.add_rms_norm(residual, branch, self.weight,
                                                        float(self.eps))
        hidden_states = residual + branch
        return hidden_states, self(hidden_states)


class SwiGLU(nn.Module):
    """Llama-style gated feed-forward network."""

    def __init__(
        self, hidden_size: int, intermediate_size: int, *, use_triton_swiglu: bool = False
    ) -> None:
        super().__init__()
        self.gate_projection = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.up_projection = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.down_projection = nn.Linear(intermediate_size, hidden_size, bias=False)
        self.use_triton_swiglu = use_triton_swiglu
        # Not in the reference (so not a constructor argument; set it on the module): run
        # gate_projection, up_projection and the activation as one tcgen05 GEMM with a
        # SwiGLU epilogue (bf16/fp16 CUDA inputs; otherwise the three-step path below).
        # Same parameters, so checkpoints are unaffected.
        self.fuse_gate_up = False
        self._triton_fallback_warned = False

    def activation(self, gate: Tensor, up: Tensor) -> Tensor:
        """``silu(gate) * up`` on the kernel path when enabled and on CUDA."""

        if self.use_triton_swiglu:
            if gate.is_cuda:
                return torch.ops.picotron_b200.swiglu(gate, up)
            _warn_once(self, "SwiGLU", RuntimeError("sm_100a SwiGLU requires CUDA tensors."))
        return F.silu(gate) * up

    def forward(self, hidden_states: Tensor) -> Tensor:
        if (self.fuse_gate_up and hidden_states.is_cuda
                and self._compute_dtype(hidden_states) in (torch.bfloat16, torch.float16)):
            dtype = self._compute_dtype(hidden_states)
            x = hidden_states.to(dtype)
            w_gate = self.gate_projection.weight.to(dtype)
            w_up = self.up_projection.weight.to(dtype)
            down = self.down_projection
            if down.bias is None and ops.fused_down_backward_supported(x, down.weight):
                # Both activation passes inside tensor-core GEMMs: the forward's epilogue and
                # the backward's (the down projection's input gradient never reaches HBM).
                return ops.swiglu_mlp(x, w_gate, w_up, down.weight.to(dtype))
            activated = torch.ops.picotron_b200.swiglu_gate_up(x, w_gate, w_up)[0]
            return down(activated)
        gate = self.gate_projection(hidden_states)
        up = self.up_projection(hidden_states)
        return self.down_projection(self.activation(gate, up))

    @staticmethod
    def _compute_dtype(hidden_states: Tensor) -> torch.dtype:
        """The dtype nn.Linear would compute in: the autocast dtype when autocast is on."""

        if torch.is_autocast_enabled("cuda"):
            return torch.get_autocast_dtype("cuda")
        return hidden_states.dtype


def rotary_cos_sin(
    sequence_length: int,
    head_dim: int,
    theta: float,
    *,
    device: torch.device,
    dtype: torch.dtype,
) -> tuple[Tensor, Tensor]:
    """RoPE cosine/sine tables ``[S, D/2]`` (reference nn/rope.py:13-32).

    ``inv_freq = 1 / theta^(arange(0, D, 2) / D)`` in fp32, angles = outer(positions,
    inv_freq), cos/sin computed in fp32 and cast to ``dtype``.
    """

    if head_dim % 2 != 0:
        raise ValueError("RoPE requires an even attention head dimension.")
    if theta <= 0:
        raise ValueError("rope_theta must be positive.")
    inverse_frequencies = 1.0 / (
        theta ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.float32) / head_dim)
    )
    positions = torch.arange(sequence_length, device=device, dtype=torch.float32)
    angles = torch.outer(positions, inverse_frequencies)
    return angles.cos().to(dtype=dtype), angles.sin().to(dtype=dtype)


def apply_rotary_embedding(states: Tensor, cosine: Tensor, sine: Tensor) -> Tensor:
    """Eager interleaved-pair RoPE of ``(batch, heads, sequence, head_dim)`` states
    (reference nn/rope.py:35-51); its gradient is computed by autograd."""

    if states.size(-1) != cosine.size(-1) * 2:
        raise ValueError("RoPE table dimension does not match the attention head dimension.")
    cosine = cosine.unsqueeze(0).unsqueeze(0)
    sine = sine.unsqueeze(0).unsqueeze(0)
    even_states = states[..., 0::2]
    odd_states = states[..., 1::2]
    rotated = torch.stack(
        (even_states * cosine - odd_states * sine, even_states * sine + odd_states * cosine),
        dim=-1,
    )
    return rotated.flatten(start_dim=-2)


class RotaryEmbedding(nn.Module):
    """Apply standard (interleaved-pair) RoPE to attention query and key tensors."""

    def __init__(
        self, head_dim: int, theta: float = 10_000.0, *, use_triton_rope: bool = False
    ) -> None:
        super().__init__()
        if head_dim % 2 != 0:
            raise ValueError("RoPE requires an even attention head dimension.")
        if theta <= 0:
            raise ValueError("rope_theta must be positive.")
        self.head_dim = head_dim
        self.theta = theta
        self.use_triton_rope = use_triton_rope
        self._triton_fallback_warned = False
        # Tables depend only on (S, D, theta, device, dtype); the reference rebuilds them
        # every call (nn/rope.py:79-85), this module builds each one once.
        self._tables: dict[tuple, tuple[Tensor, Tensor]] = {}

    def _cos_sin(self, sequence_length: int, device: torch.device, dtype: torch.dtype):
        key = (sequence_length, str(device), dtype)
        tables = self._tables.get(key)
        if tables is None:
            tables = rotary_cos_sin(
                sequence_length, self.head_dim, self.theta, device=device, dtype=dtype
            )
            self._tables[key] = tables
        return tables

    def forward(self, query: Tensor, key: Tensor) -> tuple[Tensor, Tensor]:
        """Rotate query and key using their shared sequence positions."""

        if (
            query.size(0) != key.size(0)
            or query.size(-2) != key.size(-2)
            or query.size(-1) != key.size(-1)
        ):
            raise ValueError("RoPE query and key must share batch, sequence, and head dimensions.")
        cosine, sine = self._cos_sin(query.size(-2), query.device, query.dtype)
        if self.use_triton_rope:
            if query.is_cuda and key.is_cuda:
                layout = ops.LAYOUTS["interleaved"]
                if query.dtype == key.dtype and query.device == key.device:
                    return torch.ops.picotron_b200.rope_qk(query, key, cosine, sine, layout)
                return (
                    torch.ops.picotron_b200.rope(query, cosine, sine, layout),
                    torch.ops.picotron_b200.rope(key, cosine, sine, layout),
                )
            _warn_once(self, "RoPE", RuntimeError("sm_100a RoPE requires CUDA tensors."))
        return (
            apply_rotary_embedding(query, cosine, sine),
            apply_rotary_embedding(key, cosine, sine),
        )
