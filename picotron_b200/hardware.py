"""Capability report and forward/backward probe of the sm_100a hot path.

``detect_triton_support`` keeps the reference's name, keywords and ``TritonReport`` fields
(src/picotron/utils/hardware.py:31-38, 93-108). "installed" now means that
``libpicotron_b200.so`` loads, and "hardware_compatible" that the device is compute
capability 10.0 (the library carries sm_100a code only).

``probe_hot_path`` is the runtime check of the reference's notebook probe
(examples/kaggle_demo_pretrain_sft_dpo.ipynb, cells 166-181): it runs the three modules
with their switches on through one forward and backward on the device, asserts that none
fell back, and compares values and gradients with an fp32 evaluation of the same
formulas on the same device.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from picotron_b200 import _capi


@dataclass(frozen=True, slots=True)
class TritonReport:
    """Accelerated-kernel status; disabled unless explicitly requested."""

    enabled: bool
    installed: bool
    hardware_compatible: bool
    available: bool


def _device_index(device: int | torch.device | None) -> int | None:
    if not torch.cuda.is_available():
        return None
    if device is None:
        return torch.cuda.current_device()
    if isinstance(device, int):
        return device
    device = torch.device(device)
    if device.type != "cuda":
        return None
    return device.index if device.index is not None else torch.cuda.current_device()


def detect_triton_support(
    *, enabled: bool = False, device: int | torch.device | None = None
) -> TritonReport:
    """Report whether the sm_100a kernels can run, without enabling them implicitly."""

    installed = _capi.is_available()
    index = _device_index(device)
    compatible = False
    if installed and index is not None:
        status, _, _, _ = _capi.probe(index)
        compatible = status == _capi.PT_OK
    return TritonReport(
        enabled=enabled,
        installed=installed,
        hardware_compatible=compatible,
        available=enabled and installed and compatible,
    )


@dataclass(frozen=True)
class ProbeResult:
    device: str
    max_errors: dict[str, float]


def probe_hot_path(device: int | torch.device | None = None, seed: int = 0) -> ProbeResult:
    """Run RMSNorm -> SwiGLU activation and RoPE fwd+bwd once with the switches on.

    Raises AssertionError when a module fell back or a value or gradient is off by more
    than fp32 tolerance (1e-4 relative to the tensor's magnitude).
    """

    from picotron_b200.modules import RMSNorm, RotaryEmbedding, SwiGLU, apply_rotary_embedding

    index = _device_index(device)
    if index is None:
        raise RuntimeError("probe_hot_path needs a CUDA device")
    dev = torch.device("cuda", index)
    gen = torch.Generator(device="cpu").manual_seed(seed)
    errors: dict[str, float] = {}

    def rel(a: torch.Tensor, b: torch.Tensor) -> float:
        a, b = a.detach().float(), b.detach().float()
        return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))

    hidden, inter, tokens = 64, 96, 48
    norm = RMSNorm(hidden, use_triton_rmsnorm=True).to(dev)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(hidden, generator=gen))
    mlp = SwiGLU(hidden, inter, use_triton_swiglu=True).to(dev)
    x = torch.randn(2, tokens // 2, hidden, generator=gen).to(dev).requires_grad_(True)
    y = norm(x)
    gate, up = mlp.gate_projection(y), mlp.up_projection(y)
    act = mlp.activation(gate, up)
    dact = torch.randn(act.shape, generator=gen).to(dev)
    grads = torch.autograd.grad(act, (x, norm.weight), dact)

    xr = x.detach().clone().requires_grad_(True)
    wr = norm.weight.detach().clone().requires_grad_(True)
    yr = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + norm.eps) * wr
    gr, ur = mlp.gate_projection(yr), mlp.up_projection(yr)
    ar = torch.nn.functional.silu(gr) * ur
    grads_r = torch.autograd.grad(ar, (xr, wr), dact)
    errors["rmsnorm_swiglu_out"] = rel(act, ar)
    errors["rmsnorm_dx"] = rel(grads[0], grads_r[0])
    errors["rmsnorm_dweight"] = rel(grads[1], grads_r[1])

    rope = RotaryEmbedding(16, theta=500_000.0, use_triton_rope=True)
    # Query as the attention layer makes it: a [B, H, S, D] view of [B, S, H, D] memory.
    q_base = torch.randn(2, 16, 4, 16, generator=gen).to(dev).requires_grad_(True)
    q = q_base.transpose(1, 2)
    k = torch.randn(2, 2, 16, 16, generator=gen).to(dev)
    qo, ko = rope(q, k)
    dq = torch.randn(qo.shape, generator=gen).to(dev)
    gq = torch.autograd.grad(qo, q_base, dq)[0]
    cos, sin = rope._cos_sin(16, dev, q.dtype)
    qe = q_base.detach().clone().requires_grad_(True)
    qr = apply_rotary_embedding(qe.transpose(1, 2), cos, sin)
    gqr = torch.autograd.grad(qr, qe, dq)[0]
    errors["rope_out"] = rel(qo, qr)
    errors["rope_dx"] = rel(gq, gqr)

    for module in (norm, mlp, rope):
        assert not module._triton_fallback_warned, f"{type(module).__name__} fell back"
    bad = {k: v for k, v in errors.items() if not v <= 1e-4}
    assert not bad, f"probe mismatch: {bad}"
    return ProbeResult(device=str(dev), max_errors=errors)
