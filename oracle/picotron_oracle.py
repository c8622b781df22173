"""CPU restatement of picotron's RMSNorm / SwiGLU / RoPE arithmetic (test oracle).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``. Every function cites the
reference file and lines whose arithmetic it restates. ``mode="eager"`` reproduces the
reference's PyTorch CPU computation op for op (same dtypes, same operation order);
``mode="exact"`` evaluates the same formula in float64 and returns float64.
"""

from __future__ import annotations

import torch
from torch import Tensor
from torch.nn import functional as F

MODES = ("eager", "exact")


def _check_mode(mode: str) -> None:
    if mode not in MODES:
        raise ValueError(f"mode must be one of {MODES}, got {mode!r}")


# --------------------------------------------------------------------------- RMSNorm --


def rms_norm_forward(x: Tensor, weight: Tensor, eps: float, mode: str = "eager"):
    """Returns (y, inverse_rms).

    eager: ``_inverse_rms`` + ``_pytorch_forward`` (picotron
    src/picotron/nn/triton_kernels/rmsnorm.py:49-60): r = rsqrt(mean(x.float()^2) + eps),
    y = (x.float() * r * w.float()).to(x.dtype). The fused Triton forward (:25-46) computes
    the same fp32 expression and stores in the x dtype.
    exact: the same formula in float64, unrounded.
    """

    _check_mode(mode)
    if mode == "exact":
        xd, wd = x.double(), weight.double()
        inv = torch.rsqrt(xd.square().mean(dim=-1, keepdim=True) + eps)
        return xd * inv * wd, inv
    values = x.float()
    inv = torch.rsqrt(values.square().mean(dim=-1, keepdim=True) + eps)
    return (values * inv * weight.float()).to(dtype=x.dtype), inv


def rms_norm_backward(x: Tensor, weight: Tensor, dy: Tensor, eps: float, mode: str = "eager",
                      inverse_rms: Tensor | None = None):
    """Returns (dx, dweight).

    eager: ``_RMSNormAutogradFunction.backward`` (rmsnorm.py:109-134):
      g = dy * w; dot_mean = mean(g * x); dx = r * (g - x * r^2 * dot_mean);
      dw = sum_rows(dy * x * r); all fp32, dx cast to x dtype, dw to w dtype.
      ``inverse_rms``: the r the forward saved (rmsnorm.py:103-104, as returned by
      rms_norm_forward); without it r is recomputed, with the same bits.
    exact: the same in float64, unrounded.
    """

    _check_mode(mode)
    if mode == "exact":
        xd, wd, gd = x.double(), weight.double(), dy.double()
        inv = torch.rsqrt(xd.square().mean(dim=-1, keepdim=True) + eps)
        g = gd * wd
        dot_mean = (g * xd).mean(dim=-1, keepdim=True)
        dx = inv * (g - xd * inv.square() * dot_mean)
        dw = (gd * xd * inv).reshape(-1, weight.numel()).sum(dim=0)
        return dx, dw
    if inverse_rms is None:
        inverse_rms = torch.rsqrt(x.float().square().mean(dim=-1, keepdim=True) + eps)
    x32, w32, g32 = x.float(), weight.float(), dy.float()
    weighted_grad = g32 * w32
    dot_mean = (weighted_grad * x32).mean(dim=-1, keepdim=True)
    dx = inverse_rms * (weighted_grad - x32 * inverse_rms.square() * dot_mean)
    dw = (g32 * x32 * inverse_rms).reshape(-1, weight.numel()).sum(dim=0)
    return dx.to(dtype=x.dtype), dw.to(dtype=weight.dtype)


def add_rms_norm_forward(residual: Tensor, branch: Tensor, weight: Tensor, eps: float,
                         mode: str = "eager"):
    """Returns (h, y, inverse_rms) for the residual add followed by RMSNorm.

    The caller restated is DecoderBlock.forward_with_auxiliary_loss
    (src/picotron/models/picotron_decoder.py:116-123): ``h = residual + branch`` (one PyTorch
    add in the tensors' dtype, so the fp32 sum rounded once) and then the block's RMSNorm
    module on h (rms_norm_forward above). h is materialised by the reference in that dtype
    in both modes; exact evaluates the RMSNorm of that stored h in float64.
    """

    _check_mode(mode)
    h = residual + branch
    y, inv = rms_norm_forward(h, weight, eps, mode)
    return h, y, inv


def add_rms_norm_backward(h: Tensor, weight: Tensor, dy: Tensor, dh: Tensor | None, eps: float,
                          mode: str = "eager"):
    """Returns (dx, dweight): the gradient of residual and of branch (they are equal) and
    of the weight, for the add + RMSNorm pair of picotron_decoder.py:116-123.

    Autograd of the reference: the RMSNorm backward at h (rms_norm_backward above, dx cast to
    the dtype) plus dh, the gradient reaching h through its other use, accumulated in that
    dtype. exact: the float64 RMSNorm gradient plus dh, unrounded.
    """

    _check_mode(mode)
    dx, dw = rms_norm_backward(h, weight, dy, eps, mode)
    if dh is not None:
        dx = dx + (dh.double() if mode == "exact" else dh)
    return dx, dw


# ---------------------------------------------------------------------------- SwiGLU --


def swiglu_forward(gate: Tensor, up: Tensor, mode: str = "eager") -> Tensor:
    """eager: ``F.silu(gate) * up`` in the input dtype (picotron
    src/picotron/nn/triton_kernels/swiglu.py:63-64 and nn/feedforward.py:42), i.e. SiLU
    rounded to the input dtype, then the product rounded again. (The Triton forward,
    swiglu.py:26-41, instead rounds once from fp32: g * (1/(1+exp(-g))) * u.)
    exact: g * sigmoid(g) * u in float64, unrounded."""

    _check_mode(mode)
    if mode == "exact":
        g, u = gate.double(), up.double()
        return g * torch.sigmoid(g) * u
    return F.silu(gate) * up


def gate_up_forward(x: Tensor, w_gate: Tensor, w_up: Tensor, mode: str = "eager"):
    """Returns (gate, up, activated) of SwiGLU.forward up to the down projection (picotron
    src/picotron/nn/feedforward.py:27-42): gate = gate_projection(x) = x @ w_gate^T,
    up = up_projection(x) = x @ w_up^T (nn.Linear without bias, in the input dtype),
    activated = F.silu(gate) * up (swiglu_forward above).
    exact: the two products and the activation in float64, unrounded."""

    _check_mode(mode)
    if mode == "exact":
        xd = x.double()
        g, u = xd @ w_gate.double().t(), xd @ w_up.double().t()
        return g, u, swiglu_forward(g, u, "exact")
    g, u = F.linear(x, w_gate), F.linear(x, w_up)
    return g, u, swiglu_forward(g, u, "eager")


def down_swiglu_backward(dy: Tensor, w_down: Tensor, gate: Tensor, up: Tensor,
                         mode: str = "eager"):
    """Returns (d_act, dgate, dup): the gradient that reaches the activation through
    SwiGLU.down_projection (src/picotron/nn/feedforward.py:43, an nn.Linear without bias, so
    d_act = dy @ w_down), then the activation's backward (swiglu_backward below).
    eager: the matmul in the input dtype (what autograd of F.linear computes) and the
    reference's backward op for op. exact: d_act in float64, then the float64 backward."""

    _check_mode(mode)
    if mode == "exact":
        d_act = dy.double() @ w_down.double()
    else:
        d_act = dy @ w_down
    dgate, dup = swiglu_backward(gate, up, d_act, mode)
    return d_act, dgate, dup


def swiglu_backward(gate: Tensor, up: Tensor, dout: Tensor, mode: str = "eager"):
    """Returns (dgate, dup).

    eager: ``_SwiGLUAutogradFunction.backward`` (swiglu.py:71-81) op for op in the input
    dtype: s = sigmoid(g); silu = g * s; dsilu = s * (1 + g * (1 - s));
    dgate = dout * up * dsilu; dup = dout * silu.
    exact: the same in float64, unrounded."""

    _check_mode(mode)
    if mode == "exact":
        gate, up, dout = gate.double(), up.double(), dout.double()
    sigmoid_gate = torch.sigmoid(gate)
    silu_gate = gate * sigmoid_gate
    silu_derivative = sigmoid_gate * (1 + gate * (1 - sigmoid_gate))
    return dout * up * silu_derivative, dout * silu_gate


# --------------------------------------------------------------------- cross-entropy --


def _ce_rows(logits: Tensor, targets: Tensor):
    # [N, V] / [N] or [B, V, S] / [B, S] (class dimension 1) as [rows, V] / [rows].
    if logits.dim() == 3:
        return logits.movedim(1, -1).reshape(-1, logits.size(1)), targets.reshape(-1)
    return logits, targets


def cross_entropy_forward(logits: Tensor, targets: Tensor, ignore_index: int = -100,
                          mode: str = "eager") -> Tensor:
    """Mean cross-entropy as the training loop computes it (picotron
    src/picotron/training/train_loop.py:141-145: F.cross_entropy(logits[:, :-1, :]
    .transpose(1, 2), input_ids[:, 1:]) through CrossEntropyWithFallback,
    nn/triton_kernels/cross_entropy.py:102-112; mean over the targets != ignore_index).
    eager: F.cross_entropy on the logits upcast to fp32 (what CUDA autocast does for
    cross_entropy; a no-op for the reference's fp32 CPU path), fp32 result.
    exact: log-sum-exp and the mean in float64."""

    _check_mode(mode)
    if mode == "eager":
        return F.cross_entropy(logits.float(), targets, ignore_index=ignore_index)
    x, t = _ce_rows(logits.double(), targets)
    keep = t != ignore_index
    lse = torch.logsumexp(x, dim=1)
    picked = x.gather(1, t.clamp(0, x.size(1) - 1).unsqueeze(1)).squeeze(1)
    return ((lse - picked) * keep).sum() / keep.sum()


def cross_entropy_backward(logits: Tensor, targets: Tensor, grad: float = 1.0,
                           ignore_index: int = -100, mode: str = "eager") -> Tensor:
    """Gradient of cross_entropy_forward with respect to the logits, in the logits' layout.
    eager: PyTorch autograd of the eager form, cast to the logits dtype (the gradient
    flowing back through autocast's fp32 cast). exact: (softmax - onehot) * grad / count in
    float64, zero for ignored rows."""

    _check_mode(mode)
    if mode == "eager":
        x = logits.detach().float().requires_grad_(True)
        loss = F.cross_entropy(x, targets, ignore_index=ignore_index)
        (dx,) = torch.autograd.grad(loss, (x,), torch.tensor(grad, dtype=torch.float32))
        return dx.to(logits.dtype)
    x = logits.double()
    rows, t = _ce_rows(x, targets)
    keep = (t != ignore_index).double()
    p = torch.softmax(rows, dim=1)
    onehot = torch.zeros_like(p).scatter_(1, t.clamp(0, rows.size(1) - 1).unsqueeze(1), 1.0)
    d = (p - onehot) * (keep * grad / keep.sum()).unsqueeze(1)
    if logits.dim() == 3:
        d = d.reshape(logits.size(0), logits.size(2), logits.size(1)).movedim(-1, 1)
    return d


# --------------------------------------------------------------------------- AdamW --


def adamw_step(param: Tensor, grad: Tensor, exp_avg: Tensor, exp_avg_sq: Tensor, step: int,
               lr: float, betas: tuple[float, float], eps: float, weight_decay: float,
               maximize: bool = False, mode: str = "eager"):
    """One AdamW step of one parameter; returns (param, exp_avg, exp_avg_sq), new tensors.

    The reference's optimizer step is torch.optim.AdamW built by the training loop
    (src/picotron/training/train_loop.py:302-325; its fused extension point,
    nn/triton_kernels/adamw.py:14-24, always falls back to it). eager: that optimizer's
    update op for op in fp32 (torch/optim/adam.py, decoupled weight decay): param *= 1 - lr*wd;
    exp_avg.lerp_(grad, 1 - beta1); exp_avg_sq = exp_avg_sq * beta2 + (1 - beta2) * grad^2;
    denom = sqrt(exp_avg_sq) / sqrt(1 - beta2^step) + eps;
    param += -(lr / (1 - beta1^step)) * exp_avg / denom; `step` is the count after this step.
    exact: the same formula in float64 from the same inputs."""

    _check_mode(mode)
    beta1, beta2 = betas
    if maximize:
        grad = -grad
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    if mode == "exact":
        p, g, m, v = param.double(), grad.double(), exp_avg.double(), exp_avg_sq.double()
        p = p * (1 - lr * weight_decay)
        m = m + (1 - beta1) * (g - m)
        v = v * beta2 + (1 - beta2) * g * g
        denom = v.sqrt() / bc2 ** 0.5 + eps
        return p - (lr / bc1) * m / denom, m, v
    p, m, v = param.clone(), exp_avg.clone(), exp_avg_sq.clone()
    if weight_decay != 0:
        p.mul_(1 - lr * weight_decay)
    m.lerp_(grad, 1 - beta1)
    v.mul_(beta2).addcmul_(grad, grad, value=1 - beta2)
    denom = (v.sqrt() / bc2 ** 0.5).add_(eps)
    p.addcdiv_(m, denom, value=-(lr / bc1))
    return p, m, v


# ------------------------------------------------------------------------------ RoPE --


def rotary_cos_sin(sequence_length: int, head_dim: int, theta: float, dtype: torch.dtype):
    """``rotary_cos_sin`` (picotron src/picotron/nn/rope.py:13-32) on CPU:
    inv = 1 / theta^(arange(0, D, 2) / D) in fp32; angles = outer(arange(S), inv);
    returns (cos(angles), sin(angles)) cast to ``dtype``."""

    if head_dim % 2 != 0:
        raise ValueError("RoPE requires an even attention head dimension.")
    inverse_frequencies = 1.0 / (
        theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim)
    )
    positions = torch.arange(sequence_length, dtype=torch.float32)
    angles = torch.outer(positions, inverse_frequencies)
    return angles.cos().to(dtype=dtype), angles.sin().to(dtype=dtype)


def _rope_eager(states: Tensor, cosine: Tensor, sine: Tensor) -> Tensor:
    # apply_rotary_embedding, picotron src/picotron/nn/rope.py:35-51.
    cosine = cosine.unsqueeze(0).unsqueeze(0)
    sine = sine.unsqueeze(0).unsqueeze(0)
    even_states = states[..., 0::2]
    odd_states = states[..., 1::2]
    rotated = torch.stack(
        (even_states * cosine - odd_states * sine, even_states * sine + odd_states * cosine),
        dim=-1,
    )
    return rotated.flatten(start_dim=-2)


def rope_forward(states: Tensor, cosine: Tensor, sine: Tensor, mode: str = "eager",
                 layout: str = "interleaved") -> Tensor:
    """Interleaved layout (the reference's): out[2i] = e*c - o*s, out[2i+1] = e*s + o*c,
    with (e, o) = (x[2i], x[2i+1]) and c, s = tables[seq, i] (nn/rope.py:42-51).
    eager evaluates in the states/table dtype op for op; exact in float64.

    layout="rotate_half" has no counterpart in the reference: it is the Llama/HF
    convention out[i] = x[i]*c[i] - x[i+D/2]*s[i], out[i+D/2] = x[i+D/2]*c[i] + x[i]*s[i],
    restated here for the labelled rotate-half variant of the kernels."""

    _check_mode(mode)
    if mode == "exact":
        states, cosine, sine = states.double(), cosine.double(), sine.double()
    if layout == "interleaved":
        return _rope_eager(states, cosine, sine)
    if layout != "rotate_half":
        raise ValueError(f"unknown layout {layout!r}")
    half = states.size(-1) // 2
    c, s = cosine[None, None], sine[None, None]
    x1, x2 = states[..., :half], states[..., half:]
    return torch.cat((x1 * c - x2 * s, x2 * c + x1 * s), dim=-1)


def rope_backward(dout: Tensor, cosine: Tensor, sine: Tensor, mode: str = "eager",
                  layout: str = "interleaved") -> Tensor:
    """Gradient of ``rope_forward`` with respect to the states.

    eager: what the reference's training path computes, i.e. torch autograd through the
    eager ``apply_rotary_embedding`` graph (nn/rope.py:35-51) in the states dtype.
    exact: the transposed rotation in float64: d_e = dy_e*c + dy_o*s,
    d_o = -dy_e*s + dy_o*c (interleaved), unrounded."""

    _check_mode(mode)
    if mode == "eager":
        x = torch.zeros(dout.shape, dtype=dout.dtype, requires_grad=True)
        with torch.enable_grad():
            out = rope_forward(x, cosine, sine, "eager", layout)
            (grad,) = torch.autograd.grad(out, x, dout)
        return grad
    return rope_forward(dout, cosine, -sine, "exact", layout)
