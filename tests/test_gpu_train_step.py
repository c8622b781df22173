"""A few training steps of a small decoder-shaped model with every kernel switch on, against
the same model on the reference's eager paths (switches off), from identical weights.

The model strings the hot path together the way picotron's decoder and training loop do:
RMSNorm -> q/k projections viewed as [B, H, S, D] -> RoPE on q and k -> (a cheap stand-in
for attention that mixes q and k) -> the residual add fused into the MLP norm -> SwiGLU MLP
-> output projection -> the loop's cross-entropy call on ``logits[:, :-1].transpose(1, 2)``
-> backward -> the AdamW step object. Each op is held to the float64 oracle elsewhere; this
test checks that the pieces compose (autograd plumbing, saved tensors, dtype handling,
in-place optimizer state) and that the two paths train alike.
"""

from __future__ import annotations

import pytest
import torch
from torch import nn

import gpu_utils as gu
from picotron_b200.kernels import AdamWStepWithFallback, CrossEntropyWithFallback
from picotron_b200.modules import RMSNorm, RotaryEmbedding, SwiGLU

pytestmark = pytest.mark.gpu

B, S, HEADS, D, VOCAB, INTER = 2, 64, 4, 32, 512, 384
HIDDEN = HEADS * D


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    gu.require_gpu()


class TinyDecoder(nn.Module):
    def __init__(self, kernels: bool, fuse_gate_up: bool = False) -> None:
        super().__init__()
        self.embedding = nn.Embedding(VOCAB, HIDDEN)
        self.attention_norm = RMSNorm(HIDDEN, 1e-5, use_triton_rmsnorm=kernels)
        self.q_proj = nn.Linear(HIDDEN, HIDDEN, bias=False)
        self.k_proj = nn.Linear(HIDDEN, HIDDEN, bias=False)
        self.rope = RotaryEmbedding(D, 10_000.0, use_triton_rope=kernels)
        self.mlp_norm = RMSNorm(HIDDEN, 1e-5, use_triton_rmsnorm=kernels)
        self.mlp = SwiGLU(HIDDEN, INTER, use_triton_swiglu=kernels)
        self.mlp.fuse_gate_up = fuse_gate_up
        self.final_norm = RMSNorm(HIDDEN, 1e-5, use_triton_rmsnorm=kernels)
        self.output = nn.Linear(HIDDEN, VOCAB, bias=False)

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        x = self.embedding(ids)
        n = self.attention_norm(x)
        q = self.q_proj(n).view(B, S, HEADS, D).transpose(1, 2)  # [B,H,S,D] views
        k = self.k_proj(n).view(B, S, HEADS, D).transpose(1, 2)
        q, k = self.rope(q, k)
        mixed = q * torch.sigmoid((q * k).sum(-1, keepdim=True) / D ** 0.5) + k
        attention_output = mixed.transpose(1, 2).reshape(B, S, HIDDEN)
        h, normed = self.mlp_norm.forward_with_residual(x, attention_output)
        h = h + self.mlp(normed)
        return self.output(self.final_norm(h))


def _train(kernels: bool, steps: int, autocast: bool = False, fuse_gate_up: bool = False):
    torch.manual_seed(1234)
    model = TinyDecoder(kernels, fuse_gate_up).to(gu.DEV)
    with torch.no_grad():
        for m in (model.attention_norm, model.mlp_norm, model.final_norm):
            m.weight.copy_(gu.randn((HIDDEN,), 71, scale=0.05, shift=1.0))
    optimizer = torch.optim.AdamW(model.parameters(), lr=1e-3, weight_decay=0.1)
    loss_fn = CrossEntropyWithFallback(use_triton=kernels)
    stepper = AdamWStepWithFallback(use_triton=kernels)
    g = torch.Generator().manual_seed(99)
    losses = []
    for _ in range(steps):
        ids = torch.randint(0, VOCAB, (B, S), generator=g).to(gu.DEV)
        optimizer.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
            logits = model(ids)
            loss = loss_fn(logits[:, :-1, :].transpose(1, 2), ids[:, 1:])
        loss.backward()
        stepper.step(optimizer)
        losses.append(float(loss.detach()))
    assert not loss_fn._fallback_warned and not stepper._fallback_warned
    for m in (model.attention_norm, model.mlp_norm, model.final_norm, model.mlp, model.rope):
        assert not m._triton_fallback_warned
    return losses, {n: p.detach().clone() for n, p in model.named_parameters()}


def _assert_params_close(params_k, params_e, atol, rtol, max_fraction):
    # Adam normalizes each update, so an element whose gradient is pure rounding noise on
    # both paths can move by up to about the learning rate per step in either direction;
    # such elements are allowed as a small fraction, everything else must agree tightly.
    for name, b in params_e.items():
        a = params_k[name]
        diff = (a.float() - b.float()).abs()
        fraction = (diff > atol + rtol * b.float().abs()).float().mean().item()
        assert fraction <= max_fraction, f"{name}: {fraction:.3%} of elements differ"
        assert diff.max().item() <= 1e-2, f"{name}: max difference {diff.max().item():.3e}"


def test_fp32_training_steps_match_the_eager_paths():
    steps = 3
    losses_k, params_k = _train(True, steps)
    losses_e, params_e = _train(False, steps)
    # fp32 everywhere: the kernel and eager paths differ only in summation order and in the
    # kernels' single roundings, so losses agree to ~1e-6 and the parameters after three
    # AdamW steps to ~1e-5 (the step size is 1e-3).
    torch.testing.assert_close(torch.tensor(losses_k), torch.tensor(losses_e), rtol=2e-5, atol=0)
    _assert_params_close(params_k, params_e, atol=1e-5, rtol=1e-4, max_fraction=1e-3)


def test_bf16_autocast_steps_with_the_fused_gate_up_gemm():
    steps = 3
    losses_k, params_k = _train(True, steps, autocast=True, fuse_gate_up=True)
    losses_e, params_e = _train(False, steps, autocast=True)
    # bf16 activations round differently on the two paths (the eager path rounds every
    # intermediate, the kernels once), so only the training trajectory is compared: losses
    # within 1 % and nearly all parameters within 1e-4 + 1 %.
    torch.testing.assert_close(torch.tensor(losses_k), torch.tensor(losses_e), rtol=1e-2, atol=0)
    _assert_params_close(params_k, params_e, atol=1e-4, rtol=1e-2, max_fraction=2e-2)
