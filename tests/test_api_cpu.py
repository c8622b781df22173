"""Drop-in API checks without a GPU: module constructors, parameter names (checkpoint
layout), config keys, the reference's CPU warn-and-eager contract, error types, and the
fake (meta) implementations of the custom ops used by torch.compile."""

from __future__ import annotations

import dataclasses

import pytest
import torch
from torch.nn import functional as F

import picotron_b200 as pb
from picotron_b200 import ops
from picotron_b200.config import ConfigValidationError, TritonKernelsConfig
from picotron_b200.kernels import (
    TritonRMSNormUnavailable,
    TritonRoPEUnavailable,
    TritonSwiGLUUnavailable,
    rms_norm_with_pytorch_forward,
    swiglu_with_pytorch_forward,
    triton_apply_rotary_embedding,
    triton_rms_norm,
    triton_swiglu,
)
from picotron_b200.modules import RMSNorm, RotaryEmbedding, SwiGLU


def test_kernel_entry_points_import_without_cuda():
    # reference tests/test_triton_rmsnorm_swiglu_rope.py:17-20
    assert callable(triton_rms_norm)
    assert callable(triton_swiglu)
    assert callable(triton_apply_rotary_embedding)


def test_detect_support_reports_unavailable_without_gpu():
    # reference tests/test_triton_kernels.py:11-16
    report = pb.detect_triton_support()
    assert not report.enabled
    assert not report.available
    assert report.installed  # the library itself loads on any Linux host
    report = pb.detect_triton_support(enabled=True)
    assert report.enabled and not report.available


def test_enabled_modules_warn_and_use_eager_math_on_cpu():
    # reference tests/test_triton_rmsnorm_swiglu_rope.py:23-49 (same messages, same values)
    hidden_states = torch.randn(2, 3, 8)
    norm = RMSNorm(8, use_triton_rmsnorm=True)
    with pytest.warns(RuntimeWarning, match="Triton RMSNorm unavailable"):
        normalized = norm(hidden_states)
    expected = hidden_states * torch.rsqrt(hidden_states.pow(2).mean(dim=-1, keepdim=True) + norm.eps)
    torch.testing.assert_close(normalized, expected * norm.weight)
    assert norm._triton_fallback_warned

    swiglu = SwiGLU(8, 16, use_triton_swiglu=True)
    with pytest.warns(RuntimeWarning, match="Triton SwiGLU unavailable"):
        fused_output = swiglu(hidden_states)
    expected_swiglu = swiglu.down_projection(
        F.silu(swiglu.gate_projection(hidden_states)) * swiglu.up_projection(hidden_states)
    )
    torch.testing.assert_close(fused_output, expected_swiglu)

    query, key = torch.randn(2, 4, 3, 8), torch.randn(2, 4, 3, 8)
    kernel_rope = RotaryEmbedding(8, use_triton_rope=True)
    native_rope = RotaryEmbedding(8)
    with pytest.warns(RuntimeWarning, match="Triton RoPE unavailable"):
        kq, kk = kernel_rope(query, key)
    nq, nk = native_rope(query, key)
    torch.testing.assert_close(kq, nq)
    torch.testing.assert_close(kk, nk)


def test_warning_is_emitted_once():
    norm = RMSNorm(8, use_triton_rmsnorm=True)
    with pytest.warns(RuntimeWarning):
        norm(torch.randn(2, 8))
    import warnings

    with warnings.catch_warnings():
        warnings.simplefilter("error")
        norm(torch.randn(2, 8))


def test_functional_entry_points_raise_typed_errors_on_cpu():
    x = torch.randn(4, 8)
    with pytest.raises(TritonRMSNormUnavailable):
        triton_rms_norm(x, torch.ones(8), 1e-6)
    with pytest.raises(TritonSwiGLUUnavailable):
        triton_swiglu(x, x)
    cos, sin = torch.ones(3, 4), torch.zeros(3, 4)
    with pytest.raises(TritonRoPEUnavailable):
        triton_apply_rotary_embedding(torch.randn(1, 2, 3, 8), cos, sin)
    for exc in (TritonRMSNormUnavailable, TritonSwiGLUUnavailable, TritonRoPEUnavailable):
        assert issubclass(exc, RuntimeError)


def test_ops_raise_on_cpu_tensors():
    with pytest.raises(TritonRMSNormUnavailable, match="CUDA"):
        torch.ops.picotron_b200.rms_norm(torch.randn(2, 8), torch.ones(8), 1e-6)
    with pytest.raises(TritonSwiGLUUnavailable, match="CUDA"):
        torch.ops.picotron_b200.swiglu(torch.randn(2, 8), torch.randn(2, 8))


def test_checkpoint_parameter_names_match_reference():
    # reference parameter names (picotron_decoder.py:27, feedforward.py:20-22)
    assert list(RMSNorm(16).state_dict()) == ["weight"]
    assert RMSNorm(16).weight.dtype == torch.float32
    assert torch.equal(RMSNorm(16).weight.detach(), torch.ones(16))
    assert list(SwiGLU(16, 32).state_dict()) == [
        "gate_projection.weight", "up_projection.weight", "down_projection.weight"]
    assert list(RotaryEmbedding(8).state_dict()) == []
    assert RMSNorm(16).eps == 1e-6


def test_constructor_signatures_match_reference():
    import inspect

    sig = inspect.signature(RMSNorm.__init__)
    assert list(sig.parameters) == ["self", "hidden_size", "eps", "use_triton_rmsnorm"]
    assert sig.parameters["use_triton_rmsnorm"].kind is inspect.Parameter.KEYWORD_ONLY
    sig = inspect.signature(SwiGLU.__init__)
    assert list(sig.parameters) == ["self", "hidden_size", "intermediate_size", "use_triton_swiglu"]
    sig = inspect.signature(RotaryEmbedding.__init__)
    assert list(sig.parameters) == ["self", "head_dim", "theta", "use_triton_rope"]
    assert sig.parameters["theta"].default == 10_000.0
    with pytest.raises(ValueError):
        RotaryEmbedding(7)
    with pytest.raises(ValueError):
        RotaryEmbedding(8, theta=0)


def test_triton_kernels_config_keys_and_strictness():
    cfg = TritonKernelsConfig()
    assert [f.name for f in dataclasses.fields(cfg)] == [
        "rmsnorm", "swiglu", "rope", "attention", "cross_entropy", "adamw"]
    assert not any(dataclasses.asdict(cfg).values())
    with pytest.raises(ConfigValidationError):
        TritonKernelsConfig(rmsnorm=1)
    with pytest.raises(ConfigValidationError, match="Unknown"):
        TritonKernelsConfig.from_mapping({"rmsnorm": True, "layernorm": True})
    cfg = TritonKernelsConfig.from_mapping({"rmsnorm": True, "rope": True})
    assert cfg.module_kwargs() == {"use_triton_rmsnorm": True, "use_triton_swiglu": False,
                                   "use_triton_rope": True}
    assert RMSNorm(8, **{k: v for k, v in cfg.module_kwargs().items()
                         if k == "use_triton_rmsnorm"}).use_triton_rmsnorm


def test_eager_rmsnorm_backward_matches_native():
    # reference tests/test_triton_rmsnorm_backward.py:13-32, against this package's
    # API-compatibility entry point.
    torch.manual_seed(23)
    eps = 1e-6
    dy = torch.randn(2, 3, 8)
    x = torch.randn(2, 3, 8, requires_grad=True)
    w = torch.randn(8, requires_grad=True)
    out = rms_norm_with_pytorch_forward(x, w, eps)
    (out * dy).sum().backward()
    xn = x.detach().clone().requires_grad_(True)
    wn = w.detach().clone().requires_grad_(True)
    outn = xn * torch.rsqrt(xn.square().mean(dim=-1, keepdim=True) + eps) * wn
    (outn * dy).sum().backward()
    torch.testing.assert_close(out, outn, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(x.grad, xn.grad, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(w.grad, wn.grad, rtol=1e-5, atol=1e-6)


def test_eager_swiglu_backward_matches_native():
    # reference tests/test_triton_swiglu_backward.py:9-26
    torch.manual_seed(31)
    dy = torch.randn(2, 3, 7, dtype=torch.float64)
    g = torch.randn(2, 3, 7, dtype=torch.float64, requires_grad=True)
    u = torch.randn(2, 3, 7, dtype=torch.float64, requires_grad=True)
    out = swiglu_with_pytorch_forward(g, u)
    (out * dy).sum().backward()
    gn = g.detach().clone().requires_grad_(True)
    un = u.detach().clone().requires_grad_(True)
    (F.silu(gn) * un * dy).sum().backward()
    torch.testing.assert_close(g.grad, gn.grad, rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(u.grad, un.grad, rtol=1e-10, atol=1e-10)


def test_fake_implementations_on_meta_tensors():
    x = torch.empty(3, 5, 64, device="meta", dtype=torch.bfloat16)
    w = torch.empty(64, device="meta", dtype=torch.float32)
    y = torch.ops.picotron_b200.rms_norm(x, w, 1e-6)
    assert y.shape == x.shape and y.dtype == x.dtype and y.device.type == "meta"
    dx, dw = torch.ops.picotron_b200.rms_norm_backward(x, x, w, 1e-6)
    assert dx.shape == x.shape and dw.shape == w.shape and dw.dtype == w.dtype
    g = torch.empty(7, 96, device="meta", dtype=torch.bfloat16)
    assert torch.ops.picotron_b200.swiglu(g, g).shape == g.shape
    dg, du = torch.ops.picotron_b200.swiglu_backward(g, g, g)
    assert dg.shape == g.shape and du.shape == g.shape
    q = torch.empty(2, 5, 4, 16, device="meta", dtype=torch.bfloat16).transpose(1, 2)
    cos = torch.empty(5, 8, device="meta", dtype=torch.bfloat16)
    out = torch.ops.picotron_b200.rope(q, cos, cos, ops.LAYOUTS["interleaved"])
    assert out.shape == q.shape and out.stride() == q.stride()


def test_rotary_tables_match_reference_formula():
    cos, sin = pb.rotary_cos_sin(16, 32, 500_000.0, device=torch.device("cpu"),
                                 dtype=torch.bfloat16)
    from oracle import picotron_oracle as po

    rc, rs = po.rotary_cos_sin(16, 32, 500_000.0, torch.bfloat16)
    assert torch.equal(cos, rc) and torch.equal(sin, rs)


def test_next_step_entry_points_on_cpu():
    # The loss and optimizer-step objects keep the reference's CPU contract: with the switch
    # on and CPU tensors they warn once (reference message) and use PyTorch.
    from picotron_b200.kernels import (
        AdamWStepWithFallback,
        CrossEntropyWithFallback,
        TritonAdamWUnavailable,
        TritonCrossEntropyUnavailable,
        fused_add_rms_norm,
        swiglu_gate_up,
        triton_adamw_step,
        triton_cross_entropy,
    )

    logits, targets = torch.randn(2, 7, 5), torch.randint(0, 7, (2, 5))
    loss_fn = CrossEntropyWithFallback(use_triton=True)
    with pytest.warns(RuntimeWarning, match="Triton cross-entropy unavailable"):
        loss = loss_fn(logits, targets)
    torch.testing.assert_close(loss, F.cross_entropy(logits, targets))
    with pytest.raises(TritonCrossEntropyUnavailable):
        triton_cross_entropy(logits[:, :, 0], targets[:, 0])

    p = torch.nn.Parameter(torch.randn(4))
    p.grad = torch.randn(4)
    opt = torch.optim.AdamW([p], lr=1e-2)
    ref = torch.optim.AdamW([q := torch.nn.Parameter(p.detach().clone())], lr=1e-2)
    q.grad = p.grad.clone()
    with pytest.raises(TritonAdamWUnavailable):
        triton_adamw_step(opt)
    assert len(opt.state[p]) == 0  # refused before touching the state
    with pytest.warns(RuntimeWarning, match="Triton AdamW unavailable"):
        AdamWStepWithFallback(use_triton=True).step(opt)
    ref.step()
    assert torch.equal(p, q)

    with pytest.raises(TritonRMSNormUnavailable):
        fused_add_rms_norm(torch.randn(2, 8), torch.randn(2, 8), torch.ones(8), 1e-6)
    with pytest.raises(TritonSwiGLUUnavailable):
        swiglu_gate_up(torch.randn(2, 8), torch.randn(16, 8), torch.randn(16, 8))
    # Module hooks take the eager steps on CPU.
    norm = RMSNorm(8, use_triton_rmsnorm=False)
    r, b = torch.randn(2, 8), torch.randn(2, 8)
    h, y = norm.forward_with_residual(r, b)
    torch.testing.assert_close(h, r + b)
    torch.testing.assert_close(y, norm(r + b))
    mlp = SwiGLU(8, 16)
    mlp.fuse_gate_up = True
    x = torch.randn(3, 8)
    torch.testing.assert_close(
        mlp(x), mlp.down_projection(F.silu(mlp.gate_projection(x)) * mlp.up_projection(x)))


def test_fake_implementations_of_next_step_ops():
    x = torch.empty(3, 5, 64, device="meta", dtype=torch.bfloat16)
    w = torch.empty(64, device="meta", dtype=torch.float32)
    h, y = torch.ops.picotron_b200.add_rms_norm(x, x, w, 1e-6)
    assert h.shape == x.shape and y.shape == x.shape
    wg = torch.empty(96, 64, device="meta", dtype=torch.bfloat16)
    act, g, u = torch.ops.picotron_b200.swiglu_gate_up(x, wg, wg)
    assert act.shape == (3, 5, 96) and g.shape == act.shape and u.dtype == torch.bfloat16
    wd = torch.empty(64, 96, device="meta", dtype=torch.bfloat16)
    dg, du = torch.ops.picotron_b200.swiglu_down_backward(x, wd, g, u)
    assert dg.shape == g.shape and du.shape == u.shape and dg.dtype == torch.bfloat16
    logits = torch.empty(2, 1000, 7, device="meta", dtype=torch.bfloat16)
    targets = torch.empty(2, 7, device="meta", dtype=torch.long)
    loss, lse, mean = torch.ops.picotron_b200.cross_entropy(logits, targets, -100)
    assert loss.shape == () and lse.shape == (14,) and mean.shape == (2,)
    q = torch.empty(2, 5, 4, 16, device="meta", dtype=torch.bfloat16).transpose(1, 2)
    k = torch.empty(2, 5, 1, 16, device="meta", dtype=torch.bfloat16).transpose(1, 2)
    cos = torch.empty(5, 8, device="meta", dtype=torch.bfloat16)
    qo, ko = torch.ops.picotron_b200.rope_qk(q, k, cos, cos, ops.LAYOUTS["interleaved"])
    assert qo.shape == q.shape and ko.shape == k.shape
