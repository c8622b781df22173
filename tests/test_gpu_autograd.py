"""The torch custom ops, autograd, drop-in modules, probe and error paths on the GPU."""

from __future__ import annotations

import ctypes

import pytest
import torch
from torch.nn import functional as F

import gpu_utils as gu
import picotron_b200 as pb
from oracle import picotron_oracle as po
from oracle import tolerance
from picotron_b200 import _capi
from picotron_b200.errors import TritonRMSNormUnavailable, TritonSwiGLUUnavailable
from picotron_b200.modules import RMSNorm, RotaryEmbedding, SwiGLU

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    gu.require_gpu()


def test_detect_support_and_probe():
    report = pb.detect_triton_support(enabled=True, device=0)
    assert report.installed and report.hardware_compatible and report.available
    result = pb.probe_hot_path(0)
    assert all(v <= 1e-4 for v in result.max_errors.values()), result


def test_rms_norm_op_autograd_matches_oracle():
    x = gu.randn((4, 33, 4096), 1, torch.bfloat16).requires_grad_(True)
    w = gu.randn(4096, 2, torch.float32, 0.02, 1.0).requires_grad_(True)
    dy = gu.randn((4, 33, 4096), 3, torch.bfloat16)
    y = pb.triton_rms_norm(x, w, 1e-5)
    assert y.dtype == x.dtype and y.shape == x.shape
    dx, dw = torch.autograd.grad(y, (x, w), dy)
    assert dw.dtype == w.dtype
    ye, _ = po.rms_norm_forward(x.detach(), w.detach(), 1e-5, "exact")
    dxe, dwe = po.rms_norm_backward(x.detach(), w.detach(), dy, 1e-5, "exact")
    tolerance.assert_close(y, ye, "y")
    tolerance.assert_close(dx, dxe, "dx")
    tolerance.assert_close(dw, dwe, "dw")


def test_rms_norm_fp32_residual_stream():
    # Under autocast the reference feeds RMSNorm an fp32 residual with an fp32 weight.
    x = gu.randn((2, 64, 4096), 4, torch.float32).requires_grad_(True)
    norm = RMSNorm(4096, use_triton_rmsnorm=True).to(gu.DEV)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = norm(x)
    assert y.dtype == torch.float32
    dy = gu.randn(y.shape, 5, torch.float32)
    dx, dw = torch.autograd.grad(y, (x, norm.weight), dy)
    ye, _ = po.rms_norm_forward(x.detach(), norm.weight.detach(), 1e-6, "exact")
    dxe, dwe = po.rms_norm_backward(x.detach(), norm.weight.detach(), dy, 1e-6, "exact")
    tolerance.assert_close(y, ye, "y")
    tolerance.assert_close(dx, dxe, "dx")
    tolerance.assert_close(dw, dwe, "dw")
    assert not norm._triton_fallback_warned


def test_fused_add_rms_norm_autograd_matches_two_step_eager():
    # forward_with_residual == (h = residual + branch, norm(h)) with gradients through both
    # outputs, as in the decoder block (the residual stream h is used again downstream).
    shape = (2, 50, 4096)
    res = gu.randn(shape, 71, torch.bfloat16).requires_grad_(True)
    br = gu.randn(shape, 72, torch.bfloat16).requires_grad_(True)
    norm = RMSNorm(4096, eps=1e-5, use_triton_rmsnorm=True).to(gu.DEV)
    with torch.no_grad():
        norm.weight.copy_(gu.randn(4096, 73, torch.float32, 0.02, 1.0))
    h, y = norm.forward_with_residual(res, br)
    dy = gu.randn(shape, 74, torch.bfloat16)
    dh = gu.randn(shape, 75, torch.bfloat16)
    dres, dbr, dw = torch.autograd.grad((y, h), (res, br, norm.weight), (dy, dh))
    assert torch.equal(h, res.detach() + br.detach())
    ye, _ = po.rms_norm_forward(h.detach(), norm.weight.detach(), 1e-5, "exact")
    dxe, dwe = po.add_rms_norm_backward(h.detach(), norm.weight.detach(), dy, dh, 1e-5, "exact")
    tolerance.assert_close(y, ye, "y")
    tolerance.assert_close(dres, dxe, "dresidual")
    tolerance.assert_close(dbr, dxe, "dbranch")
    tolerance.assert_close(dw, dwe, "dw")
    # Only y used downstream: the norm gradient alone.
    h2, y2 = pb.fused_add_rms_norm(res, br, norm.weight, 1e-5)
    (dres2,) = torch.autograd.grad(y2, (res,), dy)
    dxe2, _ = po.rms_norm_backward(h2.detach(), norm.weight.detach(), dy, 1e-5, "exact")
    tolerance.assert_close(dres2, dxe2, "dresidual (y only)")


def test_fused_gate_up_module_matches_three_step_path():
    # SwiGLU with fuse_gate_up (tcgen05 GEMM + activation epilogue) against the same module
    # run as gate/up Linear + the SwiGLU kernel, forward and backward, under bf16 autocast
    # with fp32 parameters (the reference's training setup).
    torch.manual_seed(0)
    mlp = SwiGLU(512, 1024, use_triton_swiglu=True).to(gu.DEV)
    x = gu.randn((4, 96, 512), 91, torch.float32).requires_grad_(True)
    dy = gu.randn((4, 96, 512), 92, torch.bfloat16)
    grads = []
    outs = []
    for fused in (False, True):
        mlp.fuse_gate_up = fused
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = mlp(x)
        outs.append(y.float())
        grads.append(torch.autograd.grad(y, (x, mlp.gate_projection.weight,
                                             mlp.up_projection.weight,
                                             mlp.down_projection.weight), dy))
    # Same math; only the GEMMs' fp32 summation order differs: compare normwise.
    for a, b, name in zip((outs[1], *grads[1]), (outs[0], *grads[0]),
                          ("y", "dx", "dw_gate", "dw_up", "dw_down")):
        err = (a.float() - b.float()).abs().max().item()
        assert err <= 2 ** -6 * b.float().abs().max().item(), (name, err)


def test_swiglu_op_autograd_and_module():
    mlp = SwiGLU(256, 512, use_triton_swiglu=True).to(gu.DEV).to(torch.bfloat16)
    gate = gu.randn((3, 17, 512), 6, torch.bfloat16, 2.0).requires_grad_(True)
    up = gu.randn((3, 17, 512), 7, torch.bfloat16, 2.0).requires_grad_(True)
    out = pb.triton_swiglu(gate, up)
    dy = gu.randn(out.shape, 8, torch.bfloat16)
    dg, du = torch.autograd.grad(out, (gate, up), dy)
    tolerance.assert_close(out, po.swiglu_forward(gate.detach(), up.detach(), "exact"), "out")
    dge, due = po.swiglu_backward(gate.detach(), up.detach(), dy, "exact")
    tolerance.assert_close(dg, dge, "dgate")
    tolerance.assert_close(du, due, "dup")
    h = gu.randn((3, 17, 256), 9, torch.bfloat16)
    ref = mlp.down_projection(F.silu(mlp.gate_projection(h).float()).bfloat16()
                              * mlp.up_projection(h))
    torch.testing.assert_close(mlp(h), ref, rtol=2e-2, atol=2e-2)
    assert not mlp._triton_fallback_warned


def test_rotary_module_on_attention_views():
    rope = RotaryEmbedding(128, theta=500_000.0, use_triton_rope=True)
    q_mem = gu.randn((2, 64, 8, 128), 10, torch.bfloat16).requires_grad_(True)
    k_mem = gu.randn((2, 64, 2, 128), 11, torch.bfloat16).requires_grad_(True)
    q, k = q_mem.transpose(1, 2), k_mem.transpose(1, 2)
    qo, ko = rope(q, k)
    assert qo.stride() == q.stride()  # output keeps the [B, S, H, D] memory layout
    dq = gu.randn(qo.shape, 12, torch.bfloat16)
    dk = gu.randn(ko.shape, 13, torch.bfloat16)
    gq, gk = torch.autograd.grad((qo, ko), (q_mem, k_mem), (dq, dk))
    cos, sin = po.rotary_cos_sin(64, 128, 500_000.0, torch.bfloat16)
    cos, sin = cos.to(gu.DEV), sin.to(gu.DEV)
    tolerance.assert_close(qo, po.rope_forward(q.detach(), cos, sin, "exact"), "q")
    tolerance.assert_close(ko, po.rope_forward(k.detach(), cos, sin, "exact"), "k")
    tolerance.assert_close(gq.transpose(1, 2), po.rope_backward(dq, cos, sin, "exact"), "dq")
    tolerance.assert_close(gk.transpose(1, 2), po.rope_backward(dk, cos, sin, "exact"), "dk")
    assert not rope._triton_fallback_warned


def test_rotate_half_functional_layout():
    x = gu.randn((2, 4, 32, 64), 14, torch.bfloat16)
    cos, sin = po.rotary_cos_sin(32, 64, 10_000.0, torch.bfloat16)
    cos, sin = cos.to(gu.DEV), sin.to(gu.DEV)
    out = pb.triton_apply_rotary_embedding(x, cos, sin, layout="rotate_half")
    tolerance.assert_close(out, po.rope_forward(x, cos, sin, "exact", "rotate_half"), "rh")


def test_torch_compile_traces_the_custom_ops():
    def block(x, w, gate, up):
        return pb.triton_rms_norm(x, w, 1e-6).sum() + pb.triton_swiglu(gate, up).float().sum()

    x = gu.randn((8, 1024), 15, torch.bfloat16).requires_grad_(True)
    w = gu.randn(1024, 16, torch.float32, 0.1, 1.0).requires_grad_(True)
    g = gu.randn((8, 2048), 17, torch.bfloat16).requires_grad_(True)
    u = gu.randn((8, 2048), 18, torch.bfloat16).requires_grad_(True)
    eager = block(x, w, g, u)
    grads_eager = torch.autograd.grad(eager, (x, w, g, u))
    compiled = torch.compile(block, backend="aot_eager", fullgraph=True)
    out = compiled(x, w, g, u)
    grads = torch.autograd.grad(out, (x, w, g, u))
    torch.testing.assert_close(out, eager)
    for a, b in zip(grads, grads_eager):
        assert torch.equal(a, b)


def test_checkpoint_recompute_is_bit_identical():
    from torch.utils.checkpoint import checkpoint

    norm = RMSNorm(2048, use_triton_rmsnorm=True).to(gu.DEV)
    mlp = SwiGLU(2048, 4096, use_triton_swiglu=True).to(gu.DEV)
    x = gu.randn((4, 32, 2048), 19, torch.float32)

    def layer(h):
        return mlp(norm(h))

    x1 = x.clone().requires_grad_(True)
    layer(x1).square().mean().backward()
    g_plain = (x1.grad.clone(), norm.weight.grad.clone())
    norm.zero_grad(set_to_none=True)
    mlp.zero_grad(set_to_none=True)
    x2 = x.clone().requires_grad_(True)
    checkpoint(layer, x2, use_reentrant=False).square().mean().backward()
    assert torch.equal(x2.grad, g_plain[0])
    assert torch.equal(norm.weight.grad, g_plain[1])


def test_capi_rejects_host_pointers_without_launching():
    host = torch.zeros(1024, dtype=torch.bfloat16).pin_memory()
    dev = torch.zeros(1024, dtype=torch.bfloat16, device=gu.DEV)
    lib = _capi.library()
    status = lib.pt_swiglu_fwd(host.data_ptr(), dev.data_ptr(), dev.data_ptr(), 1024,
                               _capi.PT_BFLOAT16, None)
    assert status == _capi.PT_ERR_DEVICE and "gate" in _capi.last_error()
    buf = ctypes.create_string_buffer(4096)
    status = lib.pt_swiglu_fwd(dev.data_ptr(), ctypes.addressof(buf), dev.data_ptr(), 1024,
                               _capi.PT_BFLOAT16, None)
    assert status == _capi.PT_ERR_DEVICE
    with pytest.raises(TritonSwiGLUUnavailable):
        torch.ops.picotron_b200.swiglu(dev, host)


def test_capi_rejects_unsupported_dtype_pair():
    x = torch.zeros((4, 64), dtype=torch.bfloat16, device=gu.DEV)
    w = torch.zeros(64, dtype=torch.float16, device=gu.DEV)
    with pytest.raises(_capi.PtError) as info:
        gu.rmsnorm_fwd(x, w, 1e-6)
    assert info.value.status == _capi.PT_ERR_UNSUPPORTED_DTYPE
    # the op layer widens such weights to fp32 instead
    y = torch.ops.picotron_b200.rms_norm(x + 1, w + 1, 1e-6)
    assert torch.isfinite(y.float()).all()


def test_op_errors_are_typed():
    x = torch.zeros((4, 64), dtype=torch.bfloat16, device=gu.DEV)
    with pytest.raises(TritonRMSNormUnavailable, match="hidden size"):
        torch.ops.picotron_b200.rms_norm(x, torch.ones(32, device=gu.DEV), 1e-6)
    with pytest.raises(TritonRMSNormUnavailable, match="dtype"):
        torch.ops.picotron_b200.rms_norm(x.double(), torch.ones(64, device=gu.DEV), 1e-6)


def test_bounded_wait_timeout_is_reported_and_the_context_survives():
    # Failure detection without a GPU fault: a wait on a barrier that nothing arrives at gives
    # up after ~5 ms of SM clock, the device error word reads 1 (then 0 once taken), and the
    # next kernels run normally.
    assert _capi.take_device_error() == 0
    _capi.selftest_wait_timeout(10_000_000, gu.stream())
    torch.cuda.synchronize()
    assert _capi.take_device_error() == 1
    assert _capi.take_device_error() == 0
    x = gu.randn((64, 512), 95, torch.bfloat16)
    w = gu.randn((512,), 96, torch.float32, scale=0.02, shift=1.0)
    y = gu.rmsnorm_fwd(x, w, 1e-5)
    ye, _ = po.rms_norm_forward(x.cpu(), w.cpu(), 1e-5, "exact")
    tolerance.assert_close(y, ye, "rmsnorm after a reported timeout")
    assert _capi.take_device_error() == 0
    with pytest.raises(_capi.PtError):
        _capi.selftest_wait_timeout(0, gu.stream())
