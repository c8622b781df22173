"""PyTorch custom ops (``torch.ops.picotron_b200.*``) over the C ABI, with autograd.

Ops, each an opaque ``torch.library.custom_op`` with a fake (meta) implementation so
``torch.compile`` can trace around it, and an autograd formula that calls the matching
backward op:

* ``rms_norm(x, weight, eps) -> y``                  (reference rmsnorm.py:87-160)
* ``rms_norm_backward(dy, x, weight, eps) -> (dx, dweight)``
* ``add_rms_norm(residual, branch, weight, eps) -> (h, y)``  (reference
  picotron_decoder.py:116-123: ``h = residual + branch`` then RMSNorm of h, fused)
* ``add_rms_norm_backward(dy, dh, h, weight, eps) -> (dx, dweight)``
* ``swiglu(gate, up) -> out``                        (reference swiglu.py:56-101)
* ``swiglu_backward(dout, gate, up) -> (dgate, dup)``
* ``swiglu_gate_up(x, w_gate, w_up) -> (act, gate, up)``  (reference feedforward.py:27-42:
  the gate and up projections and the activation as one tcgen05 GEMM with a SwiGLU epilogue)
* ``cross_entropy(logits, targets, ignore_index) -> (loss, row_lse, mean_out)``
  (reference train_loop.py:95-97,141-145: F.cross_entropy, mean over non-ignored rows)
* ``cross_entropy_backward(grad, logits, targets, row_lse, mean_out, ignore_index) -> dlogits``
* ``rope(x, cosine, sine, layout) -> out``           (reference nn/rope.py:35-51)
* ``rope_backward(dy, cosine, sine, layout) -> dx``
* ``rope_qk(q, k, cosine, sine, layout) -> (q_out, k_out)``  (query and key in one launch,
  reference nn/rope.py:70-107) and ``rope_qk_backward``

All ops run only on CUDA tensors of a compute-capability-10.0 device and launch on the
current stream of the tensors' device. Any failure raises the reference's exception
type for that op (``Triton*Unavailable``); there is no fallback path.
"""

from __future__ import annotations

import torch
from torch import Tensor

from picotron_b200 import _capi
from picotron_b200.errors import (
    TritonCrossEntropyUnavailable,
    TritonRMSNormUnavailable,
    TritonRoPEUnavailable,
    TritonSwiGLUUnavailable,
)

DTYPE_CODES = {
    torch.float32: _capi.PT_FLOAT32,
    torch.float16: _capi.PT_FLOAT16,
    torch.bfloat16: _capi.PT_BFLOAT16,
}

# RMSNorm (x dtype, weight dtype) pairs built into the library. Other weight dtypes are
# converted to float32 (an exact widening for fp16/bf16) before the call.
_RMSNORM_PAIRS = {
    (torch.float32, torch.float32),
    (torch.float16, torch.float16),
    (torch.float16, torch.float32),
    (torch.bfloat16, torch.bfloat16),
    (torch.bfloat16, torch.float32),
}

LAYOUTS = {"interleaved": _capi.PT_ROPE_INTERLEAVED, "rotate_half": _capi.PT_ROPE_ROTATE_HALF}

_device_ok: dict[int, bool] = {}


def check_device(device: torch.device, error_type: type[Exception]) -> None:
    """Raise ``error_type`` unless ``device`` is a CUDA device this library can run on."""

    if device.type != "cuda":
        raise error_type(f"requires CUDA tensors; got a tensor on {device}")
    index = device.index if device.index is not None else torch.cuda.current_device()
    ok = _device_ok.get(index)
    if ok is None:
        try:
            status, major, minor, _ = _capi.probe(index)
        except _capi.LibraryUnavailable as error:
            raise error_type(str(error)) from error
        ok = status == _capi.PT_OK
        _device_ok[index] = ok
        if not ok:
            raise error_type(_capi.last_error())
    if not ok:
        raise error_type(f"cuda:{index} is not a compute capability 10.0 (sm_100a) device")


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class _OnDevice:
    """Make ``device`` current for the duration of a C-ABI call (no-op when it is)."""

    __slots__ = ("index", "previous")

    def __init__(self, device: torch.device) -> None:
        self.index = device.index
        self.previous = None

    def __enter__(self) -> None:
        current = torch.cuda.current_device()
        if self.index is not None and current != self.index:
            self.previous = current
            torch.cuda.set_device(self.index)

    def __exit__(self, *exc) -> None:
        if self.previous is not None:
            torch.cuda.set_device(self.previous)


def _dtype_code(t: Tensor, error_type: type[Exception]) -> int:
    code = DTYPE_CODES.get(t.dtype)
    if code is None:
        raise error_type(f"unsupported dtype {t.dtype}; expected float32, float16 or bfloat16")
    return code


def _as_rows(t: Tensor, hidden: int) -> Tensor:
    """View ``t`` as [rows, hidden] with contiguous columns, copying only if impossible."""

    if t.dim() >= 1 and t.stride(-1) == 1:
        try:
            view = t.view(-1, hidden)
            if view.stride(1) == 1:
                return view
        except RuntimeError:
            pass
    return t.contiguous().view(-1, hidden)


# --------------------------------------------------------------------------- RMSNorm --


def _rms_weight(x: Tensor, weight: Tensor) -> Tensor:
    if (x.dtype, weight.dtype) in _RMSNORM_PAIRS:
        return weight.contiguous()
    return weight.to(torch.float32).contiguous()


def _validate_rms(x: Tensor, weight: Tensor) -> int:
    check_device(x.device, TritonRMSNormUnavailable)
    if weight.device != x.device:
        raise TritonRMSNormUnavailable("RMSNorm weight must be on the input's device.")
    if x.dim() < 1 or weight.dim() != 1 or x.size(-1) != weight.numel():
        raise TritonRMSNormUnavailable("RMSNorm hidden size must match the weight size.")
    _dtype_code(x, TritonRMSNormUnavailable)
    _dtype_code(weight, TritonRMSNormUnavailable)
    return x.size(-1)


@torch.library.custom_op("picotron_b200::rms_norm", mutates_args=())
def rms_norm(x: Tensor, weight: Tensor, eps: float) -> Tensor:
    hidden = _validate_rms(x, weight)
    w = _rms_weight(x, weight)
    y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    if x.numel() == 0:
        return y
    xr = _as_rows(x, hidden)
    yr = y.view(-1, hidden)
    with _OnDevice(x.device):
        _capi.rmsnorm_fwd(
            xr.data_ptr(), xr.stride(0), w.data_ptr(), yr.data_ptr(), yr.stride(0), None,
            xr.size(0), hidden, DTYPE_CODES[x.dtype], DTYPE_CODES[w.dtype], float(eps),
            _stream(x.device), TritonRMSNormUnavailable,
        )
    return y


@rms_norm.register_fake
def _rms_norm_fake(x: Tensor, weight: Tensor, eps: float) -> Tensor:
    return torch.empty(x.shape, dtype=x.dtype, device=x.device)


@torch.library.custom_op("picotron_b200::rms_norm_backward", mutates_args=())
def rms_norm_backward(dy: Tensor, x: Tensor, weight: Tensor, eps: float) -> tuple[Tensor, Tensor]:
    hidden = _validate_rms(x, weight)
    if dy.shape != x.shape:
        raise TritonRMSNormUnavailable("RMSNorm grad_output must have the input's shape.")
    if dy.dtype != x.dtype:
        dy = dy.to(x.dtype)
    w = _rms_weight(x, weight)
    dx = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    dw = torch.empty(weight.shape, dtype=weight.dtype, device=x.device)
    xr = _as_rows(x, hidden)
    dyr = _as_rows(dy, hidden)
    dxr = dx.view(-1, hidden)
    rows = xr.size(0)
    x_code, w_code = DTYPE_CODES[x.dtype], DTYPE_CODES[w.dtype]
    with _OnDevice(x.device):
        stream = _stream(x.device)
        num_partials = _capi.rmsnorm_bwd_num_partials(rows, hidden, x_code, w_code,
                                                      TritonRMSNormUnavailable)
        partials = torch.empty((num_partials, hidden), dtype=torch.float32, device=x.device)
        _capi.rmsnorm_bwd(
            dyr.data_ptr(), dyr.stride(0), xr.data_ptr(), xr.stride(0), w.data_ptr(), None,
            dxr.data_ptr(), dxr.stride(0), partials.data_ptr(), num_partials, rows, hidden,
            x_code, w_code, float(eps), stream, TritonRMSNormUnavailable,
        )
        _capi.rmsnorm_dw_reduce(partials.data_ptr(), num_partials, hidden, dw.data_ptr(),
                                DTYPE_CODES[dw.dtype], stream, TritonRMSNormUnavailable)
    return dx, dw


@rms_norm_backward.register_fake
def _rms_norm_backward_fake(dy: Tensor, x: Tensor, weight: Tensor, eps: float):
    return (torch.empty(x.shape, dtype=x.dtype, device=x.device),
            torch.empty(weight.shape, dtype=weight.dtype, device=x.device))


def _rms_setup(ctx, inputs, output) -> None:
    x, weight, eps = inputs
    ctx.save_for_backward(x, weight)
    ctx.eps = eps


def _rms_backward(ctx, grad: Tensor):
    x, weight = ctx.saved_tensors
    dx, dw = torch.ops.picotron_b200.rms_norm_backward(grad, x, weight, ctx.eps)
    return dx, dw, None


rms_norm.register_autograd(_rms_backward, setup_context=_rms_setup)


def _validate_add_rms(residual: Tensor, branch: Tensor, weight: Tensor) -> int:
    hidden = _validate_rms(residual, weight)
    if branch.device != residual.device:
        raise TritonRMSNormUnavailable("residual and branch must be on the same device.")
    if branch.shape != residual.shape or branch.dtype != residual.dtype:
        raise TritonRMSNormUnavailable(
            "fused add + RMSNorm requires residual and branch of the same shape and dtype.")
    return hidden


@torch.library.custom_op("picotron_b200::add_rms_norm", mutates_args=())
def add_rms_norm(residual: Tensor, branch: Tensor, weight: Tensor,
                 eps: float) -> tuple[Tensor, Tensor]:
    hidden = _validate_add_rms(residual, branch, weight)
    w = _rms_weight(residual, weight)
    h = torch.empty(residual.shape, dtype=residual.dtype, device=residual.device)
    y = torch.empty(residual.shape, dtype=residual.dtype, device=residual.device)
    if residual.numel() == 0:
        return h, y
    rr, br = _as_rows(residual, hidden), _as_rows(branch, hidden)
    hr, yr = h.view(-1, hidden), y.view(-1, hidden)
    with _OnDevice(residual.device):
        _capi.add_rmsnorm_fwd(
            rr.data_ptr(), rr.stride(0), br.data_ptr(), br.stride(0), w.data_ptr(),
            hr.data_ptr(), hr.stride(0), yr.data_ptr(), yr.stride(0), None, rr.size(0), hidden,
            DTYPE_CODES[residual.dtype], DTYPE_CODES[w.dtype], float(eps),
            _stream(residual.device), TritonRMSNormUnavailable,
        )
    return h, y


@add_rms_norm.register_fake
def _add_rms_norm_fake(residual: Tensor, branch: Tensor, weight: Tensor, eps: float):
    return (torch.empty(residual.shape, dtype=residual.dtype, device=residual.device),
            torch.empty(residual.shape, dtype=residual.dtype, device=residual.device))


@torch.library.custom_op("picotron_b200::add_rms_norm_backward", mutates_args=())
def add_rms_norm_backward(dy: Tensor, dh: Tensor | None, h: Tensor, weight: Tensor,
                          eps: float) -> tuple[Tensor, Tensor]:
    hidden = _validate_rms(h, weight)
    if dy.shape != h.shape or (dh is not None and dh.shape != h.shape):
        raise TritonRMSNormUnavailable("fused add + RMSNorm gradients must have h's shape.")
    if dy.dtype != h.dtype:
        dy = dy.to(h.dtype)
    if dh is not None and dh.dtype != h.dtype:
        dh = dh.to(h.dtype)
    w = _rms_weight(h, weight)
    dx = torch.empty(h.shape, dtype=h.dtype, device=h.device)
    dw = torch.empty(weight.shape, dtype=weight.dtype, device=h.device)
    hr, dyr, dxr = _as_rows(h, hidden), _as_rows(dy, hidden), dx.view(-1, hidden)
    dhr = _as_rows(dh, hidden) if dh is not None else None
    rows = hr.size(0)
    x_code, w_code = DTYPE_CODES[h.dtype], DTYPE_CODES[w.dtype]
    with _OnDevice(h.device):
        stream = _stream(h.device)
        num_partials = _capi.add_rmsnorm_bwd_num_partials(rows, hidden, x_code, w_code,
                                                          TritonRMSNormUnavailable)
        partials = torch.empty((num_partials, hidden), dtype=torch.float32, device=h.device)
        _capi.add_rmsnorm_bwd(
            dyr.data_ptr(), dyr.stride(0), dhr.data_ptr() if dhr is not None else None,
            dhr.stride(0) if dhr is not None else 0, hr.data_ptr(), hr.stride(0), w.data_ptr(),
            None, dxr.data_ptr(), dxr.stride(0), partials.data_ptr(), num_partials, rows,
            hidden, x_code, w_code, float(eps), stream, TritonRMSNormUnavailable,
        )
        _capi.rmsnorm_dw_reduce(partials.data_ptr(), num_partials, hidden, dw.data_ptr(),
                                DTYPE_CODES[dw.dtype], stream, TritonRMSNormUnavailable)
    return dx, dw


@add_rms_norm_backward.register_fake
def _add_rms_norm_backward_fake(dy, dh, h, weight, eps):
    return (torch.empty(h.shape, dtype=h.dtype, device=h.device),
            torch.empty(weight.shape, dtype=weight.dtype, device=h.device))


def _add_rms_setup(ctx, inputs, output) -> None:
    _, _, weight, eps = inputs
    h, _ = output
    ctx.save_for_backward(h, weight)
    ctx.eps = eps


def _add_rms_backward(ctx, grad_h, grad_y):
    h, weight = ctx.saved_tensors
    if grad_y is None:
        grad_y = torch.zeros_like(h)
    dx, dw = torch.ops.picotron_b200.add_rms_norm_backward(grad_y, grad_h, h, weight, ctx.eps)
    return dx, dx, dw, None


add_rms_norm.register_autograd(_add_rms_backward, setup_context=_add_rms_setup)


# ---------------------------------------------------------------------------- SwiGLU --


def _validate_swiglu(gate: Tensor, up: Tensor) -> None:
    check_device(gate.device, TritonSwiGLUUnavailable)
    if up.device != gate.device:
        raise TritonSwiGLUUnavailable("SwiGLU gate and up must be on the same device.")
    if gate.shape != up.shape or gate.dtype != up.dtype:
        raise TritonSwiGLUUnavailable("SwiGLU requires gate and up of the same shape and dtype.")
    _dtype_code(gate, TritonSwiGLUUnavailable)


@torch.library.custom_op("picotron_b200::swiglu", mutates_args=())
def swiglu(gate: Tensor, up: Tensor) -> Tensor:
    _validate_swiglu(gate, up)
    g, u = gate.contiguous(), up.contiguous()
    out = torch.empty(gate.shape, dtype=gate.dtype, device=gate.device)
    if gate.numel() == 0:
        return out
    with _OnDevice(gate.device):
        _capi.swiglu_fwd(g.data_ptr(), u.data_ptr(), out.data_ptr(), g.numel(),
                         DTYPE_CODES[g.dtype], _stream(gate.device), TritonSwiGLUUnavailable)
    return out


@swiglu.register_fake
def _swiglu_fake(gate: Tensor, up: Tensor) -> Tensor:
    return torch.empty(gate.shape, dtype=gate.dtype, device=gate.device)


@torch.library.custom_op("picotron_b200::swiglu_backward", mutates_args=())
def swiglu_backward(dout: Tensor, gate: Tensor, up: Tensor) -> tuple[Tensor, Tensor]:
    _validate_swiglu(gate, up)
    if dout.shape != gate.shape:
        raise TritonSwiGLUUnavailable("SwiGLU grad_output must have the input's shape.")
    if dout.dtype != gate.dtype:
        dout = dout.to(gate.dtype)
    o, g, u = dout.contiguous(), gate.contiguous(), up.contiguous()
    dg = torch.empty(gate.shape, dtype=gate.dtype, device=gate.device)
    du = torch.empty(gate.shape, dtype=gate.dtype, device=gate.device)
    if gate.numel() == 0:
        return dg, du
    with _OnDevice(gate.device):
        _capi.swiglu_bwd(o.data_ptr(), g.data_ptr(), u.data_ptr(), dg.data_ptr(), du.data_ptr(),
                         g.numel(), DTYPE_CODES[g.dtype], _stream(gate.device),
                         TritonSwiGLUUnavailable)
    return dg, du


@swiglu_backward.register_fake
def _swiglu_backward_fake(dout: Tensor, gate: Tensor, up: Tensor):
    return (torch.empty(gate.shape, dtype=gate.dtype, device=gate.device),
            torch.empty(gate.shape, dtype=gate.dtype, device=gate.device))


def _swiglu_setup(ctx, inputs, output) -> None:
    gate, up = inputs
    ctx.save_for_backward(gate, up)


def _swiglu_bwd(ctx, grad: Tensor):
    gate, up = ctx.saved_tensors
    dg, du = torch.ops.picotron_b200.swiglu_backward(grad, gate, up)
    return dg, du


swiglu.register_autograd(_swiglu_bwd, setup_context=_swiglu_setup)


def _validate_gate_up(x: Tensor, w_gate: Tensor, w_up: Tensor) -> tuple[int, int]:
    check_device(x.device, TritonSwiGLUUnavailable)
    if w_gate.device != x.device or w_up.device != x.device:
        raise TritonSwiGLUUnavailable("x, w_gate and w_up must be on the same device.")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise TritonSwiGLUUnavailable(
            f"the fused gate/up GEMM takes bfloat16 or float16 inputs, not {x.dtype}")
    if w_gate.dtype != x.dtype or w_up.dtype != x.dtype:
        raise TritonSwiGLUUnavailable("w_gate and w_up must have the dtype of x.")
    if (x.dim() < 1 or w_gate.dim() != 2 or w_gate.shape != w_up.shape
            or w_gate.size(1) != x.size(-1)):
        raise TritonSwiGLUUnavailable("expected x [..., k] and w_gate, w_up [n, k].")
    return w_gate.size(0), x.size(-1)


@torch.library.custom_op("picotron_b200::swiglu_gate_up", mutates_args=())
def swiglu_gate_up(x: Tensor, w_gate: Tensor, w_up: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    n, k = _validate_gate_up(x, w_gate, w_up)
    out_shape = (*x.shape[:-1], n)
    act = torch.empty(out_shape, dtype=x.dtype, device=x.device)
    gate = torch.empty(out_shape, dtype=x.dtype, device=x.device)
    up = torch.empty(out_shape, dtype=x.dtype, device=x.device)
    if act.numel() == 0:
        return act, gate, up
    x2 = _as_rows(x, k)
    if x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    wg, wu = w_gate.contiguous(), w_up.contiguous()
    with _OnDevice(x.device):
        _capi.swiglu_gemm_fwd(
            x2.data_ptr(), x2.stride(0), wg.data_ptr(), wu.data_ptr(), k, act.data_ptr(), n,
            gate.data_ptr(), up.data_ptr(), n, x2.size(0), n, k, DTYPE_CODES[x.dtype],
            _stream(x.device), TritonSwiGLUUnavailable,
        )
    return act, gate, up


@swiglu_gate_up.register_fake
def _swiglu_gate_up_fake(x: Tensor, w_gate: Tensor, w_up: Tensor):
    shape = (*x.shape[:-1], w_gate.size(0))
    return tuple(torch.empty(shape, dtype=x.dtype, device=x.device) for _ in range(3))


def _gate_up_setup(ctx, inputs, output) -> None:
    x, w_gate, w_up = inputs
    _, gate, up = output
    ctx.save_for_backward(x, w_gate, w_up, gate, up)
    ctx.set_materialize_grads(False)


def _gate_up_backward(ctx, d_act, d_gate, d_up):
    # dgate, dup from the fused activation backward, then the projections' backward as
    # plain library GEMMs (reference: autograd of the two nn.Linear, feedforward.py:27-28).
    x, w_gate, w_up, gate, up = ctx.saved_tensors
    n, k = w_gate.shape
    if d_act is not None:
        dg, du = torch.ops.picotron_b200.swiglu_backward(d_act, gate, up)
    else:
        dg, du = torch.zeros_like(gate), torch.zeros_like(up)
    if d_gate is not None:
        dg = dg + d_gate
    if d_up is not None:
        du = du + d_up
    x2, dg2, du2 = x.reshape(-1, k), dg.reshape(-1, n), du.reshape(-1, n)
    dx = (dg2 @ w_gate).addmm_(du2, w_up).reshape(x.shape)
    return dx, dg2.t() @ x2, du2.t() @ x2


swiglu_gate_up.register_autograd(_gate_up_backward, setup_context=_gate_up_setup)


def fused_down_backward_supported(x: Tensor, w_down: Tensor) -> bool:
    """True when pt_swiglu_gemm_bwd takes the MLP's shapes (intermediate size a multiple of
    64, hidden size a multiple of 8)."""

    return w_down.dim() == 2 and w_down.size(1) % 64 == 0 and w_down.size(0) % 8 == 0


@torch.library.custom_op("picotron_b200::swiglu_down_backward", mutates_args=())
def swiglu_down_backward(d_out: Tensor, w_down: Tensor, gate: Tensor,
                         up: Tensor) -> tuple[Tensor, Tensor]:
    """(dgate, dup) from the down projection's output gradient: d_act = d_out @ w_down and
    the SwiGLU backward in one tcgen05 GEMM (pt_swiglu_gemm_bwd); d_act stays on chip."""

    check_device(d_out.device, TritonSwiGLUUnavailable)
    if not (d_out.dtype == w_down.dtype == gate.dtype == up.dtype) or d_out.dtype not in (
            torch.bfloat16, torch.float16):
        raise TritonSwiGLUUnavailable("the fused down-projection backward takes one dtype, "
                                      "bfloat16 or float16")
    k, n = w_down.shape
    if (d_out.size(-1) != k or gate.shape != up.shape or gate.size(-1) != n
            or gate.shape[:-1] != d_out.shape[:-1]):
        raise TritonSwiGLUUnavailable("expected d_out [..., k], w_down [k, n], gate, up [..., n]")
    dgate = torch.empty(gate.shape, dtype=gate.dtype, device=gate.device)
    dup = torch.empty(gate.shape, dtype=gate.dtype, device=gate.device)
    if dgate.numel() == 0:
        return dgate, dup
    d2 = _as_rows(d_out, k)
    if d2.stride(0) % 8 or d2.data_ptr() % 16:
        d2 = d2.contiguous()
    g2, u2 = gate.reshape(-1, n).contiguous(), up.reshape(-1, n).contiguous()
    wd = w_down.contiguous()
    wdt = torch.empty((n, k), dtype=wd.dtype, device=wd.device)  # both operands read along k
    with _OnDevice(d_out.device):
        _capi.transpose_2d(wd.data_ptr(), wd.stride(0), wdt.data_ptr(), k, k, n,
                           DTYPE_CODES[wd.dtype], _stream(d_out.device), TritonSwiGLUUnavailable)
        _capi.swiglu_gemm_bwd(
            d2.data_ptr(), d2.stride(0), wdt.data_ptr(), k, g2.data_ptr(), u2.data_ptr(), n,
            dgate.data_ptr(), dup.data_ptr(), n, None, 0, d2.size(0), n, k,
            DTYPE_CODES[d_out.dtype], _stream(d_out.device), TritonSwiGLUUnavailable,
        )
    return dgate, dup


@swiglu_down_backward.register_fake
def _swiglu_down_backward_fake(d_out, w_down, gate, up):
    return (torch.empty(gate.shape, dtype=gate.dtype, device=gate.device),
            torch.empty(gate.shape, dtype=gate.dtype, device=gate.device))


class _SwiGLUMLP(torch.autograd.Function):
    """down_projection(silu(gate_projection(x)) * up_projection(x)) without biases (reference
    SwiGLU.forward, feedforward.py:27-43). Forward: the gate/up GEMMs with the activation in
    their epilogue, then the down projection (library GEMM). Backward: the down projection's
    weight gradient (library GEMM), its input gradient with the activation's backward in the
    epilogue (pt_swiglu_gemm_bwd), then the gate/up projections' gradients (library GEMMs)."""

    @staticmethod
    def forward(ctx, x, w_gate, w_up, w_down):
        act, gate, up = torch.ops.picotron_b200.swiglu_gate_up(x, w_gate, w_up)
        ctx.save_for_backward(x, w_gate, w_up, w_down, act, gate, up)
        return torch.nn.functional.linear(act, w_down)

    @staticmethod
    def backward(ctx, d_out):
        x, w_gate, w_up, w_down, act, gate, up = ctx.saved_tensors
        n, k = w_gate.shape
        d_out = d_out.to(x.dtype)
        d2 = d_out.reshape(-1, w_down.size(0))
        dw_down = d2.t() @ act.reshape(-1, n)
        dg, du = torch.ops.picotron_b200.swiglu_down_backward(d_out, w_down, gate, up)
        x2, dg2, du2 = x.reshape(-1, k), dg.reshape(-1, n), du.reshape(-1, n)
        dx = (dg2 @ w_gate).addmm_(du2, w_up).reshape(x.shape)
        return dx, dg2.t() @ x2, du2.t() @ x2, dw_down


def swiglu_mlp(x: Tensor, w_gate: Tensor, w_up: Tensor, w_down: Tensor) -> Tensor:
    """The SwiGLU MLP with both activation passes fused into tensor-core GEMMs."""

    return _SwiGLUMLP.apply(x, w_gate, w_up, w_down)


# --------------------------------------------------------------------- cross-entropy --


def _ce_geometry(logits: Tensor, targets: Tensor):
    """(outer, inner, logits strides, targets strides) of F.cross_entropy's layouts:
    logits [N, V] with targets [N], or logits [B, V, S] with targets [B, S] (class dim 1,
    which must have unit stride)."""

    if logits.dim() == 2 and targets.dim() == 1 and targets.size(0) == logits.size(0):
        return logits.size(0), 1, (logits.stride(0), 0), (targets.stride(0), 0)
    if (logits.dim() == 3 and targets.dim() == 2 and targets.size(0) == logits.size(0)
            and targets.size(1) == logits.size(2)):
        return (logits.size(0), logits.size(2), (logits.stride(0), logits.stride(2)),
                (targets.stride(0), targets.stride(1)))
    raise TritonCrossEntropyUnavailable(
        "cross-entropy expects logits [N, V] with targets [N], or [B, V, S] with targets [B, S]")


def _ce_inputs(logits: Tensor, targets: Tensor) -> tuple[Tensor, Tensor]:
    check_device(logits.device, TritonCrossEntropyUnavailable)
    if targets.device != logits.device:
        raise TritonCrossEntropyUnavailable("logits and targets must be on the same device.")
    if targets.dtype != torch.long:
        raise TritonCrossEntropyUnavailable("cross-entropy targets must be int64 class indices.")
    _dtype_code(logits, TritonCrossEntropyUnavailable)
    if logits.dim() not in (2, 3) or logits.stride(1) != 1:
        # The class dimension must be contiguous: move it last (one copy).
        if logits.dim() in (2, 3):
            logits = logits.movedim(1, -1).contiguous().movedim(-1, 1)
    return logits, targets


@torch.library.custom_op("picotron_b200::cross_entropy", mutates_args=())
def cross_entropy(logits: Tensor, targets: Tensor,
                  ignore_index: int) -> tuple[Tensor, Tensor, Tensor]:
    logits, targets = _ce_inputs(logits, targets)
    outer, inner, lstr, tstr = _ce_geometry(logits, targets)
    rows = outer * inner
    row_loss = torch.empty(rows, dtype=torch.float32, device=logits.device)
    row_lse = torch.empty(rows, dtype=torch.float32, device=logits.device)
    mean_out = torch.empty(2, dtype=torch.float32, device=logits.device)
    with _OnDevice(logits.device):
        _capi.cross_entropy_fwd(
            logits.data_ptr(), logits.size(1), outer, inner, lstr, targets.data_ptr(), tstr,
            int(ignore_index), row_loss.data_ptr(), row_lse.data_ptr(), mean_out.data_ptr(),
            DTYPE_CODES[logits.dtype], _stream(logits.device), TritonCrossEntropyUnavailable,
        )
    return mean_out[0].clone(), row_lse, mean_out


@cross_entropy.register_fake
def _cross_entropy_fake(logits: Tensor, targets: Tensor, ignore_index: int):
    rows = targets.numel()
    return (torch.empty((), dtype=torch.float32, device=logits.device),
            torch.empty(rows, dtype=torch.float32, device=logits.device),
            torch.empty(2, dtype=torch.float32, device=logits.device))


@torch.library.custom_op("picotron_b200::cross_entropy_backward", mutates_args=())
def cross_entropy_backward(grad: Tensor, logits: Tensor, targets: Tensor, row_lse: Tensor,
                           mean_out: Tensor, ignore_index: int) -> Tensor:
    logits_c, targets = _ce_inputs(logits, targets)
    outer, inner, lstr, tstr = _ce_geometry(logits_c, targets)
    vocab = logits_c.size(1)
    # Class dimension innermost in memory: [N, V], or [B, S, V] seen as [B, V, S].
    if logits.dim() == 2:
        dlogits = torch.empty((outer, vocab), dtype=logits.dtype, device=logits.device)
        dstr = (dlogits.stride(0), 0)
    else:
        buf = torch.empty((outer, inner, vocab), dtype=logits.dtype, device=logits.device)
        dlogits = buf.transpose(1, 2)
        dstr = (buf.stride(0), buf.stride(1))
    if outer * inner == 0:
        return dlogits
    g = grad.to(torch.float32).contiguous()
    with _OnDevice(logits.device):
        _capi.cross_entropy_bwd(
            logits_c.data_ptr(), vocab, outer, inner, lstr, targets.data_ptr(), tstr,
            int(ignore_index), row_lse.data_ptr(), mean_out.data_ptr(), g.data_ptr(),
            dlogits.data_ptr(), dstr, DTYPE_CODES[logits.dtype], _stream(logits.device),
            TritonCrossEntropyUnavailable,
        )
    return dlogits


@cross_entropy_backward.register_fake
def _cross_entropy_backward_fake(grad, logits, targets, row_lse, mean_out, ignore_index):
    return torch.empty_like(logits)


def _ce_setup(ctx, inputs, output) -> None:
    logits, targets, ignore_index = inputs
    _, row_lse, mean_out = output
    ctx.save_for_backward(logits, targets, row_lse, mean_out)
    ctx.ignore_index = ignore_index
    ctx.set_materialize_grads(False)


def _ce_backward(ctx, grad, _grad_lse, _grad_mean):
    logits, targets, row_lse, mean_out = ctx.saved_tensors
    if grad is None:
        return None, None, None
    dlogits = torch.ops.picotron_b200.cross_entropy_backward(grad, logits, targets, row_lse,
                                                             mean_out, ctx.ignore_index)
    return dlogits, None, None


cross_entropy.register_autograd(_ce_backward, setup_context=_ce_setup)


# ------------------------------------------------------------------------------ RoPE --


def _validate_rope(x: Tensor, cosine: Tensor, sine: Tensor, layout: int) -> None:
    check_device(x.device, TritonRoPEUnavailable)
    if cosine.device != x.device or sine.device != x.device:
        raise TritonRoPEUnavailable("RoPE tables must be on the states' device.")
    if layout not in (_capi.PT_ROPE_INTERLEAVED, _capi.PT_ROPE_ROTATE_HALF):
        raise TritonRoPEUnavailable(f"unknown RoPE layout {layout}")
    if (
        x.dim() != 4
        or x.size(-1) % 2 != 0
        or cosine.dim() != 2
        or cosine.shape != sine.shape
        or cosine.size(-1) * 2 != x.size(-1)
        or cosine.size(0) != x.size(-2)
        or cosine.dtype != sine.dtype
    ):
        raise TritonRoPEUnavailable(
            "RoPE requires states [B, H, S, D] and cosine/sine tables [S, D/2] of one dtype."
        )
    _dtype_code(x, TritonRoPEUnavailable)
    _dtype_code(cosine, TritonRoPEUnavailable)


def _rope_launch(direction: str, x: Tensor, cosine: Tensor, sine: Tensor, layout: int) -> Tensor:
    _validate_rope(x, cosine, sine, layout)
    if x.stride(-1) != 1:
        x = x.contiguous()
    if cosine.stride(-1) != 1 or sine.stride(-1) != 1 or cosine.stride(0) != sine.stride(0):
        cosine, sine = cosine.contiguous(), sine.contiguous()
    table = cosine if cosine.dtype in (x.dtype, torch.float32) else None
    if table is None:
        cosine, sine = cosine.to(torch.float32), sine.to(torch.float32)
    # Same memory layout as the input when it is dense (e.g. the [B,S,H,D] memory of a
    # transposed attention view), else contiguous.
    out = torch.empty_like(x)
    if out.stride(-1) != 1:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    if x.numel() == 0:
        return out
    with _OnDevice(x.device):
        _capi.rope(direction, x.data_ptr(), x.stride(), out.data_ptr(), out.stride(),
                   x.shape, cosine.data_ptr(), sine.data_ptr(), cosine.stride(0), layout,
                   DTYPE_CODES[x.dtype], DTYPE_CODES[cosine.dtype], _stream(x.device),
                   TritonRoPEUnavailable)
    return out


@torch.library.custom_op("picotron_b200::rope", mutates_args=())
def rope(x: Tensor, cosine: Tensor, sine: Tensor, layout: int) -> Tensor:
    return _rope_launch("fwd", x, cosine, sine, layout)


@rope.register_fake
def _rope_fake(x: Tensor, cosine: Tensor, sine: Tensor, layout: int) -> Tensor:
    out = torch.empty_like(x)
    return out if out.stride(-1) == 1 else torch.empty(x.shape, dtype=x.dtype, device=x.device)


@torch.library.custom_op("picotron_b200::rope_backward", mutates_args=())
def rope_backward(dy: Tensor, cosine: Tensor, sine: Tensor, layout: int) -> Tensor:
    return _rope_launch("bwd", dy, cosine, sine, layout)


@rope_backward.register_fake
def _rope_backward_fake(dy: Tensor, cosine: Tensor, sine: Tensor, layout: int) -> Tensor:
    out = torch.empty_like(dy)
    return out if out.stride(-1) == 1 else torch.empty(dy.shape, dtype=dy.dtype, device=dy.device)


def _rope_setup(ctx, inputs, output) -> None:
    x, cosine, sine, layout = inputs
    ctx.save_for_backward(cosine, sine)
    ctx.layout = layout


def _rope_bwd(ctx, grad: Tensor):
    cosine, sine = ctx.saved_tensors
    dx = torch.ops.picotron_b200.rope_backward(grad, cosine, sine, ctx.layout)
    # The angle tables are constants of the position grid: no gradient flows to them.
    return dx, None, None, None


rope.register_autograd(_rope_bwd, setup_context=_rope_setup)


def _rope_prepare(x: Tensor, cosine: Tensor, sine: Tensor, layout: int):
    _validate_rope(x, cosine, sine, layout)
    if x.stride(-1) != 1:
        x = x.contiguous()
    out = torch.empty_like(x)
    if out.stride(-1) != 1:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    return x, out


def _rope_qk_launch(direction: str, q: Tensor, k: Tensor, cosine: Tensor, sine: Tensor,
                    layout: int) -> tuple[Tensor, Tensor]:
    if q.dtype != k.dtype or q.device != k.device:
        raise TritonRoPEUnavailable("query and key must share dtype and device.")
    q, q_out = _rope_prepare(q, cosine, sine, layout)
    k, k_out = _rope_prepare(k, cosine, sine, layout)
    if cosine.stride(-1) != 1 or sine.stride(-1) != 1 or cosine.stride(0) != sine.stride(0):
        cosine, sine = cosine.contiguous(), sine.contiguous()
    if cosine.dtype not in (q.dtype, torch.float32):
        cosine, sine = cosine.to(torch.float32), sine.to(torch.float32)
    if q.numel() == 0 and k.numel() == 0:
        return q_out, k_out
    with _OnDevice(q.device):
        _capi.rope_qk(direction, q.data_ptr(), q.stride(), q_out.data_ptr(), q_out.stride(),
                      q.shape, k.data_ptr(), k.stride(), k_out.data_ptr(), k_out.stride(),
                      k.shape, cosine.data_ptr(), sine.data_ptr(), cosine.stride(0), layout,
                      DTYPE_CODES[q.dtype], DTYPE_CODES[cosine.dtype], _stream(q.device),
                      TritonRoPEUnavailable)
    return q_out, k_out


@torch.library.custom_op("picotron_b200::rope_qk", mutates_args=())
def rope_qk(q: Tensor, k: Tensor, cosine: Tensor, sine: Tensor,
            layout: int) -> tuple[Tensor, Tensor]:
    return _rope_qk_launch("fwd", q, k, cosine, sine, layout)


def _rope_qk_fake(q, k, cosine, sine, layout):
    return _rope_fake(q, cosine, sine, layout), _rope_fake(k, cosine, sine, layout)


rope_qk.register_fake(_rope_qk_fake)


@torch.library.custom_op("picotron_b200::rope_qk_backward", mutates_args=())
def rope_qk_backward(dq: Tensor, dk: Tensor, cosine: Tensor, sine: Tensor,
                     layout: int) -> tuple[Tensor, Tensor]:
    return _rope_qk_launch("bwd", dq, dk, cosine, sine, layout)


rope_qk_backward.register_fake(_rope_qk_fake)


def _rope_qk_setup(ctx, inputs, output) -> None:
    q, k, cosine, sine, layout = inputs
    ctx.save_for_backward(cosine, sine)
    ctx.layout = layout
    ctx.q_meta = (q.shape, q.dtype, q.device)
    ctx.k_meta = (k.shape, k.dtype, k.device)
    ctx.set_materialize_grads(False)


def _rope_qk_bwd(ctx, dq: Tensor | None, dk: Tensor | None):
    cosine, sine = ctx.saved_tensors
    if dq is None:
        dq = torch.zeros(ctx.q_meta[0], dtype=ctx.q_meta[1], device=ctx.q_meta[2])
    if dk is None:
        dk = torch.zeros(ctx.k_meta[0], dtype=ctx.k_meta[1], device=ctx.k_meta[2])
    gq, gk = torch.ops.picotron_b200.rope_qk_backward(dq, dk, cosine, sine, ctx.layout)
    return gq, gk, None, None, None


rope_qk.register_autograd(_rope_qk_bwd, setup_context=_rope_qk_setup)
