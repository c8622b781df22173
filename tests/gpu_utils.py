"""Helpers for the ``-m gpu`` tests: seeded inputs and direct C-ABI calls on torch buffers.

The wrappers below call the library's C entry points (through ``picotron_b200._capi``)
with raw device addresses, exactly as a non-Python caller of ``include/picotron_b200.h``
would; they allocate outputs with torch only for convenience.
"""

from __future__ import annotations

import torch

from picotron_b200 import _capi
from picotron_b200.ops import DTYPE_CODES

DEV = torch.device("cuda", 0)


def require_gpu() -> None:
    """GPU tests fail (not skip) when no usable device or library is present."""

    assert torch.cuda.is_available(), "the gpu tests need a CUDA device"
    status, major, minor, sms = _capi.probe(0)
    assert status == _capi.PT_OK, f"device 0 rejected by pt_probe: {_capi.last_error()}"


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


# Bounds on the ulp statistics of a full-size 16-bit output against the float64 oracle.
# An output computed in fp32 and rounded once, with no cancelling subtraction (RMSNorm y,
# SwiGLU out and dup), is within half an ulp plus a few fp32 ulps: max_ulp <= 1. Where the
# formula subtracts nearly equal terms (RMSNorm dx, SwiGLU dgate near 1 + g(1 - s) = 0,
# RoPE e*c - o*s, GEMM sums), fp32 evaluation error of about 2^-23 of the terms exceeds 2
# ulp of the result only when |result| < about 2^-16 of the terms: a few elements in 10^5
# for these distributions, which the tolerance's 2^-16 max floor admits. Those are counted
# (floor_only) and bounded here.
# A GEMM output is a sum of K products accumulated in fp32: its error is about
# sqrt(K) * 2^-24 of the sum of |terms|, so at K = 4096 the outputs smaller than about
# 2^-10 of that sum (about one in 10^4 for these inputs) exceed 2 ulp, inside the floor.
MAX_ULP_ROUNDED_ONCE = 1.0
MAX_FRAC_OVER_2ULP_CANCELLING = 1e-4
MAX_FRAC_OVER_2ULP_GEMM_K4096 = 1e-3


def full_size_parity(out: torch.Tensor, exact: torch.Tensor, what: str, cancels: bool,
                     dtype: torch.dtype | None = None,
                     max_frac_over_2ulp: float = MAX_FRAC_OVER_2ULP_CANCELLING):
    """assert_close plus the ulp statistics of a full-size output: asserts the bounds above
    for 16-bit outputs and appends one JSON line per output to $PT_PARITY_LOG when set."""

    import json
    import os

    from oracle import tolerance

    r = tolerance.assert_close(out, exact, what, dtype)
    dt = dtype or out.dtype
    rec = {"what": what, "dtype": str(dt).replace("torch.", ""), "numel": r.numel,
           "max_abs": r.max_abs, "max_ulp": r.max_ulp, "frac_over_2ulp": r.frac_over_2ulp,
           "floor_only": r.floor_only, "cancels": cancels}
    path = os.environ.get("PT_PARITY_LOG")
    if path:
        with open(path, "a") as fh:
            fh.write(json.dumps(rec) + "\n")
    if dt != torch.float32:
        if cancels:
            assert r.frac_over_2ulp <= max_frac_over_2ulp, f"{what}: {r}"
        else:
            assert r.max_ulp <= MAX_ULP_ROUNDED_ONCE and r.floor_only == 0, f"{what}: {r}"
    return r


def randn(shape, seed: int, dtype=torch.float32, scale: float = 1.0, shift: float = 0.0,
          device=DEV) -> torch.Tensor:
    """N(shift, scale^2) drawn on CPU in fp32 from a seeded generator, then cast (so CPU
    and GPU tests see identical bits)."""

    g = torch.Generator().manual_seed(seed)
    t = torch.randn(shape, generator=g) * scale + shift
    return t.to(dtype).to(device)


def rmsnorm_fwd(x2d: torch.Tensor, w: torch.Tensor, eps: float, want_rstd: bool = False):
    rows, hidden = x2d.shape
    y = torch.empty((rows, hidden), dtype=x2d.dtype, device=x2d.device)
    rstd = torch.empty(rows, dtype=torch.float32, device=x2d.device) if want_rstd else None
    _capi.rmsnorm_fwd(x2d.data_ptr(), x2d.stride(0), w.data_ptr(), y.data_ptr(), y.stride(0),
                      rstd.data_ptr() if rstd is not None else None, rows, hidden,
                      DTYPE_CODES[x2d.dtype], DTYPE_CODES[w.dtype], eps, stream())
    return (y, rstd) if want_rstd else y


def rmsnorm_bwd(dy2d, x2d, w, eps, num_partials=None, rstd=None, return_partials=False):
    rows, hidden = x2d.shape
    xc, wc = DTYPE_CODES[x2d.dtype], DTYPE_CODES[w.dtype]
    if num_partials is None:
        num_partials = _capi.rmsnorm_bwd_num_partials(rows, hidden, xc, wc)
    dx = torch.empty((rows, hidden), dtype=x2d.dtype, device=x2d.device)
    partials = torch.full((num_partials, hidden), float("nan"), dtype=torch.float32,
                          device=x2d.device)
    dw = torch.empty(hidden, dtype=w.dtype, device=x2d.device)
    _capi.rmsnorm_bwd(dy2d.data_ptr(), dy2d.stride(0), x2d.data_ptr(), x2d.stride(0),
                      w.data_ptr(), rstd.data_ptr() if rstd is not None else None,
                      dx.data_ptr(), dx.stride(0), partials.data_ptr(), num_partials, rows,
                      hidden, xc, wc, eps, stream())
    _capi.rmsnorm_dw_reduce(partials.data_ptr(), num_partials, hidden, dw.data_ptr(),
                            DTYPE_CODES[w.dtype], stream())
    if return_partials:
        return dx, dw, partials
    return dx, dw


def swiglu_fwd(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(g)
    _capi.swiglu_fwd(g.data_ptr(), u.data_ptr(), out.data_ptr(), g.numel(), DTYPE_CODES[g.dtype],
                     stream())
    return out


def swiglu_bwd(dout, g, u):
    dg, du = torch.empty_like(g), torch.empty_like(g)
    _capi.swiglu_bwd(dout.data_ptr(), g.data_ptr(), u.data_ptr(), dg.data_ptr(), du.data_ptr(),
                     g.numel(), DTYPE_CODES[g.dtype], stream())
    return dg, du


def rope(direction: str, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
         layout: str = "interleaved", out: torch.Tensor | None = None) -> torch.Tensor:
    code = {"interleaved": _capi.PT_ROPE_INTERLEAVED, "rotate_half": _capi.PT_ROPE_ROTATE_HALF}
    if out is None:
        out = torch.empty_like(x)
    _capi.rope(direction, x.data_ptr(), x.stride(), out.data_ptr(), out.stride(), x.shape,
               cos.data_ptr(), sin.data_ptr(), cos.stride(0), code[layout],
               DTYPE_CODES[x.dtype], DTYPE_CODES[cos.dtype], stream())
    return out


def add_rmsnorm_fwd(res2d, br2d, w, eps, h_out=None):
    rows, hidden = res2d.shape
    h = torch.empty_like(res2d) if h_out is None else h_out
    y = torch.empty_like(res2d)
    _capi.add_rmsnorm_fwd(res2d.data_ptr(), res2d.stride(0), br2d.data_ptr(), br2d.stride(0),
                          w.data_ptr(), h.data_ptr(), h.stride(0), y.data_ptr(), y.stride(0),
                          None, rows, hidden, DTYPE_CODES[res2d.dtype], DTYPE_CODES[w.dtype],
                          eps, stream())
    return h, y


def add_rmsnorm_bwd(dy2d, dh2d, h2d, w, eps, num_partials=None, dx_out=None):
    rows, hidden = h2d.shape
    xc, wc = DTYPE_CODES[h2d.dtype], DTYPE_CODES[w.dtype]
    if num_partials is None:
        num_partials = _capi.add_rmsnorm_bwd_num_partials(rows, hidden, xc, wc)
    dx = torch.empty_like(h2d) if dx_out is None else dx_out
    partials = torch.full((num_partials, hidden), float("nan"), dtype=torch.float32,
                          device=h2d.device)
    dw = torch.empty(hidden, dtype=w.dtype, device=h2d.device)
    _capi.add_rmsnorm_bwd(dy2d.data_ptr(), dy2d.stride(0),
                          dh2d.data_ptr() if dh2d is not None else None,
                          dh2d.stride(0) if dh2d is not None else 0, h2d.data_ptr(),
                          h2d.stride(0), w.data_ptr(), None, dx.data_ptr(), dx.stride(0),
                          partials.data_ptr(), num_partials, rows, hidden, xc, wc, eps, stream())
    _capi.rmsnorm_dw_reduce(partials.data_ptr(), num_partials, hidden, dw.data_ptr(), wc,
                            stream())
    return dx, dw


def swiglu_gemm(x2d, wg, wu, save_preact=True):
    m, k = x2d.shape
    n = wg.size(0)
    act = torch.empty((m, n), dtype=x2d.dtype, device=x2d.device)
    g = torch.empty_like(act) if save_preact else None
    u = torch.empty_like(act) if save_preact else None
    _capi.swiglu_gemm_fwd(x2d.data_ptr(), x2d.stride(0), wg.data_ptr(), wu.data_ptr(),
                          wg.stride(0), act.data_ptr(), act.stride(0),
                          g.data_ptr() if save_preact else None,
                          u.data_ptr() if save_preact else None, n, m, n, k,
                          DTYPE_CODES[x2d.dtype], stream())
    return act, g, u


def cross_entropy(logits, targets, ignore_index=-100, grad=None, want_grad=True):
    """C-ABI forward (+ backward) on [N, V] / [N] or [B, V, S] / [B, S] (class stride 1).
    Returns (mean loss, row_loss, dlogits or None); dlogits is dense [N, V] / [B, S, V]
    seen in the logits' layout."""

    if logits.dim() == 2:
        outer, inner = logits.size(0), 1
        ls, ts = (logits.stride(0), 0), (targets.stride(0), 0)
    else:
        outer, inner = logits.size(0), logits.size(2)
        ls, ts = (logits.stride(0), logits.stride(2)), (targets.stride(0), targets.stride(1))
    vocab = logits.size(1)
    rows = outer * inner
    row_loss = torch.empty(rows, dtype=torch.float32, device=logits.device)
    row_lse = torch.empty_like(row_loss)
    mean = torch.empty(2, dtype=torch.float32, device=logits.device)
    code = DTYPE_CODES[logits.dtype]
    _capi.cross_entropy_fwd(logits.data_ptr(), vocab, outer, inner, ls, targets.data_ptr(), ts,
                            ignore_index, row_loss.data_ptr(), row_lse.data_ptr(),
                            mean.data_ptr(), code, stream())
    if not want_grad:
        return mean[0], row_loss, None
    if logits.dim() == 2:
        d = torch.empty((outer, vocab), dtype=logits.dtype, device=logits.device)
        ds = (d.stride(0), 0)
        dview = d
    else:
        d = torch.empty((outer, inner, vocab), dtype=logits.dtype, device=logits.device)
        ds = (d.stride(0), d.stride(1))
        dview = d.transpose(1, 2)
    g = None if grad is None else torch.tensor([grad], dtype=torch.float32, device=logits.device)
    _capi.cross_entropy_bwd(logits.data_ptr(), vocab, outer, inner, ls, targets.data_ptr(), ts,
                            ignore_index, row_lse.data_ptr(), mean.data_ptr(),
                            g.data_ptr() if g is not None else None, d.data_ptr(), ds, code,
                            stream())
    return mean[0], row_loss, dview


def rope_qk(direction: str, q, k, cos, sin, layout: str = "interleaved"):
    code = {"interleaved": _capi.PT_ROPE_INTERLEAVED, "rotate_half": _capi.PT_ROPE_ROTATE_HALF}
    qo, ko = torch.empty_like(q), torch.empty_like(k)
    _capi.rope_qk(direction, q.data_ptr(), q.stride(), qo.data_ptr(), qo.stride(), q.shape,
                  k.data_ptr(), k.stride(), ko.data_ptr(), ko.stride(), k.shape, cos.data_ptr(),
                  sin.data_ptr(), cos.stride(0), code[layout], DTYPE_CODES[q.dtype],
                  DTYPE_CODES[cos.dtype], stream())
    return qo, ko


def fused_workspace(rows: int, hidden: int, x_dtype, w_dtype, add: bool = False):
    """A zeroed workspace of the size pt_(add_)rmsnorm_bwd_fused asks for."""

    query = _capi.add_rmsnorm_bwd_fused_workspace if add else _capi.rmsnorm_bwd_fused_workspace
    floats = query(rows, hidden, DTYPE_CODES[x_dtype], DTYPE_CODES[w_dtype])
    return torch.zeros(floats, dtype=torch.float32, device=DEV)


def rmsnorm_bwd_fused(dy2d, x2d, w, eps, rstd=None, ws=None):
    rows, hidden = x2d.shape
    if ws is None:
        ws = fused_workspace(rows, hidden, x2d.dtype, w.dtype)
    dx = torch.empty((rows, hidden), dtype=x2d.dtype, device=x2d.device)
    dw = torch.full((hidden,), float("nan"), dtype=w.dtype, device=x2d.device)
    _capi.rmsnorm_bwd_fused(dy2d.data_ptr(), dy2d.stride(0), x2d.data_ptr(), x2d.stride(0),
                            w.data_ptr(), rstd.data_ptr() if rstd is not None else None,
                            dx.data_ptr(), dx.stride(0), dw.data_ptr(), ws.data_ptr(),
                            ws.numel(), rows, hidden, DTYPE_CODES[x2d.dtype],
                            DTYPE_CODES[w.dtype], eps, stream())
    return dx, dw


def add_rmsnorm_bwd_fused(dy2d, dh2d, h2d, w, eps, ws=None):
    rows, hidden = h2d.shape
    if ws is None:
        ws = fused_workspace(rows, hidden, h2d.dtype, w.dtype, add=True)
    dx = torch.empty_like(h2d)
    dw = torch.full((hidden,), float("nan"), dtype=w.dtype, device=h2d.device)
    _capi.add_rmsnorm_bwd_fused(dy2d.data_ptr(), dy2d.stride(0),
                                dh2d.data_ptr() if dh2d is not None else None,
                                dh2d.stride(0) if dh2d is not None else 0, h2d.data_ptr(),
                                h2d.stride(0), w.data_ptr(), None, dx.data_ptr(), dx.stride(0),
                                dw.data_ptr(), ws.data_ptr(), ws.numel(), rows, hidden,
                                DTYPE_CODES[h2d.dtype], DTYPE_CODES[w.dtype], eps, stream())
    return dx, dw
