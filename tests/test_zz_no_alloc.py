"""The allocation-free RMSNorm backward (pt_rmsnorm_bwd_noalloc) through the C ABI.

It exists for callers that cannot allocate device memory (a runtime whose pool owns all
device memory, a step that must not synchronise on cudaMalloc/cudaFree, an FFI binding
without an allocator). On consecutive calls that reuse its internal scratch it must give the
same dx and dweight as pt_rmsnorm_bwd with a caller-provided partials buffer (bit for bit
when both use the same partial count), and both must be within the parity tolerance of the
float64 oracle. Also covered: a partial count that the scratch clamps to an odd number (the
last partial row is zeroed), rows so wide that one partial row fits, an empty call after a
non-empty one (dweight must be exactly zero, not the earlier call's sums), and sizes beyond
the scratch. This file is collected last so that a failure here cannot hide any other test.
"""

from __future__ import annotations

import pytest
import torch

import gpu_utils as gu
from oracle import picotron_oracle as po
from oracle import tolerance
from picotron_b200 import _capi
from picotron_b200.ops import DTYPE_CODES

pytestmark = pytest.mark.gpu

SCRATCH_FLOATS = 1 << 22  # the documented size of the library's scratch array


def _noalloc(dy, x, w, eps):
    rows, hidden = x.shape
    dx = torch.empty_like(x)
    dw = torch.full((hidden,), float("nan"), dtype=w.dtype, device=x.device)
    _capi.rmsnorm_bwd_noalloc(dy.data_ptr(), dy.stride(0), x.data_ptr(), x.stride(0),
                              w.data_ptr(), None, dx.data_ptr(), dx.stride(0), dw.data_ptr(),
                              rows, hidden, DTYPE_CODES[x.dtype], DTYPE_CODES[w.dtype], eps,
                              gu.stream())
    return dx, dw


def _partials_used(rows, hidden, xd, wd):
    """The partial count the no-alloc call runs with: the allocating call's, clamped to the
    rows of the scratch array."""

    p = _capi.rmsnorm_bwd_num_partials(rows, hidden, DTYPE_CODES[xd], DTYPE_CODES[wd])
    return min(p, SCRATCH_FLOATS // hidden)


@pytest.mark.parametrize("xd,wd,shape", [
    (torch.bfloat16, torch.float32, (16384, 4096)),  # the flagship shape: full partial count
    (torch.float32, torch.float32, (1000, 2048)),
    (torch.bfloat16, torch.bfloat16, (37, 1000)),    # generic path
    (torch.bfloat16, torch.float32, (4096, 7168)),   # wide rows: the big-CTA pipeline
    (torch.bfloat16, torch.float32, (1024, 14400)),  # the scratch clamps to 291 partial rows
], ids=str)
def test_noalloc_matches_allocating_backward_and_oracle_on_two_calls(xd, wd, shape):
    gu.require_gpu()
    rows, hidden = shape
    p = _partials_used(rows, hidden, xd, wd)
    for call in range(2):
        x = gu.randn(shape, 100 + call, xd)
        dy = gu.randn(shape, 200 + call, xd)
        w = gu.randn(hidden, 300 + call, wd, 0.02, 1.0)
        dx_ref, dw_ref = gu.rmsnorm_bwd(dy, x, w, 1e-5, num_partials=p)
        dx, dw = _noalloc(dy, x, w, 1e-5)
        torch.cuda.synchronize()
        assert torch.equal(dx, dx_ref), f"dx call {call}"
        assert torch.equal(dw, dw_ref), f"dw call {call}"
        dxe, dwe = po.rms_norm_backward(x, w, dy, 1e-5, "exact")
        tolerance.assert_close(dx, dxe, f"dx vs oracle, call {call}", xd)
        tolerance.assert_close(dw, dwe, f"dw vs oracle, call {call}", wd)
        del dxe, dwe
        assert _capi.take_device_error() == 0
    torch.cuda.empty_cache()


def test_noalloc_odd_clamped_partial_count():
    gu.require_gpu()
    # The scratch holds 291 rows of 14400 floats, fewer than any device's partial count
    # for 1024 rows: an odd count, whose last row the backward writes as zeros.
    rows, hidden = 1024, 14400
    p = _partials_used(rows, hidden, torch.bfloat16, torch.float32)
    assert p == SCRATCH_FLOATS // hidden == 291
    x = gu.randn((rows, hidden), 401, torch.bfloat16)
    dy = gu.randn((rows, hidden), 402, torch.bfloat16)
    w = gu.randn(hidden, 403, torch.float32, 0.02, 1.0)
    dx, dw = _noalloc(dy, x, w, 1e-5)
    _, dwe = po.rms_norm_backward(x, w, dy, 1e-5, "exact")
    tolerance.assert_close(dw, dwe, "dw with an odd partial count", torch.float32)


def test_noalloc_one_partial_row_when_rows_are_very_wide():
    gu.require_gpu()
    hidden = (1 << 21) + 8  # one partial row of this width fits in the scratch, two do not
    assert SCRATCH_FLOATS // hidden == 1
    x = gu.randn((3, hidden), 501, torch.float32)
    dy = gu.randn((3, hidden), 502, torch.float32)
    w = gu.randn(hidden, 503, torch.float32, 0.02, 1.0)
    dx, dw = _noalloc(dy, x, w, 1e-5)
    dxe, dwe = po.rms_norm_backward(x, w, dy, 1e-5, "exact")
    tolerance.assert_close(dx, dxe, "dx, one partial row", torch.float32)
    tolerance.assert_close(dw, dwe, "dw, one partial row", torch.float32)


def test_noalloc_empty_call_after_a_full_one_gives_zero_dweight():
    gu.require_gpu()
    x = gu.randn((4096, 4096), 601, torch.bfloat16)
    w = gu.randn(4096, 602, torch.float32, 0.02, 1.0)
    _noalloc(x, x, w, 1e-5)  # leaves non-zero partial sums in the scratch
    empty = torch.empty((0, 4096), dtype=torch.bfloat16, device=gu.DEV)
    dx, dw = _noalloc(empty, empty, w, 1e-5)
    torch.cuda.synchronize()
    assert dx.numel() == 0
    assert torch.equal(dw, torch.zeros_like(dw))


def test_noalloc_rejects_rows_wider_than_its_scratch():
    gu.require_gpu()
    x = torch.zeros(8, device=gu.DEV)
    hidden = SCRATCH_FLOATS + 8
    with pytest.raises(_capi.PtError) as info:
        _capi.rmsnorm_bwd_noalloc(x.data_ptr(), hidden, x.data_ptr(), hidden, x.data_ptr(), None,
                                  x.data_ptr(), hidden, x.data_ptr(), 1, hidden,
                                  _capi.PT_FLOAT32, _capi.PT_FLOAT32, 1e-5, gu.stream())
    assert info.value.status == _capi.PT_ERR_SHAPE
    assert "scratch" in info.value.message
