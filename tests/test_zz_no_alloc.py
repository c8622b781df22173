"""The allocation-free RMSNorm backward (pt_rmsnorm_bwd_noalloc) through the C ABI.

It exists for callers that cannot allocate device memory (a runtime whose pool owns all
device memory, a step that must not synchronise on cudaMalloc/cudaFree, an FFI binding
without an allocator). It must give the same dx and dweight as pt_rmsnorm_bwd with a
caller-provided partials buffer, on consecutive calls that reuse its internal scratch.
This file is collected last so that a failure here cannot hide any other test.
"""

from __future__ import annotations

import pytest
import torch

import gpu_utils as gu
from oracle import tolerance
from picotron_b200 import _capi
from picotron_b200.ops import DTYPE_CODES

pytestmark = pytest.mark.gpu


def _noalloc(dy, x, w, eps):
    rows, hidden = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty(hidden, dtype=w.dtype, device=x.device)
    _capi.rmsnorm_bwd_noalloc(dy.data_ptr(), dy.stride(0), x.data_ptr(), x.stride(0),
                              w.data_ptr(), None, dx.data_ptr(), dx.stride(0), dw.data_ptr(),
                              rows, hidden, DTYPE_CODES[x.dtype], DTYPE_CODES[w.dtype], eps,
                              gu.stream())
    return dx, dw


@pytest.mark.parametrize("xd,wd,shape", [
    (torch.bfloat16, torch.float32, (4096, 4096)),
    (torch.float32, torch.float32, (1000, 2048)),
    (torch.bfloat16, torch.bfloat16, (37, 1000)),   # generic path
])
def test_noalloc_matches_allocating_backward_on_two_calls(xd, wd, shape):
    gu.require_gpu()
    rows, hidden = shape
    for call in range(2):
        x = gu.randn(shape, 100 + call, xd)
        dy = gu.randn(shape, 200 + call, xd)
        w = gu.randn(hidden, 300 + call, wd, 0.02, 1.0)
        dx_ref, dw_ref = gu.rmsnorm_bwd(dy, x, w, 1e-5)
        dx, dw = _noalloc(dy, x, w, 1e-5)
        torch.cuda.synchronize()
        tolerance.assert_close(dx, dx_ref.double(), f"dx call {call}", xd)
        tolerance.assert_close(dw, dw_ref.double(), f"dw call {call}",
                               wd if wd != torch.float32 else torch.float32)
        assert _capi.take_device_error() == 0


def test_noalloc_rejects_rows_wider_than_its_scratch():
    gu.require_gpu()
    x = torch.zeros(8, device=gu.DEV)
    hidden = (1 << 21) + 8
    with pytest.raises(_capi.PtError) as info:
        _capi.rmsnorm_bwd_noalloc(x.data_ptr(), hidden, x.data_ptr(), hidden, x.data_ptr(), None,
                                  x.data_ptr(), hidden, x.data_ptr(), 1, hidden,
                                  _capi.PT_FLOAT32, _capi.PT_FLOAT32, 1e-5, gu.stream())
    assert info.value.status == _capi.PT_ERR_SHAPE
    assert "scratch" in info.value.message
