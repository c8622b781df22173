"""The RMSNorm backward with its dweight reduction in the same launch
(pt_rmsnorm_bwd_fused, pt_add_rmsnorm_bwd_fused), through the C ABI.

It must give the bits of the two-launch pair (pt_rmsnorm_bwd with
pt_rmsnorm_bwd_num_partials partial rows, then pt_rmsnorm_dw_reduce), on the fast
pipeline and on the generic rows it hands to the two kernels; reuse one workspace across
calls of any shape without clearing it (the grid barrier's counter is left ready by every
call); and reject a workspace that is too small or misaligned.
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


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    gu.require_gpu()


CASES = [
    (torch.bfloat16, torch.float32, (4096, 4096)),
    (torch.bfloat16, torch.bfloat16, (1000, 2048)),
    (torch.float16, torch.float32, (333, 8192)),
    (torch.float32, torch.float32, (777, 4096)),
    (torch.bfloat16, torch.float32, (5, 4096)),     # fewer rows than resident CTAs
    (torch.bfloat16, torch.float32, (1, 64)),       # one CTA: the barrier of a single CTA
    (torch.bfloat16, torch.float32, (300, 1000)),   # hidden not a multiple of 8: generic rows
    (torch.float32, torch.float32, (64, 13)),       # generic rows
]


@pytest.mark.parametrize("xd,wd,shape", CASES, ids=str)
@pytest.mark.parametrize("with_rstd", [False, True])
def test_bit_identical_to_the_two_launch_pair(xd, wd, shape, with_rstd):
    rows, hidden = shape
    x = gu.randn(shape, 41, xd)
    dy = gu.randn(shape, 42, xd)
    w = gu.randn(hidden, 43, wd, 0.02, 1.0)
    rstd = gu.rmsnorm_fwd(x, w, 1e-5, want_rstd=True)[1] if with_rstd else None
    dx_ref, dw_ref = gu.rmsnorm_bwd(dy, x, w, 1e-5, rstd=rstd)
    dx, dw = gu.rmsnorm_bwd_fused(dy, x, w, 1e-5, rstd=rstd)
    torch.cuda.synchronize()
    assert torch.equal(dx, dx_ref)
    assert torch.equal(dw, dw_ref)
    _, dwe = po.rms_norm_backward(x, w, dy, 1e-5, "exact")
    tolerance.assert_close(dw, dwe, f"dw {shape}", wd)
    assert _capi.take_device_error() == 0


def test_one_workspace_serves_many_shapes_without_clearing():
    # The largest problem sizes the workspace; every other call reuses it as it was left.
    shapes = [(8192, 4096), (3, 4096), (2048, 2048), (1, 4096), (8192, 4096), (0, 4096)]
    ws = gu.fused_workspace(8192, 4096, torch.bfloat16, torch.float32)
    w = gu.randn(4096, 51, torch.float32, 0.02, 1.0)
    for i, (rows, hidden) in enumerate(shapes):
        x = gu.randn((rows, hidden), 60 + i, torch.bfloat16)
        dy = gu.randn((rows, hidden), 70 + i, torch.bfloat16)
        ww = w[:hidden].contiguous()
        dx, dw = gu.rmsnorm_bwd_fused(dy, x, ww, 1e-5, ws=ws)
        if rows == 0:
            assert torch.equal(dw, torch.zeros_like(dw))
            continue
        dx_ref, dw_ref = gu.rmsnorm_bwd(dy, x, ww, 1e-5)
        assert torch.equal(dx, dx_ref) and torch.equal(dw, dw_ref), (rows, hidden)
    torch.cuda.synchronize()
    # The barrier counter's low 31 bits are back at zero.
    assert (ws[:1].view(torch.int32).item() & 0x7FFFFFFF) == 0
    assert _capi.take_device_error() == 0


@pytest.mark.parametrize("with_dh", [True, False])
def test_fused_add_backward_matches_the_pair(with_dh):
    n, hd = 2048, 4096
    h = gu.randn((n, hd), 81, torch.bfloat16)
    dy = gu.randn((n, hd), 82, torch.bfloat16)
    dh = gu.randn((n, hd), 83, torch.bfloat16) if with_dh else None
    w = gu.randn(hd, 84, torch.float32, 0.02, 1.0)
    dx_ref, dw_ref = gu.add_rmsnorm_bwd(dy, dh, h, w, 1e-5)
    dx, dw = gu.add_rmsnorm_bwd_fused(dy, dh, h, w, 1e-5)
    torch.cuda.synchronize()
    assert torch.equal(dx, dx_ref) and torch.equal(dw, dw_ref)


def test_rejects_small_or_misaligned_workspace():
    x = gu.randn((64, 4096), 91, torch.bfloat16)
    w = gu.randn(4096, 92, torch.float32)
    ws = gu.fused_workspace(64, 4096, torch.bfloat16, torch.float32)
    code = (DTYPE_CODES[torch.bfloat16], DTYPE_CODES[torch.float32])
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    with pytest.raises(_capi.PtError) as info:
        _capi.rmsnorm_bwd_fused(x.data_ptr(), 4096, x.data_ptr(), 4096, w.data_ptr(), None,
                                dx.data_ptr(), 4096, dw.data_ptr(), ws.data_ptr(),
                                ws.numel() - 1, 64, 4096, *code, 1e-5, gu.stream())
    assert info.value.status == _capi.PT_ERR_SHAPE
    with pytest.raises(_capi.PtError) as info:
        _capi.rmsnorm_bwd_fused(x.data_ptr(), 4096, x.data_ptr(), 4096, w.data_ptr(), None,
                                dx.data_ptr(), 4096, dw.data_ptr(), ws[16:].data_ptr(),
                                ws.numel() - 16, 64, 4096, *code, 1e-5, gu.stream())
    assert info.value.status == _capi.PT_ERR_INVALID_ARGUMENT
