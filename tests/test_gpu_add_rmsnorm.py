"""Fused residual add + RMSNorm (pt_add_rmsnorm_fwd / pt_add_rmsnorm_bwd) vs the oracle.

h = residual + branch must equal PyTorch's own add bit for bit (the reference stores that
tensor); y, dx and dweight are held to the float64 oracle with the library's tolerances
(oracle/tolerance.py): fp32 outputs within 1e-5 abs + 1e-5 rel; bf16/fp16 outputs within
2 ulp of the float64 value plus a 2^-16 * max|ref| fp32-accumulation floor.
"""

from __future__ import annotations

import pytest
import torch

import golden_io
import gpu_utils as gu
from oracle import picotron_oracle as po
from oracle import tolerance

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    gu.require_gpu()


def _check(res, br, w, dy, dh, eps, what, **kw):
    h, y = gu.add_rmsnorm_fwd(res, br, w, eps)
    dx, dw = gu.add_rmsnorm_bwd(dy, dh, h, w, eps, **kw)
    torch.cuda.synchronize()
    assert torch.equal(h, res + br), f"{what}: h differs from residual + branch"
    he, ye, _ = po.add_rms_norm_forward(res.cpu(), br.cpu(), w.cpu(), eps, "exact")
    dxe, dwe = po.add_rms_norm_backward(he, w.cpu(), dy.cpu(), None if dh is None else dh.cpu(),
                                        eps, "exact")
    tolerance.assert_close(y, ye, f"{what} y")
    tolerance.assert_close(dx, dxe, f"{what} dx")
    tolerance.assert_close(dw, dwe, f"{what} dw")
    return h, y, dx, dw


def test_golden_fixture():
    t, meta = golden_io.load("add_rmsnorm_bf16")
    eps = float(meta["eps"])
    dev = {k: v.to(gu.DEV) for k, v in t.items()}
    h, y, dx, dw = _check(dev["residual"], dev["branch"], dev["w"], dev["dy"], dev["dh"], eps,
                          "golden")
    assert torch.equal(h.cpu(), t["h"])
    tolerance.assert_close(y, t["y"].double(), "golden y vs reference", torch.bfloat16)
    tolerance.assert_close(dw, t["dw"].double(), "golden dw vs reference", torch.float32)


PAIRS = [
    (torch.float32, torch.float32),
    (torch.bfloat16, torch.bfloat16),
    (torch.bfloat16, torch.float32),
    (torch.float16, torch.float16),
    (torch.float16, torch.float32),
]
SHAPES = [(1, 128), (37, 4096), (300, 4096), (16, 1000), (7, 6), (40, 16384), (149, 1024)]


@pytest.mark.parametrize("xd,wd", PAIRS, ids=lambda d: str(d).split(".")[-1])
@pytest.mark.parametrize("shape", SHAPES, ids=str)
def test_dtypes_and_shapes(xd, wd, shape):
    rows, hd = shape
    res = gu.randn(shape, 21, xd)
    br = gu.randn(shape, 22, xd, scale=0.5)
    w = gu.randn(hd, 23, wd, scale=0.1, shift=1.0)
    dy = gu.randn(shape, 24, xd)
    dh = gu.randn(shape, 25, xd)
    _check(res, br, w, dy, dh, 1e-5, f"{xd}/{wd}{shape}")


def test_in_place_residual_and_gradient():
    # h_out may be the residual buffer itself, dx may be dh.
    n, hd = 300, 4096
    res = gu.randn((n, hd), 31, torch.bfloat16)
    br = gu.randn((n, hd), 32, torch.bfloat16)
    w = gu.randn(hd, 33, torch.float32, 0.02, 1.0)
    dy = gu.randn((n, hd), 34, torch.bfloat16)
    dh = gu.randn((n, hd), 35, torch.bfloat16)
    h_ref, y_ref = gu.add_rmsnorm_fwd(res, br, w, 1e-5)
    dx_ref, dw_ref = gu.add_rmsnorm_bwd(dy, dh, h_ref, w, 1e-5)
    res_inplace = res.clone()
    h, y = gu.add_rmsnorm_fwd(res_inplace, br, w, 1e-5, h_out=res_inplace)
    dh_inplace = dh.clone()
    dx, dw = gu.add_rmsnorm_bwd(dy, dh_inplace, h_ref, w, 1e-5, dx_out=dh_inplace)
    assert torch.equal(res_inplace, h_ref) and torch.equal(y, y_ref)
    assert torch.equal(dh_inplace, dx_ref) and torch.equal(dw, dw_ref)


def test_without_residual_gradient_is_plain_backward():
    n, hd = 64, 4096
    x = gu.randn((n, hd), 41, torch.bfloat16)
    w = gu.randn(hd, 42, torch.float32, 0.02, 1.0)
    dy = gu.randn((n, hd), 43, torch.bfloat16)
    dx, dw = gu.add_rmsnorm_bwd(dy, None, x, w, 1e-5)
    dx2, dw2 = gu.rmsnorm_bwd(dy, x, w, 1e-5)
    assert torch.equal(dx, dx2) and torch.equal(dw, dw2)


def test_generic_path_misaligned_rows():
    n, hd = 64, 4096
    flat = gu.randn(n * hd + 1, 51, torch.bfloat16)
    res = flat[1:].view(n, hd)                       # 2-byte offset: generic kernels
    br = gu.randn((n, hd), 52, torch.bfloat16)
    w = gu.randn(hd, 53, torch.float32, 0.02, 1.0)
    dy = gu.randn((n, hd), 54, torch.bfloat16)
    dflat = gu.randn(n * hd + 1, 55, torch.bfloat16)
    dh = dflat[1:].view(n, hd)
    _check(res, br, w, dy, dh, 1e-5, "misaligned")


def test_rejects_bad_aliasing():
    x = gu.randn((4, 256), 61, torch.bfloat16)
    w = gu.randn(256, 62, torch.float32)
    from picotron_b200 import _capi
    with pytest.raises(_capi.PtError):
        _capi.add_rmsnorm_fwd(x.data_ptr(), 256, x.data_ptr(), 256, w.data_ptr(), x.data_ptr(),
                              256, x.data_ptr(), 256, None, 4, 256, _capi.PT_BFLOAT16,
                              _capi.PT_FLOAT32, 1e-5, gu.stream())


def test_full_size_config2_bf16():
    n, hd = 16384, 4096
    res = gu.randn((n, hd), 0, torch.bfloat16)
    br = gu.randn((n, hd), 3, torch.bfloat16)
    w = gu.randn(hd, 1, torch.float32, 0.02, 1.0)
    dy = gu.randn((n, hd), 2, torch.bfloat16)
    dh = gu.randn((n, hd), 4, torch.bfloat16)
    h, y = gu.add_rmsnorm_fwd(res, br, w, 1e-5)
    assert torch.equal(h, res + br)
    dx, dw = gu.add_rmsnorm_bwd(dy, dh, h, w, 1e-5)
    ye, _ = po.rms_norm_forward(h, w, 1e-5, "exact")        # float64 on the GPU
    gu.full_size_parity(y, ye, "cfg2 add+rmsnorm y", cancels=False)
    del ye
    dxe, dwe = po.add_rms_norm_backward(h, w, dy, dh, 1e-5, "exact")
    gu.full_size_parity(dx, dxe, "cfg2 add+rmsnorm dx", cancels=True)
    gu.full_size_parity(dw, dwe, "cfg2 add+rmsnorm dw", cancels=True)
    del dxe, dwe
    torch.cuda.empty_cache()
