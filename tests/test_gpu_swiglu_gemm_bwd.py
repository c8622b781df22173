"""The down projection's input gradient with the SwiGLU backward in its epilogue
(pt_swiglu_gemm_bwd, tcgen05), through the C ABI, against the float64 oracle.

As for the forward GEMM: d_act (stored on request) is held to the float64 product of the same
bf16 inputs within the GEMM bound, and dgate / dup to the float64 activation backward of the
kernel's own rounded d_act, gate and up within the standard tolerance. Shapes cover one CTA
(m <= 128), CTA pairs, a partial last row block, and a last column tile narrower than 128 in
each half of d_act. Without dact_out the gradients are the same bits.
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


def _inputs(m, n, k, seed, dtype=torch.bfloat16):
    dy = gu.randn((m, k), seed, dtype)
    w_down = gu.randn((k, n), seed + 1, dtype, scale=2 * n ** -0.5)  # nn.Linear(n -> k).weight
    gate = gu.randn((m, n), seed + 2, dtype, scale=2.0)
    up = gu.randn((m, n), seed + 3, dtype, scale=2.0)
    return dy, w_down, gate, up


def _bwd(dy, w_down, gate, up, want_dact=True):
    m, k = dy.shape
    n = w_down.size(1)
    wdt = w_down.t().contiguous()
    dg, du = torch.empty_like(gate), torch.empty_like(gate)
    da = torch.empty_like(gate) if want_dact else None
    _capi.swiglu_gemm_bwd(dy.data_ptr(), dy.stride(0), wdt.data_ptr(), wdt.stride(0),
                          gate.data_ptr(), up.data_ptr(), gate.stride(0), dg.data_ptr(),
                          du.data_ptr(), dg.stride(0), da.data_ptr() if da is not None else None,
                          n, m, n, k, DTYPE_CODES[dy.dtype], gu.stream())
    return dg, du, da


@pytest.mark.parametrize("m,n,k", [(100, 256, 128), (512, 512, 256), (300, 320, 136),
                                   (1024, 1536, 512)], ids=str)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=str)
def test_shapes_and_tails_against_float64(m, n, k, dtype):
    dy, w_down, gate, up = _inputs(m, n, k, 11, dtype)
    dg, du, da = _bwd(dy, w_down, gate, up)
    torch.cuda.synchronize()
    dae, _, _ = po.down_swiglu_backward(dy, w_down, gate, up, "exact")
    tolerance.assert_close(da, dae, f"d_act {m}x{n}x{k}")
    dge, due = po.swiglu_backward(gate, up, da, "exact")
    tolerance.assert_close(dg, dge, f"dgate {m}x{n}x{k}")
    tolerance.assert_close(du, due, f"dup {m}x{n}x{k}")
    dg2, du2, _ = _bwd(dy, w_down, gate, up, want_dact=False)
    torch.cuda.synchronize()
    assert torch.equal(dg2, dg) and torch.equal(du2, du)
    assert _capi.take_device_error() == 0


def test_matches_library_gemm_plus_activation_kernel():
    # The unfused path it replaces: cuBLAS for d_act, then this library's SwiGLU backward.
    dy, w_down, gate, up = _inputs(2048, 2048, 1024, 21)
    dg, du, _ = _bwd(dy, w_down, gate, up, want_dact=False)
    d_act = dy @ w_down
    dg_ref, du_ref = gu.swiglu_bwd(d_act, gate, up)
    torch.cuda.synchronize()
    for got, ref, what in ((dg, dg_ref, "dgate"), (du, du_ref, "dup")):
        scale = ref.float().abs().max().item()
        assert (got.float() - ref.float()).abs().max().item() <= 0.02 * scale, what


def test_llama_mlp_shape_row_sample():
    # Config 3/5 shapes: dy [16384, 4096], w_down [4096, 14336]: float64 parity on a row sample.
    m, n, k = 16384, 14336, 4096
    dy, w_down, gate, up = _inputs(m, n, k, 31)
    dg, du, da = _bwd(dy, w_down, gate, up)
    torch.cuda.synchronize()
    rows = torch.arange(0, m, 97, device=gu.DEV)
    dae = dy[rows].double() @ w_down.double()
    gu.full_size_parity(da[rows], dae, "llama down-proj dgrad d_act (row sample)", cancels=True,
                        max_frac_over_2ulp=gu.MAX_FRAC_OVER_2ULP_GEMM_K4096)
    del dae
    dge, due = po.swiglu_backward(gate[rows], up[rows], da[rows], "exact")
    gu.full_size_parity(dg[rows], dge, "llama fused swiglu-bwd dgate (row sample)", cancels=True)
    gu.full_size_parity(du[rows], due, "llama fused swiglu-bwd dup (row sample)", cancels=False)
    assert _capi.take_device_error() == 0
    torch.cuda.empty_cache()


def test_rejects_unsupported_shapes_and_aliasing():
    dy, w_down, gate, up = _inputs(128, 96, 64, 41)
    wdt = w_down.t().contiguous()
    out = torch.empty_like(gate)
    code = DTYPE_CODES[torch.bfloat16]
    with pytest.raises(_capi.PtError) as info:  # n = 96 is not a multiple of 64
        _capi.swiglu_gemm_bwd(dy.data_ptr(), 64, wdt.data_ptr(), 64, gate.data_ptr(),
                              up.data_ptr(), 96, out.data_ptr(), out.data_ptr(), 96, None, 0,
                              128, 96, 64, code, gu.stream())
    assert info.value.status == _capi.PT_ERR_SHAPE
    dy, w_down, gate, up = _inputs(128, 128, 64, 42)
    wdt = w_down.t().contiguous()
    out = torch.empty_like(gate)
    with pytest.raises(_capi.PtError) as info:  # dgate written over gate
        _capi.swiglu_gemm_bwd(dy.data_ptr(), 64, wdt.data_ptr(), 64, gate.data_ptr(),
                              up.data_ptr(), 128, gate.data_ptr(), out.data_ptr(), 128, None, 0,
                              128, 128, 64, code, gu.stream())
    assert info.value.status == _capi.PT_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32], ids=str)
@pytest.mark.parametrize("rows,cols,pad", [(4096, 1536, 0), (130, 70, 0), (64, 8, 3), (1, 1, 0)],
                         ids=str)
def test_transpose_is_exact(dtype, rows, cols, pad):
    # pad > 0 gives row strides that are not multiples of 8 (the element-wise path).
    src = gu.randn((rows, cols + pad), 51, dtype)[:, :cols]
    dst_buf = torch.full((cols, rows + pad), -7.0, dtype=dtype, device=gu.DEV)
    dst = dst_buf[:, :rows]
    _capi.transpose_2d(src.data_ptr(), src.stride(0), dst.data_ptr(), dst.stride(0), rows, cols,
                       DTYPE_CODES[dtype], gu.stream())
    torch.cuda.synchronize()
    assert torch.equal(dst, src.t())
    if pad:
        assert torch.equal(dst_buf[:, rows:], torch.full_like(dst_buf[:, rows:], -7.0))
