"""Fused gate/up GEMM + SwiGLU epilogue (pt_swiglu_gemm_fwd, tcgen05) vs the oracle.

gate and up are held to the float64 products (oracle gate_up_forward "exact") and act to
the float64 activation of the kernel's own stored gate and up, both with the library's
16-bit tolerance (oracle/tolerance.py: 2 ulp of the float64 value plus a 2^-16 * max|ref|
fp32-accumulation floor). The float64 products run on the GPU.
"""

from __future__ import annotations

import pytest
import torch

import golden_io
import gpu_utils as gu
from oracle import picotron_oracle as po
from oracle import tolerance
from picotron_b200 import _capi

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    gu.require_gpu()


def _check(x, wg, wu, what):
    act, g, u = gu.swiglu_gemm(x, wg, wu)
    torch.cuda.synchronize()
    assert _capi.take_device_error() == 0, f"{what}: the kernel reported a wait timeout"
    ge, ue, _ = po.gate_up_forward(x, wg, wu, "exact")
    tolerance.assert_close(g, ge, f"{what} gate")
    tolerance.assert_close(u, ue, f"{what} up")
    tolerance.assert_close(act, po.swiglu_forward(g, u, "exact"), f"{what} act")
    return act, g, u


def test_golden_fixture():
    t, _ = golden_io.load("gate_up_bf16")
    x, wg, wu = (t[k].to(gu.DEV) for k in ("x", "w_gate", "w_up"))
    act, g, u = _check(x, wg, wu, "golden")
    # Against the reference module's own bf16 outputs (CPU GEMM, then F.silu(g) * u rounded
    # twice): same math up to fp32 summation order and the activation's extra rounding.
    tolerance.assert_close(g, t["gate"].double(), "golden gate vs reference", torch.bfloat16)
    tolerance.assert_close(u, t["up"].double(), "golden up vs reference", torch.bfloat16)


SHAPES = [(128, 128, 64), (1, 8, 8), (256, 512, 4096), (300, 264, 200), (77, 1000, 136),
          (1024, 2048, 1024), (129, 384, 4104)]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("shape", SHAPES, ids=str)
def test_shapes_and_tails(dtype, shape):
    m, n, k = shape
    scale = k ** -0.5
    x = gu.randn((m, k), 81, dtype)
    wg = gu.randn((n, k), 82, dtype, scale=2 * scale)
    wu = gu.randn((n, k), 83, dtype, scale=2 * scale)
    _check(x, wg, wu, f"{dtype}{shape}")


def test_without_saved_preactivations_and_strided_x():
    m, n, k = 384, 512, 1024
    base = gu.randn((m, k + 64), 84, torch.bfloat16)
    x = base[:, 32:32 + k]                # row stride k + 64, 64-byte offset
    wg = gu.randn((n, k), 85, torch.bfloat16, scale=k ** -0.5)
    wu = gu.randn((n, k), 86, torch.bfloat16, scale=k ** -0.5)
    act, g, u = gu.swiglu_gemm(x, wg, wu)
    act2, _, _ = gu.swiglu_gemm(x.contiguous(), wg, wu, save_preact=False)
    assert torch.equal(act, act2)
    tolerance.assert_close(act, po.swiglu_forward(g, u, "exact"), "strided act")


def test_strided_outputs_leave_neighbours_untouched():
    # act into columns [8, 8 + n) of a wider buffer, gate and up side by side in one [m, 2n]
    # buffer; the padding columns and the rows past m keep their sentinel.
    m, n, k = 200, 264, 512
    x = gu.randn((m, k), 92, torch.bfloat16)
    wg = gu.randn((n, k), 93, torch.bfloat16, scale=k ** -0.5)
    wu = gu.randn((n, k), 94, torch.bfloat16, scale=k ** -0.5)
    sentinel = 7.0
    act_buf = torch.full((m + 3, n + 24), sentinel, dtype=torch.bfloat16, device=gu.DEV)
    pre_buf = torch.full((m + 3, 2 * n), sentinel, dtype=torch.bfloat16, device=gu.DEV)
    act, g, u = act_buf[:m, 8:8 + n], pre_buf[:m, :n], pre_buf[:m, n:]
    _capi.swiglu_gemm_fwd(x.data_ptr(), k, wg.data_ptr(), wu.data_ptr(), k, act.data_ptr(),
                          act.stride(0), g.data_ptr(), u.data_ptr(), pre_buf.stride(0), m, n, k,
                          _capi.PT_BFLOAT16, gu.stream())
    torch.cuda.synchronize()
    assert _capi.take_device_error() == 0
    ea, eg, eu = gu.swiglu_gemm(x, wg, wu)
    assert torch.equal(act, ea) and torch.equal(g, eg) and torch.equal(u, eu)
    assert bool((act_buf[:, :8] == sentinel).all()) and bool((act_buf[:, 8 + n:] == sentinel).all())
    assert bool((act_buf[m:] == sentinel).all()) and bool((pre_buf[m:] == sentinel).all())


def test_deterministic():
    m, n, k = 512, 1024, 2048
    x = gu.randn((m, k), 87, torch.bfloat16)
    wg = gu.randn((n, k), 88, torch.bfloat16, scale=k ** -0.5)
    wu = gu.randn((n, k), 89, torch.bfloat16, scale=k ** -0.5)
    a1, g1, u1 = gu.swiglu_gemm(x, wg, wu)
    a2, g2, u2 = gu.swiglu_gemm(x, wg, wu)
    assert torch.equal(a1, a2) and torch.equal(g1, g2) and torch.equal(u1, u2)


def test_rejects_unsupported_shapes():
    x = gu.randn((16, 20), 90, torch.bfloat16)
    w = gu.randn((16, 20), 91, torch.bfloat16)
    out = torch.empty((16, 16), dtype=torch.bfloat16, device=gu.DEV)
    with pytest.raises(_capi.PtError):        # k = 20 is not a multiple of 8
        _capi.swiglu_gemm_fwd(x.data_ptr(), 20, w.data_ptr(), w.data_ptr(), 20, out.data_ptr(),
                              16, None, None, 16, 16, 16, 20, _capi.PT_BFLOAT16, gu.stream())
    with pytest.raises(_capi.PtError):        # float32 is not a tensor-core input here
        _capi.swiglu_gemm_fwd(x.data_ptr(), 20, w.data_ptr(), w.data_ptr(), 20, out.data_ptr(),
                              16, None, None, 16, 16, 16, 16, _capi.PT_FLOAT32, gu.stream())


def test_llama_mlp_shape_against_library_gemm():
    # Config 3/5 shapes: x [16384, 4096], w [14336, 4096]. The float64 reference of a
    # 16384 x 14336 x 4096 product is too slow here, so: full parity on a row sample
    # (float64 on the GPU) and a whole-tensor comparison with cuBLAS + the SwiGLU kernel.
    m, n, k = 16384, 14336, 4096
    x = gu.randn((m, k), 0, torch.bfloat16)
    wg = gu.randn((n, k), 1, torch.bfloat16, scale=2 * k ** -0.5)
    wu = gu.randn((n, k), 2, torch.bfloat16, scale=2 * k ** -0.5)
    act, g, u = gu.swiglu_gemm(x, wg, wu)
    torch.cuda.synchronize()
    rows = torch.arange(0, m, 61, device=gu.DEV)
    ge, ue, _ = po.gate_up_forward(x[rows], wg, wu, "exact")
    gu.full_size_parity(g[rows], ge, "llama gate_up gemm gate (row sample)", cancels=True,
                        max_frac_over_2ulp=gu.MAX_FRAC_OVER_2ULP_GEMM_K4096)
    gu.full_size_parity(u[rows], ue, "llama gate_up gemm up (row sample)", cancels=True,
                        max_frac_over_2ulp=gu.MAX_FRAC_OVER_2ULP_GEMM_K4096)
    del ge, ue
    gu.full_size_parity(act[rows], po.swiglu_forward(g[rows], u[rows], "exact"),
                        "llama gate_up gemm act (row sample)", cancels=False)
    ref_g = x @ wg.t()
    assert (g.float() - ref_g.float()).abs().max().item() <= 0.05 * ref_g.float().abs().max().item()
    del ref_g
    torch.cuda.empty_cache()
