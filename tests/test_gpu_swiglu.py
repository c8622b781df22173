"""SwiGLU forward/backward kernels vs the float64 oracle, through the C ABI."""

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


def _check(g, u, dy, what):
    out = gu.swiglu_fwd(g, u)
    dg, du = gu.swiglu_bwd(dy, g, u)
    torch.cuda.synchronize()
    oute = po.swiglu_forward(g, u, "exact")
    dge, due = po.swiglu_backward(g, u, dy, "exact")
    tolerance.assert_close(out, oute, f"{what} out")
    tolerance.assert_close(dg, dge, f"{what} dgate")
    tolerance.assert_close(du, due, f"{what} dup")
    return out, dg, du


@pytest.mark.parametrize("case", ["cfg1_swiglu_f32", "swiglu_bf16", "reftest_swiglu_f64"])
def test_golden_fixtures(case):
    t, _ = golden_io.load(case)
    dtype = t["gate"].dtype if t["gate"].dtype != torch.float64 else torch.float32
    g, u, dy = (t[k].to(dtype).to(gu.DEV) for k in ("gate", "up", "dy"))
    out, dg, du = _check(g, u, dy, case)
    if t["gate"].dtype == torch.float32:
        # the reference's fp32 output itself, within the fp32 tolerance
        tolerance.assert_close(out, t["out"].double(), f"{case} vs reference")
        tolerance.assert_close(dg, t["dgate"].double(), f"{case} dgate vs reference")


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16],
                         ids=lambda d: str(d).split(".")[-1])
@pytest.mark.parametrize("n", [1, 7, 8, 9, 4095, 32768, 1_000_003])
def test_sizes_and_tails(dtype, n):
    g = gu.randn(n, 1, dtype, 2.0)
    u = gu.randn(n, 2, dtype, 2.0)
    dy = gu.randn(n, 3, dtype)
    _check(g, u, dy, f"{dtype} n={n}")


def test_misaligned_pointers_take_the_scalar_path():
    base = gu.randn(100_001, 4, torch.bfloat16, 2.0)
    g, u = base[1:50_001], base[50_001:]
    dy = gu.randn(50_000, 5, torch.bfloat16)
    _check(g, u, dy, "misaligned")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16],
                         ids=lambda d: str(d).split(".")[-1])
def test_32_and_16_byte_vector_paths_agree(dtype):
    # 32-byte aligned arrays take the 32-byte vector kernels, arrays 16 bytes off it the
    # 16-byte ones; both give the same bits, tails included.
    n = 65_543
    dy, g, u = (gu.randn(n, seed, dtype, 2.0) for seed in (6, 7, 8))
    outs = []
    for off_bytes in (0, 16):
        off = off_bytes // dy.element_size()
        placed = []
        for t in (dy, g, u):  # the same values, starting off_bytes past a 256-byte boundary
            buf = torch.empty(n + 64, dtype=dtype, device=gu.DEV)
            buf[off:off + n].copy_(t)
            placed.append(buf[off:off + n])
        outs.append((gu.swiglu_fwd(placed[1], placed[2]),) + gu.swiglu_bwd(*placed))
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip(outs[0], outs[1]))
    _check(g, u, dy, f"32-byte path {dtype}")


def test_saturated_and_special_values():
    vals = torch.tensor([0.0, -0.0, 1.0, -1.0, 20.0, -20.0, 88.0, -88.0, 100.0, -100.0, 3e4,
                         -3e4, -1.2785, 1e-20, -1e-20, 5.0, -5.0, 0.5], dtype=torch.float32)
    g = vals.repeat(64).to(gu.DEV)
    u = torch.linspace(-3, 3, g.numel()).to(gu.DEV)
    dy = torch.linspace(2, -2, g.numel()).to(gu.DEV)
    for dtype in (torch.float32, torch.bfloat16):
        _check(g.to(dtype), u.to(dtype), dy.to(dtype), f"special {dtype}")


def test_empty_is_a_noop():
    e = torch.empty(0, dtype=torch.bfloat16, device=gu.DEV)
    assert gu.swiglu_fwd(e, e).numel() == 0


def test_full_size_config3_bf16():
    # gate, up [16384, 14336] ~ N(0,1) * 2, dy ~ N(0,1).
    shape = (16384, 14336)
    g = gu.randn(shape, 0, torch.bfloat16, 2.0)
    u = gu.randn(shape, 1, torch.bfloat16, 2.0)
    dy = gu.randn(shape, 2, torch.bfloat16)
    out = gu.swiglu_fwd(g, u)
    gu.full_size_parity(out, po.swiglu_forward(g, u, "exact"), "cfg3 swiglu out", cancels=False)
    del out
    dg, du = gu.swiglu_bwd(dy, g, u)
    dge, due = po.swiglu_backward(g, u, dy, "exact")
    gu.full_size_parity(dg, dge, "cfg3 swiglu dgate", cancels=True)
    gu.full_size_parity(du, due, "cfg3 swiglu dup", cancels=False)
    del dg, du, dge, due
    torch.cuda.empty_cache()
