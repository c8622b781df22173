"""RoPE forward/backward kernels vs the float64 oracle, through the C ABI."""

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


def _tables(s, d, theta, dtype):
    cos, sin = po.rotary_cos_sin(s, d, theta, dtype)
    return cos.to(gu.DEV), sin.to(gu.DEV)


def _check(x, dy, cos, sin, layout, what, full_size=False):
    out = gu.rope("fwd", x, cos, sin, layout)
    dx = gu.rope("bwd", dy, cos, sin, layout)
    torch.cuda.synchronize()
    assert out.stride() == x.stride()
    check = ((lambda o, e, w: gu.full_size_parity(o, e, w, cancels=True)) if full_size
             else tolerance.assert_close)
    check(out, po.rope_forward(x, cos, sin, "exact", layout), f"{what} fwd")
    check(dx, po.rope_backward(dy, cos, sin, "exact", layout), f"{what} bwd")


@pytest.mark.parametrize("case", ["rope_bf16", "rope_f32"])
def test_golden_fixtures(case):
    t, meta = golden_io.load(case)
    q = t["q"].to(gu.DEV).transpose(1, 2)        # [B, H, S, D] view of [B, S, H, D] memory
    dy = t["dy"].to(gu.DEV).transpose(1, 2)
    cos, sin = t["cos"].to(gu.DEV), t["sin"].to(gu.DEV)
    _check(q, dy, cos, sin, "interleaved", case)
    out = gu.rope("fwd", q, cos, sin)
    dq = gu.rope("bwd", dy, cos, sin)
    ref_dtype = torch.float32 if q.dtype == torch.float32 else q.dtype
    if q.dtype == torch.float32:
        tolerance.assert_close(out.contiguous(), t["out"].double(), f"{case} vs reference")
        tolerance.assert_close(dq.transpose(1, 2).contiguous(), t["dq"].double(),
                               f"{case} dq vs reference", ref_dtype)


@pytest.mark.parametrize("layout", ["interleaved", "rotate_half"])
@pytest.mark.parametrize("dtype,tdtype", [(torch.bfloat16, torch.bfloat16),
                                          (torch.bfloat16, torch.float32),
                                          (torch.float16, torch.float16),
                                          (torch.float32, torch.float32)],
                         ids=["bf16", "bf16_f32tab", "f16", "f32"])
@pytest.mark.parametrize("geom", [(2, 4, 16, 128), (1, 3, 5, 64), (2, 2, 7, 16), (1, 2, 3, 6),
                                  (3, 1, 9, 8)], ids=str)
def test_layouts_dtypes_geometries(layout, dtype, tdtype, geom):
    b, h, s, d = geom
    cos, sin = _tables(s, d, 500_000.0, tdtype)
    # contiguous [B, H, S, D]
    x = gu.randn(geom, 1, dtype)
    dy = gu.randn(geom, 2, dtype)
    _check(x, dy, cos, sin, layout, f"contig {geom}")
    # transposed view of [B, S, H, D] memory (the attention layer's layout)
    xt = gu.randn((b, s, h, d), 3, dtype).transpose(1, 2)
    dyt = gu.randn((b, s, h, d), 4, dtype).transpose(1, 2)
    _check(xt, dyt, cos, sin, layout, f"view {geom}")


def test_misaligned_and_strided_table():
    d = 64
    cos_big, sin_big = _tables(10, d + 8, 10_000.0, torch.bfloat16)
    cos, sin = _tables(10, d, 10_000.0, torch.bfloat16)
    wide_c = torch.zeros(10, d // 2 + 4, dtype=torch.bfloat16, device=gu.DEV)
    wide_s = torch.zeros_like(wide_c)
    wide_c[:, : d // 2] = cos
    wide_s[:, : d // 2] = sin
    x = gu.randn(2 * 3 * 10 * d + 1, 5, torch.bfloat16)[1:].view(2, 3, 10, d)
    dy = gu.randn((2, 3, 10, d), 6, torch.bfloat16)
    _check(x, dy, wide_c[:, : d // 2], wide_s[:, : d // 2], "interleaved", "misaligned")


def test_roundtrip_is_identity_fp32():
    x = gu.randn((2, 8, 64, 128), 7, torch.float32)
    cos, sin = _tables(64, 128, 500_000.0, torch.float32)
    for layout in ("interleaved", "rotate_half"):
        back = gu.rope("bwd", gu.rope("fwd", x, cos, sin, layout), cos, sin, layout)
        torch.testing.assert_close(back, x, rtol=1e-5, atol=1e-5)


def test_relative_position_property_on_gpu():
    torch.manual_seed(0)
    head_dim = 8
    q = torch.randn(1, 1, 1, head_dim).expand(-1, -1, 12, -1).clone().to(gu.DEV)
    k = torch.randn(1, 1, 1, head_dim).expand(-1, -1, 12, -1).clone().to(gu.DEV)
    cos, sin = _tables(12, head_dim, 10_000.0, torch.float32)
    rq, rk = gu.rope("fwd", q, cos, sin), gu.rope("fwd", k, cos, sin)
    torch.testing.assert_close((rq[:, :, 2] * rk[:, :, 5]).sum(), (rq[:, :, 6] * rk[:, :, 9]).sum())


def test_full_size_config4_bf16():
    # BASELINE config 4 geometry: q [8,2048,32,128], k [8,2048,8,128] as [B,S,H,D] memory,
    # theta 5e5, positions 0..2047; interleaved (the reference) and rotate-half.
    cos, sin = _tables(2048, 128, 500_000.0, torch.bfloat16)
    for heads, seed in ((32, 0), (8, 1)):
        x = gu.randn((8, 2048, heads, 128), seed, torch.bfloat16).transpose(1, 2)
        dy = gu.randn((8, 2048, heads, 128), seed + 10, torch.bfloat16).transpose(1, 2)
        for layout in ("interleaved", "rotate_half"):
            _check(x, dy, cos, sin, layout, f"cfg4 rope h={heads} {layout}", full_size=True)
    torch.cuda.empty_cache()


@pytest.mark.parametrize("layout", ["interleaved", "rotate_half"])
@pytest.mark.parametrize("direction", ["fwd", "bwd"])
def test_query_and_key_in_one_launch(layout, direction):
    # [B, S, H, D] memory seen as [B, H, S, D]; k with fewer heads (grouped-query attention).
    from oracle import picotron_oracle as po
    q = gu.randn((2, 96, 8, 128), 201, torch.bfloat16).transpose(1, 2)
    k = gu.randn((2, 96, 2, 128), 202, torch.bfloat16).transpose(1, 2)
    cos, sin = po.rotary_cos_sin(96, 128, 500_000.0, torch.bfloat16)
    cos, sin = cos.to(gu.DEV), sin.to(gu.DEV)
    qo, ko = gu.rope_qk(direction, q, k, cos, sin, layout)
    assert torch.equal(qo, gu.rope(direction, q, cos, sin, layout))
    assert torch.equal(ko, gu.rope(direction, k, cos, sin, layout))
    # One tensor on the vector path, the other (odd offset) on the scalar path.
    flat = gu.randn(k.numel() + 1, 203, torch.bfloat16)
    k_odd = flat[1:].view(2, 96, 2, 128).transpose(1, 2)
    qo2, ko2 = gu.rope_qk(direction, q, k_odd, cos, sin, layout)
    assert torch.equal(qo2, qo)
    assert torch.equal(ko2, gu.rope(direction, k_odd, cos, sin, layout))


@pytest.mark.parametrize("layout", ["interleaved", "rotate_half"])
@pytest.mark.parametrize("dtype,tdtype", [(torch.bfloat16, torch.bfloat16),
                                          (torch.float16, torch.float32),
                                          (torch.float32, torch.float32)], ids=str)
def test_rows_path_is_bit_identical_to_the_vector_path(layout, dtype, tdtype):
    # The same values as the [B,H,S,D] view of [B,S,H,D] memory (contiguous (b, s) rows: the
    # rows path for interleaved pairs) and as a contiguous [B,H,S,D] tensor (the vector path).
    b, s, h, d = 2, 40, 6, 64
    cos, sin = _tables(s, d, 10_000.0, tdtype)
    rows_view = gu.randn((b, s, h, d), 31, dtype).transpose(1, 2)
    dense = rows_view.contiguous()
    for direction in ("fwd", "bwd"):
        r = gu.rope(direction, rows_view, cos, sin, layout)
        v = gu.rope(direction, dense, cos, sin, layout)
        assert torch.equal(r.contiguous(), v), f"{direction} {layout}"
    tolerance.assert_close(gu.rope("fwd", rows_view, cos, sin, layout),
                           po.rope_forward(rows_view, cos, sin, "exact", layout), "rows fwd")
