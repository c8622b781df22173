"""Parity tolerances between the CUDA kernels and the float64 oracle (TEST INFRASTRUCTURE).

* float32 outputs: |out - exact| <= 1e-5 + 1e-5 * |exact| (max abs/rel error 1e-5).
* bfloat16 / float16 outputs: |out - exact| <= 2 ulp(exact) + 2^-16 * max|exact|, where
  ulp(v) is the spacing of the output format at |v| (2^(floor(log2|v|) - 7) for bf16,
  - 10 for fp16). The first term is the "2 ulps" of the target; the second is the noise
  floor of fp32 accumulation in formulas that cancel (RMSNorm dx, SwiGLU dgate near
  1 + g(1 - s) = 0, RoPE e*c - o*s): fp32 evaluation error there is a few 2^-24 of the
  cancelling terms, which the floor covers with a margin of about 64x, while it stays
  far below one ulp for every element that does not cancel.

``compare`` returns the statistics and the pass/fail verdict; ``assert_close`` raises with
the worst offenders.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

FP32_ATOL = 1e-5
FP32_RTOL = 1e-5
LOWP_ULPS = 2.0
LOWP_FLOOR = 2.0**-16

_MANTISSA_BITS = {torch.bfloat16: 7, torch.float16: 10}
_MIN_EXP = {torch.bfloat16: -126, torch.float16: -14}


def ulp(exact: Tensor, dtype: torch.dtype) -> Tensor:
    """Spacing of ``dtype`` at |exact| (float64), subnormal spacing below the normal range."""

    a = exact.double().abs()
    bits = _MANTISSA_BITS[dtype]
    e = torch.floor(torch.log2(a.clamp_min(2.0 ** _MIN_EXP[dtype])))
    return torch.exp2(e - bits)


@dataclass
class Comparison:
    ok: bool
    max_abs: float
    max_ulp: float  # max |err| / ulp(exact); 0 for fp32
    frac_over_2ulp: float
    violations: int
    numel: int
    worst: list
    floor_only: int = 0  # elements over 2 ulp that pass only through the 2^-16 max floor

    def __str__(self) -> str:
        return (f"ok={self.ok} max_abs={self.max_abs:.3e} max_ulp={self.max_ulp:.2f} "
                f"frac>2ulp={self.frac_over_2ulp:.2e} floor_only={self.floor_only} "
                f"violations={self.violations}/{self.numel} worst={self.worst}")


def compare(out: Tensor, exact: Tensor, dtype: torch.dtype | None = None) -> Comparison:
    """Compare a kernel output (any float dtype) with the float64 oracle value.

    Runs on the tensors' device (so full-size checks stay on the GPU); only scalars and
    the first few offenders come back to the host.
    """

    dtype = dtype or out.dtype
    out64 = out.detach().double().reshape(-1)
    ex = exact.detach().double().reshape(-1).to(out64.device)
    if out64.shape != ex.shape:
        raise ValueError(f"shape mismatch {tuple(out.shape)} vs {tuple(exact.shape)}")
    n = ex.numel()
    if n == 0:
        return Comparison(True, 0.0, 0.0, 0.0, 0, 0, [])
    finite = torch.isfinite(out64)
    err = (out64 - ex).abs()
    floor_only = 0
    if dtype == torch.float32:
        bound = FP32_ATOL + FP32_RTOL * ex.abs()
        max_ulp = 0.0
        over2 = 0.0
    else:
        u = ulp(ex, dtype)
        ulps = err / u
        bound = LOWP_ULPS * u + LOWP_FLOOR * ex.abs().max()
        max_ulp = float(ulps.max())
        over = ulps > LOWP_ULPS
        over2 = float(over.double().mean())
        floor_only = int((over & (err <= bound)).sum())
        del ulps, u, over
    bad = (~finite) | (err > bound)
    violations = int(bad.sum())
    worst = []
    if violations:
        idx = torch.nonzero(bad).reshape(-1)[:5]
        worst = [(int(i), float(out64[i]), float(ex[i])) for i in idx]
    return Comparison(
        ok=violations == 0,
        max_abs=float(err.max()),
        max_ulp=max_ulp,
        frac_over_2ulp=over2,
        violations=violations,
        numel=n,
        worst=worst,
        floor_only=floor_only,
    )


def assert_close(out: Tensor, exact: Tensor, what: str = "", dtype: torch.dtype | None = None):
    result = compare(out, exact, dtype)
    if not result.ok:
        raise AssertionError(f"{what}: {result}")
    return result
