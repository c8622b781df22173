"""Pins the oracle against the reference's own outputs (``tests/golden``).

The fixtures were produced by running the reference (picotron) itself
(``tests/golden/make_golden.py``). The oracle's ``eager`` form must reproduce them bit for
bit (same PyTorch CPU ops in the same order, one thread); its ``exact`` (float64) form
must agree within the fp32 tolerance on the fp32/fp64 cases and, on the bf16 RMSNorm cases
(where the reference upcasts to fp32 internally), within the bf16 tolerance.
"""

from __future__ import annotations

import pytest
import torch

import golden_io
from oracle import picotron_oracle as po
from oracle import tolerance


@pytest.fixture(autouse=True)
def _one_thread():
    previous = torch.get_num_threads()
    torch.set_num_threads(1)
    yield
    torch.set_num_threads(previous)


def test_all_golden_cases_present():
    assert set(golden_io.cases()) == {
        "cfg1_rmsnorm_f32", "cfg1_swiglu_f32", "reftest_rmsnorm_f32", "reftest_swiglu_f64",
        "rmsnorm_bf16", "rmsnorm_bf16_wf32", "swiglu_bf16", "rope_bf16", "rope_f32",
        "add_rmsnorm_bf16", "gate_up_bf16", "ce_f32", "ce_bf16", "adamw_f32",
    }


@pytest.mark.parametrize("case", ["cfg1_rmsnorm_f32", "reftest_rmsnorm_f32", "rmsnorm_bf16",
                                  "rmsnorm_bf16_wf32"])
def test_rmsnorm_oracle_matches_reference(case):
    t, meta = golden_io.load(case)
    eps = float(meta["eps"])
    y, _ = po.rms_norm_forward(t["x"], t["w"], eps, "eager")
    dx, dw = po.rms_norm_backward(t["x"], t["w"], t["dy"], eps, "eager")
    assert torch.equal(y, t["y"])
    assert torch.equal(dx, t["dx"])
    assert torch.equal(dw, t["dw"])
    ye, _ = po.rms_norm_forward(t["x"], t["w"], eps, "exact")
    dxe, dwe = po.rms_norm_backward(t["x"], t["w"], t["dy"], eps, "exact")
    tolerance.assert_close(t["y"], ye, f"{case} y")
    tolerance.assert_close(t["dx"], dxe, f"{case} dx")
    tolerance.assert_close(t["dw"], dwe, f"{case} dw")


def test_add_rmsnorm_oracle_matches_reference():
    t, meta = golden_io.load("add_rmsnorm_bf16")
    eps = float(meta["eps"])
    h, y, _ = po.add_rms_norm_forward(t["residual"], t["branch"], t["w"], eps, "eager")
    dx, dw = po.add_rms_norm_backward(h, t["w"], t["dy"], t["dh"], eps, "eager")
    assert torch.equal(h, t["h"]) and torch.equal(y, t["y"])
    assert torch.equal(dx, t["dresidual"]) and torch.equal(dx, t["dbranch"])
    assert torch.equal(dw, t["dw"])
    he, ye, _ = po.add_rms_norm_forward(t["residual"], t["branch"], t["w"], eps, "exact")
    dxe, dwe = po.add_rms_norm_backward(he, t["w"], t["dy"], t["dh"], eps, "exact")
    assert torch.equal(he, t["h"])  # h is stored in bf16 by the reference in both modes
    tolerance.assert_close(t["y"], ye, "add_rmsnorm y")
    tolerance.assert_close(t["dw"], dwe, "add_rmsnorm dw")
    # The reference rounds the norm's dx to bf16 before adding dh (two roundings), so near
    # cancellations it is off by up to a bf16 ulp of the operands: reported, bounded loosely.
    stats = tolerance.compare(t["dresidual"], dxe)
    assert stats.max_abs <= 2.0 ** -7 * float(dxe.abs().max())


def test_gate_up_oracle_matches_reference():
    t, _ = golden_io.load("gate_up_bf16")
    g, u, act = po.gate_up_forward(t["x"], t["w_gate"], t["w_up"], "eager")
    assert torch.equal(g, t["gate"]) and torch.equal(u, t["up"]) and torch.equal(act, t["act"])
    ge, ue, _ = po.gate_up_forward(t["x"], t["w_gate"], t["w_up"], "exact")
    tolerance.assert_close(t["gate"], ge, "gate_up gate")
    tolerance.assert_close(t["up"], ue, "gate_up up")


@pytest.mark.parametrize("case", ["ce_f32", "ce_bf16"])
def test_cross_entropy_oracle_matches_reference(case):
    t, _ = golden_io.load(case)
    logits, ids = t["logits"], t["input_ids"]
    view, targets = logits[:, :-1, :].transpose(1, 2), ids[:, 1:]
    loss = po.cross_entropy_forward(view, targets, mode="eager")
    d = po.cross_entropy_backward(view, targets, mode="eager")
    full = torch.zeros_like(logits)
    full[:, :-1, :] = d.transpose(1, 2)
    assert torch.equal(loss, t["loss"])
    assert torch.equal(full, t["dlogits"])
    tolerance.assert_close(t["loss"], po.cross_entropy_forward(view, targets, mode="exact"),
                           f"{case} loss", torch.float32)
    de = po.cross_entropy_backward(view, targets, mode="exact")
    fe = torch.zeros(logits.shape, dtype=torch.float64)
    fe[:, :-1, :] = de.transpose(1, 2)
    tolerance.assert_close(t["dlogits"], fe, f"{case} dlogits")


def _replay_adamw(t, meta, mode):
    out = []
    for i in range(3):
        p = t[f"p{i}_init"]
        m, v = torch.zeros_like(p), torch.zeros_like(p)
        if mode == "exact":
            p, m, v = p.double(), m.double(), v.double()
        for k in range(int(meta["steps"])):
            p, m, v = po.adamw_step(p, t[f"g{i}_s{k}"], m, v, k + 1, float(meta["lr"]),
                                    (float(meta["beta1"]), float(meta["beta2"])),
                                    float(meta["eps"]), float(meta["weight_decay"]), mode=mode)
        out.append((p, m, v))
    return out


def test_adamw_oracle_matches_reference():
    t, meta = golden_io.load("adamw_f32")
    for i, (p, m, v) in enumerate(_replay_adamw(t, meta, "eager")):
        assert torch.equal(p, t[f"p{i}"]) and torch.equal(m, t[f"m{i}"])
        assert torch.equal(v, t[f"v{i}"])
    for i, (p, m, v) in enumerate(_replay_adamw(t, meta, "exact")):
        tolerance.assert_close(t[f"p{i}"], p, f"adamw p{i}")
        tolerance.assert_close(t[f"m{i}"], m, f"adamw m{i}")
        tolerance.assert_close(t[f"v{i}"], v, f"adamw v{i}")


@pytest.mark.parametrize("case", ["cfg1_swiglu_f32", "reftest_swiglu_f64", "swiglu_bf16"])
def test_swiglu_oracle_matches_reference(case):
    t, _ = golden_io.load(case)
    out = po.swiglu_forward(t["gate"], t["up"], "eager")
    dg, du = po.swiglu_backward(t["gate"], t["up"], t["dy"], "eager")
    assert torch.equal(out, t["out"])
    assert torch.equal(dg, t["dgate"])
    assert torch.equal(du, t["dup"])
    oute = po.swiglu_forward(t["gate"], t["up"], "exact")
    dge, due = po.swiglu_backward(t["gate"], t["up"], t["dy"], "exact")
    if t["gate"].dtype in (torch.float32, torch.float64):
        tolerance.assert_close(t["out"], oute, f"{case} out", torch.float32)
        tolerance.assert_close(t["dgate"], dge, f"{case} dgate", torch.float32)
        tolerance.assert_close(t["dup"], due, f"{case} dup", torch.float32)
    else:
        # The reference's bf16 backward rounds after every op; it is reported, not pinned.
        stats = tolerance.compare(t["dgate"], dge)
        assert stats.max_abs > 0


@pytest.mark.parametrize("case", ["rope_f32", "rope_bf16"])
def test_rope_oracle_matches_reference(case):
    t, meta = golden_io.load(case)
    q = t["q"]  # [B, S, H, D] memory
    view = q.transpose(1, 2)
    cos, sin = po.rotary_cos_sin(view.size(-2), view.size(-1), float(meta["theta"]), q.dtype)
    assert torch.equal(cos, t["cos"]) and torch.equal(sin, t["sin"])
    out = po.rope_forward(view, cos, sin, "eager")
    assert torch.equal(out.contiguous(), t["out"])
    dq = po.rope_backward(t["dy"].transpose(1, 2), cos, sin, "eager")
    assert torch.equal(dq.transpose(1, 2).contiguous(), t["dq"])
    oute = po.rope_forward(view, cos, sin, "exact")
    dqe = po.rope_backward(t["dy"].transpose(1, 2), cos, sin, "exact")
    if q.dtype == torch.float32:
        tolerance.assert_close(t["out"], oute.contiguous(), f"{case} out")
        tolerance.assert_close(t["dq"], dqe.transpose(1, 2).contiguous(), f"{case} dq")


def test_rope_exact_backward_is_adjoint_of_forward():
    # <R x, y> == <x, R^T y> for the float64 rotation and its transpose.
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, 3, 7, 16, generator=g, dtype=torch.float64)
    y = torch.randn(2, 3, 7, 16, generator=g, dtype=torch.float64)
    cos, sin = po.rotary_cos_sin(7, 16, 10_000.0, torch.float64)
    for layout in ("interleaved", "rotate_half"):
        lhs = (po.rope_forward(x, cos, sin, "exact", layout) * y).sum()
        rhs = (x * po.rope_backward(y, cos, sin, "exact", layout)).sum()
        assert abs(float(lhs - rhs)) < 1e-10


def test_rope_relative_position_property():
    # The reference's own property test (tests/test_rope.py:10-23) on the oracle.
    torch.manual_seed(0)
    head_dim = 8
    base_q = torch.randn(1, 1, 1, head_dim).expand(-1, -1, 12, -1).clone()
    base_k = torch.randn(1, 1, 1, head_dim).expand(-1, -1, 12, -1).clone()
    cos, sin = po.rotary_cos_sin(12, head_dim, 10_000.0, torch.float32)
    rq = po.rope_forward(base_q, cos, sin)
    rk = po.rope_forward(base_k, cos, sin)
    torch.testing.assert_close((rq[:, :, 2] * rk[:, :, 5]).sum(), (rq[:, :, 6] * rk[:, :, 9]).sum())


def test_tolerance_rejects_a_planted_error():
    # A mistake planted in the oracle's output must be caught by the checker.
    t, meta = golden_io.load("rmsnorm_bf16")
    ye, _ = po.rms_norm_forward(t["x"], t["w"], float(meta["eps"]), "exact")
    good = ye.to(torch.bfloat16)
    assert tolerance.compare(good, ye).ok
    bad = good.clone()
    flat = bad.view(-1)
    flat[123] = (flat[123].float() * 1.03).to(torch.bfloat16)  # ~4 ulp at bf16 precision
    assert not tolerance.compare(bad, ye).ok
