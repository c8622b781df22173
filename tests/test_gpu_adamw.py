"""Fused AdamW step (pt_adamw_step) against torch.optim.AdamW on the same GPU, bit for bit.

The reference's optimizer step is torch.optim.AdamW (its fused extension point always falls
back to it), which on CUDA runs the multi-tensor path; the fused kernel must reproduce its
parameters and state exactly. The oracle (float64) and the reference's own CPU results
(golden fixture) are checked with the fp32 tolerance (1e-5 abs + 1e-5 rel).
"""

from __future__ import annotations

import warnings

import pytest
import torch

import golden_io
import gpu_utils as gu
from oracle import picotron_oracle as po
from oracle import tolerance
from picotron_b200.kernels import AdamWStepWithFallback, triton_adamw_step

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    gu.require_gpu()


SHAPES = [(4096, 1024), (14336,), (1, 1), (257, 3), (1000,), (65537,)]


def _params(seed, shapes=SHAPES, misaligned=False):
    g = torch.Generator().manual_seed(seed)
    out = []
    for s in shapes:
        t = torch.randn(s, generator=g)
        if misaligned:  # a parameter whose storage starts 4 bytes past a 16-byte boundary
            base = torch.empty(t.numel() + 1)
            base[1:] = t.reshape(-1)
            t = base[1:].view(s)
        out.append(torch.nn.Parameter(t.to(gu.DEV)))
    return out


def _twin(params):
    return [torch.nn.Parameter(p.detach().clone()) for p in params]


def _grads(params, seed, step):
    g = torch.Generator().manual_seed(seed * 1000 + step)
    return [torch.randn(p.shape, generator=g).to(gu.DEV) * (0.5 + step) for p in params]


def _run(opt_fused, opt_ref, pf, pr, seed, steps):
    for k in range(steps):
        for a, b, gr in zip(pf, pr, _grads(pf, seed, k)):
            a.grad, b.grad = gr.clone(), gr.clone()
        triton_adamw_step(opt_fused)
        opt_ref.step()
    torch.cuda.synchronize()


def _assert_same(opt_fused, opt_ref, pf, pr):
    for a, b in zip(pf, pr):
        assert torch.equal(a, b), (a - b).abs().max()
        sa, sb = opt_fused.state[a], opt_ref.state[b]
        assert torch.equal(sa["exp_avg"], sb["exp_avg"])
        assert torch.equal(sa["exp_avg_sq"], sb["exp_avg_sq"])
        assert sa["step"].item() == sb["step"].item() and sa["step"].device == sb["step"].device


def test_bit_identical_to_torch_adamw():
    # The reference builds AdamW with defaults (train_loop.py:302-325): on CUDA that is the
    # multi-tensor path, which the fused kernel reproduces exactly.
    pf = _params(1)
    pr = _twin(pf)
    kw = dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    opt_f = torch.optim.AdamW(pf, **kw)
    opt_r = torch.optim.AdamW(pr, **kw)
    _run(opt_f, opt_r, pf, pr, 1, 5)
    _assert_same(opt_f, opt_r, pf, pr)


def test_close_to_torch_single_tensor_adamw():
    # PyTorch's single-tensor CUDA path (foreach=False) rounds its final addcdiv differently
    # from its multi-tensor path (about one ulp apart); the fused kernel follows the latter.
    pf = _params(4)
    pr = _twin(pf)
    kw = dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    opt_f = torch.optim.AdamW(pf, **kw)
    opt_r = torch.optim.AdamW(pr, foreach=False, **kw)
    _run(opt_f, opt_r, pf, pr, 4, 5)
    for a, b in zip(pf, pr):
        tolerance.assert_close(a.detach(), b.detach().double(), "single-tensor param",
                               torch.float32)
        assert torch.equal(opt_f.state[a]["exp_avg"], opt_r.state[b]["exp_avg"])
        assert torch.equal(opt_f.state[a]["exp_avg_sq"], opt_r.state[b]["exp_avg_sq"])


def test_param_groups_maximize_and_misaligned_storage():
    pf = _params(2, misaligned=True)
    pr = _twin(pf)
    groups = lambda ps: [{"params": ps[:3], "lr": 1e-3, "weight_decay": 0.0},  # noqa: E731
                         {"params": ps[3:], "lr": 5e-3, "weight_decay": 0.3}]
    kw = dict(betas=(0.8, 0.99), eps=1e-6, maximize=True)
    opt_f, opt_r = torch.optim.AdamW(groups(pf), **kw), torch.optim.AdamW(groups(pr), **kw)
    _run(opt_f, opt_r, pf, pr, 2, 4)
    _assert_same(opt_f, opt_r, pf, pr)


def test_interleaves_with_pytorch_steps_and_lr_changes():
    pf = _params(3)
    pr = _twin(pf)
    kw = dict(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.05)
    opt_f, opt_r = torch.optim.AdamW(pf, **kw), torch.optim.AdamW(pr, **kw)
    for k in range(6):
        for a, b, gr in zip(pf, pr, _grads(pf, 3, k)):
            a.grad, b.grad = gr.clone(), gr.clone()
        lr = 1e-3 * (0.5 ** k)
        for grp in opt_f.param_groups + opt_r.param_groups:
            grp["lr"] = lr
        (opt_f.step if k % 2 else (lambda: triton_adamw_step(opt_f)))()
        opt_r.step()
    torch.cuda.synchronize()
    _assert_same(opt_f, opt_r, pf, pr)


def test_golden_fixture_and_oracle():
    t, meta = golden_io.load("adamw_f32")
    params = [torch.nn.Parameter(t[f"p{i}_init"].to(gu.DEV)) for i in range(3)]
    opt = torch.optim.AdamW(params, lr=float(meta["lr"]),
                            betas=(float(meta["beta1"]), float(meta["beta2"])),
                            eps=float(meta["eps"]), weight_decay=float(meta["weight_decay"]))
    for k in range(int(meta["steps"])):
        for i, p in enumerate(params):
            p.grad = t[f"g{i}_s{k}"].to(gu.DEV)
        triton_adamw_step(opt)
    for i, p in enumerate(params):
        st = opt.state[p]
        tolerance.assert_close(p.detach(), t[f"p{i}"].double(), f"p{i} vs reference",
                               torch.float32)
        tolerance.assert_close(st["exp_avg"], t[f"m{i}"].double(), f"m{i} vs reference",
                               torch.float32)
        tolerance.assert_close(st["exp_avg_sq"], t[f"v{i}"].double(), f"v{i} vs reference",
                               torch.float32)
        pe = t[f"p{i}_init"].double()
        me, ve = torch.zeros_like(pe), torch.zeros_like(pe)
        for k in range(int(meta["steps"])):
            pe, me, ve = po.adamw_step(pe, t[f"g{i}_s{k}"], me, ve, k + 1, float(meta["lr"]),
                                       (float(meta["beta1"]), float(meta["beta2"])),
                                       float(meta["eps"]), float(meta["weight_decay"]),
                                       mode="exact")
        tolerance.assert_close(p.detach(), pe, f"p{i} vs exact")


def test_step_object_falls_back_for_uncovered_optimizers():
    p = torch.nn.Parameter(torch.randn(10, device=gu.DEV))
    p.grad = torch.randn(10, device=gu.DEV)
    sgd = torch.optim.SGD([p], lr=0.1)
    before = p.detach().clone()
    stepper = AdamWStepWithFallback(use_triton=True)
    with warnings.catch_warnings(record=True) as caught:
        warnings.simplefilter("always")
        stepper.step(sgd)
    assert any("Triton AdamW unavailable; using PyTorch fallback" in str(w.message)
               for w in caught)
    torch.testing.assert_close(p.detach(), before - 0.1 * p.grad)
    # A covered optimizer takes the fused path without warning.
    q = torch.nn.Parameter(torch.randn(10, device=gu.DEV))
    q.grad = torch.randn(10, device=gu.DEV)
    adam = torch.optim.AdamW([q], lr=1e-3)
    with warnings.catch_warnings():
        warnings.simplefilter("error")
        AdamWStepWithFallback(use_triton=True).step(adam)
    assert adam.state[q]["step"].item() == 1.0
