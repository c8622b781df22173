"""Generate the golden fixtures by running the reference (picotron) itself on CPU.

Run in the build container, where the reference is mounted read-only:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference-src DIR

It imports the reference's own hot-path functions
(``picotron.nn.triton_kernels.rmsnorm.rms_norm_with_pytorch_forward``,
``picotron.nn.triton_kernels.swiglu.swiglu_with_pytorch_forward``,
``picotron.nn.rope.rotary_cos_sin`` / ``apply_rotary_embedding``), runs each forward and
``.backward(dy)`` on seeded inputs, and stores inputs and outputs in ``tests/golden``.
Inputs are drawn on CPU in float32 from ``torch.Generator().manual_seed(seed)`` and then
cast, so every consumer sees the same bits. One thread, so CPU reductions are ordered
the same way on every run. The fixtures are committed; this script is not needed at test
time and nothing at test time reads the reference.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
from pathlib import Path

import torch

sys.dont_write_bytecode = True
HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import golden_io  # noqa: E402


def _gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def _rms(ref, x, w, dy, eps):
    xg = x.clone().requires_grad_(True)
    wg = w.clone().requires_grad_(True)
    y = ref.rms_norm_with_pytorch_forward(xg, wg, eps)
    y.backward(dy)
    return {"y": y.detach(), "dx": xg.grad, "dw": wg.grad}


def _add_rms(ref, residual, branch, w, dy, dh, eps):
    """The decoder block's residual add followed by the norm (picotron_decoder.py:116-123),
    with the reference's RMSNorm autograd function; dh is the gradient reaching h through
    its other use (the residual stream)."""

    rg = residual.clone().requires_grad_(True)
    bg = branch.clone().requires_grad_(True)
    wg = w.clone().requires_grad_(True)
    h = rg + bg
    y = ref.rms_norm_with_pytorch_forward(h, wg, eps)
    torch.autograd.backward([y, h], [dy, dh])
    return {"h": h.detach(), "y": y.detach(), "dresidual": rg.grad, "dbranch": bg.grad,
            "dw": wg.grad}


def _gate_up(ffn_mod, x, hidden, inter, seed):
    """The reference's SwiGLU module (feedforward.py:13-43) up to its down projection."""

    torch.manual_seed(seed)
    mlp = ffn_mod.SwiGLU(hidden, inter).to(x.dtype)
    gate = mlp.gate_projection(x)
    up = mlp.up_projection(x)
    activated = torch.nn.functional.silu(gate) * up  # feedforward.py:42
    return {"w_gate": mlp.gate_projection.weight.detach(), "w_up": mlp.up_projection.weight.detach(),
            "gate": gate.detach(), "up": up.detach(), "act": activated.detach()}


def _ce(ce_mod, logits, input_ids, upcast):
    """The training loop's loss call (train_loop.py:95-97,141-145) on [B, S, V] logits, with
    the reference's CrossEntropyWithFallback; `upcast` applies CUDA autocast's fp32 cast."""

    lg = logits.clone().requires_grad_(True)
    x = lg.float() if upcast else lg
    loss = ce_mod.CrossEntropyWithFallback(use_triton=False)(
        x[:, :-1, :].transpose(1, 2), input_ids[:, 1:])
    loss.backward()
    return {"loss": loss.detach(), "dlogits": lg.grad}


def _adamw(adamw_mod, shapes, steps, seed):
    """AdamW as the training loop builds it (train_loop.py:302-325: lr, betas, eps,
    weight_decay), stepped through the reference's AdamWStepWithFallback with its fused
    switch on (which falls back to optimizer.step(), adamw.py:27-45)."""

    g = _gen(seed)
    params = [torch.nn.Parameter(torch.randn(s, generator=g)) for s in shapes]
    init = [p.detach().clone() for p in params]
    opt = torch.optim.AdamW(params, lr=3e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    stepper = adamw_mod.AdamWStepWithFallback(use_triton=True)
    out = {f"p{i}_init": t for i, t in enumerate(init)}
    import warnings
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", RuntimeWarning)
        for k in range(steps):
            for i, p in enumerate(params):
                p.grad = torch.randn(p.shape, generator=g) * (0.5 + k)
                out[f"g{i}_s{k}"] = p.grad.clone()
            stepper.step(opt)
    for i, p in enumerate(params):
        out[f"p{i}"] = p.detach().clone()
        out[f"m{i}"] = opt.state[p]["exp_avg"].clone()
        out[f"v{i}"] = opt.state[p]["exp_avg_sq"].clone()
    return out


def _swiglu(ref, g, u, dy):
    gg = g.clone().requires_grad_(True)
    ug = u.clone().requires_grad_(True)
    out = ref.swiglu_with_pytorch_forward(gg, ug)
    out.backward(dy)
    return {"out": out.detach(), "dgate": gg.grad, "dup": ug.grad}


def _rope(rope_mod, q_phys, theta, dy_phys):
    """q_phys is [B, S, H, D] memory; the reference sees the [B, H, S, D] transposed view."""

    qg = q_phys.clone().requires_grad_(True)
    view = qg.transpose(1, 2)
    cos, sin = rope_mod.rotary_cos_sin(view.size(-2), view.size(-1), theta, device=q_phys.device,
                                       dtype=q_phys.dtype)
    out = rope_mod.apply_rotary_embedding(view, cos, sin)
    out.backward(dy_phys.transpose(1, 2))
    return {"cos": cos, "sin": sin, "out": out.detach().contiguous(), "dq": qg.grad}


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-src", default=os.environ.get("PICOTRON_REFERENCE_SRC"),
                        help="the reference's src directory (or set PICOTRON_REFERENCE_SRC)")
    args = parser.parse_args()
    if not args.reference_src:
        parser.error("give --reference-src or set PICOTRON_REFERENCE_SRC")
    sys.path.insert(0, args.reference_src)
    torch.set_num_threads(1)
    from picotron.nn import feedforward as ffn_mod
    from picotron.nn.triton_kernels import adamw as adamw_mod
    from picotron.nn.triton_kernels import cross_entropy as ce_mod
    from picotron.nn import rope as rope_mod
    from picotron.nn.triton_kernels import rmsnorm as rms_ref
    from picotron.nn.triton_kernels import swiglu as swiglu_ref

    written = []

    # BASELINE config 1, RMSNorm part: fp32 x[128,128], gamma = 1 + 0.1 N(0,1), eps 1e-6.
    g = _gen(0)
    x = torch.randn(128, 128, generator=g)
    w = 1 + 0.1 * torch.randn(128, generator=g)
    dy = torch.randn(128, 128, generator=g)
    res = _rms(rms_ref, x, w, dy, 1e-6)
    written.append(golden_io.save("cfg1_rmsnorm_f32", {"x": x, "w": w, "dy": dy, **res},
                                  {"eps": 1e-6, "seed": 0}))

    # BASELINE config 1, SwiGLU part: fp32 gate, up [128, 256] ~ N(0,1), dy ~ N(0,1).
    g = _gen(0)
    gate = torch.randn(128, 256, generator=g)
    up = torch.randn(128, 256, generator=g)
    dy = torch.randn(128, 256, generator=g)
    res = _swiglu(swiglu_ref, gate, up, dy)
    written.append(golden_io.save("cfg1_swiglu_f32", {"gate": gate, "up": up, "dy": dy, **res},
                                  {"seed": 0}))

    # The reference's own RMSNorm test inputs (tests/test_triton_rmsnorm_backward.py:16-21):
    # torch.manual_seed(23); dy, x [2,3,8], w [8] (signed weights), eps 1e-6.
    torch.manual_seed(23)
    dy = torch.randn(2, 3, 8)
    x = torch.randn(2, 3, 8)
    w = torch.randn(8)
    res = _rms(rms_ref, x, w, dy, 1e-6)
    written.append(golden_io.save("reftest_rmsnorm_f32", {"x": x, "w": w, "dy": dy, **res},
                                  {"eps": 1e-6, "seed": 23}))

    # The reference's own SwiGLU test inputs (tests/test_triton_swiglu_backward.py:12-15).
    torch.manual_seed(31)
    dy = torch.randn(2, 3, 7, dtype=torch.float64)
    gate = torch.randn(2, 3, 7, dtype=torch.float64)
    up = torch.randn(2, 3, 7, dtype=torch.float64)
    res = _swiglu(swiglu_ref, gate, up, dy)
    written.append(golden_io.save("reftest_swiglu_f64", {"gate": gate, "up": up, "dy": dy, **res},
                                  {"seed": 31}))

    # BASELINE config 2 shape family, bf16: x[8, 4096] ~ N(0,1), gamma = 1 + 0.02 N(0,1),
    # eps 1e-5; gamma in bf16 and in fp32 (the module's parameter dtype).
    g = _gen(0)
    x = torch.randn(8, 4096, generator=g).to(torch.bfloat16)
    wf = 1 + 0.02 * torch.randn(4096, generator=g)
    dy = torch.randn(8, 4096, generator=g).to(torch.bfloat16)
    res = _rms(rms_ref, x, wf.to(torch.bfloat16), dy, 1e-5)
    written.append(golden_io.save("rmsnorm_bf16", {"x": x, "w": wf.to(torch.bfloat16), "dy": dy,
                                                   **res}, {"eps": 1e-5, "seed": 0}))
    res = _rms(rms_ref, x, wf, dy, 1e-5)
    written.append(golden_io.save("rmsnorm_bf16_wf32", {"x": x, "w": wf, "dy": dy, **res},
                                  {"eps": 1e-5, "seed": 0}))

    # Fused residual add + RMSNorm (the next-step row of the hot path), config 2 family,
    # bf16: residual, branch, dy, dh [8, 4096] ~ N(0,1), gamma = 1 + 0.02 N(0,1) in fp32.
    g = _gen(3)
    residual = torch.randn(8, 4096, generator=g).to(torch.bfloat16)
    branch = torch.randn(8, 4096, generator=g).to(torch.bfloat16)
    wf = 1 + 0.02 * torch.randn(4096, generator=g)
    dy = torch.randn(8, 4096, generator=g).to(torch.bfloat16)
    dh = torch.randn(8, 4096, generator=g).to(torch.bfloat16)
    res = _add_rms(rms_ref, residual, branch, wf, dy, dh, 1e-5)
    written.append(golden_io.save("add_rmsnorm_bf16", {"residual": residual, "branch": branch,
                                                       "w": wf, "dy": dy, "dh": dh, **res},
                                  {"eps": 1e-5, "seed": 3}))

    # SwiGLU MLP up to the down projection (the next-step row: gate/up GEMMs + activation),
    # bf16, hidden 64, intermediate 128, x [32, 64] ~ N(0,1), the module's own weight init.
    g = _gen(4)
    x = torch.randn(32, 64, generator=g).to(torch.bfloat16)
    res = _gate_up(ffn_mod, x, 64, 128, 4)
    written.append(golden_io.save("gate_up_bf16", {"x": x, **res}, {"seed": 4}))

    # Cross-entropy as the training loop calls it: logits [B=2, S=9, V=1000] ~ N(0,1) * 3,
    # input_ids uniform in [0, V) with two positions set to -100 (ignored); fp32 logits (the
    # reference's CPU training dtype) and bf16 logits under autocast's fp32 cast.
    g = _gen(5)
    logits = torch.randn(2, 9, 1000, generator=g) * 3
    ids = torch.randint(0, 1000, (2, 9), generator=g)
    ids[0, 4] = -100
    ids[1, 8] = -100
    res = _ce(ce_mod, logits, ids, upcast=False)
    written.append(golden_io.save("ce_f32", {"logits": logits, "input_ids": ids, **res},
                                  {"seed": 5}))
    lb = logits.to(torch.bfloat16)
    res = _ce(ce_mod, lb, ids, upcast=True)
    written.append(golden_io.save("ce_bf16", {"logits": lb, "input_ids": ids, **res},
                                  {"seed": 5}))

    # AdamW through the reference's optimizer-step object: three fp32 parameters, 4 steps,
    # lr 3e-3, betas (0.9, 0.95), eps 1e-8, weight decay 0.1.
    res = _adamw(adamw_mod, [(64, 32), (100,), (7, 13)], 4, 6)
    written.append(golden_io.save("adamw_f32", res,
                                  {"seed": 6, "steps": 4, "lr": 3e-3, "beta1": 0.9,
                                   "beta2": 0.95, "eps": 1e-8, "weight_decay": 0.1}))

    # BASELINE config 3 family, bf16: gate, up ~ N(0,1) * 2, dy ~ N(0,1), [16, 1024].
    g = _gen(0)
    gate = (torch.randn(16, 1024, generator=g) * 2).to(torch.bfloat16)
    up = (torch.randn(16, 1024, generator=g) * 2).to(torch.bfloat16)
    dy = torch.randn(16, 1024, generator=g).to(torch.bfloat16)
    res = _swiglu(swiglu_ref, gate, up, dy)
    written.append(golden_io.save("swiglu_bf16", {"gate": gate, "up": up, "dy": dy, **res},
                                  {"seed": 0}))

    # BASELINE config 4 family, bf16: q as [B, S, H, D] = [2, 16, 4, 32] memory, theta 5e5.
    g = _gen(0)
    q = torch.randn(2, 16, 4, 32, generator=g).to(torch.bfloat16)
    dq = torch.randn(2, 16, 4, 32, generator=g).to(torch.bfloat16)
    res = _rope(rope_mod, q, 500_000.0, dq)
    written.append(golden_io.save("rope_bf16", {"q": q, "dy": dq, **res},
                                  {"theta": 500_000.0, "seed": 0}))

    # fp32 RoPE, the reference test's geometry (tests/test_rope.py: head_dim 8, theta 1e4,
    # 12 positions), with 3 heads and batch 2.
    g = _gen(1)
    q = torch.randn(2, 12, 3, 8, generator=g)
    dq = torch.randn(2, 12, 3, 8, generator=g)
    res = _rope(rope_mod, q, 10_000.0, dq)
    written.append(golden_io.save("rope_f32", {"q": q, "dy": dq, **res},
                                  {"theta": 10_000.0, "seed": 1}))

    manifest = {
        "generator": "tests/golden/make_golden.py",
        "torch": torch.__version__,
        "threads": torch.get_num_threads(),
        "files": {p.name: hashlib.sha256(p.read_bytes()).hexdigest() for p in written},
    }
    (HERE / "MANIFEST.json").write_text(json.dumps(manifest, indent=1) + "\n")
    for p in written:
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
