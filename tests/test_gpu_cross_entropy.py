"""Cross-entropy forward/backward kernels (pt_cross_entropy_fwd / _bwd) vs the oracle.

The mean loss is held to the float64 oracle with the fp32 tolerance (1e-5 abs + 1e-5 rel),
the logits gradient with the tolerance of its dtype (oracle/tolerance.py: fp32 1e-5 abs +
1e-5 rel; bf16/fp16 2 ulp of the float64 value plus a 2^-16 * max|ref| floor).
"""

from __future__ import annotations

import pytest
import torch
from torch.nn import functional as F

import golden_io
import gpu_utils as gu
from oracle import picotron_oracle as po
from oracle import tolerance
from picotron_b200 import _capi
from picotron_b200.kernels import CrossEntropyWithFallback, triton_cross_entropy

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    gu.require_gpu()


def _targets(shape, vocab, seed, ignore_every=0):
    g = torch.Generator().manual_seed(seed)
    t = torch.randint(0, vocab, shape, generator=g)
    if ignore_every:
        t.view(-1)[::ignore_every] = -100
    return t.to(gu.DEV)


def _check(logits, targets, what, grad=None):
    loss, _, d = gu.cross_entropy(logits, targets, grad=grad)
    torch.cuda.synchronize()
    assert _capi.take_device_error() == 0, what
    tolerance.assert_close(loss, po.cross_entropy_forward(logits, targets, mode="exact"),
                           f"{what} loss", torch.float32)
    de = po.cross_entropy_backward(logits, targets, 1.0 if grad is None else grad, mode="exact")
    tolerance.assert_close(d, de, f"{what} dlogits")
    return loss, d


@pytest.mark.parametrize("case", ["ce_f32", "ce_bf16"])
def test_golden_fixtures_training_view(case):
    t, _ = golden_io.load(case)
    logits, ids = t["logits"].to(gu.DEV), t["input_ids"].to(gu.DEV)
    view, targets = logits[:, :-1, :].transpose(1, 2), ids[:, 1:]   # strided, read in place
    loss, d = _check(view, targets, case)
    tolerance.assert_close(loss, t["loss"].double(), f"{case} loss vs reference", torch.float32)
    full = torch.zeros_like(logits)
    full[:, :-1, :] = d.transpose(1, 2)
    tolerance.assert_close(full, t["dlogits"].double(), f"{case} dlogits vs reference",
                           logits.dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16],
                         ids=["f32", "bf16", "f16"])
@pytest.mark.parametrize("rows,vocab", [(1, 1), (5, 7), (64, 1000), (33, 50257), (8, 128256),
                                        (300, 4096)])
def test_shapes_dtypes_and_ignored_rows(dtype, rows, vocab):
    logits = gu.randn((rows, vocab), 101, dtype, scale=4.0)
    targets = _targets((rows,), vocab, 102, ignore_every=5 if rows > 5 else 0)
    _check(logits, targets, f"{dtype} {rows}x{vocab}", grad=0.5)


def test_misaligned_and_strided_rows():
    vocab = 1001
    base = gu.randn((40, vocab + 3), 103, torch.bfloat16, scale=3.0)
    logits = base[:, 1:1 + vocab]                         # odd row stride, 2-byte offset
    targets = _targets((40,), vocab, 104, ignore_every=7)
    _check(logits, targets, "misaligned")


def test_out_of_range_target_poisons_the_loss():
    logits = gu.randn((4, 100), 105, torch.float32)
    targets = torch.tensor([1, 2, 100, 3], device=gu.DEV)
    loss, rows, _ = gu.cross_entropy(logits, targets, want_grad=False)
    torch.cuda.synchronize()
    assert torch.isnan(loss) and torch.isnan(rows[2]) and torch.isfinite(rows[[0, 1, 3]]).all()
    assert _capi.take_device_error() == 2
    assert _capi.take_device_error() == 0


def test_all_ignored_is_nan_like_pytorch():
    logits = gu.randn((3, 10), 106, torch.float32)
    targets = torch.full((3,), -100, device=gu.DEV)
    loss, _, _ = gu.cross_entropy(logits, targets, want_grad=False)
    assert torch.isnan(loss) and torch.isnan(F.cross_entropy(logits, targets))


def test_module_and_autograd_on_the_training_call():
    # CrossEntropyWithFallback as the training loop calls it, under bf16 autocast.
    b, s, v = 2, 65, 32000
    logits = gu.randn((b, s, v), 107, torch.bfloat16, scale=3.0).requires_grad_(True)
    ids = _targets((b, s), v, 108)
    loss_fn = CrossEntropyWithFallback(use_triton=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss = loss_fn(logits[:, :-1, :].transpose(1, 2), ids[:, 1:])
    assert loss.dtype == torch.float32 and not loss_fn._fallback_warned
    (loss * 3.0).backward()
    view = logits.detach()[:, :-1, :].transpose(1, 2)
    tolerance.assert_close(loss, po.cross_entropy_forward(view, ids[:, 1:], mode="exact"),
                           "module loss", torch.float32)
    de = po.cross_entropy_backward(view, ids[:, 1:], 3.0, mode="exact")
    full = torch.zeros(logits.shape, dtype=torch.float64, device=gu.DEV)
    full[:, :-1, :] = de.transpose(1, 2)
    tolerance.assert_close(logits.grad, full, "module dlogits")
    # The reference's function name, 2-D and inference-style.
    flat = logits.detach()[:, 0, :]
    with torch.no_grad():
        l2 = triton_cross_entropy(flat, ids[:, 0])
    assert l2.dtype == torch.bfloat16
    torch.testing.assert_close(l2.float(), F.cross_entropy(flat.float(), ids[:, 0]),
                               rtol=8e-3, atol=0)


def test_llama_vocab_full_size():
    # 16384 tokens x 128256 vocabulary, bf16 (4.2 GB of logits): exact float64 parity on a
    # row sample, the whole mean against PyTorch's fp32 loss.
    n, v = 16384, 128256
    logits = gu.randn((n, v), 109, torch.bfloat16, scale=2.0)
    targets = _targets((n,), v, 110)
    loss, rows, d = gu.cross_entropy(logits, targets)
    torch.cuda.synchronize()
    sample = torch.arange(0, n, 97, device=gu.DEV)
    x = logits[sample].double()
    lse = torch.logsumexp(x, dim=1)
    exact_rows = lse - x.gather(1, targets[sample].unsqueeze(1)).squeeze(1)
    tolerance.assert_close(rows[sample], exact_rows, "row losses (sample)", torch.float32)
    p = torch.softmax(x, dim=1)
    p[torch.arange(sample.numel(), device=gu.DEV), targets[sample]] -= 1.0
    gu.full_size_parity(d[sample], p / n, "llama vocab ce dlogits (row sample)", cancels=True)
    del x, p
    ref = F.cross_entropy(logits.float(), targets)
    assert abs(loss.item() - ref.item()) <= 1e-5 * abs(ref.item()) + 1e-5
    del d
    torch.cuda.empty_cache()
