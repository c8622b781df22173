"""The hot path under CUDA graph capture.

A decoder block's hot-path pieces (RMSNorm, the fused residual add + RMSNorm, the SwiGLU
activation, the tcgen05 gate/up GEMM and the down projection's fused input gradient, RoPE on
q and k), forward and backward through the drop-in modules and ops, are captured once in a
torch CUDA graph and replayed on new inputs. Every kernel of the path is deterministic, so a replay gives the same bits as an
eager call on the same inputs. The capture includes the RMSNorm backward's dweight reduce,
which is launched as a programmatic dependent of the backward kernel, and no host
synchronisation may happen inside the path (capture fails on one).
"""

from __future__ import annotations

import pytest
import torch

import gpu_utils as gu
import picotron_b200 as pb
from picotron_b200 import _capi
from picotron_b200.modules import RMSNorm, RotaryEmbedding

pytestmark = pytest.mark.gpu

B, S, H, I, HEADS, KV_HEADS, D = 2, 64, 1024, 2048, 8, 2, 128


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    gu.require_gpu()


def _modules():
    norm = RMSNorm(H, eps=1e-5, use_triton_rmsnorm=True).to(gu.DEV)
    norm2 = RMSNorm(H, eps=1e-5, use_triton_rmsnorm=True).to(gu.DEV)
    rope = RotaryEmbedding(D, theta=500_000.0, use_triton_rope=True)
    with torch.no_grad():
        norm.weight.copy_(gu.randn(H, 90, torch.float32, 0.02, 1.0))
        norm2.weight.copy_(gu.randn(H, 91, torch.float32, 0.02, 1.0))
    w_gate = gu.randn((I, H), 92, torch.bfloat16, H ** -0.5)
    w_up = gu.randn((I, H), 93, torch.bfloat16, H ** -0.5)
    w_down = gu.randn((H, I), 94, torch.bfloat16, I ** -0.5)
    return norm, norm2, rope, w_gate, w_up, w_down


def _block(mods, x, branch, dz, dh, gate, up, dout, dy_down, q_mem, k_mem, dq):
    """Forward + backward of the pieces (this library's kernels only, no library GEMM whose
    algorithm choice could differ under capture); returns every output and gradient."""

    norm, norm2, rope, w_gate, w_up, w_down = mods
    x = x.detach().requires_grad_(True)
    branch = branch.detach().requires_grad_(True)
    gate = gate.detach().requires_grad_(True)
    up = up.detach().requires_grad_(True)
    q_mem = q_mem.detach().requires_grad_(True)
    # Fused residual add + RMSNorm, then RMSNorm, forward and backward.
    h, y = norm2.forward_with_residual(x, branch)
    z = norm(y)
    dx, dbranch, dw, dw2 = torch.autograd.grad((z, h), (x, branch, norm.weight, norm2.weight),
                                               (dz, dh))
    # SwiGLU activation, forward and backward.
    act = pb.triton_swiglu(gate, up)
    dgate, dup = torch.autograd.grad(act, (gate, up), dout)
    # The tcgen05 gate/up GEMM with the SwiGLU epilogue, and the down projection's input
    # gradient with the SwiGLU backward in its epilogue.
    act_k, gate_k, up_k = torch.ops.picotron_b200.swiglu_gate_up(z.detach().view(-1, H), w_gate,
                                                                 w_up)
    dgate_k, dup_k = torch.ops.picotron_b200.swiglu_down_backward(dy_down, w_down, gate_k, up_k)
    # RoPE on q and k in the attention layout, forward and backward.
    qo, ko = rope(q_mem.transpose(1, 2), k_mem.transpose(1, 2))
    (dq_mem,) = torch.autograd.grad(qo, (q_mem,), dq)
    # Detached, so that no output keeps this call's autograd graph alive into the next call.
    return tuple(t.detach() for t in (h, y, z, dx, dbranch, dw, dw2, act, dgate, dup, act_k,
                                      gate_k, up_k, dgate_k, dup_k, qo, ko, dq_mem))


def _inputs(seed):
    bf = torch.bfloat16
    return (gu.randn((B, S, H), seed, bf), gu.randn((B, S, H), seed + 1, bf),
            gu.randn((B, S, H), seed + 2, bf), gu.randn((B, S, H), seed + 3, bf),
            gu.randn((B * S, I), seed + 4, bf, 2.0), gu.randn((B * S, I), seed + 5, bf, 2.0),
            gu.randn((B * S, I), seed + 6, bf), gu.randn((B * S, H), seed + 7, bf),
            gu.randn((B, S, HEADS, D), seed + 8, bf), gu.randn((B, S, KV_HEADS, D), seed + 9, bf),
            gu.randn((B, HEADS, S, D), seed + 10, bf))


def test_block_replays_bit_exact():
    mods = _modules()
    static = _inputs(1)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm-up: kernel attributes, RoPE tables, allocator pools
        for _ in range(2):
            _block(mods, *static)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = _block(mods, *static)
    for seed in (11, 21, 31):
        fresh = _inputs(seed)
        for dst, src in zip(static, fresh):
            dst.copy_(src)
        graph.replay()
        replayed = [t.clone() for t in captured]
        eager = _block(mods, *fresh)
        torch.cuda.synchronize()
        for i, (got, want) in enumerate(zip(replayed, eager)):
            assert got.shape == want.shape and torch.equal(got, want), f"output {i}, seed {seed}"
    # A second replay on the same inputs gives the same bits again.
    graph.replay()
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip(replayed, captured))
    assert _capi.take_device_error() == 0
    del graph
