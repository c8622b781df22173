"""Benchmark of the RMSNorm + SwiGLU (+ RoPE) hot path on B200; prints one JSON line.

Default workload: a Llama-3-8B-shaped norm/activation stack, bf16,
32 layers x (2 RMSNorm h4096 + SwiGLU i14336), forward then backward, 16384 tokens per GPU
(4 x 4096), data-parallel over N GPUs; the 64 RMSNorm weight gradients (fp32) are averaged
over the ranks in NCCL all-reduces of 8 layers each (layer 0 alone in the last one), each
issued as soon as the backward has produced its layers and overlapping the backward of the
layers below. Every layer has its own inputs (x for both norms, gate, up, and the upstream
gradients), all larger than L2, so no L2 flush is needed.

Numbers reported (rank 0 prints, other ranks stay silent):
* ``value``: tokens/s of the whole job = N x 16384 / (max over ranks of the CUDA-event
  time of one step), inputs resident in HBM, kernels called through the C ABI.
* ``e2e``: the same metric through the public API (``picotron_b200.kernels``, torch ops
  with autograd), with each step's inputs copied from pinned host memory (on a copy stream,
  each layer's compute starting once its own inputs have landed) and the reduced weight
  gradients read back to the host inside the timed region.
* ``roofline``: the dominant kernel (SwiGLU backward) -- algorithmic bytes per launch /
  its mean CUDA-event duration inside the timed region, against MEASURED_PEAKS.json.
* ``per_kernel``: every kernel of the step, timed in instrumented steps after the timed
  region; ``rope_cfg4``: BASELINE config 4 (RoPE q+k forward and backward);
  ``library_baseline``: the reference's own GPU path (Triton forwards + eager backwards,
  from the reference installed under baseline/_ref) on the same inputs.
* ``cpu_baseline``: the reference's PyTorch CPU path (the reference itself from
  baseline/_ref, else the oracle's eager form) on one full layer of the workload, rank 0 at
  N=1 only.

``--impl reference`` times only that CPU path (rank 0; other ranks exit 0): each "step" is
one full layer at 16384 tokens, and ``value`` extrapolates to the 32-layer stack.

Run: ``python bench.py [--gpus N --steps K --warmup W]``; for N>1 under torchrun.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

# Under torchrun NCCL logs its INIT lines (communicator size, rank, channels, NVLS) into a
# per-process file, which each rank copies to stderr once its communicator exists; set
# before torch loads NCCL, since NCCL reads these once.
if int(os.environ.get("WORLD_SIZE", "1")) > 1:
    if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION", "WARN"):
        os.environ["NCCL_DEBUG"] = "INFO"
    os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
    os.environ["NCCL_DEBUG_FILE"] = f"/tmp/pt_nccl_{os.getpid()}.log"
    # The dweight all-reduces are 32-256 KB, latency-bound, and overlap kernels that fill
    # every SM: without NVLink SHARP (NVLS) their exposed wait stayed at 47-147 us per step in
    # 4 of 4 two-GPU runs, while with it about one run in three waited 1.6-2.4 ms per step
    # throughout (B200, same box and build). The environment can still turn it back on.
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")

import torch

ROOT = Path(__file__).resolve().parent

# The contract is one JSON line on stdout from rank 0. Libraries may print to stdout (NCCL's
# version banner does), so file descriptor 1 points at stderr for the whole run and the
# result line goes to the real stdout, kept here.
_RESULT_OUT = None


def _claim_stdout() -> None:
    global _RESULT_OUT
    if _RESULT_OUT is None:
        sys.stdout.flush()
        _RESULT_OUT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)


def emit(line: dict) -> None:
    """Writes the result line to the real stdout."""

    out = _RESULT_OUT if _RESULT_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def copy_nccl_log_to_stderr(rank: int) -> None:
    path = os.environ.get("NCCL_DEBUG_FILE", "")
    if not path.startswith("/tmp/pt_nccl_"):
        return
    try:
        text = Path(path).read_text()
        Path(path).unlink()
    except OSError:
        return
    block = "".join(f"[rank {rank}] {line}\n" for line in text.splitlines())
    sys.stderr.write(block)  # one write per rank, so ranks do not interleave within a line
    sys.stderr.flush()
METRIC = "RMSNorm+SwiGLU fwd+bwd tokens/s & HBM GB/s (bf16, h4096/i14336) at 1–8 B200"
HIDDEN, INTER = 4096, 14336
EPS = 1e-5
BF16 = 2


# --------------------------------------------------------------------------- helpers --


def measured_peaks(key: str = "hbm_gbs") -> tuple[float, str]:
    """A peak from MEASURED_PEAKS.json (``hbm_gbs``, ``bf16_tflops`` (burst) or
    ``bf16_tflops_sustained`` (seconds of back-to-back GEMMs under the power cap)), else the
    pool's fallback figure."""

    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data[key]), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0,
                "bf16_tflops_sustained": 1400.0}[key], "fallback"


def time_library_adamw(work, steps: int) -> float:
    """ms per step of torch.optim.AdamW.step() on copies of the same parameters."""

    params = [torch.nn.Parameter(p.clone()) for p in work.params]
    for p, g in zip(params, work.grads):
        p.grad = g
    opt = torch.optim.AdamW(params, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    for _ in range(2):
        opt.step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        opt.step()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    del opt, params
    torch.cuda.empty_cache()
    return ms


def time_library_mlpact(work, stream: int, steps: int) -> float:
    """ms per step of the unfused path the two fused GEMMs replace: cuBLAS (torch.matmul) for
    gate, up and d_act = dy @ w_down, and this library's SwiGLU forward and backward kernels."""

    c = work.capi
    n = work.tokens * INTER
    d_act = torch.empty_like(work.act)

    def step(i: int) -> None:
        x, dy = work.x[i % 2], work.dy[i % 2]
        torch.matmul(x, work.wg.t(), out=work.g)
        torch.matmul(x, work.wu.t(), out=work.u)
        c.swiglu_fwd(work.g.data_ptr(), work.u.data_ptr(), work.act.data_ptr(), n,
                     c.PT_BFLOAT16, stream)
        torch.matmul(dy, work.wd, out=d_act)
        c.swiglu_bwd(d_act.data_ptr(), work.g.data_ptr(), work.u.data_ptr(), work.dg.data_ptr(),
                     work.du.data_ptr(), n, c.PT_BFLOAT16, stream)

    for i in range(3):
        step(i)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(steps):
        step(i)
    b.record()
    torch.cuda.synchronize()
    del d_act
    return a.elapsed_time(b) / steps


def time_library_ce(work, steps: int) -> float:
    """ms per step of PyTorch's own cross-entropy forward + backward on the same logits."""

    import torch.nn.functional as F

    def step(i: int) -> None:
        x = work.logits[i % 2].float().requires_grad_(True)
        loss = F.cross_entropy(x, work.targets)
        loss.backward()
        work.dlogits.copy_(x.grad)

    for i in range(2):
        step(i)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(steps):
        step(i)
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def time_library_mlpup(work, stream: int, steps: int) -> float:
    """ms per step of the unfused path the fused GEMM replaces: two cuBLAS GEMMs (torch
    matmul) for gate and up, then this library's SwiGLU forward kernel."""

    c = work.capi
    n = work.tokens * INTER

    def step(i: int) -> None:
        x = work.x[i % 2]
        torch.matmul(x, work.wg.t(), out=work.g)
        torch.matmul(x, work.wu.t(), out=work.u)
        c.swiglu_fwd(work.g.data_ptr(), work.u.data_ptr(), work.act.data_ptr(), n,
                     c.PT_BFLOAT16, stream)

    for i in range(3):
        step(i)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(steps):
        step(i)
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def traffic_per_launch(kernel: str, units: int) -> tuple[float | None, float | None]:
    """(traffic bytes of one launch of ``kernel`` at ``units`` tokens (parameters for AdamW),
    traffic / algorithmic bytes) from the committed ncu table profiles/traffic.json, where
    traffic = DRAM reads + the bytes the SMs store into L2 of one captured launch. The
    table's launch is scaled by units: every kernel's bytes grow in proportion, except the
    gate/up GEMM's two weights, which are read once whatever the tokens."""

    path = ROOT / "profiles" / "traffic.json"
    try:
        entry = json.loads(path.read_text())["kernels"][kernel]
        t = float(entry["traffic_bytes_per_launch"])
        scale = units / float(entry["params"] if "params" in entry else entry["tokens"])
        fixed = 2 * INTER * HIDDEN * BF16 if kernel == "swiglu_gemm" else 0.0
        return (t - fixed) * scale + fixed, float(entry["traffic_over_algorithmic"])
    except Exception:
        return None, None


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuids: list[str]) -> None:
        self.uuids = {u.lower().replace("gpu-", "") for u in uuids}
        self.proc = None
        self.out_path = None

    def __enter__(self):
        try:
            self.out_path = f"/tmp/pt_clocks_{os.getpid()}.csv"
            self.fh = open(self.out_path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.fh, stderr=subprocess.DEVNULL)
            # The first sample can take a second or more on an 8-GPU host: let it land
            # before the timed region starts (at most 5 s).
            deadline = time.monotonic() + 5.0
            while time.monotonic() < deadline and self.proc.poll() is None:
                if Path(self.out_path).stat().st_size > 0:
                    break
                time.sleep(0.05)
        except Exception:
            self.proc = None
        return self

    def mark(self) -> None:
        """Only samples taken after this call count (the timed region starts here)."""

        try:
            self.skip = len(Path(self.out_path).read_text().splitlines())
        except (OSError, TypeError):
            self.skip = 0

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        if self.proc is None or self.out_path is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, sm_max, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in Path(self.out_path).read_text().splitlines()[getattr(self, "skip", 0):]:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            uuid = parts[0].lower().replace("gpu-", "")
            if self.uuids and uuid not in self.uuids:
                continue
            try:
                sm.append(float(parts[1]))
                sm_max.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        try:
            os.unlink(self.out_path)
        except OSError:
            pass
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(sm_max),
                "power_w_max": max(power) if power else None, "samples": len(sm),
                "reasons": sorted(reasons)}


def init_distributed(gpus: int, high_priority_nccl: bool = True):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != gpus:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={world}; launch N>1 under torchrun")
    if world > 1:
        import torch.distributed as dist

        from picotron_b200.dist import nccl_options

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local),
                                pg_options=nccl_options() if high_priority_nccl else None)
        dist.barrier()  # the communicator exists (and has logged its INIT lines) after this
        copy_nccl_log_to_stderr(rank)
    return world, rank, local


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int, device) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- CPU reference path --


REF_DIR = ROOT / "baseline" / "_ref"


def import_reference():
    """The reference package installed under baseline/_ref (pip --target), or None.

    Returns (rms_norm_with_pytorch_forward, swiglu_with_pytorch_forward, triton_rms_norm,
    triton_swiglu) from picotron.nn.triton_kernels, imported from that directory only."""

    if not (REF_DIR / "picotron" / "__init__.py").is_file():
        return None
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import picotron

    if Path(picotron.__file__).resolve().parent != (REF_DIR / "picotron").resolve():
        raise SystemExit(f"'picotron' resolved to {picotron.__file__}, not {REF_DIR}")
    from picotron.nn.triton_kernels.rmsnorm import rms_norm_with_pytorch_forward, triton_rms_norm
    from picotron.nn.triton_kernels.swiglu import swiglu_with_pytorch_forward, triton_swiglu

    return rms_norm_with_pytorch_forward, swiglu_with_pytorch_forward, triton_rms_norm, triton_swiglu


def cpu_reference_layer(tokens: int, seed: int = 0):
    """One layer of the stack (2 RMSNorm + SwiGLU, forward then backward) on the
    reference's PyTorch CPU path, bf16 activations and fp32 weights like the GPU run.

    With the reference installed under baseline/_ref this runs the reference itself:
    ``rms_norm_with_pytorch_forward`` and ``swiglu_with_pytorch_forward``
    (src/picotron/nn/triton_kernels/rmsnorm.py:163, swiglu.py:104, its CPU entry points),
    then one autograd backward through their ``autograd.Function``s (the RMSNorm forward
    saves the inverse RMS and the backward consumes it, rmsnorm.py:95-134). Without it, the
    oracle's eager restatement in the same order (the forward's inverse RMS handed to the
    backward). Returns (run, kind)."""

    g = torch.Generator().manual_seed(seed)
    xs = [torch.randn(tokens, HIDDEN, generator=g).bfloat16() for _ in range(2)]
    dys = [torch.randn(tokens, HIDDEN, generator=g).bfloat16() for _ in range(2)]
    ws = [(1 + 0.02 * torch.randn(HIDDEN, generator=g)) for _ in range(2)]
    gate = (torch.randn(tokens, INTER, generator=g) * 2).bfloat16()
    up = (torch.randn(tokens, INTER, generator=g) * 2).bfloat16()
    dout = torch.randn(tokens, INTER, generator=g).bfloat16()

    ref = import_reference()
    if ref is not None:
        rms_fwd, swiglu_fwd = ref[0], ref[1]
        params = [torch.nn.Parameter(w) for w in ws]

        def run():
            for p in params:
                p.grad = None
            xin = [x.detach().requires_grad_(True) for x in xs]
            gi, ui = gate.detach().requires_grad_(True), up.detach().requires_grad_(True)
            ys = [rms_fwd(x, p, EPS) for x, p in zip(xin, params)]
            out = swiglu_fwd(gi, ui)
            torch.autograd.backward([out, ys[1], ys[0]], [dout, dys[1], dys[0]])

        return run, "reference"

    from oracle import picotron_oracle as po

    def run():
        saved = [po.rms_norm_forward(x, w, EPS, "eager")[1] for x, w in zip(xs, ws)]
        po.swiglu_forward(gate, up, "eager")
        po.swiglu_backward(gate, up, dout, "eager")
        for x, w, dy, inv in zip(xs, ws, dys, saved):
            po.rms_norm_backward(x, w, dy, EPS, "eager", inverse_rms=inv)

    return run, "port"


def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def time_cpu_reference(tokens: int, steps: int, warmup: int, layers: int) -> dict:
    """Times ``steps`` passes of one full layer of the stack on the host cores.

    The timed unit is one layer at ``tokens`` tokens; ``value`` (tokens/s of the whole
    ``layers``-layer stack) is the one extrapolation: mean layer time x ``layers``."""

    cores = cpu_cores()
    torch.set_num_threads(cores)
    run, kind = cpu_reference_layer(tokens)
    for _ in range(warmup):
        run()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    per_layer = statistics.fmean(times)
    value = tokens / (per_layer * layers)
    what = ("the reference itself (baseline/_ref: rms_norm_with_pytorch_forward, "
            "swiglu_with_pytorch_forward, autograd backward)" if kind == "reference" else
            "the oracle's eager restatement of the reference (baseline/_ref not installed)")
    return {
        "value": value,
        "unit": "tokens/s",
        "cores": cores,
        "cpu_model": cpu_model(),
        "kind": kind,
        "sample": (f"1 full layer of the {layers}-layer stack (2 RMSNorm h{HIDDEN} + SwiGLU "
                   f"i{INTER}, fwd+bwd, bf16) at {tokens} tokens, {what}; mean of {steps} "
                   f"after {warmup} warm-up; tokens/s = {tokens} / (mean layer time x {layers})"),
        "seconds_per_layer": per_layer,
        "layer_times_s": times,
        "extrapolation": {"timed_unit": f"1 layer x {tokens} tokens", "layers_timed": 1,
                          "layers": layers, "factor": layers},
    }


# ----------------------------------------------------------------------- GPU stack --


class Stack:
    """Device-resident inputs of the config-5 stack and its step through the C ABI."""

    def __init__(self, layers: int, tokens: int, device: torch.device, seed: int,
                 fused_dw: bool = False) -> None:
        from picotron_b200 import _capi
        from picotron_b200.dist import DWeightBucket

        self.capi = _capi
        self.lib = _capi.library()
        self.layers, self.tokens, self.device = layers, tokens, device
        gen = torch.Generator(device=device).manual_seed(seed)
        bf = torch.bfloat16
        self.x = torch.randn((layers, 2, tokens, HIDDEN), generator=gen, device=device, dtype=bf)
        self.dy = torch.randn((layers, 2, tokens, HIDDEN), generator=gen, device=device, dtype=bf)
        self.gate = torch.randn((layers, tokens, INTER), generator=gen, device=device, dtype=bf)
        self.gate.mul_(2)
        self.up = torch.randn((layers, tokens, INTER), generator=gen, device=device, dtype=bf)
        self.up.mul_(2)
        self.dout = torch.randn((layers, tokens, INTER), generator=gen, device=device, dtype=bf)
        self.w = 1 + 0.02 * torch.randn((layers, 2, HIDDEN), generator=gen, device=device)
        # outputs are write-only here; their consumers (GEMMs) are outside this path
        # Two buffers per output, alternated by layer (dx by norm): consecutive kernels never
        # write the same addresses, so no kernel's stores can merge in L2 with the last one's.
        self.y = [torch.empty((tokens, HIDDEN), device=device, dtype=bf) for _ in range(2)]
        self.dx = [torch.empty((tokens, HIDDEN), device=device, dtype=bf) for _ in range(2)]
        self.act = [torch.empty((tokens, INTER), device=device, dtype=bf) for _ in range(2)]
        self.dg = [torch.empty((tokens, INTER), device=device, dtype=bf) for _ in range(2)]
        self.du = [torch.empty((tokens, INTER), device=device, dtype=bf) for _ in range(2)]
        self.bucket = DWeightBucket([HIDDEN] * (2 * layers), device)
        self.num_partials = _capi.rmsnorm_bwd_num_partials(tokens, HIDDEN, _capi.PT_BFLOAT16,
                                                           _capi.PT_FLOAT32)
        self.partials = torch.empty((self.num_partials, HIDDEN), device=device,
                                    dtype=torch.float32)
        # The RMSNorm backward and the dweight reduce as two launches (the default: 3 % faster
        # per norm on B200 than one cooperative launch, whose grid barrier costs more than the
        # kernel boundary it saves), or both in one launch (--rms-bwd fused).
        self.fused_dw = fused_dw
        self.workspace = torch.zeros(
            _capi.rmsnorm_bwd_fused_workspace(tokens, HIDDEN, _capi.PT_BFLOAT16,
                                              _capi.PT_FLOAT32), device=device)
        self.launches_per_step = layers * (6 if fused_dw else 8)
        # All-reduce buckets of the dweights, by first layer: 8 layers (16 norms, 256 KB)
        # each, except that layer 0 forms its own bucket (2 norms, 32 KB). The backward runs
        # from the last layer down, so each bucket's all-reduce overlaps the backward of the
        # layers below it; only layer 0's small one is left at the end of the step.
        self.bucket_starts = sorted(s for s in {0, 1} | set(range(0, layers, 8)) if s < layers)
        # When a list, each step appends the (start, end) events around its final waits for
        # the all-reduces: the collective time the backward did not hide.
        self.wait_events: list | None = None
        self.events_per_step = layers  # one (start, end) pair per SwiGLU backward launch
        self.dominant = ("swiglu_bwd_vec32 (SwiGLU backward)", 5 * tokens * INTER * BF16)
        self.traffic_key = "swiglu_bwd"
        t = tokens
        # Algorithmic bytes of one launch of each kernel of the step (inputs read once,
        # outputs written once); the dweight reduce moves its fp32 partial rows.
        self.kernel_bytes = {
            "rmsnorm_fwd": 2 * t * HIDDEN * BF16,
            "swiglu_fwd": 3 * t * INTER * BF16,
            "swiglu_bwd": 5 * t * INTER * BF16,
            "rmsnorm_bwd": 3 * t * HIDDEN * BF16,
            "rmsnorm_dw_reduce": self.num_partials * HIDDEN * 4,
        }

    # algorithmic bytes (each input read once, each output written once)
    def bytes_per_step(self) -> int:
        t = self.tokens
        rms = 2 * t * HIDDEN * BF16 + 3 * t * HIDDEN * BF16          # fwd + bwd
        swi = 3 * t * INTER * BF16 + 5 * t * INTER * BF16
        return self.layers * (2 * rms + swi)

    def _check(self, status: int, name: str) -> None:
        if status != 0:
            raise RuntimeError(f"{name}: {self.capi.last_error()}")

    def _launch(self, name: str, timer: dict | None, fn) -> None:
        if timer is None:
            self._check(fn(), name)
            return
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        self._check(fn(), name)
        b.record()
        timer.setdefault(name, []).append((a, b))

    def step_launches(self, stream: int) -> dict:
        """The launches of one step grouped by kernel, in step order, each a callable that
        returns the C ABI status (no collectives)."""

        lib, L, T = self.lib, self.layers, self.tokens
        f32, b16 = self.capi.PT_FLOAT32, self.capi.PT_BFLOAT16
        y = [t.data_ptr() for t in self.y]
        act = [t.data_ptr() for t in self.act]
        part, P = self.partials.data_ptr(), self.num_partials
        ws, ws_floats = self.workspace.data_ptr(), self.workspace.numel()
        out: dict = {}

        def add(name, fn):
            out.setdefault(name, []).append(fn)

        for l in range(L):
            for k in range(2):
                add("rmsnorm_fwd", lambda l=l, k=k: lib.pt_rmsnorm_fwd(
                    self.x[l, k].data_ptr(), HIDDEN, self.w[l, k].data_ptr(), y[k], HIDDEN, None,
                    T, HIDDEN, b16, f32, EPS, stream))
            add("swiglu_fwd", lambda l=l: lib.pt_swiglu_fwd(
                self.gate[l].data_ptr(), self.up[l].data_ptr(), act[l % 2], T * INTER, b16, stream))
        for l in reversed(range(L)):
            add("swiglu_bwd", lambda l=l: lib.pt_swiglu_bwd(
                self.dout[l].data_ptr(), self.gate[l].data_ptr(), self.up[l].data_ptr(),
                self.dg[l % 2].data_ptr(), self.du[l % 2].data_ptr(), T * INTER, b16, stream))
            for k in (1, 0):
                if self.fused_dw:
                    add("rmsnorm_bwd", lambda l=l, k=k: lib.pt_rmsnorm_bwd_fused(
                        self.dy[l, k].data_ptr(), HIDDEN, self.x[l, k].data_ptr(), HIDDEN,
                        self.w[l, k].data_ptr(), None, self.dx[k].data_ptr(), HIDDEN,
                        self.bucket.slot(2 * l + k).data_ptr(), ws, ws_floats, T, HIDDEN, b16,
                        f32, EPS, stream))
                    continue
                add("rmsnorm_bwd", lambda l=l, k=k: lib.pt_rmsnorm_bwd(
                    self.dy[l, k].data_ptr(), HIDDEN, self.x[l, k].data_ptr(), HIDDEN,
                    self.w[l, k].data_ptr(), None, self.dx[k].data_ptr(), HIDDEN, part, P, T,
                    HIDDEN, b16, f32, EPS, stream))
                add("rmsnorm_dw_reduce", lambda l=l, k=k: lib.pt_rmsnorm_dw_reduce(
                    part, P, HIDDEN, self.bucket.slot(2 * l + k).data_ptr(), f32, stream))
        return out

    def step(self, stream: int, world: int, swiglu_bwd_events: list | None = None,
             timer: dict | None = None) -> None:
        """One forward + backward of the stack. ``swiglu_bwd_events``: (start, end) event
        pairs recorded around the SwiGLU backward launches. ``timer``: when given, every
        launch is bracketed by events, collected per kernel name (an instrumented step)."""

        lib, L, T = self.lib, self.layers, self.tokens
        f32, b16 = self.capi.PT_FLOAT32, self.capi.PT_BFLOAT16
        y = [t.data_ptr() for t in self.y]
        act = [t.data_ptr() for t in self.act]
        for l in range(L):
            for k in range(2):
                self._launch("rmsnorm_fwd", timer, lambda: lib.pt_rmsnorm_fwd(
                    self.x[l, k].data_ptr(), HIDDEN, self.w[l, k].data_ptr(), y[k], HIDDEN, None,
                    T, HIDDEN, b16, f32, EPS, stream))
            self._launch("swiglu_fwd", timer, lambda: lib.pt_swiglu_fwd(
                self.gate[l].data_ptr(), self.up[l].data_ptr(), act[l % 2], T * INTER, b16, stream))
        part, P = self.partials.data_ptr(), self.num_partials
        ws, ws_floats = self.workspace.data_ptr(), self.workspace.numel()
        pending = []
        starts = self.bucket_starts
        for l in reversed(range(L)):
            if swiglu_bwd_events is not None:
                start, end = swiglu_bwd_events[l]
                start.record()
            self._launch("swiglu_bwd", timer, lambda: lib.pt_swiglu_bwd(
                self.dout[l].data_ptr(), self.gate[l].data_ptr(), self.up[l].data_ptr(),
                self.dg[l % 2].data_ptr(), self.du[l % 2].data_ptr(), T * INTER, b16, stream))
            if swiglu_bwd_events is not None:
                end.record()
            for k in (1, 0):
                if self.fused_dw:
                    self._launch("rmsnorm_bwd", timer, lambda: lib.pt_rmsnorm_bwd_fused(
                        self.dy[l, k].data_ptr(), HIDDEN, self.x[l, k].data_ptr(), HIDDEN,
                        self.w[l, k].data_ptr(), None, self.dx[k].data_ptr(), HIDDEN,
                        self.bucket.slot(2 * l + k).data_ptr(), ws, ws_floats, T, HIDDEN, b16,
                        f32, EPS, stream))
                    continue
                self._launch("rmsnorm_bwd", timer, lambda: lib.pt_rmsnorm_bwd(
                    self.dy[l, k].data_ptr(), HIDDEN, self.x[l, k].data_ptr(), HIDDEN,
                    self.w[l, k].data_ptr(), None, self.dx[k].data_ptr(), HIDDEN, part, P, T,
                    HIDDEN, b16, f32, EPS, stream))
                self._launch("rmsnorm_dw_reduce", timer, lambda: lib.pt_rmsnorm_dw_reduce(
                    part, P, HIDDEN, self.bucket.slot(2 * l + k).data_ptr(), f32, stream))
            if l in starts:
                # This bucket's layers are done: average their dweights over the ranks on
                # the process group's stream while the earlier layers' backward runs.
                i = starts.index(l)
                stop = starts[i + 1] if i + 1 < len(starts) else L
                pending.append(self.bucket.all_reduce_async(2 * l, 2 * stop))
        if self.wait_events is not None:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
        for p in pending:
            p.wait()
        if self.wait_events is not None:
            b.record()
            self.wait_events.append((a, b))


class OpWorkload:
    """One hot-path op (3, 4) forward + backward per step through the C
    ABI, on `tokens` rows with rotating input sets larger than L2. Used for per-kernel
    measurement and for small ncu captures; the default workload is the stack."""

    def __init__(self, op: str, tokens: int, device: torch.device, seed: int,
                 fused_dw: bool = False, adamw_layers: int = 4) -> None:
        from picotron_b200 import _capi

        self.capi, self.lib, self.op, self.tokens, self.device = _capi, _capi.library(), op, tokens, device
        self.fused_dw = fused_dw
        gen = torch.Generator(device=device).manual_seed(seed)
        bf = torch.bfloat16
        sets = 3
        if op == "rmsnorm":
            self.x = [torch.randn((tokens, HIDDEN), generator=gen, device=device, dtype=bf)
                      for _ in range(sets)]
            self.dy = [torch.randn((tokens, HIDDEN), generator=gen, device=device, dtype=bf)
                       for _ in range(sets)]
            self.w = 1 + 0.02 * torch.randn(HIDDEN, generator=gen, device=device)
            self.y = torch.empty((tokens, HIDDEN), device=device, dtype=bf)
            self.dx = torch.empty_like(self.y)
            self.dw = torch.empty(HIDDEN, device=device)
            self.P = _capi.rmsnorm_bwd_num_partials(tokens, HIDDEN, _capi.PT_BFLOAT16, _capi.PT_FLOAT32)
            self.part = torch.empty((self.P, HIDDEN), device=device)
            self.ws = torch.zeros(_capi.rmsnorm_bwd_fused_workspace(
                tokens, HIDDEN, _capi.PT_BFLOAT16, _capi.PT_FLOAT32), device=device)
            self.bytes = 5 * tokens * HIDDEN * BF16
            self.launches_per_step = 2 if fused_dw else 3
            self.dominant = ("rmsnorm_ws (backward, with the dweight reduction)",
                             3 * tokens * HIDDEN * BF16)
        elif op == "addnorm":
            # Fused residual add + RMSNorm (the next-step row): h = res + branch, y = norm(h);
            # backward dx = norm_bwd(dy, h) + dh. Config 2 shapes and distributions.
            mk = lambda: [torch.randn((tokens, HIDDEN), generator=gen, device=device, dtype=bf)
                          for _ in range(sets)]
            self.res, self.br, self.dy, self.dhs = mk(), mk(), mk(), mk()
            self.w = 1 + 0.02 * torch.randn(HIDDEN, generator=gen, device=device)
            self.h = [torch.empty((tokens, HIDDEN), device=device, dtype=bf) for _ in range(sets)]
            self.y = torch.empty((tokens, HIDDEN), device=device, dtype=bf)
            self.dx = torch.empty_like(self.y)
            self.dw = torch.empty(HIDDEN, device=device)
            self.P = _capi.add_rmsnorm_bwd_num_partials(tokens, HIDDEN, _capi.PT_BFLOAT16,
                                                        _capi.PT_FLOAT32)
            self.part = torch.empty((self.P, HIDDEN), device=device)
            self.ws = torch.zeros(_capi.add_rmsnorm_bwd_fused_workspace(
                tokens, HIDDEN, _capi.PT_BFLOAT16, _capi.PT_FLOAT32), device=device)
            self.bytes = 8 * tokens * HIDDEN * BF16
            self.launches_per_step = 2 if fused_dw else 3
            self.dominant = ("rmsnorm_ws (fused add, backward, with the dweight reduction)",
                             4 * tokens * HIDDEN * BF16)
        elif op == "mlpup":
            # SwiGLU fused into the gate/up GEMM (the next-step row): x [tokens, 4096] bf16,
            # w_gate, w_up [14336, 4096] bf16; act, gate and up written (the training forward).
            k = HIDDEN
            self.x = [torch.randn((tokens, k), generator=gen, device=device, dtype=bf)
                      for _ in range(2)]
            self.wg = torch.randn((INTER, k), generator=gen, device=device, dtype=bf) * 2 * k ** -0.5
            self.wu = torch.randn((INTER, k), generator=gen, device=device, dtype=bf) * 2 * k ** -0.5
            self.act = torch.empty((tokens, INTER), device=device, dtype=bf)
            self.g, self.u = torch.empty_like(self.act), torch.empty_like(self.act)
            self.flops = 2 * 2 * tokens * INTER * k
            self.bytes = (tokens * k + 2 * INTER * k + 3 * tokens * INTER) * BF16
            self.launches_per_step = 1
            self.dominant = ("swiglu_gemm_kernel", self.flops)
        elif op == "mlpact":
            # The MLP's activation in training, both directions on the tensor cores: the gate/up
            # GEMMs with the SwiGLU epilogue (act, gate, up written), then the down
            # projection's input gradient d_act = dy @ w_down with the SwiGLU backward in its
            # epilogue (dgate, dup written), w_down transposed once per step for it.
            k = HIDDEN
            self.x = [torch.randn((tokens, k), generator=gen, device=device, dtype=bf)
                      for _ in range(2)]
            self.dy = [torch.randn((tokens, k), generator=gen, device=device, dtype=bf)
                       for _ in range(2)]
            self.wg = torch.randn((INTER, k), generator=gen, device=device, dtype=bf) * 2 * k ** -0.5
            self.wu = torch.randn((INTER, k), generator=gen, device=device, dtype=bf) * 2 * k ** -0.5
            self.wd = torch.randn((k, INTER), generator=gen, device=device, dtype=bf) * 2 * INTER ** -0.5
            self.wdt = torch.empty((INTER, k), device=device, dtype=bf)
            self.act = torch.empty((tokens, INTER), device=device, dtype=bf)
            self.g, self.u = torch.empty_like(self.act), torch.empty_like(self.act)
            self.dg, self.du = torch.empty_like(self.act), torch.empty_like(self.act)
            self.flops = 2 * 2 * tokens * INTER * k + 2 * tokens * INTER * k
            # fwd: x, w_gate, w_up in, act, gate, up out; w_down transposed (in + out); bwd:
            # dy, w_down^T, gate, up in, dgate, dup out.
            self.bytes = ((tokens * k + 2 * INTER * k + 3 * tokens * INTER) + 2 * INTER * k
                          + (tokens * k + INTER * k + 4 * tokens * INTER)) * BF16
            self.launches_per_step = 3
            self.dominant = ("swiglu_gemm_bwd_pair_kernel (d_act GEMM + SwiGLU backward)",
                             2 * tokens * INTER * k)
        elif op == "ce":
            # Cross-entropy forward + backward over a Llama-3 vocabulary (the next-step row):
            # logits [tokens, 128256] bf16 ~ N(0, 2^2), uniform targets.
            self.vocab = 128256
            self.logits = [torch.randn((tokens, self.vocab), generator=gen, device=device,
                                       dtype=bf) * 2 for _ in range(2)]
            self.targets = torch.randint(0, self.vocab, (tokens,), generator=gen, device=device)
            self.row_loss = torch.empty(tokens, device=device)
            self.row_lse = torch.empty(tokens, device=device)
            self.mean = torch.empty(2, device=device)
            self.dlogits = torch.empty_like(self.logits[0])
            self.bytes = 3 * tokens * self.vocab * BF16
            self.launches_per_step = 3
            self.dominant = ("ce_bwd_kernel", 2 * tokens * self.vocab * BF16)
        elif op == "adamw":
            # One fused AdamW step over the fp32 parameters of 4 Llama-3-8B decoder layers
            # (q, k, v, o, gate, up, down projections and the two norm weights per layer:
            # 218 M parameters a layer), lr 3e-4, betas (0.9, 0.95), eps 1e-8, wd 0.1.
            shapes = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096),
                      (14336, 4096), (4096, 14336), (4096,), (4096,)] * adamw_layers
            self.params = [torch.randn(s_, generator=gen, device=device) for s_ in shapes]
            self.grads = [torch.randn(s_, generator=gen, device=device) for s_ in shapes]
            self.m = [torch.zeros(s_, device=device) for s_ in shapes]
            self.v = [torch.zeros(s_, device=device) for s_ in shapes]
            self.nparams = sum(p_.numel() for p_ in self.params)
            self.step_count = 0
            self.bytes = 28 * self.nparams
            self.launches_per_step = 1
            self.units, self.unit = self.nparams, "params/s"
            self.dominant = ("adamw_kernel", 28 * self.nparams)
        elif op == "swiglu":
            mk = lambda scale: [torch.randn((tokens, INTER), generator=gen, device=device, dtype=bf) * scale
                                for _ in range(sets)]
            self.g, self.u, self.do = mk(2.0), mk(2.0), mk(1.0)
            self.out = torch.empty((tokens, INTER), device=device, dtype=bf)
            self.dg, self.du = torch.empty_like(self.out), torch.empty_like(self.out)
            self.bytes = 8 * tokens * INTER * BF16
            self.launches_per_step = 2
            self.dominant = ("swiglu_bwd_vec32", 5 * tokens * INTER * BF16)
        elif op in ("rope", "rope_rh"):
            op_name = op
            # rope: the reference's interleaved pairs; rope_rh: the rotate-half pairing that
            # BASELINE config 4 names (same bytes, same kernel, other pair layout).
            self.rope_layout = (_capi.PT_ROPE_ROTATE_HALF if op == "rope_rh"
                                else _capi.PT_ROPE_INTERLEAVED)
            op = self.op = "rope"
            # BASELINE config 4 per 2048-token sequence: q [B,S,32,128], k [B,S,8,128] memory.
            b = max(1, tokens // 2048)
            self.q = [torch.randn((b, 2048, 32, 128), generator=gen, device=device, dtype=bf)
                      for _ in range(sets)]
            self.k = [torch.randn((b, 2048, 8, 128), generator=gen, device=device, dtype=bf)
                      for _ in range(sets)]
            self.qo, self.ko = torch.empty_like(self.q[0]), torch.empty_like(self.k[0])
            from picotron_b200.modules import rotary_cos_sin

            self.cos, self.sin = rotary_cos_sin(2048, 128, 500000.0, device=device, dtype=bf)
            self.bytes = 4 * (self.q[0].numel() + self.k[0].numel()) * BF16
            self.launches_per_step = 2
            kernel = "rope_vec" if op_name == "rope_rh" else "rope_rows"
            self.dominant = (f"{kernel} (q and k, forward)",
                             2 * (self.q[0].numel() + self.k[0].numel()) * BF16)
            self.tokens = b * 2048
        else:
            raise SystemExit(f"unknown workload {op}")
        self.i = 0
        self.events_per_step = 1
        if not hasattr(self, "units"):
            self.units, self.unit = self.tokens, "tokens/s"
        self.traffic_key = {"rmsnorm": "rmsnorm_bwd", "swiglu": "swiglu_bwd", "rope": "rope_fwd",
                            "addnorm": "add_rmsnorm_bwd", "mlpup": "swiglu_gemm",
                            "mlpact": "swiglu_gemm_bwd",
                            "ce": "ce_bwd", "adamw": "adamw"}[op]

    def bytes_per_step(self) -> int:
        return self.bytes

    def rope_launch(self, direction: str, i: int, stream: int) -> None:
        """One query+key RoPE launch on input set i: forward from (q, k) into (qo, ko),
        backward from (qo, ko) into (q, k), on the attention layer's [B, H, S, D] view."""

        c = self.capi
        if direction == "fwd":
            q, k, qo, ko = self.q[i], self.k[i], self.qo, self.ko
        else:
            q, k, qo, ko = self.qo, self.ko, self.q[i], self.k[i]
        qv, kv, qov, kov = q.transpose(1, 2), k.transpose(1, 2), qo.transpose(1, 2), ko.transpose(1, 2)
        c.rope_qk(direction, qv.data_ptr(), qv.stride(), qov.data_ptr(), qov.stride(), qv.shape,
                  kv.data_ptr(), kv.stride(), kov.data_ptr(), kov.stride(), kv.shape,
                  self.cos.data_ptr(), self.sin.data_ptr(), self.cos.stride(0), self.rope_layout,
                  c.PT_BFLOAT16, c.PT_BFLOAT16, stream)

    def _check(self, status: int, name: str) -> None:
        if status != 0:
            raise RuntimeError(f"{name}: {self.capi.last_error()}")

    def step(self, stream: int, world: int, dominant_events: list | None = None) -> None:
        lib, c, T = self.lib, self.capi, self.tokens
        i = self.i % 3
        self.i += 1
        ev = dominant_events[0] if dominant_events else None
        if self.op == "rmsnorm":
            self._check(lib.pt_rmsnorm_fwd(self.x[i].data_ptr(), HIDDEN, self.w.data_ptr(),
                                           self.y.data_ptr(), HIDDEN, None, T, HIDDEN,
                                           c.PT_BFLOAT16, c.PT_FLOAT32, EPS, stream), "fwd")
            if ev: ev[0].record()
            if self.fused_dw:
                self._check(lib.pt_rmsnorm_bwd_fused(
                    self.dy[i].data_ptr(), HIDDEN, self.x[i].data_ptr(), HIDDEN, self.w.data_ptr(),
                    None, self.dx.data_ptr(), HIDDEN, self.dw.data_ptr(), self.ws.data_ptr(),
                    self.ws.numel(), T, HIDDEN, c.PT_BFLOAT16, c.PT_FLOAT32, EPS, stream), "bwd")
                if ev: ev[1].record()
                return
            self._check(lib.pt_rmsnorm_bwd(self.dy[i].data_ptr(), HIDDEN, self.x[i].data_ptr(),
                                           HIDDEN, self.w.data_ptr(), None, self.dx.data_ptr(),
                                           HIDDEN, self.part.data_ptr(), self.P, T, HIDDEN,
                                           c.PT_BFLOAT16, c.PT_FLOAT32, EPS, stream), "bwd")
            self._check(lib.pt_rmsnorm_dw_reduce(self.part.data_ptr(), self.P, HIDDEN,
                                                 self.dw.data_ptr(), c.PT_FLOAT32, stream), "red")
            if ev: ev[1].record()
        elif self.op == "addnorm":
            self._check(lib.pt_add_rmsnorm_fwd(self.res[i].data_ptr(), HIDDEN, self.br[i].data_ptr(),
                                               HIDDEN, self.w.data_ptr(), self.h[i].data_ptr(),
                                               HIDDEN, self.y.data_ptr(), HIDDEN, None, T, HIDDEN,
                                               c.PT_BFLOAT16, c.PT_FLOAT32, EPS, stream), "fwd")
            if ev: ev[0].record()
            if self.fused_dw:
                self._check(lib.pt_add_rmsnorm_bwd_fused(
                    self.dy[i].data_ptr(), HIDDEN, self.dhs[i].data_ptr(), HIDDEN,
                    self.h[i].data_ptr(), HIDDEN, self.w.data_ptr(), None, self.dx.data_ptr(),
                    HIDDEN, self.dw.data_ptr(), self.ws.data_ptr(), self.ws.numel(), T, HIDDEN,
                    c.PT_BFLOAT16, c.PT_FLOAT32, EPS, stream), "bwd")
                if ev: ev[1].record()
                return
            self._check(lib.pt_add_rmsnorm_bwd(self.dy[i].data_ptr(), HIDDEN, self.dhs[i].data_ptr(),
                                               HIDDEN, self.h[i].data_ptr(), HIDDEN,
                                               self.w.data_ptr(), None, self.dx.data_ptr(), HIDDEN,
                                               self.part.data_ptr(), self.P, T, HIDDEN,
                                               c.PT_BFLOAT16, c.PT_FLOAT32, EPS, stream), "bwd")
            self._check(lib.pt_rmsnorm_dw_reduce(self.part.data_ptr(), self.P, HIDDEN,
                                                 self.dw.data_ptr(), c.PT_FLOAT32, stream), "red")
            if ev: ev[1].record()
        elif self.op == "mlpup":
            if ev: ev[0].record()
            x = self.x[i % 2]
            c.swiglu_gemm_fwd(x.data_ptr(), HIDDEN, self.wg.data_ptr(), self.wu.data_ptr(), HIDDEN,
                              self.act.data_ptr(), INTER, self.g.data_ptr(), self.u.data_ptr(),
                              INTER, T, INTER, HIDDEN, c.PT_BFLOAT16, stream)
            if ev: ev[1].record()
        elif self.op == "mlpact":
            x, dy = self.x[i % 2], self.dy[i % 2]
            c.swiglu_gemm_fwd(x.data_ptr(), HIDDEN, self.wg.data_ptr(), self.wu.data_ptr(), HIDDEN,
                              self.act.data_ptr(), INTER, self.g.data_ptr(), self.u.data_ptr(),
                              INTER, T, INTER, HIDDEN, c.PT_BFLOAT16, stream)
            c.transpose_2d(self.wd.data_ptr(), INTER, self.wdt.data_ptr(), HIDDEN, HIDDEN, INTER,
                           c.PT_BFLOAT16, stream)
            if ev: ev[0].record()
            c.swiglu_gemm_bwd(dy.data_ptr(), HIDDEN, self.wdt.data_ptr(), HIDDEN, self.g.data_ptr(),
                              self.u.data_ptr(), INTER, self.dg.data_ptr(), self.du.data_ptr(),
                              INTER, None, 0, T, INTER, HIDDEN, c.PT_BFLOAT16, stream)
            if ev: ev[1].record()
        elif self.op == "ce":
            lg = self.logits[i % 2]
            c.cross_entropy_fwd(lg.data_ptr(), self.vocab, T, 1, (self.vocab, 0),
                                self.targets.data_ptr(), (1, 0), -100, self.row_loss.data_ptr(),
                                self.row_lse.data_ptr(), self.mean.data_ptr(), c.PT_BFLOAT16,
                                stream)
            if ev: ev[0].record()
            c.cross_entropy_bwd(lg.data_ptr(), self.vocab, T, 1, (self.vocab, 0),
                                self.targets.data_ptr(), (1, 0), -100, self.row_lse.data_ptr(),
                                self.mean.data_ptr(), None, self.dlogits.data_ptr(),
                                (self.vocab, 0), c.PT_BFLOAT16, stream)
            if ev: ev[1].record()
        elif self.op == "adamw":
            self.step_count += 1
            n = len(self.params)
            if ev: ev[0].record()
            c.adamw_step([p_.data_ptr() for p_ in self.params],
                         [g_.data_ptr() for g_ in self.grads],
                         [m_.data_ptr() for m_ in self.m], [v_.data_ptr() for v_ in self.v],
                         [p_.numel() for p_ in self.params], [self.step_count] * n, [3e-4] * n,
                         [0.1] * n, 0.9, 0.95, 1e-8, False, stream)
            if ev: ev[1].record()
        elif self.op == "swiglu":
            n = T * INTER
            self._check(lib.pt_swiglu_fwd(self.g[i].data_ptr(), self.u[i].data_ptr(),
                                          self.out.data_ptr(), n, c.PT_BFLOAT16, stream), "fwd")
            if ev: ev[0].record()
            self._check(lib.pt_swiglu_bwd(self.do[i].data_ptr(), self.g[i].data_ptr(),
                                          self.u[i].data_ptr(), self.dg.data_ptr(),
                                          self.du.data_ptr(), n, c.PT_BFLOAT16, stream), "bwd")
            if ev: ev[1].record()
        else:
            # Query and key in one launch per direction, as RotaryEmbedding.forward calls it.
            if dominant_events is None:
                self.rope_launch("fwd", i, stream)
                self.rope_launch("bwd", i, stream)
                return
            # Events: the first pair brackets the forward launch, a second pair (if given)
            # the backward launch.
            for d, (q, k, qo, ko, direction) in enumerate(
                    ((self.q[i], self.k[i], self.qo, self.ko, "fwd"),
                     (self.qo, self.ko, self.q[i], self.k[i], "bwd"))):
                qv, kv = q.transpose(1, 2), k.transpose(1, 2)
                qov, kov = qo.transpose(1, 2), ko.transpose(1, 2)
                pair = dominant_events[d] if dominant_events and d < len(dominant_events) else None
                if pair: pair[0].record()
                c.rope_qk(direction, qv.data_ptr(), qv.stride(), qov.data_ptr(), qov.stride(),
                          qv.shape, kv.data_ptr(), kv.stride(), kov.data_ptr(), kov.stride(),
                          kv.shape, self.cos.data_ptr(), self.sin.data_ptr(), self.cos.stride(0),
                          self.rope_layout, c.PT_BFLOAT16, c.PT_BFLOAT16, stream)
                if pair: pair[1].record()


def per_kernel_block(stack: Stack, stream: int, world: int, steps: int, peak: float) -> dict:
    """Mean duration of every kernel of the stack's step, after the timed region: for each
    kernel, its launches of one step (over the stack's own inputs, in step order) run back
    to back between one pair of CUDA events, ``steps`` times; max over ranks. One event pair
    per kernel keeps event overhead out of the per-launch figure."""

    out = {}
    total_us = 0.0
    for name, fns in stack.step_launches(stream).items():
        for fn in fns[:2]:
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            for fn in fns:
                stack._check(fn(), name)
        b.record()
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1e3 / (steps * len(fns))
        us = max_over_ranks(us, world, stack.device)
        nbytes = stack.kernel_bytes[name]
        gbs = nbytes / (us * 1e-6) / 1e9
        out[name] = {"launches_per_step": len(fns), "mean_us": us, "bytes_per_launch": nbytes,
                     "gbs": gbs, "frac_of_hbm_peak": gbs / peak}
        total_us += us * len(fns)
    out["sum_us_per_step"] = total_us
    out["how"] = (f"after the timed region: each kernel's launches of one step, over the "
                  f"stack's inputs, back to back between one event pair, {steps} times; mean "
                  "per launch, max over ranks")
    return out


def rope_cfg4_block(device, stream: int, world: int, steps: int, warmup: int,
                    peak: float) -> dict:
    """BASELINE config 4 (q [8,2048,32,128], k [8,2048,8,128] bf16 in the attention layer's
    [B,S,H,D] memory, theta 5e5, positions 0..2047): the query+key RoPE launch forward and
    backward, CUDA events around each, for the reference's interleaved pairs and for the
    rotate-half pairing config 4 names."""

    out = {}
    for op, label in (("rope", "interleaved"), ("rope_rh", "rotate_half")):
        work = OpWorkload(op, 16384, device, seed=4321)
        for _ in range(warmup):
            work.step(stream, world)
        torch.cuda.synchronize()
        us = {}
        for direction in ("fwd", "bwd"):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for i in range(steps):
                work.rope_launch(direction, i % 3, stream)
            b.record()
            torch.cuda.synchronize()
            us[direction] = max_over_ranks(a.elapsed_time(b) * 1e3 / steps, world, device)
        launch_bytes = work.bytes // 2
        out[label] = {
            "fwd_us": us["fwd"], "bwd_us": us["bwd"],
            "bytes_per_launch": launch_bytes,
            "fwd_frac_of_hbm_peak": launch_bytes / (us["fwd"] * 1e-6) / 1e9 / peak,
            "bwd_frac_of_hbm_peak": launch_bytes / (us["bwd"] * 1e-6) / 1e9 / peak,
            "tokens_per_s_fwd_bwd": work.tokens / ((us["fwd"] + us["bwd"]) * 1e-6),
            "kernel": "rope_rows" if op == "rope" else "rope_vec",
        }
        del work
    out["how"] = (f"after {warmup} warm-up steps, {steps} launches per direction back to back "
                  "over 3 rotating input sets (each larger than L2) between one event pair, "
                  "max over ranks")
    torch.cuda.empty_cache()
    return out


def time_reference_gpu_stack(stack: Stack, steps: int, warmup: int, world: int) -> dict:
    """The reference's own GPU path on the same inputs: its Triton RMSNorm and SwiGLU
    forwards and its eager PyTorch backwards (``triton_rms_norm`` and ``triton_swiglu`` of
    src/picotron/nn/triton_kernels/{rmsnorm,swiglu}.py, imported from the reference
    installed under baseline/_ref), all layers forward then all backward, as the stack runs.
    The dweight all-reduce is left out (per-rank timing only). Nothing of this repository
    runs on that path."""

    why = None
    ms = float("inf")
    try:
        ref = import_reference()
        if ref is None:
            why = "the reference is not installed under baseline/_ref"
        else:
            _, _, rms_ref, swiglu_ref = ref
            weights = [torch.nn.Parameter(stack.w[l, k].clone()) for l in range(stack.layers)
                       for k in range(2)]

            def one_step():
                for w in weights:
                    w.grad = None
                saved = []
                for l in range(stack.layers):
                    xa = stack.x[l, 0].detach().requires_grad_(True)
                    xm = stack.x[l, 1].detach().requires_grad_(True)
                    g = stack.gate[l].detach().requires_grad_(True)
                    u = stack.up[l].detach().requires_grad_(True)
                    saved.append((rms_ref(xa, weights[2 * l], EPS),
                                  rms_ref(xm, weights[2 * l + 1], EPS), swiglu_ref(g, u)))
                for l in reversed(range(stack.layers)):
                    ya, ym, out = saved.pop()
                    torch.autograd.backward([out, ym, ya],
                                            [stack.dout[l], stack.dy[l, 1], stack.dy[l, 0]])

            for _ in range(warmup):
                one_step()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(steps):
                one_step()
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / steps
            del weights
    except Exception as exc:  # recorded, not raised: the reference may not run here
        why = f"{type(exc).__name__}: {str(exc).splitlines()[0] if str(exc) else ''}"[:300]
    torch.cuda.empty_cache()
    ms = max_over_ranks(ms, world, stack.device)  # every rank takes this collective
    if why is not None or ms == float("inf"):
        return {"unavailable": why or "failed on another rank"}
    return {
        "what": ("the reference's GPU path: Triton forwards + eager PyTorch backwards "
                 "(triton_rms_norm, triton_swiglu from baseline/_ref), same inputs, all 32 "
                 "layers, without the dweight all-reduce"),
        "ms_per_step": ms,
        "steps": steps,
        "value": world * stack.tokens / (ms / 1e3),
        "unit": "tokens/s",
    }


def e2e_run(stack: Stack, steps: int, warmup: int, world: int) -> dict:
    """The stack through the public API with host inputs (see the module docstring)."""

    from picotron_b200.kernels import triton_rms_norm, triton_swiglu

    dev = stack.device
    T = stack.tokens
    pin = dict(
        x=torch.empty((2, T, HIDDEN), dtype=torch.bfloat16).pin_memory(),
        dy=torch.empty((2, T, HIDDEN), dtype=torch.bfloat16).pin_memory(),
        gate=torch.empty((T, INTER), dtype=torch.bfloat16).pin_memory(),
        up=torch.empty((T, INTER), dtype=torch.bfloat16).pin_memory(),
        dout=torch.empty((T, INTER), dtype=torch.bfloat16).pin_memory(),
    )
    # Host copies of layer 0's inputs; every layer's device buffers are refilled from them.
    pin["x"].copy_(stack.x[0])
    pin["dy"].copy_(stack.dy[0])
    pin["gate"].copy_(stack.gate[0])
    pin["up"].copy_(stack.up[0])
    pin["dout"].copy_(stack.dout[0])
    weights = [torch.nn.Parameter(stack.w[l, k].clone()) for l in range(stack.layers)
               for k in range(2)]
    result_host = torch.empty(stack.bucket.buffer.numel(), dtype=torch.float32).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in pin.values()) * stack.layers
    d2h = result_host.numel() * 4

    copy_stream = torch.cuda.Stream(device=dev)

    def one_step():
        for w in weights:
            w.grad = None
        # Host-to-device copies run on their own stream, each layer's compute waiting only
        # for its own inputs, so the compute of layer l overlaps the copies of the layers
        # after it (an input pipeline's prefetch). The copy stream first waits for everything
        # the compute stream has queued, so no buffer is overwritten while still in use.
        main = torch.cuda.current_stream(dev)
        copy_stream.wait_stream(main)
        ready = []
        with torch.cuda.stream(copy_stream):
            for l in range(stack.layers):
                stack.x[l].copy_(pin["x"], non_blocking=True)
                stack.dy[l].copy_(pin["dy"], non_blocking=True)
                stack.gate[l].copy_(pin["gate"], non_blocking=True)
                stack.up[l].copy_(pin["up"], non_blocking=True)
                stack.dout[l].copy_(pin["dout"], non_blocking=True)
                event = torch.cuda.Event()
                event.record(copy_stream)
                ready.append(event)
        for l in range(stack.layers):
            main.wait_event(ready[l])
            xa = stack.x[l, 0].detach().requires_grad_(True)
            xm = stack.x[l, 1].detach().requires_grad_(True)
            g = stack.gate[l].detach().requires_grad_(True)
            u = stack.up[l].detach().requires_grad_(True)
            ya = triton_rms_norm(xa, weights[2 * l], EPS)
            ym = triton_rms_norm(xm, weights[2 * l + 1], EPS)
            out = triton_swiglu(g, u)
            torch.autograd.backward([out, ym, ya],
                                    [stack.dout[l], stack.dy[l, 1], stack.dy[l, 0]])
        torch.cat([w.grad for w in weights], out=stack.bucket.buffer)
        stack.bucket.all_reduce()
        result_host.copy_(stack.bucket.buffer)  # synchronous read of the step's result

    for _ in range(warmup):
        one_step()
    torch.cuda.synchronize()
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        one_step()
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world, dev) / steps
    return {"value": world * T / (ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": ms, "steps": steps,
            "path": "picotron_b200.kernels.triton_rms_norm / triton_swiglu (torch ops + autograd)"}


# ------------------------------------------------------------------------------ main --


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: 30 for the stack, 300 for mlpup / mlpact, and "
                         "for the other per-op workloads as many as fill about 0.6 s, so that "
                         "the clock sampler sees the timed region)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--tokens", type=int, default=16384, help="tokens per GPU")
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--rms-bwd", choices=["fused", "pair"], default="pair",
                    help="RMSNorm backward: dweight reduced by a second kernel (pair, the "
                         "faster on B200) or in the same cooperative launch (fused)")
    ap.add_argument("--nccl-stream", choices=["high", "normal"], default="high",
                    help="priority of the NCCL stream that runs the dweight all-reduces")
    ap.add_argument("--adamw-layers", type=int, default=4,
                    help="adamw: Llama-3-8B decoder layers whose parameters are stepped")
    ap.add_argument("--no-extras", action="store_true",
                    help="stack: skip the config-4 RoPE block and the reference GPU path")
    ap.add_argument("--cpu-tokens", type=int, default=16384,
                    help="tokens of the one layer the CPU reference path times")
    ap.add_argument("--workload", choices=["stack", "rmsnorm", "swiglu", "rope", "rope_rh", "addnorm", "mlpup",
                                           "mlpact", "ce", "adamw"],
                    default="stack",
                    help="stack = BASELINE config 5 (the headline); rmsnorm, swiglu, rope are "
                         "configs 2, 3 and 4, one op forward+backward per step, for per-kernel "
                         "measurement; addnorm = fused residual add + RMSNorm at config 2 shapes; "
                         "mlpup = the gate/up GEMMs with the SwiGLU epilogue (tcgen05); "
                         "ce = cross-entropy forward + backward over a 128256 vocabulary; "
                         "adamw = one fused AdamW step over 4 Llama-3-8B layers of parameters")
    args = ap.parse_args()
    auto_steps = args.steps is None
    if args.steps is None:
        args.steps = 300 if args.workload in ("mlpup", "mlpact") else 30
    _claim_stdout()
    if args.workload != "stack":
        args.no_e2e = True
        args.no_cpu_baseline = True
    if args.warmup < 3 and args.impl == "ours":
        print("note: warm-up raised to the minimum of 3 steps", file=sys.stderr)
        args.warmup = 3

    names = {"stack": "llama3-8b norm/act stack (BASELINE config 5)",
             "rmsnorm": "RMSNorm fwd+bwd bf16 h4096 (BASELINE config 2)",
             "swiglu": "SwiGLU fwd+bwd bf16 i14336 (BASELINE config 3)",
             "rope": "RoPE q+k fwd+bwd bf16 (BASELINE config 4), interleaved pairs (reference)",
             "rope_rh": "RoPE q+k fwd+bwd bf16 (BASELINE config 4), rotate-half pairs",
             "addnorm": "fused residual add + RMSNorm fwd+bwd bf16 h4096 (config 2 shapes)",
             "mlpup": "gate/up GEMMs + SwiGLU epilogue fwd bf16 4096->14336 (config 3/5 shapes)",
             "mlpact": ("MLP activation fwd+bwd on the tensor cores bf16 (config 3/5 shapes): "
                        "gate/up GEMMs + SwiGLU epilogue, d_act GEMM + SwiGLU backward epilogue"),
             "ce": "cross-entropy fwd+bwd bf16, vocab 128256 (Llama-3 head)",
             "adamw": (f"AdamW step, fp32 params of {args.adamw_layers} Llama-3-8B decoder "
                       f"layers ({218.2 * args.adamw_layers:.0f} M)")}
    config = {
        "workload": names[args.workload],
        "layers": args.layers,
        "tokens_per_gpu": args.tokens,
        "hidden": HIDDEN,
        "intermediate": INTER,
        "global_batch": max(1, args.gpus * args.tokens // 4096),
        "seq_len": 4096,
        "parallelism": f"dp{args.gpus}",
        "eps": EPS,
        "weight_dtype": "float32",
        "nccl_stream": f"{args.nccl_stream} priority",
        "nccl_nvls": os.environ.get("NCCL_NVLS_ENABLE", "default") if args.gpus > 1 else None,
        "rmsnorm_backward": ("dweight reduced in the same launch" if args.rms_bwd == "fused"
                             else "dweight reduced by a second kernel, launched as a "
                                  "programmatic dependent of the backward"),
        "l2": "no flush: every layer has its own inputs, each larger than the 126 MB L2",
    }

    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        ref = time_cpu_reference(args.cpu_tokens, args.steps, args.warmup, args.layers)
        # A "step" of this arm is the timed unit it ran: one full layer of the stack at
        # --cpu-tokens tokens. Only `value` extrapolates, to the 32-layer stack.
        line = {
            "metric": METRIC, "impl": "reference", "value": ref["value"], "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ref["seconds_per_layer"] * 1e3,
            "step_unit": ref["extrapolation"]["timed_unit"],
            "extrapolation": ref["extrapolation"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) inputs of the BASELINE shapes)",
            "config": dict(config, tokens_per_gpu=args.cpu_tokens),
            "cpu_baseline": {k: ref[k] for k in ("value", "unit", "cores", "cpu_model", "kind",
                                                 "sample")},
            "e2e": {"value": ref["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
        emit(line)
        return

    world, rank, local = init_distributed(args.gpus, args.nccl_stream == "high")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    import picotron_b200  # noqa: F401  (loads the library; fails loudly if it is missing)
    from picotron_b200 import _capi

    status, major, minor, sms = _capi.probe(local)
    if status != 0:
        raise SystemExit(f"device rejected: {_capi.last_error()}")

    if args.workload == "stack":
        work = Stack(args.layers, args.tokens, device, seed=1234 + rank,
                     fused_dw=args.rms_bwd == "fused")
    else:
        work = OpWorkload(args.workload, args.tokens, device, seed=1234 + rank,
                          fused_dw=args.rms_bwd == "fused", adamw_layers=args.adamw_layers)
    stream = torch.cuda.current_stream(device).cuda_stream
    torch.cuda.synchronize()

    for _ in range(args.warmup):
        work.step(stream, world)
    torch.cuda.synchronize()
    if auto_steps and world == 1 and args.workload not in ("stack", "mlpup", "mlpact"):
        # Per-op workloads take well under a millisecond per step: without --steps, time as
        # many as fill about 0.6 s, so that the clock sampler sees the timed region.
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(3):
            work.step(stream, world)
        b.record()
        torch.cuda.synchronize()
        args.steps = max(args.steps, int(math.ceil(600.0 / max(a.elapsed_time(b) / 3, 1e-3))))

    E = work.events_per_step
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(E * args.steps)]
    # The GPUs this job runs on (local rank r uses device r): idle GPUs of a larger box must
    # not enter the clock record.
    uuids = []
    for i in range(min(world, torch.cuda.device_count())):
        try:
            uuids.append(str(torch.cuda.get_device_properties(i).uuid))
        except Exception:
            pass
    if args.workload == "stack" and world > 1:
        work.wait_events = []
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(uuids if rank == 0 else []) as clocks:
        clocks.mark()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for s in range(args.steps):
            work.step(stream, world, ev[s * E:(s + 1) * E])
        end.record()
        torch.cuda.synchronize()
        barrier(world)
    elapsed = start.elapsed_time(end)
    ms = max_over_ranks(elapsed, world, device) / args.steps
    exposed_us = None
    if getattr(work, "wait_events", None):
        exposed_us = max_over_ranks(
            statistics.fmean(a.elapsed_time(b) for a, b in work.wait_events) * 1e3, world, device)
        work.wait_events = None
    dom_ms = statistics.fmean(a.elapsed_time(b) for a, b in ev)
    dom_ms = max_over_ranks(dom_ms, world, device)

    peak, peak_kind = measured_peaks()
    bytes_step = work.bytes_per_step()
    dom_name, dom_bytes = work.dominant
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9
    traffic, traffic_ratio = traffic_per_launch(
        work.traffic_key, work.nparams if args.workload == "adamw" else work.tokens)
    tensor_bound = args.workload in ("mlpup", "mlpact")
    library_ms = None
    library_what = None
    if args.workload == "adamw":
        library_ms = time_library_adamw(work, args.steps)
        library_what = ("torch.optim.AdamW.step() (its default CUDA multi-tensor path, what "
                        "the reference runs) on the same parameters")
    if args.workload == "ce":
        library_ms = time_library_ce(work, args.steps)
        library_what = ("PyTorch F.cross_entropy forward + backward on the bf16 logits "
                        "upcast to fp32 (what CUDA autocast runs)")
    if tensor_bound:
        # A tensor-core contraction: FLOPs per launch over the cuBLAS bf16 peak. The step is
        # 32 layers of GEMMs back to back (seconds of tensor-core work over the timed steps),
        # which runs under the 1 kW power cap at a lower SM clock than a burst: the sustained
        # figure is the denominator; the burst fraction is reported beside it.
        achieved = dom_bytes / (dom_ms / 1e3) / 1e12
        tpeak, tpeak_kind = measured_peaks("bf16_tflops_sustained")
        tburst, _ = measured_peaks("bf16_tflops")
        if args.workload == "mlpup":
            library_ms = time_library_mlpup(work, stream, args.steps)
            library_what = "cuBLAS gate and up GEMMs (torch.matmul) + this library's SwiGLU kernel"
        else:
            library_ms = time_library_mlpact(work, stream, args.steps)
            library_what = ("cuBLAS gate, up and d_act GEMMs (torch.matmul) + this library's "
                            "SwiGLU forward and backward kernels")

    per_kernel = rope_cfg4 = reference_gpu = None
    if args.workload == "stack":
        # Untimed extras, after the timed region: every kernel of the step on its own
        # clock, config 4 (RoPE), and the reference's own GPU path on the same inputs.
        per_kernel = per_kernel_block(work, stream, world, 2, peak)
        if not args.no_extras:
            rope_cfg4 = rope_cfg4_block(device, stream, world, 30, 3, peak)
            reference_gpu = time_reference_gpu_stack(work, 3, 2, world)

    e2e = None
    if not args.no_e2e:
        e2e = e2e_run(work, max(1, args.e2e_steps), 1, world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ref = time_cpu_reference(args.cpu_tokens, 3, 1, args.layers)
        cpu = {k: ref[k] for k in ("value", "unit", "cores", "cpu_model", "kind", "sample",
                                   "extrapolation")}

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": world * getattr(work, "units", work.tokens) / (ms / 1e3),
            "unit": getattr(work, "unit", "tokens/s"),
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) inputs of the BASELINE shapes, on device)",
            "config": config,
            "hbm_gbs_per_gpu": bytes_step / (ms / 1e3) / 1e9,
            "hbm_frac_per_gpu": bytes_step / (ms / 1e3) / 1e9 / peak,
            "roofline": {
                "kernel": dom_name,
                "bound": "hbm",
                "achieved": achieved,
                "peak": peak,
                "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                "unit": "GB/s",
                "frac": achieved / peak,
                "traffic": traffic,
                "traffic_over_algorithmic": traffic_ratio,
                "traffic_source": "profiles/traffic.json: ncu DRAM reads + SM-issued L2 writes",
                "algorithmic_bytes_per_launch": dom_bytes,
                "mean_launch_us": dom_ms * 1e3,
            } if not tensor_bound else {
                "kernel": dom_name,
                "bound": "tensor",
                "achieved": achieved,
                "peak": tpeak,
                "peak_source": f"{tpeak_kind} bf16_tflops_sustained (MEASURED_PEAKS.json): "
                               "cuBLAS bf16 GEMMs back to back for seconds, under the power cap",
                "unit": "TFLOP/s",
                "frac": achieved / tpeak,
                "burst_peak": tburst,
                "frac_of_burst": achieved / tburst,
                "traffic": traffic,
                "traffic_over_algorithmic": traffic_ratio,
                "traffic_source": "profiles/traffic.json: ncu DRAM reads + SM-issued L2 writes",
                "algorithmic_flops_per_launch": dom_bytes,
                "mean_launch_us": dom_ms * 1e3,
            },
            "library_baseline": reference_gpu if library_ms is None else {
                "what": library_what,
                "ms_per_step": library_ms,
                "value": world * getattr(work, "units", work.tokens) / (library_ms / 1e3),
                "unit": getattr(work, "unit", "tokens/s"),
            },
            "per_kernel": per_kernel,
            "dweight_allreduce": None if args.workload != "stack" or world == 1 else {
                "buckets_per_step": len(work.bucket_starts),
                "last_bucket": "layer 0 (2 norms, 32 KB)",
                "exposed_us_per_step": exposed_us,
                "how": "CUDA events around the step's final waits for its all-reduces (the "
                       "time the compute stream waits for NCCL after its last kernel), mean "
                       "over the timed steps, max over ranks",
            },
            "rope_cfg4": rope_cfg4,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": work.launches_per_step * args.steps,
            "clocks": clocks.summary() if rank == 0 else None,
        }
        emit(line)

    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
