"""CPU oracle for the RMSNorm / SwiGLU / RoPE hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and
its ``--impl reference`` arm) may import this package, and only as the checker or as the
timed CPU baseline. The product (``picotron_b200``) never imports it and has no code path
that runs it.

``picotron_oracle`` restates the reference's arithmetic (picotron, the files cited in each
function) in two forms:

* ``eager``: the reference's own PyTorch CPU arithmetic op for op, in the reference's
  dtypes (what ``rms_norm_with_pytorch_forward`` / ``swiglu_with_pytorch_forward`` /
  ``apply_rotary_embedding`` compute on CPU). This is the timed CPU baseline.
* ``exact``: the same formulas evaluated in float64 from the same (already rounded)
  inputs, left unrounded. This is the tolerance target for the CUDA kernels.

Pinning: ``tests/golden/make_golden.py`` imports the reference itself and records its
outputs on seeded inputs into ``tests/golden/*.npz``; ``tests/test_oracle_golden.py``
checks the eager form against those outputs bit for bit and the exact form within the
fp32 tolerance.
"""
