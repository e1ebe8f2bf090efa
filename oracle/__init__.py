"""CPU oracle for the Qwen3 prefill/decode hot path. TEST INFRASTRUCTURE ONLY.

This package restates, in plain PyTorch on the CPU, the algorithm of the reference engine
(mamadou-wane/inference-performance-engineering, `src/ipe/ops.py`, `src/ipe/forward.py`,
`src/ipe/engine.py`) so that the CUDA path can be checked against it:

- `oracle.qwen3`: the operators, the uncached forward, the fp64 oracle and the cached engine,
  each function citing the reference lines it follows.
- `oracle.accuracy`: the reference's accuracy rule (`tests/needs_torch/accuracy.py:16-45`).

Only `tests/`, `__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference` legs of
`bench.py` may import this package, and only as the checker or the timed CPU baseline. The
product path (`ipe_b200`) never imports it.

Parity pin: `tests/golden/make_golden.py` runs the reference itself and commits its outputs under
`tests/golden/`; `tests/test_oracle.py` checks this restatement against them.
"""
