"""CPU oracle for the qwen3_5 MTP speculative-decoding step — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU in plain torch, the reference's algorithm for the path the
CUDA library implements (giapnguyen74/lollm `src/qwen3_5/*`, `src/generate.py`,
`src/attention.py`), each function citing the reference file:line it follows. It is the
checker, never the product: only `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of `bench.py` may import it. The product path
(`lollm_b200`) never imports it and fails loudly when its CUDA library is missing.

Parity is pinned: `tests/golden/make_golden.py` runs the reference itself (importable in
the development container) on seeded weights/inputs and stores its outputs under
`tests/golden/`; `tests/test_oracle_golden.py` checks this oracle against those fixtures.
Behaviour the reference does not define (k>1 MTP draft chaining, the lossless p/q
speculative sampler driven by caller uniforms, ragged per-sequence cache lengths) is
restated here from its published definition and marked as such where it appears.
"""
