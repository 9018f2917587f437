"""CPU oracle for the duo mixer hot path.  TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference's algorithms for the token-mixing hot path of its Qwen3.5 engine.
It is the checker that the CUDA path is compared against, and the CPU baseline that bench.py times beside it.
Nothing in the product path (the `duo` package and its CUDA library) may import it: only `tests/`,
`__graft_entry__.smoke()` and bench.py's CPU-baseline / reference arm do.

Modules
  q8      int8 group quantisation, dequantisation, matvec and embedding gather, restated from the reference's WGSL
          (engine/kernels.js:5-47, 55-94, 205-221) in numpy.  Pinned by known-answer tests that follow the WGSL
          semantics (round half to even, zero groups get scale 1).
  mixer   Gated DeltaNet and gated attention ops in torch fp32 on the CPU, restated from the third-party module the
          reference's PyTorch tools run (Hugging Face transformers 5.5.0, models/qwen3_5/modeling_qwen3_5.py) and
          from the reference's WGSL (engine/kernels_qwen35.js).  Pinned against outputs of that module, committed as
          fixtures under tests/golden/ together with the script that made them.
  model   The full Qwen3.5 text decoder forward with the engine's row/position/push/vec semantics
          (engine/model.js:404-466), on dequantised int8 weights or float weights.
  hf      Harness around the transformers model itself (random init, forced pure-torch paths, push and vec hooks as
          in tests/engine_ref.py).  Only usable where transformers is importable.
"""
