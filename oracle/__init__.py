"""CPU oracle for the decoder hot path (test infrastructure, never shipped).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this package, and only to check or time the CUDA path.
The product path (``kinetic-rt_b200``) never calls into it.

Modules:
  fused_layer  -- RMSNorm + QKV projection + RoPE, restating the reference's
                  PyTorch functions (tests/test_fusion.py:11-51).
  paged_kv     -- BlockManager address arithmetic and the K/V scatter
                  (include/BlockManager.h:29-95, src/GraphWrapper.cpp:139-145).
  gemm_ar      -- row-parallel sharding (scripts/export_hf.py:62-65) and the
                  allreduce-sum semantics (tests/mock_rccl.h:27-76).
  attention    -- paged decode attention over the pool layout above (no
                  reference counterpart; standard GQA scaled-dot-product).
  bf16         -- bfloat16 <-> float32 conversion with round-to-nearest-even.

Parity pins: tests/golden/ holds vectors produced by the reference's own
PyTorch functions and by its Triton kernel (interpreter mode) together with
the script that made them (tests/golden/make_golden.py).
"""
