"""CPU oracle for the minifield-training hot path (TEST INFRASTRUCTURE ONLY).

This package is a NumPy restatement of the reference algorithms that the CUDA
kernels in ``minifield_training_b200`` replace. It exists to check those
kernels and to time a CPU baseline. Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference`` arm) may
import it, and only as the checker or the timed CPU baseline. The product
package never imports it and has no CPU fallback.

Parity pinning: the reference (Python/JAX, jax 0.7.2) cannot be imported here
because jax is not installed. The oracle is pinned instead against every
known-answer test the reference's own test-suite holds for this path
(``tests/kernels/test_attention.py``, ``test_bidirectional.py``,
``test_quantization.py``, ``test_linear.py``); those values live in
``tests/golden/`` together with the script that writes them. The int8
per-channel and int4 group-128 fake quantizers have no reference
implementation: their parity is unpinned and follows the stated definition.

Modules:
  attention  -- masked GQA attention forward/backward (dense, packed, prefix,
                bidirectional, cached) with the reference's mask semantics.
  quant      -- fake quantizers: reference ternary/NF4 g128 (FP16 scale) and
                int8 per-channel / int4 g128 symmetric with STE masks.
  linear     -- full_linear and the SwiGLU QAT FFN forward/backward.
  decode     -- KV-cache append + single-query cached attention.
  bf16       -- round-to-nearest-even bfloat16 helpers.
"""
