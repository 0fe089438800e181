"""CPU restatement of BigRig's MoE expert hot path -- TEST INFRASTRUCTURE ONLY.

This package is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The product path (``bigrig_b200``) runs
hand-written sm_100a CUDA through a C-ABI library and raises when that library
is missing; it never routes through anything here.

What each module restates (reference paths are relative to the BigRig tree):

* ``affine``  -- the MLX affine 4/8-bit format the reference stores experts in:
  codes packed little-endian into uint32 words, one fp16/bf16 scale and bias
  per group of 64 input elements, ``w = scale * q + bias``
  (bigrig_engine/stream.py:144-151 manifest ``quant`` block,
  bigrig_engine/direct.py:110-142, tests/test_plan_invariance.py:61-62).
* ``moe``     -- the SwiGLU expert ``down(silu(gate(x)) * up(x))`` over
  dequantised weights, unreduced per (token, k) as StreamingSwitchGLU returns it
  (bigrig_engine/stream.py:1278-1318, 1523-1525), and the router-weighted
  combine the calling MoE block applies afterwards.
* ``router``  -- top-k selection and the two softmax orders the model families
  use (softmax-then-top-k, top-k-then-softmax), summarised by
  bigrig_engine/adapter.py:74-92; the next-layer predictor's softmax/top-m
  (bigrig_engine/stream.py:1436-1439).
* ``permute`` -- the stable token->expert permutation and its inverse
  (bigrig_engine/stream.py:1246-1250, 1275-1276, 1527-1531, 1559-1560).

Parity status: the reference's arithmetic lives in MLX (mlx>=0.29,
mlx-lm>=0.28, floor-pinned in pyproject.toml:31-33, no lockfile), which is not
installed here or on the GPU box.  The formulas above are therefore pinned to
the reference's own by-hand oracle (tests/test_plan_invariance.py:149-160) and
to the manifest byte layouts it ships (data/blobs/*.manifest.json); MLX's own
rounding inside ``mx.dequantize``/``mx.quantized_matmul`` is unpinned.  The
pool and eviction policies are pinned to golden miss counts produced by the
reference's own pure-Python pool/policy code (tests/golden/).
"""
