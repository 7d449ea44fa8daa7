"""CPU oracle for the Branch Folding verification path (TEST INFRASTRUCTURE).

This package is a plain-numpy restatement of ActFold's per-layer folding
algorithm. It exists only to check the CUDA product: ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import it, nothing under ``actfold_b200/`` does.

Pinning: every function here is checked against golden vectors produced by
running the reference implementation itself (``tests/golden/make_golden.py``
imports ActFold and writes ``tests/golden/*.npz``); the checks live in
``tests/test_oracle_golden.py``.

Modules:
  numerics  -- bf16/fp16 rounding helpers (round-to-nearest-even)
  gate      -- SimilarityGate.forward (actfold/core/similarity_gate.py:43-103)
  rows      -- merge_stable_divergent / gather_cached_activations and the
               stable/divergent compaction (actfold/core/fused_ops.py:38-87, 206-324)
  cache     -- ActivationCache put/get/LRU semantics (actfold/core/activation_cache.py:50-175)
  folding   -- FoldedTransformerLayer.forward (actfold/core/folded_transformer.py:60-203)
  llada     -- LLaDA-architecture block and model arithmetic (restated from the
               architecture description; no LLaDA code ships with the reference)
  demo      -- demo.py's SyntheticTransformerLayer / SyntheticTransformer (demo.py:41-97)
"""
