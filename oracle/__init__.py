"""CPU oracle for the expert-cache hot path.  TEST INFRASTRUCTURE ONLY.

This package is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs may import
it.  The product path (``vllm_expert_cache``) never imports anything from here and fails
loudly when its CUDA library is missing.

Contents
--------
``policy``    pure-Python/numpy restatement of one ``expert_cache_manage`` call, the
              fused remap and the gather (byte copy), state layout identical to the
              C-ABI's.  It follows the reference's numpy model ``ref_step``
              (tests/test_policy.py:83-132) and the kernel it models
              (kernels/expert_cache.hip:191-282, 106-189, 286-314), plus the remap in
              vllm_expert_cache/cache.py:108-110.
``policy.c``  the same step in plain C (fast enough to replay the 4096-step traces and to
              serve as the timed CPU baseline); loaded through ``policy_c``.
``hashing``   the chained state digest used by the golden fixtures.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own ``ref_step``
(extracted from its test file) and its own trace generators
(tests/compare_policies.py:51-73) in the build container and commits their outputs as
fixtures; ``tests/test_oracle.py`` checks both restatements against every fixture and
against the twelve published miss counts (README.md:179-184).
"""
