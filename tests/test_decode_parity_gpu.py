"""End-to-end greedy decode through vLLM: the cached model against the fully resident one.

A 4-layer model with the Qwen3-30B-A3B layer shapes (hidden 2048, 32q/4kv x 128, 128
experts of moe_intermediate 768, top-8), random-init W8A8 int8 experts, loaded through the
product's own ``vllm.general_plugins`` entry point.  Both engines run vLLM's deterministic
(batch-invariant) kernels and replay the same sticky-Zipf routing trace in every layer, so
the cache really churns: 16 of 128 experts fit, and every decode step installs experts
over the host link.  The 128-token prefill is wider than the slots and reads through.

Pinned: the greedy tokens are identical to the resident run's and the chosen tokens'
logprobs are within 1e-2 (they are expected to be equal; the tolerance is the bf16 bound
this check allows).  The cached run must have armed every layer, installed experts, and
had no step-kernel wait run out.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

LOGPROB_TOL = 1e-2


def test_cached_decode_matches_resident_under_churn(tmp_path):
    import bench_decode as bd
    torch.cuda.empty_cache()              # leave the engines the memory earlier tests cached
    a = bd.parser().parse_args([
        "--layers", "4", "--gen", "32", "--slots", "16", "--routing", "sticky-zipf",
        "--deterministic", "--no-offload-baseline", "--gpu-util", "0.3",
        "--offload-gb", "16", "--mode-timeout", "900", "--logdir", str(tmp_path)])
    got = bd.run_suite(a, echo=False)
    assert not got["summary"]["failed"], got["summary"]["failed"]
    by = {r["mode"]: r for r in got["results"]}
    cached = by["slots16-churn"]
    stats = cached["cache"]
    assert stats["armed_layers"] == 4, stats
    assert stats["installs"] > 0, stats            # the cache actually swapped experts
    assert stats["step_wait_timeouts"] == 0, stats
    assert cached["tokens_match_resident"], (
        f"first divergent token {cached['first_divergent_token']}, resident top-2 gap "
        f"there {cached['resident_top2_gap_at_divergence']}")
    assert cached["max_abs_logprob_diff"] <= LOGPROB_TOL, cached["max_abs_logprob_diff"]
