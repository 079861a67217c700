"""bench_decode.py's benchmark-only pieces, on CPU: the trace-routing override that makes the
churn workload (every layer replays its own sticky-Zipf trace, one row per token, wrapping
at the end and restarting on reset), the mode plan, and the comparison with the resident
run."""

from __future__ import annotations

import numpy as np
import torch

import bench_decode as bd
from synthetic import sticky_zipf_trace


class Router:
    """A router stand-in: returns uniform weights and ids 0..k-1 for every token."""

    def __init__(self, E=16, k=4):
        self.global_num_experts, self.k = E, k

    def select_experts(self, hidden_states, router_logits, *, input_ids=None):
        n = hidden_states.size(0)
        w = torch.full((n, self.k), 1.0 / self.k)
        return w, torch.arange(self.k, dtype=torch.int32).repeat(n, 1)


def test_trace_routing_replays_the_layer_trace(monkeypatch):
    monkeypatch.setattr(bd, "TRACE_ROWS", 6)
    r = Router()
    wrap = bd._TraceRouting(r, seed=1003)
    want = sticky_zipf_trace(1003, steps=6, E=16, k=4)
    x = torch.zeros(1, 8)
    rows = []
    for _ in range(8):                                  # one token per call, wraps at 6
        w, ids = wrap(x, None)
        assert ids.dtype == torch.int32 and tuple(ids.shape) == (1, 4)
        assert torch.equal(w, torch.full((1, 4), 0.25))  # the router's weights are kept
        rows.append(ids[0].numpy())
    np.testing.assert_array_equal(np.stack(rows), want[[0, 1, 2, 3, 4, 5, 0, 1]])
    w, ids = wrap(torch.zeros(5, 8), None)              # a 5-token step continues from row 2
    np.testing.assert_array_equal(ids.numpy(), want[[2, 3, 4, 5, 0]])
    wrap.reset()
    _, ids = wrap(x, None)
    np.testing.assert_array_equal(ids[0].numpy(), want[0])


def test_plan_and_compare():
    a = bd.parser().parse_args(["--slots", "16", "64", "--routing", "model", "sticky-zipf",
                                "--launch", "single", "two"])
    names = [m["name"] for m in bd.plan_modes(a)]
    assert names[:2] == ["resident", "offload"]
    assert "slots64-two-launch" in names and "slots16-churn" in names
    assert all(m.get("routing") == "sticky-zipf" for m in bd.plan_modes(a)
               if m["name"].endswith("-churn"))
    base = {"mode": "resident", "decode_tok_s": 200.0, "tokens": [1, 2, 3, 4],
            "logprobs": [-0.1, -0.2, -0.3, -0.4], "gaps": [1.0, 0.5, 0.0156, 2.0]}
    r = {"mode": "slots16", "decode_tok_s": 150.0, "tokens": [1, 2, 9, 9],
         "logprobs": [-0.1, -0.2005, -1.0, -1.0], "gaps": [0, 0, 0, 0]}
    bd.compare(r, base)
    assert r["frac_of_resident"] == 0.75 and not r["tokens_match_resident"]
    assert r["first_divergent_token"] == 2
    assert abs(r["max_abs_logprob_diff"] - 0.0005) < 1e-9   # only positions before it
    assert r["resident_top2_gap_at_divergence"] == 0.0156


def test_bench_decode_object(monkeypatch):
    """bench.py's decode object from a stubbed suite: the cached fraction is taken against
    the faster resident engine, the spread between the two is reported beside it."""
    import bench

    def result(mode, tps, frac, installs=None):
        cache = None if installs is None else {"timed_installs_per_layer_step": installs,
                                               "installs_per_layer_step": installs,
                                               "layer_steps": 10, "installs": 1,
                                               "armed_layers": 48, "step_wait_timeouts": 0}
        return {"mode": mode, "decode_tok_s": tps, "frac_of_resident": frac,
                "tokens_match_resident": True, "max_abs_logprob_diff": 0.0,
                "first_divergent_token": None, "resident_top2_gap_at_divergence": None,
                "cache": cache}

    modes_seen = []

    def fake_suite(args, modes, echo=True):
        modes_seen.extend(m["name"] for m in modes)
        res = [result("resident", 250.0, 1.0), result("offload", 25.0, 0.1),
               result("slots64", 240.0, 0.96, 0.0), result("resident-churn", 240.0, 1.0),
               result("slots64-churn", 150.0, 0.625, 0.44),
               result("resident-again", 300.0, 1.2)]
        return {"results": res, "ok": True,
                "summary": {"all_within_1e-2_before_divergence": True, "skipped": [],
                            "failed": {}, "wall_s": 1.0}}

    monkeypatch.setattr(bd, "run_suite", fake_suite)
    a = bench.parse(["--decode-slots", "64"])
    out = bench.decode_leg(a)
    assert modes_seen == ["resident", "offload", "slots64", "resident-churn",
                          "slots64-churn", "resident-again"]
    assert out["frac_of_resident"] == 0.8            # 240 / max(250, 300)
    assert out["frac_of_first_resident"] == 0.96
    assert out["resident_spread"] == 0.2
    assert out["churn"]["frac_of_resident"] == 0.625
    assert out["cached"]["timed_installs_per_layer_step"] == 0.0


def test_repeat_interleaves_and_averages(monkeypatch, tmp_path):
    rates = iter([250.0, 240.0, 270.0, 250.0, 260.0, 245.0])   # R, C, R, C, R, C
    order = []

    def fake_run_mode(mode, args, model_dir, site, logdir):
        order.append(mode["name"])
        return {"mode": mode["name"], "decode_tok_s": next(rates), "tokens": [1, 2],
                "logprobs": [-0.1, -0.1], "gaps": [1.0, 1.0], "cache": None}

    monkeypatch.setattr(bd, "run_mode", fake_run_mode)
    a = bd.parser().parse_args(["--slots", "64", "--no-offload-baseline", "--repeat", "3",
                                "--logdir", str(tmp_path)])
    got = bd.run_suite(a, echo=False)
    assert order == ["resident#0", "slots64#0", "resident#1", "slots64#1", "resident#2",
                     "slots64#2"]
    rep = got["summary"]["repeated"]
    assert rep["resident"]["mean_tok_s"] == 260.0 and rep["slots64"]["mean_tok_s"] == 245.0
    assert rep["slots64"]["mean_frac_of_resident"] == round(245.0 / 260.0, 4)
    assert rep["slots64"]["min"] == 240.0 and rep["slots64"]["max"] == 250.0
