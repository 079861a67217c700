#!/usr/bin/env python
"""End-to-end decode through vLLM with the expert cache (BASELINE configs 3-5 family).

Synthetic Qwen3-30B-A3B-shaped W8A8 model (48 layers, hidden 2048, 32q/4kv heads of
128, 128 experts of moe_intermediate 768, top-8, vocab 151936), random-init weights:
normal(0, 0.02), quantised per output channel to int8 with fp32 scales (compressed-
tensors "int-quantized", dynamic per-token int8 activations; lm_head and the router stay
bf16).  Greedy decode at batch 1 from a seeded random 128-token prompt.

Modes, each in its own process (vLLM engine), same weights:

  resident      experts in HBM, cache off                    (the 100% reference)
  offload       --cpu-offload-params experts, cache off      (vLLM's uncached offload)
  slots=S       offload + EXPERT_CACHE_SLOTS=S               (the product)

The expert cache is loaded exactly as in production: through its vllm.general_plugins
entry point.  The synthetic weights come from a load format registered by a second,
benchmark-only general plugin (`register_synthetic_loader` below), so every vLLM process
(including tensor-parallel workers) initialises the same deterministic weights.  Both
entry points are declared in a throw-away site directory put on PYTHONPATH.

Printed: one JSON line per mode (decode tok/s, fraction of resident, tokens identical to
resident, max |logprob difference| of the chosen tokens) and a summary line.

    python bench_decode.py [--arch qwen3-30b-a3b] [--quant int8-experts] [--tp 1]
                           [--slots 16 32 64 96] [--gen 512] [--batch 1]
    python bench_decode.py --arch mixtral-8x7b --quant bf16 --slots 2 4 6 --gen 64
    python bench_decode.py --batch 8 --slots 32 --split-wide 0 4 --parity-batch ...
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
import zlib
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "vllm-expert-cache_b200"
LOAD_FORMAT = "synthetic_w8a8"

QWEN3_30B_A3B = {
    "architectures": ["Qwen3MoeForCausalLM"], "model_type": "qwen3_moe",
    "attention_bias": False, "attention_dropout": 0.0,
    "bos_token_id": 151643, "eos_token_id": 151645, "decoder_sparse_step": 1,
    "head_dim": 128, "hidden_act": "silu", "hidden_size": 2048,
    "initializer_range": 0.02, "intermediate_size": 6144, "max_position_embeddings": 4096,
    "max_window_layers": 48, "mlp_only_layers": [], "moe_intermediate_size": 768,
    "norm_topk_prob": True, "num_attention_heads": 32, "num_experts": 128,
    "num_experts_per_tok": 8, "num_hidden_layers": 48, "num_key_value_heads": 4,
    "output_router_logits": False, "rms_norm_eps": 1e-6, "rope_scaling": None,
    "rope_theta": 1000000.0, "router_aux_loss_coef": 0.001, "sliding_window": None,
    "tie_word_embeddings": False, "torch_dtype": "bfloat16", "use_cache": True,
    "use_sliding_window": False, "vocab_size": 151936,
}

MIXTRAL_8X7B = {
    "architectures": ["MixtralForCausalLM"], "model_type": "mixtral",
    "attention_dropout": 0.0, "bos_token_id": 1, "eos_token_id": 2, "hidden_act": "silu",
    "hidden_size": 4096, "initializer_range": 0.02, "intermediate_size": 14336,
    "max_position_embeddings": 32768, "num_attention_heads": 32, "num_experts_per_tok": 2,
    "num_hidden_layers": 32, "num_key_value_heads": 8, "num_local_experts": 8,
    "output_router_logits": False, "rms_norm_eps": 1e-5, "rope_theta": 1000000.0,
    "router_aux_loss_coef": 0.02, "sliding_window": None, "tie_word_embeddings": False,
    "torch_dtype": "bfloat16", "use_cache": True, "vocab_size": 32000,
}

# the Qwen3-235B-A22B shape (94 layers; runs here truncated with
# --layers so that the offloaded experts fit the host's pinned memory).
QWEN3_235B_A22B = dict(QWEN3_30B_A3B, hidden_size=4096, num_attention_heads=64,
                       num_key_value_heads=4, moe_intermediate_size=1536,
                       intermediate_size=12288, num_hidden_layers=94, max_window_layers=94)

MODELS = {"qwen3-30b-a3b": (QWEN3_30B_A3B, 151936), "mixtral-8x7b": (MIXTRAL_8X7B, 32000),
          "qwen3-235b-a22b": (QWEN3_235B_A22B, 151936)}

W8A8_INT8 = {  # int8 weights + dynamic per-token int8 activations
    "quant_method": "compressed-tensors", "format": "int-quantized",
    "quantization_status": "compressed", "kv_cache_scheme": None,
    "global_compression_ratio": None, "ignore": ["lm_head", "re:.*mlp.gate$"],
    "config_groups": {"group_0": {
        "targets": ["Linear"], "output_activations": None,
        "input_activations": {"num_bits": 8, "type": "int", "symmetric": True,
                              "strategy": "token", "dynamic": True, "group_size": None,
                              "block_structure": None, "actorder": None,
                              "observer": None, "observer_kwargs": {}},
        "weights": {"num_bits": 8, "type": "int", "symmetric": True, "strategy": "channel",
                    "dynamic": False, "group_size": None, "block_structure": None,
                    "actorder": None, "observer": "minmax", "observer_kwargs": {}},
    }},
}


W8A8_FP8 = {   # fp8 e4m3 weights (per channel) + dynamic per-token fp8 activations
    "quant_method": "compressed-tensors", "format": "float-quantized",
    "quantization_status": "compressed", "kv_cache_scheme": None,
    "global_compression_ratio": None, "ignore": ["lm_head", "re:.*mlp.gate$"],
    "config_groups": {"group_0": {
        "targets": ["Linear"], "output_activations": None,
        "input_activations": {"num_bits": 8, "type": "float", "symmetric": True,
                              "strategy": "token", "dynamic": True, "group_size": None,
                              "block_structure": None, "actorder": None,
                              "observer": None, "observer_kwargs": {}},
        "weights": {"num_bits": 8, "type": "float", "symmetric": True, "strategy": "channel",
                    "dynamic": False, "group_size": None, "block_structure": None,
                    "actorder": None, "observer": "minmax", "observer_kwargs": {}},
    }},
}


def quant_config(kind: str):
    """``int8``: W8A8 int8 on every Linear; ``int8-experts``: the same with attention left
    in bf16 (vLLM's CUTLASS int8 scaled-mm does not run on SM100, its fused-MoE int8 path
    does); ``fp8``: W8A8 fp8; ``bf16``: unquantised."""
    import copy
    if kind == "bf16":
        return None
    if kind == "fp8":
        return copy.deepcopy(W8A8_FP8)
    q = copy.deepcopy(W8A8_INT8)
    if kind == "int8-experts":
        q["ignore"] = q["ignore"] + ["re:.*self_attn.*"]
    return q


# ---------------------------------------------------------------------------------------
# benchmark-only vLLM plugin: deterministic synthetic W8A8 weights

def _seed(name: str, base: int = 1234) -> int:
    return (base * 1000003 + zlib.crc32(name.encode())) & 0x7FFFFFFF


# Experts drawn per random call while initialising a quantised expert tensor (one fp32
# chunk of 16 Qwen3-30B-A3B w13 slabs is 200 MB of scratch).
INIT_CHUNK = 16


def init_synthetic_weights(model, std: float = 0.02) -> None:
    """normal(0, std) everywhere; int8 / fp8 weights quantised per output row with their
    fp32 ``*_scale`` set to absmax/qmax (127 / 448); norm weights 1.  Every tensor draws
    from its own generator seeded by its name, on the tensor's device, in fixed chunks of
    experts, so resident and offloaded runs (UVA views of host memory are CUDA tensors)
    initialise identical weights."""
    import torch
    params = dict(model.named_parameters())
    quantised = {torch.int8: 127.0, torch.float8_e4m3fn: 448.0}
    with torch.no_grad():
        for name, p in params.items():
            if p.dtype in quantised:
                qmax = quantised[p.dtype]
                scale = params.get(name + "_scale")
                if scale is None:
                    raise RuntimeError(f"int8 parameter {name} has no {name}_scale")
                g = torch.Generator(device=p.device).manual_seed(_seed(name))
                lead = p.shape[0] if p.dim() == 3 else 1
                qv = p.view(lead, *p.shape[-2:])
                sv = scale.view(lead, p.shape[-2], -1)
                for e0 in range(0, lead, INIT_CHUNK):   # a chunk of experts at a time
                    e1 = min(lead, e0 + INIT_CHUNK)
                    w = torch.randn((e1 - e0,) + tuple(qv.shape[1:]), generator=g,
                                    device=p.device, dtype=torch.float32) * std
                    s = w.abs().amax(dim=-1, keepdim=True).clamp_min(1e-8) / qmax
                    q = (w / s).clamp_(-qmax, qmax)
                    if p.dtype == torch.int8:
                        q = torch.round(q)
                    qv[e0:e1].copy_(q.to(p.dtype))
                    sv[e0:e1].copy_(s.to(sv.dtype).expand_as(sv[e0:e1]))
            elif name.endswith("_scale") and name[:-6] in params \
                    and params[name[:-6]].dtype in quantised:
                continue                     # written with its weight
            elif torch.is_floating_point(p):
                if "norm" in name:
                    p.fill_(1.0)
                else:
                    g = torch.Generator(device=p.device).manual_seed(_seed(name))
                    p.copy_(torch.randn(p.shape, generator=g, device=p.device,
                                        dtype=torch.float32).mul_(std).to(p.dtype))


def cache_stats_on_worker(worker) -> list:
    """collective_rpc target: every armed layer's counters, the tensors it mirrors, every
    name bound to slot storage during a cached step, a digest of its policy state (equal
    on every tensor-parallel rank when the ranks stayed in step) and a consistency check
    of that state (table[e] = s exactly when slot_expert[s] = e)."""
    import hashlib

    import numpy as np
    model = worker.model_runner.get_model()
    out = []
    for m in model.modules():
        c = getattr(m, "_expert_cache", None)
        if c is not None:
            st = c.stats()
            st["mirrored"] = {n: list(c.slots[n].shape) for n in c.names}
            st["bound"] = sorted(c.bound)
            st["method"] = type(m.quant_method).__name__
            st["prefetch_linked"] = c.next is not None
            table, se = c.table.cpu().numpy(), c.slot_expert.cpu().numpy()
            h = hashlib.blake2b(digest_size=8)
            for t in (table, c.map_cold.cpu().numpy(), se, c.slot_stamp.cpu().numpy(),
                      c.step.cpu().numpy()):
                h.update(np.ascontiguousarray(t).tobytes())
            st["state_digest"] = h.hexdigest()
            occupied = se >= 0
            st["consistent"] = bool(
                all(table[e] == s for s, e in enumerate(se) if e >= 0) and
                int((table >= 0).sum()) == int(occupied.sum()))
            out.append(st)
    return out


# Benchmark-only routing override: with BENCH_DECODE_ROUTING=sticky-zipf every MoE layer's
# routing ids replay that layer's own sticky-Zipf trace (the config-1 locality model: each
# of the 8 positions keeps the previous token's expert with p=0.7, else draws Zipf(1.1)
# over a seeded permutation), one trace row per token, seeds 1000 + layer index.  The
# router's top-k weights are kept.  A device counter per layer picks the row, so the
# override runs inside vLLM's CUDA graphs (3 small torch kernels per layer per decode
# step, paid by every mode that uses the override, resident included).
ROUTING_ENV = "BENCH_DECODE_ROUTING"
TRACE_ROWS = 4096


class _TraceRouting:
    def __init__(self, router, seed: int):
        self.router, self.seed = router, seed
        self.orig = router.select_experts
        self.tr = self.ctr = self.ar = None

    def _init(self, ids):
        import torch
        from synthetic import sticky_zipf_trace
        k = ids.size(1)
        E = int(self.router.global_num_experts)
        tr = sticky_zipf_trace(self.seed, steps=TRACE_ROWS, E=E, k=k)
        self.tr = torch.from_numpy(tr).to(device=ids.device, dtype=ids.dtype)
        self.ctr = torch.zeros(1, dtype=torch.int64, device=ids.device)

    def reset(self):
        if self.ctr is not None:
            self.ctr.zero_()

    def __call__(self, hidden_states, router_logits, *, input_ids=None):
        import torch
        w, ids = self.orig(hidden_states, router_logits, input_ids=input_ids)
        if ids.dim() != 2:
            return w, ids
        if self.tr is None:
            self._init(ids)
        n = ids.size(0)
        if n == 1:
            idx = self.ctr
        else:
            if self.ar is None or self.ar.numel() < n:
                self.ar = torch.arange(max(n, 8192), dtype=torch.int64, device=ids.device)
            idx = (self.ctr + self.ar[:n]).remainder_(TRACE_ROWS)
        new = self.tr.index_select(0, idx)
        self.ctr.add_(n).remainder_(TRACE_ROWS)     # always a valid row index
        return w, new


def install_trace_routing(model) -> int:
    """Wrap every FusedMoE layer's router (in model order) with its trace replay."""
    from vllm.model_executor.layers.fused_moe.layer import FusedMoE
    n = 0
    for m in model.modules():
        if isinstance(m, FusedMoE) and getattr(m, "router", None) is not None:
            m.router.select_experts = _TraceRouting(m.router, 1000 + n)
            n += 1
    return n


def reset_routing_on_worker(worker) -> int:
    """collective_rpc target: restart every layer's trace at row 0."""
    model = worker.model_runner.get_model()
    n = 0
    for m in model.modules():
        r = getattr(getattr(m, "router", None), "select_experts", None)
        if isinstance(r, _TraceRouting):
            r.reset()
            n += 1
    return n


def register_synthetic_loader() -> None:
    """vllm.general_plugins entry point of the benchmark (not of the product)."""
    import os
    from vllm.model_executor.model_loader import register_model_loader
    from vllm.model_executor.model_loader.dummy_loader import DummyModelLoader

    class SyntheticW8A8Loader(DummyModelLoader):
        def load_weights(self, model, model_config) -> None:
            init_synthetic_weights(model)
            if os.environ.get(ROUTING_ENV) == "sticky-zipf":
                install_trace_routing(model)

    register_model_loader(LOAD_FORMAT)(SyntheticW8A8Loader)


# ---------------------------------------------------------------------------------------
# parent: model directory, plugin site, one child process per mode

def write_model_dir(path: Path, layers: int, max_len: int, quant: str,
                    model: str = "qwen3-30b-a3b") -> None:
    cfg = dict(MODELS[model][0])
    if layers:
        cfg["num_hidden_layers"] = layers
        if "max_window_layers" in cfg:
            cfg["max_window_layers"] = layers
    cfg["max_position_embeddings"] = max(max_len, 4096)
    q = quant_config(quant)
    if q is not None:
        cfg["quantization_config"] = q
    path.mkdir(parents=True, exist_ok=True)
    (path / "config.json").write_text(json.dumps(cfg, indent=1))
    (path / "generation_config.json").write_text(json.dumps(
        {"bos_token_id": cfg["bos_token_id"], "eos_token_id": cfg["eos_token_id"],
         "do_sample": False}))


def write_plugin_site(path: Path) -> None:
    """dist-info entry points for the product plugin and the benchmark loader."""
    for dist, ep in (("vllm_expert_cache-0.3.0", "expert_cache = vllm_expert_cache:install"),
                     ("expert_cache_bench-0.0.0",
                      "synthetic_w8a8 = bench_decode:register_synthetic_loader")):
        d = path / f"{dist}.dist-info"
        d.mkdir(parents=True, exist_ok=True)
        name, ver = dist.rsplit("-", 1)
        (d / "METADATA").write_text(f"Metadata-Version: 2.1\nName: {name}\nVersion: {ver}\n")
        (d / "entry_points.txt").write_text(f"[vllm.general_plugins]\n{ep}\n")


def run_mode(mode: dict, args, model_dir: Path, site: Path, logdir: Path) -> dict:
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(site), str(PKG), str(ROOT),
                                         env.get("PYTHONPATH", "")])
    env["VLLM_PLUGINS"] = "expert_cache,synthetic_w8a8"
    env.setdefault("VLLM_LOGGING_LEVEL", "INFO")
    if args.debug_calls:
        env["EXPERT_CACHE_DEBUG"] = str(args.debug_calls)
    env.pop("EXPERT_CACHE_SLOTS", None)
    env["EXPERT_CACHE_DISABLE"] = "0" if mode.get("slots") else "1"
    if mode.get("slots"):
        env["EXPERT_CACHE_SLOTS"] = str(mode["slots"])
    env["EXPERT_CACHE_POLICY"] = args.policy
    env["EXPERT_CACHE_STATS"] = "1" if args.stats else "0"
    env.pop("EXPERT_CACHE_SPLIT_WIDE", None)
    env["EXPERT_CACHE_PREFETCH"] = str(mode.get("prefetch") or 0)
    if mode.get("policy"):
        env["EXPERT_CACHE_POLICY"] = mode["policy"]
    env.pop(ROUTING_ENV, None)
    if mode.get("routing"):
        env[ROUTING_ENV] = mode["routing"]
    if mode.get("split"):
        env["EXPERT_CACHE_SPLIT_WIDE"] = str(mode["split"])
    env["EXPERT_CACHE_EP"] = "1" if args.ep else "0"
    env["EXPERT_CACHE_SINGLE_LAUNCH"] = "0" if mode.get("two_launch") else "1"
    if args.deterministic:
        env["VLLM_BATCH_INVARIANT"] = "1"   # vLLM's deterministic (batch-invariant) kernels
    # the counters are fetched with collective_rpc(<function>), which vLLM pickles
    env["VLLM_ALLOW_INSECURE_SERIALIZATION"] = "1"
    log = logdir / f"decode_{mode['name']}.log"
    cmd = [sys.executable, str(Path(__file__).resolve()), "--child",
           json.dumps(mode), "--model", str(model_dir), "--tp", str(args.tp),
           "--prompt", str(args.prompt), "--gen", str(args.gen), "--seed", str(args.seed),
           "--batch", str(args.batch), "--vocab", str(MODELS[args.arch][1]),
           "--gpu-util", str(args.gpu_util), "--moe-backend", args.moe_backend,
           "--temperature", str(args.temperature), "--reps", str(args.reps)]
    if args.ep:
        cmd.append("--ep")
    if args.parity_batch:
        cmd.append("--parity-batch")
    if args.no_autotune or args.deterministic:
        cmd.append("--no-autotune")
    t0 = time.time()
    with open(log, "w") as f:
        rc = subprocess.run(cmd, env=env, stdout=subprocess.PIPE, stderr=f, text=True,
                            timeout=args.mode_timeout)
    with open(log, "a") as f:            # vLLM's loggers (and ours) write to stdout
        f.write(rc.stdout)
    res = None
    for line in rc.stdout.splitlines():
        if line.startswith("{\"decode_result\""):
            res = json.loads(line)["decode_result"]
    if rc.returncode != 0 or res is None:
        tail = log.read_text()[-3000:]
        raise RuntimeError(f"mode {mode['name']} failed rc={rc.returncode}:\n{tail}")
    res["wall_s"] = round(time.time() - t0, 1)
    text = log.read_text()
    res["armed_log"] = [ln.split("expert-cache", 1)[1].strip()[:160]
                        for ln in text.splitlines() if "active on" in ln][:1]
    return res


def child(mode: dict, a) -> None:
    import numpy as np
    from vllm import LLM, SamplingParams
    kw = dict(model=a.model, skip_tokenizer_init=True, load_format=LOAD_FORMAT,
              dtype="bfloat16", tensor_parallel_size=a.tp, max_model_len=a.prompt + a.gen + 16,
              gpu_memory_utilization=a.gpu_util, max_num_seqs=a.batch, seed=a.seed,
              enable_prefix_caching=False, disable_log_stats=False)
    if a.moe_backend != "auto":
        kw["moe_backend"] = a.moe_backend
    if a.no_autotune:
        kw["enable_flashinfer_autotune"] = False
    if mode.get("offload"):
        kw.update(cpu_offload_gb=mode["offload_gb"], cpu_offload_params={"experts"})
    if a.ep:
        kw["enable_expert_parallel"] = True
    t0 = time.time()
    llm = LLM(**kw)
    init_s = time.time() - t0
    rng = np.random.default_rng(a.seed)
    prompts = [{"prompt_token_ids": rng.integers(0, a.vocab, size=a.prompt).tolist()}
               for _ in range(a.batch)]
    greedy = dict(temperature=0.0, ignore_eos=True, detokenize=False)
    # timed runs: greedy, or seeded sampling so the input token changes every step (a
    # random-init model's greedy output repeats one token, which makes routing repeat)
    timed = greedy if a.temperature == 0 else dict(
        temperature=a.temperature, seed=a.seed, ignore_eos=True, detokenize=False)

    def generate(p, sp):
        # with the trace routing, every generate starts each layer's trace at row 0, so all
        # modes see the same routing sequence
        if mode.get("routing"):
            llm.collective_rpc(reset_routing_on_worker)
        return llm.generate(p, sp, use_tqdm=False)

    generate(prompts, SamplingParams(max_tokens=32, **timed))  # warm
    # parity run: the first prompt alone, or (--parity-batch) the whole batch so that its
    # decode steps have the timed runs' width; sequences are concatenated in prompt order
    refs = generate(prompts if a.parity_batch else prompts[:1],
                    SamplingParams(max_tokens=a.gen, logprobs=2, **greedy))
    tokens, lps, gaps = [], [], []
    for r in refs:
        ref = r.outputs[0]
        tokens += list(ref.token_ids)
        lps += [float(d[t].logprob) for d, t in zip(ref.logprobs, ref.token_ids)]
        # top-1 minus top-2 logprob per position: how close each greedy choice was to a tie
        for d in ref.logprobs:
            v = sorted((float(x.logprob) for x in d.values()), reverse=True)
            gaps.append(v[0] - v[1] if len(v) > 1 else float("inf"))
    def installs_now():
        if not mode.get("slots"):
            return None
        ranks = llm.collective_rpc(cache_stats_on_worker)
        layers = ranks[0] if ranks else []
        return (sum(x.get("installs", 0) for x in layers),
                sum(x["steps"] for x in layers))

    before = installs_now()
    times = {}
    engine_decode = []
    for n in (1, a.gen):
        best = None
        for _ in range(a.reps):
            if mode.get("routing"):
                llm.collective_rpc(reset_routing_on_worker)
            t = time.perf_counter()
            outs = llm.generate(prompts, SamplingParams(max_tokens=n, **timed), use_tqdm=False)
            dt = time.perf_counter() - t
            best = dt if best is None else min(best, dt)
            if n == a.gen:
                # the engine's own clock: first token (end of prefill) to last token
                ts = [(o.metrics.first_token_ts, o.metrics.last_token_ts) for o in outs
                      if getattr(o, "metrics", None) is not None]
                if len(ts) == len(outs) and all(b > a_ for a_, b in ts):
                    engine_decode.append(max(b for _, b in ts) - min(a_ for a_, _ in ts))
        times[n] = best
    # decode tokens of the whole batch per second of decode: timed by the engine between
    # each request's first and last token (no prefill in it); the wall-clock difference
    # t(gen) - t(1) is kept beside it
    after = installs_now()
    wall_tps = a.batch * (a.gen - 1) / (times[a.gen] - times[1])
    decode_tps = (a.batch * (a.gen - 1) / min(engine_decode)) if engine_decode else wall_tps
    cache = None
    if mode.get("slots"):
        per_rank = llm.collective_rpc(cache_stats_on_worker)
        layers = per_rank[0] if per_rank else []
        if layers:
            steps = sum(x["steps"] for x in layers)
            installs = sum(x.get("installs", 0) for x in layers)
            cache = {"armed_layers": len(layers), "layer_steps": steps,
                     "mirrored": layers[0]["mirrored"], "bound": layers[0]["bound"],
                     "method": layers[0]["method"],
                     "step_wait_timeouts": sum(x.get("step_timeouts", 0) for x in layers)}
            cache["prefetch_linked"] = sum(bool(x.get("prefetch_linked")) for x in layers)
            cache["consistent"] = all(x["consistent"] for r in per_rank for x in r)
            cache["ranks"] = len(per_rank)
            cache["ranks_identical"] = all(
                [x["state_digest"] for x in r] == [x["state_digest"] for x in layers]
                for r in per_rank)
            if before is not None and after is not None and after[1] > before[1]:
                # only the timed generations (their prefills read through and add no steps)
                cache["timed_installs_per_layer_step"] = round(
                    (after[0] - before[0]) / (after[1] - before[1]), 4)
            if "installs" in layers[0]:
                cache.update(installs=installs,
                             installs_per_layer_step=round(installs / max(steps, 1), 4),
                             bytes_per_install=layers[0].get("bytes_per_install"))
            if "prefetch_installs" in layers[0]:
                pf = sum(x["prefetch_installs"] for x in layers)
                cache.update(prefetch_installs=pf,
                             prefetch_installs_per_layer_step=round(pf / max(steps, 1), 4))
    out = {"mode": mode["name"], "slots": mode.get("slots"), "split_wide": mode.get("split", 0),
           "prefetch": mode.get("prefetch") or 0, "routing": mode.get("routing") or "model",
           "policy": mode.get("policy") or a.policy,
           "offload": bool(mode.get("offload")),
           "tp": a.tp, "ep": a.ep, "batch": a.batch, "init_s": round(init_s, 1), "prefill_s": round(times[1], 4),
           "gen_s": round(times[a.gen], 4), "decode_tok_s": round(decode_tps, 2),
           "decode_tok_s_wall": round(wall_tps, 2),
           "decode_timer": "engine first-to-last token" if engine_decode else "wall t(gen)-t(1)",
           "cache": cache, "tokens": tokens, "logprobs": lps, "gaps": gaps}
    print(json.dumps({"decode_result": out}), flush=True)


def parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser()
    ap.add_argument("--arch", choices=sorted(MODELS), default="qwen3-30b-a3b")
    ap.add_argument("--layers", type=int, default=0, help="0 = the architecture's own")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--gpu-util", type=float, default=0.55)
    ap.add_argument("--vocab", type=int, default=151936)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--ep", action="store_true",
                    help="vLLM expert parallelism across the TP ranks "
                         "(--enable-expert-parallel); cached modes set EXPERT_CACHE_EP=1")
    ap.add_argument("--slots", type=int, nargs="*", default=[16, 32, 64, 96])
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--gen", type=int, default=512)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--policy", default="lfu")
    ap.add_argument("--policies", nargs="*", default=[],
                    help="EXPERT_CACHE_POLICY values: every slot count runs once per value "
                         "(default: --policy alone)")
    ap.add_argument("--quant", choices=["int8", "int8-experts", "fp8", "bf16"],
                    default="int8-experts")
    ap.add_argument("--offload-gb", type=float, default=64.0)
    ap.add_argument("--no-offload-baseline", action="store_true")
    ap.add_argument("--no-resident", action="store_true",
                    help="skip the resident mode: the first mode run is the comparison base")
    ap.add_argument("--stats", action="store_true",
                    help="EXPERT_CACHE_STATS=1: also count installs of the two-launch path "
                         "and of prefetches (one small kernel per layer-step each); the "
                         "single-launch step counts its own installs either way")
    ap.add_argument("--moe-backend", default="auto",
                    help="vLLM MoE backend; the cache needs a modular (non-monolithic) one, "
                         "e.g. 'triton' where vLLM's default would be flashinfer_trtllm")
    ap.add_argument("--no-autotune", action="store_true",
                    help="disable FlashInfer's start-up autotuning (a source of run-to-run "
                         "kernel choice, and slow on host-resident weights)")
    ap.add_argument("--deterministic", action="store_true",
                    help="VLLM_BATCH_INVARIANT=1 and no autotuning in every mode, to compare "
                         "tokens and logprobs without the engine's own run-to-run spread")
    ap.add_argument("--temperature", type=float, default=0.0,
                    help="timed runs only: 0 = greedy; > 0 = seeded sampling (the parity "
                         "run stays greedy)")
    ap.add_argument("--routing", nargs="*", default=["model"],
                    choices=["model", "sticky-zipf"],
                    help="'model': the random-init router's own choice; 'sticky-zipf': every "
                         "layer replays its own config-1 trace (benchmark-only override). "
                         "Each kind runs its own resident / offload / slots modes and is "
                         "compared with its own resident run")
    ap.add_argument("--debug-calls", type=int, default=0,
                    help="EXPERT_CACHE_DEBUG: log the first N MoE calls per armed layer")
    ap.add_argument("--control", action="store_true",
                    help="run the resident mode twice to measure the engine's own spread")
    ap.add_argument("--split-wide", type=int, nargs="*", default=[],
                    help="EXPERT_CACHE_SPLIT_WIDE values: every slot count runs once per "
                         "value (0 = the reference's read-through of wide steps)")
    ap.add_argument("--prefetch", type=int, nargs="*", default=[],
                    help="EXPERT_CACHE_PREFETCH values (predictions per token, 0 = off): "
                         "every slot count runs once per value")
    ap.add_argument("--launch", nargs="*", default=["single"], choices=["single", "two"],
                    help="cached step form: one expert_cache_step launch, or two launches "
                         "(EXPERT_CACHE_SINGLE_LAUNCH=0); every slot count runs once per value")
    ap.add_argument("--parity-batch", action="store_true",
                    help="greedy parity run over the whole batch instead of its first prompt")
    ap.add_argument("--reps", type=int, default=2, help="timed generations per length; the "
                    "best is kept")
    ap.add_argument("--mode-timeout", type=int, default=1200)
    ap.add_argument("--repeat", type=int, default=1,
                    help="run the whole mode list this many times, interleaved (resident, "
                         "cached, resident, cached, ...), and report each mode's mean and "
                         "spread: engines of one configuration differ by several percent")
    ap.add_argument("--budget-s", type=float, default=0,
                    help="stop starting new modes once this much wall time has passed "
                         "(0 = no limit); skipped modes are listed in the summary")
    ap.add_argument("--logdir", default=str(Path(tempfile.gettempdir()) / "expert_cache_decode"),
                    help="per-mode engine logs")
    ap.add_argument("--child", default=None)
    ap.add_argument("--model", default=None)
    return ap


def plan_modes(a) -> list[dict]:
    """Every mode of the run, grouped by routing kind; the first mode of a kind that keeps
    the experts resident is that kind's comparison base."""
    modes = []
    for routing in a.routing:
        tag = "" if routing == "model" else "-churn"
        extra = {} if routing == "model" else {"routing": routing}
        if not a.no_resident:
            modes.append({"name": "resident" + tag, **extra})
        if a.control:
            modes.append({"name": "resident-again" + tag, **extra})
        if not a.no_offload_baseline:
            modes.append({"name": "offload" + tag, "offload": True,
                          "offload_gb": a.offload_gb, **extra})
        for pol in (a.policies or [None]):
            for sl in a.slots:
                for v in (a.split_wide or [0]):
                    for f in (a.prefetch or [0]):
                        for launch in a.launch:
                            name = (f"slots{sl}" + (f"-{pol}" if pol else "") +
                                    (f"-split{v}" if v else "") +
                                    (f"-prefetch{f}" if f else "") +
                                    ("-two-launch" if launch == "two" else "") + tag)
                            modes.append({"name": name, "slots": sl, "split": v,
                                          "prefetch": f, "policy": pol, "offload": True,
                                          "two_launch": launch == "two",
                                          "offload_gb": a.offload_gb, **extra})
    return modes


def compare(r: dict, base: dict) -> dict:
    """Speed and greedy parity of one mode against its base (resident) run."""
    r["base_mode"] = base["mode"]
    r["frac_of_resident"] = round(r["decode_tok_s"] / base["decode_tok_s"], 4)
    r["tokens_match_resident"] = r["tokens"] == base["tokens"]
    first = next((i for i, (x, y) in enumerate(zip(r["tokens"], base["tokens"])) if x != y),
                 None)
    r["first_divergent_token"] = first
    # logprobs of the same chosen tokens: every position before the first divergence
    upto = len(r["tokens"]) if first is None else first
    r["max_abs_logprob_diff"] = max(
        (abs(x - y) for x, y in zip(r["logprobs"][:upto], base["logprobs"][:upto])),
        default=0.0)
    # at a divergence: how close the resident run's own top-2 were (a near-tie flip)
    r["resident_top2_gap_at_divergence"] = (None if first is None
                                            else round(base["gaps"][first], 5))
    return r


def run_suite(a, modes=None, echo=True) -> dict:
    """Run every mode (one vLLM engine process each) and compare each with its base."""
    logdir = Path(a.logdir)
    logdir.mkdir(parents=True, exist_ok=True)
    tmp = Path(tempfile.mkdtemp(prefix="expert_cache_decode_"))
    model_dir, site = tmp / "model", tmp / "site"
    write_model_dir(model_dir, a.layers, a.prompt + a.gen + 16, a.quant, a.arch)
    write_plugin_site(site)
    modes = plan_modes(a) if modes is None else modes
    if a.repeat > 1:
        modes = [dict(m, name=f"{m['name']}#{i}") for i in range(a.repeat) for m in modes]
    t0 = time.time()
    results, skipped, failed = [], [], {}
    bases: dict[str, dict] = {}
    for m in modes:
        if a.budget_s and time.time() - t0 > a.budget_s:
            skipped.append(m["name"])
            continue
        try:
            r = run_mode(m, a, model_dir, site, logdir)
        except Exception as e:        # report and go on: one mode must not sink the rest
            failed[m["name"]] = repr(e)[-600:]
            continue
        kind = m.get("routing") or "model"
        if kind not in bases and not m.get("offload"):
            bases[kind] = r
        base = bases.get(kind, r)
        compare(r, base)
        slim = {k: v for k, v in r.items() if k not in ("logprobs", "gaps")}
        slim["tokens"] = r["tokens"][:16]
        slim.update(moe_backend=a.moe_backend, deterministic=a.deterministic,
                    temperature=a.temperature,
                    arch=a.arch, layers=a.layers or MODELS[a.arch][0]["num_hidden_layers"],
                    prompt=a.prompt, gen=a.gen, quant=a.quant, parity_batch=a.parity_batch)
        if echo:
            print(json.dumps(slim), flush=True)
        results.append(slim)
    # the chosen tokens' logprobs within 1e-2 of the resident run's at every position the
    # two runs share (before any divergence); divergences are reported with the resident
    # run's own top-1/top-2 margin at that position
    ok = all(r["max_abs_logprob_diff"] <= 1e-2 for r in results) and not failed
    repeated = {}
    if a.repeat > 1:
        for r in results:
            repeated.setdefault(r["mode"].split("#")[0], []).append(r["decode_tok_s"])
        base_mean = None
        for name, v in repeated.items():
            mean = sum(v) / len(v)
            repeated[name] = {"mean_tok_s": round(mean, 2), "min": min(v), "max": max(v),
                              "runs": v}
            if base_mean is None and name.startswith("resident"):
                base_mean = mean
        for name, v in repeated.items():
            if base_mean:
                v["mean_frac_of_resident"] = round(v["mean_tok_s"] / base_mean, 4)
    summary = {"summary": "decode", "all_within_1e-2_before_divergence": ok,
               "repeated": repeated,
               "tokens_identical": {r["mode"]: r["tokens_match_resident"] for r in results},
               "decode_tok_s": {r["mode"]: r["decode_tok_s"] for r in results},
               "frac_of_resident": {r["mode"]: r["frac_of_resident"] for r in results},
               "skipped": skipped, "failed": failed, "wall_s": round(time.time() - t0, 1)}
    if echo:
        print(json.dumps(summary), flush=True)
    return {"results": results, "summary": summary, "ok": ok}


def main(argv=None):
    a = parser().parse_args(argv)
    if a.child:
        return child(json.loads(a.child), a)
    return 0 if run_suite(a)["ok"] else 1


if __name__ == "__main__":
    sys.exit(main() or 0)
