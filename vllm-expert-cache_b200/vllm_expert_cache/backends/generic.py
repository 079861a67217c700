"""Arming: attach an ExpertSlotCache to every cacheable vLLM MoE layer.

Scheme-agnostic by the same three conventions the reference relies on
(vllm_expert_cache/backends/generic.py:1-23):

  1. ``method.apply`` reads the expert weights off the layer;
  2. every per-expert scale / zero point / bias reaches the kernel through
     ``method.get_fused_moe_quant_config(layer)``, which reads named layer attributes;
  3. the built kernel keeps that config in ``method.moe_kernel.fused_experts.quant_config``.

So arming discovers the per-expert tensors by shape (dim 0 == E, aliases grouped by
storage), hangs slot buffers on the layer, re-runs the scheme's own config factory under
slot binding to get a slot-bound config, refuses the layer if any per-expert tensor
stayed on full [E] storage, and wraps ``method.apply`` on the instance.  A cached step
swaps the slot buffers, the slot-bound config and ``global_num_experts = S`` in around the
original ``apply`` and restores everything afterwards; a step wider than the slots calls
the original untouched (or, opted in with EXPERT_CACHE_SPLIT_WIDE, runs as a few cached
steps over consecutive token chunks).  An expert-parallel layer (opted in with
EXPERT_CACHE_EP) caches its local experts and keeps its routing ids global: the step
binds a composed global id -> slot map as ``layer.expert_map`` instead of remapping the
ids.  The hook is vLLM's single post-load call site,
``model_loader.utils.process_weights_after_loading``, rebound wherever it was imported by
name.  Refusals are logged and leave the layer on the stock path.
"""

from __future__ import annotations

import contextlib
import itertools
import sys

import torch

from ..cache import ExpertSlotCache
from ..config import settings

# FusedMoEQuantConfig descriptors and the fields that can carry a per-expert tensor.
_QUANT_DESCS = ("_a1", "_a2", "_w1", "_w2")
_QUANT_FIELDS = ("scale", "alpha_or_gscale", "zp", "bias")
# Registered names of the two expert weight matrices, plain and packed spellings.
_WEIGHT_PAIRS = (("w13_weight", "w2_weight"), ("w13_weight_packed", "w2_weight_packed"))
# Expert-parallel bookkeeping vLLM registers on the layer (fused_moe/layer.py:516-531):
# indexed by expert id but not expert data, so never mirrored into slots.
_EP_BUFFERS = frozenset({"_expert_map", "expert_mask", "expert_global_to_physical",
                         "expert_physical_to_global", "expert_local_to_global"})
# Activation quant dtypes whose scales are per block of one row (vLLM's string dtypes).
_MICRO_SCALED = frozenset({"nvfp4", "mxfp4", "mxfp6_e3m2", "mxfp6_e2m3", "mxfp8"})

_installed = False
# One side stream per device carries every layer's next-layer prefetch.
_side_streams: dict[int, torch.cuda.Stream] = {}


def _set_tensor(layer, name: str, t: torch.Tensor) -> None:
    """Rebind ``layer.<name>`` without tripping nn.Module's Parameter registration."""
    if name in layer._parameters:
        layer._parameters[name] = t
    elif name in layer._buffers:
        layer._buffers[name] = t
    else:
        setattr(layer, name, t)


def _per_expert_tensors(layer, num_experts: int) -> dict[str, list[str]]:
    """Expert-major storages of ``layer``, each with every name that reaches it.

    Registered parameters and buffers are listed without de-duplication (an alias
    registered under two names must keep both names), then plain tensor attributes
    (the packed families alias ``w13_weight = w13_weight_packed`` as a bare attribute).
    Names are grouped by storage so one slot buffer serves every alias; the first name of
    a group is the one sources are read from.
    """
    by_storage: dict[int, list[str]] = {}
    found = itertools.chain(
        layer.named_parameters(recurse=False, remove_duplicate=False),
        layer.named_buffers(recurse=False, remove_duplicate=False),
        ((k, v) for k, v in vars(layer).items() if isinstance(v, torch.Tensor)))
    for name, t in found:
        if not isinstance(t, torch.Tensor) or t.dim() < 1 or t.size(0) != num_experts:
            continue
        if name in _EP_BUFFERS:
            continue
        names = by_storage.setdefault(t.data_ptr(), [])
        if name not in names:
            names.append(name)
    return {names[0]: names for names in by_storage.values()}


def _leaked_full_tensors(cfg, num_experts: int) -> list[str]:
    """Per-expert tensors the slot-bound quant config still holds at full [E] size.

    Such a tensor would be indexed with slot ids and serve the wrong expert's rows, so a
    non-empty answer refuses the layer.
    """
    leaked = []
    for dname in _QUANT_DESCS:
        desc = getattr(cfg, dname, None)
        if desc is None:
            continue
        for field in _QUANT_FIELDS:
            t = getattr(desc, field, None)
            if isinstance(t, torch.Tensor) and t.dim() >= 1 and t.size(0) == num_experts:
                leaked.append(f"{dname}.{field}{tuple(t.shape)}")
    return leaked


def _token_local(cfg) -> str | None:
    """Why a token of this quant config does not compute independently of the others in
    its step, or None when it does.

    The one coupling in a FusedMoEQuantConfig is a dynamic per-tensor activation scale:
    ``_a1`` / ``_a2`` with a quant dtype, no static scale, and the PER_TENSOR group shape
    (or none).  Serving such a step in chunks would quantise each chunk against its own
    maximum.  Token-local are: per-token shapes, K-blocked shapes (vLLM records a block
    quantiser's activation shape as the weight block, e.g. (128, 128), and quantises per
    token group), static scales, and the micro-scaled formats, whose scales cover 16 or 32
    elements of one row (vllm/model_executor/layers/fused_moe/config.py:69-97, 488-560).
    """
    if cfg is None:
        return None
    for dname in ("_a1", "_a2"):
        desc = getattr(cfg, dname, None)
        dtype = getattr(desc, "dtype", None)
        if dtype is None or dtype in _MICRO_SCALED:
            continue
        if getattr(desc, "scale", None) is not None:
            continue                                  # static scale
        shape = getattr(desc, "shape", None)
        if shape is not None and (getattr(shape, "row", -1), getattr(shape, "col", -1)) \
                != (-1, -1):
            continue                                  # per token / per token group
        return f"{dname} is quantised with a dynamic per-tensor scale"
    return None


@contextlib.contextmanager
def _slot_bound(layer, cache: ExpertSlotCache):
    """Point every mirrored name at its slot buffer inside the block; restore after."""
    saved = {name: getattr(layer, name) for name in cache.bound}
    try:
        for name, slot in cache.bound.items():
            _set_tensor(layer, name, slot)
        yield
    finally:
        for name, t in saved.items():
            _set_tensor(layer, name, t)


def _decline(layer, method, num_experts: int) -> str | None:
    """Why this layer cannot be cached correctly, or None."""
    if method.is_monolithic:
        return "monolithic method (routing happens inside apply_monolithic)"
    kernel = getattr(method, "moe_kernel", None)
    if kernel is None:
        return "method has no moe_kernel (legacy non-modular path)"
    if getattr(kernel, "fused_experts", None) is None:
        return "moe_kernel exposes no fused_experts to rebind"
    if getattr(layer, "eplb_state", None) is not None or getattr(layer, "enable_eplb", False):
        # vLLM's expert load balancer rewrites the layer's expert rows and expert_map in
        # place between steps (rearrange_expert_weights_inplace); the cache's table and
        # slot contents would stay keyed by the old placement and serve wrong experts.
        return ("expert load balancing (EPLB) rearranges the expert weights between "
                "steps")
    if getattr(layer, "expert_map", None) is not None:
        if not settings.ep:
            return "expert parallelism active (layer.expert_map is set)"
        return _decline_ep(method, kernel)
    if getattr(layer, "use_ep", False):
        # EP whose kernel takes no expert map: routing ids are global while the layer's
        # weights are local, so a slot remap over the local count would be meaningless.
        return "expert parallelism without an expert_map (the kernel is not given one)"
    return None


def _decline_ep(method, kernel) -> str | None:
    """Why an expert-parallel layer cannot be cached through its expert map, or None.

    The composed map only works where the stock kernel reaches every expert through
    ``layer.expert_map``: the method passes it (``disable_expert_map`` unset,
    vllm/model_executor/layers/fused_moe/fused_moe_modular_method.py:36-40, 108), the
    kernel supports it, and tokens arrive in the standard (num_tokens, hidden) format;
    batched all-to-all formats index experts by local position instead.
    """
    if getattr(method, "disable_expert_map", False):
        return "expert parallelism with the expert map disabled for this method"
    supports = getattr(kernel, "supports_expert_map", None)
    if callable(supports) and not supports():
        return "expert parallelism with a kernel that does not take an expert map"
    fmt = getattr(getattr(kernel, "prepare_finalize", None), "activation_format", None)
    name = getattr(fmt, "name", None)
    if name != "Standard":
        return (f"expert parallelism with the {name or 'unknown'} activation format (only "
                "the standard format reaches the experts through expert_map)")
    return None


def _expert_map_name(layer) -> str:
    """Where ``layer.expert_map`` is stored: vLLM registers it as the ``_expert_map``
    buffer behind a read-only property (fused_moe/layer.py:516-521, 1318-1322)."""
    return "_expert_map" if "_expert_map" in layer._buffers else "expert_map"


def _router_weight(layer) -> torch.Tensor | None:
    """The layer's router weight [E, hidden]: vLLM hands the model's gate to FusedMoE,
    which keeps it on its runner (fused_moe/layer.py:426-431, runner/moe_runner.py:238)."""
    for owner in (getattr(layer, "runner", None), layer):
        w = getattr(getattr(owner, "gate", None), "weight", None)
        if isinstance(w, torch.Tensor):
            return w
    return None


def _prefetch_unusable(w: torch.Tensor | None, cache: ExpertSlotCache) -> str | None:
    """Why the pregate kernel cannot score with this router weight, or None."""
    if w is None:
        return "no router weight on the layer"
    if w.dtype != torch.bfloat16 or w.dim() != 2 or w.size(0) != cache.E:
        return f"router weight {tuple(w.shape)} {w.dtype} is not bf16 [{cache.E}, hidden]"
    if not w.is_contiguous() or w.size(1) % 8 or w.size(1) > 16384 or w.data_ptr() % 16:
        return "router weight layout (contiguous rows, hidden % 8, <= 16384, 16 B aligned)"
    if cache.E > 2048:
        return "more than 2048 experts"
    return None


def _link_prefetch(armed: list, logger) -> int:
    """Chain consecutive armed layers so each predicts and prefetches the next one's
    experts.  ``armed``: (layer, cache) in model order.  Expert-parallel layers are not
    linked (their routing ids are global, their caches local)."""
    linked = 0
    for (li, ci), (lj, cj) in zip(armed, armed[1:]):
        if getattr(li, "expert_map", None) is not None or \
                getattr(lj, "expert_map", None) is not None:
            continue
        w = _router_weight(lj)
        why = _prefetch_unusable(w, cj)
        if why is not None:
            logger.info("expert-cache: no prefetch into %s -- %s", type(lj).__name__, why)
            continue
        ci.next, ci.next_gate = cj, w
        ci.pred = torch.empty((ci.S,), dtype=torch.int32, device=ci.device)
        ci.prefetch_top = settings.prefetch
        linked += 1
    return linked


def _prefetch_allowed() -> bool:
    """A fork must be joined inside the same CUDA graph: allowed eagerly and in vLLM's
    FULL graphs, not while it captures PIECEWISE graphs (the next layer's MoE lies in
    another piece)."""
    try:
        from vllm.forward_context import get_forward_context, is_forward_context_available
    except Exception:
        return True
    if not is_forward_context_available():
        return True
    mode = getattr(get_forward_context(), "cudagraph_runtime_mode", None)
    return getattr(mode, "name", "NONE") != "PIECEWISE"


def _fork_prefetch(cache: ExpertSlotCache, x: torch.Tensor, k: int) -> None:
    """Predict the next layer's routing from this layer's MoE input and install its top
    ``prefetch_top`` experts per token on the side stream; the next layer's apply joins
    before touching its cache."""
    nxt = cache.next
    if not nxt.routed_is_step:
        # The next layer's `routed` does not hold its last real step (its last call was a
        # prefetch, a split chunk or a read-through), so a prefetch could evict experts
        # that step needs: skip until the next layer has run a full cached step again.
        return
    T = x.size(0)
    k = min(k, cache.prefetch_top)
    if T * k > cache.pred.numel() or x.dim() != 2 or x.dtype != torch.bfloat16 or \
            x.stride(1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16:
        return
    if not _prefetch_allowed():
        return
    dev = cache.device.index if cache.device.index is not None else \
        torch.cuda.current_device()
    side = _side_streams.get(dev)
    if side is None:
        side = _side_streams[dev] = torch.cuda.Stream(device=cache.device)
    if nxt.ready is None:
        nxt.ready = torch.cuda.Event()
    main = torch.cuda.current_stream(cache.device)
    side.wait_stream(main)              # x is written and this layer's gather is enqueued
    x.record_stream(side)
    with torch.cuda.stream(side):
        pred = cache.pred[:T * k]
        ExpertSlotCache.pregate(x, cache.next_gate, k, pred)
        nxt.prefetch(pred)
        nxt.ready.record(side)
    nxt.pending = True


def _join_prefetch(cache: ExpertSlotCache) -> None:
    if cache.pending:
        torch.cuda.current_stream(cache.device).wait_event(cache.ready)
        cache.pending = False


def _weight_names(layer) -> tuple[str, str] | None:
    for pair in _WEIGHT_PAIRS:
        if all(isinstance(getattr(layer, n, None), torch.Tensor) for n in pair):
            return pair
    return None


def arm(layer, method, logger) -> bool:
    """Attach a slot cache to one MoE layer; True when the cache is live."""
    kind = type(method).__name__
    names = _weight_names(layer)
    if names is None:
        present = sorted(n for n, _ in layer.named_parameters(recurse=False))
        if any("w13" in n or "w2" in n for n in present):
            logger.warning("expert-cache: not caching %s -- no recognised expert weight "
                           "pair; the layer registers %s", kind, ", ".join(present))
        return False
    w13_name, w2_name = names
    num_experts = getattr(layer, w13_name).size(0)
    slots = settings.slots_for(num_experts)
    if slots >= num_experts:
        return False            # everything fits already; a cache would duplicate VRAM

    reason = _decline(layer, method, num_experts)
    if reason is not None:
        logger.warning("expert-cache: not caching %s -- %s", kind, reason)
        return False

    groups = _per_expert_tensors(layer, num_experts)
    owner_of = {n: canon for canon, group in groups.items() for n in group}
    for name in (w13_name, w2_name):
        if name not in owner_of:
            logger.warning("expert-cache: not caching %s -- %s is not a directly-owned "
                           "expert-major tensor (found: %s)", kind, name,
                           ", ".join(sorted(owner_of)) or "none")
            return False
    required = set(groups[owner_of[w13_name]]) | set(groups[owner_of[w2_name]])
    try:
        cache = ExpertSlotCache(layer, groups.keys(), num_experts, slots,
                                getattr(layer, w13_name).device, required=required)
    except ValueError as e:
        logger.warning("expert-cache: not caching %s -- %s", kind, e)
        return False

    # One Parameter wrapper per slot storage, shared by all its registered aliases;
    # plain-attribute aliases get the bare tensor.
    cache.bound = {}
    for canon, group in groups.items():
        if canon not in cache.slots:
            continue
        slot = cache.slots[canon]
        param = torch.nn.Parameter(slot, requires_grad=False)
        for name in group:
            cache.bound[name] = param if name in layer._parameters else slot
    if cache.skipped:
        logger.info("expert-cache: not mirroring %s (not 16-byte aligned per expert); the "
                    "leak check decides whether that matters", ", ".join(cache.skipped))

    with _slot_bound(layer, cache):
        slot_cfg = method.get_fused_moe_quant_config(layer)
    if slot_cfg is not None:
        leaked = _leaked_full_tensors(slot_cfg, num_experts)
        if leaked:
            logger.warning("expert-cache: not caching %s -- these per-expert tensors "
                           "stayed bound to full [%d] storage after slot binding and would "
                           "be indexed by slot id: %s", kind, num_experts, ", ".join(leaked))
            return False

    stock_apply = method.apply
    debug_left = [settings.debug_calls]
    ep_name = _expert_map_name(layer) if getattr(layer, "expert_map", None) is not None \
        else None
    split_max = settings.split_wide
    if split_max:
        why = _token_local(slot_cfg)
        if why is not None:
            logger.info("expert-cache: not splitting wide steps of %s -- %s", kind, why)
            split_max = 0
    split = [split_max]

    def cached(layer, x, topk_weights, topk_ids, shared_experts, shared_experts_input,
               fork=True):
        experts = method.moe_kernel.fused_experts
        saved = (experts.quant_config, method.moe_quant_config, layer.global_num_experts)
        if ep_name is None:
            ids = cache.refresh(topk_ids)
            cache.routed_is_step = fork       # a split chunk flags only its own tokens
            layer.global_num_experts = cache.S
            # one prefetch per real step: a prefetch parks the experts flagged by the call
            # before it, which must be this layer's step, not another prefetch
            if fork and cache.next is not None and topk_ids.dim() == 2 and \
                    isinstance(x, torch.Tensor):
                _fork_prefetch(cache, x, topk_ids.size(1))
        else:
            # Expert parallel: the routing ids stay global; the layer's expert map is
            # replaced by the composed global id -> slot map for this step.
            ids = topk_ids
            full_map = getattr(layer, ep_name)
            _set_tensor(layer, ep_name, cache.refresh_ep(topk_ids, full_map))
        experts.quant_config = slot_cfg
        method.moe_quant_config = slot_cfg
        try:
            with _slot_bound(layer, cache):
                return stock_apply(layer, x, topk_weights, ids, shared_experts,
                                   shared_experts_input)
        finally:
            experts.quant_config, method.moe_quant_config, layer.global_num_experts = saved
            if ep_name is not None:
                _set_tensor(layer, ep_name, full_map)

    def chunk_tokens(x, topk_ids, shared_experts) -> int:
        """Tokens per chunk when this wide step may be split, else 0 (read through)."""
        if not split[0] or shared_experts is not None or topk_ids.dim() != 2:
            return 0
        if not isinstance(x, torch.Tensor) or x.size(0) != topk_ids.size(0):
            return 0
        per = cache.S // max(1, topk_ids.size(1))
        if per < 1 or -(-topk_ids.size(0) // per) > split[0]:
            return 0
        return per

    # vLLM calls apply by keyword: these parameter names are part of the contract.
    def apply(layer, x, topk_weights, topk_ids, shared_experts=None,
              shared_experts_input=None):
        _join_prefetch(cache)            # a prefetch into this layer may be in flight
        fits = cache.fits(topk_ids)
        per = 0 if fits else chunk_tokens(x, topk_ids, shared_experts)
        if debug_left[0] > 0:
            debug_left[0] -= 1
            path = ("cached" if fits else
                    f"split {-(-topk_ids.size(0) // per)}" if per else "read-through")
            logger.warning("expert-cache debug: %s topk_ids %s %s -> %s", kind,
                           tuple(topk_ids.shape), topk_ids.dtype, path)
        if fits:
            return cached(layer, x, topk_weights, topk_ids, shared_experts,
                          shared_experts_input)
        if not per:
            cache.routed_is_step = False      # read through: `routed` is not this step's
            return stock_apply(layer, x, topk_weights, topk_ids, shared_experts,
                               shared_experts_input)
        # Each chunk is an ordinary cached step over consecutive tokens; a token's output
        # depends only on its own row (checked by _token_local at arm time).
        outs = []
        for lo in range(0, topk_ids.size(0), per):
            out = cached(layer, x[lo:lo + per], topk_weights[lo:lo + per],
                         topk_ids[lo:lo + per], None, None, fork=False)
            if not isinstance(out, torch.Tensor):
                logger.warning("expert-cache: %s apply returned %s, not a tensor; wide "
                               "steps read through from now on", kind, type(out).__name__)
                split[0] = 0
                return stock_apply(layer, x, topk_weights, topk_ids, shared_experts,
                                   shared_experts_input)
            outs.append(out)
        return torch.cat(outs, dim=0)

    method.apply = apply
    layer._expert_cache = cache
    return True


def _arm_model(model, logger, method_base) -> None:
    armed = declined = 0
    first = None
    chain = []
    seen: set[int] = set()
    for _, module in model.named_modules():
        method = getattr(module, "quant_method", None)
        if not isinstance(method, method_base):
            continue
        if id(method) in seen:
            # A quant_method shared by two layers would bind its slot config to the first
            # layer's buffers and serve the second from them: leave the extras uncached.
            logger.warning("expert-cache: %s instance is shared across layers; leaving the "
                           "extra layers uncached", type(method).__name__)
            declined += 1
            continue
        try:
            if arm(module, method, logger):
                armed += 1
                seen.add(id(method))
                first = first or module._expert_cache
                chain.append((module, module._expert_cache))
            else:
                declined += 1
        except Exception as e:   # never break serving: the layer keeps the stock path
            logger.warning("expert-cache: disabled for layer (%r)", e)
            module._expert_cache = None
            declined += 1
    if first is None:
        logger.info("expert-cache: no cacheable MoE layer found; staying out of the way")
        return
    from .. import __version__
    logger.info("expert-cache %s active on %d MoE layer(s) (%d declined): %d/%d experts "
                "resident, mirroring %s, policy=%s", __version__, armed, declined, first.S,
                first.E, "+".join(first.names), settings.policy)
    if settings.prefetch:
        logger.info("expert-cache: next-layer prefetch linked %d of %d layer pairs",
                    _link_prefetch(chain, logger), max(len(chain) - 1, 0))


def install(logger) -> bool:
    """Wrap vLLM's post-load hook so every MoE layer is armed once weights are final."""
    global _installed
    if _installed:
        return True
    try:
        from vllm.model_executor.layers.fused_moe.fused_moe_method_base import (
            FusedMoEMethodBase)
        from vllm.model_executor.model_loader import utils as loader_utils
    except Exception as e:
        logger.debug("expert-cache: vLLM MoE interfaces unavailable (%r)", e)
        return False

    stock = loader_utils.process_weights_after_loading

    def process_weights_after_loading(model, model_config, target_device):
        stock(model, model_config, target_device)
        if not settings.disabled:
            _arm_model(model, logger, FusedMoEMethodBase)

    # base_loader imports the function by name, so rebind every module holding it as
    # well as the defining module (patching only the latter leaves the hook inert).
    # Module dicts are read directly: getattr on lazy modules (transformers') would
    # import or alias-resolve names as a side effect.
    rebound = []
    for modname, mod in list(sys.modules.items()):
        namespace = getattr(mod, "__dict__", None) if mod is not None else None
        if isinstance(namespace, dict) and \
                namespace.get("process_weights_after_loading") is stock:
            setattr(mod, "process_weights_after_loading", process_weights_after_loading)
            rebound.append(modname.rsplit(".", 1)[-1])
    loader_utils.process_weights_after_loading = process_weights_after_loading
    logger.info("expert-cache: hooked the MoE loader in %s", ", ".join(rebound) or "utils")
    _installed = True
    return True
