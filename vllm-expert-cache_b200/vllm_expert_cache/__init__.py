"""Device-side expert cache for vLLM MoE models, built for NVIDIA B200 (sm_100a).

A bounded set of experts stays in HBM "slots"; the rest stay where vLLM's
``--cpu-offload-params experts`` put them (pinned host memory mapped into the GPU's
address space).  vLLM loads this package through its ``vllm.general_plugins`` entry point
(``expert_cache = vllm_expert_cache:install``); installing it is the whole integration.
``EXPERT_CACHE_DISABLE=1`` turns it off.
"""

from __future__ import annotations

from .config import settings

__all__ = ["install", "settings"]
__version__ = "0.3.0+b200"


def _logger():
    # vLLM attaches handlers to the "vllm" logger tree only; a logger outside it would
    # print nothing in a real server (reference vllm_expert_cache/__init__.py:21-29).
    try:
        from vllm.logger import init_logger
        return init_logger("vllm.expert_cache")
    except Exception:  # vLLM absent: plain logging under the same name
        import logging
        return logging.getLogger("vllm.expert_cache")


def install() -> None:
    """Plugin entry point: hook vLLM's post-load step so every MoE layer gets armed."""
    log = _logger()
    if settings.disabled:
        log.info("expert-cache: disabled by EXPERT_CACHE_DISABLE")
        return
    from .backends import generic
    if not generic.install(log):
        log.info("expert-cache: could not hook vLLM's MoE loader; staying out of the way")
