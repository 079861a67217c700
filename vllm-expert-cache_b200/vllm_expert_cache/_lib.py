"""ctypes binding of libexpertcache.so (the B200 build of the reference's C-ABI).

Search order, as in the reference (vllm_expert_cache/_lib.py:17-33): $EXPERT_CACHE_LIB,
then ``libexpertcache.so`` beside this package, then /usr/local/lib.  A missing library
raises FileNotFoundError; there is no fallback path.  The handle is loaded once per
process.  Argument types are the reference's (_lib.py:41-53) plus the fused-remap,
expert-parallel, prefetch and single-launch step entry points this build adds.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

# Six (dst, src, bytes) triples per gather call (reference _lib.py:61).
GATHER_SLOTS = 6
# Largest slot count of the single-launch step (EXPERT_CACHE_STEP_MAX_SLOTS).
STEP_MAX_SLOTS = 256

_P, _I, _L = ctypes.c_void_p, ctypes.c_int, ctypes.c_long
MANAGE_ARGTYPES = [_P] + [_I] * 5 + [_P] * 8 + [_I] * 2 + [_P]
MANAGE_REMAP_ARGTYPES = [_P] + [_I] * 5 + [_P] * 8 + [_I] * 2 + [_P, _I, _P]
MANAGE_EP_ARGTYPES = [_P, _I, _P] + [_I] * 5 + [_P] * 8 + [_I] * 2 + [_P, _P]
PREFETCH_ARGTYPES = [_P] + [_I] * 5 + [_P] * 8 + [_I, _P]
PREGATE_ARGTYPES = [_P, _I, _I, _I, _P, _I, _I, _P, _P]
GATHER_ARGTYPES = [_P, _P, _L] * GATHER_SLOTS + [_P, _P, _I, _I, _P]
STEP_ARGTYPES = ([_P] + [_I] * 5 + [_P] * 8 + [_I] * 2 + [_P, _I] + [_P, _P, _L] * GATHER_SLOTS
                 + [_I, _I, _P, _I, _P])

_handle = None


def _candidates():
    yield os.environ.get("EXPERT_CACHE_LIB")
    yield str(Path(__file__).resolve().parent / "libexpertcache.so")
    yield "/usr/local/lib/libexpertcache.so"


def library_path() -> str:
    for cand in _candidates():
        if cand and Path(cand).is_file():
            return cand
    raise FileNotFoundError(
        "libexpertcache.so not found: build it with "
        "`python vllm-expert-cache_b200/build_lib.py` (nvcc, sm_100a) so it lands beside "
        "this package, or set EXPERT_CACHE_LIB to its path.")


def bind(h: ctypes.CDLL) -> ctypes.CDLL:
    h.expert_cache_manage.restype = _I
    h.expert_cache_manage.argtypes = MANAGE_ARGTYPES
    h.expert_cache_manage_remap.restype = _I
    h.expert_cache_manage_remap.argtypes = MANAGE_REMAP_ARGTYPES
    h.expert_cache_manage_ep.restype = _I
    h.expert_cache_manage_ep.argtypes = MANAGE_EP_ARGTYPES
    h.expert_cache_prefetch.restype = _I
    h.expert_cache_prefetch.argtypes = PREFETCH_ARGTYPES
    h.expert_cache_pregate.restype = _I
    h.expert_cache_pregate.argtypes = PREGATE_ARGTYPES
    h.expert_cache_gather.restype = _I
    h.expert_cache_gather.argtypes = GATHER_ARGTYPES
    h.expert_cache_step.restype = _I
    h.expert_cache_step.argtypes = STEP_ARGTYPES
    return h


def lib() -> ctypes.CDLL:
    """The bound library, loaded on first use."""
    global _handle
    if _handle is None:
        _handle = bind(ctypes.CDLL(library_path()))
    return _handle
