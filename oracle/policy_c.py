"""ctypes binding of oracle/policy.c.  TEST INFRASTRUCTURE ONLY."""

from __future__ import annotations

import ctypes

import numpy as np

from .build import OUT, build
from .policy import CacheState

_H = None


def lib():
    global _H
    if _H is None:
        build()
        h = ctypes.CDLL(str(OUT))
        P, I = ctypes.c_void_p, ctypes.c_int
        h.oracle_manage.restype = I
        h.oracle_manage.argtypes = [P, I, I, I, I, I] + [P] * 8 + [I, I]
        h.oracle_run.restype = ctypes.c_longlong
        h.oracle_run.argtypes = [P, I, I, I, I, I, I] + [P] * 8 + [I, I, P]
        h.oracle_remap.restype = None
        h.oracle_remap.argtypes = [P, I, I, P, P, I]
        h.oracle_gather.restype = None
        h.oracle_gather.argtypes = [I, P, P, P, P, P]
        _H = h
    return _H


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return ctypes.c_void_p(a.ctypes.data)


def _state_ptrs(st: CacheState):
    return [_p(st.table), _p(st.map_cold), _p(st.slot_expert), _p(st.slot_stamp),
            _p(st.routed), _p(st.step), _p(st.miss), _p(st.n_miss)]


def manage(st: CacheState, ids, max_distinct, max_inserts, policy, decay) -> int:
    """One step in place; returns the C rc (0 / -1).  Same contract as policy.manage."""
    ids = np.ascontiguousarray(np.asarray(ids).reshape(-1), dtype=np.int32)
    return lib().oracle_manage(_p(ids), ids.size, st.E, st.S, max_distinct, max_inserts,
                               *_state_ptrs(st), policy, decay)


def run(st: CacheState, trace, max_distinct, max_inserts, policy, decay):
    """Replay ``trace`` ([steps, mk] int) in place; returns per-step n_miss (int32)."""
    trace = np.ascontiguousarray(trace, dtype=np.int32)
    steps, mk = trace.shape
    nm = np.zeros(steps, dtype=np.int32)
    rc = lib().oracle_run(_p(trace), steps, mk, st.E, st.S, max_distinct, max_inserts,
                          *_state_ptrs(st), policy, decay, _p(nm))
    if rc < 0:
        raise ValueError("oracle_run refused the arguments")
    return nm


def remap(table: np.ndarray, ids, out_elem_bytes: int = 4) -> np.ndarray:
    ids = np.ascontiguousarray(np.asarray(ids).reshape(-1), dtype=np.int32)
    out = np.empty(ids.size, dtype=np.int64 if out_elem_bytes == 8 else np.int32)
    lib().oracle_remap(_p(ids), ids.size, table.shape[0], _p(table), _p(out),
                       out_elem_bytes)
    return out


def gather(dsts, srcs, nbytes, miss, n_miss) -> None:
    n = len(dsts)
    D = (ctypes.c_void_p * n)(*[d.ctypes.data for d in dsts])
    S_ = (ctypes.c_void_p * n)(*[s.ctypes.data for s in srcs])
    B = (ctypes.c_long * n)(*nbytes)
    miss = np.ascontiguousarray(miss, dtype=np.int32)
    n_miss = np.ascontiguousarray(n_miss, dtype=np.int32)
    lib().oracle_gather(n, D, S_, B, _p(miss), _p(n_miss))
