"""Helpers for the GPU tests: device mirrors of the oracle state, C-ABI call wrappers and
UVA views of pinned host memory (what vLLM's ``--cpu-offload-params experts`` hands the
cache)."""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from oracle.policy import CacheState

DEV = "cuda:0"
FIELDS = ("table", "map_cold", "slot_expert", "slot_stamp", "routed", "step", "miss",
          "n_miss")


def lib():
    import build_lib
    build_lib.build()
    from vllm_expert_cache import _lib
    return _lib.lib()


def stream_ptr():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def p(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


class DeviceState:
    """The eight state tensors on the GPU, initialised from an oracle CacheState."""

    def __init__(self, st: CacheState, device=DEV):
        self.E, self.S = st.E, st.S
        for f in FIELDS:
            setattr(self, f, torch.from_numpy(getattr(st, f).copy()).to(device))

    def ptrs(self):
        return [p(getattr(self, f)) for f in FIELDS]

    def host(self) -> dict:
        return {f: getattr(self, f).cpu().numpy() for f in FIELDS}


def manage(h, ds: DeviceState, ids_t: torch.Tensor, md, mi, policy, decay, out=None):
    if out is None:
        rc = h.expert_cache_manage(p(ids_t), ids_t.numel(), ds.E, ds.S, md, mi, *ds.ptrs(),
                                   policy, decay, stream_ptr())
    else:
        rc = h.expert_cache_manage_remap(p(ids_t), ids_t.numel(), ds.E, ds.S, md, mi,
                                         *ds.ptrs(), policy, decay, p(out),
                                         out.element_size(), stream_ptr())
    assert rc == 0, f"manage rc={rc}"


def gather(h, triples, miss, n_miss, chunks=16, lanes=64):
    """triples: list of (dst_ptr, src_ptr, bytes) with up to 6 entries (padded here)."""
    triples = list(triples) + [triples[-1]] * (6 - len(triples))
    args = []
    for d, s, b in triples:
        args += [ctypes.c_void_p(d), ctypes.c_void_p(s), ctypes.c_long(b)]
    return h.expert_cache_gather(*args, p(miss), p(n_miss), chunks, lanes, stream_ptr())


def compare_state(ds_host: dict, st: CacheState, nins: int, tag: str) -> None:
    """Every field after a step, including the miss-list entries the kernel defines."""
    for f in ("table", "map_cold", "slot_expert", "slot_stamp", "routed", "step", "n_miss"):
        np.testing.assert_array_equal(ds_host[f], getattr(st, f), err_msg=f"{tag}: {f}")
    n = int(st.n_miss[0])
    got, want = ds_host["miss"], st.miss
    np.testing.assert_array_equal(got[0:2 * nins:2], want[0:2 * nins:2],
                                  err_msg=f"{tag}: miss experts")
    np.testing.assert_array_equal(got[1:2 * n:2], want[1:2 * n:2], err_msg=f"{tag}: miss slots")


def device_ptr_of_pinned(host: torch.Tensor) -> int:
    from synthetic import host_device_pointer
    return host_device_pointer(host)


def uva_view(host: torch.Tensor) -> torch.Tensor:
    """A CUDA tensor aliasing pinned host memory (reads cross the host link)."""
    from synthetic import uva_view as _view
    return _view(host, DEV)
