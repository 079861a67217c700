"""Seeded synthetic inputs for the benchmarks and tests: routing traces and W8A8 slabs.

Benchmark and test helper only: it sits beside ``bench.py`` and is not part of the
installed ``vllm_expert_cache`` plugin.  No real checkpoint or captured routing is
available, so the benchmarks and tests use these stand-ins, sized and distributed like
the workloads the cache is measured on:

* :func:`sticky_zipf_trace` -- decode routing with temporal locality: 8 distinct experts
  per token; each position keeps the previous token's expert with probability ``p_keep``,
  otherwise draws from a Zipf(``s``) law over a seeded permutation of the expert ids,
  rejecting ids already chosen for this token.
* :func:`qwen3_30b_a3b_experts` -- per-expert W8A8 slabs of a Qwen3-30B-A3B MoE layer
  (w13 int8 [2*768, 2048], w2 int8 [2048, 768], fp32 per-output-row scales), uniform int8
  weights and scales uniform in [1e-3, 1e-2].
"""

from __future__ import annotations

import numpy as np
import torch

# Qwen3-30B-A3B MoE layer: hidden 2048, moe_intermediate 768, 128 experts, top-8.
QWEN3_30B = dict(E=128, top_k=8, hidden=2048, inter=768)


def sticky_zipf_trace(seed: int, steps: int = 4096, E: int = 128, k: int = 8,
                      s: float = 1.1, p_keep: float = 0.7, tokens: int = 1) -> np.ndarray:
    """``[steps, tokens*k]`` int32 routing ids; each token's ``k`` ids are distinct."""
    if k > E:
        raise ValueError("top-k larger than the expert count")
    rng = np.random.default_rng(seed)
    perm = rng.permutation(E).astype(np.int32)
    w = np.arange(1, E + 1, dtype=np.float64) ** (-s)
    cdf = np.cumsum(w / w.sum())
    cdf[-1] = 1.0
    out = np.empty((steps, tokens, k), dtype=np.int32)
    prev = [None] * tokens
    for t in range(steps):
        for tok in range(tokens):
            chosen: list[int] = []
            last = prev[tok]
            for j in range(k):
                if last is not None and rng.random() < p_keep and last[j] not in chosen:
                    chosen.append(int(last[j]))
                    continue
                while True:
                    e = int(perm[int(np.searchsorted(cdf, rng.random(), side="right"))])
                    if e not in chosen:
                        break
                chosen.append(e)
            out[t, tok] = chosen
            prev[tok] = chosen
    return out.reshape(steps, tokens * k)


def qwen3_30b_a3b_experts(E: int = 128, seed: int = 0, tp: int = 1, pin: bool = True,
                          hidden: int = 2048, inter: int = 768) -> dict[str, torch.Tensor]:
    """Host-resident W8A8 expert tensors in vLLM's registration order.

    Shapes follow vLLM's compressed-tensors W8A8 int8 MoE method: ``w13_weight``
    [E, 2*inter/tp, hidden], ``w2_weight`` [E, hidden, inter/tp], ``w13_weight_scale``
    [E, 2*inter/tp, 1] and ``w2_weight_scale`` [E, hidden, 1] (fp32).
    """
    g = torch.Generator().manual_seed(seed)
    i = inter // tp
    shapes = {
        "w13_weight": ((E, 2 * i, hidden), torch.int8),
        "w2_weight": ((E, hidden, i), torch.int8),
        "w13_weight_scale": ((E, 2 * i, 1), torch.float32),
        "w2_weight_scale": ((E, hidden, 1), torch.float32),
    }
    out = {}
    for name, (shape, dt) in shapes.items():
        t = torch.empty(shape, dtype=dt, pin_memory=pin)
        if dt == torch.int8:
            t.copy_(torch.randint(-128, 128, shape, dtype=torch.int8, generator=g))
        else:
            t.copy_(torch.rand(shape, generator=g) * 9e-3 + 1e-3)
        out[name] = t
    return out


def bytes_per_expert(t: torch.Tensor) -> int:
    return (t.numel() // t.shape[0]) * t.element_size()


# ---------------------------------------------------------------------------------------
# UVA views of pinned host memory: what vLLM's expert offload leaves on the layer.

_TYPESTR = {torch.int8: "|i1", torch.uint8: "|u1", torch.int16: "<i2", torch.int32: "<i4",
            torch.int64: "<i8", torch.float16: "<f2", torch.float32: "<f4"}


def host_device_pointer(host: torch.Tensor) -> int:
    """Device address of a pinned host tensor (``cudaHostGetDevicePointer``)."""
    import ctypes
    if not host.is_pinned():
        raise ValueError("host tensor is not pinned")
    torch.cuda.init()
    rt = ctypes.CDLL("libcudart.so.12")
    rt.cudaHostGetDevicePointer.restype = ctypes.c_int
    rt.cudaHostGetDevicePointer.argtypes = [ctypes.POINTER(ctypes.c_void_p),
                                            ctypes.c_void_p, ctypes.c_uint]
    dp = ctypes.c_void_p()
    rc = rt.cudaHostGetDevicePointer(ctypes.byref(dp), ctypes.c_void_p(host.data_ptr()), 0)
    if rc != 0:
        raise RuntimeError(f"cudaHostGetDevicePointer failed rc={rc}")
    return int(dp.value)


class _CudaArray:
    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3,
                                         "strides": None}


def uva_view(host: torch.Tensor, device: str | torch.device = "cuda") -> torch.Tensor:
    """A CUDA tensor aliasing ``host`` (pinned): every read crosses the host link.

    The caller keeps ``host`` alive for as long as the view is used.
    """
    ptr = host_device_pointer(host)
    try:
        if host.dtype == torch.bfloat16:
            return torch.as_tensor(_CudaArray(ptr, host.shape, "<i2"), device=device).view(
                torch.bfloat16)
        return torch.as_tensor(_CudaArray(ptr, host.shape, _TYPESTR[host.dtype]),
                               device=device)
    except (RuntimeError, TypeError):
        # torch refused a host-resident interface pointer: use vLLM's own view op, the
        # one its UVA offloader calls (vllm/model_executor/offloader/uva.py)
        from vllm.utils.torch_utils import get_accelerator_view_from_cpu_tensor
        return get_accelerator_view_from_cpu_tensor(host)
