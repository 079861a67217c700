"""Per-MoE-layer expert slot cache: state tensors plus the per-forward step driver.

The full expert tensors stay where vLLM's offloader put them (pinned host memory seen by
the GPU through UVA); this class adds ``S`` device-resident slots per expert tensor and
the policy state that decides which experts occupy them.  One cached forward step is one
``expert_cache_step`` launch (S <= 256):

  1. its first CTA runs the policy step on the routed ids -- hits refreshed, victims
     chosen among slots this step does not need, table / miss list rewritten -- and
     remaps the routing ids expert -> slot;
  2. then all its CTAs copy every missing expert's slabs from host memory into their new
     slots (six tensors per launch; a wider set adds ``expert_cache_gather`` launches).

With more than 256 slots (or EXPERT_CACHE_SINGLE_LAUNCH=0) the same step is two launches,
``expert_cache_manage_remap`` then ``expert_cache_gather``.

Nothing reads a device value back, so the step is recorded into CUDA graphs like any
other kernel sequence; every rank that sees the same routing evolves the same state.

Interface and behaviour follow the reference class ``ExpertSlotCache``
(vllm_expert_cache/cache.py:38-163): constructor arguments, the 16-byte slab rule, the
``fits`` shape gate, ``remap`` semantics and ``refresh``'s return value.  The difference
is that the remap runs inside the manage kernel instead of as torch ops.
"""

from __future__ import annotations

import ctypes

import torch

from ._lib import GATHER_SLOTS, STEP_MAX_SLOTS, lib
from .config import settings


def _bytes_per_expert(t: torch.Tensor) -> int:
    return (t.numel() // t.shape[0]) * t.element_size()


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


class ExpertSlotCache:
    """``num_slots`` of ``num_experts`` experts resident in device memory."""

    def __init__(self, owner, source_names, num_experts: int, num_slots: int, device,
                 required=()):
        # Sources are looked up on `owner` at every step: vLLM's offloader moves them to
        # host memory after weight loading, so a pointer taken here would dangle.
        self.owner = owner
        self.names = list(source_names)
        self.E = int(num_experts)
        self.S = int(num_slots)
        self.device = torch.device(device)

        self.slots: dict[str, torch.Tensor] = {}
        self.skipped: list[str] = []
        fatal = []
        for name in self.names:
            full = getattr(owner, name).data
            nbytes = _bytes_per_expert(full)
            if nbytes % 16:
                # The gather moves 16-byte vectors.  A ragged weight would be handed to
                # the GEMM half-copied, so it is fatal; a ragged auxiliary tensor is left
                # unmirrored and the caller's leak check decides whether it matters.
                where = fatal if name in required else self.skipped
                where.append(f"{name}{tuple(full.shape)}={nbytes}B")
                continue
            self.slots[name] = torch.empty((self.S,) + tuple(full.shape[1:]),
                                           dtype=full.dtype, device=self.device)
        if fatal:
            raise ValueError("per-expert slab must be a multiple of 16 bytes, but these "
                             "are not: " + ", ".join(fatal))
        self.names = [n for n in self.names if n in self.slots]
        # Names -> tensors bound on the layer during a cached step (arming may widen it
        # with aliases and Parameter wrappers).
        self.bound: dict[str, torch.Tensor] = dict(self.slots)

        dev = self.device
        self.table = torch.full((self.E,), -1, dtype=torch.int32, device=dev)
        self.map_cold = torch.arange(self.E, dtype=torch.int32, device=dev)
        self.slot_expert = torch.full((self.S,), -1, dtype=torch.int32, device=dev)
        self.slot_stamp = torch.zeros((self.S,), dtype=torch.int64, device=dev)
        self.routed = torch.zeros((self.E,), dtype=torch.uint8, device=dev)
        self.step = torch.zeros((1,), dtype=torch.int64, device=dev)
        self.miss = torch.zeros((2 * self.S,), dtype=torch.int32, device=dev)
        self.n_miss = torch.zeros((1,), dtype=torch.int32, device=dev)
        # expert_cache_step's per-launch words, its count of timed-out waits ([5]) and its
        # running install count (int64 at [6])
        self.sync = torch.zeros((8,), dtype=torch.int32, device=dev)

        # Opt-in counter: installs summed over every cached step (device int64, no sync).
        self.miss_total = (torch.zeros((1,), dtype=torch.int64, device=dev)
                           if settings.stats else None)

        # Next-layer prefetch wiring (set by the arming code when EXPERT_CACHE_PREFETCH=1):
        # the next armed layer's cache and router weight, a buffer for the predicted ids,
        # and this layer's own in-flight marker (event on the side stream + flag).
        self.next: ExpertSlotCache | None = None
        self.next_gate: torch.Tensor | None = None
        self.pred: torch.Tensor | None = None
        self.prefetch_top = 0           # predictions per token to prefetch
        self.ready = None
        self.pending = False
        # True while `routed` holds this layer's last full cached step (set by the arming
        # code after such a step; cleared by a prefetch, a split chunk or a read-through).
        # A prefetch parks the experts flagged in `routed`, so it is only issued when this
        # holds.
        self.routed_is_step = False
        self.prefetch_total = (torch.zeros((1,), dtype=torch.int64, device=dev)
                               if settings.stats else None)

        self.policy = settings.policy_code
        self.decay = settings.decay
        self.chunks = settings.chunks
        self.lanes = settings.lanes
        self.single_launch = settings.single_launch and self.S <= STEP_MAX_SLOTS
        self._state_args = None

    # ---------------------------------------------------------------------------------
    def fits(self, topk_ids: torch.Tensor) -> bool:
        """Can this step be served from slots?  ``tokens x top_k <= S``: shape only, so
        no device sync; prefill and wide batches fail it and read through."""
        return topk_ids.numel() <= self.S

    def remap(self, topk_ids: torch.Tensor) -> torch.Tensor:
        """``table[topk_ids]`` as torch ops (the reference's remap); ``refresh`` does the
        same inside the manage kernel."""
        return self.table[topk_ids.to(torch.int64)].to(topk_ids.dtype)

    def _state(self):
        if self._state_args is None:
            self._state_args = (
                _ptr(self.table), _ptr(self.map_cold), _ptr(self.slot_expert),
                _ptr(self.slot_stamp), _ptr(self.routed), _ptr(self.step),
                _ptr(self.miss), _ptr(self.n_miss))
        return self._state_args

    def refresh(self, topk_ids: torch.Tensor) -> torch.Tensor:
        """Run one cached step and return the routing ids in slot space."""
        h = lib()
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        ids = topk_ids
        if ids.dtype != torch.int32 or not ids.is_contiguous():
            ids = ids.to(torch.int32).contiguous()
        mk = ids.numel()
        wide = topk_ids.dtype in (torch.int32, torch.int64)
        out = torch.empty(topk_ids.shape, dtype=topk_ids.dtype if wide else torch.int32,
                          device=self.device)
        args = (_ptr(ids), mk, self.E, self.S, min(self.E, mk), self.S, *self._state(),
                self.policy, self.decay, _ptr(out), out.element_size())
        if self.single_launch:
            groups = self._gather_groups()
            rc = h.expert_cache_step(*args, *groups[0], self.chunks, self.lanes,
                                     _ptr(self.sync), 0, stream)
            if rc != 0:
                raise RuntimeError(f"expert_cache_step failed rc={rc}")
            self._gather(h, stream, groups[1:])
        else:
            rc = h.expert_cache_manage_remap(*args, stream)
            if rc != 0:
                raise RuntimeError(f"expert_cache_manage_remap failed rc={rc}")
            self._gather(h, stream)
            if self.miss_total is not None:     # the step kernel counts its own installs
                self.miss_total.add_(self.n_miss)
        return out if wide else out.to(topk_ids.dtype)

    def refresh_ep(self, topk_ids: torch.Tensor, expert_map: torch.Tensor) -> torch.Tensor:
        """One cached step of an expert-parallel layer.

        ``topk_ids`` are global expert ids and ``expert_map`` (int32 [E_global], vLLM's
        global id -> local expert or -1) selects this rank's experts, which are the
        cache's E.  Returns the composed map global id -> slot (int32 [E_global], -1 where
        the expert is not resident here) to pass as the stock kernel's ``expert_map``; the
        routing ids themselves stay global.  One ``expert_cache_manage_ep`` launch, then
        the gather.
        """
        h = lib()
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        ids = topk_ids
        if ids.dtype != torch.int32 or not ids.is_contiguous():
            ids = ids.to(torch.int32).contiguous()
        emap = expert_map
        if emap.dtype != torch.int32 or not emap.is_contiguous():
            emap = emap.to(torch.int32).contiguous()
        mk = ids.numel()
        out = torch.empty((emap.numel(),), dtype=torch.int32, device=self.device)
        rc = h.expert_cache_manage_ep(
            _ptr(ids), mk, _ptr(emap), emap.numel(), self.E, self.S, min(self.E, mk),
            self.S, *self._state(), self.policy, self.decay, _ptr(out), stream)
        if rc != 0:
            raise RuntimeError(f"expert_cache_manage_ep failed rc={rc}")
        if self.miss_total is not None:
            self.miss_total.add_(self.n_miss)
        self._gather(h, stream)
        return out

    def prefetch(self, pred_ids: torch.Tensor) -> None:
        """Install the predicted experts that are missing (``expert_cache_prefetch``, then
        the gather) on the current stream.  ``pred_ids``: int32, contiguous, on device.
        The layer's own next step still installs whatever it routes, so a wrong
        prediction costs transfers, never results."""
        h = lib()
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        mk = pred_ids.numel()
        rc = h.expert_cache_prefetch(_ptr(pred_ids), mk, self.E, self.S, min(self.E, mk),
                                     self.S, *self._state(), self.policy, stream)
        if rc != 0:
            raise RuntimeError(f"expert_cache_prefetch failed rc={rc}")
        if self.prefetch_total is not None:
            self.prefetch_total.add_(self.n_miss)
        self.routed_is_step = False       # `routed` now holds the predicted flags
        self._gather(h, stream)

    @staticmethod
    def pregate(x: torch.Tensor, gate_w: torch.Tensor, k: int, out: torch.Tensor) -> None:
        """``out[t*k + r]`` = the r-th best expert of token t under router ``gate_w``
        (``expert_cache_pregate``; bf16 x rows with unit inner stride)."""
        h = lib()
        stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
        rc = h.expert_cache_pregate(_ptr(x), x.size(0), x.stride(0), x.size(1), _ptr(gate_w),
                                    gate_w.size(0), k, _ptr(out), stream)
        if rc != 0:
            raise RuntimeError(f"expert_cache_pregate failed rc={rc}")

    def stats(self) -> dict:
        """Host snapshot of the counters (synchronises; call outside the hot path)."""
        sync = self.sync.cpu()
        step_installs = int(sync[6:8].view(torch.int64)[0])
        out = {"experts": self.E, "slots": self.S, "steps": int(self.step.item()),
               "step_timeouts": int(sync[5])}
        if self.single_launch or self.miss_total is not None:
            # the single-launch step counts installs itself; the two-launch path (S > 256,
            # EXPERT_CACHE_SINGLE_LAUNCH=0, EP steps) only with EXPERT_CACHE_STATS=1
            other = int(self.miss_total.item()) if self.miss_total is not None else 0
            out["installs"] = step_installs + other
            out["bytes_per_install"] = sum(_bytes_per_expert(getattr(self.owner, n).data)
                                           for n in self.names)
        if self.prefetch_total is not None:
            out["prefetch_installs"] = int(self.prefetch_total.item())
        return out

    def step_timeouts(self) -> int:
        """CTAs of ``expert_cache_step`` whose wait for the policy step ran out, summed over
        every call (0 in normal operation; synchronises, so call it outside the hot path)."""
        return int(self.sync[5].item())

    def _gather_groups(self) -> list[list]:
        """The (dst, src, bytes) arguments of every gather launch, six triples each."""
        triples = []
        for name in self.names:
            src = getattr(self.owner, name).data
            triples.append((_ptr(self.slots[name]), _ptr(src),
                            ctypes.c_long(_bytes_per_expert(src))))
        groups = []
        for i in range(0, len(triples), GATHER_SLOTS):
            group = triples[i:i + GATHER_SLOTS]
            # pad with the group's last triple: the kernel copies a repeated triple once
            group += [group[-1]] * (GATHER_SLOTS - len(group))
            groups.append([x for tr in group for x in tr])
        return groups

    def _gather(self, h, stream, groups=None) -> None:
        for args in (self._gather_groups() if groups is None else groups):
            rc = h.expert_cache_gather(*args, _ptr(self.miss), _ptr(self.n_miss),
                                       self.chunks, self.lanes, stream)
            if rc != 0:
                raise RuntimeError(f"expert_cache_gather failed rc={rc}")
