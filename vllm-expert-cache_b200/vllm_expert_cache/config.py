"""Runtime settings, read from the environment on every access.

Names, defaults and quirks are the reference's (vllm_expert_cache/config.py:8-47,
cache.py:96-97, _lib.py:18, README.md:103-116):

  EXPERT_CACHE_SLOTS      absolute slot count (unset: use FRACTION)
  EXPERT_CACHE_FRACTION   0.5     fraction of the experts kept resident
  EXPERT_CACHE_POLICY     lfu     'lfu' (frequency + decay) or 'lru'; anything else -> lru
  EXPERT_CACHE_DECAY      64      LFU halving period in steps, 0 = never
  EXPERT_CACHE_DISABLE    0       '1' turns the cache off
  EXPERT_CACHE_LIB        -       explicit path of libexpertcache.so
  EXPERT_CACHE_CHUNKS     16      gather CTA budget = CHUNKS * LANES
  EXPERT_CACHE_LANES      64
  EXPERT_CACHE_DEBUG      0       N > 0 logs the first N MoE calls of each armed layer
                                  (routing shape and cached / read-through path); new,
                                  off by default
  EXPERT_CACHE_STATS      0       '1' keeps a device-side running total of installs per
                                  layer (one extra tiny kernel per cached step; new in
                                  this build, off by default)
  EXPERT_CACHE_SPLIT_WIDE 0       N > 0 serves a step wider than the slots as up to N
                                  cached chunks of S // top_k tokens when the layer's
                                  activation quantisation is per token (new, off by
                                  default: 0 keeps the reference's read-through)
  EXPERT_CACHE_EP         0       '1' caches expert-parallel layers (standard activation
                                  format, vLLM expert_map) instead of refusing them as the
                                  reference does (new, off by default)
  EXPERT_CACHE_PREFETCH   0       N > 0 predicts each armed layer's routing from the
                                  previous layer's MoE input and installs the top N
                                  predicted experts per token on a side stream while that
                                  layer computes (new, off by default)
  EXPERT_CACHE_SINGLE_LAUNCH 1    '1': a cached step with S <= 256 is one
                                  expert_cache_step launch; '0': two launches (manage +
                                  remap, then gather), the form used above 256 slots (new)

``slots_for(E)`` clamps to [1, E]: EXPERT_CACHE_SLOTS=0 means one slot, not "off".
"""

from __future__ import annotations

import os

_POLICIES = {"lru": 0, "lfu": 1}


def _env(name: str, default: str | None = None) -> str | None:
    return os.environ.get(name, default)


class Settings:
    @property
    def disabled(self) -> bool:
        return _env("EXPERT_CACHE_DISABLE", "0") == "1"

    @property
    def slots(self) -> int | None:
        v = _env("EXPERT_CACHE_SLOTS")
        return int(v) if v else None

    @property
    def fraction(self) -> float:
        return float(_env("EXPERT_CACHE_FRACTION", "0.5"))

    @property
    def policy(self) -> str:
        return _env("EXPERT_CACHE_POLICY", "lfu").strip().lower()

    @property
    def policy_code(self) -> int:
        return _POLICIES.get(self.policy, 0)

    @property
    def decay(self) -> int:
        return int(_env("EXPERT_CACHE_DECAY", "64"))

    @property
    def chunks(self) -> int:
        return int(_env("EXPERT_CACHE_CHUNKS", "16"))

    @property
    def lanes(self) -> int:
        return int(_env("EXPERT_CACHE_LANES", "64"))

    @property
    def debug_calls(self) -> int:
        return int(_env("EXPERT_CACHE_DEBUG", "0") or 0)

    @property
    def stats(self) -> bool:
        return _env("EXPERT_CACHE_STATS", "0") == "1"

    @property
    def split_wide(self) -> int:
        return max(0, int(_env("EXPERT_CACHE_SPLIT_WIDE", "0") or 0))

    @property
    def ep(self) -> bool:
        return _env("EXPERT_CACHE_EP", "0") == "1"

    @property
    def prefetch(self) -> int:
        return max(0, int(_env("EXPERT_CACHE_PREFETCH", "0") or 0))

    @property
    def single_launch(self) -> bool:
        return _env("EXPERT_CACHE_SINGLE_LAUNCH", "1") != "0"

    def slots_for(self, num_experts: int) -> int:
        want = self.slots
        if want is None:
            want = round(num_experts * self.fraction)
        return max(1, min(int(want), int(num_experts)))


settings = Settings()
