"""Chained digest of the cache state after every step.  TEST INFRASTRUCTURE ONLY.

``chain = blake2b(chain || table || map_cold || slot_expert || slot_stamp || step)``
(little-endian bytes, 8-byte digest) after each step, so one 8-byte value pins the full
state after every step of a trace; the golden fixtures store it per trace.
"""

from __future__ import annotations

import hashlib

import numpy as np

SEED = b"expert-cache-state-chain"


def start() -> bytes:
    return hashlib.blake2b(SEED, digest_size=8).digest()


def fold(chain: bytes, table, map_cold, slot_expert, slot_stamp, step) -> bytes:
    h = hashlib.blake2b(chain, digest_size=8)
    for a, dt in ((table, "<i4"), (map_cold, "<i4"), (slot_expert, "<i4"),
                  (slot_stamp, "<i8"), (step, "<i8")):
        h.update(np.ascontiguousarray(np.asarray(a).reshape(-1), dtype=dt).tobytes())
    return h.digest()


def as_u64(chain: bytes) -> int:
    return int.from_bytes(chain, "little")
