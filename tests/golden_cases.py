"""Shared access to tests/golden/golden.npz (written by tests/golden/make_golden.py)."""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from synthetic import sticky_zipf_trace

# The twelve published miss counts: README.md:179-184 of the reference, (LRU, LFU).
PUBLISHED = {
    ("zipf", 16): (2392, 1980), ("zipf", 32): (1555, 1239), ("zipf", 64): (758, 674),
    ("interleaved", 16): (2289, 1899), ("interleaved", 32): (1347, 1096),
    ("interleaved", 64): (489, 363),
}


@dataclass
class Case:
    key: str
    E: int
    S: int
    md: int
    mi: int
    policy: int
    decay: int
    trace: np.ndarray
    hot: np.ndarray
    nmiss: np.ndarray
    pairs: np.ndarray
    chain: int
    final: dict


def cases(g, prefix: str = ""):
    for key in g["cases"].tolist():
        if key.startswith(prefix):
            yield load(g, key)


def load(g, key: str) -> Case:
    f = lambda k: g[f"{key}/{k}"]  # noqa: E731
    if f"{key}/trace" in g.files:
        trace = f("trace").astype(np.int32)
    else:  # cfg1:seed<k>:p<policy> -- regenerated, checked by digest
        seed = int(key.split(":")[1][4:])
        trace = sticky_zipf_trace(seed, steps=4096)
    return Case(key, int(f("E")), int(f("S")), int(f("md")), int(f("mi")),
                int(f("policy")), int(f("decay")), trace, f("hot"), f("nmiss"),
                f("pairs"), int(f("chain")[0]),
                dict(table=f("final_table"), map_cold=f("final_cold"),
                     slot_expert=f("final_se"), slot_stamp=f("final_st"),
                     step=f("final_step")))
