"""Compile the C restatement of the policy step.  TEST INFRASTRUCTURE ONLY.

    python oracle/build.py      ->  oracle/_build/liboracle.so

The reference's own kernels are HIP for AMD (kernels/expert_cache.hip) and cannot be
built with the tools in this image (no hipcc, no ROCm), so there is no ``oracle/_ref``
build; the reference is pinned through its Python model instead (tests/golden/).
"""

from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_build" / "liboracle.so"


def build(force: bool = False) -> Path:
    src = HERE / "policy.c"
    if OUT.exists() and not force and OUT.stat().st_mtime >= src.stat().st_mtime:
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    cmd = ["gcc", "-O2", "-std=c11", "-Wall", "-Wextra", "-fPIC", "-shared",
           str(src), "-o", str(OUT)]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
