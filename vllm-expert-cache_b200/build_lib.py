"""Build libexpertcache.so for B200 (sm_100a) and check its exports.

    python vllm-expert-cache_b200/build_lib.py [--verbose]

Output: vllm-expert-cache_b200/vllm_expert_cache/libexpertcache.so -- beside the Python
package, which is where vllm_expert_cache/_lib.py looks after EXPERT_CACHE_LIB.  This
replaces the reference's hipcc build (kernels/build.sh:26-38), keeping its export check.
"""

from __future__ import annotations

import os
import re
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
SRC = HERE / "csrc" / "expert_cache.cu"
HEADER = ROOT / "include" / "expert_cache.h"
OUT = HERE / "vllm_expert_cache" / "libexpertcache.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo",
         "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared"]


def exported_symbols(path: Path = HEADER) -> list[str]:
    """Every function the public header declares."""
    text = path.read_text()
    return re.findall(r"^EXPERT_CACHE_API\s+int\s+(expert_cache_\w+)\s*\(", text, flags=re.M)


def build(force: bool = False, verbose: bool = False) -> Path:
    deps = [SRC, HEADER]
    if (OUT.exists() and not force
            and OUT.stat().st_mtime >= max(p.stat().st_mtime for p in deps)):
        return OUT
    cmd = [NVCC, *FLAGS, "-I", str(ROOT / "include"), str(SRC), "-o", str(OUT)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    check_exports(OUT)
    return OUT


def check_exports(path: Path = OUT) -> None:
    out = subprocess.run(["nm", "-D", "--defined-only", str(path)], check=True,
                         capture_output=True, text=True).stdout
    have = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in exported_symbols() if s not in have]
    if missing:
        raise RuntimeError(f"{path}: missing exports {missing}")


if __name__ == "__main__":
    print(build(force=True, verbose="--verbose" in sys.argv))
