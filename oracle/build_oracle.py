"""Build recipe for the CPU oracle (test infrastructure; see lssm_oracle.cpp).

Compiles oracle/lssm_oracle.cpp into oracle/_build/liblssm_oracle.so with g++,
OpenMP and a portable x86-64-v3 target (the .so travels to the GPU box, whose
host CPU may differ from the build container's).
"""

from __future__ import annotations

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_build" / "liblssm_oracle.so"


def build(force: bool = False) -> Path:
    src = HERE / "lssm_oracle.cpp"
    if OUT.exists() and not force and OUT.stat().st_mtime >= src.stat().st_mtime:
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    cmd = ["g++", "-O3", "-fopenmp", "-fPIC", "-shared", "-std=c++17", "-march=x86-64-v3",
           "-ffp-contract=off", "-o", str(OUT), str(src)]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(force=True))
