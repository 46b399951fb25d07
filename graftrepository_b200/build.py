"""Build recipe for libgrm_b200.so (sm_100a only).

The library is compiled in-tree so the built .so travels with the checkout:
``python -m graftrepository_b200.build`` or ``__graft_entry__.build()``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB = PKG / "libgrm_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-std=c++17", "-O3", "-lineinfo", "--shared", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    mtime = LIB.stat().st_mtime
    deps = sources() + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > mtime for p in deps)


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found: the sm_100a library cannot be built")
    return exe


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE}",
           *[str(s) for s in sources()], "-o", str(tmp)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    env = dict(os.environ)
    # the host compiler must be a plain gcc (some images point CC at wrappers)
    subprocess.run(cmd, check=True, env=env)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
