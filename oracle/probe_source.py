"""Writes the CUDA source that one of the reference's probe scripts compiles.

TEST INFRASTRUCTURE ONLY (used by oracle/Makefile's ``ref_cuda`` target).

scripts/grm_mla_cuda_probe.py and scripts/grm_gqa_cuda_probe.py hold their
CUDA code as a module-level string ``CUDA_SOURCE`` that their ``build_probe``
writes to a file and compiles with nvcc (scripts/grm_mla_cuda_probe.py:551-569,
scripts/grm_gqa_cuda_probe.py:610-628).  This helper reads that string out of
the script with ``ast`` (without importing the module) and writes it where the
Makefile compiles it, under oracle/_ref/ (git-ignored, never committed).

    python oracle/probe_source.py <probe script> <output .cu>
"""

import ast
import sys
from pathlib import Path


def cuda_source(script: Path) -> str:
    tree = ast.parse(script.read_text(encoding="utf-8"), filename=str(script))
    for node in tree.body:
        if (isinstance(node, ast.Assign) and len(node.targets) == 1
                and isinstance(node.targets[0], ast.Name)
                and node.targets[0].id == "CUDA_SOURCE"
                and isinstance(node.value, ast.Constant) and isinstance(node.value.value, str)):
            return node.value.value
    raise SystemExit(f"{script}: no module-level CUDA_SOURCE string")


if __name__ == "__main__":
    src, out = Path(sys.argv[1]), Path(sys.argv[2])
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(cuda_source(src), encoding="utf-8")
