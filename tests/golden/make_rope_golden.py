"""Generate tests/golden/rope_law.npz from the REFERENCE's own rotary functions.

Run in a container that has the GraftRepository checkout (the path in
oracle/reference_root, or GRM_REFERENCE_ROOT):

    python tests/golden/make_rope_golden.py

The reference's device rotation (tensor_cuda's ``F.apply_rotary``) is not part
of its tree, but the reference states the same law in Python twice:

* ``rope(t, cs, sn) = t * cs + concat(-t2, t1) * sn`` and the table builder
  ``rope_tables(D, theta, n_real)`` (full rotary and p-RoPE, fp64) in
  tests/gemma4_int4_sim.py:60-76;
* ``_deepseek_rope_prep``, the pair permutation applied before rotate-half
  for the MLA positional key part, in core/deepseek_v2_lite_tc.py:99-103.

Neither module can be imported here (one loads model weights at import, the
other needs tensor_cuda), so this script takes exactly those three function
definitions out of the reference sources with ``ast`` and executes them
unchanged: the two numpy functions on numpy arrays, the permutation (written
for tensor_cuda's torch-style tensors) on a torch tensor.  The expected
outputs are the reference functions' fp64 results on bf16 key values at mount
seats; the fixture keeps them as fp64 so the test can state its tolerance
against the exact value.
"""

from __future__ import annotations

import ast
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

import oracle as O  # noqa: E402

REF = O.reference_root()

# (name, width, offset, dim, heads, pair_swap, theta, n_real, seats, tokens, layers)
CASES = [
    ("mla_kpe", 288, 256, 32, 1, True, 1e4, 16, [5, 100, 170], 24, 2),
    ("gqa_k", 256, 0, 128, 2, False, 1e6, 64, [0, 64], 16, 2),
    ("p_rope", 192, 64, 64, 2, False, 1e6, 16, [17, 120], 16, 2),
]
S = 256   # table rows (positions 0 .. S-1)


def _functions(path: Path, names: set[str], env: dict) -> dict:
    tree = ast.parse(path.read_text(), filename=str(path))
    defs = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in names]
    missing = names - {d.name for d in defs}
    if missing:
        raise SystemExit(f"{path}: no top-level definition of {sorted(missing)}")
    ns = dict(env)
    exec(compile(ast.Module(body=defs, type_ignores=[]), str(path), "exec"), ns)
    return ns


def _bf16_bits(f32):
    u = np.ascontiguousarray(f32, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _to_f64(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def main() -> None:
    gem = _functions(REF / "tests" / "gemma4_int4_sim.py", {"rope", "rope_tables"},
                     {"np": np, "S": S})
    ds = _functions(REF / "core" / "deepseek_v2_lite_tc.py", {"_deepseek_rope_prep"}, {})
    out = {}
    for ci, (name, W, off, dim, heads, swap, theta, n_real, seats, T, L) in enumerate(CASES):
        rng = np.random.default_rng(700 + ci)
        arena = _bf16_bits(rng.standard_normal((L, S, W)).astype(np.float32) * 2.0)
        cs, sn = gem["rope_tables"](dim, theta, n_real)        # fp64 [S, dim]
        want = np.empty((len(seats), L, T, heads * dim), np.float64)
        for g, s in enumerate(seats):
            t = _to_f64(arena[:, s:s + T, off:off + heads * dim]).reshape(L, T, heads, dim)
            for layer in range(L):
                x = t[layer]                                    # [T, heads, dim]
                if swap:   # written for torch-style tensors: transpose(-1, -2) swaps two axes
                    x = ds["_deepseek_rope_prep"](torch.from_numpy(x)).numpy()
                want[g, layer] = gem["rope"](x, cs[s:s + T], sn[s:s + T]).reshape(T, heads * dim)
        p = f"{name}_"
        end = max(seats) + T   # the test rebuilds an arena of `end` rows around these windows
        out[p + "windows"] = np.stack([arena[:, s:s + T] for s in seats])   # [G, L, T, W] bf16
        out[p + "cos"] = cs[:end]
        out[p + "sin"] = sn[:end]
        out[p + "seats"] = np.asarray(seats, np.int64)
        out[p + "want"] = want
        out[p + "meta"] = np.array([W, off, dim, heads, int(swap), T, L], np.int64)
    # the plain full-rotary tables (n_real = dim / 2) for the table-construction check
    cs, sn = gem["rope_tables"](32, 1e4, 16)
    out["tables32_cos"], out["tables32_sin"] = cs[:64], sn[:64]
    np.savez_compressed(HERE / "rope_law.npz", **out)
    print("wrote", HERE / "rope_law.npz")


if __name__ == "__main__":
    main()
