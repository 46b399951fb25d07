"""ctypes bindings for the CPU parity oracle (TEST INFRASTRUCTURE ONLY).

See the package docstring: only tests, smoke() and bench.py's CPU-baseline legs
may use this module.  It wraps ``liboracle.so`` (the C restatement in
``grm_oracle.c``) and, when it was built here, the reference's own runtime in
``_ref/libgrm_ref*.so``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def reference_root() -> Path:
    """The GraftRepository checkout: $GRM_REFERENCE_ROOT, else the single
    default written in oracle/reference_root (also read by oracle/Makefile
    and the build hook)."""
    env = os.environ.get("GRM_REFERENCE_ROOT")
    if env:
        return Path(env)
    return Path((HERE / "reference_root").read_text().strip())


LIB_PATH = HERE / "liboracle.so"
REF_LIB_PATH = HERE / "_ref" / "libgrm_ref.so"
REF_OMP_LIB_PATH = HERE / "_ref" / "libgrm_ref_omp.so"

__all__ = [
    "ensure_built", "lib", "ref_available", "RefStore", "reference_root",
    "f32_to_f16_bits", "f16_bits_to_f32", "f32_to_bf16_bits", "bf16_bits_to_f32",
    "mla_row_norms", "mla_scores", "mla_route", "topk",
    "gqa_scores", "gqa_route",
    "quant_ref", "dequant_ref", "quant_packed", "dequant_packed", "packed_group_bytes",
    "mount_scatter", "mount_rope", "swap_splice",
    "ROUTE_DEFAULTS", "split_keys", "route_allowed", "lexical_hits", "mla_route_policy",
    "gqa_route_policy", "mla_route_multi", "mla_int4_arena", "mla_int4_scores", "mla_int4_route",
]

_P = ctypes.c_void_p
_I64 = ctypes.c_int64


def ensure_built(ref_root: str | os.PathLike | None = None, with_ref: bool = False) -> None:
    """Compile liboracle.so (and, if asked and the sources exist, the
    reference runtime) with oracle/Makefile."""
    targets = ["oracle"]
    if with_ref:
        root = Path(ref_root) if ref_root else reference_root()
        if (root / "cpp" / "grm_runtime.cpp").is_file():
            targets.append("ref")
    src = HERE / "grm_oracle.c"
    stale = LIB_PATH.exists() and src.exists() and src.stat().st_mtime > LIB_PATH.stat().st_mtime
    need = (not LIB_PATH.exists()) or stale or (
        "ref" in targets and not (REF_LIB_PATH.exists() and REF_OMP_LIB_PATH.exists()))
    if not need:
        return
    cmd = ["make", "-s", "-C", str(HERE), *targets]
    if with_ref:
        cmd.append(f"REF_ROOT={root}")
    subprocess.run(cmd, check=True)


_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        ensure_built()
        L = ctypes.CDLL(str(LIB_PATH))
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f32_to_f16.argtypes = [ctypes.c_float]
        L.orc_f32_to_bf16.restype = ctypes.c_uint16
        L.orc_f32_to_bf16.argtypes = [ctypes.c_float]
        L.orc_mla_row_norms.argtypes = [_P, _I64, _I64, _P]
        L.orc_mla_row_norms.restype = None
        L.orc_mla_query_norm.argtypes = [_P, _I64]
        L.orc_mla_query_norm.restype = ctypes.c_double
        L.orc_mla_scores.argtypes = [_P, _P, _I64, _I64, _P, _P]
        L.orc_mla_scores.restype = None
        L.orc_mla_int4_arena.argtypes = [_P, _P, _I64, _I64, _P, _P]
        L.orc_mla_int4_arena.restype = None
        L.orc_mla_int4_scores.argtypes = [_P, _P, _I64, _I64, _P, _P]
        L.orc_mla_int4_scores.restype = None
        L.orc_mla_int4_route.argtypes = [_P, _P, _I64, _I64, _P, _I64, _I64, _P, _P]
        L.orc_mla_int4_route.restype = _I64
        L.orc_topk.argtypes = [_P, _P, _I64, _I64, _P, _P]
        L.orc_topk.restype = _I64
        L.orc_gqa_scores.argtypes = [_P, _P, _I64, _I64, _I64, _P, _I64, _I64, _P]
        L.orc_gqa_scores.restype = None
        L.orc_quant_ref.argtypes = [_P, _I64, ctypes.c_int, ctypes.c_int, _P, _P]
        L.orc_quant_ref.restype = None
        L.orc_dequant_ref.argtypes = [_P, _P, _I64, ctypes.c_int, _P, _P]
        L.orc_dequant_ref.restype = None
        L.orc_packed_group_bytes.argtypes = [ctypes.c_int, ctypes.c_int]
        L.orc_packed_group_bytes.restype = _I64
        L.orc_quant_packed.argtypes = [_P, _I64, ctypes.c_int, ctypes.c_int, _P, _P]
        L.orc_quant_packed.restype = ctypes.c_int
        L.orc_dequant_packed.argtypes = [_P, _P, _I64, ctypes.c_int, ctypes.c_int, _P]
        L.orc_dequant_packed.restype = ctypes.c_int
        L.orc_mount_scatter.argtypes = [_P, _I64, _I64, _I64, _I64, _P, _P, _I64]
        L.orc_mount_scatter.restype = ctypes.c_int
        L.orc_mount_rope.argtypes = [_P, _I64, _I64, _I64, _I64, _P, _I64, _P, _P, _I64, _I64,
                                     _I64, ctypes.c_int]
        L.orc_mount_rope.restype = ctypes.c_int
        L.orc_swap_splice.argtypes = [_P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _P,
                                      ctypes.POINTER(_I64)]
        L.orc_swap_splice.restype = ctypes.c_int
        _LIB = L
    return _LIB


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


# ------------------------------------------------------------------ floats

def f32_to_bf16_bits(x) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even (NaN -> quiet NaN)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u.astype(np.uint64) + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) & 0x8000).astype(np.uint16) | np.uint16(0x7FC0), r)


def bf16_bits_to_f32(b) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_f16_bits(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def f16_bits_to_f32(h) -> np.ndarray:
    return np.ascontiguousarray(h, dtype=np.uint16).view(np.float16).astype(np.float32)


# --------------------------------------------------------------------- MLA

def mla_row_norms(rows) -> np.ndarray:
    r = np.ascontiguousarray(rows, dtype=np.float32)
    out = np.empty(r.shape[0], dtype=np.float32)
    lib().orc_mla_row_norms(_ptr(r), r.shape[0], r.shape[1], _ptr(out))
    return out


def mla_scores(rows, query, norms=None) -> np.ndarray:
    r = np.ascontiguousarray(rows, dtype=np.float32)
    q = np.ascontiguousarray(query, dtype=np.float32).reshape(-1)
    if q.shape[0] != r.shape[1]:
        raise ValueError("query dim does not match rows")
    nrm = mla_row_norms(r) if norms is None else np.ascontiguousarray(norms, dtype=np.float32)
    out = np.empty(r.shape[0], dtype=np.float32)
    lib().orc_mla_scores(_ptr(r), _ptr(nrm), r.shape[0], r.shape[1], _ptr(q), _ptr(out))
    return out


def topk(scores, k: int, ids=None) -> tuple[np.ndarray, np.ndarray, int]:
    s = np.ascontiguousarray(scores, dtype=np.float32)
    idp = None
    if ids is not None:
        idp = np.ascontiguousarray(ids, dtype=np.uint64)
    out_ids = np.empty(k, dtype=np.uint64)
    out_s = np.empty(k, dtype=np.float32)
    got = lib().orc_topk(_ptr(s), None if idp is None else _ptr(idp), s.shape[0], k,
                         _ptr(out_ids), _ptr(out_s))
    return out_ids, out_s, int(got)


def mla_route(rows, query, k: int, norms=None) -> tuple[np.ndarray, np.ndarray]:
    """Exact reference MLA route: (ids uint64[k] with UINT64_MAX fill, scores)."""
    ids, s, _ = topk(mla_scores(rows, query, norms), k)
    return ids, s


def mla_int4_arena(rows, norms=None) -> tuple[np.ndarray, np.ndarray]:
    """The reference's INT4 route arena (cpp/grm_runtime.cpp:3241-3266):
    (int8 values [n, dim] in [-7, 7], fp32 norm scales [n])."""
    r = np.ascontiguousarray(rows, dtype=np.float32)
    nrm = mla_row_norms(r) if norms is None else np.ascontiguousarray(norms, dtype=np.float32)
    vals = np.empty(r.shape, dtype=np.int8)
    ns = np.empty(r.shape[0], dtype=np.float32)
    lib().orc_mla_int4_arena(_ptr(r), _ptr(nrm), r.shape[0], r.shape[1], _ptr(vals), _ptr(ns))
    return vals, ns


def mla_int4_scores(rows, query, norms=None) -> np.ndarray:
    """Bulk INT4 scores of every row (int4_mla_row_score, default build)."""
    vals, ns = mla_int4_arena(rows, norms)
    q = np.ascontiguousarray(query, dtype=np.float32).reshape(-1)
    out = np.empty(vals.shape[0], dtype=np.float32)
    lib().orc_mla_int4_scores(_ptr(vals), _ptr(ns), vals.shape[0], vals.shape[1], _ptr(q),
                              _ptr(out))
    return out


def mla_int4_route(rows, query, k: int, refine_m: int = 4096, norms=None):
    """route_mla_int4 (cpp/grm_runtime.cpp:4363-4482): exact top-k among the
    refine_m best INT4 bulk scores.  (ids uint64[k], exact scores)."""
    r = np.ascontiguousarray(rows, dtype=np.float32)
    nrm = mla_row_norms(r) if norms is None else np.ascontiguousarray(norms, dtype=np.float32)
    q = np.ascontiguousarray(query, dtype=np.float32).reshape(-1)
    ids = np.empty(k, dtype=np.uint64)
    sc = np.empty(k, dtype=np.float32)
    lib().orc_mla_int4_route(_ptr(r), _ptr(nrm), r.shape[0], r.shape[1], _ptr(q), k,
                             int(refine_m), _ptr(ids), _ptr(sc))
    return ids, sc


def mla_route_multi(rows, entry_row_offsets, query, k: int, norms=None):
    """route_mla_arena over multi-row entries (exact_mla_entry_score,
    cpp/grm_runtime.cpp:3518-3545): an entry scores the max of its finite row
    scores, NaN (dropped) if none; (score desc, entry asc)."""
    s = mla_scores(rows, query, norms)
    off = np.asarray(entry_row_offsets, dtype=np.int64)
    n = off.shape[0] - 1
    best = np.full(n, np.nan, dtype=np.float32)
    for e in range(n):
        seg = s[off[e]:off[e + 1]]
        seg = seg[np.isfinite(seg)]
        if seg.size:
            best[e] = seg.max()
    ids, sc, _ = topk(best, k)
    return ids, sc


# ------------------------------------------------------------ route policy

# RouterIndex::Entry defaults (cpp/grm_runtime.hpp:488-492): kind, scope,
# durability, mutability of a node whose metadata was never set.
ROUTE_DEFAULTS = ("turn", "conversation", "session", "ephemeral")


def split_keys(blob) -> list[str]:
    """split_lexical_keys (cpp/grm_runtime.cpp:5196-5208): '\n'-separated,
    empty items dropped.  A list/tuple is taken as already split (empties
    dropped the same way)."""
    if blob is None:
        return []
    if isinstance(blob, (list, tuple)):
        return [str(x) for x in blob if str(x) != ""]
    return [x for x in str(blob).split("\n") if x != ""]


def route_allowed(n: int, cats=None, active=None, filters=None) -> np.ndarray:
    """entry_allowed (cpp/grm_runtime.cpp:3056-3105): active and, for every
    category with a non-empty filter list, the node's value is in the list.
    cats: 4 sequences of per-node values (None entries / arrays: defaults)."""
    ok = np.ones(n, dtype=bool) if active is None else np.asarray(active, dtype=bool).copy()
    for k in range(4):
        f = split_keys(filters[k]) if filters is not None else []
        if not f:
            continue
        fs = set(f)
        col = cats[k] if cats is not None else None
        for i in range(n):
            v = col[i] if col is not None and col[i] else ROUTE_DEFAULTS[k]
            if v not in fs:
                ok[i] = False
    return ok


def lexical_hits(query_keys, node_keys) -> int:
    """lexical_hit_count (cpp/grm_runtime.cpp:3107-3150): query keys counted
    with multiplicity, each hit when the node carries it."""
    ks = set(split_keys(node_keys))
    return sum(1 for q in split_keys(query_keys) if q in ks)


def mla_route_policy(rows, query, k: int, *, node_lexical=None, cats=None, active=None,
                     query_lexical=None, filters=None, norms=None):
    """route_mla_arena with its lexical and filter channels
    (cpp/grm_runtime.cpp:4299-4361): S = exact score + float(hits)/float(m)
    in fp32 for allowed nodes; non-finite dropped; (S desc, id asc)."""
    r = np.ascontiguousarray(rows, dtype=np.float32)
    n = r.shape[0]
    s = mla_scores(r, query, norms)
    qk = split_keys(query_lexical)
    m = len(qk)
    if m:
        hits = np.array([lexical_hits(qk, node_lexical[i] if node_lexical is not None else None)
                         for i in range(n)], dtype=np.float32)
        s = (s + hits / np.float32(m)).astype(np.float32)
    else:
        s = (s + np.float32(0.0)).astype(np.float32)
    s[~route_allowed(n, cats, active, filters)] = np.nan
    ids, sc, _ = topk(s, k)
    return ids, sc


# --------------------------------------------------------------------- GQA

def gqa_scores(keys_bf16, token_offsets, kv_heads: int, head_dim: int, query) -> np.ndarray:
    k = np.ascontiguousarray(keys_bf16, dtype=np.uint16).reshape(-1)
    off = np.ascontiguousarray(token_offsets, dtype=np.uint64)
    q = np.ascontiguousarray(query, dtype=np.float32)
    if q.ndim == 2:
        q = q[:, None, :]
    qh, qt, qd = q.shape
    if qd != head_dim or qh % kv_heads:
        raise ValueError("query shape does not match the bank")
    n = off.shape[0] - 1
    out = np.empty(n, dtype=np.float32)
    lib().orc_gqa_scores(_ptr(k), _ptr(off), n, kv_heads, head_dim, _ptr(q), qh, qt, _ptr(out))
    return out


def gqa_route(keys_bf16, token_offsets, kv_heads, head_dim, query, k: int):
    ids, s, _ = topk(gqa_scores(keys_bf16, token_offsets, kv_heads, head_dim, query), k)
    return ids, s


def gqa_route_policy(keys_bf16, token_offsets, kv_heads: int, head_dim: int, query, k: int, *,
                     node_lexical=None, cats=None, active=None, query_lexical=None,
                     filters=None):
    """route_gqa_raw with its lexical and filter channels
    (cpp/grm_runtime.cpp:4498-4867).  Without lexical keys: raw order over
    the allowed nodes.  With them: norm = max |raw| + 1e-8 (fp32) over the
    allowed nodes with a finite raw, S = raw / norm + float(hits)/float(m)."""
    raw = gqa_scores(keys_bf16, token_offsets, kv_heads, head_dim, query)
    n = raw.shape[0]
    have = route_allowed(n, cats, active, filters) & np.isfinite(raw)
    qk = split_keys(query_lexical)
    m = len(qk)
    if m == 0:
        s = raw.copy()
    else:
        max_abs = np.float32(np.max(np.abs(raw[have]), initial=np.float32(0.0)))
        norm = np.float32(max_abs + np.float32(1.0e-8))
        hits = np.array([lexical_hits(qk, node_lexical[i] if node_lexical is not None else None)
                         for i in range(n)], dtype=np.float32)
        with np.errstate(invalid="ignore"):
            s = ((raw / norm).astype(np.float32) + hits / np.float32(m)).astype(np.float32)
    s[~have] = np.nan
    ids, sc, _ = topk(s, k)
    return ids, sc


# ------------------------------------------------------------------- quant

def quant_ref(x, bits: int, group: int = 32) -> tuple[np.ndarray, np.ndarray]:
    """graft_quant.quantize_symmetric_group32 over the flat value stream."""
    xf = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    if xf.size % group:
        raise ValueError("value count not divisible by group")
    ng = xf.size // group
    codes = np.empty(xf.size, dtype=np.int8)
    scales = np.empty(ng, dtype=np.float32)
    lib().orc_quant_ref(_ptr(xf), ng, group, bits, _ptr(codes), _ptr(scales))
    return codes, scales


def dequant_ref(codes, scales, group: int = 32) -> tuple[np.ndarray, np.ndarray]:
    """-> (fp16 bits, bf16 bits) of fp32(code)*scale (fp16 first, then bf16)."""
    c = np.ascontiguousarray(codes, dtype=np.int8).reshape(-1)
    s = np.ascontiguousarray(scales, dtype=np.float32).reshape(-1)
    if c.size != s.size * group:
        raise ValueError("codes/scales size mismatch")
    f16 = np.empty(c.size, dtype=np.uint16)
    bf = np.empty(c.size, dtype=np.uint16)
    lib().orc_dequant_ref(_ptr(c), _ptr(s), s.size, group, _ptr(f16), _ptr(bf))
    return f16, bf


def packed_group_bytes(bits: int, group: int = 64) -> int:
    return group * bits // 8


def quant_packed(x, bits: int, group: int = 64) -> tuple[np.ndarray, np.ndarray]:
    xf = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    if xf.size % group:
        raise ValueError("value count not divisible by group")
    ng = xf.size // group
    codes = np.empty(ng * packed_group_bytes(bits, group), dtype=np.uint8)
    scales = np.empty(ng, dtype=np.uint16)
    rc = lib().orc_quant_packed(_ptr(xf), ng, group, bits, _ptr(codes), _ptr(scales))
    if rc != 0:
        raise ValueError("unsupported packed format")
    return codes, scales


def dequant_packed(codes, scales_f16, bits: int, group: int = 64) -> np.ndarray:
    c = np.ascontiguousarray(codes, dtype=np.uint8).reshape(-1)
    s = np.ascontiguousarray(scales_f16, dtype=np.uint16).reshape(-1)
    out = np.empty(s.size * group, dtype=np.uint16)
    rc = lib().orc_dequant_packed(_ptr(c), _ptr(s), s.size, group, bits, _ptr(out))
    if rc != 0:
        raise ValueError("unsupported packed format")
    return out


def mount_scatter(values_bf16, seats, arena_bf16) -> np.ndarray:
    """values [G, L, T, W] bf16 bits; arena [L, S, W] bf16 bits (modified copy)."""
    v = np.ascontiguousarray(values_bf16, dtype=np.uint16)
    a = np.array(arena_bf16, dtype=np.uint16, copy=True, order="C")
    st = np.ascontiguousarray(seats, dtype=np.int64)
    G, L, T, W = v.shape
    rc = lib().orc_mount_scatter(_ptr(v), G, L, T, W, _ptr(st), _ptr(a), a.shape[1])
    if rc != 0:
        raise ValueError("seat out of range")
    return a


def mount_rope(arena_bf16, grafts: int, layers: int, tokens: int, seats, cos, sin, offset: int,
               dim: int, pair_swap: bool = False) -> np.ndarray:
    """Re-RoPE of the mounted rows' rope heads at their seats (orc_mount_rope).
    arena [L, S, W] bf16 bits (modified copy); cos/sin [rows, dim] fp32."""
    a = np.array(arena_bf16, dtype=np.uint16, copy=True, order="C")
    L, S, W = a.shape
    st = np.ascontiguousarray(seats, dtype=np.int64)
    c = np.ascontiguousarray(cos, dtype=np.float32)
    sn = np.ascontiguousarray(sin, dtype=np.float32)
    rc = lib().orc_mount_rope(_ptr(a), grafts, layers, tokens, W, _ptr(st), S, _ptr(c), _ptr(sn),
                              c.shape[0], offset, dim, 1 if pair_swap else 0)
    if rc != 0:
        raise ValueError("bad rope arguments")
    return a


def swap_splice(old, mount, sink_tokens: int, old_mount_tokens: int) -> np.ndarray:
    """old [outer, T_in, inner] / mount [outer, n, inner] (any dtype) ->
    sink | mount | live tail, as DeviceArena::apply_swap_tensor."""
    o = np.ascontiguousarray(old)
    m = np.ascontiguousarray(mount, dtype=o.dtype)
    outer, tin, inner = o.shape
    n = m.shape[1]
    row = inner * o.itemsize
    tail_start = min(sink_tokens + old_mount_tokens, tin)
    out_t = sink_tokens + n + (tin - tail_start)
    out = np.empty((outer, out_t, inner), dtype=o.dtype)
    got = _I64(0)
    rc = lib().orc_swap_splice(_ptr(o), outer, tin, _ptr(m), n, row, sink_tokens,
                               old_mount_tokens, _ptr(out), ctypes.byref(got))
    if rc != 0:
        raise ValueError("input cache shorter than arena sink")
    return out


# ------------------------------------------- the reference's own runtime

def ref_available(omp: bool = False) -> bool:
    return (REF_OMP_LIB_PATH if omp else REF_LIB_PATH).exists()


def _c_array(vals, n: int):
    """(char* [n]) of per-node strings; lists are '\n'-joined; None -> NULL."""
    if vals is None:
        return None
    a = (ctypes.c_char_p * n)()
    for i, v in enumerate(vals):
        if isinstance(v, (list, tuple)):
            v = "\n".join(v)
        a[i] = None if v is None else str(v).encode()
    return a


class RefStore:
    """A reference ``grm_store_handle`` loaded with one route bank, driven
    through the reference's C ABI (``cpp/grm_runtime_c.h``)."""

    _libs: dict = {}

    def __init__(self, omp: bool = False):
        path = REF_OMP_LIB_PATH if omp else REF_LIB_PATH
        if not path.exists():
            raise FileNotFoundError(f"reference runtime not built: {path}")
        L = RefStore._libs.get(str(path))
        if L is None:
            L = ctypes.CDLL(str(path))
            L.refd_mla_create.restype = _P
            L.refd_mla_create.argtypes = [_P, ctypes.c_uint64, ctypes.c_uint64]
            L.refd_mla_route.restype = ctypes.c_int
            L.refd_mla_route.argtypes = [_P, _P, ctypes.c_uint64, ctypes.c_uint64, _P, _P]
            L.refd_mla_create_policy.restype = _P
            L.refd_mla_create_policy.argtypes = [_P, ctypes.c_uint64, ctypes.c_uint64] + [_P] * 6
            L.refd_mla_route_policy.restype = ctypes.c_int
            L.refd_mla_route_policy.argtypes = [_P, _P, ctypes.c_uint64] + [ctypes.c_char_p] * 5 + [
                ctypes.c_uint64, _P, _P]
            L.refd_mla_create_multi.restype = _P
            L.refd_mla_create_multi.argtypes = [_P, ctypes.c_uint64, ctypes.c_uint64, _P,
                                                ctypes.c_uint64]
            L.refd_gqa_create_policy.restype = _P
            L.refd_gqa_create_policy.argtypes = [_P, _P, ctypes.c_uint64, ctypes.c_uint64,
                                                 ctypes.c_uint64] + [_P] * 6
            L.refd_gqa_route_policy.restype = ctypes.c_int
            L.refd_gqa_route_policy.argtypes = [_P, _P] + [ctypes.c_uint64] * 3 + [
                ctypes.c_char_p] * 5 + [ctypes.c_uint64, _P, _P]
            L.refd_gqa_create.restype = _P
            L.refd_gqa_create.argtypes = [_P, _P, ctypes.c_uint64, ctypes.c_uint64,
                                          ctypes.c_uint64]
            L.refd_gqa_route.restype = ctypes.c_int
            L.refd_gqa_route.argtypes = [_P, _P, ctypes.c_uint64, ctypes.c_uint64,
                                         ctypes.c_uint64, ctypes.c_uint64, _P, _P]
            L.refd_swap.restype = ctypes.c_int
            L.refd_swap.argtypes = [ctypes.c_uint64] * 3 + [_P, ctypes.c_uint64,
                                    ctypes.c_uint64, _P] + [ctypes.c_uint64] * 3 + [
                                    _P, ctypes.c_uint64, _P, _P]
            L.refd_last_error.restype = ctypes.c_char_p
            L.refd_last_error.argtypes = [_P]
            L.refd_destroy.restype = None
            L.refd_destroy.argtypes = [_P]
            RefStore._libs[str(path)] = L
        self._L = L
        self._h = None
        self.kind = None

    def load_mla(self, rows) -> "RefStore":
        r = np.ascontiguousarray(rows, dtype=np.float32)
        self._keep = r
        h = self._L.refd_mla_create(_ptr(r), r.shape[0], r.shape[1])
        if not h:
            raise RuntimeError("reference MLA store load failed")
        self._h, self.kind, self.dim = h, "mla", r.shape[1]
        del self._keep
        return self

    def load_mla_policy(self, rows, node_lexical=None, cats=None, active=None) -> "RefStore":
        """MLA store with per-node lexical keys, route metadata and active flags."""
        r = np.ascontiguousarray(rows, dtype=np.float32)
        n = r.shape[0]
        lex = _c_array(node_lexical, n)
        cs = [_c_array(cats[k], n) if cats is not None else None for k in range(4)]
        act = None if active is None else np.ascontiguousarray(active, dtype=np.uint8)
        self._keep_c = (lex, cs, act)
        h = self._L.refd_mla_create_policy(_ptr(r), n, r.shape[1], lex, cs[0], cs[1], cs[2],
                                           cs[3], None if act is None else _ptr(act))
        if not h:
            raise RuntimeError("reference MLA store load failed")
        self._h, self.kind, self.dim = h, "mla", r.shape[1]
        return self

    def route_policy(self, query, k: int, lexical=None, filters=None) -> list[int]:
        """grm_store_route_filtered with '\n'-joined blobs."""
        def blob(v):
            if v is None:
                return b""
            if isinstance(v, (list, tuple)):
                v = "\n".join(str(x) for x in v)
            return str(v).encode()
        f = list(filters) if filters is not None else [None] * 4
        out = np.zeros(k, dtype=np.uint64)
        cnt = ctypes.c_uint64(0)
        q = np.ascontiguousarray(query, dtype=np.float32)
        if self.kind == "mla":
            rc = self._L.refd_mla_route_policy(self._h, _ptr(q), q.size, blob(lexical),
                                               blob(f[0]), blob(f[1]), blob(f[2]), blob(f[3]), k,
                                               _ptr(out), ctypes.addressof(cnt))
        else:
            if q.ndim == 2:
                q = np.ascontiguousarray(q[:, None, :])
            rc = self._L.refd_gqa_route_policy(self._h, _ptr(q), q.shape[0], q.shape[1],
                                               q.shape[2], blob(lexical), blob(f[0]), blob(f[1]),
                                               blob(f[2]), blob(f[3]), k, _ptr(out),
                                               ctypes.addressof(cnt))
        if rc != 0:
            raise RuntimeError(self._L.refd_last_error(self._h).decode())
        return [int(x) for x in out[: cnt.value]]

    def load_mla_multi(self, rows, entry_row_offsets) -> "RefStore":
        """MLA store whose node e carries rows off[e] .. off[e+1]-1 as its
        route keys (grm_store_set_route_list with key_count > 1)."""
        r = np.ascontiguousarray(rows, dtype=np.float32)
        off = np.ascontiguousarray(entry_row_offsets, dtype=np.uint64)
        h = self._L.refd_mla_create_multi(_ptr(r), r.shape[0], r.shape[1], _ptr(off),
                                          off.shape[0] - 1)
        if not h:
            raise RuntimeError("reference MLA store load failed")
        self._h, self.kind, self.dim = h, "mla", r.shape[1]
        return self

    def load_gqa_policy(self, keys_bf16, token_offsets, kv_heads: int, head_dim: int,
                        node_lexical=None, cats=None, active=None) -> "RefStore":
        """GQA store with per-node lexical keys, route metadata and active flags."""
        k = np.ascontiguousarray(keys_bf16, dtype=np.uint16).reshape(-1)
        off = np.ascontiguousarray(token_offsets, dtype=np.uint64)
        n = off.shape[0] - 1
        lex = _c_array(node_lexical, n)
        cs = [_c_array(cats[j], n) if cats is not None else None for j in range(4)]
        act = None if active is None else np.ascontiguousarray(active, dtype=np.uint8)
        self._keep_c = (lex, cs, act)
        h = self._L.refd_gqa_create_policy(_ptr(k), _ptr(off), n, kv_heads, head_dim, lex, cs[0],
                                           cs[1], cs[2], cs[3],
                                           None if act is None else _ptr(act))
        if not h:
            raise RuntimeError("reference GQA store load failed")
        self._h, self.kind, self.dim = h, "gqa", head_dim
        return self

    def load_gqa(self, keys_bf16, token_offsets, kv_heads: int, head_dim: int) -> "RefStore":
        k = np.ascontiguousarray(keys_bf16, dtype=np.uint16).reshape(-1)
        off = np.ascontiguousarray(token_offsets, dtype=np.uint64)
        h = self._L.refd_gqa_create(_ptr(k), _ptr(off), off.shape[0] - 1, kv_heads, head_dim)
        if not h:
            raise RuntimeError("reference GQA store load failed")
        self._h, self.kind, self.dim = h, "gqa", head_dim
        return self

    def route(self, query, k: int) -> list[int]:
        out = np.zeros(k, dtype=np.uint64)
        cnt = ctypes.c_uint64(0)
        q = np.ascontiguousarray(query, dtype=np.float32)
        if self.kind == "mla":
            rc = self._L.refd_mla_route(self._h, _ptr(q), q.size, k, _ptr(out),
                                        ctypes.addressof(cnt))
        else:
            if q.ndim == 2:
                q = np.ascontiguousarray(q[:, None, :])
            rc = self._L.refd_gqa_route(self._h, _ptr(q), q.shape[0], q.shape[1], q.shape[2],
                                        k, _ptr(out), ctypes.addressof(cnt))
        if rc != 0:
            raise RuntimeError(self._L.refd_last_error(self._h).decode())
        return [int(x) for x in out[: cnt.value]]

    def swap(self, old, mount, sink_tokens: int, width: int, old_mount_tokens: int):
        o = np.ascontiguousarray(old)
        m = np.ascontiguousarray(mount, dtype=o.dtype)
        outer, tin, inner = o.shape
        n = m.shape[1]
        cap = outer * (sink_tokens + n + tin) * inner * o.itemsize
        out = np.zeros(cap, dtype=np.uint8)
        got_len = ctypes.c_uint64(0)
        got_t = ctypes.c_uint64(0)
        rc = self._L.refd_swap(sink_tokens, width, old_mount_tokens, _ptr(o), outer, tin,
                               _ptr(m), n, inner, o.itemsize, _ptr(out), cap,
                               ctypes.addressof(got_len), ctypes.addressof(got_t))
        if rc != 0:
            raise RuntimeError("reference apply_swap_tensor failed")
        return out[: got_len.value].view(o.dtype).reshape(outer, int(got_t.value), inner)

    def close(self) -> None:
        if self._h:
            self._L.refd_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
