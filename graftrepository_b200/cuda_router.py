"""B200 route sidecars: the drop-in for GraftRepository's CUDA route banks.

This module mirrors the public surface of ``core/grm_cuda_router.py`` (names,
argument meaning, receipts and error behaviour) so that
``NativeGraftStore.configure_cuda_{mla,gqa}_route_bank(..., sidecar=...)``
(core/grm_native.py:1498-1531, :1590-1624) and the arena's ``route_*_cuda``
calls use the sm_100a library unchanged:

* ``CudaRouterUnavailable``           core/grm_cuda_router.py:18
* ``CudaRouteReceipt``                :22-32
* ``validate_/..._route_bank_signature`` :35-75, :293-332
* ``CudaGQARouteSidecar`` / ``Bank``  :87-282 (the bank is CSR-ragged here)
* ``CudaMLARouteSidecar`` / ``Bank``  :344-539
* ``PaddedGQARouteSidecar``           the arena's dense padded GQA bank plus its
  ``row_token_counts`` receipt (core/graft_arena.py:2980-3042) -> CSR

Every route goes through ``libgrm_b200.so``; there is no host fallback inside
this module.  Exactly as in the reference, a UINT64_MAX sentinel (fewer finite
scores than ``topk``) raises ``RuntimeError`` so the caller falls back to its
CPU route (core/grm_cuda_router.py:465-475).
"""

from __future__ import annotations

import ctypes
import hashlib
import time
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import _lib
from ._lib import (GRM_B200_BF16, GRM_B200_F16, GRM_B200_F32, MAX_TOPK, CudaRouterUnavailable,
                   GrmB200Error)

__all__ = [
    "CudaRouterUnavailable", "CudaRouteReceipt", "GrmB200Error",
    "validate_mla_route_bank", "mla_route_bank_signature",
    "validate_gqa_route_bank", "gqa_route_bank_signature", "dense_to_csr",
    "CudaMLARouteSidecar", "CudaMLARouteBank", "CudaGQARouteSidecar", "CudaGQARouteBank",
    "PaddedGQARouteSidecar", "DeviceQueries", "upload_queries",
]

UINT64_MAX = np.iinfo(np.uint64).max


@dataclass(frozen=True)
class CudaRouteReceipt:
    """Same fields as core/grm_cuda_router.py:22-32."""
    device_route_ms_total: float
    device_route_ms_per_query: float
    route_wall_ms: float
    route_wall_ms_first: float
    route_wall_ms_min: float
    route_wall_ms_runs: tuple[float, ...]
    device_route_ms_runs: tuple[float, ...]
    measured_queries: int
    route_repeats: int


def _receipt(route_walls, device_times, measured, repeats) -> CudaRouteReceipt:
    return CudaRouteReceipt(
        device_route_ms_total=device_times[-1],
        device_route_ms_per_query=device_times[-1] / measured,
        route_wall_ms=route_walls[-1],
        route_wall_ms_first=route_walls[0],
        route_wall_ms_min=float(min(route_walls)),
        route_wall_ms_runs=tuple(route_walls),
        device_route_ms_runs=tuple(device_times),
        measured_queries=measured,
        route_repeats=repeats,
    )


def _blake(arrays) -> str:
    digest = hashlib.blake2b(digest_size=16)
    for a in arrays:
        digest.update(str(a.shape).encode("ascii"))
        digest.update(a.dtype.str.encode("ascii"))
        digest.update(memoryview(np.ascontiguousarray(a).view(np.uint8)))
    return digest.hexdigest()


# ----------------------------------------------------------------- helpers

class DeviceQueries:
    """Owning device query buffer with the ``.handle`` / ``.shape`` contract of
    the reference's CudaDeviceQueryPtr (scripts/grm_mla_cuda_probe.py:790-811)."""

    def __init__(self, handle: ctypes.c_void_p, shape):
        self.handle = handle
        self.shape = tuple(int(x) for x in shape)

    def close(self) -> None:
        if self.handle:
            _lib.load().grm_b200_free_device_ptr(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def upload_queries(queries: np.ndarray) -> DeviceQueries:
    """Upload fp32 queries to a fresh device buffer (the reference's test-only
    ``upload_queries``, scripts/grm_mla_cuda_probe.py:628-641)."""
    q = np.ascontiguousarray(queries, dtype=np.float32)
    handle = ctypes.c_void_p()
    L = _lib.load()
    rc = L.grm_b200_upload(q.ctypes.data, q.nbytes, ctypes.byref(handle))
    _lib.check(rc, _lib.thread_error)
    return DeviceQueries(handle, q.shape)


def _device_ptr(device_queries) -> int:
    """Accept a reference-style ``.handle`` object or a CUDA torch tensor."""
    if hasattr(device_queries, "data_ptr"):
        return int(device_queries.data_ptr())
    h = device_queries.handle
    return int(h.value if isinstance(h, ctypes.c_void_p) else h)


_U64MAX = np.uint64(np.iinfo(np.uint64).max)


def _blob(values) -> bytes:
    """A '\\n'-joined filter or key blob (core/grm_native.py:1367-1381)."""
    if values is None:
        return b""
    if isinstance(values, (str, bytes)):
        values = (values,)
    vals = [v.decode() if isinstance(v, bytes) else str(v) for v in values
            if v is not None and str(v) != ""]
    return "\n".join(vals).encode("utf-8")


def _c_strings(values, n: int, *, join: bool = False):
    """A (char* [n]) array for per-row / per-query strings; None -> NULL."""
    if values is None:
        return None
    if len(values) != n:
        raise ValueError(f"expected {n} entries, got {len(values)}")
    arr = (ctypes.c_char_p * n)()
    for i, v in enumerate(values):
        if v is None:
            arr[i] = None
        elif join and not isinstance(v, (str, bytes)):
            arr[i] = _blob(v)
        else:
            arr[i] = v if isinstance(v, bytes) else str(v).encode("utf-8")
    return arr


def _set_policy(fn, handle, err, n, lexical_keys, kinds, scopes, durabilities, mutabilities,
                active) -> None:
    arrays = [_c_strings(lexical_keys, n, join=True)]
    arrays += [_c_strings(v, n) for v in (kinds, scopes, durabilities, mutabilities)]
    act = None
    if active is not None:
        act = np.ascontiguousarray(active, dtype=np.uint8).reshape(-1)
        if act.shape[0] != n:
            raise ValueError("active must have one entry per bank row")
    rc = fn(handle, *[None if a is None else ctypes.addressof(a) for a in arrays],
            None if act is None else act.ctypes.data)
    _lib.check(rc, err)


def _query_lexical(lexical_keys, count: int):
    """One key list per query; a single list (or blob) for a single query."""
    lex = lexical_keys
    if lex is not None and count == 1 and (isinstance(lex, str) or (
            len(lex) > 0 and all(isinstance(x, str) for x in lex))):
        lex = [lex]
    return _c_strings(lex, count, join=True)


def _fits(values: np.ndarray, dtype) -> bool:
    """True when every value survives a round trip through `dtype` bit-exactly
    (NaN payloads aside), so a narrower bank keeps the reference's values."""
    if values.size == 0:
        return True
    narrowed = values.astype(dtype).astype(np.float32)
    same = (narrowed == values) | (np.isnan(narrowed) & np.isnan(values))
    return bool(np.all(same))


def _bf16_bits(values: np.ndarray) -> np.ndarray:
    u = values.view(np.uint32)
    return ((u.astype(np.uint64) + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _fits_bf16(values: np.ndarray) -> bool:
    u = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
    finite = np.isfinite(values)
    return bool(np.all(((u & 0xFFFF) == 0) | ~finite))


# --------------------------------------------------------------------- MLA

def validate_mla_route_bank(rows, node_ids=None) -> tuple[np.ndarray, np.ndarray]:
    """core/grm_cuda_router.py:293-314: shape (nodes, dim), dense ids by default."""
    rows_np = np.ascontiguousarray(rows, dtype=np.float32)
    if rows_np.ndim != 2:
        raise ValueError("MLA CUDA route bank must have shape (nodes, dim)")
    if any(int(d) <= 0 for d in rows_np.shape):
        raise ValueError("MLA CUDA route bank dimensions must be nonzero")
    if node_ids is None:
        ids_np = np.arange(rows_np.shape[0], dtype=np.uint64)
    else:
        ids_np = np.ascontiguousarray(node_ids, dtype=np.uint64).reshape(-1)
    if ids_np.shape[0] != rows_np.shape[0]:
        raise ValueError("node_ids length must match MLA route-bank nodes")
    return rows_np, ids_np


def mla_route_bank_signature(rows, node_ids) -> str:
    """Deterministic content signature (core/grm_cuda_router.py:317-332)."""
    rows_np, ids_np = validate_mla_route_bank(rows, node_ids)
    return _blake([rows_np, ids_np])


class CudaMLARouteBank:
    """Device-resident MLA centroid bank (core/grm_cuda_router.py:408-539)."""

    def __init__(self, handle: ctypes.c_void_p, node_ids: np.ndarray, *, nodes: int, dim: int,
                 setup_wall_ms: float, signature: str | None = None, dtype: int = GRM_B200_F16):
        self._h = handle
        self.node_ids = np.ascontiguousarray(node_ids, dtype=np.uint64)
        self.nodes = int(nodes)
        self.dim = int(dim)
        self.setup_wall_ms = float(setup_wall_ms)
        self.signature = signature
        self.dtype = dtype
        self.last_scores: np.ndarray | None = None
        self._fn_route = _lib.load().grm_b200_mla_route

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def _err(self) -> str:
        msg = _lib.load().grm_b200_mla_last_error(self._h)
        return msg.decode() if msg else ""

    def close(self) -> None:
        if self._h:
            _lib.load().grm_b200_mla_bank_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _route_raw(self, fn, qarg, count: int, topk: int, warmup: int):
        out = np.empty((count, topk), dtype=np.uint64)
        scores = np.empty((count, topk), dtype=np.float32)
        elapsed = ctypes.c_float(0.0)
        t0 = time.perf_counter_ns()
        rc = fn(self._h, qarg, count, self.dim, warmup, topk, out.ctypes.data,
                scores.ctypes.data, ctypes.byref(elapsed))
        wall = (time.perf_counter_ns() - t0) / 1.0e6
        _lib.check(rc, self._err)
        return out, scores, float(elapsed.value), wall

    def _finish(self, rows, scores, walls, devs, count, warmup, repeats):
        if rows.size and int(rows.max()) >= self.node_ids.shape[0]:
            raise RuntimeError("CUDA MLA route returned an out-of-range row ID")
        self.last_scores = scores
        mapped = self.node_ids[rows]
        measured = max(1, int(count) - int(warmup))
        return mapped, _receipt(walls, devs, measured, repeats)

    def route_topk(self, queries, *, topk: int, warmup: int = 0, route_repeats: int = 1):
        """core/grm_cuda_router.py:433-489: returns (node ids [Q, topk],
        receipt); the exact scores of the last call are in ``last_scores``."""
        if self._h is None:
            raise RuntimeError("CUDA MLA route bank is closed")
        q = np.ascontiguousarray(queries, dtype=np.float32)
        if q.ndim == 1:
            q = q[None, ...]
        if q.ndim != 2:
            raise ValueError("MLA CUDA queries must have shape (queries, dim) or (dim,)")
        if q.shape[1] != self.dim:
            raise ValueError("query dim does not match rows")
        if int(topk) <= 0:
            raise ValueError("topk must be positive")
        if int(topk) > MAX_TOPK:
            raise ValueError(f"topk must be <= {MAX_TOPK}")
        repeats = max(1, int(route_repeats))
        walls, devs = [], []
        rows = scores = None
        for _ in range(repeats):
            rows, scores, dev, wall = self._route_raw(
                self._fn_route, q.ctypes.data, q.shape[0], int(topk), int(warmup))
            walls.append(wall)
            devs.append(dev)
        return self._finish(rows, scores, walls, devs, q.shape[0], warmup, repeats)

    def route_topk_device(self, device_queries, *, topk: int, warmup: int = 0,
                          route_repeats: int = 1):
        """core/grm_cuda_router.py:491-539 (device-resident queries)."""
        if self._h is None:
            raise RuntimeError("CUDA MLA route bank is closed")
        if int(topk) <= 0:
            raise ValueError("topk must be positive")
        shape = tuple(device_queries.shape)
        count, dim = (1, shape[0]) if len(shape) == 1 else shape
        if dim != self.dim:
            raise ValueError("query dim does not match rows")
        repeats = max(1, int(route_repeats))
        walls, devs = [], []
        rows = scores = None
        for _ in range(repeats):
            rows, scores, dev, wall = self._route_raw(
                _lib.load().grm_b200_mla_route_device, _device_ptr(device_queries), count,
                int(topk), int(warmup))
            walls.append(wall)
            devs.append(dev)
        return self._finish(rows, scores, walls, devs, count, warmup, repeats)

    def route_topk_int4(self, queries, *, topk: int, refine_m: int = 4096,
                        route_repeats: int = 1):
        """The reference's INT4 bulk/refine mode (route_mla_int4,
        cpp/grm_runtime.cpp:4363-4482; GRM_ROUTER_INT4=1 with
        GRM_ROUTER_INT4_REFINE_M=refine_m): exact top-k among the refine_m
        best INT4 bulk scores.  Returns (node ids [Q, topk], receipt) with the
        same sentinel law as route_topk; exact scores in ``last_scores``."""
        if self._h is None:
            raise RuntimeError("CUDA MLA route bank is closed")
        q = np.ascontiguousarray(queries, dtype=np.float32)
        if q.ndim == 1:
            q = q[None, ...]
        if q.ndim != 2 or q.shape[1] != self.dim:
            raise ValueError("query dim does not match rows")
        if int(topk) <= 0 or int(topk) > MAX_TOPK:
            raise ValueError(f"topk must be in 1..{MAX_TOPK}")
        if int(refine_m) < 0:
            raise ValueError("refine_m must be >= 0")
        fn = _lib.load().grm_b200_mla_route_int4
        repeats = max(1, int(route_repeats))
        walls, devs = [], []
        rows = scores = None
        for _ in range(repeats):
            rows = np.empty((q.shape[0], int(topk)), dtype=np.uint64)
            scores = np.empty((q.shape[0], int(topk)), dtype=np.float32)
            elapsed = ctypes.c_float(0.0)
            t0 = time.perf_counter_ns()
            rc = fn(self._h, q.ctypes.data, q.shape[0], self.dim, int(topk), int(refine_m),
                    rows.ctypes.data, scores.ctypes.data, ctypes.byref(elapsed))
            walls.append((time.perf_counter_ns() - t0) / 1.0e6)
            _lib.check(rc, self._err)
            devs.append(float(elapsed.value))
        return self._finish(rows, scores, walls, devs, q.shape[0], 0, repeats)

    def route_int4_async(self, queries_ptr: int, count: int, topk: int, out_ids_ptr: int,
                         out_scores_ptr: int, stream: int = 0, id_offset: int = 0,
                         refine_m: int = 4096) -> None:
        """Stream-ordered INT4-mode route with device outputs (no host sync)."""
        rc = _lib.load().grm_b200_mla_route_int4_async(self._h, queries_ptr, count, topk,
                                                       int(refine_m), id_offset, out_ids_ptr,
                                                       out_scores_ptr, stream)
        _lib.check(rc, self._err)

    def route_async(self, queries_ptr: int, count: int, topk: int, out_ids_ptr: int,
                    out_scores_ptr: int, stream: int = 0, id_offset: int = 0) -> None:
        """Stream-ordered route with device outputs (no host sync)."""
        rc = _lib.load().grm_b200_mla_route_async(self._h, queries_ptr, count, topk, id_offset,
                                                  out_ids_ptr, out_scores_ptr, stream)
        _lib.check(rc, self._err)

    def reserve(self, max_queries: int) -> None:
        _lib.check(_lib.load().grm_b200_mla_reserve(self._h, int(max_queries)), self._err)

    def stats(self) -> tuple[int, int]:
        a, b = ctypes.c_uint64(0), ctypes.c_uint64(0)
        _lib.check(_lib.load().grm_b200_mla_stats(self._h, ctypes.byref(a), ctypes.byref(b)),
                   self._err)
        return int(a.value), int(b.value)

    def set_route_policy(self, *, lexical_keys=None, kinds=None, scopes=None,
                         durabilities=None, mutabilities=None, active=None) -> None:
        """Per-row route policy data (RouterIndex::Entry lexical_keys, kind,
        scope, durability, mutability, active; cpp/grm_runtime.hpp:483-494),
        one entry per bank row.  lexical_keys[i]: a sequence of keys or a
        '\n'-joined string; None values keep the reference's defaults."""
        _set_policy(_lib.load().grm_b200_mla_bank_set_policy, self._h, self._err, self.nodes,
                    lexical_keys, kinds, scopes, durabilities, mutabilities, active)

    def route_policy_topk(self, queries, *, topk: int, lexical_keys=None, kinds=(), scopes=(),
                          durabilities=(), mutabilities=()):
        """route_mla_arena with its lexical bonus and filters
        (cpp/grm_runtime.cpp:4299-4361) on the device: (node ids [Q, topk],
        policy scores [Q, topk]); lexical_keys: one key list per query (or
        one list for a single query)."""
        if self._h is None:
            raise RuntimeError("CUDA MLA route bank is closed")
        q = np.ascontiguousarray(queries, dtype=np.float32)
        if q.ndim == 1:
            q = q[None, ...]
        if q.ndim != 2 or q.shape[1] != self.dim:
            raise ValueError("query dim does not match rows")
        if not 0 < int(topk) <= MAX_TOPK:
            raise ValueError(f"topk must be in 1..{MAX_TOPK}")
        count = q.shape[0]
        lex_arr = _query_lexical(lexical_keys, count)
        out = np.empty((count, int(topk)), dtype=np.uint64)
        scores = np.empty((count, int(topk)), dtype=np.float32)
        elapsed = ctypes.c_float(0.0)
        rc = _lib.load().grm_b200_mla_route_policy(
            self._h, q.ctypes.data, count, self.dim, int(topk),
            None if lex_arr is None else ctypes.addressof(lex_arr), _blob(kinds), _blob(scopes),
            _blob(durabilities), _blob(mutabilities), out.ctypes.data, scores.ctypes.data,
            ctypes.byref(elapsed))
        _lib.check(rc, self._err)
        self.last_scores = scores
        self._last_elapsed_ms = float(elapsed.value)
        if np.any((out != _U64MAX) & (out >= self.node_ids.shape[0])):
            raise RuntimeError("CUDA MLA route returned an out-of-range row ID")
        mapped = np.where(out == _U64MAX, _U64MAX, self.node_ids[np.minimum(out, self.nodes - 1)])
        return mapped, scores

    def route(self, query, lexical_keys=(), topk=3, kinds=(), scopes=(), durabilities=(),
              mutabilities=()) -> list[int]:
        """NativeGraftStore.route's signature (core/grm_native.py:1446-1469):
        the ranked node ids of one query, lexical bonus and filters applied."""
        ids, _ = self.route_policy_topk(np.asarray(query, dtype=np.float32).reshape(1, -1),
                                        topk=int(topk), lexical_keys=[list(lexical_keys or ())],
                                        kinds=kinds, scopes=scopes, durabilities=durabilities,
                                        mutabilities=mutabilities)
        return [int(x) for x in ids[0] if x != _U64MAX]

    def paths(self) -> dict:
        """Which kernels serve this bank: bulk single-query scan, tensor-core
        batch route, or the exact kernel only."""
        f = ctypes.c_int(0)
        _lib.check(_lib.load().grm_b200_mla_paths(self._h, ctypes.byref(f)), self._err)
        return {"bulk": bool(f.value & 1), "batch": bool(f.value & 2),
                "exact_only": bool(f.value & 4)}


class CudaMLARouteSidecar:
    """core/grm_cuda_router.py:344-405.  ``build`` loads (building in-tree if
    needed) the sm_100a library instead of compiling a probe per attach."""

    def __init__(self, lib_path: Path | None = None, *, device: int = 0):
        self._lib = _lib.load()
        self.lib_path = Path(lib_path) if lib_path else _lib.LIB_PATH
        self.device = int(device)

    @classmethod
    def build(cls, build_dir: Path | None = None, *, nvcc: str = "nvcc",
              device: int = 0) -> "CudaMLARouteSidecar":
        del build_dir, nvcc  # the library is prebuilt in-tree (graftrepository_b200/build.py)
        return cls(device=device)

    def create_bank(self, rows, node_ids=None, *, signature=None,
                    dtype: str = "auto") -> CudaMLARouteBank:
        rows_np, ids_np = validate_mla_route_bank(rows, node_ids)
        if signature is None:
            signature = mla_route_bank_signature(rows_np, ids_np)
        use_f16 = dtype == "f16" or (dtype == "auto" and _fits(rows_np, np.float16))
        payload = rows_np.astype(np.float16) if use_f16 else rows_np
        code = GRM_B200_F16 if use_f16 else GRM_B200_F32
        return self.create_bank_raw(payload, code, ids_np, signature=signature)

    def create_bank_raw(self, rows: np.ndarray, dtype_code: int, node_ids=None, *,
                        signature=None) -> CudaMLARouteBank:
        """Attach an already-typed bank (fp16 or fp32 ndarray) without checks."""
        arr = np.ascontiguousarray(rows)
        nodes, dim = arr.shape
        ids = np.arange(nodes, dtype=np.uint64) if node_ids is None else node_ids
        handle = ctypes.c_void_p()
        t0 = time.perf_counter_ns()
        rc = self._lib.grm_b200_mla_bank_create(arr.ctypes.data, dtype_code, nodes, dim,
                                                self.device, ctypes.byref(handle))
        setup = (time.perf_counter_ns() - t0) / 1.0e6
        _lib.check(rc, _lib.thread_error)
        return CudaMLARouteBank(handle, ids, nodes=nodes, dim=dim, setup_wall_ms=setup,
                                signature=signature, dtype=dtype_code)

    def create_bank_multi(self, rows, entry_row_offsets, node_ids=None, *,
                          signature=None) -> CudaMLARouteBank:
        """A bank of multi-row entries: entry e owns rows
        entry_row_offsets[e] .. entry_row_offsets[e+1]-1 (a digest's own
        centroid and its child_cents) and scores the max of its rows."""
        r32 = np.ascontiguousarray(rows, dtype=np.float32)
        if r32.ndim != 2:
            raise ValueError("rows must have shape (rows, dim)")
        off = np.ascontiguousarray(entry_row_offsets, dtype=np.uint64).reshape(-1)
        entries = off.shape[0] - 1
        ids = np.arange(entries, dtype=np.uint64) if node_ids is None else \
            np.ascontiguousarray(node_ids, dtype=np.uint64).reshape(-1)
        if ids.shape[0] != entries:
            raise ValueError("node_ids length must match the entries")
        if _fits(r32, np.float16):
            arr, code = r32.astype(np.float16), GRM_B200_F16
        else:
            arr, code = r32, GRM_B200_F32
        handle = ctypes.c_void_p()
        t0 = time.perf_counter_ns()
        rc = self._lib.grm_b200_mla_bank_create_multi(arr.ctypes.data, code, arr.shape[0],
                                                      arr.shape[1], off.ctypes.data, entries,
                                                      self.device, ctypes.byref(handle))
        setup = (time.perf_counter_ns() - t0) / 1.0e6
        _lib.check(rc, _lib.thread_error)
        return CudaMLARouteBank(handle, ids, nodes=entries, dim=arr.shape[1],
                                setup_wall_ms=setup, signature=signature, dtype=code)

    def create_bank_device(self, rows_ptr: int, dtype_code: int, nodes: int, dim: int,
                           node_ids=None, *, signature=None) -> CudaMLARouteBank:
        handle = ctypes.c_void_p()
        t0 = time.perf_counter_ns()
        rc = self._lib.grm_b200_mla_bank_create_device(rows_ptr, dtype_code, nodes, dim,
                                                       ctypes.byref(handle))
        setup = (time.perf_counter_ns() - t0) / 1.0e6
        _lib.check(rc, _lib.thread_error)
        ids = np.arange(nodes, dtype=np.uint64) if node_ids is None else node_ids
        return CudaMLARouteBank(handle, ids, nodes=nodes, dim=dim, setup_wall_ms=setup,
                                signature=signature, dtype=dtype_code)

    def close(self) -> None:
        pass


# --------------------------------------------------------------------- GQA

def validate_gqa_route_bank(keys, node_ids=None) -> tuple[np.ndarray, np.ndarray]:
    """core/grm_cuda_router.py:35-57: dense (nodes, kv_heads, key_tokens, head_dim)."""
    keys_np = np.ascontiguousarray(keys, dtype=np.float32)
    if keys_np.ndim != 4:
        raise ValueError("GQA CUDA route bank must have shape "
                         "(nodes, kv_heads, key_tokens, head_dim)")
    if any(int(d) <= 0 for d in keys_np.shape):
        raise ValueError("GQA CUDA route bank dimensions must be nonzero")
    if node_ids is None:
        ids_np = np.arange(keys_np.shape[0], dtype=np.uint64)
    else:
        ids_np = np.ascontiguousarray(node_ids, dtype=np.uint64).reshape(-1)
    if ids_np.shape[0] != keys_np.shape[0]:
        raise ValueError("node_ids length must match GQA route-bank nodes")
    return keys_np, ids_np


def gqa_route_bank_signature(keys, node_ids) -> str:
    """core/grm_cuda_router.py:60-75."""
    keys_np, ids_np = validate_gqa_route_bank(keys, node_ids)
    return _blake([keys_np, ids_np])


def dense_to_csr(keys: np.ndarray, token_counts=None) -> tuple[np.ndarray, np.ndarray]:
    """Strip the zero padding of a dense (nodes, kv_heads, Tmax, head_dim) bank
    (core/graft_arena.py:2980-3042) back to CSR values + token offsets.
    Without ``token_counts`` every node keeps Tmax tokens, which routes
    identically (zero keys score |q.0| = 0 and best starts at 0)."""
    n, kh, tmax, d = keys.shape
    counts = np.full(n, tmax, dtype=np.int64) if token_counts is None else \
        np.asarray(token_counts, dtype=np.int64).reshape(-1)
    if counts.shape[0] != n or np.any(counts < 0) or np.any(counts > tmax):
        raise ValueError("token_counts must have one entry per node within [0, Tmax]")
    off = np.zeros(n + 1, dtype=np.uint64)
    off[1:] = np.cumsum(counts)
    vals = np.empty(int(off[-1]) * kh * d, dtype=keys.dtype)
    for i in range(n):
        t = int(counts[i])
        a = int(off[i]) * kh * d
        vals[a: a + kh * t * d] = keys[i, :, :t, :].reshape(-1)
    return vals, off


class CudaGQARouteBank:
    """Device-resident ragged GQA key bank (core/grm_cuda_router.py:159-282)."""

    def __init__(self, handle: ctypes.c_void_p, node_ids: np.ndarray, *, kv_heads: int,
                 head_dim: int, setup_wall_ms: float, signature=None, keepalive=None):
        self._h = handle
        self.node_ids = np.ascontiguousarray(node_ids, dtype=np.uint64)
        self.kv_heads = int(kv_heads)
        self.head_dim = int(head_dim)
        self.setup_wall_ms = float(setup_wall_ms)
        self.signature = signature
        self.last_scores: np.ndarray | None = None
        self._keepalive = keepalive

    def _err(self) -> str:
        msg = _lib.load().grm_b200_gqa_last_error(self._h)
        return msg.decode() if msg else ""

    def close(self) -> None:
        if self._h:
            _lib.load().grm_b200_gqa_bank_destroy(self._h)
            self._h = None
        self._keepalive = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _run(self, fn, qarg, count, heads, qtok, topk, warmup):
        out = np.empty((count, topk), dtype=np.uint64)
        scores = np.empty((count, topk), dtype=np.float32)
        elapsed = ctypes.c_float(0.0)
        t0 = time.perf_counter_ns()
        rc = fn(self._h, qarg, count, heads, qtok, warmup, topk, out.ctypes.data,
                scores.ctypes.data, ctypes.byref(elapsed))
        wall = (time.perf_counter_ns() - t0) / 1.0e6
        _lib.check(rc, self._err)
        return out, scores, float(elapsed.value), wall

    def _finish(self, rows, scores, walls, devs, count, warmup, repeats):
        if rows.size and int(rows.max()) >= self.node_ids.shape[0]:
            raise RuntimeError("CUDA GQA route returned an out-of-range row ID")
        self.last_scores = scores
        return self.node_ids[rows], _receipt(walls, devs, max(1, int(count) - int(warmup)),
                                             repeats)

    def route_topk(self, queries, *, topk: int, warmup: int = 0, route_repeats: int = 1):
        """core/grm_cuda_router.py:183-231: queries (Q, H, qt, D) or (H, qt, D)."""
        if self._h is None:
            raise RuntimeError("CUDA GQA route bank is closed")
        q = np.ascontiguousarray(queries, dtype=np.float32)
        if q.ndim == 3:
            q = q[None, ...]
        if q.ndim != 4:
            raise ValueError("GQA CUDA queries must have shape "
                             "(queries, heads, tokens, dim) or (heads, tokens, dim)")
        if int(topk) <= 0:
            raise ValueError("topk must be positive")
        if int(topk) > MAX_TOPK:
            raise ValueError(f"topk must be <= {MAX_TOPK}")
        if q.shape[3] != self.head_dim:
            raise ValueError("query head_dim does not match the bank")
        repeats = max(1, int(route_repeats))
        walls, devs = [], []
        rows = scores = None
        for _ in range(repeats):
            rows, scores, dev, wall = self._run(
                _lib.load().grm_b200_gqa_route, q.ctypes.data, q.shape[0], q.shape[1],
                q.shape[2], int(topk), int(warmup))
            walls.append(wall)
            devs.append(dev)
        return self._finish(rows, scores, walls, devs, q.shape[0], warmup, repeats)

    def set_route_policy(self, *, lexical_keys=None, kinds=None, scopes=None,
                         durabilities=None, mutabilities=None, active=None) -> None:
        """Per-node route policy data, as CudaMLARouteBank.set_route_policy."""
        _set_policy(_lib.load().grm_b200_gqa_bank_set_policy, self._h, self._err,
                    int(self.node_ids.shape[0]), lexical_keys, kinds, scopes, durabilities,
                    mutabilities, active)

    def route_policy_topk(self, queries, *, topk: int, lexical_keys=None, kinds=(), scopes=(),
                          durabilities=(), mutabilities=()):
        """route_gqa_raw with its lexical bonus and filters
        (cpp/grm_runtime.cpp:4498-4867) on the device: (node ids [Q, topk],
        scores [Q, topk]: S with lexical keys, raw without)."""
        if self._h is None:
            raise RuntimeError("CUDA GQA route bank is closed")
        q = np.ascontiguousarray(queries, dtype=np.float32)
        if q.ndim == 3:
            q = q[None, ...]
        if q.ndim != 4 or q.shape[3] != self.head_dim:
            raise ValueError("GQA queries must have shape (queries, heads, tokens, head_dim)")
        if not 0 < int(topk) <= MAX_TOPK:
            raise ValueError(f"topk must be in 1..{MAX_TOPK}")
        count = q.shape[0]
        lex_arr = _query_lexical(lexical_keys, count)
        out = np.empty((count, int(topk)), dtype=np.uint64)
        scores = np.empty((count, int(topk)), dtype=np.float32)
        elapsed = ctypes.c_float(0.0)
        rc = _lib.load().grm_b200_gqa_route_policy(
            self._h, q.ctypes.data, count, q.shape[1], q.shape[2], int(topk),
            None if lex_arr is None else ctypes.addressof(lex_arr), _blob(kinds), _blob(scopes),
            _blob(durabilities), _blob(mutabilities), out.ctypes.data, scores.ctypes.data,
            ctypes.byref(elapsed))
        _lib.check(rc, self._err)
        self.last_scores = scores
        n = self.node_ids.shape[0]
        if np.any((out != _U64MAX) & (out >= n)):
            raise RuntimeError("CUDA GQA route returned an out-of-range row ID")
        mapped = np.where(out == _U64MAX, _U64MAX, self.node_ids[np.minimum(out, n - 1)])
        return mapped, scores

    def route_gqa(self, query, lexical_keys=(), topk=3, kinds=(), scopes=(), durabilities=(),
                  mutabilities=()) -> list[int]:
        """NativeGraftStore.route_gqa's signature (core/grm_native.py:1471-1496)."""
        q = np.asarray(query, dtype=np.float32)
        if q.ndim != 3:
            raise ValueError("GQA query must have shape (heads, tokens, dim)")
        ids, _ = self.route_policy_topk(q[None], topk=int(topk),
                                        lexical_keys=[list(lexical_keys or ())], kinds=kinds,
                                        scopes=scopes, durabilities=durabilities,
                                        mutabilities=mutabilities)
        return [int(x) for x in ids[0] if x != _U64MAX]

    def route_topk_device(self, device_queries, *, topk: int, warmup: int = 0,
                          route_repeats: int = 1):
        """core/grm_cuda_router.py:233-282."""
        if self._h is None:
            raise RuntimeError("CUDA GQA route bank is closed")
        if int(topk) <= 0:
            raise ValueError("topk must be positive")
        count, heads, qtok, _ = tuple(device_queries.shape)
        repeats = max(1, int(route_repeats))
        walls, devs = [], []
        rows = scores = None
        for _ in range(repeats):
            rows, scores, dev, wall = self._run(
                _lib.load().grm_b200_gqa_route_device, _device_ptr(device_queries), count,
                heads, qtok, int(topk), int(warmup))
            walls.append(wall)
            devs.append(dev)
        return self._finish(rows, scores, walls, devs, count, warmup, repeats)

    def stats(self) -> tuple[int, int]:
        a, b = ctypes.c_uint64(0), ctypes.c_uint64(0)
        _lib.check(_lib.load().grm_b200_gqa_stats(self._h, ctypes.byref(a), ctypes.byref(b)),
                   self._err)
        return int(a.value), int(b.value)

    def paths(self) -> dict:
        """Which scan serves this bank: the tensor-core approximate pass, and
        whether its key tiles are TMA-staged."""
        f = ctypes.c_int(0)
        _lib.check(_lib.load().grm_b200_gqa_paths(self._h, ctypes.byref(f)), self._err)
        return {"fast": bool(f.value & 1), "tma": bool(f.value & 2)}


class CudaGQARouteSidecar:
    """core/grm_cuda_router.py:87-156."""

    def __init__(self, lib_path: Path | None = None, *, device: int = 0):
        self._lib = _lib.load()
        self.lib_path = Path(lib_path) if lib_path else _lib.LIB_PATH
        self.device = int(device)

    @classmethod
    def build(cls, build_dir: Path | None = None, *, nvcc: str = "nvcc",
              device: int = 0) -> "CudaGQARouteSidecar":
        del build_dir, nvcc
        return cls(device=device)

    def create_bank(self, keys, node_ids=None, *, signature=None, token_counts=None):
        """Dense padded bank as the arena passes it today
        (core/graft_arena.py:3140-3141); ``token_counts`` (the arena's
        ``row_token_counts`` receipt) strips the padding."""
        keys_np, ids_np = validate_gqa_route_bank(keys, node_ids)
        if signature is None:
            signature = gqa_route_bank_signature(keys_np, ids_np)
        vals, off = dense_to_csr(keys_np, token_counts)
        return self.create_bank_csr(vals, off, keys_np.shape[1], keys_np.shape[3], ids_np,
                                    signature=signature)

    def create_bank_csr(self, values, token_offsets, kv_heads: int, head_dim: int,
                        node_ids=None, *, signature=None, dtype: str = "auto"):
        """CSR bank: values = concatenated per-node [kv_heads, T_i, head_dim]
        blocks; fp32 values, or bf16 bit patterns as uint16 (dtype='bf16')."""
        off = np.ascontiguousarray(token_offsets, dtype=np.uint64)
        n = off.shape[0] - 1
        if n <= 0 or off[0] != 0 or np.any(off[1:] < off[:-1]):
            raise ValueError("token_offsets must start at 0 and be non-decreasing")
        vals = np.ascontiguousarray(values)
        if vals.size != int(off[-1]) * kv_heads * head_dim:
            raise ValueError("values size does not match token_offsets")
        if dtype == "bf16" or vals.dtype == np.uint16:
            payload, code = vals.astype(np.uint16, copy=False), GRM_B200_BF16
        else:
            f = np.ascontiguousarray(vals, dtype=np.float32)
            if dtype in ("auto", "bf16") and _fits_bf16(f):
                payload, code = (f.view(np.uint32) >> 16).astype(np.uint16), GRM_B200_BF16
            elif dtype in ("auto", "f16") and _fits(f, np.float16):
                payload, code = f.astype(np.float16), GRM_B200_F16
            else:
                payload, code = f, GRM_B200_F32
        ids = np.arange(n, dtype=np.uint64) if node_ids is None else \
            np.ascontiguousarray(node_ids, dtype=np.uint64).reshape(-1)
        if ids.shape[0] != n:
            raise ValueError("node_ids length must match GQA route-bank nodes")
        handle = ctypes.c_void_p()
        t0 = time.perf_counter_ns()
        rc = self._lib.grm_b200_gqa_bank_create(payload.ctypes.data, code, off.ctypes.data, n,
                                                kv_heads, head_dim, self.device,
                                                ctypes.byref(handle))
        setup = (time.perf_counter_ns() - t0) / 1.0e6
        _lib.check(rc, _lib.thread_error)
        return CudaGQARouteBank(handle, ids, kv_heads=kv_heads, head_dim=head_dim,
                                setup_wall_ms=setup, signature=signature)

    def create_bank_padded(self, keys, node_ids, row_token_counts, *, signature=None):
        """The arena's dense zero-padded bank plus its padding receipt
        (``row_token_counts``, core/graft_arena.py:3026-3041): stored as CSR."""
        return self.create_bank(keys, node_ids, signature=signature,
                                token_counts=row_token_counts)

    def create_bank_device(self, keys_ptr: int, dtype_code: int, token_offsets, kv_heads: int,
                           head_dim: int, node_ids=None, *, signature=None, keepalive=None):
        """Borrow keys already on the current device (no copy)."""
        off = np.ascontiguousarray(token_offsets, dtype=np.uint64)
        n = off.shape[0] - 1
        handle = ctypes.c_void_p()
        t0 = time.perf_counter_ns()
        rc = self._lib.grm_b200_gqa_bank_create_device(keys_ptr, dtype_code, off.ctypes.data, n,
                                                       kv_heads, head_dim, ctypes.byref(handle))
        setup = (time.perf_counter_ns() - t0) / 1.0e6
        _lib.check(rc, _lib.thread_error)
        ids = np.arange(n, dtype=np.uint64) if node_ids is None else node_ids
        return CudaGQARouteBank(handle, ids, kv_heads=kv_heads, head_dim=head_dim,
                                setup_wall_ms=setup, signature=signature, keepalive=keepalive)

    def close(self) -> None:
        pass


class PaddedGQARouteSidecar:
    """Sidecar for ``NativeGraftStore.configure_cuda_gqa_route_bank(...,
    sidecar=...)`` (core/grm_native.py:1498-1531) while the arena still passes
    its dense zero-padded bank (core/graft_arena.py:2980-3042): the store
    calls ``create_bank(route_bank, node_ids, signature=...)`` and this adapter
    hands the arena's ``row_token_counts`` padding receipt along, so the
    device bank is CSR (no padded bytes are stored or streamed).  Routing
    results equal the padded law's (a zero key scores |q.0| = 0, which never
    raises a node's maximum)."""

    def __init__(self, sidecar: CudaGQARouteSidecar, row_token_counts):
        self.sidecar = sidecar
        self.row_token_counts = np.ascontiguousarray(row_token_counts, dtype=np.int64).reshape(-1)

    @classmethod
    def build(cls, row_token_counts, build_dir: Path | None = None, *, nvcc: str = "nvcc",
              device: int = 0) -> "PaddedGQARouteSidecar":
        return cls(CudaGQARouteSidecar.build(build_dir, nvcc=nvcc, device=device),
                   row_token_counts)

    def create_bank(self, keys, node_ids=None, *, signature=None):
        return self.sidecar.create_bank_padded(keys, node_ids, self.row_token_counts,
                                               signature=signature)

    def close(self) -> None:
        self.sidecar.close()
