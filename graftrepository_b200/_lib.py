"""ctypes binding of libgrm_b200.so (the sm_100a route/mount library).

There is no CPU fallback: if the library is missing or a call fails, this
module raises.  ``CudaRouterUnavailable`` mirrors the reference's exception of
the same name (core/grm_cuda_router.py:18) so callers that fall back to the CPU
route on it keep working unchanged.
"""

from __future__ import annotations

import ctypes
import os
import re
import threading
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("GRM_B200_LIB", PKG / "libgrm_b200.so"))
HEADER = PKG.parent / "include" / "grm_b200.h"

GRM_B200_F32 = 0
GRM_B200_F16 = 1
GRM_B200_BF16 = 2
MAX_TOPK = 32

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_U64 = ctypes.c_uint64
_SZ = ctypes.c_size_t


class CudaRouterUnavailable(RuntimeError):
    """Raised when the sm_100a route library cannot be loaded or built."""


class GrmB200Error(RuntimeError):
    """A libgrm_b200 call returned a non-zero status."""

    def __init__(self, rc: int, message: str):
        super().__init__(f"{message} (status {rc})")
        self.rc = rc


_SIGS = {
    "grm_b200_mla_bank_create": (_I, [_P, _I, _I64, _I, _I, _P]),
    "grm_b200_mla_bank_create_device": (_I, [_P, _I, _I64, _I, _P]),
    "grm_b200_mla_bank_create_multi": (_I, [_P, _I, _I64, _I, _P, _I64, _I, _P]),
    "grm_b200_mla_route": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P]),
    "grm_b200_mla_route_device": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P]),
    "grm_b200_mla_route_async": (_I, [_P, _P, _I, _I, _U64, _P, _P, _P]),
    "grm_b200_mla_scan_async": (_I, [_P, _P, _I, _I, _U64, _P, _P, _P]),
    "grm_b200_mla_resolve_async": (_I, [_P, _P, _I, _I, _U64, _P, _P, _P]),
    "grm_b200_mla_reserve": (_I, [_P, _I]),
    "grm_b200_mla_bank_destroy": (_I, [_P]),
    "grm_b200_mla_last_error": (ctypes.c_char_p, [_P]),
    "grm_b200_mla_row_norms_device": (_P, [_P]),
    "grm_b200_mla_stats": (_I, [_P, _P, _P]),
    "grm_b200_mla_paths": (_I, [_P, _P]),
    "grm_b200_mla_bank_set_policy": (_I, [_P, _P, _P, _P, _P, _P, _P]),
    "grm_b200_mla_route_policy": (_I, [_P, _P, _I, _I, _I, _P, ctypes.c_char_p,
                                       ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p,
                                       _P, _P, _P]),
    "grm_b200_gqa_paths": (_I, [_P, _P]),
    "grm_b200_gqa_bank_set_policy": (_I, [_P, _P, _P, _P, _P, _P, _P]),
    "grm_b200_gqa_route_policy": (_I, [_P, _P, _I, _I, _I, _I, _P, ctypes.c_char_p,
                                       ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p,
                                       _P, _P, _P]),
    "grm_b200_mla_route_noalloc": (_I, [_P, _I64, _I, _P, _I, _I, _P, _P, _P]),
    "grm_b200_mla_route_int4": (_I, [_P, _P, _I, _I, _I, _I64, _P, _P, _P]),
    "grm_b200_mla_route_int4_async": (_I, [_P, _P, _I, _I, _I64, _U64, _P, _P, _P]),
    "grm_b200_gqa_bank_create": (_I, [_P, _I, _P, _I64, _I, _I, _I, _P]),
    "grm_b200_gqa_bank_create_device": (_I, [_P, _I, _P, _I64, _I, _I, _P]),
    "grm_b200_gqa_route": (_I, [_P, _P, _I, _I, _I, _I, _I, _P, _P, _P]),
    "grm_b200_gqa_route_device": (_I, [_P, _P, _I, _I, _I, _I, _I, _P, _P, _P]),
    "grm_b200_gqa_route_async": (_I, [_P, _P, _I, _I, _I, _I, _U64, _P, _P, _P]),
    "grm_b200_gqa_bank_destroy": (_I, [_P]),
    "grm_b200_gqa_last_error": (ctypes.c_char_p, [_P]),
    "grm_b200_gqa_stats": (_I, [_P, _P, _P]),
    "grm_b200_mount_ref": (_I, [_P, _P, _I64, _I64, _I64, _I64, _P, _P, _I64, _P]),
    "grm_b200_mount_packed": (_I, [_P, _P, _I, _I, _I64, _I64, _I64, _I64, _P, _P, _I64, _P]),
    "grm_b200_upload_rows": (_I, [_P, _P, _I, _I64, _P, _I64, _P]),
    "grm_b200_mount_packed_rope": (_I, [_P, _P, _I, _I, _I64, _I64, _I64, _I64, _P, _P, _I64, _P,
                                        _P]),
    "grm_b200_mount_ref_rope": (_I, [_P, _P, _I64, _I64, _I64, _I64, _P, _P, _I64, _P, _P]),
    "grm_b200_arena_splice": (_I, [_P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _P, _P, _P]),
    "grm_b200_merge_topk": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P]),
    "grm_b200_merge_topk_strided": (_I, [_P, ctypes.c_int64, _P, ctypes.c_int64, _I, _I, _I, _I,
                                         _P, _P, _P]),
    "grm_b200_upload": (_I, [_P, _SZ, _P]),
    "grm_b200_free_device_ptr": (_I, [_P]),
    "grm_b200_last_error": (ctypes.c_char_p, []),
    "grm_b200_version": (ctypes.c_char_p, []),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def header_symbols() -> list[str]:
    """Every function declared in include/grm_b200.h."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(grm_b200_\w+)\s*\(", text)))


def load() -> ctypes.CDLL:
    """Load the library (building it in-tree first when nvcc is available and
    the .so is missing).  Raises CudaRouterUnavailable, never falls back."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            try:
                from .build import build
                build()
            except Exception as exc:  # pragma: no cover - depends on toolchain
                raise CudaRouterUnavailable(
                    f"libgrm_b200.so missing and could not be built: {exc}") from exc
        try:
            lib = ctypes.CDLL(str(LIB_PATH))
        except OSError as exc:
            raise CudaRouterUnavailable(f"cannot load {LIB_PATH}: {exc}") from exc
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def thread_error() -> str:
    msg = load().grm_b200_last_error()
    return msg.decode() if msg else ""


def check(rc: int, message_fn) -> None:
    if rc != 0:
        raise GrmB200Error(int(rc), message_fn())


def cuda_available() -> bool:
    try:
        import torch
        return bool(torch.cuda.is_available())
    except Exception:  # pragma: no cover
        return False
