"""Packed graft payloads straight to the device (no host dequant).

The reference stores a graft node as ``pack_kv_arrays`` fields
(core/graft_quant.py:177-217): per tensor ``name`` the int8 codes
``{name}_codes`` (..., groups, 32), the fp32 scales ``{name}_scales``
(..., groups, 1) and the original shape ``{name}_shape``, plus
``format_version``, ``storage_bits`` and ``group_size``.  At mount it
dequantises on the host (``unpack_kv_arrays``, :233-279) and uploads fp16
(core/graft_arena.py:3479-3492).  Here the fields are checked exactly as
``unpack_kv_arrays`` checks them (fail-closed, same messages), the codes and
scales are uploaded as stored, and the fused mount kernel dequantises them
into the arena (optionally with the re-RoPE of the positional columns).

Node layouts: an MLA node is ``{"c": [L, S, 256], "kpe": [L, S, 32]}``
(core/graft_arena.py:464-477) and mounts as arena rows ``[c | kpe]``; a GQA
node is ``{"k": [L, H, S, D]}`` (:3459-3477) and mounts as L*H slices of S
rows of D values.  Tensors of one node share every axis but the last, whose
widths add up to the arena row.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib

__all__ = ["FORMAT_VERSION", "SUPPORTED_BITS", "GraftQuantFormatError", "PackedTensor",
           "read_packed", "upload_packed", "mount_payloads"]

FORMAT_VERSION = 1                      # core/graft_quant.py:70
SUPPORTED_BITS = (16, 8, 6, 4, 3, 2)    # :71
GROUP_SIZE = 32                         # :69


class GraftQuantFormatError(ValueError):
    """Unknown or unsupported packed format (core/graft_quant.py:75-77)."""


@dataclass
class PackedTensor:
    codes: np.ndarray    # int8 (..., groups, group)
    scales: np.ndarray   # float32 (..., groups, 1)
    shape: tuple         # the original (pre-group) shape
    bits: int


def _validate_bits(bits: int) -> None:
    if bits not in SUPPORTED_BITS:
        raise GraftQuantFormatError(
            f"unsupported storage_bits {bits!r}; supported: {SUPPORTED_BITS}")


def _scalar_int_field(payload, name: str) -> int:
    arr = np.asarray(payload[name])
    if arr.shape == ():
        return int(arr)
    if arr.size == 1:
        return int(arr.reshape(-1)[0])
    raise GraftQuantFormatError(
        f"unpack_kv_arrays: field {name!r} must be scalar-like, got shape {arr.shape}")


def _keys(payload):
    return payload.files if hasattr(payload, "files") else payload.keys()


def read_packed(payload, names) -> dict[str, PackedTensor]:
    """The checks of unpack_kv_arrays (core/graft_quant.py:233-279), without
    the dequant: codes and scales as stored, plus the shape and bit depth."""
    if "format_version" not in _keys(payload):
        raise GraftQuantFormatError(
            "unpack_kv_arrays: payload has no format_version field "
            "(not a packed graft payload, or a corrupt/foreign file)")
    version = _scalar_int_field(payload, "format_version")
    if version != FORMAT_VERSION:
        raise GraftQuantFormatError(
            f"unpack_kv_arrays: unknown format_version {version} "
            f"(this build only understands {FORMAT_VERSION})")
    bits = _scalar_int_field(payload, "storage_bits")
    _validate_bits(bits)
    if bits == 16:
        raise GraftQuantFormatError(
            "unpack_kv_arrays: storage_bits=16 encoded in a packed payload "
            "is invalid (16 is never packed, see pack_kv_arrays)")
    out = {}
    for name in names:
        ck, sk, hk = f"{name}_codes", f"{name}_scales", f"{name}_shape"
        keys = _keys(payload)
        if ck not in keys or sk not in keys or hk not in keys:
            raise GraftQuantFormatError(f"unpack_kv_arrays: payload missing {ck}/{sk}/{hk}")
        codes = np.ascontiguousarray(payload[ck])
        scales = np.ascontiguousarray(payload[sk])
        shape = tuple(int(v) for v in np.asarray(payload[hk]))
        # the device mount reads the stored layout directly: check it
        if codes.dtype != np.int8 or scales.dtype != np.float32:
            raise GraftQuantFormatError(f"{name}: codes must be int8 and scales float32")
        if len(shape) < 1 or shape[-1] % GROUP_SIZE or codes.size != int(np.prod(shape)) or \
                codes.shape[-1] != GROUP_SIZE or scales.size * GROUP_SIZE != codes.size:
            raise GraftQuantFormatError(f"{name}: codes/scales do not match shape {shape}")
        out[name] = PackedTensor(codes, scales, shape, bits)
    return out


def _node_layout(tensors: dict[str, PackedTensor], names):
    """(slices, tokens, width, per-name widths) of one node."""
    lead = None
    widths = []
    for n in names:
        shp = tensors[n].shape
        if len(shp) < 2:
            raise ValueError(f"{n}: need at least (tokens, width), got {shp}")
        if lead is None:
            lead = shp[:-1]
        elif shp[:-1] != lead:
            raise ValueError(f"tensors of one node must share all axes but the last: {names}")
        widths.append(shp[-1])
    tokens = lead[-1]
    slices = int(np.prod(lead[:-1])) if len(lead) > 1 else 1
    return slices, tokens, int(sum(widths)), widths


def upload_packed(nodes, names, *, device=None, stream=None):
    """Upload the codes and scales of `nodes` (each a read_packed result, or
    a raw payload) to the device, interleaving the named tensors row by row
    into arena rows.  Returns (codes int8 [G, slices, tokens*width], scales
    fp32 [G, slices, tokens*width/32], slices, tokens, width)."""
    import torch

    nodes = [n if all(isinstance(v, PackedTensor) for v in n.values()) else read_packed(n, names)
             for n in nodes]
    slices, tokens, width, widths = _node_layout(nodes[0], names)
    for n in nodes[1:]:
        if _node_layout(n, names)[:3] != (slices, tokens, width):
            raise ValueError("every node of one mount must have the same layout")
    G = len(nodes)
    rows = slices * tokens
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    codes = torch.empty((G, slices, tokens * width), dtype=torch.int8, device=dev)
    scales = torch.empty((G, slices, tokens * width // GROUP_SIZE), dtype=torch.float32,
                         device=dev)
    st = torch.cuda.current_stream(dev) if stream is None else stream
    L = _lib.load()
    n = len(names)
    for g, node in enumerate(nodes):
        for arrs, dst, esz, per in ((
                [node[k].codes for k in names], codes[g], 1, 1),
                ([node[k].scales for k in names], scales[g], 4, GROUP_SIZE)):
            ptrs = (ctypes.c_void_p * n)(*[a.ctypes.data for a in arrs])
            rb = (ctypes.c_int64 * n)(*[w // per * esz for w in widths])
            rc = L.grm_b200_upload_rows(ptrs, rb, n, rows, dst.data_ptr(),
                                        width // per * esz, st.cuda_stream)
            _lib.check(rc, _lib.thread_error)
    st.synchronize()  # the host arrays may go away after this call
    return codes, scales, slices, tokens, width


def mount_payloads(arena, payloads, seats, names, *, rope=None, stream=None) -> None:
    """Mount packed node payloads into an ArenaMount (arena [slices, seats,
    width]): upload codes and scales as stored, then one fused dequant (+
    re-RoPE) kernel.  Payloads of one call share their layout."""
    codes, scales, slices, tokens, width = upload_packed(payloads, names, stream=stream)
    if slices != arena.layers or width != arena.width:
        raise ValueError(f"payload layout ({slices} slices x {width}) does not match the arena "
                         f"({arena.layers} x {arena.width})")
    arena.mount_ref(codes, scales, seats, tokens, rope=rope, stream=stream)
