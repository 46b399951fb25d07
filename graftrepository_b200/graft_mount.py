"""Fused dequantise + scatter mount of routed grafts into the device arena.

Host-side mirror of the mount half of GraftRepository's per-turn step:
``ArenaCache.swap`` pages the picked grafts in through ``unpack_node``
(core/graft_arena.py:3479-3492: ``graft_quant.unpack_kv_arrays`` on the CPU,
then an fp16 -> bf16 upload per layer) and splices them into the arena seats
(:1933-1995).  Here the codes and scales are uploaded as they are stored and
one kernel dequantises and writes bf16 rows straight into the preallocated
arena ``[layers, seats, width]``; with a ``RopeSpec`` the same kernel also
re-RoPEs the positional columns at their arena seats (``_graft_block``,
core/graft_arena.py:1848-1859).

Two storage formats:

* ``"ref"`` -- core/graft_quant.py's format (``pack_kv_arrays``): int8 codes,
  groups of 32 on the value stream, fp32 scales; the mounted bytes equal
  ``bf16(dequantize_symmetric_group32(...))`` bit for bit.
* ``"packed"`` -- bit-packed 8/6/4-bit codes, groups of 64 on the flattened
  (token, value) stream of each (graft, layer), fp16 scales (the same
  quantisation law with the scale rounded to fp16 before the codes are taken).
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import _lib

__all__ = ["quantize_packed", "packed_group_bytes", "ArenaMount", "mount_ref", "mount_packed",
           "arena_splice", "RopeSpec", "rope_tables"]

GROUP_PACKED = 64


def packed_group_bytes(bits: int, group: int = GROUP_PACKED) -> int:
    return group * bits // 8


def _qmax(bits: int) -> int:
    return (1 << (bits - 1)) - 1


def quantize_packed(values: np.ndarray, bits: int, group: int = GROUP_PACKED):
    """Quantise fp32 values [..., n] (n % group == 0) to the packed format:
    returns (codes uint8 [..., n*bits/8], scales fp16 [..., n/group])."""
    if bits not in (8, 6, 4):
        raise ValueError("packed mount supports 8, 6 and 4 bits")
    x = np.ascontiguousarray(values, dtype=np.float32)
    lead, n = x.shape[:-1], x.shape[-1]
    if n % group:
        raise ValueError(f"value stream length {n} not divisible by group {group}")
    xg = x.reshape(-1, group)
    qmax = _qmax(bits)
    s16 = (np.abs(xg).max(axis=1) / np.float32(qmax)).astype(np.float16)
    s16 = np.where(s16 == 0, np.float16(1.0), s16)
    s16 = np.where(np.isinf(s16), np.float16(65504.0), s16)
    s = s16.astype(np.float32)[:, None]
    c = np.clip(np.round(xg / s), -qmax - 1, qmax).astype(np.int32)
    if bits == 8:
        packed = (c & 0xFF).astype(np.uint8)
    elif bits == 4:
        u = (c & 0xF).astype(np.uint8)
        packed = (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)
    else:
        u = (c & 0x3F).astype(np.uint32).reshape(xg.shape[0], group // 4, 4)
        w = u[..., 0] | (u[..., 1] << 6) | (u[..., 2] << 12) | (u[..., 3] << 18)
        packed = np.stack([w & 0xFF, (w >> 8) & 0xFF, (w >> 16) & 0xFF], axis=-1).astype(np.uint8)
    codes = packed.reshape(*lead, n * bits // 8)
    scales = s16.reshape(*lead, n // group)
    return codes, scales


class _RopeC(ctypes.Structure):
    _fields_ = [("cos_device", ctypes.c_void_p), ("sin_device", ctypes.c_void_p),
                ("rows", ctypes.c_int64), ("offset", ctypes.c_int64), ("dim", ctypes.c_int64),
                ("pair_swap", ctypes.c_int)]


class RopeSpec:
    """Re-RoPE of mounted rows: device fp32 ``cos``/``sin`` tables ``[rows, dim]``
    (``emb = cat([pos*inv, pos*inv])``, as the models build ``rope_cos``),
    the first positional column ``offset`` of a row (MLA: 256, after the latent;
    GQA: 0) and the rotary head width ``dim`` (MLA k_pe: 32; GQA: head_dim).
    ``pair_swap`` selects the ``ROPE_PAIR_SWAP`` layout (DeepSeek)."""

    def __init__(self, cos, sin, offset: int, dim: int, pair_swap: bool = False):
        self.cos, self.sin = cos, sin
        self.offset, self.dim, self.pair_swap = int(offset), int(dim), bool(pair_swap)

    def c(self) -> _RopeC:
        for t in (self.cos, self.sin):
            if hasattr(t, "shape") and (tuple(t.shape[1:]) != (self.dim,) or
                                        getattr(t, "dtype", None) is not None and
                                        "float32" not in str(t.dtype)):
                raise ValueError("rope tables must be fp32 [rows, dim]")
        if hasattr(self.cos, "shape") and self.cos.shape != self.sin.shape:
            raise ValueError("rope cos and sin tables differ in shape")
        return _RopeC(_ptr(self.cos), _ptr(self.sin), int(self.cos.shape[0]), self.offset,
                      self.dim, 1 if self.pair_swap else 0)


def rope_tables(rows: int, dim: int, theta: float = 10000.0, factors=None):
    """fp32 (cos, sin) [rows, dim] the way the reference models build them
    (core/minicpm3_tc.py:345-355): inv = 1/theta^(2i/dim) [/ factors],
    emb = cat([pos*inv, pos*inv])."""
    inv = 1.0 / (theta ** (np.arange(0, dim, 2, np.float32) / dim))
    if factors is not None:
        inv = inv / np.asarray(factors, np.float32)
    ang = np.arange(rows, dtype=np.float32)[:, None] * inv[None, :]
    emb = np.concatenate([ang, ang], axis=-1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def _ptr(t) -> int:
    if hasattr(t, "data_ptr"):
        return int(t.data_ptr())
    return int(t)


def _stream(stream) -> int:
    if stream is None:
        return 0
    if hasattr(stream, "cuda_stream"):
        return int(stream.cuda_stream)
    return int(stream)


def mount_ref(codes, scales, seats, arena, *, layers: int, tokens: int, width: int,
              rope: RopeSpec | None = None, stream=None) -> None:
    """codes int8 [G, layers, tokens*width], scales fp32 [G, layers, tokens*width/32]
    and arena bf16 [layers, seats, width] are device tensors (or pointers)."""
    st = np.ascontiguousarray(seats, dtype=np.int64)
    arena_seats = int(arena.shape[1]) if hasattr(arena, "shape") else None
    if arena_seats is None:
        raise ValueError("arena must be a tensor with a shape")
    L = _lib.load()
    if rope is None:
        rc = L.grm_b200_mount_ref(_ptr(codes), _ptr(scales), st.shape[0], layers, tokens, width,
                                  st.ctypes.data, _ptr(arena), arena_seats, _stream(stream))
    else:
        spec = rope.c()
        rc = L.grm_b200_mount_ref_rope(_ptr(codes), _ptr(scales), st.shape[0], layers, tokens,
                                       width, st.ctypes.data, _ptr(arena), arena_seats,
                                       ctypes.addressof(spec), _stream(stream))
    _lib.check(rc, _lib.thread_error)


def mount_packed(codes, scales, seats, arena, *, bits: int, layers: int, tokens: int, width: int,
                 group: int = GROUP_PACKED, rope: RopeSpec | None = None, stream=None) -> None:
    st = np.ascontiguousarray(seats, dtype=np.int64)
    L = _lib.load()
    if rope is None:
        rc = L.grm_b200_mount_packed(_ptr(codes), _ptr(scales), bits, group, st.shape[0], layers,
                                     tokens, width, st.ctypes.data, _ptr(arena),
                                     int(arena.shape[1]), _stream(stream))
    else:
        spec = rope.c()
        rc = L.grm_b200_mount_packed_rope(_ptr(codes), _ptr(scales), bits, group, st.shape[0],
                                          layers, tokens, width, st.ctypes.data, _ptr(arena),
                                          int(arena.shape[1]), ctypes.addressof(spec),
                                          _stream(stream))
    _lib.check(rc, _lib.thread_error)


def arena_splice(old, mount, out, *, outer: int, input_tokens: int, mount_tokens: int,
                 row_bytes: int, sink_tokens: int, old_mount_tokens: int, stream=None) -> int:
    """Device DeviceArena::apply_swap_tensor; returns the output token count."""
    got = ctypes.c_int64(0)
    rc = _lib.load().grm_b200_arena_splice(_ptr(old), outer, input_tokens,
                                           _ptr(mount) if mount is not None else 0, mount_tokens,
                                           row_bytes, sink_tokens, old_mount_tokens, _ptr(out),
                                           ctypes.byref(got), _stream(stream))
    _lib.check(rc, _lib.thread_error)
    return int(got.value)


class ArenaMount:
    """A preallocated bf16 arena ``[layers, seats, width]`` on one device."""

    def __init__(self, layers: int, seats: int, width: int, device: str = "cuda:0", fill=None):
        import torch

        self.layers, self.seats, self.width = int(layers), int(seats), int(width)
        self.arena = torch.empty((layers, seats, width), dtype=torch.bfloat16, device=device)
        if fill is not None:
            self.arena.view(torch.int16).fill_(int(np.uint16(fill).view(np.int16)))

    def mount_ref(self, codes, scales, seats, tokens: int, rope: RopeSpec | None = None,
                  stream=None) -> None:
        mount_ref(codes, scales, seats, self.arena, layers=self.layers, tokens=tokens,
                  width=self.width, rope=rope, stream=stream)

    def mount_packed(self, codes, scales, seats, tokens: int, bits: int,
                     rope: RopeSpec | None = None, stream=None) -> None:
        mount_packed(codes, scales, seats, self.arena, bits=bits, layers=self.layers,
                     tokens=tokens, width=self.width, rope=rope, stream=stream)
