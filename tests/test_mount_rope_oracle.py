"""The re-RoPE mount oracle (orc_mount_rope) against a numpy restatement of the
reference's rotation of the positional key part at the mount seats
(core/graft_arena.py:339-367 `_pair_swap_last` / `_rope_tensor` /
`_rope_block_at`, applied at seats n_sink.. by `_graft_block`, :1848-1859):
x' = pair_swap(x), out = bf16(x' * cos[pos] + rotate_half(x') * sin[pos]).
`apply_rotary` lives in the reference's compiled tensor library, which is not
part of the reference tree, so the restatement follows the standard
rotate-half form the Python fallback calls."""

import numpy as np
import pytest

import oracle as O
from graftrepository_b200 import graft_mount


def _bf16_bits(f32):
    u = np.ascontiguousarray(f32, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) & 0x8000 | 0x7FC0).astype(np.uint16), r)


def _to_f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def _pair_swap_last(x):
    d = x.shape[-1]
    return x.reshape(x.shape[:-1] + (d // 2, 2)).swapaxes(-1, -2).reshape(x.shape)


def _rotate_half(x):
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def numpy_mount_rope(arena, seats, tokens, cos, sin, offset, dim, pair_swap):
    a = arena.copy()
    L, S, W = a.shape
    heads = (W - offset) // dim
    for s in seats:
        pos = np.arange(s, s + tokens)
        blk = a[:, s:s + tokens, offset:offset + heads * dim].reshape(L, tokens, heads, dim)
        x = _to_f32(blk)
        if pair_swap:
            x = _pair_swap_last(x)
        c = cos[pos][None, :, None, :]
        sn = sin[pos][None, :, None, :]
        out = (x * c).astype(np.float32) + (_rotate_half(x) * sn).astype(np.float32)
        a[:, s:s + tokens, offset:offset + heads * dim] = _bf16_bits(out).reshape(
            L, tokens, heads * dim)
    return a


def _arena(seed, L, S, W):
    rng = np.random.default_rng(seed)
    return _bf16_bits(rng.standard_normal((L, S, W)).astype(np.float32) * 3.0)


@pytest.mark.parametrize("W,offset,dim", [(288, 256, 32), (256, 0, 128), (192, 64, 64),
                                          (288, 96, 96)])
@pytest.mark.parametrize("pair_swap", [False, True])
def test_oracle_rope_matches_numpy_restatement(W, offset, dim, pair_swap):
    L, S, T = 3, 300, 17
    arena = _arena(W + dim, L, S, W)
    seats = np.array([4, 40, 200], np.int64)
    cos, sin = graft_mount.rope_tables(S, dim)
    got = O.mount_rope(arena, 3, L, T, seats, cos, sin, offset, dim, pair_swap)
    want = numpy_mount_rope(arena, seats, T, cos, sin, offset, dim, pair_swap)
    assert np.array_equal(got, want)
    # rows outside the mount seats and the position-free columns keep their bytes
    touched = np.zeros(S, bool)
    for s in seats:
        touched[s:s + T] = True
    assert np.array_equal(got[:, ~touched], arena[:, ~touched])
    assert np.array_equal(got[:, :, :offset], arena[:, :, :offset])


def test_rope_tables_follow_the_model_construction():
    cos, sin = graft_mount.rope_tables(64, 32, theta=10000.0)
    assert cos.shape == (64, 32) and cos.dtype == np.float32
    assert np.array_equal(cos[:, :16], cos[:, 16:])
    assert np.array_equal(cos[0], np.ones(32, np.float32))
    assert np.array_equal(sin[0], np.zeros(32, np.float32))
    inv = 1.0 / (10000.0 ** (np.arange(0, 32, 2, dtype=np.float32) / 32))
    assert np.allclose(sin[5, :16], np.sin(5 * inv), atol=1e-6)


def test_rope_then_inverse_is_near_identity():
    """Rotation composition, the reference's un-RoPE (-sin) of a cache slice:
    the round trip returns the stored values within two bf16 roundings."""
    L, S, W, T = 2, 64, 288, 20
    arena = _arena(9, L, S, W)
    cos, sin = graft_mount.rope_tables(S, 32)
    seats = np.array([10], np.int64)
    fwd = O.mount_rope(arena, 1, L, T, seats, cos, sin, 256, 32)
    back = O.mount_rope(fwd, 1, L, T, seats, cos, -sin, 256, 32)
    x0 = _to_f32(arena[:, 10:30, 256:])
    x1 = _to_f32(back[:, 10:30, 256:])
    assert np.allclose(x0, x1, rtol=2e-2, atol=6e-2)
    assert not np.array_equal(fwd, arena)


@pytest.mark.parametrize("offset,dim", [(250, 32), (0, 7), (300, 32)])
def test_oracle_rope_rejects_bad_layouts(offset, dim):
    arena = _arena(1, 1, 40, 288)
    cos, sin = graft_mount.rope_tables(40, 32)
    with pytest.raises(ValueError):
        O.mount_rope(arena, 1, 1, 4, [0], cos, sin, offset, dim)


def test_oracle_rope_rejects_seats_past_the_tables():
    arena = _arena(1, 1, 100, 288)
    cos, sin = graft_mount.rope_tables(50, 32)
    with pytest.raises(ValueError):
        O.mount_rope(arena, 1, 1, 8, [45], cos, sin, 256, 32)
