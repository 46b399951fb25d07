"""The re-RoPE mount oracle (orc_mount_rope) against a numpy restatement of the
reference's rotation of the positional key part at the mount seats
(core/graft_arena.py:339-367 `_pair_swap_last` / `_rope_tensor` /
`_rope_block_at`, applied at seats n_sink.. by `_graft_block`, :1848-1859):
x' = pair_swap(x), out = bf16(x' * cos[pos] + rotate_half(x') * sin[pos]).
`apply_rotary` lives in the reference's compiled tensor library, which is not
part of the reference tree, so the restatement follows the standard
rotate-half form the Python fallback calls.  The same law as the reference
writes it in Python (rope / rope_tables of tests/gemma4_int4_sim.py:60-76 and
_deepseek_rope_prep of core/deepseek_v2_lite_tc.py:99-103), executed by
tests/golden/make_rope_golden.py, pins the oracle to a stated tolerance."""

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


GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden" / "rope_law.npz"


@pytest.mark.parametrize("name", ["mla_kpe", "gqa_k", "p_rope"])
def test_oracle_rope_matches_the_reference_rotary_functions(name):
    """orc_mount_rope against the reference's own rotation law, executed by
    tests/golden/make_rope_golden.py: rope() and rope_tables() of
    tests/gemma4_int4_sim.py:60-76 (full rotary and p-RoPE tables, fp64) and
    the pair permutation _deepseek_rope_prep of core/deepseek_v2_lite_tc.py:99-103.
    The reference computes in fp64; the mount computes x*cos + rot(x)*sin in
    fp32 with the tables rounded to fp32, then rounds to bf16.  Tolerance:
    every value within one bf16 ulp of the reference's fp64 value (2^-8
    relative, plus 1e-5 absolute for results that cancel to near zero), and
    at least 99.9% of them equal to its round-to-nearest-even bf16 (all of them
    are, on this fixture)."""
    g = np.load(GOLDEN)
    W, off, dim, heads, swap, T, L = (int(v) for v in g[f"{name}_meta"])
    windows, seats = g[f"{name}_windows"], g[f"{name}_seats"]
    cos, sin = g[f"{name}_cos"], g[f"{name}_sin"]
    S = cos.shape[0]
    arena = np.zeros((L, S, W), np.uint16)
    for w, s in zip(windows, seats):
        arena[:, s:s + T] = w
    got = O.mount_rope(arena, len(seats), L, T, seats, cos.astype(np.float32),
                       sin.astype(np.float32), off, dim, bool(swap))
    want = g[f"{name}_want"]
    for gi, s in enumerate(seats):
        mine = _to_f32(got[:, s:s + T, off:off + heads * dim]).astype(np.float64)
        ref = want[gi]
        assert np.all(np.abs(mine - ref) <= np.abs(ref) * 2.0 ** -8 + 1e-5), (name, s)
        exact = np.mean(mine == _to_f32(_bf16_bits(ref.astype(np.float32))))
        assert exact >= 0.999, (name, s, exact)
        # the position-free columns keep their bytes
        assert np.array_equal(got[:, s:s + T, :off], arena[:, s:s + T, :off])


def test_rope_tables_match_the_reference_table_builder():
    """graft_mount.rope_tables (fp32, the construction of core/minicpm3_tc.py:345-355)
    against the reference's fp64 rope_tables (tests/gemma4_int4_sim.py:60-65) for
    full rotary at dim 32, theta 1e4: equal to fp32 angle rounding (pos * 2^-24)."""
    g = np.load(GOLDEN)
    want_c, want_s = g["tables32_cos"], g["tables32_sin"]
    cos, sin = graft_mount.rope_tables(want_c.shape[0], 32, theta=1e4)
    tol = np.arange(want_c.shape[0])[:, None] * 2.0 ** -22 + 1e-7
    assert np.all(np.abs(cos - want_c) <= tol)
    assert np.all(np.abs(sin - want_s) <= tol)
