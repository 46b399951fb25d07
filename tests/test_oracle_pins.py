"""Pin the C restatement against the reference's own runtime (cpp/grm_runtime.cpp
compiled from its sources into oracle/_ref/) on seeded fuzz cases larger than
the committed goldens.  CPU only; skipped where the reference was not built."""

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built here")


@pytest.mark.parametrize("seed,n,dim", [(1234, 2000, 256), (5678, 1200, 16), (7, 777, 128)])
def test_mla_restatement_equals_reference_runtime(seed, n, dim):
    rng = np.random.default_rng(seed)
    rows = rng.standard_normal((n, dim)).astype(np.float32)
    rows[::97] = rows[3]                          # tie groups
    rows[5, 1] = np.nan
    qs = rng.standard_normal((4, dim)).astype(np.float32)
    qs[1] = rows[3]
    with O.RefStore().load_mla(rows) as st:
        for q in qs:
            ids, _ = O.mla_route(rows, q, 16)
            want = st.route(q, 16)
            got = [int(x) for x in ids if x != np.iinfo(np.uint64).max]
            assert got == want


@pytest.mark.parametrize("qt", [1, 2, 4])
@pytest.mark.parametrize("kv,h", [(4, 16), (8, 8), (2, 8)])
def test_gqa_restatement_equals_reference_runtime(qt, kv, h):
    rng = np.random.default_rng(100 * qt + kv)
    n, d = 30, 32
    T = rng.integers(0, 40, n)
    T[0] = 0
    off = np.zeros(n + 1, np.uint64)
    off[1:] = np.cumsum(T)
    keys = O.f32_to_bf16_bits(rng.standard_normal(int(off[-1]) * kv * d).astype(np.float32))
    q = rng.standard_normal((h, qt, d)).astype(np.float32)
    ids, _ = O.gqa_route(keys, off, kv, d, q, 12)
    with O.RefStore().load_gqa(keys, off, kv, d) as st:
        want = st.route(q, 12)
    got = [int(x) for x in ids if x != np.iinfo(np.uint64).max]
    assert got == want
