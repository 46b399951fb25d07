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


def _policy_case(seed, n, dim):
    rng = np.random.default_rng(seed)
    rows = rng.standard_normal((n, dim)).astype(np.float32)
    rows[::53] = rows[7]                          # tie groups
    vocab = [f"tok{i}" for i in range(60)] + ["common"]
    lex = []
    for i in range(n):
        keys = list(rng.choice(vocab[:-1], rng.integers(0, 4), replace=False))
        if i % 3 == 0:
            keys.append("common")
        lex.append(keys if keys else None)
    kinds = [str(rng.choice(["turn", "doc", "fact", "custom", ""])) for _ in range(n)]
    scopes = [str(rng.choice(["conversation", "project", "user", "odd scope"])) for _ in range(n)]
    active = rng.random(n) > 0.08
    return rows, lex, [kinds, scopes, None, None], active, rng


@pytest.mark.parametrize("seed,n,dim", [(21, 900, 64), (22, 1500, 128), (23, 400, 16)])
def test_mla_policy_restatement_equals_reference_runtime(seed, n, dim):
    """Lexical bonus, filters (known, unknown and default values) and
    inactive nodes: route_mla_arena through grm_store_route_filtered."""
    rows, lex, cats, active, rng = _policy_case(seed, n, dim)
    cases = [
        ([], None),
        (["tok1", "tok2"], None),
        (["common"], None),
        (["tok3", "tok3", "nosuchkey"], [["doc", "custom"], None, None, None]),
        (["tok4", "common"], [["turn"], ["project", "user"], None, None]),
        ([], [None, ["odd scope"], ["session"], None]),
        (["tok5"], [None, None, ["permanent"], None]),      # excludes every node
        (["tok6"], [None, None, None, ["ephemeral", "stable"]]),
    ]
    with O.RefStore().load_mla_policy(rows, lex, cats, active) as st:
        for qlex, filt in cases:
            q = rng.standard_normal(dim).astype(np.float32)
            for k in (1, 5, 16):
                want = st.route_policy(q, k, qlex, filt)
                ids, _ = O.mla_route_policy(rows, q, k, node_lexical=lex, cats=cats,
                                            active=active, query_lexical=qlex, filters=filt)
                got = [int(x) for x in ids if x != np.iinfo(np.uint64).max]
                assert got == want, (qlex, filt, k)


@pytest.mark.parametrize("seed,qt", [(31, 1), (32, 4), (33, 2)])
def test_gqa_policy_restatement_equals_reference_runtime(seed, qt):
    """The GQA lexical law (raw / (max raw + 1e-8) + hits / m), filters and
    inactive nodes through grm_store_route_gqa."""
    rng = np.random.default_rng(seed)
    n, kv, d, h = 70, 4, 32, 16
    T = rng.integers(0, 30, n)
    T[0] = T[9] = 0
    off = np.zeros(n + 1, np.uint64)
    off[1:] = np.cumsum(T)
    keys = O.f32_to_bf16_bits(rng.standard_normal(int(off[-1]) * kv * d).astype(np.float32))
    vocab = [f"t{i}" for i in range(15)]
    lex = [list(rng.choice(vocab, rng.integers(0, 3), replace=False)) for _ in range(n)]
    kinds = [str(rng.choice(["turn", "doc", "custom", ""])) for _ in range(n)]
    muts = [str(rng.choice(["ephemeral", "stable", "weird"])) for _ in range(n)]
    active = rng.random(n) > 0.1
    cats = [kinds, None, None, muts]
    with O.RefStore().load_gqa_policy(keys, off, kv, d, lex, cats, active) as st:
        for t in range(12):
            q = rng.standard_normal((h, qt, d)).astype(np.float32)
            qlex = list(rng.choice(vocab + ["absent"], rng.integers(0, 4)))
            filt = [[None] * 4, [["doc", "custom"], None, None, None],
                    [None, None, None, ["weird", "stable"]], [["turn"], None, None, ["x"]]][t % 4]
            for k in (1, 7):
                want = st.route_policy(q, k, qlex, filt)
                ids, _ = O.gqa_route_policy(keys, off, kv, d, q, k, node_lexical=lex, cats=cats,
                                            active=active, query_lexical=qlex, filters=filt)
                got = [int(x) for x in ids if x != np.iinfo(np.uint64).max]
                assert got == want, (t, qlex, filt, k)


@pytest.mark.parametrize("seed,dim", [(41, 64), (42, 256)])
def test_mla_multi_row_restatement_equals_reference_runtime(seed, dim):
    """Entries of several rows (digest + child centroids) score the max of
    their rows: route_mla_arena over entry_row_offsets."""
    rng = np.random.default_rng(seed)
    E = 400
    counts = rng.integers(1, 6, E)
    off = np.zeros(E + 1, np.uint64)
    off[1:] = np.cumsum(counts)
    rows = rng.standard_normal((int(off[-1]), dim)).astype(np.float32)
    rows[int(off[7]):int(off[8])] = rows[int(off[3])]   # ties across entries
    rows[int(off[11]), 0] = np.nan                        # one bad row of an entry
    with O.RefStore().load_mla_multi(rows, off) as st:
        for _ in range(8):
            q = rng.standard_normal(dim).astype(np.float32)
            for k in (1, 5, 16):
                want = st.route(q, k)
                ids, _ = O.mla_route_multi(rows, off, q, k)
                got = [int(x) for x in ids if x != np.iinfo(np.uint64).max]
                assert got == want


def test_config1_exact_recipe_equals_reference_runtime():
    """BASELINE config 1 as written: default_rng(0), 10,000 x 256 N(0,1) rows
    L2-normalised in fp32 and stored fp16, the query the generator's next draw,
    top-3."""
    from graftrepository_b200 import synth

    rows16, qs = synth.mla_config(0, 10_000)
    rows = rows16.astype(np.float32)
    ids, _ = O.mla_route(rows, qs[0], 3)
    with O.RefStore().load_mla(rows) as st:
        assert [int(x) for x in ids] == st.route(qs[0], 3)


def test_config4_longest_nodes_equal_reference_runtime():
    """The tail of config 4's length distribution (lognormal(ln 192, 0.8)
    clipped 8..4096, 100,000 nodes): its 20 longest nodes, eight of them at
    4,096 tokens, routed by the reference runtime (4 layers x 8 kv heads on the
    head axis, 128 query heads) and by the restatement."""
    from graftrepository_b200 import synth

    lengths = synth.gqa_lengths(3, 100_000, "lognormal")
    top = np.sort(np.argsort(-lengths, kind="stable")[:20])
    sub = lengths[top]
    assert int((sub == 4096).sum()) == 8
    keys, off = synth.gqa_bank(3, sub)
    q = synth.gqa_query(3)[0]
    ids, _ = O.gqa_route(keys, off, 32, 128, q, 5)
    with O.RefStore().load_gqa(keys, off, 32, 128) as st:
        want = st.route(q, 5)
    assert [int(x) for x in ids] == want


@pytest.mark.parametrize("seed,n,dim,m", [(51, 3000, 256, 200), (52, 1500, 64, 64),
                                          (53, 800, 128, 5000), (54, 5000, 256, 4096)])
def test_mla_int4_restatement_equals_reference_runtime(seed, n, dim, m, monkeypatch):
    """The INT4 bulk/refine route (GRM_ROUTER_INT4=1, route_mla_int4,
    cpp/grm_runtime.cpp:4363-4482) of the reference runtime's default build
    against the restatement: fp16-valued rows (duplicate rows, a NaN row, an
    Inf row, a zero row), refine sets smaller than, equal to and larger than
    the bank."""
    rng = np.random.default_rng(seed)
    rows = rng.standard_normal((n, dim)).astype(np.float32)
    rows /= np.linalg.norm(rows, axis=1, keepdims=True)
    rows = rows.astype(np.float16).astype(np.float32)
    rows[::97] = rows[3]
    rows[5, 1] = np.nan
    rows[6, 2] = np.inf
    rows[7] = 0.0
    qs = rng.standard_normal((5, dim)).astype(np.float32)
    qs[1] = rows[3]
    qs[2] *= 1e-6
    monkeypatch.setenv("GRM_ROUTER_INT4", "1")
    monkeypatch.setenv("GRM_ROUTER_INT4_REFINE_M", str(m))
    with O.RefStore().load_mla(rows) as st:
        for q in qs:
            for k in (1, 3, 16):
                ids, _ = O.mla_int4_route(rows, q, k, refine_m=m)
                want = st.route(q, k)
                got = [int(x) for x in ids if x != np.iinfo(np.uint64).max]
                assert got == want, (k, got, want)


def test_mla_int4_restatement_rounding_order_equals_reference_runtime(monkeypatch):
    """Rows that are permutations of one integer vector, queried with equal
    values in every dim: the INT4 bulk ranking is decided by the rounding of
    the sequential fp32 sum alone (the refine scores all tie), so this pins the
    restatement's bulk arithmetic -- separately rounded products and sums in
    element order -- to the reference runtime's default build."""
    rng = np.random.default_rng(66)
    base = rng.integers(-7, 8, 256).astype(np.float32)
    base[0], base[1] = 7.0, -7.0
    rows = np.stack([base[rng.permutation(256)] for _ in range(3000)]).astype(np.float32)
    qs = [np.full(256, 0.7317093, np.float32),
          np.where(np.arange(256) % 3 == 0, -1.3371, 0.4142).astype(np.float32)]
    monkeypatch.setenv("GRM_ROUTER_INT4", "1")
    for m in (1, 16, 700):
        monkeypatch.setenv("GRM_ROUTER_INT4_REFINE_M", str(m))
        with O.RefStore().load_mla(rows) as st:
            for q in qs:
                for k in (1, 5):
                    ids, _ = O.mla_int4_route(rows, q, k, refine_m=m)
                    got = [int(x) for x in ids if x != np.iinfo(np.uint64).max]
                    assert got == st.route(q, k), (m, k)


def test_mla_int4_mode_differs_from_the_exact_route():
    """With a small refine set the INT4 mode's answer can differ from the exact
    route (the bulk pass decides which rows are refined): the restatement must
    reproduce that, not the exact answer."""
    rng = np.random.default_rng(55)
    n, dim = 20_000, 64
    rows = rng.standard_normal((n, dim)).astype(np.float32)
    norms = O.mla_row_norms(rows)
    diffs = 0
    for _ in range(20):
        q = rng.standard_normal(dim).astype(np.float32)
        a, _ = O.mla_int4_route(rows, q, 16, refine_m=16, norms=norms)
        b, _ = O.mla_route(rows, q, 16, norms=norms)
        diffs += int(not np.array_equal(a, b))
    assert diffs > 0
