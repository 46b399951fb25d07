"""Route policy on the GPU (lexical bonus, kind/scope/durability/mutability
filters, inactive nodes) through grm_b200_mla_route_policy, against the CPU
oracle's restatement of route_mla_arena (cpp/grm_runtime.cpp:4299-4361, pinned
to the reference runtime in test_oracle_pins.py): ids and policy scores
bit-exact."""

import numpy as np
import pytest

import oracle as O
from graftrepository_b200 import synth
from graftrepository_b200.cuda_router import CudaMLARouteSidecar

pytestmark = pytest.mark.gpu
U64MAX = np.iinfo(np.uint64).max


@pytest.fixture(scope="module")
def sidecar():
    return CudaMLARouteSidecar(device=0)


def make_policy(seed, n, n_common=3):
    rng = np.random.default_rng(seed)
    vocab = [f"k{i}" for i in range(max(50, n // 20))]
    common = [f"common{i}" for i in range(n_common)]
    lex = []
    for i in range(n):
        keys = list(rng.choice(vocab, rng.integers(0, 4), replace=False))
        for j, c in enumerate(common):
            if i % (2 + j) == 0:
                keys.append(c)
        lex.append(keys)
    kinds = [str(rng.choice(["turn", "doc", "fact", "digest", "custom"])) for _ in range(n)]
    scopes = [str(rng.choice(["conversation", "project", "user", ""])) for _ in range(n)]
    durs = [str(rng.choice(["session", "permanent", "volatile"])) for _ in range(n)]
    active = rng.random(n) > 0.05
    return lex, [kinds, scopes, durs, None], active, vocab, common


def check(bank, rows, qs, k, lex, cats, active, qlex, filt):
    ids, sc = bank.route_policy_topk(qs, topk=k, lexical_keys=qlex,
                                     kinds=filt[0] or (), scopes=filt[1] or (),
                                     durabilities=filt[2] or (), mutabilities=filt[3] or ())
    norms = O.mla_row_norms(rows)
    for i, q in enumerate(qs):
        want, want_s = O.mla_route_policy(rows, q, k, node_lexical=lex, cats=cats, active=active,
                                          query_lexical=qlex[i], filters=filt, norms=norms)
        assert np.array_equal(ids[i], want), (i, ids[i], want)
        fin = want != U64MAX
        assert np.array_equal(sc[i][fin], want_s[fin]), (i, sc[i], want_s)


@pytest.mark.parametrize("dim,n", [(64, 5000), (128, 20000), (256, 70001)])
def test_lexical_and_filters_match_oracle(sidecar, dim, n):
    rows = synth.mla_bank(dim + 3 * n, n, dim).astype(np.float32)
    lex, cats, active, vocab, common = make_policy(dim, n)
    bank = sidecar.create_bank(rows)
    bank.set_route_policy(lexical_keys=lex, kinds=cats[0], scopes=cats[1], durabilities=cats[2],
                          active=active)
    qs = synth.mla_queries(n + 5, 4, dim)
    qlex = [[vocab[1], vocab[2]], [common[0]], [vocab[3], vocab[3], "absent-key"],
            [common[1], common[2], vocab[7]]]
    nofilt = [None] * 4
    for k in (1, 5, 16, 32):
        check(bank, rows, qs, k, lex, cats, active, qlex, nofilt)
    for filt in ([["doc", "custom"], None, None, None],
                 [None, ["conversation", "nosuch"], ["permanent"], None],
                 [["turn", "fact"], ["project"], None, ["ephemeral"]],
                 [["era"], None, None, None]):
        check(bank, rows, qs, 8, lex, cats, active, qlex, filt)
        check(bank, rows, qs, 8, lex, cats, active, [[]] * 4, filt)
    bank.close()


def test_policy_defaults_without_set(sidecar):
    """No policy data: every node is active with the reference defaults, so a
    filter on a default value keeps every node and any other value none."""
    rows = synth.mla_bank(41, 3000).astype(np.float32)
    qs = synth.mla_queries(42, 2)
    bank = sidecar.create_bank(rows)
    ids, _ = bank.route_policy_topk(qs, topk=5, lexical_keys=[["x"], []], kinds=["turn"])
    for i, q in enumerate(qs):
        want, _ = O.mla_route(rows, q, 5)
        assert np.array_equal(ids[i], want)
    ids, _ = bank.route_policy_topk(qs, topk=5, kinds=["doc"])
    assert np.all(ids == U64MAX)
    bank.close()


def test_lexical_ties_and_store_route_signature(sidecar):
    """Duplicate rows with equal hits tie on S: lower row first.  The
    NativeGraftStore.route-shaped call returns the same ids as the batch form."""
    rng = np.random.default_rng(43)
    base = rng.standard_normal((5, 128)).astype(np.float32)
    rows = np.repeat(base, 400, axis=0).astype(np.float16).astype(np.float32)
    n = rows.shape[0]
    lex = [["a"] if i % 7 == 0 else (["a", "b"] if i % 11 == 0 else []) for i in range(n)]
    bank = sidecar.create_bank(rows)
    bank.set_route_policy(lexical_keys=lex)
    q = base[2] + 0.01
    for qlex in (["a"], ["a", "b"], ["b", "b"]):
        ids, sc = bank.route_policy_topk(q, topk=16, lexical_keys=qlex)
        want, want_s = O.mla_route_policy(rows, q, 16, node_lexical=lex, query_lexical=qlex)
        assert np.array_equal(ids[0], want)
        assert np.array_equal(sc[0], want_s)
        assert bank.route(q, qlex, 16) == [int(x) for x in want if x != U64MAX]
    bank.close()


def test_nan_rows_and_queries_under_policy(sidecar):
    rows = synth.mla_bank(44, 2000).astype(np.float32)
    rows[3, 0] = np.nan
    rows[8, 1] = np.inf
    lex = [["hot"] if i in (3, 8, 9, 10) else [] for i in range(2000)]
    bank = sidecar.create_bank(rows)
    bank.set_route_policy(lexical_keys=lex)
    qs = synth.mla_queries(45, 3)
    qs[1] = 0.0
    qs[2, 4] = np.nan
    qlex = [["hot"], ["hot"], ["hot"]]
    check(bank, rows, qs, 6, lex, None, None, qlex, [None] * 4)
    bank.close()


# ----------------------------------------------------------------------- GQA

def gqa_bank(seed, n, kv=8, d=128, tmax=300):
    rng = np.random.default_rng(seed)
    T = rng.integers(0, tmax, n)
    T[::17] = 0
    off = np.zeros(n + 1, np.uint64)
    off[1:] = np.cumsum(T)
    keys = O.f32_to_bf16_bits(rng.standard_normal(int(off[-1]) * kv * d).astype(np.float32))
    return keys, off, rng


@pytest.mark.parametrize("qt", [1, 4])
def test_gqa_lexical_and_filters_match_oracle(qt):
    from graftrepository_b200.cuda_router import CudaGQARouteSidecar

    n, kv, d, h = 600, 8, 128, 32
    keys, off, rng = gqa_bank(50 + qt, n, kv, d)
    vocab = [f"g{i}" for i in range(40)]
    lex = [list(rng.choice(vocab, rng.integers(0, 4), replace=False)) + (["hot"] if i % 5 == 0 else [])
           for i in range(n)]
    kinds = [str(rng.choice(["turn", "doc", "fact"])) for _ in range(n)]
    durs = [str(rng.choice(["session", "permanent"])) for _ in range(n)]
    active = rng.random(n) > 0.07
    cats = [kinds, None, durs, None]
    side = CudaGQARouteSidecar(device=0)
    bank = side.create_bank_csr(keys.view(np.uint16), off, kv, d)
    bank.set_route_policy(lexical_keys=lex, kinds=kinds, durabilities=durs, active=active)
    qs = rng.standard_normal((4, h, qt, d)).astype(np.float32)
    qlex = [[], ["hot"], [vocab[1], vocab[2], "absent"], [vocab[3], vocab[3]]]
    for filt in ([None] * 4, [["doc", "fact"], None, None, None],
                 [None, None, ["permanent"], None], [["era"], None, None, None]):
        for k in (1, 5, 16):
            ids, sc = bank.route_policy_topk(qs, topk=k, lexical_keys=qlex,
                                             kinds=filt[0] or (), durabilities=filt[2] or ())
            for i in range(4):
                want, want_s = O.gqa_route_policy(keys, off, kv, d, qs[i], k, node_lexical=lex,
                                                  cats=cats, active=active,
                                                  query_lexical=qlex[i], filters=filt)
                assert np.array_equal(ids[i], want), (filt, k, i, ids[i], want)
                fin = want != U64MAX
                assert np.array_equal(sc[i][fin], want_s[fin])
    assert bank.route_gqa(qs[1][:, :, :], ["hot"], 5) == [
        int(x) for x in O.gqa_route_policy(keys, off, kv, d, qs[1], 5, node_lexical=lex,
                                           cats=cats, active=active, query_lexical=["hot"])[0]
        if x != U64MAX]
    bank.close()
