"""Ragged GQA route parity on the GPU through the C ABI, against the reference
goldens and the CPU oracle (ids and scores bit-exact)."""

import numpy as np
import pytest

import oracle as O
from graftrepository_b200 import _lib, synth
from graftrepository_b200.cuda_router import CudaGQARouteSidecar, upload_queries

pytestmark = pytest.mark.gpu
U64MAX = np.iinfo(np.uint64).max


@pytest.fixture(scope="module")
def sidecar():
    return CudaGQARouteSidecar(device=0)


def raw_route(bank, q, k):
    q = np.ascontiguousarray(q, dtype=np.float32)
    if q.ndim == 3:
        q = q[None]
    ids, scores, _, _ = bank._run(_lib.load().grm_b200_gqa_route, q.ctypes.data, q.shape[0],
                                  q.shape[1], q.shape[2], k, 0)
    return ids, scores


def check(bank, keys, off, kh, d, qs, k):
    ids, scores = raw_route(bank, qs, k)
    for i, q in enumerate(qs):
        want, want_s = O.gqa_route(keys, off, kh, d, q, k)
        assert np.array_equal(ids[i], want), (i, ids[i], want)
        fin = want != U64MAX
        assert np.array_equal(scores[i][fin], want_s[fin]), (i, scores[i], want_s)


@pytest.mark.parametrize("name", ["gqa_d128.npz", "gqa_d64_l4.npz"])
def test_golden_vectors(sidecar, golden, name):
    g = golden(name)
    kh, d, k = int(g["kv_heads"]), int(g["head_dim"]), int(g["topk"])
    bank = sidecar.create_bank_csr(g["keys_bf16"], g["token_offsets"], kh, d, dtype="bf16")
    for key in ("q1", "q4", "qnan"):
        ids, scores = raw_route(bank, g[key], k)
        assert np.array_equal(ids, g[key + "_ids"]), key
        for i, q in enumerate(g[key]):
            _, want_s = O.gqa_route(g["keys_bf16"], g["token_offsets"], kh, d, q, k)
            fin = g[key + "_ids"][i] != U64MAX
            assert np.array_equal(scores[i][fin], want_s[fin]), (key, i)
    bank.close()


def _ragged(seed, n, kh, d, tmax, zero_nodes=(), nan_node=None, dup=None):
    rng = np.random.default_rng(seed)
    T = rng.integers(1, tmax + 1, n)
    for z in zero_nodes:
        T[z] = 0
    if dup:
        T[dup[0]] = T[dup[1]]
    off = synth.offsets(T)
    keys = synth.bf16_bits(rng.standard_normal(int(off[-1]) * kh * d, dtype=np.float32))
    if dup:
        a, b = dup
        ka = slice(int(off[a]) * kh * d, int(off[a + 1]) * kh * d)
        kb = slice(int(off[b]) * kh * d, int(off[b + 1]) * kh * d)
        keys[ka] = keys[kb]
    if nan_node is not None:
        keys[int(off[nan_node]) * kh * d + 3] = 0x7FC0
    return keys, off


@pytest.mark.parametrize("group,qt", [(4, 1), (1, 1), (2, 2), (8, 1), (4, 4), (4, 2), (16, 1)])
def test_random_ragged(sidecar, group, qt):
    kh, d = 8, 128
    keys, off = _ragged(group * 10 + qt, 70, kh, d, 150, zero_nodes=(3, 40), nan_node=9,
                        dup=(30, 50))
    bank = sidecar.create_bank_csr(keys, off, kh, d, dtype="bf16")
    assert bank.paths() == {"fast": True, "tma": True}
    rng = np.random.default_rng(qt)
    qs = rng.standard_normal((3, kh * group, qt, d), dtype=np.float32)
    for k in (1, 3, 16):
        check(bank, keys, off, kh, d, qs, k)
    bank.close()


@pytest.mark.parametrize("group,qt", [(4, 1), (8, 1), (4, 4), (16, 1)])
def test_refine_near_ties_and_overflowing_bound(sidecar, group, qt):
    """Near ties: in two nodes every token of a kv head is one base row with a
    single element nudged by one bf16 ulp, so the tokens' dots differ far
    inside the approximate pass's error bound and only the exact dots can
    order them (both scaled by 4, so that they rank in the top 16 and are
    always refined).  Overflowing bound: one node scaled by 1e28, where |q||k|
    exceeds the approximation's range and every token is refined exactly."""
    kh, d = 8, 128
    keys, off = _ragged(group * 7 + qt, 60, kh, d, 120)
    T = np.diff(off).astype(np.int64)
    rng = np.random.default_rng(group + qt)
    for node in (5, 17):
        t = int(T[node])
        base = int(off[node]) * kh * d
        blk = keys[base: base + t * kh * d].reshape(kh, t, d)
        blk[:] = synth.bf16_bits(O.bf16_bits_to_f32(blk[:, :1, :]) * np.float32(4.0))
        for h in range(kh):
            for tok in range(1, t):
                j = int(rng.integers(0, d))
                bits = int(blk[h, tok, j])
                if bits & 0x7FFF not in (0, 0x7F7F):
                    blk[h, tok, j] = bits + int(rng.choice([-1, 1]))
    big = 40
    sl = slice(int(off[big]) * kh * d, int(off[big + 1]) * kh * d)
    keys[sl] = synth.bf16_bits(O.bf16_bits_to_f32(keys[sl]) * np.float32(1e28))
    bank = sidecar.create_bank_csr(keys, off, kh, d, dtype="bf16")
    assert bank.paths() == {"fast": True, "tma": True}
    qs = np.random.default_rng(qt).standard_normal((2, kh * group, qt, d), dtype=np.float32)
    for k in (3, 16):
        check(bank, keys, off, kh, d, qs, k)
    ids, _ = raw_route(bank, qs, 16)
    assert ids[:, 0].tolist() == [big, big]
    assert all({5, 17} <= set(r.tolist()) for r in ids)
    bank.close()


def test_dim64_and_generic_dim(sidecar):
    for d in (64, 96):
        keys, off = _ragged(d, 40, 4, d, 60)
        bank = sidecar.create_bank_csr(keys, off, 4, d, dtype="bf16")
        qs = np.random.default_rng(d).standard_normal((2, 16, 1, d), dtype=np.float32)
        check(bank, keys, off, 4, d, qs, 5)
        bank.close()


def test_fp16_and_fp32_banks(sidecar):
    rng = np.random.default_rng(77)
    T = rng.integers(0, 50, 30)
    off = synth.offsets(T)
    vals = rng.standard_normal(int(off[-1]) * 4 * 128).astype(np.float32)
    q = rng.standard_normal((2, 16, 1, 128), dtype=np.float32)
    for kind in ("f16", "f32"):
        v = vals.astype(np.float16).astype(np.float32) if kind == "f16" else vals
        bank = sidecar.create_bank_csr(v, off, 4, 128, dtype=kind)
        ids, scores = raw_route(bank, q, 6)
        for i in range(2):
            want_s_all = _oracle_scores_f32(v, off, 4, 128, q[i])
            want, want_s, _ = O.topk(want_s_all, 6)
            assert np.array_equal(ids[i], want), kind
            fin = want != U64MAX
            assert np.array_equal(scores[i][fin], want_s[fin]), kind
        bank.close()


def _oracle_scores_f32(vals, off, kh, d, q):
    """The reference law on fp32 keys, via the reference runtime when present,
    else via a bf16-exact split (only used for fp16-representable values)."""
    # fp32 keys are not bf16 bit patterns: evaluate the law in numpy-free C by
    # splitting each fp32 key k = hi + lo is not exact, so use the reference
    # runtime order directly: sequential fp32 per dot.
    n = off.shape[0] - 1
    out = np.empty(n, np.float32)
    inv = np.float32(1.0) / np.sqrt(np.float32(d))
    H, qt, _ = q.shape
    rep = H // kh
    for i in range(n):
        T = int(off[i + 1] - off[i])
        if T == 0:
            out[i] = 0.0
            continue
        blk = vals[int(off[i]) * kh * d: int(off[i + 1]) * kh * d].reshape(kh, T, d)
        if not np.all(np.isfinite(blk)):
            out[i] = np.nan
            continue
        total = np.float32(0.0)
        for h in range(H):
            best = np.float32(0.0)
            for qi in range(qt):
                prods = (q[h, qi][None, :] * blk[h // rep]).astype(np.float32)
                dots = np.zeros(T, np.float32)
                for j in range(d):
                    dots = (dots + prods[:, j]).astype(np.float32)
                v = (np.abs(dots) * inv).astype(np.float32).max()
                best = max(best, v)
            total = np.float32(total + best)
        out[i] = np.float32(total / np.float32(H))
    return out


def test_dense_padded_bank_equals_csr(sidecar):
    keys, off = _ragged(5, 20, 4, 128, 30)
    T = np.diff(off).astype(np.int64)
    dense = np.zeros((20, 4, 30, 128), np.float32)
    f = O.bf16_bits_to_f32(keys)
    for i in range(20):
        dense[i, :, : T[i]] = f[int(off[i]) * 512: int(off[i + 1]) * 512].reshape(4, T[i], 128)
    q = np.random.default_rng(1).standard_normal((16, 1, 128), dtype=np.float32)
    b1 = sidecar.create_bank(dense, token_counts=T)
    b2 = sidecar.create_bank(dense)                 # padding kept: identical law
    i1, _ = b1.route_topk(q, topk=5)
    i2, _ = b2.route_topk(q, topk=5)
    want, _ = O.gqa_route(keys, off, 4, 128, q, 5)
    assert i1[0].tolist() == want.tolist() == i2[0].tolist()
    dq = upload_queries(q[None])
    i3, _ = b1.route_topk_device(dq, topk=5)
    assert np.array_equal(i1, i3)
    dq.close()
    b1.close()
    b2.close()


def test_full_size_config3(sidecar):
    """512 nodes, T ~ U{16..1024}, [4 layers x 8 kv heads, T, 128] bf16, 128 query heads."""
    lengths = synth.gqa_lengths(2, 512)
    keys, off = synth.gqa_bank(2, lengths)
    q = synth.gqa_query(2, count=2)
    bank = CudaGQARouteSidecar(device=0).create_bank_csr(keys, off, 32, 128, dtype="bf16")
    ids, scores = raw_route(bank, q, 3)
    for i in range(2):
        want, want_s = O.gqa_route(keys, off, 32, 128, q[i], 3)
        assert np.array_equal(ids[i], want)
        assert np.array_equal(scores[i], want_s)
    routes, refined = bank.stats()
    assert routes == 2 and refined >= 6
    bank.close()


def test_async_route_device_outputs_and_offset(sidecar):
    import torch

    keys, off = _ragged(12, 50, 8, 128, 200, zero_nodes=(7,), dup=(10, 11))
    bank = sidecar.create_bank_csr(keys, off, 8, 128, dtype="bf16")
    qs = np.random.default_rng(12).standard_normal((3, 32, 1, 128), dtype=np.float32)
    want_ids, want_s = raw_route(bank, qs, 4)
    dq = torch.from_numpy(qs).cuda()
    ids = torch.empty((3, 4), dtype=torch.int64, device="cuda")
    sc = torch.empty((3, 4), dtype=torch.float32, device="cuda")
    rc = _lib.load().grm_b200_gqa_route_async(bank._h, dq.data_ptr(), 3, 32, 1, 4, 1000,
                                              ids.data_ptr(), sc.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    got = ids.cpu().numpy().view(np.uint64)
    assert np.array_equal(got, want_ids + 1000)
    assert np.array_equal(sc.cpu().numpy(), want_s)
    bank.close()


def test_config4_lognormal_subset(sidecar):
    """Config 4's length distribution (lognormal(ln 192, 0.8) clipped 8..4096,
    100,000 nodes, default_rng(3)) on a subset the oracle finishes in seconds:
    the 20 longest nodes (eight at 4,096 tokens) plus the longest node prefix
    that keeps the subset under 400k tokens.  Long nodes exercise the per-item
    chunk count, the work-item list and the key-norm bounds."""
    lengths = synth.gqa_lengths(3, 100_000, "lognormal")
    idx = synth.longest_plus_prefix(lengths, 20, 400_000)
    sub = lengths[idx]
    assert int((sub == 4096).sum()) == 8 and int(sub.sum()) <= 400_000
    keys, off = synth.gqa_bank(3, sub)
    qs = synth.gqa_query(3, count=2)
    bank = sidecar.create_bank_csr(keys, off, 32, 128, dtype="bf16")
    assert bank.paths() == {"fast": True, "tma": True}
    for k in (3, 16):
        ids, scores = raw_route(bank, qs, k)
        for i in range(2):
            want, want_s = O.gqa_route(keys, off, 32, 128, qs[i], k)
            assert np.array_equal(ids[i], want), (k, i, ids[i], want)
            assert np.array_equal(scores[i], want_s), (k, i)
    bank.close()
