"""MLA route parity on the GPU, through the C ABI (graftrepository_b200.cuda_router
-> libgrm_b200.so), against the reference goldens and the CPU oracle.
Ids and scores must be bit-exact."""

import numpy as np
import pytest

import oracle as O
from graftrepository_b200 import synth
from graftrepository_b200.cuda_router import CudaMLARouteSidecar, upload_queries

pytestmark = pytest.mark.gpu
U64MAX = np.iinfo(np.uint64).max


@pytest.fixture(scope="module")
def sidecar():
    return CudaMLARouteSidecar(device=0)


def raw_route(bank, qs, k):
    """Row ids + scores straight from the C ABI (no node-id mapping, no sentinel raise)."""
    from graftrepository_b200 import _lib

    q = np.ascontiguousarray(qs, dtype=np.float32).reshape(-1, bank.dim)
    ids, scores, _, _ = bank._route_raw(_lib.load().grm_b200_mla_route, q.ctypes.data,
                                        q.shape[0], k, 0)
    return ids, scores


def _check(bank, rows_f32, qs, k):
    ids, scores = raw_route(bank, qs, k)
    for i, q in enumerate(qs):
        want, want_s = O.mla_route(rows_f32, q, k)
        assert np.array_equal(ids[i], want), (i, ids[i], want)
        fin = want != U64MAX
        assert np.array_equal(scores[i][fin], want_s[fin]), (i, scores[i], want_s)
        assert np.all(np.isnan(scores[i][~fin]))


@pytest.mark.parametrize("name", ["mla_d256.npz", "mla_d64.npz"])
def test_golden_vectors(sidecar, golden, name):
    g = golden(name)
    rows = g["rows_f16"].view(np.float16).astype(np.float32)
    k = int(g["topk"])
    bank = sidecar.create_bank(rows)
    assert bank.dtype == 1  # exactly representable -> fp16 bank
    out, scores = raw_route(bank, g["queries"], k)
    assert np.array_equal(out, g["ids"])
    fin = g["ids"] != U64MAX
    np.testing.assert_allclose(scores[fin], g["scores"][fin], rtol=1e-6, atol=1e-7)
    for i, q in enumerate(g["queries"]):
        _, want_s = O.mla_route(rows, q, k)
        assert np.array_equal(scores[i][fin[i]], want_s[fin[i]])
    bank.close()


@pytest.mark.parametrize("n", [1, 31, 1000, 65537])
@pytest.mark.parametrize("dim", [64, 128, 256, 512])
def test_random_banks_fp16(sidecar, n, dim):
    rows = synth.mla_bank(n + dim, n, dim).astype(np.float32)
    qs = synth.mla_queries(n, 3, dim)
    bank = sidecar.create_bank(rows)
    for k in (1, 3, 16):
        _check(bank, rows, qs, k)
    bank.close()


@pytest.mark.parametrize("dim", [96, 256])
def test_fp32_bank_and_generic_dim(sidecar, dim):
    rng = np.random.default_rng(dim)
    rows = rng.standard_normal((5000, dim)).astype(np.float32)   # not fp16-representable
    qs = rng.standard_normal((2, dim)).astype(np.float32)
    bank = sidecar.create_bank(rows)
    assert bank.dtype == 0
    _check(bank, rows, qs, 5)
    bank.close()


def test_topk_32_and_sentinel_fill(sidecar):
    rows = synth.mla_bank(3, 20).astype(np.float32)
    rows[4, 0] = np.nan
    qs = synth.mla_queries(3, 2)
    bank = sidecar.create_bank(rows)
    got, _ = raw_route(bank, qs, 32)
    for i, q in enumerate(qs):
        want, _ = O.mla_route(rows, q, 32)
        assert np.array_equal(got[i], want)
        assert np.sum(got[i] != U64MAX) == 19
    with pytest.raises(RuntimeError):     # the sentinel law: fewer finite than topk
        bank.route_topk(qs, topk=25)
    bank.close()


def test_ties_force_the_exact_fallback(sidecar):
    rng = np.random.default_rng(9)
    base = rng.standard_normal((4, 256)).astype(np.float32)
    rows = np.repeat(base, 3000, axis=0)                      # 12000 rows, 4 tie groups
    rows = rows.astype(np.float16).astype(np.float32)
    q = base[2].astype(np.float16).astype(np.float32)[None]
    bank = sidecar.create_bank(rows)
    _check(bank, rows, q, 16)
    routes, fallbacks = bank.stats()
    assert fallbacks >= 1
    bank.close()


def test_unsafe_queries(sidecar):
    rows = synth.mla_bank(5, 3000).astype(np.float32)
    rows[7] = 0.0
    qs = synth.mla_queries(5, 5)
    qs[0] = 0.0
    qs[1] *= 1e-30
    qs[2] *= 1e25
    qs[3, 9] = np.inf
    bank = sidecar.create_bank(rows)
    raw = raw_route(bank, qs, 8)
    for i, q in enumerate(qs):
        want, want_s = O.mla_route(rows, q, 8)
        assert np.array_equal(raw[0][i], want), i
        fin = want != U64MAX
        assert np.array_equal(raw[1][i][fin], want_s[fin]), i
    bank.close()


def test_device_entry_matches_host_entry(sidecar):
    rows = synth.mla_bank(6, 20000).astype(np.float32)
    qs = synth.mla_queries(6, 6)
    bank = sidecar.create_bank(rows, node_ids=np.arange(20000, dtype=np.uint64) * 3 + 11)
    host_ids, rh = bank.route_topk(qs, topk=5, warmup=2)
    dq = upload_queries(qs)
    dev_ids, rd = bank.route_topk_device(dq, topk=5, warmup=2)
    assert np.array_equal(host_ids, dev_ids)
    assert rh.measured_queries == 4 and rd.measured_queries == 4
    assert np.all((host_ids - 11) % 3 == 0)
    dq.close()
    bank.close()


def test_async_route_with_offsets_and_merge(sidecar):
    import torch

    from graftrepository_b200 import _lib

    rows = synth.mla_bank(8, 50000)
    qs = synth.mla_queries(8, 4)
    halves = [rows[:20000], rows[20000:]]
    banks = [sidecar.create_bank_raw(h, 1) for h in halves]
    dq = torch.from_numpy(qs).cuda()
    k = 7
    sc = torch.empty((2, 4, k), dtype=torch.float32, device="cuda")
    ids = torch.empty((2, 4, k), dtype=torch.int64, device="cuda")
    for r, (b, off) in enumerate(zip(banks, (0, 20000))):
        b.reserve(4)
        b.route_async(dq.data_ptr(), 4, k, ids[r].data_ptr(), sc[r].data_ptr(),
                      torch.cuda.current_stream().cuda_stream, off)
    out_s = torch.empty((4, k), dtype=torch.float32, device="cuda")
    out_i = torch.empty((4, k), dtype=torch.int64, device="cuda")
    rc = _lib.load().grm_b200_merge_topk(sc.data_ptr(), ids.data_ptr(), 4, 2, k, k,
                                         out_s.data_ptr(), out_i.data_ptr(),
                                         torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    rows32 = rows.astype(np.float32)
    for i, q in enumerate(qs):
        want, want_s = O.mla_route(rows32, q, k)
        assert out_i[i].cpu().numpy().view(np.uint64).tolist() == want.tolist()
        assert np.array_equal(out_s[i].cpu().numpy(), want_s)
    for b in banks:
        b.close()


def test_full_size_config2(sidecar):
    """1,048,576 x 256 fp16 centroids (config 2): batch 1 and a batch of 64."""
    import torch

    n = 1 << 20
    rows16 = synth.mla_bank(1, n)
    qs = synth.mla_queries(1, 64)
    bank = sidecar.create_bank_raw(rows16, 1)
    ids, _ = bank.route_topk(qs, topk=3)
    rows = rows16.astype(np.float32)
    norms = O.mla_row_norms(rows)
    for i in list(range(4)) + [63]:
        want, want_s = O.mla_route(rows, qs[i], 3, norms=norms)
        assert np.array_equal(ids[i], want), i
        assert np.array_equal(bank.last_scores[i], want_s), i
    # size-independent properties over the whole batch
    s = bank.last_scores
    assert np.all(np.diff(s, axis=1) <= 0)
    assert np.all(ids < n)
    bank.close()
    torch.cuda.synchronize()


def test_async_route_resolves_ties_after_scan(sidecar):
    """The programmatic-dependent resolve kernel handles a saturated margin."""
    import torch

    rng = np.random.default_rng(44)
    base = rng.standard_normal((2, 256)).astype(np.float16)
    rows = np.repeat(base, 5000, axis=0)
    bank = sidecar.create_bank_raw(rows, 1)
    bank.reserve(2)
    qs = base.astype(np.float32)
    dq = torch.from_numpy(qs).cuda()
    ids = torch.empty((2, 6), dtype=torch.int64, device="cuda")
    sc = torch.empty((2, 6), dtype=torch.float32, device="cuda")
    bank.route_async(dq.data_ptr(), 2, 6, ids.data_ptr(), sc.data_ptr(),
                     torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    rows32 = rows.astype(np.float32)
    for i in range(2):
        want, want_s = O.mla_route(rows32, qs[i], 6)
        assert ids[i].cpu().numpy().view(np.uint64).tolist() == want.tolist()
        assert np.array_equal(sc[i].cpu().numpy(), want_s)
    bank.close()


def test_config1_exact_recipe(sidecar):
    """BASELINE config 1 as written (default_rng(0), 10,000 x 256 fp16
    unit rows, the query the generator's next draw, top-3): ids and scores
    against the oracle and ids against the reference runtime itself."""
    rows16, qs = synth.mla_config(0, 10_000)
    rows = rows16.astype(np.float32)
    bank = sidecar.create_bank(rows)
    assert bank.dtype == 1
    ids, scores = raw_route(bank, qs, 3)
    want, want_s = O.mla_route(rows, qs[0], 3)
    assert np.array_equal(ids[0], want)
    assert np.array_equal(scores[0], want_s)
    if O.ref_available():
        with O.RefStore().load_mla(rows) as st:
            assert [int(x) for x in ids[0]] == st.route(qs[0], 3)
    bank.close()
