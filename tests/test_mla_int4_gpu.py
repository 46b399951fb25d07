"""The reference's INT4 bulk/refine MLA route mode on the GPU
(grm_b200_mla_route_int4 / _async), against the CPU restatement of
route_mla_int4 (cpp/grm_runtime.cpp:4363-4482; pinned to the reference runtime
in tests/test_oracle_pins.py) and, where it was built, the reference runtime
itself with GRM_ROUTER_INT4=1.  Ids and exact scores must be bit-exact: the
mode's candidate set is decided by its INT4 bulk scores, so a single bulk
score rounded differently would change the answer."""

import os

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


def _raw(bank, qs, k, m):
    """Row ids + scores of the INT4 route without the sentinel raise."""
    import ctypes

    from graftrepository_b200 import _lib

    q = np.ascontiguousarray(qs, dtype=np.float32).reshape(-1, bank.dim)
    ids = np.empty((q.shape[0], k), dtype=np.uint64)
    sc = np.empty((q.shape[0], k), dtype=np.float32)
    ms = ctypes.c_float()
    rc = _lib.load().grm_b200_mla_route_int4(bank._h, q.ctypes.data, q.shape[0], bank.dim, k, m,
                                            ids.ctypes.data, sc.ctypes.data, ctypes.byref(ms))
    _lib.check(rc, bank._err)
    return ids, sc


def _check(bank, rows_f32, qs, k, m, norms=None):
    ids, sc = _raw(bank, qs, k, m)
    for i, q in enumerate(qs):
        want, want_s = O.mla_int4_route(rows_f32, q, k, refine_m=m, norms=norms)
        assert np.array_equal(ids[i], want), (i, k, m, ids[i], want)
        fin = want != U64MAX
        assert np.array_equal(sc[i][fin], want_s[fin]), (i, k, m)
        assert np.all(np.isnan(sc[i][~fin]))


@pytest.mark.parametrize("dim", [64, 128, 256, 512])
def test_random_banks(sidecar, dim):
    rows16 = synth.mla_bank(300 + dim, 30_011, dim)
    rows = rows16.astype(np.float32)
    qs = synth.mla_queries(300 + dim, 3, dim)
    bank = sidecar.create_bank(rows)
    for k, m in ((1, 4096), (3, 4096), (16, 16), (5, 1), (3, 40_000)):
        _check(bank, rows, qs, k, m)
    bank.close()


def test_edge_rows_and_queries(sidecar):
    """NaN / Inf / zero rows, duplicate rows, a zero query, a tiny query and a
    non-finite query (every bulk score NaN: nothing is routed)."""
    rows16, _ = synth.mla_config(61, 9_000)
    rows = rows16.astype(np.float32)
    rows[::101] = rows[3]
    rows[5, 1] = np.nan
    rows[6, 2] = np.inf
    rows[7] = 0.0
    qs = synth.mla_queries(61, 5)
    qs[1] = rows[3]
    qs[2] = 0.0
    qs[3] *= 1e-12
    qs[4, 9] = np.nan
    bank = sidecar.create_bank(rows)
    for k, m in ((3, 4096), (16, 50), (8, 8)):
        _check(bank, rows, qs, k, m)
    bank.close()


def test_fp32_bank(sidecar):
    """Values that fp16 cannot hold keep the bank fp32 (both the INT4 arena
    build and the exact refine read fp32 rows)."""
    rng = np.random.default_rng(65)
    rows = rng.standard_normal((7_000, 128)).astype(np.float32)
    qs = rng.standard_normal((3, 128)).astype(np.float32)
    bank = sidecar.create_bank(rows)
    assert bank.dtype == 0
    for k, m in ((3, 4096), (16, 100)):
        _check(bank, rows, qs, k, m)
    bank.close()


def test_ties_at_the_refine_boundary(sidecar):
    """Thousands of identical rows straddle the M-th bulk score: the lowest row
    ids win the remaining candidate slots (candidate_better)."""
    rng = np.random.default_rng(62)
    base = rng.standard_normal((4, 128)).astype(np.float32)
    rows = np.repeat(base, 3000, axis=0)
    rows = rows[rng.permutation(rows.shape[0])]
    rows = rows.astype(np.float16).astype(np.float32)
    qs = np.stack([base[1], base[2] + 0.1 * base[0]]).astype(np.float16).astype(np.float32)
    bank = sidecar.create_bank(rows)
    for k, m in ((16, 100), (5, 2999), (3, 3001), (32, 7000)):
        _check(bank, rows, qs, k, m)
    bank.close()


def test_against_the_reference_runtime(sidecar, monkeypatch):
    if not O.ref_available():
        pytest.skip("reference runtime not built")
    rows16 = synth.mla_bank(63, 20_000)
    rows = rows16.astype(np.float32)
    qs = synth.mla_queries(63, 3)
    bank = sidecar.create_bank(rows)
    monkeypatch.setenv("GRM_ROUTER_INT4", "1")
    for m in (64, 4096):
        monkeypatch.setenv("GRM_ROUTER_INT4_REFINE_M", str(m))
        ids, _ = _raw(bank, qs, 5, m)
        with O.RefStore().load_mla(rows) as st:
            for i, q in enumerate(qs):
                assert [int(x) for x in ids[i]] == st.route(q, 5), (m, i)
    bank.close()


def test_public_api_and_async_entry(sidecar):
    import torch

    rows16 = synth.mla_bank(64, 50_000)
    rows = rows16.astype(np.float32)
    qs = synth.mla_queries(64, 4)
    bank = sidecar.create_bank(rows, node_ids=np.arange(50_000, dtype=np.uint64) * 2 + 1)
    ids, receipt = bank.route_topk_int4(qs, topk=3)
    assert receipt.measured_queries == 4
    raw, sc = _raw(bank, qs, 3, 4096)
    assert np.array_equal(ids, raw * 2 + 1)
    assert np.array_equal(bank.last_scores, sc)
    dq = torch.from_numpy(qs).cuda()
    oi = torch.empty((4, 3), dtype=torch.int64, device="cuda")
    os_ = torch.empty((4, 3), dtype=torch.float32, device="cuda")
    bank.route_int4_async(dq.data_ptr(), 4, 3, oi.data_ptr(), os_.data_ptr(),
                          torch.cuda.current_stream().cuda_stream, id_offset=1000)
    torch.cuda.synchronize()
    assert np.array_equal(oi.cpu().numpy().view(np.uint64), raw + 1000)
    assert np.array_equal(os_.cpu().numpy(), sc)
    # the exact route on the same bank is unaffected by the INT4 arena
    ex_ids, _ = bank.route_topk(qs[:1], topk=3)
    want, _ = O.mla_route(rows, qs[0], 3)
    assert np.array_equal(ex_ids[0], want * 2 + 1)
    bank.close()


def test_full_size_config2(sidecar):
    """1,048,576 x 256 fp16 (config 2) in the INT4 mode with the reference's
    default refine set (4,096)."""
    n = 1 << 20
    rows16, qs = synth.mla_config(1, n, queries=3)
    bank = sidecar.create_bank_raw(rows16, 1)
    rows = rows16.astype(np.float32)
    norms = O.mla_row_norms(rows)
    ids, sc = _raw(bank, qs, 3, 4096)
    for i, q in enumerate(qs):
        want, want_s = O.mla_int4_route(rows, q, 3, refine_m=4096, norms=norms)
        assert np.array_equal(ids[i], want), i
        assert np.array_equal(sc[i], want_s), i
    bank.close()


def _permutation_bank(seed, n, dim):
    """Rows that are permutations of one integer vector (values -7..7, so the
    INT4 arena holds them exactly and every row has the same norm and norm
    scale): with a query whose values are all equal, every row's bulk dot is
    the same multiset of rounded products summed in a different order, so the
    bulk ranking -- and with it the refine set -- is decided by fp32 rounding
    alone.  A bulk pass that fused a multiply into an add, or summed in another
    order, picks a different set.  The exact scores all tie (the fp64 sums are
    exact), so the answer lists the refine set's lowest row ids."""
    rng = np.random.default_rng(seed)
    base = rng.integers(-7, 8, dim).astype(np.float32)
    base[0], base[1] = 7.0, -7.0
    rows = np.stack([base[rng.permutation(dim)] for _ in range(n)])
    return rows.astype(np.float16).astype(np.float32)


def test_bulk_rounding_order_decides_the_refine_set(sidecar):
    rows = _permutation_bank(66, 20_000, 256)
    q_const = np.full(256, 0.7317093, np.float32)
    q_alt = np.where(np.arange(256) % 3 == 0, -1.3371, 0.4142).astype(np.float32)
    qs = np.stack([q_const, q_alt])
    bank = sidecar.create_bank(rows)
    for k, m in ((1, 1), (3, 3), (16, 16), (5, 4096), (8, 19_000)):
        _check(bank, rows, qs, k, m)
    bank.close()
