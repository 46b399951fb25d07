"""Batched MLA route (tensor-core path, top-k <= 16) parity on the GPU, through
the C ABI, against the CPU oracle: ids and scores bit-exact for batches of
2..130 queries, including chunking past 64 queries, queries outside the batch
path's safe range, margin-saturating ties, banks that cannot be batched and the
async entry."""

import numpy as np
import pytest

import oracle as O
from graftrepository_b200 import _lib, synth
from graftrepository_b200.cuda_router import CudaMLARouteSidecar

pytestmark = pytest.mark.gpu
U64MAX = np.iinfo(np.uint64).max


@pytest.fixture(scope="module")
def sidecar():
    return CudaMLARouteSidecar(device=0)


def raw_route(bank, qs, k):
    q = np.ascontiguousarray(qs, dtype=np.float32).reshape(-1, bank.dim)
    ids, scores, _, _ = bank._route_raw(_lib.load().grm_b200_mla_route, q.ctypes.data,
                                        q.shape[0], k, 0)
    return ids, scores


def check(bank, rows, qs, k):
    ids, scores = raw_route(bank, qs, k)
    norms = O.mla_row_norms(rows)
    for i, q in enumerate(qs):
        want, want_s = O.mla_route(rows, q, k, norms=norms)
        assert np.array_equal(ids[i], want), (i, ids[i], want)
        fin = want != U64MAX
        assert np.array_equal(scores[i][fin], want_s[fin]), (i, scores[i], want_s)


@pytest.mark.parametrize("dim", [64, 128, 256])
@pytest.mark.parametrize("n,nq", [(3000, 2), (70001, 64), (40000, 130)])
def test_batch_matches_oracle(sidecar, dim, n, nq):
    rows = synth.mla_bank(dim + n, n, dim).astype(np.float32)
    qs = synth.mla_queries(n + 7, nq, dim)
    bank = sidecar.create_bank(rows)
    assert bank.paths()["batch"]
    for k in (1, 3, 16):
        check(bank, rows, qs, k)
    bank.close()


def test_batch_equals_single_query_routes(sidecar):
    rows = synth.mla_bank(21, 120000).astype(np.float32)
    qs = synth.mla_queries(22, 40)
    bank = sidecar.create_bank(rows)
    ids_b, s_b = raw_route(bank, qs, 8)
    for i in range(0, 40, 7):
        ids_1, s_1 = raw_route(bank, qs[i:i + 1], 8)
        assert np.array_equal(ids_b[i], ids_1[0])
        assert np.array_equal(s_b[i], s_1[0])
    bank.close()


def test_batch_unsafe_queries_take_the_exact_path(sidecar):
    rows = synth.mla_bank(31, 5000).astype(np.float32)
    qs = synth.mla_queries(32, 8)
    qs[0] = 0.0
    qs[1] *= 1e-4          # |q| below the batch path's 2^-8
    qs[2, 5] = np.nan
    qs[3] *= 1e25          # |q| above the safe range
    bank = sidecar.create_bank(rows)
    check(bank, rows, qs, 5)
    assert bank.stats()[1] >= 4
    bank.close()


def test_batch_ties_force_the_exact_fallback(sidecar):
    rng = np.random.default_rng(33)
    base = rng.standard_normal((3, 128)).astype(np.float32)
    rows = np.repeat(base, 2000, axis=0).astype(np.float16).astype(np.float32)
    qs = np.stack([base[1], base[2], base[0] + 0.01]).astype(np.float32)
    bank = sidecar.create_bank(rows)
    assert bank.paths()["batch"]
    check(bank, rows, qs, 16)
    assert bank.stats()[1] >= 2
    bank.close()


def test_small_norm_rows_disable_the_batch_path(sidecar):
    rows = synth.mla_bank(34, 4000, 128).astype(np.float32)
    rows[17] *= 0.25       # norm 0.25 < 1/2: outside the batch path's proven range
    rows[18] = 0.0
    qs = synth.mla_queries(35, 5, 128)
    bank = sidecar.create_bank(rows)
    assert not bank.paths()["batch"] and bank.paths()["bulk"]
    check(bank, rows, qs, 4)
    bank.close()


@pytest.mark.parametrize("n,k,valid", [(40, 32, 32), (12, 16, 10)])
def test_batch_nan_rows_and_sentinels(sidecar, n, k, valid):
    """k <= 16 runs on the tensor-core path, k = 32 loops the single-query scan."""
    rows = synth.mla_bank(36, n).astype(np.float32)
    rows[3, 1] = np.nan
    rows[9, 0] = np.inf
    qs = synth.mla_queries(37, 3)
    bank = sidecar.create_bank(rows)
    assert bank.paths()["batch"]
    ids, scores = raw_route(bank, qs, k)
    for i, q in enumerate(qs):
        want, want_s = O.mla_route(rows, q, k)
        assert np.array_equal(ids[i], want)
        assert np.sum(ids[i] != U64MAX) == valid
        fin = want != U64MAX
        assert np.array_equal(scores[i][fin], want_s[fin])
    bank.close()


def test_batch_async_entry_with_offset(sidecar):
    import torch

    rows16 = synth.mla_bank(38, 90000)
    qs = synth.mla_queries(39, 64)
    bank = sidecar.create_bank_raw(rows16, 1)
    bank.reserve(64)
    dq = torch.from_numpy(qs).cuda()
    k = 5
    ids = torch.empty((64, k), dtype=torch.int64, device="cuda")
    sc = torch.empty((64, k), dtype=torch.float32, device="cuda")
    bank.route_async(dq.data_ptr(), 64, k, ids.data_ptr(), sc.data_ptr(),
                     torch.cuda.current_stream().cuda_stream, 5000)
    torch.cuda.synchronize()
    got = ids.cpu().numpy().view(np.uint64)
    rows = rows16.astype(np.float32)
    norms = O.mla_row_norms(rows)
    for i in (0, 1, 31, 32, 63):
        want, want_s = O.mla_route(rows, qs[i], k, norms=norms)
        assert np.array_equal(got[i], want + 5000)
        assert np.array_equal(sc[i].cpu().numpy(), want_s)
    bank.close()
