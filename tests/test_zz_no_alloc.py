"""The allocation-free MLA route (grm_b200_mla_route_noalloc) against the CPU
oracle and the bank entry point (grm_b200_mla_route).

Callers that cannot allocate device memory while routing -- an engine whose
pool owns all of HBM, a route issued during CUDA-graph capture, a decode loop
that cannot take an allocation's implicit synchronisation -- pass their own
fp16 rows, queries and output buffers and the library works in a fixed scratch
array.  This file is collected last so that a run stopping at the first failure
has already run every other test; it passes alone in a fresh process too.

Ids and scores must equal the oracle's (and the bank route's) exactly -- the
tolerance of every parity test here: bit-exact -- on two calls in a row,
because the shared scratch keeps the previous call's contents.
"""

import numpy as np
import pytest

import oracle as O
from graftrepository_b200 import _lib, synth
from graftrepository_b200.cuda_router import CudaMLARouteSidecar

pytestmark = pytest.mark.gpu
U64MAX = np.iinfo(np.uint64).max


def _noalloc(rows_t, q_t, k):
    import torch

    lib = _lib.load()
    nq = q_t.shape[0]
    ids = torch.full((nq, k), -7, dtype=torch.int64, device="cuda")
    sc = torch.full((nq, k), -7.0, dtype=torch.float32, device="cuda")
    rc = lib.grm_b200_mla_route_noalloc(rows_t.data_ptr(), rows_t.shape[0], rows_t.shape[1],
                                        q_t.data_ptr(), nq, k, ids.data_ptr(), sc.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.thread_error()
    torch.cuda.synchronize()
    return ids.cpu().numpy().view(np.uint64), sc.cpu().numpy()


def _bank_route(rows16, qs, k):
    bank = CudaMLARouteSidecar(device=0).create_bank_raw(rows16, 1)
    ids, scores, _, _ = bank._route_raw(_lib.load().grm_b200_mla_route,
                                        np.ascontiguousarray(qs).ctypes.data, qs.shape[0], k, 0)
    bank.close()
    return ids, scores


def _oracle(rows16, qs, k, norms=None):
    rows = rows16.astype(np.float32)
    if norms is None:
        norms = O.mla_row_norms(rows)
    out = [O.mla_route(rows, q, k, norms=norms) for q in qs]
    return np.stack([o[0] for o in out]), np.stack([o[1] for o in out])


def _banks():
    rng = np.random.default_rng(31)
    tie = np.repeat(rng.standard_normal((3, 128)).astype(np.float32), 700, axis=0)
    tie_q = tie[:2].copy()
    tie_q[1] = tie[1000]
    return [
        ("random_256", synth.mla_bank(17, 200_003), synth.mla_queries(17, 5)),
        ("ties_128", tie.astype(np.float16), tie_q.astype(np.float16).astype(np.float32)),
        ("small_64", synth.mla_bank(18, 40, 64), synth.mla_queries(18, 3, 64)),
    ]


def _same(ids, scores, want_ids, want_scores):
    assert np.array_equal(ids, want_ids)
    fin = want_ids != U64MAX
    assert np.array_equal(scores[fin], want_scores[fin])
    assert np.all(np.isnan(scores[~fin]))


@pytest.mark.parametrize("case", range(3))
def test_noalloc_matches_oracle_and_bank_route_twice(case):
    import torch

    name, rows16, qs = _banks()[case]
    if name == "random_256":
        qs[1] = 0.0                      # a query outside the fast path's safe range
    k = 5 if name != "small_64" else 32
    want_ids, want_scores = _oracle(rows16, qs, k)
    bank_ids, bank_scores = _bank_route(rows16, qs, k)
    _same(bank_ids, bank_scores, want_ids, want_scores)
    rows_t = torch.from_numpy(rows16).cuda()
    q_t = torch.from_numpy(qs).cuda()
    for call in range(2):
        ids, scores = _noalloc(rows_t, q_t, k)
        _same(ids, scores, want_ids, want_scores)


def test_noalloc_sixteen_queries_on_a_large_bank():
    """The documented maximum (16 queries) on a bank of about a million rows:
    the grid narrows so that every query's scratch fits in the fixed array."""
    import torch

    n = 1_000_003
    rows16 = synth.mla_bank(19, n)
    qs = synth.mla_queries(19, 16)
    rows_t = torch.from_numpy(rows16).cuda()
    q_t = torch.from_numpy(qs).cuda()
    ids, scores = _noalloc(rows_t, q_t, 3)
    norms = O.mla_row_norms(rows16.astype(np.float32))
    for i in (0, 7, 15):
        want, want_s = _oracle(rows16, qs[i:i + 1], 3, norms=norms)
        _same(ids[i:i + 1], scores[i:i + 1], want, want_s)
    bank_ids, bank_scores = _bank_route(rows16, qs, 3)
    _same(ids, scores, bank_ids, bank_scores)
    ids2, scores2 = _noalloc(rows_t, q_t, 3)
    _same(ids2, scores2, bank_ids, bank_scores)


def test_noalloc_rejects_oversized_requests():
    import torch

    lib = _lib.load()
    rows = torch.zeros((64, 256), dtype=torch.float16, device="cuda")
    q = torch.zeros((17, 256), dtype=torch.float32, device="cuda")
    ids = torch.zeros((17, 3), dtype=torch.int64, device="cuda")
    sc = torch.zeros((17, 3), dtype=torch.float32, device="cuda")
    rc = lib.grm_b200_mla_route_noalloc(rows.data_ptr(), 64, 256, q.data_ptr(), 17, 3,
                                        ids.data_ptr(), sc.data_ptr(), 0)
    assert rc == -1 and "at most 16" in _lib.thread_error()
    rc = lib.grm_b200_mla_route_noalloc(rows.data_ptr(), 64, 96, q.data_ptr(), 1, 3,
                                        ids.data_ptr(), sc.data_ptr(), 0)
    assert rc == -1 and "dim" in _lib.thread_error()


def test_noalloc_rejects_misaligned_pointers():
    """An offset view into a caller's pool is refused before any launch."""
    import torch

    lib = _lib.load()
    pool = torch.zeros(64 * 256 + 8, dtype=torch.float16, device="cuda")
    q = torch.zeros((2, 256), dtype=torch.float32, device="cuda")
    ids = torch.zeros((2, 4), dtype=torch.int64, device="cuda")
    sc = torch.zeros((2, 4), dtype=torch.float32, device="cuda")
    rows_off = pool.data_ptr() + 2                # 2-byte offset: not 16-byte aligned
    rc = lib.grm_b200_mla_route_noalloc(rows_off, 64, 256, q.data_ptr(), 1, 3,
                                        ids.data_ptr(), sc.data_ptr(), 0)
    assert rc == -1 and "aligned" in _lib.thread_error()
    rc = lib.grm_b200_mla_route_noalloc(pool.data_ptr(), 64, 256, q.data_ptr() + 2, 1, 3,
                                        ids.data_ptr(), sc.data_ptr(), 0)
    assert rc == -1 and "aligned" in _lib.thread_error()
    rc = lib.grm_b200_mla_route_noalloc(pool.data_ptr(), 64, 256, q.data_ptr(), 1, 3,
                                        ids.data_ptr() + 4, sc.data_ptr(), 0)
    assert rc == -1 and "aligned" in _lib.thread_error()
    torch.cuda.synchronize()                      # nothing was launched; the context is fine
    assert (ids == 0).all().item()
