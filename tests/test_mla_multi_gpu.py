"""Multi-row MLA entries (a digest's centroid plus its child centroids,
core/graft_arena.py:1670-1684) on the GPU: an entry scores the max of its
finite rows (exact_mla_entry_score, cpp/grm_runtime.cpp:3518-3545).  Ids and
scores bit-exact against the oracle (pinned to the reference runtime in
test_oracle_pins.py)."""

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


def multi_bank(seed, entries, dim, max_rows=6):
    rng = np.random.default_rng(seed)
    counts = rng.integers(1, max_rows + 1, entries)
    counts[::11] = 1
    off = np.zeros(entries + 1, np.uint64)
    off[1:] = np.cumsum(counts)
    rows = synth.mla_bank(seed, int(off[-1]), dim).astype(np.float32)
    return rows, off


def check(bank, rows, off, qs, k):
    ids, rec = bank.route_topk(qs, topk=k)
    norms = O.mla_row_norms(rows)
    for i, q in enumerate(qs):
        want, want_s = O.mla_route_multi(rows, off, q, k, norms=norms)
        assert np.array_equal(ids[i], want), (i, ids[i], want)
        fin = want != U64MAX
        assert np.array_equal(bank.last_scores[i][fin], want_s[fin])


@pytest.mark.parametrize("dim,entries", [(64, 3000), (128, 20000), (256, 60000)])
def test_multi_row_entries_match_oracle(sidecar, dim, entries):
    rows, off = multi_bank(dim + entries, entries, dim)
    bank = sidecar.create_bank_multi(rows, off)
    qs = synth.mla_queries(entries + 1, 3, dim)
    for k in (1, 3, 16):
        check(bank, rows, off, qs, k)
    bank.close()


def test_multi_row_ties_nan_rows_and_unsafe_queries(sidecar):
    rows, off = multi_bank(77, 2000, 128)
    rows[int(off[5]):int(off[6])] = rows[int(off[2])]     # equal best rows: lower entry first
    rows[int(off[9]), 3] = np.nan
    rows[int(off[13]):int(off[14]), 0] = np.inf           # an entry with no finite row
    bank = sidecar.create_bank_multi(rows, off)
    qs = synth.mla_queries(78, 4, 128)
    qs[1] = rows[int(off[2])]
    qs[2] = 0.0                                            # outside the approximate pass
    qs[3] *= 1e25
    check(bank, rows, off, qs, 8)
    bank.close()


def test_multi_row_filters_and_lexical(sidecar):
    rows, off = multi_bank(79, 5000, 128)
    E = off.shape[0] - 1
    rng = np.random.default_rng(80)
    lex = [["hot"] if e % 9 == 0 else [f"k{int(x)}" for x in rng.integers(0, 50, 2)]
           for e in range(E)]
    kinds = [("digest" if e % 3 == 0 else "turn") for e in range(E)]
    bank = sidecar.create_bank_multi(rows, off)
    bank.set_route_policy(lexical_keys=lex, kinds=kinds)
    qs = synth.mla_queries(81, 2, 128)
    norms = O.mla_row_norms(rows)
    for qlex, kf in ((["hot"], ()), ([], ["digest"]), (["k3", "hot"], ["turn"])):
        ids, sc = bank.route_policy_topk(qs, topk=6, lexical_keys=[qlex, qlex], kinds=kf)
        for i, q in enumerate(qs):
            s = O.mla_scores(rows, q, norms)
            best = np.full(E, np.nan, np.float32)
            for e in range(E):
                seg = s[int(off[e]):int(off[e + 1])]
                seg = seg[np.isfinite(seg)]
                if seg.size:
                    best[e] = seg.max()
            m = len(qlex)
            if m:
                hits = np.array([O.lexical_hits(qlex, lex[e]) for e in range(E)], np.float32)
                best = (best + hits / np.float32(m)).astype(np.float32)
            else:
                best = (best + np.float32(0)).astype(np.float32)
            best[~O.route_allowed(E, [kinds, None, None, None], None, [list(kf) or None, None,
                                                                       None, None])] = np.nan
            want, want_s, _ = O.topk(best, 6)
            assert np.array_equal(ids[i], want), (qlex, kf, i)
            fin = want != U64MAX
            assert np.array_equal(sc[i][fin], want_s[fin])
    bank.close()


def test_multi_row_async_with_offset(sidecar):
    import torch

    rows, off = multi_bank(82, 8000, 256)
    bank = sidecar.create_bank_multi(rows, off)
    qs = synth.mla_queries(83, 3, 256)
    dq = torch.from_numpy(qs).cuda()
    ids = torch.empty((3, 5), dtype=torch.int64, device="cuda")
    sc = torch.empty((3, 5), dtype=torch.float32, device="cuda")
    bank.reserve(3)
    bank.route_async(dq.data_ptr(), 3, 5, ids.data_ptr(), sc.data_ptr(),
                     torch.cuda.current_stream().cuda_stream, 1000)
    torch.cuda.synchronize()
    got = ids.cpu().numpy().view(np.uint64)
    for i, q in enumerate(qs):
        want, want_s = O.mla_route_multi(rows, off, q, 5)
        assert np.array_equal(got[i], want + 1000)
        assert np.array_equal(sc[i].cpu().numpy(), want_s)
    bank.close()
