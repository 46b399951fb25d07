"""Host logic of the node-sharded route on CPU ranks (gloo, world size 2):
shard plans, the all-gather of per-shard candidates and the deterministic
merge reproduce the single-process route exactly; a rank that never reaches
the collective makes the others fail with an error instead of hanging."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from graftrepository_b200 import synth
from graftrepository_b200.sharded import (ShardedRoute, gqa_shard_range, merge_topk_host,
                                          mla_shard_range)

U64MAX = np.iinfo(np.uint64).max


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=60):
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _to_torch(ids, scores):
    return (torch.from_numpy(scores.astype(np.float32)),
            torch.from_numpy(ids.astype(np.uint64).view(np.int64)))


def _merge(gs, gi, k):
    ids, s = merge_topk_host(gs.numpy(), gi.numpy().view(np.uint64), k)
    return ids, s


def _mla_worker(rank, world, port, out):
    _init(rank, world, port)
    rows = synth.mla_bank(21, 3001).astype(np.float32)
    rows[100:160] = rows[7]                      # a tie group straddling nothing special
    qs = synth.mla_queries(21, 3)
    a, b = mla_shard_range(rows.shape[0], world, rank)

    def local(q, k):
        ids = np.full((q.shape[0], k), U64MAX, np.uint64)
        sc = np.full((q.shape[0], k), np.nan, np.float32)
        for i, qq in enumerate(q.numpy()):
            li, ls = O.mla_route(rows[a:b], qq, k)
            ok = li != U64MAX
            ids[i, ok] = li[ok] + a
            sc[i] = ls
        return _to_torch(ids, sc)

    r = ShardedRoute(None, local, _merge)
    ids, scores = r.route(torch.from_numpy(qs), 9)
    out[rank] = (ids, scores)
    dist.destroy_process_group()


def test_sharded_mla_merge_equals_global_route():
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(_mla_worker, args=(world, _port(), out), nprocs=world, join=True)
    rows = synth.mla_bank(21, 3001).astype(np.float32)
    rows[100:160] = rows[7]
    qs = synth.mla_queries(21, 3)
    for rank in range(world):
        ids, scores = out[rank]
        for i, q in enumerate(qs):
            want, want_s = O.mla_route(rows, q, 9)
            assert np.array_equal(ids[i], want)
            assert np.array_equal(scores[i], want_s)


def _gqa_worker(rank, world, port, out):
    _init(rank, world, port)
    lengths = synth.gqa_lengths(5, 60, "lognormal") // 8 + 1
    keys, off = synth.gqa_bank(5, lengths, kv_heads=4, dim=32)
    q = np.random.default_rng(3).standard_normal((1, 16, 1, 32)).astype(np.float32)
    a, b = gqa_shard_range(off, world, rank)
    sub_off = (off[a: b + 1] - off[a]).astype(np.uint64)
    sub_keys = keys[int(off[a]) * 4 * 32: int(off[b]) * 4 * 32]

    def local(qq, k):
        li, ls = O.gqa_route(sub_keys, sub_off, 4, 32, qq.numpy()[0], k)
        ok = li != U64MAX
        li = li.copy()
        li[ok] += a
        return _to_torch(li[None], ls[None])

    ids, scores = ShardedRoute(None, local, _merge).route(torch.from_numpy(q), 6)
    out[rank] = (ids, scores, a, b)
    dist.destroy_process_group()


def test_sharded_gqa_token_balanced_merge():
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(_gqa_worker, args=(world, _port(), out), nprocs=world, join=True)
    lengths = synth.gqa_lengths(5, 60, "lognormal") // 8 + 1
    keys, off = synth.gqa_bank(5, lengths, kv_heads=4, dim=32)
    q = np.random.default_rng(3).standard_normal((16, 1, 32)).astype(np.float32)
    want, want_s = O.gqa_route(keys, off, 4, 32, q, 6)
    assert out[0][2] == 0 and out[0][3] == out[1][2] and out[1][3] == 60
    for rank in range(world):
        assert np.array_equal(out[rank][0][0], want)
        assert np.array_equal(out[rank][1][0], want_s)


def test_shard_plans_cover_and_balance():
    for n, w in [(10, 3), (1 << 20, 8), (5, 8)]:
        spans = [mla_shard_range(n, w, r) for r in range(w)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(spans[i][1] == spans[i + 1][0] for i in range(w - 1))
    lengths = synth.gqa_lengths(3, 100_000, "lognormal")
    off = synth.offsets(lengths)
    spans = [gqa_shard_range(off, 8, r) for r in range(8)]
    assert spans[0][0] == 0 and spans[-1][1] == 100_000
    toks = [int(off[b] - off[a]) for a, b in spans]
    assert max(toks) / min(toks) < 1.01


def _dead_rank_worker(rank, world, port, out):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        os._exit(0)                                  # leaves between steps, no collective
    try:
        t = torch.zeros(4)
        g = torch.zeros(8)
        dist.all_gather_into_tensor(g, t)
        out[rank] = "completed"
    except Exception as exc:                          # noqa: BLE001
        out[rank] = "error:" + type(exc).__name__


def test_dead_rank_surfaces_as_error_not_hang():
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    ctx = mp.spawn(_dead_rank_worker, args=(world, _port(), out), nprocs=world, join=False)
    for p in ctx.processes:
        p.join(timeout=120)
    assert out.get(0, "").startswith("error:")
