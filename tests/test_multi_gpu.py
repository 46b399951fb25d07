"""Node-sharded route on 2+ GPUs (one process per GPU, NCCL all-gather, device
merge) equals the single-process reference route bit for bit.  Skipped on a
single GPU; NVLS is off (NCCL_NVLS_ENABLE=0) and no kernel reads peer memory."""

import os
import socket

import numpy as np
import pytest

import oracle as O
from graftrepository_b200 import synth

pytestmark = pytest.mark.gpu


def _ngpu():
    import torch
    return torch.cuda.device_count()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    import datetime

    import torch
    import torch.distributed as dist

    from graftrepository_b200.sharded import (ShardedGQARoute, ShardedMLARoute, gqa_shard_range,
                                              mla_shard_range)

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        rows = synth.mla_bank(51, 300_001)
        rows[1000:1010] = rows[5]                 # ties across the shard boundary region
        qs = synth.mla_queries(51, 4)
        a, b = mla_shard_range(rows.shape[0], world, rank)
        shard = torch.from_numpy(rows[a:b]).cuda()
        r = ShardedMLARoute(None, shard, a, 256, device=rank)
        ids, sc = r.route(torch.from_numpy(qs).cuda(), 5)
        mla = (ids.cpu().numpy().view(np.uint64), sc.cpu().numpy())
        r.close()

        lengths = synth.gqa_lengths(52, 300, "lognormal") // 4 + 1
        keys, off = synth.gqa_bank(52, lengths, kv_heads=8, dim=128)
        q = synth.gqa_query(52, q_heads=32, count=2)
        a, b = gqa_shard_range(off, world, rank)
        sub_off = (off[a:b + 1] - off[a]).astype(np.uint64)
        sub = torch.from_numpy(keys[int(off[a]) * 8 * 128:int(off[b]) * 8 * 128].view(np.int16))
        g = ShardedGQARoute(None, sub.cuda(), sub_off, a, 8, 128, device=rank)
        gids, gsc = g.route(torch.from_numpy(q).cuda(), 3)
        gqa = (gids.cpu().numpy().view(np.uint64), gsc.cpu().numpy())
        g.close()
        out[rank] = (mla, gqa)
    finally:
        dist.destroy_process_group()


def test_sharded_routes_equal_single_gpu_oracle():
    if _ngpu() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    world = min(_ngpu(), 4)
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _port(), out), nprocs=world, join=True)
    rows = synth.mla_bank(51, 300_001)
    rows[1000:1010] = rows[5]
    qs = synth.mla_queries(51, 4)
    rows32 = rows.astype(np.float32)
    lengths = synth.gqa_lengths(52, 300, "lognormal") // 4 + 1
    keys, off = synth.gqa_bank(52, lengths, kv_heads=8, dim=128)
    q = synth.gqa_query(52, q_heads=32, count=2)
    for rank in range(world):
        (mids, msc), (gids, gsc) = out[rank]
        for i, qq in enumerate(qs):
            want, want_s = O.mla_route(rows32, qq, 5)
            assert np.array_equal(mids[i], want)
            assert np.array_equal(msc[i], want_s)
        for i in range(2):
            want, want_s = O.gqa_route(keys, off, 8, 128, q[i], 3)
            assert np.array_equal(gids[i], want)
            assert np.array_equal(gsc[i], want_s)
