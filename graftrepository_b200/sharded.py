"""Node-range sharded route across 1-8 GPUs (one process per GPU).

The reference is single-process; its route is embarrassingly parallel over
nodes with one exchange step: each shard produces its local top-k with the
final reference-arithmetic score and the GLOBAL node row, the k candidates of
every shard are all-gathered (NCCL over NVLink; 8 x k x 12 bytes), and a
deterministic merge (score desc, row asc, non-finite dropped) gives the global
top-k.  Because every score is the exact per-node reference score, the merged
result equals the single-GPU route bit for bit.

Shard plans:
* MLA: equal contiguous node ranges.
* GQA: contiguous node ranges balanced by token count (CSR prefix sums), so a
  lognormal length distribution does not skew shard time.

``ShardedRoute`` holds the collective plumbing; the local route and the merge
are injected, so the same host logic runs with the sm_100a kernels and NCCL
on GPUs, and with CPU stand-ins over ``gloo`` in the host-logic tests.
"""

from __future__ import annotations

from typing import Callable

import numpy as np

U64MAX = np.iinfo(np.uint64).max

__all__ = ["mla_shard_range", "gqa_shard_range", "merge_topk_host", "ShardedRoute",
           "ShardedMLARoute", "ShardedGQARoute"]


def mla_shard_range(nodes: int, world: int, rank: int) -> tuple[int, int]:
    per = -(-nodes // world)
    a = min(nodes, rank * per)
    return a, min(nodes, a + per)


def gqa_shard_range(token_offsets, world: int, rank: int) -> tuple[int, int]:
    """Contiguous node range whose token count is ~1/world of the bank."""
    off = np.asarray(token_offsets, dtype=np.uint64)
    n = off.shape[0] - 1
    total = int(off[-1])
    cuts = [0]
    for r in range(1, world):
        target = (total * r) // world
        cuts.append(int(np.searchsorted(off, target, side="left")))
    cuts.append(n)
    cuts = np.maximum.accumulate(np.minimum(np.asarray(cuts), n))
    return int(cuts[rank]), int(cuts[rank + 1])


def merge_topk_host(scores: np.ndarray, ids: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """Host mirror of grm_b200_merge_topk: scores/ids [lists, Q, per] -> [Q, k]."""
    L, Q, P = scores.shape
    out_ids = np.full((Q, k), U64MAX, dtype=np.uint64)
    out_s = np.full((Q, k), np.nan, dtype=np.float32)
    for q in range(Q):
        s = scores[:, q, :].reshape(-1)
        i = ids[:, q, :].reshape(-1).astype(np.uint64)
        keep = np.isfinite(s) & (i != U64MAX)
        s, i = s[keep], i[keep]
        order = np.lexsort((i, -s.astype(np.float64)))[:k]
        out_ids[q, : order.size] = i[order]
        out_s[q, : order.size] = s[order]
    return out_ids, out_s


class ShardedRoute:
    """Local route -> one all-gather of (score, global row) candidates -> merge.

    ``local_route(queries, k) -> (scores [Q, k] float32, ids [Q, k] int64)`` (torch
    tensors on the process group's device; ids already global, UINT64_MAX as
    -1 for empty slots); ``merge(gathered_scores [W, Q, k], gathered_ids) ->
    (ids, scores)`` (the gathered views may be strided along W).  Scores and
    ids of a rank travel in one packed block of 16 bytes per entry (ids, then
    scores, then padding), so a route costs a single collective.  Subclasses
    may set ``local_into(queries, k, scores_out, ids_out)`` to write straight
    into the block.
    """

    local_into = None

    def __init__(self, group, local_route: Callable, merge: Callable):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.local_route = local_route
        self.merge = merge

    def route(self, queries, k: int):
        import torch

        Q = queries.shape[0]
        n = Q * k
        blk = torch.empty(16 * n, dtype=torch.uint8, device=queries.device)
        bi = blk[:8 * n].view(torch.int64).view(Q, k)
        bs = blk[8 * n:12 * n].view(torch.float32).view(Q, k)
        if self.local_into is not None:
            self.local_into(queries, k, bs, bi)
        else:
            scores, ids = self.local_route(queries, k)
            bs.copy_(scores)
            bi.copy_(ids)
        g = torch.empty(self.world * 16 * n, dtype=torch.uint8, device=queries.device)
        if self.world == 1:
            g.copy_(blk)
        else:
            self.dist.all_gather_into_tensor(g, blk, group=self.group)
        g2 = g.view(self.world, 16 * n)
        gi = g2[:, :8 * n].view(torch.int64).view(self.world, Q, k)
        gs = g2[:, 8 * n:12 * n].view(torch.float32).view(self.world, Q, k)
        return self.merge(gs, gi, k)


class ShardedMLARoute(ShardedRoute):
    """The MLA route over this rank's node range of a bank, on its GPU."""

    def __init__(self, group, rows_shard_device, first_row: int, dim: int, max_queries: int = 64,
                 device: int = 0, stream=None):
        import torch

        from . import _lib
        from .cuda_router import CudaMLARouteSidecar

        self.torch = torch
        self.first_row = int(first_row)
        self.bank = CudaMLARouteSidecar(device=device).create_bank_device(
            rows_shard_device.data_ptr(), 1 if rows_shard_device.dtype == torch.float16 else 0,
            rows_shard_device.shape[0], dim)
        self.bank.reserve(max_queries)
        self._lib = _lib.load()
        self.stream = stream
        super().__init__(group, self._local, self._merge)

    def _stream(self) -> int:
        s = self.stream or self.torch.cuda.current_stream()
        return int(s.cuda_stream)

    def _local(self, queries, k: int):
        torch = self.torch
        Q = queries.shape[0]
        s = torch.empty((Q, k), dtype=torch.float32, device=queries.device)
        i = torch.empty((Q, k), dtype=torch.int64, device=queries.device)
        self.local_into(queries, k, s, i)
        return s, i

    def local_into(self, queries, k: int, s, i):
        self.bank.route_async(queries.data_ptr(), queries.shape[0], k, i.data_ptr(), s.data_ptr(),
                              self._stream(), self.first_row)

    def _merge(self, gs, gi, k: int):
        torch = self.torch
        W, Q, P = gs.shape
        out_s = torch.empty((Q, k), dtype=torch.float32, device=gs.device)
        out_i = torch.empty((Q, k), dtype=torch.int64, device=gs.device)
        rc = self._lib.grm_b200_merge_topk_strided(gs.data_ptr(), gs.stride(0), gi.data_ptr(),
                                                   gi.stride(0), Q, W, P, k, out_s.data_ptr(),
                                                   out_i.data_ptr(), self._stream())
        if rc != 0:
            raise RuntimeError("merge_topk failed")
        return out_i, out_s

    def close(self) -> None:
        self.bank.close()


class ShardedGQARoute(ShardedRoute):
    """The ragged GQA route over this rank's token-balanced node range."""

    def __init__(self, group, keys_shard_device, token_offsets_shard, first_row: int,
                 kv_heads: int, head_dim: int, dtype_code: int = 2, device: int = 0,
                 stream=None):
        import torch

        from . import _lib
        from .cuda_router import CudaGQARouteSidecar

        self.torch = torch
        self.first_row = int(first_row)
        self.bank = CudaGQARouteSidecar(device=device).create_bank_device(
            keys_shard_device.data_ptr(), dtype_code, token_offsets_shard, kv_heads, head_dim,
            keepalive=keys_shard_device)
        self._lib = _lib.load()
        self.stream = stream
        super().__init__(group, self._local, self._merge)

    def _stream(self) -> int:
        s = self.stream or self.torch.cuda.current_stream()
        return int(s.cuda_stream)

    def _local(self, queries, k: int):
        """queries: device fp32 [Q, H, qt, D]."""
        torch = self.torch
        Q = queries.shape[0]
        s = torch.empty((Q, k), dtype=torch.float32, device=queries.device)
        i = torch.empty((Q, k), dtype=torch.int64, device=queries.device)
        self.local_into(queries, k, s, i)
        return s, i

    def local_into(self, queries, k: int, s, i):
        Q, H, qt, _ = queries.shape
        rc = self._lib.grm_b200_gqa_route_async(self.bank._h, queries.data_ptr(), Q, H, qt, k,
                                                self.first_row, i.data_ptr(), s.data_ptr(),
                                                self._stream())
        if rc != 0:
            raise RuntimeError(self.bank._err())

    _merge = ShardedMLARoute._merge

    def close(self) -> None:
        self.bank.close()
