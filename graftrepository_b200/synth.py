"""Seeded synthetic route banks and grafts with the benchmark configs' shapes.

The reference measures on real harvested banks that are not in this checkout,
so tests and the benchmark use these generators instead:

* MLA centroid banks (configs 1-2): rows N(0,1) fp32, L2-normalised per row in
  fp32, stored fp16; queries N(0,1) fp32.
* Ragged GQA banks (configs 3-4): per-node token counts uniform 16..1024 or
  lognormal(ln 192, 0.8) clipped to 8..4096; keys N(0,1) stored bf16 (round to
  nearest even), laid out per node [kv_heads, T_i, head_dim]; queries N(0,1).
* Grafts for the quantised mount (config 5): values N(0,1).

Small banks use numpy's default_rng(seed); banks too large for host memory are
drawn on the device with torch's seeded CUDA generator.
"""

from __future__ import annotations

import numpy as np

MLA_DIM = 256
GQA_LAYERS, GQA_KV_HEADS, GQA_Q_HEADS, GQA_DIM = 4, 8, 32, 128


def bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u.astype(np.uint64) + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    return np.where(nan, np.uint16(0x7FC0), r)


def mla_bank(seed: int, nodes: int, dim: int = MLA_DIM) -> np.ndarray:
    """fp16 [nodes, dim] unit-norm rows (configs 1-2)."""
    rng = np.random.default_rng(seed)
    rows = rng.standard_normal((nodes, dim), dtype=np.float32)
    rows /= np.linalg.norm(rows, axis=1, keepdims=True)
    return rows.astype(np.float16)


def mla_queries(seed: int, count: int, dim: int = MLA_DIM) -> np.ndarray:
    rng = np.random.default_rng(seed + 1000)
    return rng.standard_normal((count, dim), dtype=np.float32)


def mla_config(seed: int, nodes: int, queries: int = 1,
               dim: int = MLA_DIM) -> tuple[np.ndarray, np.ndarray]:
    """The configs' exact recipe from ONE generator: rng = default_rng(seed);
    rows N(0,1) fp32 [nodes, dim], L2-normalised per row in fp32, stored fp16;
    then the queries N(0,1) fp32 [queries, dim] as the generator's next draws
    (config 1: seed 0, 10,000 nodes, one query)."""
    rng = np.random.default_rng(seed)
    rows = rng.standard_normal((nodes, dim), dtype=np.float32)
    rows /= np.linalg.norm(rows, axis=1, keepdims=True)
    qs = rng.standard_normal((queries, dim), dtype=np.float32)
    return rows.astype(np.float16), qs


def mla_bank_device(seed: int, nodes: int, dim: int = MLA_DIM, device: str = "cuda"):
    """The same recipe drawn on the device (torch CUDA generator), fp16 tensor."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = torch.empty((nodes, dim), dtype=torch.float16, device=device)
    step = 1 << 18
    for a in range(0, nodes, step):
        b = min(nodes, a + step)
        x = torch.randn((b - a, dim), generator=g, device=device, dtype=torch.float32)
        x /= torch.linalg.vector_norm(x, dim=1, keepdim=True)
        out[a:b] = x.to(torch.float16)
    return out


def gqa_lengths(seed: int, nodes: int, kind: str = "uniform") -> np.ndarray:
    rng = np.random.default_rng(seed)
    if kind == "uniform":                  # config 3: U{16..1024}
        return rng.integers(16, 1025, nodes).astype(np.int64)
    if kind == "lognormal":                # config 4: lognormal(ln 192, 0.8) clipped 8..4096
        t = np.round(rng.lognormal(np.log(192.0), 0.8, nodes))
        return np.clip(t, 8, 4096).astype(np.int64)
    raise ValueError(kind)


def longest_plus_prefix(lengths: np.ndarray, longest: int, max_tokens: int) -> np.ndarray:
    """Node indices (ascending) of a checkable subset of a large ragged bank:
    the `longest` longest nodes (ties to the lower index) plus the longest
    contiguous prefix that keeps the subset within `max_tokens` tokens.  The
    tail of the length distribution (config 4's 4,096-token nodes) is then
    always part of the check."""
    t = np.asarray(lengths, dtype=np.int64)
    top = np.argsort(-t, kind="stable")[:longest]
    budget = max_tokens - int(t[top].sum())
    in_top = np.zeros(len(t), dtype=bool)
    in_top[top] = True
    extra = np.cumsum(np.where(in_top, 0, t))
    prefix = int(np.searchsorted(extra, budget, side="right"))
    keep = in_top.copy()
    keep[:prefix] = True
    return np.nonzero(keep)[0]


def offsets(lengths: np.ndarray) -> np.ndarray:
    off = np.zeros(len(lengths) + 1, dtype=np.uint64)
    off[1:] = np.cumsum(lengths)
    return off


def gqa_bank(seed: int, lengths: np.ndarray, kv_heads: int = GQA_LAYERS * GQA_KV_HEADS,
             dim: int = GQA_DIM) -> tuple[np.ndarray, np.ndarray]:
    """Host CSR bank: (bf16 bits uint16 [sum T * kv_heads * dim], offsets)."""
    rng = np.random.default_rng(seed + 7)
    off = offsets(lengths)
    n = int(off[-1]) * kv_heads * dim
    keys = np.empty(n, dtype=np.uint16)
    step = 1 << 26      # chunked draws: the same stream, a bounded temporary
    for a in range(0, n, step):
        b = min(n, a + step)
        keys[a:b] = bf16_bits(rng.standard_normal(b - a, dtype=np.float32))
    return keys, off


def gqa_bank_device(seed: int, lengths: np.ndarray, kv_heads: int = GQA_LAYERS * GQA_KV_HEADS,
                    dim: int = GQA_DIM, device: str = "cuda"):
    """Device CSR bank (bf16 tensor, flat) drawn with torch's CUDA generator."""
    import torch

    off = offsets(lengths)
    n = int(off[-1]) * kv_heads * dim
    g = torch.Generator(device=device)
    g.manual_seed(seed + 7)
    out = torch.empty(n, dtype=torch.bfloat16, device=device)
    step = 1 << 28
    for a in range(0, n, step):
        b = min(n, a + step)
        out[a:b] = torch.randn(b - a, generator=g, device=device, dtype=torch.float32).to(
            torch.bfloat16)
    return out, off


def gqa_query(seed: int, q_heads: int = GQA_LAYERS * GQA_Q_HEADS, q_tokens: int = 1,
              dim: int = GQA_DIM, count: int = 1) -> np.ndarray:
    rng = np.random.default_rng(seed + 2000)
    return rng.standard_normal((count, q_heads, q_tokens, dim), dtype=np.float32)


def grafts(seed: int, n_grafts: int = 3, layers: int = 62, tokens: int = 2048,
           width: int = 288) -> np.ndarray:
    """Config 5 graft values: fp32 [n_grafts, layers, tokens, width] N(0,1)."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal((n_grafts, layers, tokens, width), dtype=np.float32)


def seat_offsets(seed: int, n_grafts: int, tokens: int, arena_seats: int) -> np.ndarray:
    """Random non-overlapping runs of `tokens` seats in [0, arena_seats)."""
    rng = np.random.default_rng(seed + 99)
    free = arena_seats - n_grafts * tokens
    if free < 0:
        raise ValueError("arena too small")
    cuts = np.sort(rng.integers(0, free + 1, n_grafts))
    order = rng.permutation(n_grafts)
    seats = np.empty(n_grafts, dtype=np.int64)
    for rank, g in enumerate(order):
        seats[g] = cuts[rank] + rank * tokens
    return seats


ROUTE_KINDS = ("turn", "doc", "digest", "era", "fact", "task_state", "recall", "cull_span")


def route_policy(seed: int, nodes: int, vocab: int = 100_000, keys_per_node: int = 2):
    """Synthetic route policy data for a bank of `nodes` rows: each node
    carries `keys_per_node` lexical keys drawn Zipf-like from a vocabulary of
    `vocab` words ("w<rank>"), a kind cycling through the reference's known
    kinds, and 1 % inactive nodes.  Returns (lexical key lists, kinds, active)."""
    rng = np.random.default_rng(seed + 7)
    ranks = np.minimum(rng.zipf(1.3, size=(nodes, keys_per_node)), vocab) - 1
    lexical = [[f"w{r}" for r in row] for row in ranks.tolist()]
    kinds = [ROUTE_KINDS[i % len(ROUTE_KINDS)] for i in range(nodes)]
    active = rng.random(nodes) >= 0.01
    return lexical, kinds, active


def route_policy_query(seed: int, count: int = 3):
    """Query keys for a policy route (the arena's rare query tokens):
    `count - 1` words of Zipf rank 50..2000 (tens to a thousand nodes each at
    1M nodes) plus one key absent from the bank."""
    rng = np.random.default_rng(seed + 11)
    keys = [f"w{int(r)}" for r in rng.integers(50, 2000, count - 1)]
    return keys + ["absent-from-bank"]
