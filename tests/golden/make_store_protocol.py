"""Record how GraftRepository's own NativeGraftStore drives a CUDA route
sidecar, and what its CPU route answers, as a fixture the GPU tests replay
against this repository's sidecars.

Run where the GraftRepository checkout exists (the path in
oracle/reference_root, or GRM_REFERENCE_ROOT) after ``make -C oracle ref``:

    python tests/golden/make_store_protocol.py

The reference store is core/grm_native.py's NativeGraftStore over the
reference runtime compiled from cpp/grm_runtime.cpp (oracle/_ref/libgrm_ref.so,
loaded through GRM_RUNTIME_LIB, core/grm_native.py:148-149).  Its CUDA seam
takes an injected sidecar (configure_cuda_mla_route_bank /
configure_cuda_gqa_route_bank, core/grm_native.py:1498-1531, :1590-1624) and
then calls ``bank.route_topk`` (route_mla_cuda / route_gqa_cuda, :1542-1563,
:1635-1648).  A recording sidecar stands in for the CUDA one here: it keeps
every argument the store passes, answers each route with the store's own CPU
route (grm_store_route / grm_store_route_gqa), and raises RuntimeError where
the reference sidecar raises on its UINT64_MAX sentinel
(core/grm_cuda_router.py:465-475).  Written to tests/golden/store_protocol.npz:

* ``<case>_bank`` / ``<case>_node_ids`` / ``<case>_bank_kwargs``: the
  create_bank call the store made (route bank as passed, node ids, keyword
  names), and ``<case>_signature``: the reference's bank signature
  (mla_route_bank_signature / gqa_route_bank_signature);
* ``<case>_q<i>``, ``<case>_q<i>_kw`` (topk, warmup, route_repeats) and
  ``<case>_q<i>_want``: each route_topk call and the store's result, where
  ``want`` is the list route_mla_cuda / route_gqa_cuda returned, or
  ``[-1]`` when the call raised RuntimeError (the sentinel law);
* ``<case>_row_token_counts``: for the ragged GQA case, the padding receipt
  of the arena's dense bank (core/graft_arena.py:3026-3041).
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

import oracle as O  # noqa: E402

REF = O.reference_root()
sys.path.insert(0, str(REF))
os.environ["GRM_RUNTIME_LIB"] = str(O.oracle.REF_LIB_PATH)


class RecordingBank:
    def __init__(self, rec, answer):
        self.rec, self.answer = rec, answer
        self.signature = None

    def route_topk(self, queries, *, topk, warmup=0, route_repeats=1):
        q = np.ascontiguousarray(queries, dtype=np.float32)
        self.rec["calls"].append((q.copy(), {"topk": int(topk), "warmup": int(warmup),
                                             "route_repeats": int(route_repeats)}))
        single = q.ndim == (1 if self.rec["kind"] == "mla" else 3)
        batch = q[None] if single else q
        rows = []
        for one in batch:
            ids = self.answer(one, int(topk))
            if len(ids) < int(topk):
                raise RuntimeError("CUDA route returned an out-of-range row ID")
            rows.append(ids)
        return np.asarray(rows, dtype=np.uint64), None

    def close(self):
        pass


class RecordingSidecar:
    def __init__(self, kind, answer):
        self.rec = {"kind": kind, "calls": []}
        self.answer = answer

    def create_bank(self, route_bank, node_ids=None, **kwargs):
        self.rec["bank"] = np.ascontiguousarray(route_bank, dtype=np.float32).copy()
        self.rec["node_ids"] = np.ascontiguousarray(node_ids, dtype=np.uint64).copy()
        self.rec["bank_kwargs"] = sorted(kwargs)
        return RecordingBank(self.rec, self.answer)

    def close(self):
        pass


def mla_case(out):
    from core.grm_cuda_router import mla_route_bank_signature
    from core.grm_native import NativeGraftStore

    rng = np.random.default_rng(71)
    n, dim = 600, 256
    rows = rng.standard_normal((n, dim)).astype(np.float32)
    rows /= np.linalg.norm(rows, axis=1, keepdims=True)
    rows = rows.astype(np.float16).astype(np.float32)      # the harvested latents are fp16
    rows[40] = rows[12]                                      # a tie pair
    rows[41] = rows[12]
    rows[77, 5] = np.nan                                     # a bad row: dropped by the law
    store = NativeGraftStore(model_type="MiniCPM3_TC", num_layers=62, hidden_dim=2560,
                             vals_per_tok_layer=288, route_layer=0, payload_kind="mla",
                             latent_rank=256, rope_dim=32)
    ids = []
    for i in range(n):
        nid = store.add_node(f"graft {i}", b"", ntok=1)
        store.set_route(nid, rows[i])
        ids.append(nid)
    node_ids = np.asarray(ids, dtype=np.uint64)
    sc = RecordingSidecar("mla", lambda q, k: store.route(q, topk=k))
    store.configure_cuda_mla_route_bank(rows, node_ids, sidecar=sc)
    qs = rng.standard_normal((4, dim)).astype(np.float32)
    qs[1] = rows[12]                                         # the tie group first
    qs[2] = 0.0                                              # a zero query
    calls = [(qs[0], 3), (qs[1], 5), (qs[2], 3), (qs[3], 16), (qs[0] * np.nan, 3)]
    wants = []
    for q, k in calls:
        try:
            wants.append(store.route_mla_cuda(q, topk=k))
        except RuntimeError:
            wants.append([-1])
    _save(out, "mla", sc.rec, wants, mla_route_bank_signature(rows, node_ids))
    store.close()


def _gqa_dense(rows):
    """The arena's dense zero-padded bank and its row_token_counts receipt
    (core/graft_arena.py:2980-3042, restated: graft_arena imports tensor_cuda,
    which is not vendored)."""
    counts = [int(r.shape[1]) for r in rows]
    kh, d = rows[0].shape[0], rows[0].shape[2]
    bank = np.zeros((len(rows), kh, max(counts), d), dtype=np.float32)
    for i, r in enumerate(rows):
        bank[i, :, : r.shape[1]] = r
    return bank, counts


def gqa_case_ragged(out):
    from core.grm_cuda_router import gqa_route_bank_signature
    from core.grm_native import NativeGraftStore

    rng = np.random.default_rng(72)
    kh, d, h = 8, 128, 32
    lengths = rng.integers(1, 40, 50)
    rows = [O.bf16_bits_to_f32(O.f32_to_bf16_bits(
        rng.standard_normal((kh, int(t), d)).astype(np.float32))).reshape(kh, int(t), d)
        for t in lengths]
    rows[9] = rows[3].copy()                                 # a tie pair (same keys)
    lengths[9] = lengths[3]
    store = NativeGraftStore(model_type="Qwen3_TC", num_layers=36, hidden_dim=2560,
                             vals_per_tok_layer=2048, route_layer=0, payload_kind="gqa",
                             num_kv_heads=kh, head_dim=d)
    ids = []
    for i, r in enumerate(rows):
        nid = store.add_node(f"gqa graft {i}", b"", ntok=int(r.shape[1]))
        store.set_route_key_list(nid, [r], [])
        ids.append(nid)
    node_ids = np.asarray(ids, dtype=np.uint64)
    bank, counts = _gqa_dense(rows)
    sc = RecordingSidecar("gqa", lambda q, k: store.route_gqa(q, topk=k))
    sig = gqa_route_bank_signature(bank, node_ids)
    store.configure_cuda_gqa_route_bank(bank, node_ids, sidecar=sc, signature=sig)
    qs = rng.standard_normal((3, h, 1, d)).astype(np.float32)
    q4 = rng.standard_normal((h, 4, d)).astype(np.float32)
    calls = [(qs[0], 3), (qs[1], 5), (q4, 4), (qs[2], 16), (qs[2] * np.nan, 3)]
    wants = []
    for q, k in calls:
        try:
            wants.append(store.route_gqa_cuda(q, topk=k))
        except RuntimeError:
            wants.append([-1])
    _save(out, "gqa", sc.rec, wants, sig)
    out["gqa_row_token_counts"] = np.asarray(counts, dtype=np.int64)
    store.close()


def _save(out, case, rec, wants, signature):
    out[f"{case}_bank"] = rec["bank"]
    out[f"{case}_node_ids"] = rec["node_ids"]
    out[f"{case}_bank_kwargs"] = np.asarray(json.dumps(rec["bank_kwargs"]))
    out[f"{case}_signature"] = np.asarray(signature)
    out[f"{case}_ncalls"] = np.asarray(len(rec["calls"]))
    for i, ((q, kw), want) in enumerate(zip(rec["calls"], wants)):
        out[f"{case}_q{i}"] = q
        out[f"{case}_q{i}_kw"] = np.asarray(json.dumps(kw))
        out[f"{case}_q{i}_want"] = np.asarray(want, dtype=np.int64)


def main():
    O.ensure_built(with_ref=True)
    out = {}
    mla_case(out)
    gqa_case_ragged(out)
    np.savez_compressed(HERE / "store_protocol.npz", **out)
    print("wrote", HERE / "store_protocol.npz")


if __name__ == "__main__":
    main()
