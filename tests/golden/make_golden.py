"""Generate the committed golden vectors from the REFERENCE implementation.

Run in a container that has the GraftRepository checkout (the path in
oracle/reference_root, or GRM_REFERENCE_ROOT) and a C++ compiler:

    python tests/golden/make_golden.py [fixture ...]

Every expected output below is produced by the reference's own code:

* MLA / GQA route ids -- the reference's C++ RouterIndex, compiled from
  cpp/grm_runtime.cpp by oracle/Makefile and driven through its C ABI
  (grm_store_route cpp/grm_runtime.cpp:6767, grm_store_route_gqa :6898);
  the MLA ids are cross-checked against python_mla_reference_route
  (scripts/grm_mla_cuda_probe.py:814-832).
* MLA scores -- the python reference's own fp64 formula (same file :821-828).
* Quant codes / scales / fp16 dequant -- core/graft_quant.py
  (quantize_symmetric_group32 :93-133, dequantize_symmetric_group32 :136-144,
  pack_kv_arrays :177-217); the bf16 upload cast (core/graft_arena.py:3490)
  is stood in for by torch's fp16 -> bf16 conversion because tensor_cuda is
  not vendored.
* Arena splice -- DeviceArena::apply_swap_tensor (cpp/grm_runtime.cpp:4941)
  through grm_store_apply_swap_tensor.
* Packed payloads -- pack_kv_arrays (core/graft_quant.py:177-217) of an
  MLA-shaped node ({"c": [L, S, 256], "kpe": [L, S, 32]}, the payload of
  core/graft_arena.py:464-477) and a GQA-shaped one ({"k": [L, H, S, D]},
  :3459-3477), every field as pack_kv_arrays wrote it, with
  unpack_kv_arrays's fp16 output and its bf16 cast; plus payloads that
  unpack_kv_arrays rejects, each with the error it raised.

Inputs are seeded synthetic data with the configs' shapes at small sizes, plus
the edge cases the reference tests exercise (ties, non-finite rows, empty
ragged nodes, zero and non-finite queries).
"""

from __future__ import annotations

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


def mla_case(seed: int, n: int, dim: int, topk: int):
    from scripts.grm_mla_cuda_probe import python_mla_reference_route

    rng = np.random.default_rng(seed)
    rows = rng.standard_normal((n, dim)).astype(np.float32)
    rows /= np.linalg.norm(rows, axis=1, keepdims=True)
    rows16 = rows.astype(np.float16)
    # edge rows: exact duplicates (ties broken by lowest id), a zero row,
    # non-finite rows (dropped), a scaled copy (same cosine up to rounding)
    rows16[17] = rows16[5]
    rows16[40] = rows16[5]
    rows16[23] = 0
    rows16[31, 7] = np.float16(np.nan)
    rows16[32, 0] = np.float16(np.inf)
    rows16[50] = (rows16[60].astype(np.float32) * 2.0).astype(np.float16)
    qs = rng.standard_normal((7, dim)).astype(np.float32)
    qs[1] = rows16[5].astype(np.float32)            # top tie group {5, 17, 40}
    qs[2] = rows16[60].astype(np.float32) * 3.0     # near tie {50, 60}
    qs[3] = 0.0                                     # zero query: all scores 0
    qs[4, 3] = np.nan                               # non-finite query: empty
    qs[5] *= 1.0e-12                                # tiny query
    qs[6] *= 1.0e12                                 # huge query
    rows_f32 = rows16.astype(np.float32)
    ids = np.full((qs.shape[0], topk), np.iinfo(np.uint64).max, dtype=np.uint64)
    scores = np.full((qs.shape[0], topk), np.nan, dtype=np.float32)
    with O.RefStore().load_mla(rows_f32) as st:
        for i, q in enumerate(qs):
            got = st.route(q, topk)
            py = python_mla_reference_route(rows_f32, q, topk)
            assert got == py, (i, got, py)
            ids[i, : len(got)] = got
            qd = q.astype(np.float64)
            qn = float(np.sqrt(np.sum(qd * qd)))
            for j, nid in enumerate(got):
                r = rows_f32[nid].astype(np.float64)
                scores[i, j] = np.float32(float(np.dot(qd, r)) /
                                          (qn * float(np.sqrt(np.sum(r * r))) + 1.0e-8))
    return dict(rows_f16=rows16.view(np.uint16), queries=qs, topk=np.int64(topk),
                ids=ids, scores=scores)


def gqa_case(seed: int, n: int, kv_heads: int, q_heads: int, dim: int, tmax: int, topk: int):
    rng = np.random.default_rng(seed)
    T = rng.integers(1, tmax + 1, n)
    T[4] = 0              # empty ragged node: the reference scores it 0.0
    T[9] = 1
    off = np.zeros(n + 1, dtype=np.uint64)
    off[1:] = np.cumsum(T)
    keys = O.f32_to_bf16_bits(rng.standard_normal(int(off[-1]) * kv_heads * dim)
                              .astype(np.float32))

    def block(i):
        a, b = int(off[i]) * kv_heads * dim, int(off[i + 1]) * kv_heads * dim
        return slice(a, b)

    # node 12 duplicates node 20 (same T forced) -> exact tie, lowest id wins
    T12 = int(T[20])
    # rebuild with T[12] = T[20] so the blocks can be copied
    T[12] = T12
    off[1:] = np.cumsum(T)
    keys = O.f32_to_bf16_bits(rng.standard_normal(int(off[-1]) * kv_heads * dim)
                              .astype(np.float32))
    keys[block(12)] = keys[block(20)]
    keys[block(7).start + 11] = 0x7FC0      # NaN key -> node dropped
    q1 = rng.standard_normal((2, q_heads, 1, dim)).astype(np.float32)
    q4 = rng.standard_normal((1, q_heads, 4, dim)).astype(np.float32)
    qnan = rng.standard_normal((1, q_heads, 1, dim)).astype(np.float32)
    qnan[0, 3, 0, 5] = np.inf               # non-finite query: only T=0 nodes score
    out = {}
    with O.RefStore().load_gqa(keys, off, kv_heads, dim) as st:
        for name, qs in (("q1", q1), ("q4", q4), ("qnan", qnan)):
            ids = np.full((qs.shape[0], topk), np.iinfo(np.uint64).max, dtype=np.uint64)
            for i, q in enumerate(qs):
                got = st.route(q, topk)
                ids[i, : len(got)] = got
            out[name] = qs
            out[name + "_ids"] = ids
    return dict(keys_bf16=keys, token_offsets=off, kv_heads=np.int64(kv_heads),
                head_dim=np.int64(dim), topk=np.int64(topk), **out)


def quant_case(seed: int):
    import torch
    from core import graft_quant as GQ

    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((2, 3, 8, 96)) * 1.7).astype(np.float16)
    x[0, 0, 0, :32] = 0                      # all-zero group: scale 1
    out = {"x_f16": x.view(np.uint16)}
    for bits in (8, 6, 4, 3, 2):
        codes, scales = GQ.quantize_symmetric_group32(x, bits)
        dq = GQ.dequantize_symmetric_group32(codes, scales, x.shape)
        bf = torch.from_numpy(dq).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        payload = GQ.pack_kv_arrays({"k": x}, bits)
        assert np.array_equal(payload["k_codes"], codes)
        rt = GQ.unpack_kv_arrays(payload, ["k"])["k"]
        assert np.array_equal(rt.view(np.uint16), dq.view(np.uint16))
        out[f"codes{bits}"] = codes
        out[f"scales{bits}"] = scales
        out[f"dequant_f16_{bits}"] = dq.view(np.uint16)
        out[f"dequant_bf16_{bits}"] = bf
    return out


def packed_case(seed: int):
    import torch
    from core import graft_quant as GQ

    def bf16(x16):
        return torch.from_numpy(x16).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)

    rng = np.random.default_rng(seed)
    out = {}
    L, S = 3, 16
    c = (rng.standard_normal((L, S, 256)) * 0.8).astype(np.float16)
    kpe = (rng.standard_normal((L, S, 32)) * 2.5).astype(np.float16)
    c[1, 2, 32:64] = 0
    k = (rng.standard_normal((2, 4, 8, 64)) * 1.3).astype(np.float16)
    for tag, arrays, bits in (("mla8", {"c": c, "kpe": kpe}, 8), ("mla4", {"c": c, "kpe": kpe}, 4),
                              ("gqa6", {"k": k}, 6), ("gqa3", {"k": k}, 3)):
        payload = GQ.pack_kv_arrays(arrays, bits)
        rt = GQ.unpack_kv_arrays(payload, list(arrays))
        for key, val in payload.items():
            out[f"{tag}__{key}"] = np.asarray(val)
        for name in arrays:
            out[f"{tag}__expect_f16_{name}"] = rt[name].view(np.uint16)
            out[f"{tag}__expect_bf16_{name}"] = bf16(rt[name])
    # payloads unpack_kv_arrays rejects (fail-closed), with its error text
    base = GQ.pack_kv_arrays({"k": k}, 8)
    bad = {
        "noversion": {kk: v for kk, v in base.items() if kk != "format_version"},
        "version2": {**base, "format_version": np.asarray(2, dtype=np.int64)},
        "bits16": {**base, "storage_bits": np.asarray(16, dtype=np.int64)},
        "bits5": {**base, "storage_bits": np.asarray(5, dtype=np.int64)},
        "noscales": {kk: v for kk, v in base.items() if kk != "k_scales"},
        "vecversion": {**base, "format_version": np.asarray([1, 1], dtype=np.int64)},
    }
    for tag, payload in bad.items():
        try:
            GQ.unpack_kv_arrays(payload, ["k"])
            raise AssertionError(f"{tag} was accepted")
        except GQ.GraftQuantFormatError as exc:
            out[f"bad_{tag}__error"] = np.asarray(str(exc))
        for key, val in payload.items():
            out[f"bad_{tag}__{key}"] = np.asarray(val)
    return out


def splice_case(seed: int):
    rng = np.random.default_rng(seed)
    out = {}
    cases = [(4, 64, 7, 20, 5), (0, 16, 0, 9, 9), (3, 32, 30, 12, 6), (2, 8, 3, 2, 0)]
    for i, (sink, width, old_mount, tin, n) in enumerate(cases):
        old = rng.integers(0, 65535, (3, tin, 10), dtype=np.uint16)
        mnt = rng.integers(0, 65535, (3, n, 10), dtype=np.uint16)
        res = O.RefStore().swap(old, mnt, sink, width, old_mount)
        out[f"c{i}_params"] = np.asarray([sink, width, old_mount], dtype=np.int64)
        out[f"c{i}_old"] = old
        out[f"c{i}_mount"] = mnt
        out[f"c{i}_out"] = res
    return out


def main() -> None:
    if not (REF / "cpp" / "grm_runtime.cpp").is_file():
        raise SystemExit(f"reference checkout not found at {REF}")
    O.ensure_built(ref_root=REF, with_ref=True)
    only = sys.argv[1:]
    if only:  # regenerate the named fixtures only, e.g. packed_payload
        cases = {"packed_payload": lambda: packed_case(6)}
        for name in only:
            np.savez_compressed(HERE / f"{name}.npz", **cases[name]())
            print(name, (HERE / f"{name}.npz").stat().st_size)
        return
    np.savez_compressed(HERE / "mla_d256.npz", **mla_case(0, 512, 256, 16))
    np.savez_compressed(HERE / "mla_d64.npz", **mla_case(10, 300, 64, 5))
    np.savez_compressed(HERE / "gqa_d128.npz", **gqa_case(2, 48, 2, 8, 128, 24, 16))
    np.savez_compressed(HERE / "gqa_d64_l4.npz", **gqa_case(3, 40, 8, 32, 64, 10, 8))
    np.savez_compressed(HERE / "quant_g32.npz", **quant_case(4))
    np.savez_compressed(HERE / "splice.npz", **splice_case(5))
    np.savez_compressed(HERE / "packed_payload.npz", **packed_case(6))
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
