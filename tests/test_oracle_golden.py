"""Pin the CPU oracle against golden vectors produced by the reference itself
(tests/golden/make_golden.py): the C++ RouterIndex route, graft_quant, and
DeviceArena::apply_swap_tensor.  CPU only."""

import numpy as np
import pytest

import oracle as O

U64MAX = np.iinfo(np.uint64).max


@pytest.mark.parametrize("name", ["mla_d256.npz", "mla_d64.npz"])
def test_mla_oracle_matches_reference_golden(golden, name):
    g = golden(name)
    rows = g["rows_f16"].view(np.float16).astype(np.float32)
    k = int(g["topk"])
    for i, q in enumerate(g["queries"]):
        ids, scores = O.mla_route(rows, q, k)
        assert ids.tolist() == g["ids"][i].tolist(), i
        fin = g["ids"][i] != U64MAX
        # golden scores come from the python reference (np.dot order); the
        # oracle follows the C++ element order: equal to ~1 ulp
        np.testing.assert_allclose(scores[fin], g["scores"][i][fin], rtol=1e-6, atol=1e-7)


def test_mla_golden_edge_cases_are_present(golden):
    g = golden("mla_d256.npz")
    ids = g["ids"]
    assert ids[1][:3].tolist() == [5, 17, 40]          # duplicate rows: lowest id first
    assert np.all(ids[4] == U64MAX)                     # non-finite query: nothing
    assert ids[3][:4].tolist() == [0, 1, 2, 3]          # zero query: all 0, id order
    bad = {31, 32}
    assert not bad & set(int(x) for x in ids.reshape(-1))


@pytest.mark.parametrize("name", ["gqa_d128.npz", "gqa_d64_l4.npz"])
def test_gqa_oracle_matches_reference_golden(golden, name):
    g = golden(name)
    kh, d, k = int(g["kv_heads"]), int(g["head_dim"]), int(g["topk"])
    for key in ("q1", "q4", "qnan"):
        for i, q in enumerate(g[key]):
            ids, _ = O.gqa_route(g["keys_bf16"], g["token_offsets"], kh, d, q, k)
            assert ids.tolist() == g[key + "_ids"][i].tolist(), (key, i)


def test_gqa_golden_edge_cases(golden):
    g = golden("gqa_d128.npz")
    # non-finite query: only the empty node (T=0) scores, exactly 0
    assert g["qnan_ids"][0][0] == 4 and np.all(g["qnan_ids"][0][1:] == U64MAX)
    q1 = g["q1_ids"][0].tolist()
    assert 7 not in q1                                  # NaN key: dropped
    if 12 in q1 and 20 in q1:
        assert q1.index(12) < q1.index(20)              # exact duplicate: lowest id


@pytest.mark.parametrize("bits", [8, 6, 4, 3, 2])
def test_quant_oracle_matches_graft_quant(golden, bits):
    g = golden("quant_g32.npz")
    x = g["x_f16"].view(np.float16).astype(np.float32)
    codes, scales = O.quant_ref(x, bits)
    assert np.array_equal(codes, g[f"codes{bits}"].reshape(-1))
    assert np.array_equal(scales, g[f"scales{bits}"].reshape(-1))
    f16, bf = O.dequant_ref(g[f"codes{bits}"], g[f"scales{bits}"])
    assert np.array_equal(f16, g[f"dequant_f16_{bits}"].reshape(-1))
    assert np.array_equal(bf, g[f"dequant_bf16_{bits}"].reshape(-1))


def test_splice_oracle_matches_reference(golden):
    g = golden("splice.npz")
    i = 0
    while f"c{i}_params" in g:
        sink, width, old_mount = (int(v) for v in g[f"c{i}_params"])
        out = O.swap_splice(g[f"c{i}_old"], g[f"c{i}_mount"], sink, old_mount)
        assert np.array_equal(out, g[f"c{i}_out"]), i
        i += 1
    assert i >= 4


@pytest.mark.parametrize("bits", [8, 6, 4])
def test_packed_format_round_trip_and_bound(bits):
    rng = np.random.default_rng(bits)
    x = rng.standard_normal(64 * 300, dtype=np.float32) * 2.5
    x[:64] = 0.0
    codes, scales = O.quant_packed(x, bits)
    assert codes.size == x.size * bits // 8
    deq = O.bf16_bits_to_f32(O.dequant_packed(codes, scales, bits))
    s = O.f16_bits_to_f32(scales)
    assert np.all(s[0] == 1.0) and np.all(deq[:64] == 0.0)
    # |x - deq| <= scale/2 (rounding) + bf16 rounding of the product
    err = np.abs(x - deq).reshape(-1, 64)
    bound = s[:, None] * 0.5 + np.abs(deq.reshape(-1, 64)) * 2.0 ** -8 + 1e-30
    assert np.all(err <= bound * (1 + 1e-6))


def test_packed_quantiser_in_package_matches_oracle():
    from graftrepository_b200.graft_mount import quantize_packed

    rng = np.random.default_rng(11)
    x = rng.standard_normal((3, 2, 64 * 9), dtype=np.float32)
    for bits in (8, 6, 4):
        c, s = quantize_packed(x, bits)
        oc, os_ = O.quant_packed(x, bits)
        assert np.array_equal(c.reshape(-1), oc), bits
        assert np.array_equal(s.view(np.uint16).reshape(-1), os_), bits


def test_float_conversions_match_numpy():
    rng = np.random.default_rng(3)
    u = rng.integers(0, 2 ** 32, 100_000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    u = u[np.isfinite(u)]
    mine = np.array([O.lib().orc_f32_to_f16(float(v)) for v in u[:20000]], dtype=np.uint16)
    with np.errstate(over="ignore"):
        ref = u[:20000].astype(np.float16).view(np.uint16)
    assert np.array_equal(mine, ref)
    import torch
    t = torch.from_numpy(u).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(O.f32_to_bf16_bits(u), t)
