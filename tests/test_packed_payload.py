"""Packed graft payloads (core/graft_quant.py pack_kv_arrays fields) read
without a host dequant: the fail-closed checks of unpack_kv_arrays with its
messages, and the stored codes/scales, against payloads the reference itself
wrote (tests/golden/packed_payload.npz, tests/golden/make_golden.py)."""

import numpy as np
import pytest

import oracle as O
from graftrepository_b200 import packed

TAGS = {"mla8": ("c", "kpe"), "mla4": ("c", "kpe"), "gqa6": ("k",), "gqa3": ("k",)}


def payload(g, tag):
    pre = f"{tag}__"
    return {k[len(pre):]: g[k] for k in g if k.startswith(pre)}


@pytest.mark.parametrize("tag", sorted(TAGS))
def test_read_packed_keeps_the_stored_fields(golden, tag):
    g = golden("packed_payload.npz")
    p = payload(g, tag)
    got = packed.read_packed(p, TAGS[tag])
    for name, t in got.items():
        assert np.array_equal(t.codes, p[f"{name}_codes"])
        assert np.array_equal(t.scales, p[f"{name}_scales"])
        assert t.shape == tuple(int(x) for x in p[f"{name}_shape"])
        assert t.bits == int(p["storage_bits"])
        # the stored fields dequantise (oracle, graft_quant's law) to the
        # reference's own unpack_kv_arrays output
        f16, bf = O.dequant_ref(t.codes.reshape(-1), t.scales.reshape(-1))
        assert np.array_equal(f16.reshape(-1), p[f"expect_f16_{name}"].reshape(-1))
        assert np.array_equal(bf.reshape(-1), p[f"expect_bf16_{name}"].reshape(-1))


@pytest.mark.parametrize("tag", ["noversion", "version2", "bits16", "bits5", "noscales",
                                 "vecversion"])
def test_fail_closed_like_unpack_kv_arrays(golden, tag):
    g = golden("packed_payload.npz")
    p = payload(g, f"bad_{tag}")
    want = str(p.pop("error"))
    with pytest.raises(packed.GraftQuantFormatError) as exc:
        packed.read_packed(p, ["k"])
    assert str(exc.value) == want


def test_layout_mismatch_is_rejected(golden):
    g = golden("packed_payload.npz")
    p = payload(g, "mla8")
    p["kpe_codes"] = p["kpe_codes"][:, :-1]
    with pytest.raises(packed.GraftQuantFormatError):
        packed.read_packed(p, ["c", "kpe"])
