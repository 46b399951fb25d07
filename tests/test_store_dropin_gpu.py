"""The drop-in seam, replayed on the GPU: GraftRepository's NativeGraftStore
(core/grm_native.py) drives a CUDA route sidecar through
``configure_cuda_{mla,gqa}_route_bank(..., sidecar=...)`` and
``route_{mla,gqa}_cuda`` (core/grm_native.py:1498-1563, :1590-1648).

tests/golden/store_protocol.npz holds the exact calls the reference store
made on an injected sidecar (create_bank arguments, every route_topk query
and keyword) and the store's own answers from its CPU route
(grm_store_route / grm_store_route_gqa of the reference runtime), written by
tests/golden/make_store_protocol.py.  The reference checkout is not on the
GPU box, so these tests replay those calls against this repository's
sidecars and apply the store's own post-processing
(``[int(x) for x in mapped[0]]``): the result must equal the store's CPU
route, and a sentinel route must raise RuntimeError, as the store expects.
The GQA case goes through PaddedGQARouteSidecar with the arena's dense
zero-padded bank and its row_token_counts receipt."""

import json

import numpy as np
import pytest

from graftrepository_b200.cuda_router import (CudaGQARouteSidecar, CudaMLARouteSidecar,
                                              PaddedGQARouteSidecar)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def proto(golden):
    return golden("store_protocol.npz")


def _replay(z, case, bank):
    n = int(z[f"{case}_ncalls"])
    assert n >= 5
    for i in range(n):
        q = z[f"{case}_q{i}"]
        kw = json.loads(str(z[f"{case}_q{i}_kw"]))
        want = [int(x) for x in z[f"{case}_q{i}_want"]]
        if want == [-1]:
            with pytest.raises(RuntimeError):
                bank.route_topk(q, **kw)
            continue
        mapped, receipt = bank.route_topk(q, **kw)
        assert [int(x) for x in mapped[0].tolist()] == want, (case, i)
        assert receipt.measured_queries == 1 and receipt.route_repeats == kw["route_repeats"]


def test_mla_sidecar_replays_the_reference_store(proto):
    z = proto
    assert json.loads(str(z["mla_bank_kwargs"])) == []      # create_bank(route_bank, node_ids)
    sidecar = CudaMLARouteSidecar.build()
    bank = sidecar.create_bank(z["mla_bank"], z["mla_node_ids"])
    assert bank.signature == str(z["mla_signature"])
    _replay(z, "mla", bank)
    bank.close()
    sidecar.close()


def test_gqa_padded_sidecar_replays_the_reference_store(proto):
    z = proto
    assert json.loads(str(z["gqa_bank_kwargs"])) == ["signature"]
    sidecar = PaddedGQARouteSidecar(CudaGQARouteSidecar.build(), z["gqa_row_token_counts"])
    bank = sidecar.create_bank(z["gqa_bank"], z["gqa_node_ids"],
                               signature=str(z["gqa_signature"]))
    assert bank.signature == str(z["gqa_signature"])
    _replay(z, "gqa", bank)
    bank.close()
    # the padding kept (no receipt) routes identically: zero keys never raise a maximum
    plain = CudaGQARouteSidecar.build().create_bank(z["gqa_bank"], z["gqa_node_ids"])
    _replay(z, "gqa", plain)
    plain.close()
    sidecar.close()
