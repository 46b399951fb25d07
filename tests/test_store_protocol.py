"""CPU checks of the drop-in seam (no GPU needed).

* The sidecar classes expose the reference's public call surface
  (core/grm_cuda_router.py: CudaMLARouteSidecar / CudaGQARouteSidecar and
  their banks): every parameter the reference declares is accepted under the
  same name and kind.
* Where the GraftRepository checkout is present, the committed store-protocol
  fixture is re-recorded from the reference store and must be unchanged, so
  the GPU replay (tests/test_store_dropin_gpu.py) tracks the reference."""

import inspect
import json
import sys

import numpy as np
import pytest

import oracle as O
from graftrepository_b200 import cuda_router as ours

REF = O.reference_root()
HAVE_REF = (REF / "core" / "grm_cuda_router.py").is_file() and O.ref_available()


def _ref_module():
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import core.grm_cuda_router as ref
    return ref


@pytest.mark.skipif(not HAVE_REF, reason="GraftRepository checkout not present")
@pytest.mark.parametrize("cls,meth", [
    ("CudaMLARouteSidecar", "create_bank"), ("CudaGQARouteSidecar", "create_bank"),
    ("CudaMLARouteBank", "route_topk"), ("CudaMLARouteBank", "route_topk_device"),
    ("CudaGQARouteBank", "route_topk"), ("CudaGQARouteBank", "route_topk_device"),
    ("CudaMLARouteSidecar", "build"), ("CudaGQARouteSidecar", "build"),
])
def test_public_signatures_accept_the_reference_calls(cls, meth):
    ref = _ref_module()
    rp = inspect.signature(getattr(getattr(ref, cls), meth)).parameters
    op = inspect.signature(getattr(getattr(ours, cls), meth)).parameters
    for name, p in rp.items():
        if name in ("self", "cls"):
            continue
        if name == "nvcc" or name == "build_dir":
            assert name in op
            continue
        assert name in op, (cls, meth, name)
        assert op[name].kind == p.kind or p.kind == inspect.Parameter.POSITIONAL_OR_KEYWORD, \
            (cls, meth, name)


@pytest.mark.skipif(not HAVE_REF, reason="GraftRepository checkout not present")
def test_store_protocol_fixture_is_current(golden):
    sys.path.insert(0, str(O.oracle.HERE.parent / "tests" / "golden"))
    import make_store_protocol as mk

    out = {}
    mk.mla_case(out)
    mk.gqa_case_ragged(out)
    z = golden("store_protocol.npz")
    assert sorted(out) == sorted(z)
    for k, v in out.items():
        assert np.array_equal(np.asarray(v), z[k], equal_nan=v.dtype.kind == "f"), k


def test_padded_adapter_forwards_the_padding_receipt():
    calls = []

    class Fake:
        def create_bank_padded(self, keys, node_ids, counts, *, signature=None):
            calls.append((keys, node_ids, list(counts), signature))
            return "bank"

        def close(self):
            calls.append("closed")

    ad = ours.PaddedGQARouteSidecar(Fake(), [3, 1, 2])
    assert ad.create_bank("K", "ids", signature="sig") == "bank"
    ad.close()
    assert calls == [("K", "ids", [3, 1, 2], "sig"), "closed"]
    vals, off = ours.dense_to_csr(np.arange(2 * 1 * 3 * 2, dtype=np.float32).reshape(2, 1, 3, 2),
                                  [3, 1])
    assert off.tolist() == [0, 3, 4] and vals.tolist() == list(range(6)) + [6.0, 7.0]
