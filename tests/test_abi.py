"""The C-ABI library loads, exports every symbol include/grm_b200.h declares,
and the host-side protocol mirrors core/grm_cuda_router.py's validation.
No GPU compute (CPU only)."""

import ctypes
import subprocess

import numpy as np
import pytest

from graftrepository_b200 import _lib
from graftrepository_b200 import cuda_router as CR


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    syms = _lib.header_symbols()
    assert len(syms) >= 24
    for name in syms:
        assert hasattr(lib, name), name
    # and nothing else leaks out of the shared object
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    ours = {s for s in exported if s.startswith("grm_b200_")}
    assert ours == set(syms)


def test_handle_less_calls_validate_arguments():
    lib = _lib.load()
    bank = ctypes.c_void_p()
    rc = lib.grm_b200_mla_bank_create(None, 1, 10, 256, 0, ctypes.byref(bank))
    assert rc == -1
    assert "invalid" in _lib.thread_error()
    assert lib.grm_b200_merge_topk(None, None, 1, 1, 1, 1, None, None, None) == -1
    assert lib.grm_b200_mla_route(None, None, 1, 256, 0, 3, None, None, None) == -1
    assert lib.grm_b200_version().decode().startswith("grm_b200")


def test_mla_bank_validation_mirrors_reference():
    with pytest.raises(ValueError):
        CR.validate_mla_route_bank(np.zeros((4,), np.float32))
    with pytest.raises(ValueError):
        CR.validate_mla_route_bank(np.zeros((0, 8), np.float32))
    with pytest.raises(ValueError):
        CR.validate_mla_route_bank(np.zeros((4, 8), np.float32), node_ids=[1, 2])
    rows, ids = CR.validate_mla_route_bank(np.ones((3, 4)), node_ids=[7, 8, 9])
    assert rows.dtype == np.float32 and ids.dtype == np.uint64
    s1 = CR.mla_route_bank_signature(rows, ids)
    s2 = CR.mla_route_bank_signature(rows.copy(), ids.copy())
    assert s1 == s2 and len(s1) == 32


def test_gqa_bank_validation_and_dense_to_csr():
    with pytest.raises(ValueError):
        CR.validate_gqa_route_bank(np.zeros((2, 3, 4), np.float32))
    keys = np.arange(2 * 3 * 5 * 4, dtype=np.float32).reshape(2, 3, 5, 4)
    vals, off = CR.dense_to_csr(keys, token_counts=[2, 5])
    assert off.tolist() == [0, 2, 7]
    assert np.array_equal(vals[: 3 * 2 * 4].reshape(3, 2, 4), keys[0, :, :2])
    assert np.array_equal(vals[3 * 2 * 4:].reshape(3, 5, 4), keys[1])
    with pytest.raises(ValueError):
        CR.dense_to_csr(keys, token_counts=[6, 1])
    vals, off = CR.dense_to_csr(keys)
    assert off.tolist() == [0, 5, 10]


def test_narrowing_checks():
    x = np.array([1.0, 0.5, -3.25, np.nan], dtype=np.float32)
    assert CR._fits(x, np.float16) and CR._fits_bf16(x)
    y = np.array([1.0 + 2 ** -12], dtype=np.float32)
    assert not CR._fits(y, np.float16) and not CR._fits_bf16(y)
    z = np.array([1.0 + 2 ** -9], dtype=np.float32)
    assert CR._fits(z, np.float16) and not CR._fits_bf16(z)
