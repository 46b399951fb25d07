"""The bounded-wait error path of the bulk-copy MLA scan.

Every mbarrier wait of the streaming scan gives up after a probe limit, drains
the copies still in flight, and reports the query as failed instead of
hanging.  Normal runs never reach that path, so this test forces it: in a child
process with GRM_B200_WAIT_LIMIT=0 each wait gives up before its first probe.
The route must return status 3001 ("a bounded device wait gave up") and the
CUDA context must stay usable.  Nothing waits on a flag that is never set: the
copies complete normally and are waited for by the drain."""

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]

CHILD = r"""
import ctypes, sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
from graftrepository_b200 import _lib, synth
from graftrepository_b200.cuda_router import CudaMLARouteSidecar

rows = synth.mla_bank(23, 40_000)
bank = CudaMLARouteSidecar(device=0).create_bank_raw(rows, 1)
flags = ctypes.c_int(0)
assert _lib.load().grm_b200_mla_paths(bank._h, ctypes.byref(flags)) == 0
assert flags.value & 1, "bank is not on the bulk-copy path"
q = synth.mla_queries(23, 1)
try:
    bank.route_topk(q, topk=3)
except _lib.GrmB200Error as e:
    print("RC", e.rc, str(e))
else:
    print("RC 0")
x = torch.arange(1024, device="cuda", dtype=torch.float32)
torch.cuda.synchronize()
print("CTX", float(x.sum().item()))
bank.close()
"""


def test_bulk_scan_wait_gives_up_and_reports():
    env = dict(os.environ, GRM_B200_WAIT_LIMIT="0")
    out = subprocess.run([sys.executable, "-c", CHILD, str(ROOT)], env=env, capture_output=True,
                         text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = out.stdout.splitlines()
    rc_line = next(l for l in lines if l.startswith("RC "))
    assert rc_line.startswith("RC 3001"), rc_line
    assert "bounded device wait gave up" in rc_line
    ctx = next(l for l in lines if l.startswith("CTX "))
    assert float(ctx.split()[1]) == 1023 * 1024 / 2
