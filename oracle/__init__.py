"""CPU parity oracle for the graft route and mount hot path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
package, and only as the checker or the timed CPU baseline; the product path
(``graftrepository_b200``) never imports it and has no CPU fallback.

Two checkers live here:

* ``liboracle.so`` -- ``grm_oracle.c``, a plain-C restatement of the reference
  laws (MLA fp64 cosine route, GQA sequential-fp32 |q.k| route, group-32 quant,
  packed mount quant, mount scatter, arena splice), each function citing the
  reference file:line it follows.
* ``_ref/libgrm_ref.so`` -- the reference's own ``cpp/grm_runtime.cpp`` compiled
  from its sources (``oracle/Makefile``) plus ``ref_driver.cpp``; this pins the
  restatement (``tests/test_oracle_pins.py``) and is the timed CPU baseline.
"""

from .oracle import *  # noqa: F401,F403
