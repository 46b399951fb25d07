"""B200-native (sm_100a) graft route + mount for GraftRepository.

Drop-in for the reference's CUDA route sidecars (core/grm_cuda_router.py) and
for the device mount of routed grafts (core/graft_arena.py swap/unpack_node):

* ``cuda_router``  -- CudaMLARouteSidecar/Bank, CudaGQARouteSidecar/Bank
* ``graft_mount``  -- fused dequantise + scatter into the bf16 arena
* ``sharded``      -- node-range sharded route over 1-8 GPUs (NCCL all-gather)
* ``synth``        -- seeded synthetic banks with the benchmark configs' shapes

All compute runs in ``libgrm_b200.so`` (include/grm_b200.h); there is no CPU
fallback.  The library is loaded on first use.
"""

__version__ = "0.1.0"

from ._lib import CudaRouterUnavailable, GrmB200Error  # noqa: F401
