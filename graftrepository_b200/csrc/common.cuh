// common.cuh -- shared device helpers for the B200 graft route/mount library.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/grm_b200.h"

namespace grm_b200 {

constexpr unsigned kFull = 0xFFFFFFFFu;
constexpr uint32_t kNoRow = 0xFFFFFFFFu;

// Status codes (include/grm_b200.h).
inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? 0 : GRM_B200_CUDA_BASE + (int)e; }

// Handle-less error text, one per thread.
void set_thread_error(const char* fmt, ...);

// Per-handle error text.
struct ErrorSlot {
  std::string text;
  int set(int rc, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    text = buf;
    return rc;
  }
};

// score_node_better (GraftRepository cpp/grm_runtime.cpp:75-82): score desc,
// then row id asc.  Float comparison semantics, so -0 == +0.
__device__ __forceinline__ bool better(float sa, uint32_t ia, float sb, uint32_t ib) {
  return sa > sb || (sa == sb && ia < ib);
}

// Order-preserving float <-> int encoding for atomicMax on non-NaN floats.
__device__ __forceinline__ int float_to_ordered(float f) {
  int i = __float_as_int(f);
  return i >= 0 ? i : i ^ 0x7FFFFFFF;
}
__device__ __forceinline__ float ordered_to_float(int i) {
  return __int_as_float(i >= 0 ? i : i ^ 0x7FFFFFFF);
}
constexpr int kOrderedNegInf = (int)(0xFF800000u ^ 0x7FFFFFFFu);  // float_to_ordered(-inf)

// A warp-wide sorted top-32 list: lane i holds entry i (best first).  Empty
// entries are (-inf, kNoRow), which every finite candidate beats.
struct WarpList {
  float s;
  uint32_t id;
  __device__ __forceinline__ void init() { s = -INFINITY; id = kNoRow; }
  // Insert a warp-uniform candidate.
  __device__ __forceinline__ void insert(float cs, uint32_t cid, int lane) {
    const unsigned ahead = __ballot_sync(kFull, better(s, id, cs, cid));
    const int pos = __popc(ahead);
    const float us = __shfl_up_sync(kFull, s, 1);
    const uint32_t uid = __shfl_up_sync(kFull, id, 1);
    if (lane == pos) {
      s = cs;
      id = cid;
    } else if (lane > pos) {
      s = us;
      id = uid;
    }
  }
  // Every lane offers its own (cs, cid); finite candidates that beat the
  // current last entry are inserted one at a time.
  __device__ __forceinline__ void offer(float cs, uint32_t cid, int lane) {
    float ts = __shfl_sync(kFull, s, 31);
    uint32_t tid = __shfl_sync(kFull, id, 31);
    unsigned m = __ballot_sync(kFull, isfinite(cs) && better(cs, cid, ts, tid));
    while (m) {
      const int src = __ffs(m) - 1;
      const float bs = __shfl_sync(kFull, cs, src);
      const uint32_t bid = __shfl_sync(kFull, cid, src);
      insert(bs, bid, lane);
      m &= m - 1;
      ts = __shfl_sync(kFull, s, 31);
      tid = __shfl_sync(kFull, id, 31);
      m &= __ballot_sync(kFull, better(cs, cid, ts, tid));
    }
  }
  // offer() that also skips candidates below the list's k-th score minus
  // `margin2`.  Used where only rows within margin2 of the final k-th best
  // matter: the list's k-th score only grows, so a skipped row can never get
  // within margin2 of the final k-th best.  The list's last entry still
  // bounds the rows dropped for lack of room.
  __device__ __forceinline__ void offer_margin(float cs, uint32_t cid, int lane, int k,
                                               float margin2) {
    float ts = __shfl_sync(kFull, s, 31);
    uint32_t tid = __shfl_sync(kFull, id, 31);
    float tk = __shfl_sync(kFull, s, k - 1) - margin2;
    unsigned m = __ballot_sync(kFull, isfinite(cs) && cs >= tk && better(cs, cid, ts, tid));
    while (m) {
      const int src = __ffs(m) - 1;
      const float bs = __shfl_sync(kFull, cs, src);
      const uint32_t bid = __shfl_sync(kFull, cid, src);
      insert(bs, bid, lane);
      m &= m - 1;
      ts = __shfl_sync(kFull, s, 31);
      tid = __shfl_sync(kFull, id, 31);
      tk = __shfl_sync(kFull, s, k - 1) - margin2;
      m &= __ballot_sync(kFull, cs >= tk && better(cs, cid, ts, tid));
    }
  }
};

// 16-byte streaming load that bypasses L1 allocation (the bank is read once).
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// The same load without `volatile`, so the compiler may batch and hoist it
// (the bank is immutable while a route runs).
__device__ __forceinline__ uint4 ld_nc16(const void* p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}

// ---- mbarrier + bulk async copy (global -> shared), sm_90+ ----------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// Make initialised barriers visible to the async (TMA) proxy.
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// One probe of the barrier phase; true when the phase with `parity` completed.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after `limit` probes (each probe may block for a
// hardware-defined interval) and returns false, so no kernel can hang.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, unsigned limit) {
  for (unsigned i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from
// global memory into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, unsigned bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(smem_dst)), "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// An L2 policy that marks lines evict-first: a stream read once (the bank)
// then leaves the rest of L2 -- code, scratch, results -- in place.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// bulk_g2s with an L2 cache policy (l2_evict_first_policy for streamed data).
__device__ __forceinline__ void bulk_g2s_hint(void* smem_dst, const void* gmem_src, unsigned bytes,
                                              uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(smem_dst)), "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Order this thread's generic-proxy shared-memory accesses before later
// async-proxy (bulk copy) writes to the same buffer.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

constexpr unsigned kWaitLimit = 1u << 24;

// Probe limit of the streaming scans' bounded waits: kWaitLimit, unless the
// environment variable GRM_B200_WAIT_LIMIT (read once per process) gives
// another value.  Tests set it to 0 so that every wait gives up at once and
// the error path (drain the copies in flight, report status 3001) runs
// without any wait actually hanging.  The drain itself always uses kWaitLimit.
unsigned scan_wait_limit();

__host__ __device__ inline int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Device properties cached per device.
struct DeviceInfo {
  int sms = 0;
  int cc_major = 0;
};
int device_info(int device, DeviceInfo* out);

}  // namespace grm_b200
