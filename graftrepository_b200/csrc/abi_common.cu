// abi_common.cu -- handle-less entry points of libgrm_b200.so: thread-local
// error text, device-property cache, upload/free helpers and the top-k merge
// used after the all-gather of per-shard route results.
#include <cstdlib>
#include <cstring>

#include "common.cuh"

namespace grm_b200 {

namespace {
thread_local std::string g_thread_error;
std::mutex g_info_mu;
DeviceInfo g_info[64];
}  // namespace

void set_thread_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_thread_error = buf;
}

unsigned scan_wait_limit() {
  static const unsigned limit = [] {
    const char* v = std::getenv("GRM_B200_WAIT_LIMIT");
    if (!v || !*v) return kWaitLimit;
    char* end = nullptr;
    const unsigned long n = std::strtoul(v, &end, 10);
    return (end && *end == '\0' && n <= kWaitLimit) ? (unsigned)n : kWaitLimit;
  }();
  return limit;
}

int device_info(int device, DeviceInfo* out) {
  if (device < 0 || device >= 64) return GRM_B200_EINVAL;
  std::lock_guard<std::mutex> lock(g_info_mu);
  if (g_info[device].sms == 0) {
    cudaDeviceProp prop;
    cudaError_t e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return cuda_status(e);
    g_info[device].sms = prop.multiProcessorCount;
    g_info[device].cc_major = prop.major;
  }
  *out = g_info[device];
  return 0;
}

// Merge `lists` sorted-or-unsorted candidate lists per query into the best
// `topk` (score desc, id asc; non-finite and UINT64_MAX entries dropped).
// One warp per query; ids are 64-bit global node rows here.
__global__ void merge_topk_kernel(const float* scores, const uint64_t* ids, int64_t sstride,
                                  int64_t istride, int queries, int lists, int per_list, int topk,
                                  float* out_scores, uint64_t* out_ids) {
  const int q = blockIdx.x;
  const int lane = threadIdx.x;
  if (q >= queries) return;
  // warp list with 64-bit ids
  float ls = -INFINITY;
  uint64_t lid = UINT64_MAX;
  const int n = lists * per_list;
  for (int base = 0; base < n; base += 32) {
    const int i = base + lane;
    float cs = -INFINITY;
    uint64_t cid = UINT64_MAX;
    if (i < n) {
      const int l = i / per_list, j = i % per_list;
      cs = scores[l * sstride + (int64_t)q * per_list + j];
      cid = ids[l * istride + (int64_t)q * per_list + j];
      if (cid == UINT64_MAX) cs = -INFINITY;
    }
    auto better64 = [](float sa, uint64_t ia, float sb, uint64_t ib) {
      return sa > sb || (sa == sb && ia < ib);
    };
    float ts = __shfl_sync(kFull, ls, 31);
    uint64_t tid = __shfl_sync(kFull, lid, 31);
    unsigned m = __ballot_sync(kFull, isfinite(cs) && better64(cs, cid, ts, tid));
    while (m) {
      const int src = __ffs(m) - 1;
      const float bs = __shfl_sync(kFull, cs, src);
      const uint64_t bid = __shfl_sync(kFull, cid, src);
      const unsigned ahead = __ballot_sync(kFull, better64(ls, lid, bs, bid));
      const int pos = __popc(ahead);
      const float us = __shfl_up_sync(kFull, ls, 1);
      const uint64_t uid = __shfl_up_sync(kFull, lid, 1);
      if (lane == pos) {
        ls = bs;
        lid = bid;
      } else if (lane > pos) {
        ls = us;
        lid = uid;
      }
      m &= m - 1;
      ts = __shfl_sync(kFull, ls, 31);
      tid = __shfl_sync(kFull, lid, 31);
      m &= __ballot_sync(kFull, better64(cs, cid, ts, tid));
    }
  }
  if (lane < topk) {
    const bool ok = isfinite(ls) && lid != UINT64_MAX;
    out_scores[(int64_t)q * topk + lane] = ok ? ls : __int_as_float(0x7FC00000);
    out_ids[(int64_t)q * topk + lane] = ok ? lid : UINT64_MAX;
  }
}

}  // namespace grm_b200

using namespace grm_b200;

extern "C" {

const char* grm_b200_last_error(void) { return g_thread_error.c_str(); }

const char* grm_b200_version(void) { return "grm_b200 0.1 sm_100a"; }

int grm_b200_upload(const void* host, size_t bytes, void** out_device) {
  if (!host || !out_device || bytes == 0) {
    set_thread_error("invalid upload arguments");
    return GRM_B200_EINVAL;
  }
  *out_device = nullptr;
  void* d = nullptr;
  cudaError_t e = cudaMalloc(&d, bytes);
  if (e == cudaSuccess) e = cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    if (d) cudaFree(d);
    set_thread_error("upload failed: %s", cudaGetErrorString(e));
    return cuda_status(e);
  }
  *out_device = d;
  return 0;
}

int grm_b200_free_device_ptr(void* device) {
  if (!device) return 0;
  return cuda_status(cudaFree(device));
}

int grm_b200_merge_topk_strided(const float* scores_device, int64_t scores_list_stride,
                                const uint64_t* ids_device, int64_t ids_list_stride, int queries,
                                int lists, int per_list, int topk, float* out_scores_device,
                                uint64_t* out_ids_device, void* stream) {
  if (!scores_device || !ids_device || !out_scores_device || !out_ids_device || queries <= 0 ||
      lists <= 0 || per_list <= 0 || topk <= 0 || topk > GRM_B200_MAX_TOPK ||
      scores_list_stride < (int64_t)queries * per_list ||
      ids_list_stride < (int64_t)queries * per_list) {
    set_thread_error("invalid merge_topk arguments");
    return GRM_B200_EINVAL;
  }
  merge_topk_kernel<<<queries, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      scores_device, ids_device, scores_list_stride, ids_list_stride, queries, lists, per_list,
      topk, out_scores_device, out_ids_device);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_thread_error("merge_topk launch failed: %s", cudaGetErrorString(e));
    return cuda_status(e);
  }
  return 0;
}

int grm_b200_merge_topk(const float* scores_device, const uint64_t* ids_device, int queries,
                        int lists, int per_list, int topk, float* out_scores_device,
                        uint64_t* out_ids_device, void* stream) {
  const int64_t stride = (int64_t)queries * per_list;
  return grm_b200_merge_topk_strided(scores_device, stride, ids_device, stride, queries, lists,
                                     per_list, topk, out_scores_device, out_ids_device, stream);
}

}  // extern "C"
