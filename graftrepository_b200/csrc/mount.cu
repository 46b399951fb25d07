// mount.cu -- fused dequantise + scatter of routed grafts into the bf16 arena,
// and the arena byte splice, on sm_100a.
//
// Reference: the host dequant of core/graft_quant.py:136-144
// (dequantize_symmetric_group32: fp32(code) * fp32 scale -> fp16) called from
// GQAArenaCache.unpack_node (core/graft_arena.py:3479-3492), the fp16 -> bf16
// upload cast (:3490), and the splice of the mounted payload into the arena
// seats (core/graft_arena.py:1933-1995; host byte oracle
// DeviceArena::apply_swap_tensor, cpp/grm_runtime.cpp:4941-5064).
//
// Layout.  Every (graft, layer) slice is a contiguous stream of tokens *
// width values; it lands contiguously at arena[layer, seat .. seat+tokens).
// Both kernels are pure streams (read codes + scales once, write bf16 once):
// HBM-bound, so they use 16-byte loads/stores and a grid of SMs x resident
// blocks that strides over the work.
#include <algorithm>

#include "common.cuh"

namespace grm_b200 {
namespace mount {

constexpr int kMaxGrafts = 64;

struct Seats {
  int64_t seat[kMaxGrafts];
};

__device__ __forceinline__ uint32_t bf16x2_bits(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Reference format: int8 codes, groups of 32, fp32 scales; output
// bf16(fp16(code * scale)).  One thread per 16 values.
__global__ void __launch_bounds__(256) mount_ref_kernel(const int8_t* __restrict__ codes,
                                                        const float* __restrict__ scales,
                                                        int64_t grafts, int64_t layers,
                                                        int64_t vals, int64_t width, Seats seats,
                                                        uint16_t* __restrict__ arena,
                                                        int64_t arena_seats) {
  const int64_t per_slice = vals / 16;
  const int64_t total = grafts * layers * per_slice;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t slice = i / per_slice;
    const int64_t v0 = (i - slice * per_slice) * 16;
    const int64_t g = slice / layers, l = slice - g * layers;
    const uint4 c = ld_stream(codes + slice * vals + v0);
    const float s = __ldg(scales + (slice * vals + v0) / 32);
    const int8_t* cb = reinterpret_cast<const int8_t*>(&c);
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // fp16 first (dequantize_symmetric_group32), then the bf16 upload cast
      const float a = __half2float(__float2half_rn((float)cb[2 * j] * s));
      const float b = __half2float(__float2half_rn((float)cb[2 * j + 1] * s));
      o[j] = bf16x2_bits(a, b);
    }
    uint16_t* dst = arena + (l * arena_seats + seats.seat[g]) * width + v0;
    reinterpret_cast<uint4*>(dst)[0] = make_uint4(o[0], o[1], o[2], o[3]);
    reinterpret_cast<uint4*>(dst)[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

template <int BITS>
__device__ __forceinline__ int code_at(const uint32_t* w, int j) {
  if constexpr (BITS == 8) {
    return (int)(int8_t)((w[j >> 2] >> (8 * (j & 3))) & 0xFF);
  } else if constexpr (BITS == 4) {
    const uint32_t n = (w[j >> 3] >> (4 * (j & 7))) & 0xF;
    return (int)(n << 28) >> 28;
  } else {  // 6 bits: 4 codes per little-endian 24-bit triple
    const int bit = 6 * j;
    const int word = bit >> 5, sh = bit & 31;
    uint32_t v = w[word] >> sh;
    if (sh > 26) v |= w[word + 1] << (32 - sh);
    return (int)((v & 0x3F) << 26) >> 26;
  }
}

// Packed format: `BITS`-bit codes, groups of 64 values, fp16 scales; output
// bf16(code * scale).  One thread per group (64 values, 128 output bytes).
template <int BITS>
__global__ void __launch_bounds__(256) mount_packed_kernel(const uint8_t* __restrict__ codes,
                                                           const __half* __restrict__ scales,
                                                           int64_t grafts, int64_t layers,
                                                           int64_t vals, int64_t width, Seats seats,
                                                           uint16_t* __restrict__ arena,
                                                           int64_t arena_seats) {
  constexpr int G = 64;
  constexpr int GB = G * BITS / 8;  // bytes per group: 64 / 48 / 32
  const int64_t per_slice = vals / G;
  const int64_t total = grafts * layers * per_slice;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t slice = i / per_slice;
    const int64_t gi = i - slice * per_slice;
    const int64_t g = slice / layers, l = slice - g * layers;
    uint32_t w[GB / 4 + 1];
    const uint8_t* src = codes + i * GB;
#pragma unroll
    for (int k = 0; k < GB / 16; ++k) {
      const uint4 v = ld_stream(src + 16 * k);
      w[4 * k] = v.x;
      w[4 * k + 1] = v.y;
      w[4 * k + 2] = v.z;
      w[4 * k + 3] = v.w;
    }
    w[GB / 4] = 0;
    const float s = __half2float(scales[i]);
    uint16_t* dst = arena + (l * arena_seats + seats.seat[g]) * width + gi * G;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c0 = code_at<BITS>(w, 8 * k + 2 * j);
        const int c1 = code_at<BITS>(w, 8 * k + 2 * j + 1);
        o[j] = bf16x2_bits((float)c0 * s, (float)c1 * s);
      }
      reinterpret_cast<uint4*>(dst)[k] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// out[o] = old[o][:sink] | mount[o] | old[o][tail_start:], 16 bytes per thread.
__global__ void splice_kernel(const uint4* __restrict__ old_p, const uint4* __restrict__ mnt,
                              uint4* __restrict__ out, int64_t outer, int64_t tin, int64_t tm,
                              int64_t sink, int64_t tail_start, int64_t out_t, int64_t row16) {
  const int64_t per_outer = out_t * row16;
  const int64_t total = outer * per_outer;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = i / per_outer;
    const int64_t r = i - o * per_outer;
    const int64_t t = r / row16, c = r - t * row16;
    uint4 v;
    if (t < sink) {
      v = old_p[(o * tin + t) * row16 + c];
    } else if (t < sink + tm) {
      v = mnt[(o * tm + (t - sink)) * row16 + c];
    } else {
      v = old_p[(o * tin + tail_start + (t - sink - tm)) * row16 + c];
    }
    out[i] = v;
  }
}

int grid_for(int64_t work) {
  int dev = 0;
  cudaGetDevice(&dev);
  DeviceInfo info;
  if (device_info(dev, &info) != 0) info.sms = 148;
  return (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div64(work, 256), (int64_t)info.sms * 8));
}

bool seats_ok(const int64_t* seats, int64_t n, int64_t tokens, int64_t arena_seats, Seats* out) {
  if (!seats || n <= 0 || n > kMaxGrafts) return false;
  for (int64_t g = 0; g < n; ++g) {
    if (seats[g] < 0 || seats[g] + tokens > arena_seats) return false;
    out->seat[g] = seats[g];
  }
  return true;
}

}  // namespace mount
}  // namespace grm_b200

using namespace grm_b200;
using namespace grm_b200::mount;

extern "C" {

int grm_b200_mount_ref(const int8_t* codes_device, const float* scales_device, int64_t n_grafts,
                       int64_t layers, int64_t tokens, int64_t width, const int64_t* seats_host,
                       uint16_t* arena_device, int64_t arena_seats, void* stream) {
  Seats seats;
  if (!codes_device || !scales_device || !arena_device || layers <= 0 || tokens <= 0 ||
      width <= 0 || width % 32 != 0 || !seats_ok(seats_host, n_grafts, tokens, arena_seats, &seats)) {
    set_thread_error("invalid mount_ref arguments (grafts=%lld tokens=%lld width=%lld)",
                     (long long)n_grafts, (long long)tokens, (long long)width);
    return GRM_B200_EINVAL;
  }
  const int64_t vals = tokens * width;
  const int64_t work = n_grafts * layers * (vals / 16);
  mount_ref_kernel<<<grid_for(work), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      codes_device, scales_device, n_grafts, layers, vals, width, seats, arena_device, arena_seats);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_thread_error("mount_ref launch failed: %s", cudaGetErrorString(e));
    return cuda_status(e);
  }
  return 0;
}

int grm_b200_mount_packed(const uint8_t* codes_device, const uint16_t* scales_device, int bits,
                          int group, int64_t n_grafts, int64_t layers, int64_t tokens, int64_t width,
                          const int64_t* seats_host, uint16_t* arena_device, int64_t arena_seats,
                          void* stream) {
  Seats seats;
  const int64_t vals = tokens * width;
  if (!codes_device || !scales_device || !arena_device || layers <= 0 || tokens <= 0 ||
      width <= 0 || width % 8 != 0 || group != 64 || vals % 64 != 0 ||
      !(bits == 8 || bits == 6 || bits == 4) ||
      !seats_ok(seats_host, n_grafts, tokens, arena_seats, &seats)) {
    set_thread_error("invalid mount_packed arguments (bits=%d group=%d width=%lld)", bits, group,
                     (long long)width);
    return GRM_B200_EINVAL;
  }
  const int64_t work = n_grafts * layers * (vals / 64);
  const int grid = grid_for(work);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __half* sc = reinterpret_cast<const __half*>(scales_device);
  if (bits == 8)
    mount_packed_kernel<8><<<grid, 256, 0, s>>>(codes_device, sc, n_grafts, layers, vals, width,
                                                seats, arena_device, arena_seats);
  else if (bits == 6)
    mount_packed_kernel<6><<<grid, 256, 0, s>>>(codes_device, sc, n_grafts, layers, vals, width,
                                                seats, arena_device, arena_seats);
  else
    mount_packed_kernel<4><<<grid, 256, 0, s>>>(codes_device, sc, n_grafts, layers, vals, width,
                                                seats, arena_device, arena_seats);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_thread_error("mount_packed launch failed: %s", cudaGetErrorString(e));
    return cuda_status(e);
  }
  return 0;
}

int grm_b200_arena_splice(const void* old_device, int64_t outer, int64_t input_tokens,
                          const void* mount_device, int64_t mount_tokens, int64_t row_bytes,
                          int64_t sink_tokens, int64_t old_mount_tokens, void* out_device,
                          int64_t* out_tokens, void* stream) {
  if (!old_device || !out_device || !out_tokens || outer <= 0 || input_tokens < 0 ||
      mount_tokens < 0 || (mount_tokens > 0 && !mount_device) || row_bytes <= 0 ||
      row_bytes % 16 != 0 || sink_tokens < 0 || old_mount_tokens < 0) {
    set_thread_error("invalid arena_splice arguments");
    return GRM_B200_EINVAL;
  }
  if (input_tokens < sink_tokens) {
    // DeviceArena::apply_swap_tensor: "input cache shorter than arena sink"
    set_thread_error("input cache shorter than arena sink");
    return GRM_B200_EINVAL;
  }
  const int64_t old_end = sink_tokens + old_mount_tokens;
  const int64_t tail_start = std::min(old_end, input_tokens);
  const int64_t out_t = sink_tokens + mount_tokens + (input_tokens - tail_start);
  *out_tokens = out_t;
  const int64_t row16 = row_bytes / 16;
  const int64_t work = outer * out_t * row16;
  if (work == 0) return 0;
  splice_kernel<<<grid_for(work), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(old_device), static_cast<const uint4*>(mount_device),
      static_cast<uint4*>(out_device), outer, input_tokens, mount_tokens, sink_tokens, tail_start,
      out_t, row16);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_thread_error("arena_splice launch failed: %s", cudaGetErrorString(e));
    return cuda_status(e);
  }
  return 0;
}

}  // extern "C"
