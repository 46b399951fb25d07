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
// bf16(fp16(code * scale)).  Grid: x strides 16-value chunks of one
// (graft, layer) slice, y = slice.  Each thread handles kU consecutive chunks
// with all loads issued before any store; consecutive threads write
// consecutive 32-byte pieces, so a warp stores 1 KB contiguously.
constexpr int kU = 2;

__device__ __forceinline__ void store_bf16x16(uint16_t* dst, const float (&f)[16]) {
  uint32_t o[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = bf16x2_bits(f[2 * j], f[2 * j + 1]);
  reinterpret_cast<uint4*>(dst)[0] = make_uint4(o[0], o[1], o[2], o[3]);
  reinterpret_cast<uint4*>(dst)[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

__global__ void __launch_bounds__(256) mount_ref_kernel(const int8_t* __restrict__ codes,
                                                        const float* __restrict__ scales,
                                                        int64_t layers, int64_t vals, int64_t width,
                                                        Seats seats, uint16_t* __restrict__ arena,
                                                        int64_t arena_seats) {
  const int64_t slice = blockIdx.y;
  const int64_t g = slice / layers, l = slice - g * layers;
  const int64_t chunks = vals / 16;
  const int8_t* src = codes + slice * vals;
  const float* sc = scales + slice * (vals / 32);
  uint16_t* dst = arena + (l * arena_seats + seats.seat[g]) * width;
  for (int64_t c0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * kU; c0 < chunks;
       c0 += (int64_t)gridDim.x * blockDim.x * kU) {
    uint4 v[kU];
    float s[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (c0 + u < chunks) {
        v[u] = ld_stream(src + (c0 + u) * 16);
        s[u] = __ldg(sc + ((c0 + u) * 16) / 32);
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (c0 + u >= chunks) break;
      const int8_t* cb = reinterpret_cast<const int8_t*>(&v[u]);
      float f[16];
#pragma unroll
      for (int j = 0; j < 16; ++j)  // fp16 first (dequantize_symmetric_group32), then bf16
        f[j] = __half2float(__float2half_rn((float)cb[j] * s[u]));
      store_bf16x16(dst + (c0 + u) * 16, f);
    }
  }
}

// 16 codes of one chunk from the chunk's little-endian bit stream.
template <int BITS>
struct Chunk {
  static constexpr int kWords = 16 * BITS / 32;  // 4 / 3 / 2 words
  uint32_t w[kWords];
  __device__ __forceinline__ void load(const uint8_t* p) {
    if constexpr (BITS == 8) {
      const uint4 v = ld_stream(p);
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    } else if constexpr (BITS == 4) {
      const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
      w[0] = v.x; w[1] = v.y;
    } else {
      const uint32_t* q = reinterpret_cast<const uint32_t*>(p);
      w[0] = __ldg(q); w[1] = __ldg(q + 1); w[2] = __ldg(q + 2);
    }
  }
  __device__ __forceinline__ int code(int j) const {
    if constexpr (BITS == 8) {
      return (int)(int8_t)((w[j >> 2] >> (8 * (j & 3))) & 0xFF);
    } else if constexpr (BITS == 4) {
      return (int)(((w[j >> 3] >> (4 * (j & 7))) & 0xF) << 28) >> 28;
    } else {
      const int bit = 6 * j, word = bit >> 5, sh = bit & 31;
      uint32_t v = w[word] >> sh;
      if (sh > 26) v |= w[word + 1] << (32 - sh);
      return (int)((v & 0x3F) << 26) >> 26;
    }
  }
};

// Packed format: `BITS`-bit codes, groups of 64 values, fp16 scales; output
// bf16(code * scale).  Same grid shape as mount_ref_kernel.
template <int BITS>
__global__ void __launch_bounds__(256) mount_packed_kernel(const uint8_t* __restrict__ codes,
                                                           const __half* __restrict__ scales,
                                                           int64_t layers, int64_t vals,
                                                           int64_t width, Seats seats,
                                                           uint16_t* __restrict__ arena,
                                                           int64_t arena_seats) {
  const int64_t slice = blockIdx.y;
  const int64_t g = slice / layers, l = slice - g * layers;
  const int64_t chunks = vals / 16;
  const uint8_t* src = codes + slice * (vals * BITS / 8);
  const __half* sc = scales + slice * (vals / 64);
  uint16_t* dst = arena + (l * arena_seats + seats.seat[g]) * width;
  for (int64_t c0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * kU; c0 < chunks;
       c0 += (int64_t)gridDim.x * blockDim.x * kU) {
    Chunk<BITS> ch[kU];
    float s[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (c0 + u < chunks) {
        ch[u].load(src + (c0 + u) * (2 * BITS));  // 16 codes = 2*BITS bytes
        s[u] = __half2float(sc[(c0 + u) >> 2]);
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (c0 + u >= chunks) break;
      float f[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) f[j] = (float)ch[u].code(j) * s[u];
      store_bf16x16(dst + (c0 + u) * 16, f);
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

// x: enough 256-thread blocks for kU chunks per thread of one slice (capped,
// then grid-strided); y: one row of blocks per (graft, layer) slice.
dim3 slice_grid(int64_t slices, int64_t chunks) {
  const int64_t per = ceil_div64(chunks, 256 * kU);
  return dim3((unsigned)std::max<int64_t>(1, std::min<int64_t>(per, 1024)), (unsigned)slices);
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
  const dim3 grid = slice_grid(n_grafts * layers, vals / 16);
  mount_ref_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      codes_device, scales_device, layers, vals, width, seats, arena_device, arena_seats);
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
  const dim3 grid = slice_grid(n_grafts * layers, vals / 16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __half* sc = reinterpret_cast<const __half*>(scales_device);
  if (bits == 8)
    mount_packed_kernel<8><<<grid, 256, 0, s>>>(codes_device, sc, layers, vals, width, seats,
                                                arena_device, arena_seats);
  else if (bits == 6)
    mount_packed_kernel<6><<<grid, 256, 0, s>>>(codes_device, sc, layers, vals, width, seats,
                                                arena_device, arena_seats);
  else
    mount_packed_kernel<4><<<grid, 256, 0, s>>>(codes_device, sc, layers, vals, width, seats,
                                                arena_device, arena_seats);
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
