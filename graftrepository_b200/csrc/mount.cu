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

// Packed format, warp tiles: a warp takes tiles of kTV values of one
// (graft, layer) slice, loads the tile's codes with coalesced 16-byte loads
// into its shared-memory buffer, and writes the output as 8 rounds in which
// lane l dequantises values 256*i + 8*l .. +7, so every store instruction
// writes 512 contiguous bytes.  The grid is persistent (SMs x 8 blocks).
constexpr int kTV = 2048;

template <int BITS>
__device__ __forceinline__ void codes8(const uint32_t* sw, int v, int (&code)[8]) {
  const int b0 = v * BITS;  // bit offset of the piece (v is a multiple of 8)
  const int w = b0 >> 5, sh = b0 & 31;
  const uint64_t x = (((uint64_t)sw[w + 1] << 32) | sw[w]) >> sh;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t c = (uint32_t)(x >> (BITS * j)) & ((1u << BITS) - 1u);
    code[j] = (int)(c << (32 - BITS)) >> (32 - BITS);  // sign-extend
  }
}

template <int BITS>
__global__ void __launch_bounds__(256) mount_packed_tiled_kernel(
    const uint8_t* __restrict__ codes, const __half* __restrict__ scales, int64_t slices,
    int64_t layers, int64_t vals, int64_t width, Seats seats, uint16_t* __restrict__ arena,
    int64_t arena_seats) {
  constexpr int TB = kTV * BITS / 8;      // code bytes of a full tile: 1024 / 1536 / 2048
  constexpr int NL = TB / (16 * 32);      // 16-byte loads per lane: 2 / 3 / 4
  __shared__ uint4 sbuf[8][TB / 16 + 1];  // +1: the 64-bit window of the last piece
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t tps = ceil_div64(vals, kTV);
  const int64_t total = slices * tps;
  const uint32_t* sw = reinterpret_cast<const uint32_t*>(sbuf[warp]);
  for (int64_t t = (int64_t)blockIdx.x * 8 + warp; t < total; t += (int64_t)gridDim.x * 8) {
    const int64_t slice = t / tps, tile = t - slice * tps;
    const int64_t g = slice / layers, l = slice - g * layers;
    const int64_t v0 = tile * kTV;
    const int nv = (int)min((int64_t)kTV, vals - v0);  // a multiple of 64
    const uint8_t* src = codes + slice * (vals * BITS / 8) + v0 * BITS / 8;
    const int nb16 = nv * BITS / 128;
    uint4 r[NL];
#pragma unroll
    for (int j = 0; j < NL; ++j) {
      const int u = j * 32 + lane;
      r[j] = u < nb16 ? ld_stream(src + (int64_t)u * 16) : make_uint4(0, 0, 0, 0);
    }
    const __half* sc = scales + slice * (vals / 64) + v0 / 64;
    const float s_lane = lane < nv / 64 ? __half2float(sc[lane]) : 0.0f;
    __syncwarp();  // the previous tile's reads of the buffer are done
#pragma unroll
    for (int j = 0; j < NL; ++j) sbuf[warp][j * 32 + lane] = r[j];
    __syncwarp();
    uint16_t* dst = arena + (l * arena_seats + seats.seat[g]) * width + v0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int v = i * 256 + 8 * lane;
      const float s = __shfl_sync(kFull, s_lane, (v >> 6) & 31);
      if (v < nv) {
        int code[8];
        codes8<BITS>(sw, v, code);
        uint4 o;
        o.x = bf16x2_bits((float)code[0] * s, (float)code[1] * s);
        o.y = bf16x2_bits((float)code[2] * s, (float)code[3] * s);
        o.z = bf16x2_bits((float)code[4] * s, (float)code[5] * s);
        o.w = bf16x2_bits((float)code[6] * s, (float)code[7] * s);
        *reinterpret_cast<uint4*>(dst + v) = o;
      }
    }
  }
}

// Reference format, warp tiles (the tiling of mount_packed_tiled_kernel):
// int8 codes, one fp32 scale per 32 values (lane l holds the tile's scales l
// and 32 + l), output bf16(fp16(code * scale)).
__global__ void __launch_bounds__(256) mount_ref_tiled_kernel(
    const int8_t* __restrict__ codes, const float* __restrict__ scales, int64_t slices,
    int64_t layers, int64_t vals, int64_t width, Seats seats, uint16_t* __restrict__ arena,
    int64_t arena_seats) {
  constexpr int NL = kTV / (16 * 32);  // 4 16-byte loads per lane
  __shared__ uint4 sbuf[8][kTV / 16];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t tps = ceil_div64(vals, kTV);
  const int64_t total = slices * tps;
  const uint2* sw = reinterpret_cast<const uint2*>(sbuf[warp]);
  for (int64_t t = (int64_t)blockIdx.x * 8 + warp; t < total; t += (int64_t)gridDim.x * 8) {
    const int64_t slice = t / tps, tile = t - slice * tps;
    const int64_t g = slice / layers, l = slice - g * layers;
    const int64_t v0 = tile * kTV;
    const int nv = (int)min((int64_t)kTV, vals - v0);  // a multiple of 32
    const int8_t* src = codes + slice * vals + v0;
    const int nb16 = nv / 16;
    uint4 r[NL];
#pragma unroll
    for (int j = 0; j < NL; ++j) {
      const int u = j * 32 + lane;
      r[j] = u < nb16 ? ld_stream(src + (int64_t)u * 16) : make_uint4(0, 0, 0, 0);
    }
    const float* sc = scales + slice * (vals / 32) + v0 / 32;
    const int ng = nv / 32;
    const float s_lo = lane < ng ? __ldg(sc + lane) : 0.0f;
    const float s_hi = 32 + lane < ng ? __ldg(sc + 32 + lane) : 0.0f;
    __syncwarp();
#pragma unroll
    for (int j = 0; j < NL; ++j) sbuf[warp][j * 32 + lane] = r[j];
    __syncwarp();
    uint16_t* dst = arena + (l * arena_seats + seats.seat[g]) * width + v0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int v = i * 256 + 8 * lane;
      const int grp = v >> 5;  // 8*i + lane/4
      const float s = __shfl_sync(kFull, i < 4 ? s_lo : s_hi, grp & 31);
      if (v < nv) {
        const uint2 w = sw[v >> 3];
        const int8_t* cb = reinterpret_cast<const int8_t*>(&w);
        float f[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)  // fp16 first (dequantize_symmetric_group32), then bf16
          f[j] = __half2float(__float2half_rn((float)cb[j] * s));
        uint4 o;
        o.x = bf16x2_bits(f[0], f[1]);
        o.y = bf16x2_bits(f[2], f[3]);
        o.z = bf16x2_bits(f[4], f[5]);
        o.w = bf16x2_bits(f[6], f[7]);
        *reinterpret_cast<uint4*>(dst + v) = o;
      }
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
  const int64_t slices = n_grafts * layers;
  int dev = 0;
  cudaGetDevice(&dev);
  DeviceInfo info;
  if (device_info(dev, &info) != 0) info.sms = 148;
  const int grid = (int)std::max<int64_t>(
      1, std::min<int64_t>((int64_t)info.sms * 8, ceil_div64(slices * ceil_div64(vals, kTV), 8)));
  mount_ref_tiled_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      codes_device, scales_device, slices, layers, vals, width, seats, arena_device, arena_seats);
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __half* sc = reinterpret_cast<const __half*>(scales_device);
  const int64_t slices = n_grafts * layers;
  int dev = 0;
  cudaGetDevice(&dev);
  DeviceInfo info;
  if (device_info(dev, &info) != 0) info.sms = 148;
  const int grid = (int)std::max<int64_t>(
      1, std::min<int64_t>((int64_t)info.sms * 8, ceil_div64(slices * ceil_div64(vals, kTV), 8)));
  if (bits == 8)
    mount_packed_tiled_kernel<8><<<grid, 256, 0, s>>>(codes_device, sc, slices, layers, vals, width,
                                                      seats, arena_device, arena_seats);
  else if (bits == 6)
    mount_packed_tiled_kernel<6><<<grid, 256, 0, s>>>(codes_device, sc, slices, layers, vals, width,
                                                      seats, arena_device, arena_seats);
  else
    mount_packed_tiled_kernel<4><<<grid, 256, 0, s>>>(codes_device, sc, slices, layers, vals, width,
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
