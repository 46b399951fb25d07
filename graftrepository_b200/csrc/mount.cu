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

// Re-RoPE of the positional part of the mounted rows at their arena seats
// (core/graft_arena.py:344-367, :1848-1859).  Columns [offset, width) of a
// row are heads of `dim` values; head element j of the row at arena seat p
// becomes x'_j * cos[p][j] + r_j * sin[p][j] (two fp32 products, one add,
// one bf16 rounding), with x' = the stored bf16 values, pair-swapped
// ([x0 x2 .. x1 x3 ..]) when asked, and r = rotate_half(x').  dim == 0: no
// rope.
struct Rope {
  const float* cos;
  const float* sin;
  int offset;
  int dim;
  int pair_swap;
  int aligned;  // dim a power of two <= 256, offset % dim == 0, 16-byte aligned tables
  // aligned mode: ceil(2^32 / d) for d = rope pieces per row and d = width, so
  // n / d = umulhi(n, m) for the n the kernel divides (0: divide instead)
  uint32_t m_nrp, m_w;
};

// n / d by the precomputed multiplier m = ceil(2^32 / d), exact while
// n * d < 2^32 (the host sets m = 0 otherwise, and d's integer division runs).
__device__ __forceinline__ int div_pre(int n, uint32_t m, int d) {
  return m ? (int)__umulhi((uint32_t)n, m) : n / d;
}

__device__ __forceinline__ float bf16_round(float f) {
  return __bfloat162float(__float2bfloat16_rn(f));
}

// The 8 stored values (as floats) of slice values u .. u+7 (u a multiple of
// 8), decoded from global memory: BITS = 4/6/8 packed format, BITS = 0 the
// reference format.
template <int BITS>
__device__ __forceinline__ void stored8(const void* codes, const void* scales, int64_t slice,
                                        int64_t vals, int64_t u, float (&x)[8]) {
  if constexpr (BITS == 0) {
    const int8_t* cp = static_cast<const int8_t*>(codes) + slice * vals + u;
    const uint2 w = __ldg(reinterpret_cast<const uint2*>(cp));
    const int8_t* cb = reinterpret_cast<const int8_t*>(&w);
    const float s = __ldg(static_cast<const float*>(scales) + slice * (vals / 32) + u / 32);
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = bf16_round(__half2float(__float2half_rn((float)cb[j] * s)));
  } else {
    const uint8_t* cp = static_cast<const uint8_t*>(codes) + slice * (vals * BITS / 8) + u * BITS / 8;
    uint64_t w;
    if constexpr (BITS == 4) {
      w = __ldg(reinterpret_cast<const uint32_t*>(cp));
    } else if constexpr (BITS == 8) {
      const uint2 v = __ldg(reinterpret_cast<const uint2*>(cp));
      w = (uint64_t)v.x | ((uint64_t)v.y << 32);
    } else {  // 6 bytes, 2-byte aligned
      const uint16_t* h = reinterpret_cast<const uint16_t*>(cp);
      w = (uint64_t)__ldg(h) | ((uint64_t)__ldg(h + 1) << 16) | ((uint64_t)__ldg(h + 2) << 32);
    }
    const float s = __half2float(
        __ldg(static_cast<const __half*>(scales) + slice * (vals / 64) + u / 64));
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t c = (uint32_t)(w >> (BITS * j)) & ((1u << BITS) - 1u);
      x[j] = bf16_round((float)((int)(c << (32 - BITS)) >> (32 - BITS)) * s);
    }
  }
}

// Rotated values of the piece at slice value u (in rope head column j0 of
// the row starting at slice value rowv, arena seat pos).
template <int BITS>
__device__ __forceinline__ void rope_piece(const void* codes, const void* scales, int64_t slice,
                                           int64_t vals, int64_t head_v, int j0, int64_t pos,
                                           const Rope& rope, float (&out)[8]) {
  const int half = rope.dim / 2;
  float a[8], b[8];
  if (!rope.pair_swap) {
    stored8<BITS>(codes, scales, slice, vals, head_v + j0, a);
    stored8<BITS>(codes, scales, slice, vals, head_v + (j0 < half ? j0 + half : j0 - half), b);
  } else {
    const int base = j0 < half ? 2 * j0 : 2 * (j0 - half);
    stored8<BITS>(codes, scales, slice, vals, head_v + base, a);
    stored8<BITS>(codes, scales, slice, vals, head_v + base + 8, b);
  }
  const float* cs = rope.cos + pos * rope.dim + j0;
  const float* sn = rope.sin + pos * rope.dim + j0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float xp, r;
    if (!rope.pair_swap) {
      xp = a[k];
      r = j0 < half ? -b[k] : b[k];
    } else {  // span s[0..15] = a | b; x'_j = s[2k] or s[2k+1]
      const float ev = k < 4 ? a[2 * k] : b[2 * k - 8];
      const float od = k < 4 ? a[2 * k + 1] : b[2 * k - 7];
      xp = j0 < half ? ev : od;
      r = j0 < half ? -od : ev;
    }
    out[k] = __fadd_rn(__fmul_rn(xp, __ldg(cs + k)), __fmul_rn(r, __ldg(sn + k)));
  }
}

__device__ __forceinline__ void unpack8(uint4 o, float (&f)[8]) {
  const uint32_t w[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = __uint_as_float(w[j] << 16);
    f[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
  }
}

// Aligned rope (dim a power of two <= 256, offset % dim == 0): the store
// rounds skip the rope pieces and leave their stored bf16 values in the
// warp's buffer obuf (16 bytes per 8 values of the tile); this pass then
// takes the tile's rope pieces 32 at a time, one per lane, reads the piece
// and its partner (rotate_half: j0 +- dim/2; pair-swapped: the 16-value span
// at 2*(j0 mod dim/2)) from obuf, rotates and stores it.  A head never
// straddles a tile: tiles start at multiples of 2048 values, heads at
// multiples of dim.  Rope pieces are numbered over the slice, nrp per row.
// The tile's rope pieces [p0, p1), numbered over the slice.  The tile ends
// in row t0 + (col0 + nv) / width (a small quotient: col0 + nv < width + 2048).
__device__ __forceinline__ void rope_range(int v0, int t0, int col0, int nv, int width,
                                           const Rope& rope, int& p0, int& p1) {
  const int nrp = (width - rope.offset) >> 3;
  p0 = t0 * nrp + min(max((col0 - rope.offset) >> 3, 0), nrp);
  const int e = col0 + nv, dt = div_pre(e, rope.m_w, width);
  p1 = (t0 + dt) * nrp + min(max((e - dt * width - rope.offset) >> 3, 0), nrp);
}

__device__ __forceinline__ void rope_pass(const uint4* obuf, uint16_t* dst, int v0, int p0,
                                          int p1, int width, int64_t seat, const Rope& rope,
                                          int lane) {
  const int nrp = (width - rope.offset) >> 3;
  const int half = rope.dim >> 1;
  for (int pc = p0 + lane; pc < p1; pc += 32) {
    const int r = div_pre(pc, rope.m_nrp, nrp), q = pc - r * nrp;
    const int v = r * width + rope.offset + 8 * q - v0;  // in the tile
    const int j0 = (8 * q) & (rope.dim - 1);
    const int head = v - j0;
    const bool lo = j0 < half;  // first half: r = -x'_{partner}, by a sign-flip multiply below
    uint32_t xw[8], rw[8];  // x' and the partner values as fp32 bit patterns
    if (!rope.pair_swap) {
      const uint4 a = obuf[v >> 3];
      const uint4 b = obuf[(head + (lo ? j0 + half : j0 - half)) >> 3];
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
      const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        xw[2 * k] = aw[k] << 16;
        xw[2 * k + 1] = aw[k] & 0xFFFF0000u;
        rw[2 * k] = bw[k] << 16;
        rw[2 * k + 1] = bw[k] & 0xFFFF0000u;
      }
    } else {  // span words S[k] = (x'-even value k | x'-odd value k << 16)
      const int base = head + (lo ? 2 * j0 : 2 * (j0 - half));
      const uint4 a = obuf[base >> 3], b = obuf[(base >> 3) + 1];
      const uint32_t sw8[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      // one byte permute per value: the even (low) or odd (high) half of S[k]
      // under a zero low half; x' takes the even values in the first half of
      // the head, the partner the odd ones, and the other way round after
      const unsigned sel_x = lo ? 0x1044u : 0x3244u, sel_r = lo ? 0x3244u : 0x1044u;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        xw[k] = __byte_perm(sw8[k], 0u, sel_x);
        rw[k] = __byte_perm(sw8[k], 0u, sel_r);
      }
    }
    const float sgn = lo ? -1.0f : 1.0f;  // -(r * s) == (-r) * s, exactly
    const int at = (int)(seat + r) * rope.dim + j0;
    const float4* cs = reinterpret_cast<const float4*>(rope.cos + at);
    const float4* sn = reinterpret_cast<const float4*>(rope.sin + at);
    const float4 c0 = __ldg(cs), c1 = __ldg(cs + 1), s0 = __ldg(sn), s1 = __ldg(sn + 1);
    const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    float f[8];
#pragma unroll
    for (int k = 0; k < 8; ++k)
      f[k] = __fadd_rn(__fmul_rn(__uint_as_float(xw[k]), cv[k]),
                       __fmul_rn(__fmul_rn(__uint_as_float(rw[k]), sv[k]), sgn));
    uint4 o;
    o.x = bf16x2_bits(f[0], f[1]);
    o.y = bf16x2_bits(f[2], f[3]);
    o.z = bf16x2_bits(f[4], f[5]);
    o.w = bf16x2_bits(f[6], f[7]);
    *reinterpret_cast<uint4*>(dst + v) = o;
  }
}

// Replace the 8 packed outputs of slice value u by their rotated values when
// the piece lies in a rope head (offset and dim are multiples of 8 and 16, so
// a piece never straddles a head boundary).
template <int BITS>
__device__ __forceinline__ void rope_fix(const void* codes, const void* scales, int64_t slice,
                                         int64_t vals, int64_t u, int64_t width, int64_t seat,
                                         const Rope& rope, uint4& o) {
  const int64_t t = u / width;
  const int col = (int)(u - t * width);
  if (col < rope.offset) return;
  const int rel = col - rope.offset;
  const int h = rel / rope.dim, j0 = rel - h * rope.dim;
  float f[8];
  rope_piece<BITS>(codes, scales, slice, vals, t * width + rope.offset + (int64_t)h * rope.dim, j0,
                   seat + t, rope, f);
  o.x = bf16x2_bits(f[0], f[1]);
  o.y = bf16x2_bits(f[2], f[3]);
  o.z = bf16x2_bits(f[4], f[5]);
  o.w = bf16x2_bits(f[6], f[7]);
}

// Packed format, warp tiles: a warp takes tiles of kTV values of one
// (graft, layer) slice, loads the tile's codes with coalesced 16-byte loads
// into its shared-memory buffer, and writes the output as 8 rounds in which
// lane l dequantises values 256*i + 8*l .. +7, so every store instruction
// writes 512 contiguous bytes.  The grid is persistent (SMs x 8 blocks).
constexpr int kTV = 2048;

// Exact integer -> float decode without int-to-float conversions: a byte n
// placed under the exponent bits of 2^23 (0x4B0000nn) is the float 2^23 + n,
// and subtracting 2^23 + bias (both exact in fp32) leaves n - bias.  Codes are
// stored two's complement, so flipping their sign bit first makes n - bias the
// signed code.
__device__ __forceinline__ float magic_byte(uint32_t x, int b) {
  return __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7650 + b));
}

// Codes of the 8 values v .. v+7 of the tile's buffer as floats (v a
// multiple of 8).
template <int BITS>
__device__ __forceinline__ void decode8(const uint32_t* sw, int v, float (&f)[8]) {
  if constexpr (BITS == 4) {
    const uint32_t x = sw[v >> 3] ^ 0x88888888u;
    const uint32_t lo = x & 0x0F0F0F0Fu, hi = (x >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      f[2 * b] = magic_byte(lo, b) - 8388616.0f;       // 2^23 + 8
      f[2 * b + 1] = magic_byte(hi, b) - 8388616.0f;
    }
  } else if constexpr (BITS == 8) {
    const uint32_t x0 = sw[v >> 2] ^ 0x80808080u, x1 = sw[(v >> 2) + 1] ^ 0x80808080u;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      f[b] = magic_byte(x0, b) - 8388736.0f;           // 2^23 + 128
      f[4 + b] = magic_byte(x1, b) - 8388736.0f;
    }
  } else {  // 6 bits: 48-bit window starting at bit 6v (a multiple of 16)
    const int b0 = v * 6;
    const int w = b0 >> 5, sh = b0 & 31;
    const uint64_t x = (((uint64_t)sw[w + 1] << 32) | sw[w]) >> sh;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t c = ((uint32_t)(x >> (6 * j)) & 63u) ^ 32u;
      f[j] = __uint_as_float(c | 0x4B000000u) - 8388640.0f;  // 2^23 + 32
    }
  }
}

// Load tile t (codes into r, lane l's group scale into s_lane) and return
// its slice and tile index.
template <int BITS, int NL>
__device__ __forceinline__ void load_packed_tile(const uint8_t* codes, const __half* scales,
                                                 int64_t vals, int tps, int t, int lane,
                                                 uint4 (&r)[NL], float& s_lane, int& slice,
                                                 int& tile) {
  slice = t / tps;
  tile = t - slice * tps;
  const int v0 = tile * kTV;
  const int nv = min(kTV, (int)vals - v0);
  const uint8_t* src = codes + slice * (vals * BITS / 8) + v0 * BITS / 8;
  const int nb16 = nv * BITS / 128;
#pragma unroll
  for (int j = 0; j < NL; ++j) {
    const int u = j * 32 + lane;
    r[j] = u < nb16 ? ld_stream(src + (int64_t)u * 16) : make_uint4(0, 0, 0, 0);
  }
  const __half* sc = scales + slice * (vals / 64) + v0 / 64;
  s_lane = lane < nv / 64 ? __half2float(sc[lane]) : 0.0f;
}

template <int NL>
__device__ __forceinline__ void load_ref_tile(const int8_t* codes, const float* scales,
                                              int64_t vals, int tps, int t, int lane,
                                              uint4 (&r)[NL], float& s_lo, float& s_hi,
                                              int& slice, int& tile) {
  slice = t / tps;
  tile = t - slice * tps;
  const int v0 = tile * kTV;
  const int nv = min(kTV, (int)vals - v0);
  const int8_t* src = codes + slice * vals + v0;
  const int nb16 = nv / 16;
#pragma unroll
  for (int j = 0; j < NL; ++j) {
    const int u = j * 32 + lane;
    r[j] = u < nb16 ? ld_stream(src + (int64_t)u * 16) : make_uint4(0, 0, 0, 0);
  }
  const float* sc = scales + slice * (vals / 32) + v0 / 32;
  const int ng = nv / 32;
  s_lo = lane < ng ? __ldg(sc + lane) : 0.0f;
  s_hi = 32 + lane < ng ? __ldg(sc + 32 + lane) : 0.0f;
}

template <int BITS, int RM>
__global__ void __launch_bounds__(256, 4) mount_packed_tiled_kernel(
    const uint8_t* __restrict__ codes, const __half* __restrict__ scales, int64_t slices,
    int64_t layers, int64_t vals, int64_t width, Seats seats, uint16_t* __restrict__ arena,
    int64_t arena_seats, Rope rope) {
  constexpr int TB = kTV * BITS / 8;      // code bytes of a full tile: 1024 / 1536 / 2048
  constexpr int NL = TB / (16 * 32);      // 16-byte loads per lane: 2 / 3 / 4
  __shared__ uint4 sbuf[8][TB / 16];  // INT6's 64-bit windows end inside the tile
  __shared__ uint4 obuf[RM == 1 ? 8 : 1][RM == 1 ? kTV / 8 : 1];  // stored rope pieces
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // 32-bit tile arithmetic: the host keeps vals and slices * tiles below 2^30
  const int tps = (int)ceil_div64(vals, kTV);
  const int total = (int)slices * tps;
  const int col_step = 256 % (int)width;  // round-to-round column advance (rope)
  const uint32_t* sw = reinterpret_cast<const uint32_t*>(sbuf[warp]);
  for (int t = blockIdx.x * 8 + warp; t < total; t += gridDim.x * 8) {
    uint4 r[NL];
    float s_lane;
    int slice, tile;
    load_packed_tile<BITS, NL>(codes, scales, vals, tps, t, lane, r, s_lane, slice, tile);
    const int g = slice / (int)layers, l = slice - g * (int)layers;
    const int v0 = tile * kTV;
    const int nv = min(kTV, (int)vals - v0);  // a multiple of 64
    const int t0 = v0 / (int)width;
    const int col0 = v0 - t0 * (int)width;
    int col = 0;  // column of this lane's piece in the current round (aligned rope)
    int p0 = 0, p1 = 0;  // the tile's rope pieces (aligned rope)
    if constexpr (RM == 1) {
      col = col0 + 8 * lane;
      while (col >= width) col -= (int)width;
      rope_range(v0, t0, col0, nv, (int)width, rope, p0, p1);
    }
    __syncwarp();  // the previous tile's reads of the buffers are done
#pragma unroll
    for (int j = 0; j < NL; ++j) sbuf[warp][j * 32 + lane] = r[j];
    __syncwarp();
    uint16_t* dst = arena + (l * arena_seats + seats.seat[g]) * width + v0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int v = i * 256 + 8 * lane;
      const float s = __shfl_sync(kFull, s_lane, (v >> 6) & 31);
      uint4 o = make_uint4(0, 0, 0, 0);
      if (v < nv) {
        float c[8];
        decode8<BITS>(sw, v, c);
        o.x = bf16x2_bits(c[0] * s, c[1] * s);
        o.y = bf16x2_bits(c[2] * s, c[3] * s);
        o.z = bf16x2_bits(c[4] * s, c[5] * s);
        o.w = bf16x2_bits(c[6] * s, c[7] * s);
      }
      bool store = v < nv;
      if constexpr (RM == 1) {
        if (store && col >= rope.offset) {  // rope piece: rotated in rope_pass
          obuf[warp][v >> 3] = o;
          store = false;
        }
        col += col_step;  // col < width and col_step < width: one wrap at most
        if (col >= width) col -= (int)width;
      } else if constexpr (RM == 2) {
        if (store) rope_fix<BITS>(codes, scales, slice, vals, v0 + v, width, seats.seat[g], rope, o);
      }
      if (store) *reinterpret_cast<uint4*>(dst + v) = o;
    }
    if constexpr (RM == 1) {
      __syncwarp();
      rope_pass(obuf[warp], dst, v0, p0, p1, (int)width, seats.seat[g], rope, lane);
    }
  }
}

// Reference format, warp tiles (the tiling of mount_packed_tiled_kernel):
// int8 codes, one fp32 scale per 32 values (lane l holds the tile's scales l
// and 32 + l), output bf16(fp16(code * scale)).
template <int RM>
__global__ void __launch_bounds__(256, 4) mount_ref_tiled_kernel(
    const int8_t* __restrict__ codes, const float* __restrict__ scales, int64_t slices,
    int64_t layers, int64_t vals, int64_t width, Seats seats, uint16_t* __restrict__ arena,
    int64_t arena_seats, Rope rope) {
  constexpr int NL = kTV / (16 * 32);  // 4 16-byte loads per lane
  __shared__ uint4 sbuf[8][kTV / 16];
  __shared__ uint4 obuf[RM == 1 ? 8 : 1][RM == 1 ? kTV / 8 : 1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // 32-bit tile arithmetic: the host keeps vals and slices * tiles below 2^30
  const int tps = (int)ceil_div64(vals, kTV);
  const int total = (int)slices * tps;
  const int col_step = 256 % (int)width;  // round-to-round column advance (rope)
  const uint2* sw = reinterpret_cast<const uint2*>(sbuf[warp]);
  for (int t = blockIdx.x * 8 + warp; t < total; t += gridDim.x * 8) {
    uint4 r[NL];
    float s_lo, s_hi;
    int slice, tile;
    load_ref_tile<NL>(codes, scales, vals, tps, t, lane, r, s_lo, s_hi, slice, tile);
    const int g = slice / (int)layers, l = slice - g * (int)layers;
    const int v0 = tile * kTV;
    const int nv = min(kTV, (int)vals - v0);  // a multiple of 32
    const int t0 = v0 / (int)width;
    const int col0 = v0 - t0 * (int)width;
    int col = 0;
    int p0 = 0, p1 = 0;  // the tile's rope pieces (aligned rope)
    if constexpr (RM == 1) {
      col = col0 + 8 * lane;
      while (col >= width) col -= (int)width;
      rope_range(v0, t0, col0, nv, (int)width, rope, p0, p1);
    }
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
      uint4 o = make_uint4(0, 0, 0, 0);
      if (v < nv) {
        const uint2 w = sw[v >> 3];
        const uint32_t x0 = w.x ^ 0x80808080u, x1 = w.y ^ 0x80808080u;
        float f[8];
#pragma unroll
        for (int b = 0; b < 4; ++b) {  // fp16 first (dequantize_symmetric_group32), then bf16
          f[b] = __half2float(__float2half_rn((magic_byte(x0, b) - 8388736.0f) * s));
          f[4 + b] = __half2float(__float2half_rn((magic_byte(x1, b) - 8388736.0f) * s));
        }
        o.x = bf16x2_bits(f[0], f[1]);
        o.y = bf16x2_bits(f[2], f[3]);
        o.z = bf16x2_bits(f[4], f[5]);
        o.w = bf16x2_bits(f[6], f[7]);
      }
      bool store = v < nv;
      if constexpr (RM == 1) {
        if (store && col >= rope.offset) {  // rope piece: rotated in rope_pass
          obuf[warp][v >> 3] = o;
          store = false;
        }
        col += col_step;  // col < width and col_step < width: one wrap at most
        if (col >= width) col -= (int)width;
      } else if constexpr (RM == 2) {
        if (store) rope_fix<0>(codes, scales, slice, vals, v0 + v, width, seats.seat[g], rope, o);
      }
      if (store) *reinterpret_cast<uint4*>(dst + v) = o;
    }
    if constexpr (RM == 1) {
      __syncwarp();
      rope_pass(obuf[warp], dst, v0, p0, p1, (int)width, seats.seat[g], rope, lane);
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

}  // extern "C"

namespace {

int mount_grid(int64_t slices, int64_t vals) {
  int dev = 0;
  cudaGetDevice(&dev);
  DeviceInfo info;
  if (device_info(dev, &info) != 0) info.sms = 148;
  return (int)std::max<int64_t>(
      1, std::min<int64_t>((int64_t)info.sms * 8, ceil_div64(slices * ceil_div64(vals, kTV), 8)));
}

// Host-side rope spec -> device Rope (dim 0: none).  Seats must lie inside the
// tables' rows.
bool rope_ok(const grm_b200_rope_spec* spec, int64_t width, const Seats& seats, int64_t n_grafts,
             int64_t tokens, Rope* out) {
  *out = Rope{nullptr, nullptr, 0, 0, 0, 0, 0, 0};
  if (!spec) return true;
  if (!spec->cos_device || !spec->sin_device || spec->dim <= 0 || spec->dim % 16 != 0 ||
      spec->offset < 0 || spec->offset % 8 != 0 || spec->offset >= width ||
      (width - spec->offset) % spec->dim != 0)
    return false;
  for (int64_t g = 0; g < n_grafts; ++g)
    if (seats.seat[g] + tokens > spec->rows) return false;
  const int64_t d = spec->dim;
  const bool aligned = d <= 256 && (d & (d - 1)) == 0 && spec->offset % d == 0 &&
                       width <= (int64_t)1 << 24 &&  // 32-bit column arithmetic
                       spec->rows * d < ((int64_t)1 << 31) &&  // 32-bit table index
                       reinterpret_cast<uintptr_t>(spec->cos_device) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(spec->sin_device) % 16 == 0;
  // division multipliers of the aligned rope pass: pieces numbered up to
  // tokens * nrp are divided by nrp, in-tile column sums below width + 2048
  // by width; each is exact while numerator x divisor < 2^32
  auto magic = [](int64_t n_max, int64_t d) -> uint32_t {
    if (d <= 1 || n_max * d >= ((int64_t)1 << 32)) return 0u;
    return (uint32_t)((((uint64_t)1 << 32) + (uint64_t)d - 1) / (uint64_t)d);
  };
  const int64_t nrp = (width - spec->offset) / 8;
  *out = Rope{spec->cos_device, spec->sin_device, (int)spec->offset, (int)d,
              spec->pair_swap ? 1 : 0, aligned ? 1 : 0, magic(tokens * nrp + 32, nrp),
              magic(width + 2048, width)};
  return true;
}

// The kernels index tiles in 32-bit: a slice below 2^30 values, below 2^30
// tiles in all (a 2^30-value bf16 slice is 2 GB).
bool tiles_fit(int64_t n_grafts, int64_t layers, int64_t tokens, int64_t width) {
  constexpr int64_t kLim = (int64_t)1 << 30;
  if (tokens > kLim || width > kLim || tokens * width > kLim || layers > kLim) return false;
  return n_grafts * layers * ceil_div64(tokens * width, kTV) <= kLim;
}

// Kernel rope mode: 0 none, 1 aligned heads (rope pass from shared memory),
// 2 any other layout (partners re-read from the codes).
int rope_mode(const Rope& rope) { return rope.dim == 0 ? 0 : rope.aligned ? 1 : 2; }

int mount_ref_impl(const int8_t* codes_device, const float* scales_device, int64_t n_grafts,
                   int64_t layers, int64_t tokens, int64_t width, const int64_t* seats_host,
                   uint16_t* arena_device, int64_t arena_seats, const grm_b200_rope_spec* spec,
                   void* stream) {
  Seats seats;
  Rope rope;
  if (!codes_device || !scales_device || !arena_device || layers <= 0 || tokens <= 0 ||
      width <= 0 || width % 32 != 0 || !tiles_fit(n_grafts, layers, tokens, width) ||
      !seats_ok(seats_host, n_grafts, tokens, arena_seats, &seats) ||
      !rope_ok(spec, width, seats, n_grafts, tokens, &rope)) {
    set_thread_error("invalid mount_ref arguments (grafts=%lld tokens=%lld width=%lld)",
                     (long long)n_grafts, (long long)tokens, (long long)width);
    return GRM_B200_EINVAL;
  }
  const int64_t vals = tokens * width;
  const int64_t slices = n_grafts * layers;
  const int grid = mount_grid(slices, vals);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int mode = rope_mode(rope);
  if (mode == 1)
    mount_ref_tiled_kernel<1><<<grid, 256, 0, s>>>(codes_device, scales_device, slices, layers,
                                                   vals, width, seats, arena_device, arena_seats,
                                                   rope);
  else if (mode == 2)
    mount_ref_tiled_kernel<2><<<grid, 256, 0, s>>>(codes_device, scales_device, slices, layers,
                                                   vals, width, seats, arena_device, arena_seats,
                                                   rope);
  else
    mount_ref_tiled_kernel<0><<<grid, 256, 0, s>>>(codes_device, scales_device, slices, layers,
                                                   vals, width, seats, arena_device, arena_seats,
                                                   rope);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_thread_error("mount_ref launch failed: %s", cudaGetErrorString(e));
    return cuda_status(e);
  }
  return 0;
}

template <int BITS>
void launch_packed(int grid, cudaStream_t s, const uint8_t* codes, const __half* sc, int64_t slices,
                   int64_t layers, int64_t vals, int64_t width, const Seats& seats,
                   uint16_t* arena, int64_t arena_seats, const Rope& rope) {
  const int mode = rope_mode(rope);
  if (mode == 1)
    mount_packed_tiled_kernel<BITS, 1><<<grid, 256, 0, s>>>(codes, sc, slices, layers, vals, width,
                                                            seats, arena, arena_seats, rope);
  else if (mode == 2)
    mount_packed_tiled_kernel<BITS, 2><<<grid, 256, 0, s>>>(codes, sc, slices, layers, vals, width,
                                                            seats, arena, arena_seats, rope);
  else
    mount_packed_tiled_kernel<BITS, 0><<<grid, 256, 0, s>>>(codes, sc, slices, layers, vals, width,
                                                            seats, arena, arena_seats, rope);
}

int mount_packed_impl(const uint8_t* codes_device, const uint16_t* scales_device, int bits,
                      int group, int64_t n_grafts, int64_t layers, int64_t tokens, int64_t width,
                      const int64_t* seats_host, uint16_t* arena_device, int64_t arena_seats,
                      const grm_b200_rope_spec* spec, void* stream) {
  Seats seats;
  Rope rope;
  if (!codes_device || !scales_device || !arena_device || layers <= 0 || tokens <= 0 ||
      width <= 0 || width % 8 != 0 || group != 64 || !tiles_fit(n_grafts, layers, tokens, width) ||
      (tokens * width) % 64 != 0 ||
      !(bits == 8 || bits == 6 || bits == 4) ||
      !seats_ok(seats_host, n_grafts, tokens, arena_seats, &seats) ||
      !rope_ok(spec, width, seats, n_grafts, tokens, &rope)) {
    set_thread_error("invalid mount_packed arguments (bits=%d group=%d width=%lld)", bits, group,
                     (long long)width);
    return GRM_B200_EINVAL;
  }
  const int64_t vals = tokens * width;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __half* sc = reinterpret_cast<const __half*>(scales_device);
  const int64_t slices = n_grafts * layers;
  const int grid = mount_grid(slices, vals);
  if (bits == 8)
    launch_packed<8>(grid, s, codes_device, sc, slices, layers, vals, width, seats, arena_device,
                     arena_seats, rope);
  else if (bits == 6)
    launch_packed<6>(grid, s, codes_device, sc, slices, layers, vals, width, seats, arena_device,
                     arena_seats, rope);
  else
    launch_packed<4>(grid, s, codes_device, sc, slices, layers, vals, width, seats, arena_device,
                     arena_seats, rope);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_thread_error("mount_packed launch failed: %s", cudaGetErrorString(e));
    return cuda_status(e);
  }
  return 0;
}

}  // namespace

extern "C" {

int grm_b200_mount_ref(const int8_t* codes_device, const float* scales_device, int64_t n_grafts,
                       int64_t layers, int64_t tokens, int64_t width, const int64_t* seats_host,
                       uint16_t* arena_device, int64_t arena_seats, void* stream) {
  return mount_ref_impl(codes_device, scales_device, n_grafts, layers, tokens, width, seats_host,
                        arena_device, arena_seats, nullptr, stream);
}

int grm_b200_mount_ref_rope(const int8_t* codes_device, const float* scales_device,
                            int64_t n_grafts, int64_t layers, int64_t tokens, int64_t width,
                            const int64_t* seats_host, uint16_t* arena_device, int64_t arena_seats,
                            const grm_b200_rope_spec* rope, void* stream) {
  if (!rope) {
    set_thread_error("mount_ref_rope: rope spec is NULL");
    return GRM_B200_EINVAL;
  }
  return mount_ref_impl(codes_device, scales_device, n_grafts, layers, tokens, width, seats_host,
                        arena_device, arena_seats, rope, stream);
}

int grm_b200_mount_packed(const uint8_t* codes_device, const uint16_t* scales_device, int bits,
                          int group, int64_t n_grafts, int64_t layers, int64_t tokens, int64_t width,
                          const int64_t* seats_host, uint16_t* arena_device, int64_t arena_seats,
                          void* stream) {
  return mount_packed_impl(codes_device, scales_device, bits, group, n_grafts, layers, tokens,
                           width, seats_host, arena_device, arena_seats, nullptr, stream);
}

int grm_b200_mount_packed_rope(const uint8_t* codes_device, const uint16_t* scales_device, int bits,
                               int group, int64_t n_grafts, int64_t layers, int64_t tokens,
                               int64_t width, const int64_t* seats_host, uint16_t* arena_device,
                               int64_t arena_seats, const grm_b200_rope_spec* rope, void* stream) {
  if (!rope) {
    set_thread_error("mount_packed_rope: rope spec is NULL");
    return GRM_B200_EINVAL;
  }
  return mount_packed_impl(codes_device, scales_device, bits, group, n_grafts, layers, tokens,
                           width, seats_host, arena_device, arena_seats, rope, stream);
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

int grm_b200_upload_rows(const void* const* parts_host, const int64_t* part_row_bytes, int n_parts,
                         int64_t rows, void* dst_device, int64_t dst_row_bytes, void* stream) {
  if (!parts_host || !part_row_bytes || n_parts <= 0 || rows < 0 || !dst_device ||
      dst_row_bytes <= 0) {
    set_thread_error("invalid upload_rows arguments");
    return GRM_B200_EINVAL;
  }
  int64_t total = 0;
  for (int i = 0; i < n_parts; ++i) {
    if (!parts_host[i] || part_row_bytes[i] <= 0) {
      set_thread_error("upload_rows: part %d is empty", i);
      return GRM_B200_EINVAL;
    }
    total += part_row_bytes[i];
  }
  if (total > dst_row_bytes) {
    set_thread_error("upload_rows: parts (%lld bytes per row) exceed the row (%lld)",
                     (long long)total, (long long)dst_row_bytes);
    return GRM_B200_EINVAL;
  }
  if (rows == 0) return 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int64_t col = 0;
  for (int i = 0; i < n_parts; ++i) {
    cudaError_t e = (total == dst_row_bytes && n_parts == 1)
                        ? cudaMemcpyAsync(dst_device, parts_host[0], (size_t)(rows * total),
                                          cudaMemcpyHostToDevice, s)
                        : cudaMemcpy2DAsync(static_cast<char*>(dst_device) + col,
                                            (size_t)dst_row_bytes, parts_host[i],
                                            (size_t)part_row_bytes[i], (size_t)part_row_bytes[i],
                                            (size_t)rows, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) {
      set_thread_error("upload_rows: copy of part %d failed: %s", i, cudaGetErrorString(e));
      return cuda_status(e);
    }
    col += part_row_bytes[i];
  }
  return 0;
}

}  // extern "C"
