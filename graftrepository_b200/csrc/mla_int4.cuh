// mla_int4.cuh -- the reference's INT4 bulk/refine MLA route mode on sm_100a.
//
// Law (GraftRepository cpp/grm_runtime.cpp, default build without OpenMP):
//   arena (rebuild_mla_arena :3241-3266), per row: max_abs = max |v| (std::max,
//     NaN skipped); scale = max_abs > 0 ? max_abs / 7 : 1; value_d =
//     int8(clamp(round(v_d / scale), -7, 7)) (round half away from zero; the
//     std::min / std::max clamp maps a NaN quotient to 7); norm_scale = scale *
//     (norm > 0 ? 1 / norm : 0) with the row's fp32 norm;
//   bulk score (int4_mla_row_score :3568-3585): dot = sum_d q_d * float(value_d)
//     in fp32, element order; s = dot * norm_scale * float(1 / (qnorm + 1e-8)),
//     then `+ 0.0f` (the lexical bonus of a query without keys, :4401-4402);
//   route (route_mla_int4 :4363-4482): the M = max(topk, refine_m) best finite
//     bulk scores by (score desc, node id asc) -- all of them when M >= their
//     count -- are rescored with exact_mla_entry_score; the top-k of those by
//     score_node_better.
// Every step is reproduced bit for bit: the bulk dot uses separately rounded
// fp32 multiplies and adds in element order, the candidate set is selected
// exactly (no approximation is involved in the selection at all), and the
// refine is the exact route's fp64 arithmetic.
//
// Device layout (built by the first INT4 route of a bank and kept with it):
// values are biased nibbles (value + 8, 1..15) packed 8 per 32-bit word and 4
// words (32 values) per 16-byte quad; the quads of 64-row tiles are
// interleaved [tile][quad][64 rows] so a warp loads one quad of 64 rows as two
// coalesced 512-byte runs.  Rows are padded to whole quads with value 0
// (exact: each padded element adds q * 0 = +0 to the dot, and the final
// `+ 0.0f` erases the only difference that could make, the sign of a zero).
// At 1M x 256 that is 128 MB against the 512 MB fp16 bank the exact route
// streams.
//
// Kernels per query (each a programmatic dependent of the one before):
//   int4_bulk_kernel    bulk scores -> ordered 32-bit keys and a level-1
//                       histogram of the top 12 key bits; its last block finds
//                       the level-1 boundary bin;
//   int4_collect_kernel rows above that bin become candidates, rows in it go
//                       to a boundary list with a level-2 histogram;
//   int4_select_kernel  one block resolves the boundary exactly: the level-2
//                       and level-3 bins (the low 8 key bits), then ties at
//                       the M-th key by row id;
//   int4_refine_kernel  exact fp64 scores of the candidates, a top-k per
//                       block, and the last block's top-k of those; it also
//                       resets the header for the next route.
#pragma once

namespace grm_b200 {
namespace mla {

constexpr int kQ4Bins = 4096;  // 12-bit histogram levels
constexpr int kQ4Tile = 64;    // rows per interleaved tile
constexpr int kQ4CollThreads = 256;
constexpr int kQ4RefThreads = 64;
constexpr int kQ4StageMax = 96 * 1024;  // shared bytes for staged candidate rows per block

struct Q4Hdr {
  unsigned hist1[kQ4Bins];
  unsigned hist2[kQ4Bins];
  unsigned ncand;      // candidates appended
  unsigned nbnd;       // boundary entries appended
  unsigned done_bulk;  // blocks finished (the last one of each kernel does
  unsigned done_ref;   // the kernel's single-block step)
  int b1;              // level-1 boundary bin, -1: every finite row is a candidate
  unsigned above1;     // rows in bins above b1
  float qinv;          // float(1 / (qnorm + 1e-8))
  int err;             // a bounded wait of the refine gave up (reported as kError)
  double qnorm;        // the query's reference norm
};

// Unsigned order-preserving key of a finite float; 0 marks "no score" (no
// finite float maps to it).  -0 is canonicalised to +0 by the caller.
__device__ __forceinline__ uint32_t q4_key(float s) {
  const uint32_t u = __float_as_uint(s);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__host__ __device__ inline int q4_quads(int dim) { return (dim / 8 + 3) / 4; }

// ---- arena -------------------------------------------------------------------

// One warp per row: the INT4 values and norm scale of rebuild_mla_arena.
// Rows past `nodes` in the last tile, and words past dim / 8, hold value 0.
template <typename T>
__global__ void __launch_bounds__(256) int4_arena_kernel(const T* __restrict__ rows,
                                                          const float* __restrict__ norms,
                                                          int64_t nodes, int dim,
                                                          uint32_t* __restrict__ q4,
                                                          float* __restrict__ nscale) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int W = dim / 8, WP = 4 * q4_quads(dim);
  const int64_t padded = ceil_div64(nodes, kQ4Tile) * kQ4Tile;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < padded;
       r += warps) {
    // word k of row r: quad k / 4 of its tile, lane-row r % 64, slot k % 4
    uint32_t* tile = q4 + (r / kQ4Tile) * (int64_t)WP * kQ4Tile + (r % kQ4Tile) * 4;
    auto word_at = [&](int k) -> uint32_t& {
      return tile[(int64_t)(k / 4) * kQ4Tile * 4 + (k % 4)];
    };
    if (r >= nodes) {
      for (int k = lane; k < WP; k += 32) word_at(k) = 0x88888888u;
      continue;
    }
    const T* row = rows + r * dim;
    float max_abs = 0.0f;  // fmaxf skips NaN like std::max(max_abs, |v|) does
    for (int d = lane; d < dim; d += 32) max_abs = fmaxf(max_abs, fabsf(to_f(row[d])));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) max_abs = fmaxf(max_abs, __shfl_xor_sync(kFull, max_abs, o));
    const float norm = norms[r];
    const float inv_norm = norm > 0.0f ? __fdiv_rn(1.0f, norm) : 0.0f;
    const float scale = max_abs > 0.0f ? __fdiv_rn(max_abs, 7.0f) : 1.0f;
    if (lane == 0) nscale[r] = __fmul_rn(scale, inv_norm);
    for (int k = lane; k < WP; k += 32) {
      uint32_t w = 0x88888888u;
      if (k < W) {
        w = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float x = roundf(__fdiv_rn(to_f(row[8 * k + i]), scale));
          float t = (x < 7.0f) ? x : 7.0f;    // std::min(7.0F, x)
          t = (-7.0f < t) ? t : -7.0f;        // std::max(-7.0F, t)
          w |= (uint32_t)((int)t + 8) << (4 * i);
        }
      }
      word_at(k) = w;
    }
  }
}

// ---- block helpers ---------------------------------------------------------------

// Inclusive suffix sum over the block's threads (thread t gets the sum of the
// values of threads t .. blockDim-1).  `sh` holds blockDim / 32 words.
__device__ __forceinline__ unsigned block_suffix_sum(unsigned v, unsigned* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned t = __shfl_down_sync(kFull, v, o);
    if (lane + o < 32) v += t;
  }
  if (lane == 0) sh[warp] = v;  // warp total
  __syncthreads();
  unsigned after = 0;
  for (int w = warp + 1; w < nw; ++w) after += sh[w];
  __syncthreads();
  return v + after;
}

// The boundary bin of a histogram of `bins` (a multiple of the block size)
// for the `need` largest keys: the bin b with count(> b) < need <=
// count(>= b); -1 when the histogram holds fewer than `need`.  *above =
// count(> b) and *total = the histogram's sum (shared-memory words the caller
// reads after a barrier).  Every thread of the block calls it; `sh` holds
// blockDim / 32 + 1 words.  The histogram is read through L2 (other blocks
// wrote it).
__device__ int q4_boundary(const unsigned* hist, int bins, unsigned need, unsigned* above,
                           unsigned* total, unsigned* sh) {
  const int per = bins / (int)blockDim.x;
  const int lo = (int)threadIdx.x * per;
  unsigned mine = 0;
  for (int i = 0; i < per; ++i) mine += __ldcg(hist + lo + i);
  const unsigned incl = block_suffix_sum(mine, sh);
  const int nw = blockDim.x >> 5;
  if (threadIdx.x == 0) {
    sh[nw] = 0xFFFFFFFFu;
    *total = incl;
  }
  __syncthreads();
  const unsigned excl = incl - mine;  // keys in the chunks above this one
  if (excl < need && incl >= need) {
    unsigned run = excl;
    for (int i = per - 1; i >= 0; --i) {
      const unsigned c = __ldcg(hist + lo + i);
      if (run + c >= need) {
        sh[nw] = (unsigned)(lo + i);
        *above = run;
        break;
      }
      run += c;
    }
  }
  __syncthreads();
  const unsigned b = sh[nw];
  __syncthreads();
  return b == 0xFFFFFFFFu ? -1 : (int)b;
}

// Last-block election after every block's global writes: true in every
// thread of the one block that finishes last.
__device__ __forceinline__ bool q4_last_block(unsigned* counter, int* sh_flag) {
  __threadfence();  // every thread's writes before the ticket
  __syncthreads();
  if (threadIdx.x == 0) {
    *sh_flag = atomicAdd(counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  const bool last = *sh_flag != 0;
  if (last) __threadfence();
  return last;
}

// Warp-aggregated append of `row` when `take` (the order of the list is free).
// Every lane of the warp must call it.
__device__ __forceinline__ void q4_append(bool take, uint32_t row, unsigned* count,
                                          uint32_t* list) {
  const unsigned m = __ballot_sync(kFull, take);
  if (!m) return;
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(m) - 1;
  unsigned base = 0;
  if (lane == leader) base = atomicAdd(count, (unsigned)__popc(m));
  base = __shfl_sync(kFull, base, leader);
  if (take) list[base + __popc(m & ((1u << lane) - 1u))] = row;
}

// ---- bulk pass -----------------------------------------------------------------

// Two rows per lane (rows l and 32 + l of a 64-row tile): per element one
// exact nibble -> float conversion (2^23 + u, minus 2^23 + 8; a packed f32x2
// subtract for both rows), then one multiply and one add, each rounded
// separately, in element order.  The multiply and add are scalar
// __fmul_rn / __fadd_rn: a packed __fmul2_rn whose product feeds a packed
// __fadd2_rn was measured on sm_100a to be contracted into a fused
// multiply-add (results differing from the separately rounded pair), and
// the reference rounds both.
//
// Lanes load their quads directly.  The pass is bound by issue (conversion,
// multiply and add per element, each its own instruction), not by HBM: it
// keeps many warps per SM resident rather than staging tiles in shared
// memory, which measured slower (126 vs 114 us per 1M route) with the one
// block per SM the stages allow.  QC > 0: the dim's quad count at compile
// time (dims 64/128/256), the tile loop fully unrolled with each quad loaded
// two quads ahead; QC == 0: any dim, one quad ahead.
constexpr int kQ4BulkWarps = 8;

template <int QC>
__global__ void __launch_bounds__(kQ4BulkWarps * 32) int4_bulk_kernel(
    const uint4* __restrict__ q4, const float* __restrict__ nscale, int64_t nodes, int dim,
    const float* __restrict__ query, uint32_t* __restrict__ keys, Q4Hdr* hdr, unsigned M) {
  constexpr int NW = kQ4BulkWarps;
  // the query, zero-padded to quads * 32 values
  extern __shared__ __align__(16) unsigned char b4_smem[];
  float* const qf = reinterpret_cast<float*>(b4_smem);
  __shared__ unsigned hist[kQ4Bins];
  __shared__ float sh_qinv;
  __shared__ unsigned sh_scan[NW + 1];
  __shared__ unsigned sh_above;
  __shared__ int sh_flag;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int quads = QC > 0 ? QC : q4_quads(dim);
  const int64_t tiles = ceil_div64(nodes, kQ4Tile);
  const int64_t stride = (int64_t)gridDim.x * NW;
  const int64_t t_first = (int64_t)blockIdx.x * NW + warp;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int j = threadIdx.x; j < quads * 32; j += blockDim.x) qf[j] = j < dim ? query[j] : 0.0f;
  for (int i = threadIdx.x; i < kQ4Bins; i += blockDim.x) hist[i] = 0;
  if (threadIdx.x == 0) {
    const double qn = query_norm_seq(query, dim);
    const float qinv = (float)(1.0 / (qn + 1.0e-8));
    sh_qinv = qinv;
    if (blockIdx.x == 0) {
      hdr->qnorm = qn;
      hdr->qinv = qinv;
    }
  }
  __syncthreads();
  const float qinv = sh_qinv;
  const float2 magic = make_float2(-8388616.0f, -8388616.0f);  // -(2^23 + 8)
  // elements 32 kq .. 32 kq + 31 of both rows, in order
  auto quad = [&](float2& acc, const uint4& ua, const uint4& ub, int kq) {
    const uint32_t wa4[4] = {ua.x, ua.y, ua.z, ua.w};
    const uint32_t wb4[4] = {ub.x, ub.y, ub.z, ub.w};
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t la = wa4[w] & 0x0F0F0F0Fu, ha = (wa4[w] >> 4) & 0x0F0F0F0Fu;
      const uint32_t lb = wb4[w] & 0x0F0F0F0Fu, hb = (wb4[w] >> 4) & 0x0F0F0F0Fu;
      // the query at elements (kq*4 + w)*8 .. +7
      const float4 q0 = *reinterpret_cast<const float4*>(qf + (kq * 4 + w) * 8);
      const float4 q1 = *reinterpret_cast<const float4*>(qf + (kq * 4 + w) * 8 + 4);
      const float qe[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float qlo = qe[2 * m], qhi = qe[2 * m + 1];  // elements 2m, 2m + 1
        const unsigned sel = 0x7440u + (unsigned)m;  // [byte m, 0, 0, 0x4B]
        // the values, exact small integers (a packed subtract: nothing to fuse)
        float2 v = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(la, 0x4B000000u, sel)),
                                          __uint_as_float(__byte_perm(lb, 0x4B000000u, sel))),
                              magic);
        acc.x = __fadd_rn(acc.x, __fmul_rn(qlo, v.x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(qlo, v.y));
        v = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(ha, 0x4B000000u, sel)),
                                   __uint_as_float(__byte_perm(hb, 0x4B000000u, sel))),
                       magic);
        acc.x = __fadd_rn(acc.x, __fmul_rn(qhi, v.x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(qhi, v.y));
      }
    }
  };
  auto finish_tile = [&](int64_t t, const float2& acc) {
    const int64_t ra = t * kQ4Tile + lane, rb = ra + 32;
    if (ra < nodes) {
      const float s = __fadd_rn(__fmul_rn(__fmul_rn(acc.x, __ldg(nscale + ra)), qinv), 0.0f);
      const uint32_t key = isfinite(s) ? q4_key(s) : 0u;
      keys[ra] = key;
      if (key) atomicAdd(&hist[key >> 20], 1u);
    }
    if (rb < nodes) {
      const float s = __fadd_rn(__fmul_rn(__fmul_rn(acc.y, __ldg(nscale + rb)), qinv), 0.0f);
      const uint32_t key = isfinite(s) ? q4_key(s) : 0u;
      keys[rb] = key;
      if (key) atomicAdd(&hist[key >> 20], 1u);
    }
  };
  if constexpr (QC > 0) {
    for (int64_t t = t_first; t < tiles; t += stride) {
      const uint4* base = q4 + t * (int64_t)QC * kQ4Tile + lane;
      float2 acc = make_float2(0.0f, 0.0f);
      uint4 ra[QC], rb[QC];  // static indices only: the loop below is unrolled
      ra[0] = __ldg(base);
      rb[0] = __ldg(base + 32);
      if (QC > 1) {
        ra[1] = __ldg(base + kQ4Tile);
        rb[1] = __ldg(base + kQ4Tile + 32);
      }
#pragma unroll
      for (int kq = 0; kq < QC; ++kq) {
        if (kq + 2 < QC) {
          ra[kq + 2] = __ldg(base + (kq + 2) * kQ4Tile);
          rb[kq + 2] = __ldg(base + (kq + 2) * kQ4Tile + 32);
        }
        quad(acc, ra[kq], rb[kq], kq);
      }
      finish_tile(t, acc);
    }
  } else {
    for (int64_t t = t_first; t < tiles; t += stride) {
      const uint4* base = q4 + t * (int64_t)quads * kQ4Tile + lane;
      float2 acc = make_float2(0.0f, 0.0f);
      uint4 na = __ldg(base), nb = __ldg(base + 32);  // quad 0, loaded one quad ahead
      for (int kq = 0; kq < quads; ++kq) {
        const uint4 ua = na, ub = nb;
        if (kq + 1 < quads) {
          na = __ldg(base + (int64_t)(kq + 1) * kQ4Tile);
          nb = __ldg(base + (int64_t)(kq + 1) * kQ4Tile + 32);
        }
        quad(acc, ua, ub, kq);
      }
      finish_tile(t, acc);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kQ4Bins; i += blockDim.x)
    if (hist[i]) atomicAdd(&hdr->hist1[i], hist[i]);
  asm volatile("griddepcontrol.launch_dependents;");
  if (!q4_last_block(&hdr->done_bulk, &sh_flag)) return;
  // level 1: the bin holding the M-th largest key; with at most M finite
  // rows every one of them is a candidate (b1 = -1)
  __shared__ unsigned sh_total;
  if (threadIdx.x == 0) sh_above = 0;
  const int b1 = q4_boundary(hdr->hist1, kQ4Bins, M, &sh_above, &sh_total, sh_scan);
  if (threadIdx.x == 0) {
    hdr->b1 = sh_total <= M ? -1 : b1;
    hdr->above1 = sh_above;
    hdr->done_bulk = 0;
  }
}

// ---- selection -----------------------------------------------------------------

// Rows are taken in chunks of kQ4Chunk per block: their candidates and
// boundary entries are gathered in shared memory and appended to the global
// lists with one atomic per list and chunk (thousands of warp-level atomics
// on one counter serialise in L2).
constexpr int kQ4Chunk = 2048;

__global__ void __launch_bounds__(kQ4CollThreads) int4_collect_kernel(
    const uint32_t* __restrict__ keys, int64_t nodes, Q4Hdr* hdr, uint32_t* cand, uint2* bnd) {
  constexpr int PER = kQ4Chunk / kQ4CollThreads;  // keys per thread and chunk
  __shared__ uint32_t s_cand[kQ4Chunk];
  __shared__ uint2 s_bnd[kQ4Chunk];
  __shared__ unsigned s_nc, s_nb, s_bc, s_bb;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b1 = __ldcg(&hdr->b1);
  const bool all = b1 < 0;
  for (int64_t c0 = (int64_t)blockIdx.x * kQ4Chunk; c0 < nodes;
       c0 += (int64_t)gridDim.x * kQ4Chunk) {
    if (threadIdx.x == 0) s_nc = s_nb = 0;
    uint32_t k[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {  // independent loads first
      const int64_t r = c0 + j * kQ4CollThreads + threadIdx.x;
      k[j] = r < nodes ? __ldcg(keys + r) : 0u;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const uint32_t r = (uint32_t)(c0 + j * kQ4CollThreads + threadIdx.x);
      const int bin = (int)(k[j] >> 20);
      if (k[j] && (all || bin > b1)) {
        s_cand[atomicAdd(&s_nc, 1u)] = r;
      } else if (k[j] && bin == b1) {
        s_bnd[atomicAdd(&s_nb, 1u)] = make_uint2(k[j], r);
        atomicAdd(&hdr->hist2[(k[j] >> 8) & 0xFFFu], 1u);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      s_bc = s_nc ? atomicAdd(&hdr->ncand, s_nc) : 0u;
      s_bb = s_nb ? atomicAdd(&hdr->nbnd, s_nb) : 0u;
    }
    __syncthreads();
    for (unsigned i = threadIdx.x; i < s_nc; i += blockDim.x) cand[s_bc + i] = s_cand[i];
    for (unsigned i = threadIdx.x; i < s_nb; i += blockDim.x) bnd[s_bb + i] = s_bnd[i];
    __syncthreads();
  }
  asm volatile("griddepcontrol.launch_dependents;");
}

// One block resolves the level-1 boundary bin exactly: the level-2 bin b2
// from hist2, level 3 (the low 8 key bits) over the boundary entries of b2,
// then the rows whose key equals the M-th key, lowest rows first.  Up to
// kQ4SelThreads * kQ4SelHeld boundary entries stay in registers across the
// passes (one round of independent loads); larger boundaries are re-read.
// This block is the only writer of the candidate list now, so appends go
// through a shared-memory counter written back at the end.
constexpr int kQ4SelThreads = 1024;
constexpr int kQ4SelHeld = 8;

__global__ void __launch_bounds__(kQ4SelThreads) int4_select_kernel(
    const uint2* __restrict__ bnd, int64_t nodes, unsigned M, Q4Hdr* hdr, uint32_t* cand,
    uint32_t* tie_bits) {
  __shared__ unsigned scratch[kQ4SelThreads];
  __shared__ unsigned sh_scan[kQ4SelThreads / 32 + 1];
  __shared__ unsigned hist3[256];
  __shared__ unsigned sh_above2, sh_above3, sh_n4, sh_taken, sh_nc;
  __shared__ int sh_b3;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b1 = __ldcg(&hdr->b1);
  if (b1 < 0) {
    asm volatile("griddepcontrol.launch_dependents;");
    return;
  }
  const unsigned above1 = __ldcg(&hdr->above1);
  const unsigned nb = __ldcg(&hdr->nbnd);
  const bool held = nb <= (unsigned)(kQ4SelThreads * kQ4SelHeld);
  uint2 e[kQ4SelHeld];
#pragma unroll
  for (int j = 0; j < kQ4SelHeld; ++j) {
    const unsigned i = j * kQ4SelThreads + threadIdx.x;
    e[j] = (held && i < nb) ? __ldcg(bnd + i) : make_uint2(0u, 0u);
  }
  if (threadIdx.x < 256) hist3[threadIdx.x] = 0;
  if (threadIdx.x == 0) {
    sh_above2 = sh_n4 = sh_taken = 0;
    sh_nc = __ldcg(&hdr->ncand);
  }
  unsigned total2 = 0;
  // level 2 within b1: count(bin b1) >= M - above1 holds by construction
  const int b2 = q4_boundary(hdr->hist2, kQ4Bins, M - above1, &sh_above2, &total2, sh_scan);
  const unsigned need3 = M - above1 - sh_above2;
  const uint32_t pre2 = ((uint32_t)b1 << 12) | (uint32_t)b2;  // key >> 8 of the level-2 bin
  unsigned* const nc = &sh_nc;
  // entry j of this thread: from registers, or re-read when the boundary is large
  const unsigned rounds = held ? (unsigned)kQ4SelHeld : (nb + kQ4SelThreads - 1) / kQ4SelThreads;
  auto entry = [&](unsigned j) -> uint2 {
    const unsigned i = j * kQ4SelThreads + threadIdx.x;
    if (held) {
      uint2 v = make_uint2(0u, 0u);
#pragma unroll
      for (int h = 0; h < kQ4SelHeld; ++h)
        if ((unsigned)h == j) v = e[h];
      return v;
    }
    return i < nb ? __ldcg(bnd + i) : make_uint2(0u, 0u);
  };
  for (unsigned j = 0; j < rounds; ++j) {
    const uint2 v = entry(j);
    const bool live = j * kQ4SelThreads + threadIdx.x < nb;
    q4_append(live && (int)((v.x >> 8) & 0xFFFu) > b2, v.y, nc, cand);
    if (live && (v.x >> 8) == pre2) atomicAdd(&hist3[v.x & 0xFFu], 1u);
  }
  __syncthreads();
  if (threadIdx.x < 32) {  // level 3 over 256 bins by one warp: count(bin b2) >= need3
    const int lane = threadIdx.x;
    unsigned mine = 0;  // bins 8*lane .. 8*lane+7
#pragma unroll
    for (int i = 0; i < 8; ++i) mine += hist3[8 * lane + i];
    unsigned incl = mine;  // suffix sum over lanes
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned t = __shfl_down_sync(kFull, incl, o);
      if (lane + o < 32) incl += t;
    }
    const unsigned excl = incl - mine;
    if (excl < need3 && incl >= need3) {
      unsigned run = excl;
      for (int i = 7; i >= 0; --i) {
        const unsigned c = hist3[8 * lane + i];
        if (run + c >= need3) {
          sh_b3 = 8 * lane + i;
          sh_above3 = run;
          break;
        }
        run += c;
      }
    }
  }
  __syncthreads();
  const uint32_t T = (pre2 << 8) | (uint32_t)sh_b3;  // the M-th key
  const unsigned need4 = need3 - sh_above3;          // rows with key == T to take
  for (unsigned j = 0; j < rounds; ++j) {
    const uint2 v = entry(j);
    const bool live = j * kQ4SelThreads + threadIdx.x < nb;
    q4_append(live && (v.x >> 8) == pre2 && v.x > T, v.y, nc, cand);
    if (live && v.x == T) atomicAdd(&sh_n4, 1u);
  }
  __syncthreads();
  const unsigned n4 = sh_n4;
  if (n4 <= need4) {  // every row with the M-th key is taken (n4 == need4)
    for (unsigned j = 0; j < rounds; ++j) {
      const uint2 v = entry(j);
      const bool live = j * kQ4SelThreads + threadIdx.x < nb;
      q4_append(live && v.x == T, v.y, nc, cand);
    }
  } else {
    // more rows share the M-th key than slots remain: the lowest row ids win
    // (candidate_better, cpp/grm_runtime.cpp:4422-4428), found in row order
    // through a bitmap that is cleared again on the way
    for (unsigned j = 0; j < rounds; ++j) {
      const uint2 v = entry(j);
      const bool live = j * kQ4SelThreads + threadIdx.x < nb;
      if (live && v.x == T) atomicOr(tie_bits + (v.y >> 5), 1u << (v.y & 31u));
    }
    __syncthreads();
    const int64_t words = ceil_div64(nodes, 32);
    for (int64_t w0 = 0; w0 < words; w0 += blockDim.x) {
      const int64_t w = w0 + threadIdx.x;
      const uint32_t bits = w < words ? __ldcg(tie_bits + w) : 0u;
      const unsigned c = (unsigned)__popc(bits);
      scratch[threadIdx.x] = c;  // block inclusive scan of c (Hillis-Steele)
      __syncthreads();
      for (int o = 1; o < (int)blockDim.x; o <<= 1) {
        const unsigned v = (int)threadIdx.x >= o ? scratch[threadIdx.x - o] : 0u;
        __syncthreads();
        scratch[threadIdx.x] += v;
        __syncthreads();
      }
      const unsigned incl = scratch[threadIdx.x];
      const unsigned taken = sh_taken;
      if (bits) {
        uint32_t b = bits;
        unsigned rank = taken + incl - c;
        while (b) {
          const int bit = __ffs(b) - 1;
          b &= b - 1;
          if (rank < need4) cand[atomicAdd(nc, 1u)] = (uint32_t)(w * 32 + bit);
          ++rank;
        }
        tie_bits[w] = 0u;
      }
      __syncthreads();
      if (threadIdx.x == blockDim.x - 1) sh_taken = taken + incl;
      __syncthreads();
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) hdr->ncand = sh_nc;
  asm volatile("griddepcontrol.launch_dependents;");
}

// ---- exact refine + top-k -------------------------------------------------------

// exact_score with the row read as 16-byte vectors (dim a multiple of 8) and
// the query as doubles: the same fp64 fma chain in element order.
template <typename T>
__device__ __forceinline__ float exact_score_vec(const T* row, int dim, const double* qd,
                                                 double qnorm, float norm) {
  constexpr int E = 16 / (int)sizeof(T);
  const uint4* rv = reinterpret_cast<const uint4*>(row);
  const int nv = dim / E;
  double dot = 0.0;
  for (int c = 0; c < nv; c += 4) {
    uint4 v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = c + i < nv ? ld_nc16(rv + c + i) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (c + i < nv) {
        const T* e = reinterpret_cast<const T*>(&v[i]);
#pragma unroll
        for (int k = 0; k < E; ++k) dot = fma(qd[(c + i) * E + k], to_d(e[k]), dot);
      }
    }
  }
  return (float)(dot / (qnorm * (double)norm + 1.0e-8));
}

// The same chain over a row staged in shared memory.
template <typename T>
__device__ __forceinline__ float exact_score_smem(const uint4* rs, int dim, const double* qd,
                                                  double qnorm, float norm) {
  constexpr int E = 16 / (int)sizeof(T);
  const int nv = dim / E;
  double dot = 0.0;
#pragma unroll 2
  for (int c = 0; c < nv; ++c) {
    const uint4 v = rs[c];
    const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int k = 0; k < E; ++k) dot = fma(qd[c * E + k], to_d(e[k]), dot);
  }
  return (float)(dot / (qnorm * (double)norm + 1.0e-8));
}

// One candidate per lane, the exact route's arithmetic.  With `stage` set
// each lane copies its candidate row into the warp's shared-memory stage with
// one bulk copy (the 32 copies of a warp are in flight together and complete
// on one mbarrier; rows padded by 16 bytes, so the lanes' reads of their own
// rows hit distinct banks), then every lane runs its row's sequential fp64
// chain from there; otherwise lanes read their rows from global memory.  A
// bounded wait that gives up waits once more for the warp's copies, leaves
// the warp's candidates out and makes the route report kError.  Each block keeps its top entries (score desc, row asc,
// non-finite dropped) in slot_s / slot_id [block * topk ..]; the last block to
// finish merges the slots, writes the result and resets the header for the
// next route.
template <typename T>
__global__ void __launch_bounds__(kQ4RefThreads) int4_refine_kernel(
    const T* __restrict__ rows, const float* __restrict__ norms, int dim,
    const float* __restrict__ query, const uint32_t* __restrict__ cand, Q4Hdr* hdr,
    float* slot_s, uint32_t* slot_id, int topk, uint64_t id_offset, Result* result,
    uint64_t* out_ids, float* out_scores, int stage) {
  extern __shared__ __align__(16) unsigned char ref_smem[];
  constexpr int NW = kQ4RefThreads / 32;
  __shared__ float sh_s[NW * 32];
  __shared__ uint32_t sh_id[NW * 32];
  __shared__ int sh_flag;
  __shared__ __align__(8) uint64_t rbar[NW];
  double* const qd = reinterpret_cast<double*>(ref_smem);  // [dim]
  if (stage && (threadIdx.x & 31) == 0) {
    mbar_init(&rbar[threadIdx.x >> 5], 1);
    mbar_fence_init();
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int i = threadIdx.x; i < dim; i += blockDim.x) qd[i] = (double)query[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned n = __ldcg(&hdr->ncand);
  const double qn = __ldcg(&hdr->qnorm);
  const int nv = dim * (int)sizeof(T) / 16;       // 16-byte vectors per row
  const int rs_vec = nv + 1;                       // staged row stride (vectors)
  uint4* const stage_w = reinterpret_cast<uint4*>(ref_smem + ((8 * dim + 15) & ~15)) +
                         (size_t)warp * 32 * rs_vec;
  WarpList list;
  list.init();
  unsigned rphase = 0;
  bool failed = false;
  const unsigned row_bytes = (unsigned)(nv * 16);
  for (unsigned c0 = (blockIdx.x * NW + warp) * 32u; c0 < n && !failed;
       c0 += gridDim.x * NW * 32u) {
    const unsigned c = c0 + lane;
    const uint32_t id = c < n ? __ldcg(cand + c) : kNoRow;
    float es = -INFINITY;
    if (stage) {
      const unsigned rows_in = __popc(__ballot_sync(kFull, id != kNoRow));
      if (lane == 0) mbar_arrive_expect_tx(&rbar[warp], rows_in * row_bytes);
      __syncwarp();
      if (id != kNoRow)
        bulk_g2s(stage_w + lane * rs_vec, rows + (int64_t)id * dim, row_bytes, &rbar[warp]);
      if (!mbar_wait(&rbar[warp], rphase, kWaitLimit)) {
        mbar_wait(&rbar[warp], rphase, kWaitLimit);  // the copies still in flight
        failed = true;
        if (lane == 0) atomicOr(&hdr->err, 1);
        break;
      }
      rphase ^= 1u;
      if (c < n) es = exact_score_smem<T>(stage_w + lane * rs_vec, dim, qd, qn, __ldg(norms + id));
      __syncwarp();
      fence_proxy_async_smem();  // the next copies overwrite what this round read
    } else if (c < n) {
      es = exact_score_vec<T>(rows + (int64_t)id * dim, dim, qd, qn, __ldg(norms + id));
    }
    const bool ok = c < n && isfinite(es);
    list.offer(ok ? es : -INFINITY, ok ? id : kNoRow, lane);
  }
  block_merge<NW>(list, lane, warp, sh_s, sh_id);
  if (warp == 0 && lane < topk) {
    slot_s[blockIdx.x * topk + lane] = list.s;
    slot_id[blockIdx.x * topk + lane] = list.id;
  }
  if (!q4_last_block(&hdr->done_ref, &sh_flag)) return;
  list.init();
  const unsigned ns = gridDim.x * (unsigned)topk;
  for (unsigned j0 = warp * 32u; j0 < ns; j0 += NW * 32u) {
    const unsigned j = j0 + lane;
    list.offer(j < ns ? __ldcg(slot_s + j) : -INFINITY, j < ns ? __ldcg(slot_id + j) : kNoRow,
               lane);
  }
  __syncthreads();
  block_merge<NW>(list, lane, warp, sh_s, sh_id);
  if (warp == 0) {
    const bool ok = lane < topk && isfinite(list.s) && list.id != kNoRow;
    const unsigned m = __ballot_sync(kFull, ok);
    if (lane < topk) {
      const uint64_t id = ok ? (uint64_t)list.id + id_offset : UINT64_MAX;
      const float s = ok ? list.s : __int_as_float(0x7FC00000);
      if (result) {
        result->ids[lane] = id;
        result->scores[lane] = s;
      }
      if (out_ids) out_ids[lane] = id;
      if (out_scores) out_scores[lane] = s;
    }
    if (lane == 0 && result) {
      result->count = __popc(m);
      result->status = __ldcg(&hdr->err) ? kError : kOk;
    }
  }
  // back to the state the next route starts from
  for (int i = threadIdx.x; i < kQ4Bins; i += blockDim.x) {
    hdr->hist1[i] = 0;
    hdr->hist2[i] = 0;
  }
  if (threadIdx.x == 0) {
    hdr->ncand = 0;
    hdr->nbnd = 0;
    hdr->done_ref = 0;
    hdr->err = 0;
  }
}

}  // namespace mla
}  // namespace grm_b200
