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
// values are biased nibbles (value + 8, 1..15) packed 8 per 32-bit word; the
// words of 64-row tiles are interleaved [tile][word][64 rows] so a warp loads
// one word of 64 rows as two coalesced 128-byte lines.  At 1M x 256 that is
// 128 MB against the 512 MB fp16 bank the exact route streams.
//
// Kernels per query (each a programmatic dependent of the one before):
//   int4_bulk_kernel    bulk scores -> ordered 32-bit keys, level-1 histogram
//                       of the top 12 key bits (HBM: 4 bits per value);
//   int4_collect_kernel every block finds the level-1 boundary bin from the
//                       histogram; rows above it become candidates, rows in it
//                       go to a boundary list with a level-2 histogram;
//   int4_select_kernel  one block resolves the boundary exactly: level-2 and
//                       level-3 bins, then ties at the M-th key by row id;
//   int4_refine_kernel  exact fp64 scores of the candidates; the last block
//                       takes the top-k and resets the histograms.
#pragma once

namespace grm_b200 {
namespace mla {

constexpr int kQ4Bins = 4096;  // 12-bit histogram levels
constexpr int kQ4Tile = 64;    // rows per interleaved tile
constexpr int kQ4BulkThreads = 256;
constexpr int kQ4SelThreads = 1024;
constexpr int kQ4RefThreads = 128;

struct Q4Hdr {
  unsigned hist1[kQ4Bins];
  unsigned hist2[kQ4Bins];
  unsigned ncand;   // candidates appended
  unsigned nbnd;    // boundary entries appended
  unsigned done;    // refine blocks finished
  int b1;           // level-1 boundary bin, -1: every finite row is a candidate
  unsigned above1;  // rows in bins above b1
  float qinv;       // float(1 / (qnorm + 1e-8))
  double qnorm;     // the query's reference norm
};

// Unsigned order-preserving key of a finite float; 0 marks "no score" (no
// finite float maps to it).  -0 is canonicalised to +0 by the caller.
__device__ __forceinline__ uint32_t q4_key(float s) {
  const uint32_t u = __float_as_uint(s);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float q4_unkey(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// ---- arena -------------------------------------------------------------------

// One warp per row: the INT4 values and norm scale of rebuild_mla_arena.
// Rows past `nodes` in the last tile hold value 0.
template <typename T>
__global__ void __launch_bounds__(256) int4_arena_kernel(const T* __restrict__ rows,
                                                          const float* __restrict__ norms,
                                                          int64_t nodes, int dim,
                                                          uint32_t* __restrict__ q4,
                                                          float* __restrict__ nscale) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int W = dim / 8;
  const int64_t padded = ceil_div64(nodes, kQ4Tile) * kQ4Tile;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < padded;
       r += warps) {
    uint32_t* tile = q4 + (r / kQ4Tile) * (int64_t)W * kQ4Tile + (r % kQ4Tile);
    if (r >= nodes) {
      for (int k = lane; k < W; k += 32) tile[(int64_t)k * kQ4Tile] = 0x88888888u;
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
    for (int k = lane; k < W; k += 32) {
      uint32_t w = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float x = roundf(__fdiv_rn(to_f(row[8 * k + i]), scale));
        float t = (x < 7.0f) ? x : 7.0f;    // std::min(7.0F, x)
        t = (-7.0f < t) ? t : -7.0f;        // std::max(-7.0F, t)
        w |= (uint32_t)((int)t + 8) << (4 * i);
      }
      tile[(int64_t)k * kQ4Tile] = w;
    }
  }
}

// ---- bulk pass -----------------------------------------------------------------

// Two rows per lane (rows l and 32 + l of a 64-row tile), as the two halves of
// packed f32x2 operations: per element one exact nibble -> float conversion
// (2^23 + u, minus 2^23 + 8), one multiply and one add, each rounded
// separately, in element order.
__global__ void __launch_bounds__(kQ4BulkThreads) int4_bulk_kernel(
    const uint32_t* __restrict__ q4, const float* __restrict__ nscale, int64_t nodes, int dim,
    const float* __restrict__ query, uint32_t* __restrict__ keys, Q4Hdr* hdr) {
  extern __shared__ float2 qq[];  // [dim] (q_d, q_d)
  __shared__ unsigned hist[kQ4Bins];
  __shared__ float sh_qinv;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = query[i];
    qq[i] = make_float2(v, v);
  }
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
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int NW = kQ4BulkThreads / 32;
  const int W = dim / 8;
  const int64_t tiles = ceil_div64(nodes, kQ4Tile);
  const float2 magic = make_float2(-8388616.0f, -8388616.0f);  // -(2^23 + 8)
  for (int64_t t = (int64_t)blockIdx.x * NW + warp; t < tiles; t += (int64_t)gridDim.x * NW) {
    const uint32_t* base = q4 + t * (int64_t)W * kQ4Tile + lane;
    float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll 4
    for (int k = 0; k < W; ++k) {
      const uint32_t wa = __ldg(base + (int64_t)k * kQ4Tile);
      const uint32_t wb = __ldg(base + (int64_t)k * kQ4Tile + 32);
      const uint32_t la = wa & 0x0F0F0F0Fu, ha = (wa >> 4) & 0x0F0F0F0Fu;
      const uint32_t lb = wb & 0x0F0F0F0Fu, hb = (wb >> 4) & 0x0F0F0F0Fu;
      const float2* qk = qq + 8 * k;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const unsigned sel = 0x7440u + (unsigned)m;  // [byte m, 0, 0, 0x4B]
        float2 v = make_float2(__uint_as_float(__byte_perm(la, 0x4B000000u, sel)),
                               __uint_as_float(__byte_perm(lb, 0x4B000000u, sel)));
        acc = __fadd2_rn(acc, __fmul2_rn(qk[2 * m], __fadd2_rn(v, magic)));
        v = make_float2(__uint_as_float(__byte_perm(ha, 0x4B000000u, sel)),
                        __uint_as_float(__byte_perm(hb, 0x4B000000u, sel)));
        acc = __fadd2_rn(acc, __fmul2_rn(qk[2 * m + 1], __fadd2_rn(v, magic)));
      }
    }
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
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kQ4Bins; i += blockDim.x)
    if (hist[i]) atomicAdd(&hdr->hist1[i], hist[i]);
  asm volatile("griddepcontrol.launch_dependents;");
}

// ---- selection -----------------------------------------------------------------

// The boundary bin of a histogram of `bins` (a multiple of the block size)
// for the `need` largest keys: the bin b with count(> b) < need <=
// count(>= b); returns -1 when the whole histogram holds fewer than `need`.
// *above = count(> b), *total = the histogram's sum.  Every thread of the
// block must call it; `scratch` holds blockDim.x + 2 words.
__device__ int q4_boundary(const unsigned* hist, int bins, unsigned need, unsigned* above,
                           unsigned* total, unsigned* scratch) {
  const int per = bins / (int)blockDim.x;
  const int lo = (int)threadIdx.x * per;
  unsigned mine = 0;
  for (int i = 0; i < per; ++i) mine += hist[lo + i];
  scratch[threadIdx.x] = mine;
  __syncthreads();
  // counts of every chunk above this thread's chunk (inclusive scan from the top)
  unsigned upper = 0;
  for (int j = (int)threadIdx.x + 1; j < (int)blockDim.x; ++j) upper += scratch[j];
  if (threadIdx.x == 0) {
    scratch[blockDim.x] = 0xFFFFFFFFu;
    scratch[blockDim.x + 1] = upper + mine;
  }
  __syncthreads();
  if (upper < need && upper + mine >= need) {
    unsigned run = upper;
    for (int i = per - 1; i >= 0; --i) {
      const unsigned c = hist[lo + i];
      if (run + c >= need) {
        scratch[blockDim.x] = (unsigned)(lo + i);
        *above = run;
        break;
      }
      run += c;
    }
  }
  __syncthreads();
  const unsigned b = scratch[blockDim.x];
  *total = scratch[blockDim.x + 1];
  __syncthreads();
  return b == 0xFFFFFFFFu ? -1 : (int)b;
}

// Warp-aggregated append of `row` when `take` (returns nothing; order free).
__device__ __forceinline__ void q4_append(bool take, uint32_t row, unsigned* count,
                                          uint32_t* list) {
  const unsigned m = __ballot_sync(__activemask(), take);
  if (!m) return;
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(m) - 1;
  unsigned base = 0;
  if (lane == leader) base = atomicAdd(count, (unsigned)__popc(m));
  base = __shfl_sync(__activemask(), base, leader);
  if (take) list[base + __popc(m & ((1u << lane) - 1u))] = row;
}

__global__ void __launch_bounds__(256) int4_collect_kernel(const uint32_t* __restrict__ keys,
                                                           int64_t nodes, unsigned M,
                                                           Q4Hdr* hdr, uint32_t* cand,
                                                           uint2* bnd) {
  __shared__ unsigned scratch[258];
  __shared__ unsigned sh_above;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) sh_above = 0;
  __syncthreads();
  unsigned total = 0;
  const int b1 = q4_boundary(hdr->hist1, kQ4Bins, M, &sh_above, &total, scratch);
  __syncthreads();
  const unsigned above = sh_above;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    hdr->b1 = (total > M) ? b1 : -1;
    hdr->above1 = above;
  }
  const bool all = total <= M;
  const int64_t n_iter = ceil_div64(nodes, 32) * 32;  // whole warps take part in the appends
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n_iter;
       r += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t key = r < nodes ? keys[r] : 0u;
    const int bin = (int)(key >> 20);
    const bool in = key && (all || bin > b1);
    const bool edge = key && !all && bin == b1;
    q4_append(in, (uint32_t)r, &hdr->ncand, cand);
    const unsigned m = __ballot_sync(kFull, edge);
    if (m) {
      const int lane = threadIdx.x & 31;
      const int leader = __ffs(m) - 1;
      unsigned base = 0;
      if (lane == leader) base = atomicAdd(&hdr->nbnd, (unsigned)__popc(m));
      base = __shfl_sync(kFull, base, leader);
      if (edge) {
        bnd[base + __popc(m & ((1u << lane) - 1u))] = make_uint2(key, (uint32_t)r);
        atomicAdd(&hdr->hist2[(key >> 8) & 0xFFFu], 1u);
      }
    }
  }
  asm volatile("griddepcontrol.launch_dependents;");
}

// One block resolves the level-1 boundary bin exactly.
__global__ void __launch_bounds__(kQ4SelThreads) int4_select_kernel(
    const uint2* __restrict__ bnd, int64_t nodes, unsigned M, Q4Hdr* hdr, uint32_t* cand,
    uint32_t* tie_bits) {
  __shared__ unsigned scratch[kQ4SelThreads + 2];
  __shared__ unsigned hist3[256];
  __shared__ unsigned sh_above2, sh_above3, sh_n4, sh_taken;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b1 = hdr->b1;
  if (b1 < 0) {
    asm volatile("griddepcontrol.launch_dependents;");
    return;
  }
  const unsigned need = M - hdr->above1;
  const unsigned nb = hdr->nbnd;
  if (threadIdx.x < 256) hist3[threadIdx.x] = 0;
  if (threadIdx.x == 0) {
    sh_above2 = sh_above3 = sh_n4 = sh_taken = 0;
  }
  __syncthreads();
  unsigned total = 0;
  const int b2 = q4_boundary(hdr->hist2, kQ4Bins, need, &sh_above2, &total, scratch);
  const unsigned need3 = need - sh_above2;
  const uint32_t pre2 = ((uint32_t)b1 << 12) | (uint32_t)b2;  // key >> 8 of the level-2 bin
  const unsigned n_iter = (nb + 31u) & ~31u;
  for (unsigned i = threadIdx.x; i < n_iter; i += blockDim.x) {
    const uint2 e = i < nb ? bnd[i] : make_uint2(0u, 0u);
    const bool live = i < nb;
    const bool in = live && (int)((e.x >> 8) & 0xFFFu) > b2;
    q4_append(in, e.y, &hdr->ncand, cand);
    if (live && (e.x >> 8) == pre2) atomicAdd(&hist3[e.x & 0xFFu], 1u);
  }
  __syncthreads();
  // level 3 (the low 8 bits): 256 bins, resolved by thread 0
  int b3;
  {
    unsigned* s = scratch;
    if (threadIdx.x < 256) s[threadIdx.x] = hist3[threadIdx.x];
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned run = 0, bb = 0xFFFFFFFFu;
      for (int i = 255; i >= 0; --i) {
        if (run + s[i] >= need3) {
          bb = (unsigned)i;
          break;
        }
        run += s[i];
      }
      sh_above3 = run;
      s[256] = bb;
    }
    __syncthreads();
    b3 = (int)s[256];
    __syncthreads();
  }
  const uint32_t T = (pre2 << 8) | (uint32_t)b3;  // the M-th key
  const unsigned need4 = need3 - sh_above3;         // rows with key == T to take
  for (unsigned i = threadIdx.x; i < n_iter; i += blockDim.x) {
    const uint2 e = i < nb ? bnd[i] : make_uint2(0u, 0u);
    const bool live = i < nb;
    q4_append(live && (e.x >> 8) == pre2 && e.x > T, e.y, &hdr->ncand, cand);
    if (live && e.x == T) atomicAdd(&sh_n4, 1u);
  }
  __syncthreads();
  const unsigned n4 = sh_n4;
  if (n4 <= need4) {  // every tie is taken (n4 == need4)
    for (unsigned i = threadIdx.x; i < n_iter; i += blockDim.x) {
      const uint2 e = i < nb ? bnd[i] : make_uint2(0u, 0u);
      q4_append(i < nb && e.x == T, e.y, &hdr->ncand, cand);
    }
  } else {
    // more rows share the M-th key than remain: the lowest row ids win
    // (candidate_better, cpp/grm_runtime.cpp:4422-4428), found in row order
    // through a bitmap that is cleared again on the way
    for (unsigned i = threadIdx.x; i < nb; i += blockDim.x) {
      const uint2 e = bnd[i];
      if (e.x == T) atomicOr(tie_bits + (e.y >> 5), 1u << (e.y & 31u));
    }
    __syncthreads();
    const int64_t words = ceil_div64(nodes, 32);
    for (int64_t w0 = 0; w0 < words; w0 += blockDim.x) {
      const int64_t w = w0 + threadIdx.x;
      const uint32_t bits = w < words ? tie_bits[w] : 0u;
      const unsigned c = (unsigned)__popc(bits);
      // block exclusive scan of c
      scratch[threadIdx.x] = c;
      __syncthreads();
      for (int o = 1; o < (int)blockDim.x; o <<= 1) {
        const unsigned v = (int)threadIdx.x >= o ? scratch[threadIdx.x - o] : 0u;
        __syncthreads();
        scratch[threadIdx.x] += v;
        __syncthreads();
      }
      const unsigned incl = scratch[threadIdx.x];
      const unsigned excl = incl - c;
      const unsigned taken = sh_taken;
      if (bits) {
        uint32_t b = bits;
        unsigned rank = taken + excl;
        while (b) {
          const int bit = __ffs(b) - 1;
          b &= b - 1;
          if (rank < need4) {
            const unsigned at = atomicAdd(&hdr->ncand, 1u);
            cand[at] = (uint32_t)(w * 32 + bit);
          }
          ++rank;
        }
        tie_bits[w] = 0u;
      }
      __syncthreads();
      if (threadIdx.x == blockDim.x - 1) sh_taken = taken + incl;
      __syncthreads();
    }
  }
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
  double dot = 0.0;
  for (int c = 0; c < dim / E; c += 4) {
    uint4 v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = (c + i) * E < dim ? ld_nc16(rv + c + i) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if ((c + i) * E >= dim) break;
      const T* e = reinterpret_cast<const T*>(&v[i]);
#pragma unroll
      for (int k = 0; k < E; ++k) dot = fma(qd[(c + i) * E + k], to_d(e[k]), dot);
    }
  }
  return (float)(dot / (qnorm * (double)norm + 1.0e-8));
}

// One candidate per thread, the exact route's arithmetic; the last block to
// finish takes the top-k (score desc, row asc, non-finite dropped), writes the
// result and resets the header for the next route.
template <typename T>
__global__ void __launch_bounds__(kQ4RefThreads) int4_refine_kernel(
    const T* __restrict__ rows, const float* __restrict__ norms, int dim,
    const float* __restrict__ query, const uint32_t* __restrict__ cand, Q4Hdr* hdr,
    float* __restrict__ ex, int topk, uint64_t id_offset, Result* result, uint64_t* out_ids,
    float* out_scores) {
  extern __shared__ double qd[];  // [dim]
  __shared__ float sh_s[kQ4RefThreads];
  __shared__ uint32_t sh_id[kQ4RefThreads];
  __shared__ int sh_last;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int i = threadIdx.x; i < dim; i += blockDim.x) qd[i] = (double)query[i];
  __syncthreads();
  const unsigned n = __ldcg(&hdr->ncand);
  const double qn = __ldcg(&hdr->qnorm);
  for (unsigned c = blockIdx.x * blockDim.x + threadIdx.x; c < n; c += gridDim.x * blockDim.x) {
    const uint32_t r = cand[c];
    ex[c] = exact_score_vec<T>(rows + (int64_t)r * dim, dim, qd, qn, __ldg(norms + r));
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned ticket = atomicAdd(&hdr->done, 1u);
    sh_last = ticket == gridDim.x - 1;
  }
  __syncthreads();
  if (!sh_last) return;
  __threadfence();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int NW = kQ4RefThreads / 32;
  WarpList list;
  list.init();
  for (unsigned c0 = warp * 32; c0 < n; c0 += NW * 32) {
    const unsigned c = c0 + lane;
    const float s = c < n ? __ldcg(ex + c) : -INFINITY;
    const uint32_t id = c < n ? __ldcg(cand + c) : kNoRow;
    list.offer(isfinite(s) ? s : -INFINITY, isfinite(s) ? id : kNoRow, lane);
  }
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
      result->status = kOk;
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
    hdr->done = 0;
  }
}

}  // namespace mla
}  // namespace grm_b200
