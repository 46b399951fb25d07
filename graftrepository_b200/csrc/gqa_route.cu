// gqa_route.cu -- exact ragged GQA route on sm_100a.
//
// Law (GraftRepository cpp/grm_runtime.cpp:3588-3671, gqa_arena_key_score):
// for every query head h (kv head kh = h / (H / KH)) best_h = max over query
// tokens qi and key tokens t of |dot_fp32(q_{h,qi}, k_{kh,t})| * inv_denom,
// where the dot is accumulated in fp32 in element order with separately
// rounded products and inv_denom = 1/sqrtf(head_dim); std::max semantics
// (a NaN candidate never replaces best, which starts at 0).  score =
// (sum_h best_h, fp32, h ascending) / H.  A node with no key tokens scores
// exactly 0; a node with a non-finite key, or any node when the query is
// non-finite, scores NaN and is dropped.  The query_tokens == 4 path of the
// reference (:3673-3739) takes the max over the four dots of a key token
// before scaling, with the same std::max semantics.  Ordering: score desc,
// node asc; the first topk are returned (:4800-4838).
//
// Design.  The bank is CSR: node i owns the contiguous block
// [KH, T_i, D] at token offset off[i].  Work items are (node, kv head, 128-token
// chunk); a warp computes q.k for 16 key tokens x up to 16 query vectors per
// mma.sync.m16n8k16 (bf16 or f16 operands, fp32 accumulate), with the fp32
// query split into hi + lo halves of the key type so the products carry ~16
// bits more than one bf16 rounding.  The key slice each thread owns is 64
// contiguous bytes (the K dimension is permuted identically in A and B), so
// keys stream from HBM in full 32-byte sectors with no shared-memory staging.
// The per-(node, head) maxima are combined with atomicMax on the float bits
// (max is exact and order-independent).  A per-node error bound
// e = eps * inv_denom / H * sum_h |q_h| * Kmax(node, kh) (Kmax = largest key-
// token norm of that head, computed at attach) brackets the reference score;
// every node whose upper bound reaches the k-th largest lower bound is
// recomputed with the reference's exact sequential fp32 arithmetic, so the ids
// and scores returned are the reference's bit for bit.
#include <algorithm>
#include <cmath>
#include <type_traits>
#include <vector>

#include <cuda.h>

#include "common.cuh"
#include "route_policy.cuh"

namespace grm_b200 {
namespace gqa {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kChunk = 128;      // key tokens per work item
constexpr float kEps = 2.44140625e-4f;  // 2^-12 relative to |q||k|: >= 5x the proven bound
constexpr float kHuge = 1.0e30f;
constexpr int kRefineChunk = 256;  // candidates per unit scan (the refine's block size)

struct Result {
  int count;
  int cands;     // nodes recomputed exactly for this route
  uint64_t ids[GRM_B200_MAX_TOPK];
  float scores[GRM_B200_MAX_TOPK];
};

// One scan work item: up to kChunk key tokens of one (node, kv head).
// base: element offset of the item's first key row; ntok: rows in the item.
struct Item {
  uint64_t base;
  uint32_t node;
  uint16_t kh;
  uint16_t ntok;
};
static_assert(sizeof(Item) == 16, "one 16-byte load per item");

struct QueryInfo {
  int finite;      // every query value finite
  int fast_ok;     // the query fits the fast path (|q| range)
  int err;         // a bounded device wait gave up during this route
  float pad;
};

// ---------------------------------------------------------------- helpers

template <typename KT>
__device__ __forceinline__ float key_to_f(KT v);
template <>
__device__ __forceinline__ float key_to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float key_to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float key_to_f<float>(float v) { return v; }

template <typename KT>
__device__ __forceinline__ bool key_nonfinite_bits(KT v) { return !isfinite(key_to_f(v)); }

__device__ __forceinline__ float std_max(float a, float b) { return (a < b) ? b : a; }


// fp32 -> (hi, lo) pair of the key type, packed two per 32-bit word.
template <typename KT>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <typename KT>
__device__ __forceinline__ float round_kt(float a);
template <>
__device__ __forceinline__ float round_kt<__nv_bfloat16>(float a) { return __bfloat162float(__float2bfloat16_rn(a)); }
template <>
__device__ __forceinline__ float round_kt<__half>(float a) { return __half2float(__float2half_rn(a)); }

template <typename KT>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  if constexpr (sizeof(KT) == 2 && std::is_same<KT, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// ------------------------------------------------------------ attach kernels

// Per (node, kv head): largest key-token L2 norm (fp32, inflated by 2^-10 to
// cover its own rounding) and the node's key-finite flag.  One warp per
// (node, kv head).
template <typename KT>
__global__ void attach_stats_kernel(const KT* keys, const uint64_t* off, int64_t nodes, int kh_n,
                                    int dim, float* kmax, unsigned char* key_bad) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t pair = wid; pair < nodes * kh_n; pair += nw) {
    const int64_t node = pair / kh_n;
    const int kh = (int)(pair % kh_n);
    const int64_t T = (int64_t)(off[node + 1] - off[node]);
    const KT* base = keys + ((int64_t)off[node] * kh_n + (int64_t)kh * T) * dim;
    float mx = 0.0f;
    bool bad = false;
    for (int64_t t = 0; t < T; ++t) {
      float ss = 0.0f;
      for (int d = lane; d < dim; d += 32) {
        const float v = key_to_f(base[t * dim + d]);
        bad = bad || !isfinite(v);
        ss = fmaf(v, v, ss);
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
      mx = fmaxf(mx, sqrtf(ss));
    }
    bad = __any_sync(kFull, bad);
    if (lane == 0) {
      kmax[pair] = bad ? kHuge : mx * (1.0f + 9.765625e-4f);
      if (bad) key_bad[node] = 1;
    }
  }
}

// --------------------------------------------------------------- route kernels

struct RouteParams {
  const void* keys;
  const uint64_t* off;
  int64_t nodes;
  int kh_n;        // kv heads (layers concatenated)
  int dim;
  int heads;       // query heads H
  int qt;          // query tokens
  int group;       // H / KH
  int nv;          // query vectors per kv head = group * qt
  float inv_denom;
  const float* query;          // [H, qt, D] of this query
  const Item* items;           // work items
  int64_t n_items;
  const float* kmax;           // [N, KH]
  const unsigned char* key_bad;
  unsigned* headmax;           // [N, H] float bits, zero between routes
  float* lo;                   // [N]
  float* hi;                   // [N]
  uint32_t* cand;              // [N]
  int* cand_count;
  uint32_t* frag;              // query fragments [KH][NT][32][16]
  float* qnorm_h;              // [H] max_qi |q_{h,qi}|
  QueryInfo* qinfo;
  int* qparts;                 // [KH] per-kv-head query flags (bit 0 non-finite, bit 1 too large)
  unsigned* qcount;            // query_prep blocks finished (re-armed by the last one)
  int topk;
  int fast;                    // 1 = approximate pass available for this bank
  Result* result;
  unsigned long long* refined_total;  // nodes recomputed exactly, all routes (device counter)
  int qt4;                     // reference query_tokens == 4 path
  uint64_t* out_ids;           // optional device outputs (topk entries of this query)
  float* out_scores;
  uint64_t id_offset;          // added to returned node rows (first row of this shard)
  // route policy (lexical bonus and filters, cpp/grm_runtime.cpp:4498-4867)
  const uint32_t* allow;       // bitmap of routable nodes (nullptr: all)
  const uint32_t* hits;        // [N] lexical hits of this query (lexical routes)
  int lex_m;                   // query lexical keys; > 0 selects the normalised lexical law
  // per (node, head) approximate maxima of the scan, kept by node_bounds for
  // the filtered refine (nullptr: not kept); eps_abs as node_bounds uses it
  float* amax;
  float eps_abs;
  // query vectors transposed for the staged refine: [KH][ceil(nv/4)][D][4],
  // vector 4*v4 + j of kv head kh at dim d (zero past nv); nullptr: not used
  float* qT;
};

// Writes kv head kh's slice of p.qT (one block, any size).
__device__ __forceinline__ void write_qT(const RouteParams& p, int kh) {
  const int D = p.dim, nv4 = (p.nv + 3) >> 2;
  const int n = nv4 * D * 4;
  float* dst = p.qT + (int64_t)kh * n;
  const float* src = p.query + (int64_t)kh * p.nv * D;   // this kv head's nv vectors
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int j = i & 3, d = (i >> 2) % D, vi = ((i >> 2) / D) * 4 + j;
    dst[i] = vi < p.nv ? src[(int64_t)vi * D + d] : 0.0f;
  }
}

// K permutation shared by the query fragments and the scan kernels: thread
// c (lane & 3) holds, for each key row, the 16-byte chunks w = 0 .. D/32-1 at
// dims chunk_dim(c, w) .. +7: chunks 2c and 2c+1 of every 64-dim half.  With
// the 128-byte swizzle of the staged key tiles, the 8 threads of a quarter
// warp then read 8 different 16-byte bank groups.  k-step s takes halves
// 4*(s % 2) .. +3 of chunk s / 2.
__host__ __device__ constexpr int chunk_dim(int c, int w) { return (w / 2) * 64 + 16 * c + 8 * (w % 2); }

// Query preparation, one block per kv head: hi/lo fragments in mma B layout,
// the norms of that kv head's query heads, and the finite / range flags of
// its query values.  The last block to finish combines the flags into
// p.qinfo (and re-arms the counter).  K permutation: k-step s, slot (c, j)
// <-> dim chunk_dim(c, s / 2) + 4 * (s % 2) + j.
template <typename KT, int D, int NT>
__global__ void __launch_bounds__(128) query_prep_kernel(RouteParams p) {
  // the scan is launched chained to this kernel and waits for all of it
  asm volatile("griddepcontrol.launch_dependents;");
  constexpr int KSTEPS = D / 16;
  constexpr int NVP = NT * 4;  // padded vector count: hi cols [0, NVP), lo cols [NVP, 2 NVP)
  const int kh = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float limit =
      (sizeof(KT) == 2 && !std::is_same<KT, __nv_bfloat16>::value) ? 6.0e4f : kHuge;
  // this kv head's query values: heads [kh*group, (kh+1)*group) x qt tokens
  const float* qkh = p.query + (int64_t)kh * p.group * p.qt * D;
  const int nq = p.group * p.qt * D;
  int bad = 0, big = 0;
  for (int i = threadIdx.x; i < nq; i += blockDim.x) {
    const float v = qkh[i];
    bad |= !isfinite(v);
    big |= fabsf(v) > limit;
  }
  bad = __syncthreads_or(bad);
  big = __syncthreads_or(big);
  // head norms (max over query tokens), one warp per head
  for (int lh = warp; lh < p.group; lh += blockDim.x / 32) {
    const int h = kh * p.group + lh;
    float mx = 0.0f;
    for (int qi = 0; qi < p.qt; ++qi) {
      const float* q = p.query + ((int64_t)h * p.qt + qi) * D;
      float ss = 0.0f;
      for (int d = lane; d < D; d += 32) ss = fmaf(q[d], q[d], ss);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
      mx = fmaxf(mx, sqrtf(ss));
    }
    if (lane == 0) p.qnorm_h[h] = mx * (1.0f + 9.765625e-4f);
  }
  if constexpr (D == 128 || D == 64) {
    // fragments of this kv head: [t][lane][2*s + r]
    const int total = NT * 32 * KSTEPS;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
      const int s = i % KSTEPS;
      const int ln = (i / KSTEPS) % 32;
      const int t = i / (KSTEPS * 32);
      const int g = ln >> 2, c = ln & 3;
      const int col = t * 8 + g;
      const bool is_lo = col >= NVP;
      const int vi = is_lo ? col - NVP : col;
      float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (vi < p.nv) {
        const int lh = vi / p.qt, qi = vi % p.qt;
        const int h = kh * p.group + lh;
        const float* q = p.query + ((int64_t)h * p.qt + qi) * D;
        const int d0 = chunk_dim(c, s / 2) + 4 * (s % 2);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float x = q[d0 + j];
          const float xh = round_kt<KT>(x);
          v[j] = is_lo ? (x - xh) : xh;
        }
      }
      uint32_t* dst = p.frag + ((((int64_t)kh * NT + t) * 32 + ln) * (2 * KSTEPS));
      dst[2 * s] = pack2<KT>(v[0], v[1]);
      dst[2 * s + 1] = pack2<KT>(v[2], v[3]);
    }
  }
  if (p.qT) write_qT(p, kh);
  if (threadIdx.x == 0) {
    p.qparts[kh] = (bad ? 1 : 0) | (big ? 2 : 0);
    __threadfence();
    const unsigned ticket = atomicAdd(p.qcount, 1u);
    if (ticket == gridDim.x - 1) {
      __threadfence();
      int flags = 0;
      for (int k = 0; k < (int)gridDim.x; ++k) flags |= __ldcg(p.qparts + k);
      p.qinfo->finite = !(flags & 1);
      p.qinfo->fast_ok = !flags;
      p.qinfo->err = 0;
      *p.qcount = 0u;
    }
  }
}

// Approximate pass: one warp per work item (node, kv head, 128-token chunk).
template <typename KT, int D, int NT>
__global__ void __launch_bounds__(kThreads) gqa_scan_kernel(RouteParams p) {
  constexpr int KSTEPS = D / 16;
  constexpr int W = D / 32;         // 16-byte loads per key row per thread (D/4 dims)
  constexpr int NVP = NT * 4;
  const int lane = threadIdx.x & 31;
  // Chained launch after query_prep_kernel, whose outputs are read below.  No
  // early trigger: node_bounds_kernel is scheduled as the scan's CTAs exit.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (!p.qinfo->fast_ok) return;
  const int g = lane >> 2, c = lane & 3;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const KT* keys = static_cast<const KT*>(p.keys);
  // items are read 16 bytes at a time, the next one prefetched during this one
  uint4 cur = wid < p.n_items ? __ldg(reinterpret_cast<const uint4*>(p.items + wid))
                              : make_uint4(0, 0, 0, 0);
  for (int64_t it = wid; it < p.n_items; it += nw) {
    const uint4 nxt_raw = (it + nw < p.n_items)
                              ? __ldg(reinterpret_cast<const uint4*>(p.items + it + nw))
                              : make_uint4(0, 0, 0, 0);
    const uint64_t base_off = (uint64_t)cur.x | ((uint64_t)cur.y << 32);
    const int64_t node = (int64_t)cur.z;
    const int kh = (int)(cur.w & 0xFFFF);
    const int64_t t0 = 0;
    const int64_t tend = (int64_t)(cur.w >> 16);
    cur = nxt_raw;
    const KT* base = keys + base_off;
    // query fragments for this kv head
    uint32_t bq[NT][2 * KSTEPS];
    const uint32_t* fsrc = p.frag + ((int64_t)kh * NT * 32 + lane) * (2 * KSTEPS);
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int w = 0; w < 2 * KSTEPS; ++w) bq[t][w] = __ldg(fsrc + (int64_t)t * 32 * 2 * KSTEPS + w);
    float mx[NT][2];
#pragma unroll
    for (int t = 0; t < NT; ++t) mx[t][0] = mx[t][1] = 0.0f;
    // 16 key tokens x this thread's D/4 dims (chunk_dim) of rows g and g+8:
    // 8 MMAs per n-tile, then hi + lo and |.| max over the two rows.
    auto tile = [&](const uint32_t (&ra)[2 * KSTEPS], const uint32_t (&rb)[2 * KSTEPS]) {
      float acc[NT][4];
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
#pragma unroll
      for (int s = 0; s < KSTEPS; ++s) {
        const uint32_t a[4] = {ra[2 * s], rb[2 * s], ra[2 * s + 1], rb[2 * s + 1]};
#pragma unroll
        for (int t = 0; t < NT; ++t) mma16816<KT>(acc[t], a, bq[t][2 * s], bq[t][2 * s + 1]);
      }
      if constexpr (NT == 1) {
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = acc[0][j] + __shfl_xor_sync(kFull, acc[0][j], 2);
        mx[0][0] = fmaxf(mx[0][0], fmaxf(fabsf(o[0]), fabsf(o[2])));
        mx[0][1] = fmaxf(mx[0][1], fmaxf(fabsf(o[1]), fabsf(o[3])));
      } else {
#pragma unroll
        for (int t = 0; t < NT / 2; ++t) {
          const float o0 = acc[t][0] + acc[t + NT / 2][0];
          const float o1 = acc[t][1] + acc[t + NT / 2][1];
          const float o2 = acc[t][2] + acc[t + NT / 2][2];
          const float o3 = acc[t][3] + acc[t + NT / 2][3];
          mx[t][0] = fmaxf(mx[t][0], fmaxf(fabsf(o0), fabsf(o2)));
          mx[t][1] = fmaxf(mx[t][1], fmaxf(fabsf(o1), fabsf(o3)));
        }
      }
    };
    auto put = [](uint32_t* r, const uint4& v) {
      r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
    };
    int64_t tt = t0;
    // full pairs of tiles: 4 rows x W unchecked 16-byte loads in flight per thread
    for (; tt + 32 <= tend; tt += 32) {
      uint32_t ra0[2 * KSTEPS], rb0[2 * KSTEPS], ra1[2 * KSTEPS], rb1[2 * KSTEPS];
      const KT* p0 = base + (tt + g) * D;
#pragma unroll
      for (int w = 0; w < W; ++w) {
        const int d = chunk_dim(c, w);
        put(ra0 + 4 * w, ld_nc16(p0 + d));
        put(rb0 + 4 * w, ld_nc16(p0 + 8 * D + d));
        put(ra1 + 4 * w, ld_nc16(p0 + 16 * D + d));
        put(rb1 + 4 * w, ld_nc16(p0 + 24 * D + d));
      }
      tile(ra0, rb0);
      tile(ra1, rb1);
    }
    for (; tt < tend; tt += 16) {
      uint32_t ra[2 * KSTEPS], rb[2 * KSTEPS];
      const int64_t r0 = tt + g, r1 = tt + g + 8;
#pragma unroll
      for (int w = 0; w < W; ++w) {
        uint4 va = make_uint4(0, 0, 0, 0), vb = make_uint4(0, 0, 0, 0);
        if (r0 < tend) va = ld_nc16(base + r0 * D + chunk_dim(c, w));
        if (r1 < tend) vb = ld_nc16(base + r1 * D + chunk_dim(c, w));
        put(ra + 4 * w, va);
        put(rb + 4 * w, vb);
      }
      tile(ra, rb);
    }
    // max across the 8 row groups (lanes with equal c)
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float v = mx[t][e];
        v = fmaxf(v, __shfl_xor_sync(kFull, v, 4));
        v = fmaxf(v, __shfl_xor_sync(kFull, v, 8));
        v = fmaxf(v, __shfl_xor_sync(kFull, v, 16));
        mx[t][e] = v;
      }
    if (g == 0) {
      const int tiles = (NT == 1) ? 1 : NT / 2;
      const int cmax = (NT == 1) ? 2 : 4;
      if (c < cmax) {
#pragma unroll
        for (int t = 0; t < tiles; ++t)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int vi = t * 8 + 2 * c + e;
            if (vi < p.nv) {
              const int h = kh * p.group + vi / p.qt;
              const float best = mx[t][e] * p.inv_denom;
              atomicMax(p.headmax + node * p.heads + h, __float_as_uint(best));
            }
          }
      }
    }
    (void)NVP;
  }
}

// TMA-staged approximate pass.  The keys are viewed as one 2D tensor
// [rows, D] (rows = every (node, kv head, token)); each of the kTmaWarps warps
// of a CTA walks its work items (wid, wid + nw, ...) as 32-token sub-chunks
// and streams them through two shared-memory buffers with TMA box loads
// (64 dims x 32 rows, 128-byte swizzle, L2 evict-first), the next sub-chunk
// always in flight.  Fragments are read from shared memory in the chunk_dim
// permutation (conflict-free under the swizzle); the MMA and epilogue are
// those of gqa_scan_kernel.  Rows past an item's last token (the next kv
// head's rows, or zero fill past the tensor) are masked.  Every wait is
// bounded: a wait that gives up drains this warp's loads and sets qinfo->err.
constexpr int kTmaWarps = 12;
constexpr int kSubRows = 32;

template <int D>
struct TmaLayout {
  static constexpr int kBoxes = D / 64;
  static constexpr int kBox = kSubRows * 128;          // 4 KB: 32 rows x 64 dims
  static constexpr int kBuf = kBoxes * kBox;           // one sub-chunk
  static constexpr int kSmem = 1024 + kTmaWarps * 2 * kBuf;
};

__device__ __forceinline__ void tma_load_2d_g(void* dst, const CUtensorMap* map, int x, int y,
                                              uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

template <typename KT, int D, int NT>
__global__ void __launch_bounds__(kTmaWarps * 32, 1)
    gqa_scan_tma_kernel(const __grid_constant__ CUtensorMap tmap, RouteParams p) {
  using LY = TmaLayout<D>;
  constexpr int KSTEPS = D / 16;
  constexpr int W = D / 32;
  extern __shared__ unsigned char gsm_raw[];
  unsigned char* const gsm = gsm_raw + ((1024u - (smem_u32(gsm_raw) & 1023u)) & 1023u);
  __shared__ __align__(8) uint64_t bar[kTmaWarps][2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // Chained launch after query_prep_kernel, whose outputs are read below.  No
  // early trigger: node_bounds_kernel is scheduled as the scan's CTAs exit.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (!p.qinfo->fast_ok) return;
  const int g = lane >> 2, c = lane & 3;
  if (lane == 0) {
    mbar_init(&bar[warp][0], 1);
    mbar_init(&bar[warp][1], 1);
    mbar_fence_init();
  }
  __syncwarp();
  unsigned char* const buf0 = gsm + warp * 2 * LY::kBuf;
  const int64_t nw = (int64_t)gridDim.x * kTmaWarps;
  const uint64_t pol = l2_evict_first_policy();

  // the warp's sequence of sub-chunks: (item, sub) in item order
  struct Pos {
    int64_t it;
    int sub;
    uint64_t row;   // tensor row of the sub-chunk's first token
    int ntok;       // tokens of the item
  };
  auto item_at = [&](int64_t it, Pos& ps) {
    ps.it = it;
    ps.sub = 0;
    if (it < p.n_items) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p.items + it));
      const uint64_t base_off = (uint64_t)raw.x | ((uint64_t)raw.y << 32);
      ps.row = base_off / D;
      ps.ntok = (int)(raw.w >> 16);
    } else {
      ps.row = 0;
      ps.ntok = 0;
    }
  };
  auto advance = [&](Pos& ps) {
    if ((ps.sub + 1) * kSubRows < ps.ntok) {
      ++ps.sub;
    } else {
      item_at(ps.it + nw, ps);
    }
  };
  auto issue = [&](const Pos& ps, int b) {  // lane 0
    unsigned char* dst = buf0 + b * LY::kBuf;
    mbar_arrive_expect_tx(&bar[warp][b], LY::kBuf);
    const int y = (int)(ps.row + (uint64_t)ps.sub * kSubRows);
#pragma unroll
    for (int x = 0; x < LY::kBoxes; ++x)
      tma_load_2d_g(dst + x * LY::kBox, &tmap, 64 * x, y, &bar[warp][b], pol);
  };

  Pos cur, nxt;
  item_at((int64_t)blockIdx.x * kTmaWarps + warp, cur);
  nxt = cur;
  advance(nxt);
  unsigned phase_bits = 0u, pending_bits = 0u;
  if (cur.it < p.n_items) {
    if (lane == 0) issue(cur, 0);
    pending_bits |= 1u;
    if (nxt.it < p.n_items) {
      if (lane == 0) issue(nxt, 1);
      pending_bits |= 2u;
    }
  }
  bool failed = false;
  int b = 0;
  uint32_t bq[NT][2 * KSTEPS];
  float mx[NT][2];
  int64_t item_node = 0;
  int item_kh = 0;
  while (cur.it < p.n_items) {
    if (cur.sub == 0) {  // a new item: its kv head's query fragments, fresh maxima
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p.items + cur.it));
      item_node = (int64_t)raw.z;
      item_kh = (int)(raw.w & 0xFFFF);
      const uint32_t* fsrc = p.frag + ((int64_t)item_kh * NT * 32 + lane) * (2 * KSTEPS);
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int w = 0; w < 2 * KSTEPS; ++w)
          bq[t][w] = __ldg(fsrc + (int64_t)t * 32 * 2 * KSTEPS + w);
#pragma unroll
      for (int t = 0; t < NT; ++t) mx[t][0] = mx[t][1] = 0.0f;
    }
    if (!mbar_wait(&bar[warp][b], (phase_bits >> b) & 1u, kWaitLimit)) {
      failed = true;
      break;
    }
    phase_bits ^= 1u << b;
    pending_bits &= ~(1u << b);
    const unsigned char* sb = buf0 + b * LY::kBuf;
    const int valid = min(kSubRows, cur.ntok - cur.sub * kSubRows);
    // two 16-row tiles of this sub-chunk
#pragma unroll
    for (int tl = 0; tl < 2; ++tl) {
      uint32_t ra[2 * KSTEPS], rb[2 * KSTEPS];
      const int r0 = tl * 16 + g, r1 = r0 + 8;
#pragma unroll
      for (int w = 0; w < W; ++w) {
        const int box = w / 2, chunk = 2 * c + (w % 2);
        const uint4 va = *reinterpret_cast<const uint4*>(
            sb + box * LY::kBox + r0 * 128 + ((chunk ^ (r0 & 7)) * 16));
        const uint4 vb = *reinterpret_cast<const uint4*>(
            sb + box * LY::kBox + r1 * 128 + ((chunk ^ (r1 & 7)) * 16));
        const uint4 z = make_uint4(0, 0, 0, 0);
        const uint4 a = r0 < valid ? va : z;
        const uint4 bb = r1 < valid ? vb : z;
        ra[4 * w] = a.x; ra[4 * w + 1] = a.y; ra[4 * w + 2] = a.z; ra[4 * w + 3] = a.w;
        rb[4 * w] = bb.x; rb[4 * w + 1] = bb.y; rb[4 * w + 2] = bb.z; rb[4 * w + 3] = bb.w;
      }
      float acc[NT][4];
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
#pragma unroll
      for (int s2 = 0; s2 < KSTEPS; ++s2) {
        const uint32_t a[4] = {ra[2 * s2], rb[2 * s2], ra[2 * s2 + 1], rb[2 * s2 + 1]};
#pragma unroll
        for (int t = 0; t < NT; ++t) mma16816<KT>(acc[t], a, bq[t][2 * s2], bq[t][2 * s2 + 1]);
      }
      if constexpr (NT == 1) {
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = acc[0][j] + __shfl_xor_sync(kFull, acc[0][j], 2);
        mx[0][0] = fmaxf(mx[0][0], fmaxf(fabsf(o[0]), fabsf(o[2])));
        mx[0][1] = fmaxf(mx[0][1], fmaxf(fabsf(o[1]), fabsf(o[3])));
      } else {
#pragma unroll
        for (int t = 0; t < NT / 2; ++t) {
          const float o0 = acc[t][0] + acc[t + NT / 2][0];
          const float o1 = acc[t][1] + acc[t + NT / 2][1];
          const float o2 = acc[t][2] + acc[t + NT / 2][2];
          const float o3 = acc[t][3] + acc[t + NT / 2][3];
          mx[t][0] = fmaxf(mx[t][0], fmaxf(fabsf(o0), fabsf(o2)));
          mx[t][1] = fmaxf(mx[t][1], fmaxf(fabsf(o1), fabsf(o3)));
        }
      }
    }
    // buffer b is read: start the sub-chunk after nxt in it
    __syncwarp();
    fence_proxy_async_smem();
    Pos after = nxt;
    advance(after);
    if (after.it < p.n_items) {
      if (lane == 0) issue(after, b);
      pending_bits |= 1u << b;
    }
    const bool item_done = (cur.sub + 1) * kSubRows >= cur.ntok;
    if (item_done) {  // max across the 8 row groups, then one atomic per (node, head)
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float v = mx[t][e];
          v = fmaxf(v, __shfl_xor_sync(kFull, v, 4));
          v = fmaxf(v, __shfl_xor_sync(kFull, v, 8));
          v = fmaxf(v, __shfl_xor_sync(kFull, v, 16));
          mx[t][e] = v;
        }
      if (g == 0) {
        const int tiles = (NT == 1) ? 1 : NT / 2;
        const int cmax = (NT == 1) ? 2 : 4;
        if (c < cmax) {
#pragma unroll
          for (int t = 0; t < tiles; ++t)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int vi = t * 8 + 2 * c + e;
              if (vi < p.nv) {
                const int h = item_kh * p.group + vi / p.qt;
                atomicMax(p.headmax + item_node * p.heads + h,
                          __float_as_uint(mx[t][e] * p.inv_denom));
              }
            }
        }
      }
    }
    cur = nxt;
    nxt = after;
    b ^= 1;
  }
  if (failed) {
    for (int k = 0; k < 2; ++k)
      if ((pending_bits >> k) & 1u) mbar_wait(&bar[warp][k], (phase_bits >> k) & 1u, kWaitLimit);
    if (lane == 0) atomicOr(&p.qinfo->err, 1);
  }
}

// Per node: approximate score interval [lo, hi]; resets headmax.  One warp per node.
__global__ void node_bounds_kernel(RouteParams p, float eps_abs) {
  // Programmatic dependent launch: wait for the previous kernel's grid (a
  // no-op for a plain launch) before touching memory, then let the next one
  // be scheduled.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  const int lane = threadIdx.x & 31;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const bool qfinite = p.qinfo->finite != 0;
  const bool fast = p.fast && p.qinfo->fast_ok;
  for (int64_t node = wid; node < p.nodes; node += nw) {
    const int64_t T = (int64_t)(p.off[node + 1] - p.off[node]);
    float sum = 0.0f, err = 0.0f;
    bool forced = !fast;
    // heads lane, lane + 32, ... in order; the loads of up to eight of them
    // are issued together before any is used
    constexpr int kHB = 8;
    for (int h0 = lane; h0 < p.heads; h0 += 32 * kHB) {
      float bv[kHB], kmv[kHB], qnv[kHB];
#pragma unroll
      for (int j = 0; j < kHB; ++j) {
        const int h = h0 + 32 * j;
        bv[j] = kmv[j] = qnv[j] = 0.0f;
        if (h < p.heads) {
          bv[j] = __uint_as_float(p.headmax[node * p.heads + h]);
          kmv[j] = p.kmax[node * p.kh_n + h / p.group];
          qnv[j] = p.qnorm_h[h];
        }
      }
#pragma unroll
      for (int j = 0; j < kHB; ++j) {
        const int h = h0 + 32 * j;
        if (h >= p.heads) break;
        p.headmax[node * p.heads + h] = 0u;
        if (p.amax) p.amax[node * p.heads + h] = bv[j];
        const float mag = qnv[j] * kmv[j];
        if (!(mag < kHuge)) forced = true;
        sum += bv[j];
        err = fmaf(kEps * p.inv_denom, mag, err);
        err = fmaf(eps_abs * p.inv_denom, kmv[j], err);
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      sum += __shfl_xor_sync(kFull, sum, o);
      err += __shfl_xor_sync(kFull, err, o);
    }
    forced = __any_sync(kFull, forced);
    if (lane == 0) {
      float l, u;
      if (!policy::row_allowed(p.allow, node)) {
        l = u = __int_as_float(0x7FC00000);                 // filtered out: never scored
      } else if (T == 0) {
        l = u = 0.0f;                                       // exact: the reference returns 0
      } else if (!qfinite || p.key_bad[node]) {
        l = u = __int_as_float(0x7FC00000);                 // NaN: dropped
      } else if (forced) {
        l = -INFINITY;
        u = INFINITY;
      } else {
        const float s = sum / (float)p.heads;
        const float e = err / (float)p.heads + 4.0f * (float)(p.heads + 8) * 5.9604645e-08f * s +
                        1.0e-30f;
        l = s - e;
        u = s + e;
      }
      p.lo[node] = l;
      p.hi[node] = u;
    }
  }
}

// Candidate selection: L = k-th largest lower bound; candidates = nodes whose
// upper bound reaches L.  One block of 1024 threads.
__global__ void __launch_bounds__(1024) select_kernel(RouteParams p) {
  __shared__ float sh_s[32 * 32];
  __shared__ uint32_t sh_id[32 * 32];
  __shared__ float sh_L;
  asm volatile("griddepcontrol.wait;" ::: "memory");  // chained launch, as node_bounds_kernel
  asm volatile("griddepcontrol.launch_dependents;");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  WarpList list;
  list.init();
  for (int64_t base = (int64_t)warp * 32; base < p.nodes; base += 32 * 32) {
    const int64_t n = base + lane;
    float v = -INFINITY;
    if (n < p.nodes) {
      v = p.lo[n];
      if (!isfinite(v)) v = -INFINITY;
    }
    list.offer_margin(v, (uint32_t)n, lane, p.topk, 0.0f);  // only the k-th is needed
  }
  // the 32 warp lists merged pairwise in five rounds (offer_margin keeps the
  // k best by (score, node), so the merge order does not change the result)
#pragma unroll 1
  for (int stride = 16; stride >= 1; stride >>= 1) {
    if (warp >= stride && warp < 2 * stride) {
      sh_s[warp * 32 + lane] = list.s;
      sh_id[warp * 32 + lane] = list.id;
    }
    __syncthreads();
    if (warp < stride)
      list.offer_margin(sh_s[(warp + stride) * 32 + lane], sh_id[(warp + stride) * 32 + lane],
                        lane, p.topk, 0.0f);
    __syncthreads();
  }
  if (warp == 0) {
    const float L = __shfl_sync(kFull, list.s, p.topk - 1);
    if (lane == 0) sh_L = L;
  }
  __syncthreads();
  // Lexical routes order by raw / (max raw + 1e-8) + bonus: a node without
  // hits can reach the final top-k only if its raw is within a rounding of
  // that division (2^-23 relative) of the k-th raw, so the threshold drops by
  // 2^-21 relative; every allowed node with hits is a candidate as well.
  const float L = p.lex_m ? sh_L - fabsf(sh_L) * 4.76837158203125e-07f : sh_L;
  for (int64_t n = threadIdx.x; n < p.nodes; n += blockDim.x) {
    const float u = p.hi[n];
    const bool hit = p.lex_m && p.hits[n] && policy::row_allowed(p.allow, n);
    if ((u == u && u >= L) || hit) {  // not NaN
      const int slot = atomicAdd(p.cand_count, 1);
      p.cand[slot] = (uint32_t)n;
    }
  }
}

// Exact refine: one wave of blocks shares the warp units of all candidates,
// a unit being 32 tokens of one kv head of one candidate (tokens padded to a
// multiple of 32 per head).  Candidates go in chunks of 256: the block scans
// their unit counts in shared memory and each warp strides the flattened
// units, finding its candidate by binary search.  Each thread reads its key row
// once with 16-byte loads and computes the dots of every query vector of that
// kv head (the reference's sequential fp32 arithmetic, products and sums
// rounded separately), four vectors at a time; the query sits in shared memory
// when it fits (SMEM).  The per-head maximum is reduced across the warp first
// (fmaxf never returns a NaN over a number, matching std::max(best, v) keeping
// best), then one atomicMax on the bits of the non-negative float per warp
// and head.
template <typename KT, bool SMEM>
__global__ void __launch_bounds__(256) refine_kernel(RouteParams p) {
  extern __shared__ float sh_query[];
  asm volatile("griddepcontrol.wait;" ::: "memory");  // chained launch, as node_bounds_kernel
  asm volatile("griddepcontrol.launch_dependents;");
  __shared__ int64_t s_pref[kRefineChunk + 1];  // units before candidate i of the chunk
  const int count = *p.cand_count;
  if (count == 0) return;
  const int qvals = p.heads * p.qt * p.dim;
  if constexpr (SMEM) {
    for (int i = threadIdx.x; i < qvals; i += blockDim.x) sh_query[i] = p.query[i];
    __syncthreads();
  }
  const float* qbase = SMEM ? sh_query : p.query;
  constexpr int E = 16 / (int)sizeof(KT);       // keys per 16-byte load
  const KT* keys = static_cast<const KT*>(p.keys);
  const int lane = threadIdx.x & 31;
  const int nvec = p.group * p.qt;               // query vectors per kv head
  const int dim = p.dim;
  // 16-byte query loads when every query vector starts on a 16-byte boundary
  const bool qvec = dim % 4 == 0 && (reinterpret_cast<uintptr_t>(qbase) & 15) == 0;
  const bool qfinite = p.qinfo->finite != 0;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int c0 = 0; c0 < count; c0 += kRefineChunk) {
    const int cn = min(kRefineChunk, count - c0);
    int64_t my_units = 0;
    if ((int)threadIdx.x < cn) {
      const int64_t node = p.cand[c0 + threadIdx.x];
      const int64_t T = (int64_t)(p.off[node + 1] - p.off[node]);
      if (T > 0 && !p.key_bad[node] && qfinite) my_units = (int64_t)p.kh_n * ((T + 31) >> 5);
    }
    if (threadIdx.x == 0) s_pref[0] = 0;
    s_pref[threadIdx.x + 1] = my_units;
    __syncthreads();
#pragma unroll 1
    for (int o = 1; o < kRefineChunk; o <<= 1) {  // inclusive scan of s_pref[1..256]
      const int64_t v = (int)threadIdx.x >= o ? s_pref[threadIdx.x + 1 - o] : 0;
      __syncthreads();
      s_pref[threadIdx.x + 1] += v;
      __syncthreads();
    }
    const int64_t total = s_pref[cn];
    for (int64_t w = gw; w < total; w += nw) {
      int lo = 0, hi = cn - 1;  // the last candidate whose units start at or before w
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_pref[mid] <= w) lo = mid;
        else hi = mid - 1;
      }
      const int ci = c0 + lo;
      const int64_t node = p.cand[ci];
      const int64_t T = (int64_t)(p.off[node + 1] - p.off[node]);
      const int64_t tiles = (T + 31) >> 5;  // 32-token units per kv head
      const int64_t local = w - s_pref[lo];
      const int kh = (int)(local / tiles);
      const int64_t t = (local - (int64_t)kh * tiles) * 32 + lane;
      const bool live = t < T;
      const KT* base = keys + (int64_t)p.off[node] * p.kh_n * dim;
      unsigned* best_out = p.headmax + (int64_t)ci * p.heads;
      const KT* k = base + ((int64_t)kh * T + (live ? t : 0)) * dim;
      for (int v0 = 0; v0 < nvec; v0 += 4) {
        float dot[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const float* qv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int vi = min(v0 + j, nvec - 1);
          const int h = kh * p.group + vi / p.qt, qi = vi % p.qt;
          qv[j] = qbase + ((int64_t)h * p.qt + qi) * dim;
        }
        // dims d..d+E-1 of the four dots, in the reference's order
        auto dots_of = [&](const uint4& raw, int d) {
          const KT* kk = reinterpret_cast<const KT*>(&raw);
          if (qvec) {
#pragma unroll
            for (int e4 = 0; e4 < E; e4 += 4) {
              float4 q4[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) q4[j] = *reinterpret_cast<const float4*>(qv[j] + d + e4);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float kvf = key_to_f(kk[e4 + e]);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  dot[j] = __fadd_rn(dot[j], __fmul_rn((&q4[j].x)[e], kvf));
              }
            }
          } else {
#pragma unroll
            for (int e = 0; e < E; ++e) {
              const float kvf = key_to_f(kk[e]);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                dot[j] = __fadd_rn(dot[j], __fmul_rn(qv[j][d + e], kvf));
            }
          }
        };
        // four 16-byte row loads in flight per thread
        int d0 = 0;
        for (; d0 + 4 * E <= dim; d0 += 4 * E) {
          uint4 r[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) r[u] = *reinterpret_cast<const uint4*>(k + d0 + u * E);
#pragma unroll
          for (int u = 0; u < 4; ++u) dots_of(r[u], d0 + u * E);
        }
        for (; d0 < dim; d0 += E) dots_of(*reinterpret_cast<const uint4*>(k + d0), d0);
        if (p.qt4) {
          // vectors v0..v0+3 are the four query tokens of one head
          const float rb = std_max(std_max(fabsf(dot[0]), fabsf(dot[1])),
                                   std_max(fabsf(dot[2]), fabsf(dot[3])));
          float v = live ? __fmul_rn(rb, p.inv_denom) : 0.0f;
          if (!(v == v)) v = 0.0f;   // a NaN row never raises best
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
          if (lane == 0 && v > 0.0f)
            atomicMax(best_out + kh * p.group + v0 / 4, __float_as_uint(v));
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (v0 + j >= nvec) break;
            float v = live ? __fmul_rn(fabsf(dot[j]), p.inv_denom) : 0.0f;
            if (!(v == v)) v = 0.0f;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
            if (lane == 0 && v > 0.0f)
              atomicMax(best_out + kh * p.group + (v0 + j) / p.qt, __float_as_uint(v));
          }
        }
      }
    }
    __syncthreads();  // s_pref is rewritten for the next chunk
  }
}

// Exact refine with staged keys, for banks the TMA scan serves (16-bit keys,
// dim 64 or 128).  The work units are those of refine_kernel (32 tokens of one
// kv head of one candidate); a unit's 32 key rows are contiguous, so one pair
// of TMA boxes (the scan's tensor map: 32 rows x 64 dims, 128-byte swizzle)
// stages it in shared memory.  Each warp owns a contiguous range of the
// flattened units (consecutive tokens, then kv heads, then candidates), so
// the next unit follows from the current one without global reads, and keeps
// kRefStages units in flight in its own ring while it computes.  Lane l takes
// row l of the unit (token t0 + l) and reads its 16-byte chunks through the
// swizzle (eight lanes cover all 32 banks).  The dots are the reference's
// sequential fp32 sums of separately rounded products, four query vectors at
// a time: the query, transposed to [kh][v4][d][4] by the query kernel (p.qT),
// gives the four vectors' values at dim d in one 16-byte load.  The head
// maxima and atomics are those of refine_kernel.  Every wait is bounded: a
// wait that gives up drains the warp's loads and sets qinfo->err, which makes
// the route report an error.
//
// Filtered mode (NT > 0, p.amax set, the query on the fast path): a head's
// exact maximum is the exact dot of some (token, query vector) pair, and only
// pairs whose approximate dot comes within twice the approximation bound of
// the scan's approximate maximum can hold it.  Each unit first recomputes the
// scan's approximate dots on the tensor cores (the scan's query fragments and
// MMA over the staged rows), queues the pairs that pass that test, and the
// lanes then take the queued pairs one each for the exact sequential dot.
// The maximum over the queued pairs equals the maximum over all pairs, so the
// result is bit-identical to the unfiltered refine.  Heads whose |q||k| bound
// overflows the approximation's range queue every pair.
constexpr int kRefWarps = 12;
constexpr int kRefStages = 2;

template <int D>
struct RefLayout {
  static constexpr int kBuf = TmaLayout<D>::kBuf;  // one staged unit
  static constexpr int kQSlice = D * 16;           // one kv head's four query vectors
  static constexpr int kSmem = 1024 + kRefWarps * (kRefStages * kBuf + kQSlice);
};

template <typename KT, int D, int NT>
__global__ void __launch_bounds__(kRefWarps * 32, 1)
    refine_tma_kernel(const __grid_constant__ CUtensorMap tmap, RouteParams p) {
  using LY = TmaLayout<D>;
  constexpr int KSTEPS = D / 16;
  constexpr int W = D / 32;
  static_assert(kRefWarps * 32 >= kRefineChunk, "one candidate of a chunk per thread");
  extern __shared__ unsigned char rsm_raw[];
  unsigned char* const rsm = rsm_raw + ((1024u - (smem_u32(rsm_raw) & 1023u)) & 1023u);
  __shared__ __align__(8) uint64_t bar[kRefWarps][kRefStages];
  __shared__ int64_t s_pref[kRefineChunk + 1];  // units before candidate i of the chunk
  asm volatile("griddepcontrol.wait;" ::: "memory");  // chained launch, as node_bounds_kernel
  asm volatile("griddepcontrol.launch_dependents;");
  const int count = *p.cand_count;
  if (count == 0) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    for (int st = 0; st < kRefStages; ++st) mbar_init(&bar[warp][st], 1);
    mbar_fence_init();
  }
  __syncwarp();
  unsigned char* const buf0 = rsm + warp * kRefStages * LY::kBuf;
  // this warp's copy of the current kv head's transposed query (when a kv head
  // has at most four query vectors: the whole query does not fit beside the
  // rings, and read through L1 it misses, L1 being what the rings leave)
  float4* const qs_w = reinterpret_cast<float4*>(rsm + kRefWarps * kRefStages * LY::kBuf) +
                       warp * D;
  int cached_kh = -1;
  const uint64_t pol = l2_evict_first_policy();
  const bool qfinite = p.qinfo->finite != 0;
  const int nv4 = (p.nv + 3) >> 2;
  const int64_t gw = (int64_t)blockIdx.x * kRefWarps + warp;
  const int64_t nw = (int64_t)gridDim.x * kRefWarps;
  unsigned phase_bits = 0u, pending_bits = 0u;
  bool failed = false;
  // filtered mode: the scan's query fragments of the current kv head, the
  // thresholds of this lane's (head, vector) columns for the current
  // (node, kv head), and the warp's queue of pairs for the exact pass (it
  // takes the place of qs_w, which filtered mode does not use)
  const bool filt = NT > 0 && p.amax != nullptr && p.qinfo->fast_ok != 0;
  constexpr int NTR = NT > 0 ? NT : 1;
  constexpr int kTiles = NT <= 1 ? 1 : NT / 2;  // 8-vector column tiles after the hi/lo sum
  const int g = lane >> 2, c4 = lane & 3;
  const int cmax = NT <= 1 ? 2 : 4;  // lanes c4 < cmax hold distinct columns
  uint32_t bq[NTR][2 * KSTEPS];
  float thr[kTiles][2];
  int frag_kh = -1;
  int64_t thr_key = -1;
  uint16_t* const queue = reinterpret_cast<uint16_t*>(qs_w);
  static_assert(32 * 16 * sizeof(uint16_t) <= D * 16, "queue fits the query slice");
  const float* const qTf = reinterpret_cast<const float*>(p.qT);

  // A position in the chunk's flattened units.
  struct Unit {
    int lo;        // candidate index within the chunk
    int kh;
    int64_t T;     // tokens of the candidate
    int64_t t0;    // first token of the unit
    uint64_t o0;   // the candidate's first token
    int64_t node;
  };
  for (int c0 = 0; c0 < count; c0 += kRefineChunk) {
    const int cn = min(kRefineChunk, count - c0);
    int64_t my_units = 0;
    if ((int)threadIdx.x < cn) {
      const int64_t node = p.cand[c0 + threadIdx.x];
      const int64_t T = (int64_t)(p.off[node + 1] - p.off[node]);
      if (T > 0 && !p.key_bad[node] && qfinite) my_units = (int64_t)p.kh_n * ((T + 31) >> 5);
    }
    const bool scanner = threadIdx.x < kRefineChunk;
    if (threadIdx.x == 0) s_pref[0] = 0;
    if (scanner) s_pref[threadIdx.x + 1] = my_units;
    __syncthreads();
#pragma unroll 1
    for (int o = 1; o < kRefineChunk; o <<= 1) {  // inclusive scan of s_pref[1..256]
      const int64_t v = (scanner && (int)threadIdx.x >= o) ? s_pref[threadIdx.x + 1 - o] : 0;
      __syncthreads();
      if (scanner) s_pref[threadIdx.x + 1] += v;
      __syncthreads();
    }
    const int64_t total = failed ? 0 : s_pref[cn];
    // this warp's units [u_begin, u_end)
    const int64_t u_begin = total * gw / nw, u_end = total * (gw + 1) / nw;
    auto load_cand = [&](Unit& u) {
      const int64_t node = p.cand[c0 + u.lo];
      u.node = node;
      u.o0 = p.off[node];
      u.T = (int64_t)(p.off[node + 1] - u.o0);
    };
    auto decode = [&](int64_t w, Unit& u) {
      int lo = 0, hi = cn - 1;  // the last candidate whose units start at or before w
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_pref[mid] <= w) lo = mid;
        else hi = mid - 1;
      }
      u.lo = lo;
      load_cand(u);
      const int64_t tiles = (u.T + 31) >> 5;
      const int64_t local = w - s_pref[lo];
      u.kh = (int)(local / tiles);
      u.t0 = (local - (int64_t)u.kh * tiles) * 32;
    };
    auto advance = [&](Unit& u) {  // the next unit (valid while units remain)
      u.t0 += 32;
      if (u.t0 < u.T) return;
      u.t0 = 0;
      if (++u.kh < p.kh_n) return;
      u.kh = 0;
      do {
        ++u.lo;
      } while (u.lo < cn - 1 && s_pref[u.lo + 1] == s_pref[u.lo]);  // candidates without units
      if (u.lo < cn) load_cand(u);
    };
    auto issue = [&](const Unit& u, int st) {
      if (lane == 0) {
        const int row = (int)(u.o0 * (uint64_t)p.kh_n + (uint64_t)u.kh * u.T + u.t0);
        unsigned char* dst = buf0 + st * LY::kBuf;
        mbar_arrive_expect_tx(&bar[warp][st], LY::kBuf);
#pragma unroll
        for (int x = 0; x < LY::kBoxes; ++x)
          tma_load_2d_g(dst + x * LY::kBox, &tmap, 64 * x, row, &bar[warp][st], pol);
      }
      pending_bits |= 1u << st;
    };
    Unit cur, fetch;
    if (u_begin < u_end) {
      decode(u_begin, cur);
      fetch = cur;
    }
    int64_t w_fetch = u_begin;
    for (int st = 0; st < kRefStages && w_fetch < u_end; ++st, ++w_fetch) {
      issue(fetch, st);
      if (w_fetch + 1 < u_end) advance(fetch);
    }
    int st = 0;
    for (int64_t w = u_begin; w < u_end; ++w) {
      if (!mbar_wait(&bar[warp][st], (phase_bits >> st) & 1u, kWaitLimit)) {
        failed = true;
        break;
      }
      phase_bits ^= 1u << st;
      pending_bits &= ~(1u << st);
      const unsigned char* sb = buf0 + st * LY::kBuf;
      const bool live = cur.t0 + lane < cur.T;  // rows past the candidate's tokens are masked
      unsigned* best_out = p.headmax + (int64_t)(c0 + cur.lo) * p.heads;
      const float4* qk = reinterpret_cast<const float4*>(p.qT) + (int64_t)cur.kh * nv4 * D;
      if constexpr (NT > 0) {
        if (filt) {
          if (cur.kh != frag_kh) {
            const uint32_t* fsrc = p.frag + ((int64_t)cur.kh * NT * 32 + lane) * (2 * KSTEPS);
#pragma unroll
            for (int t = 0; t < NT; ++t)
#pragma unroll
              for (int w2 = 0; w2 < 2 * KSTEPS; ++w2)
                bq[t][w2] = __ldg(fsrc + (int64_t)t * 32 * 2 * KSTEPS + w2);
            frag_kh = cur.kh;
          }
          const int64_t key = cur.node * p.kh_n + cur.kh;
          if (key != thr_key) {
            // column (t, e) of this lane is query vector t*8 + 2*c4 + e; a
            // NaN threshold never queues (lanes without a column, vectors
            // past nv), -inf queues every live row (forced heads)
            const float km = p.kmax[key];
#pragma unroll
            for (int t = 0; t < kTiles; ++t)
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int vi = t * 8 + 2 * c4 + e;
                float th = __int_as_float(0x7FC00000);
                if (c4 < cmax && vi < p.nv) {
                  const int h = cur.kh * p.group + vi / p.qt;
                  const float qn = p.qnorm_h[h];
                  const float mag = qn * km;
                  if (!(mag < kHuge)) {
                    th = -INFINITY;
                  } else {
                    const float err = kEps * p.inv_denom * mag + p.eps_abs * p.inv_denom * km;
                    th = p.amax[cur.node * p.heads + h] - 2.0f * err;
                  }
                }
                thr[t][e] = th;
              }
            thr_key = key;
          }
          const int valid = (int)(cur.T - cur.t0 < 32 ? cur.T - cur.t0 : 32);
          const unsigned below = (1u << lane) - 1u;
          int qn_w = 0;  // pairs queued by the warp (uniform)
#pragma unroll
          for (int tl = 0; tl < 2; ++tl) {
            uint32_t ra[2 * KSTEPS], rb[2 * KSTEPS];
            const int r0 = tl * 16 + g, r1 = r0 + 8;
#pragma unroll
            for (int w2 = 0; w2 < W; ++w2) {
              const int box = w2 / 2, chunk = 2 * c4 + (w2 % 2);
              const uint4 va = *reinterpret_cast<const uint4*>(
                  sb + box * LY::kBox + r0 * 128 + ((chunk ^ (r0 & 7)) * 16));
              const uint4 vb = *reinterpret_cast<const uint4*>(
                  sb + box * LY::kBox + r1 * 128 + ((chunk ^ (r1 & 7)) * 16));
              ra[4 * w2] = va.x; ra[4 * w2 + 1] = va.y; ra[4 * w2 + 2] = va.z; ra[4 * w2 + 3] = va.w;
              rb[4 * w2] = vb.x; rb[4 * w2 + 1] = vb.y; rb[4 * w2 + 2] = vb.z; rb[4 * w2 + 3] = vb.w;
            }
            float acc[NTR][4];
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
#pragma unroll
            for (int s2 = 0; s2 < KSTEPS; ++s2) {
              const uint32_t a[4] = {ra[2 * s2], rb[2 * s2], ra[2 * s2 + 1], rb[2 * s2 + 1]};
#pragma unroll
              for (int t = 0; t < NT; ++t) mma16816<KT>(acc[t], a, bq[t][2 * s2], bq[t][2 * s2 + 1]);
            }
            // o[t][j]: j = 0/1 row r0 columns e = 0/1, j = 2/3 row r1
            float o[kTiles][4];
            if constexpr (NT == 1) {
#pragma unroll
              for (int j = 0; j < 4; ++j) o[0][j] = acc[0][j] + __shfl_xor_sync(kFull, acc[0][j], 2);
            } else {
#pragma unroll
              for (int t = 0; t < kTiles; ++t)
#pragma unroll
                for (int j = 0; j < 4; ++j) o[t][j] = acc[t][j] + acc[t + kTiles][j];
            }
#pragma unroll
            for (int t = 0; t < kTiles; ++t)
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int e = j & 1;
                const int r = (j < 2) ? r0 : r1;
                const float th = thr[t][e];
                const bool m = r < valid && (th == -INFINITY || fabsf(o[t][j]) * p.inv_denom >= th);
                const unsigned bal = __ballot_sync(kFull, m);
                if (m) queue[qn_w + __popc(bal & below)] = (uint16_t)((r << 8) | (t * 8 + 2 * c4 + e));
                qn_w += __popc(bal);
              }
          }
          __syncwarp();
          // exact pass: lane i takes queued pairs i, i + 32, ...
          for (int i = lane; i < qn_w; i += 32) {
            const int ent = queue[i];
            const int r = ent >> 8, vi = ent & 255;
            const float* qv = qTf + (((int64_t)cur.kh * nv4 + (vi >> 2)) * D) * 4 + (vi & 3);
            float dot = 0.0f;
#pragma unroll 4
            for (int c = 0; c < D / 8; ++c) {
              const uint4 raw = *reinterpret_cast<const uint4*>(
                  sb + (c / 8) * LY::kBox + r * 128 + (((c % 8) ^ (r & 7)) * 16));
              const KT* kk = reinterpret_cast<const KT*>(&raw);
#pragma unroll
              for (int e = 0; e < 8; ++e)
                dot = __fadd_rn(dot, __fmul_rn(__ldg(qv + (c * 8 + e) * 4), key_to_f(kk[e])));
            }
            float v = __fmul_rn(fabsf(dot), p.inv_denom);
            if (!(v == v)) v = 0.0f;  // a NaN row never raises best
            if (v > 0.0f) atomicMax(best_out + cur.kh * p.group + vi / p.qt, __float_as_uint(v));
          }
        }
      }
      if (!filt && nv4 == 1 && cur.kh != cached_kh) {
        __syncwarp();
        for (int i = lane; i < D; i += 32) qs_w[i] = __ldg(qk + i);
        __syncwarp();
        cached_kh = cur.kh;
      }
      for (int v4 = 0; v4 < (filt ? 0 : nv4); ++v4) {
        const float4* q = qk + (int64_t)v4 * D;
        // the four vectors' values at dim d: shared memory or global
        auto qat = [&](int d) -> float4 { return nv4 == 1 ? qs_w[d] : __ldg(q + d); };
        float dot[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int c = 0; c < D / 8; ++c) {  // 16-byte chunk c: dims 8c .. 8c+7, in order
          const uint4 raw = *reinterpret_cast<const uint4*>(
              sb + (c / 8) * LY::kBox + lane * 128 + (((c % 8) ^ (lane & 7)) * 16));
          const KT* kk = reinterpret_cast<const KT*>(&raw);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float kf = key_to_f(kk[e]);
            const float4 qv = qat(c * 8 + e);
            dot[0] = __fadd_rn(dot[0], __fmul_rn(qv.x, kf));
            dot[1] = __fadd_rn(dot[1], __fmul_rn(qv.y, kf));
            dot[2] = __fadd_rn(dot[2], __fmul_rn(qv.z, kf));
            dot[3] = __fadd_rn(dot[3], __fmul_rn(qv.w, kf));
          }
        }
        const int v0 = v4 * 4;
        if (p.qt4) {
          // vectors v0..v0+3 are the four query tokens of one head
          const float rb = std_max(std_max(fabsf(dot[0]), fabsf(dot[1])),
                                   std_max(fabsf(dot[2]), fabsf(dot[3])));
          float v = live ? __fmul_rn(rb, p.inv_denom) : 0.0f;
          if (!(v == v)) v = 0.0f;   // a NaN row never raises best
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
          if (lane == 0 && v > 0.0f)
            atomicMax(best_out + cur.kh * p.group + v0 / 4, __float_as_uint(v));
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (v0 + j >= p.nv) break;
            float v = live ? __fmul_rn(fabsf(dot[j]), p.inv_denom) : 0.0f;
            if (!(v == v)) v = 0.0f;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
            if (lane == 0 && v > 0.0f)
              atomicMax(best_out + cur.kh * p.group + (v0 + j) / p.qt, __float_as_uint(v));
          }
        }
      }
      // stage st is read: the unit kRefStages ahead goes into it
      __syncwarp();
      fence_proxy_async_smem();
      if (w_fetch < u_end) {
        issue(fetch, st);
        if (w_fetch + 1 < u_end) advance(fetch);
        ++w_fetch;
      }
      if (w + 1 < u_end) advance(cur);
      st = (st + 1 == kRefStages) ? 0 : st + 1;
    }
    __syncthreads();  // s_pref is rewritten for the next chunk
  }
  if (failed) {
    for (int k = 0; k < kRefStages; ++k)
      if ((pending_bits >> k) & 1u) mbar_wait(&bar[warp][k], (phase_bits >> k) & 1u, kWaitLimit);
    if (lane == 0) atomicOr(&p.qinfo->err, 1);
  }
}

// Final scores of the candidates (sequential fp32 head sum, as the reference)
// and the exact top-k.  One warp.  Lexical routes (lex_m > 0) rank by the
// reference's S = raw / (max raw + 1e-8) + hits / m instead
// (cpp/grm_runtime.cpp:4840-4867): the raws are kept in lo[node] by the first
// pass and the maximum over the candidates (which contain the top raw) sets
// the norm.
__global__ void finalize_kernel(RouteParams p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // chained launch, as node_bounds_kernel
  asm volatile("griddepcontrol.launch_dependents;");
  // head maxima of 32 candidates x 64 heads, staged by coalesced loads (and
  // reset for the next route in the same pass); lane c then sums candidate
  // c's heads in order from shared memory
  __shared__ float sh_best[32][65];
  const int lane = threadIdx.x;
  const int count = *p.cand_count;
  WarpList list;
  list.init();
  float max_abs = 0.0f;
  for (int base = 0; base < count; base += 32) {
    const int ci = base + lane;
    const int nc = min(32, count - base);
    float total = 0.0f;
    for (int h0 = 0; h0 < p.heads; h0 += 64) {
      const int hn = min(64, p.heads - h0);
      __syncwarp();
      // eight candidates' loads in flight at a time, then their stores
      for (int c0 = 0; c0 < nc; c0 += 8) {
        unsigned a[8], b[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const unsigned* bc = p.headmax + (int64_t)(base + c0 + j) * p.heads + h0;
          a[j] = (c0 + j < nc && lane < hn) ? bc[lane] : 0u;
          b[j] = (c0 + j < nc && lane + 32 < hn) ? bc[lane + 32] : 0u;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (c0 + j >= nc) break;
          unsigned* bc = p.headmax + (int64_t)(base + c0 + j) * p.heads + h0;
          if (lane < hn) {
            sh_best[c0 + j][lane] = __uint_as_float(a[j]);
            bc[lane] = 0u;
          }
          if (lane + 32 < hn) {
            sh_best[c0 + j][lane + 32] = __uint_as_float(b[j]);
            bc[lane + 32] = 0u;
          }
        }
      }
      __syncwarp();
      if (ci < count)
        for (int h = 0; h < hn; ++h) total = __fadd_rn(total, sh_best[lane][h]);
    }
    float score = -INFINITY;
    uint32_t node = kNoRow;
    if (ci < count) {
      node = p.cand[ci];
      const int64_t T = (int64_t)(p.off[node + 1] - p.off[node]);
      if (T == 0) {
        score = 0.0f;
      } else if (p.key_bad[node] || !p.qinfo->finite) {
        score = __int_as_float(0x7FC00000);
      } else {
        score = __fdiv_rn(total, (float)p.heads);
      }
      if (p.lex_m) {
        p.lo[node] = score;
        if (isfinite(score)) max_abs = fmaxf(max_abs, fabsf(score));
      }
    }
    if (!p.lex_m) list.offer(score, node, lane);
  }
  if (p.lex_m) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) max_abs = fmaxf(max_abs, __shfl_xor_sync(kFull, max_abs, o));
    const float norm = __fadd_rn(max_abs, 1.0e-8f);
    for (int base = 0; base < count; base += 32) {
      const int ci = base + lane;
      float S = -INFINITY;
      uint32_t node = kNoRow;
      if (ci < count) {
        node = p.cand[ci];
        const float raw = p.lo[node];
        if (isfinite(raw))
          S = __fadd_rn(__fdiv_rn(raw, norm), __fdiv_rn((float)p.hits[node], (float)p.lex_m));
      }
      list.offer(S, node, lane);
    }
  }
  const bool failed = p.qinfo->err != 0;  // a bounded wait of the scan gave up
  const bool ok = !failed && lane < p.topk && isfinite(list.s) && list.id != kNoRow;
  const unsigned m = __ballot_sync(kFull, ok);
  if (lane < p.topk) {
    const uint64_t id = ok ? (uint64_t)list.id + p.id_offset : UINT64_MAX;
    const float sc = ok ? list.s : __int_as_float(0x7FC00000);
    p.result->ids[lane] = id;
    p.result->scores[lane] = sc;
    if (p.out_ids) p.out_ids[lane] = id;
    if (p.out_scores) p.out_scores[lane] = sc;
  }
  if (lane == 0) {
    p.result->count = failed ? -1 : __popc(m);
    p.result->cands = count;
    if (p.refined_total) atomicAdd(p.refined_total, (unsigned long long)count);
    *p.cand_count = 0;
  }
}

}  // namespace gqa
}  // namespace grm_b200

using namespace grm_b200;
using namespace grm_b200::gqa;

struct grm_b200_gqa_bank {
  int device = 0;
  int dtype = GRM_B200_BF16;
  int64_t nodes = 0;
  int kh_n = 0;
  int dim = 0;
  bool owns_keys = true;
  void* d_keys = nullptr;
  uint64_t* d_off = nullptr;
  std::vector<uint64_t> h_off;
  Item* d_items = nullptr;
  int64_t n_items = 0;
  float* d_kmax = nullptr;
  unsigned char* d_key_bad = nullptr;
  unsigned* d_headmax = nullptr;
  float* d_amax = nullptr;   // [nodes, heads] scan maxima kept for the filtered refine
  int headmax_heads = 0;
  float* d_lo = nullptr;
  float* d_hi = nullptr;
  uint32_t* d_cand = nullptr;
  int* d_cand_count = nullptr;
  uint32_t* d_frag = nullptr;
  size_t frag_cap = 0;
  float* d_qnorm = nullptr;
  int qnorm_cap = 0;
  QueryInfo* d_qinfo = nullptr;
  int* d_qparts = nullptr;
  float* d_qT = nullptr;     // transposed query for refine_tma_kernel
  size_t qT_cap = 0;         // floats
  unsigned* d_qcount = nullptr;
  Result* d_result = nullptr;
  Result* h_result = nullptr;
  float* d_queries = nullptr;
  size_t dq_cap = 0;
  int grid_scan = 1;
  bool tma = false;          // scan with gqa_scan_tma_kernel
  int grid_tma = 1;
  CUtensorMap tmap;          // keys as a 2D tensor [rows, dim]
  int sms = 1;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  std::mutex mu;
  ErrorSlot err;
  uint64_t routes = 0;
  unsigned long long* d_refined = nullptr;  // counted by finalize_kernel
  grm_b200::policy::Policy pol;             // lexical keys, filter codes, active flags
};

namespace {

bool fast_bank(const grm_b200_gqa_bank* b) {
  return (b->dtype == GRM_B200_BF16 || b->dtype == GRM_B200_F16) && (b->dim == 128 || b->dim == 64);
}

int nt_for(int nv) { return nv <= 4 ? 1 : (nv <= 8 ? 2 : (nv <= 16 ? 4 : 0)); }

// Launch chained to the previous kernel of the stream (programmatic stream
// serialization); the kernel waits on that grid with griddepcontrol.wait.
template <typename... KArgs, typename... Args>
cudaError_t launch_chained(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                           cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <typename KT, int D, int NT>
void launch_fast(grm_b200_gqa_bank* b, const RouteParams& p) {
  query_prep_kernel<KT, D, NT><<<b->kh_n, 128, 0, b->stream>>>(p);
  if (b->n_items <= 0) return;
  if (b->tma)
    launch_chained(gqa_scan_tma_kernel<KT, D, NT>, dim3(b->grid_tma), dim3(kTmaWarps * 32),
                   (size_t)TmaLayout<D>::kSmem, b->stream, b->tmap, p);
  else
    launch_chained(gqa_scan_kernel<KT, D, NT>, dim3(b->grid_scan), dim3(kThreads), 0, b->stream, p);
}

template <typename KT, int D>
cudaError_t tma_smem_attr() {
  cudaError_t e = cudaSuccess;
  for (auto fn : {gqa_scan_tma_kernel<KT, D, 1>, gqa_scan_tma_kernel<KT, D, 2>,
                  gqa_scan_tma_kernel<KT, D, 4>})
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               TmaLayout<D>::kSmem);
  for (auto fn : {refine_tma_kernel<KT, D, 0>, refine_tma_kernel<KT, D, 1>,
                  refine_tma_kernel<KT, D, 2>, refine_tma_kernel<KT, D, 4>})
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, RefLayout<D>::kSmem);
  return e;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// The TMA-staged scan for 16-bit banks of dim 64/128 whose row count fits a
// tensor-map coordinate; otherwise the direct-load scan stays in use.
int setup_tma(grm_b200_gqa_bank* b, int sms) {
  b->tma = false;
  if (!(b->dtype == GRM_B200_BF16 || b->dtype == GRM_B200_F16) ||
      !(b->dim == 64 || b->dim == 128) || b->n_items <= 0)
    return 0;
  const uint64_t rows = b->h_off[b->nodes] * (uint64_t)b->kh_n;
  if (rows >= ((uint64_t)1 << 31) || (reinterpret_cast<uintptr_t>(b->d_keys) & 15) != 0) return 0;
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return 0;
  const cuuint64_t dims[2] = {(cuuint64_t)b->dim, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)b->dim * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)kSubRows};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt =
      b->dtype == GRM_B200_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (enc(&b->tmap, dt, 2, b->d_keys, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return 0;
  cudaError_t e;
  if (b->dtype == GRM_B200_BF16)
    e = b->dim == 128 ? tma_smem_attr<__nv_bfloat16, 128>() : tma_smem_attr<__nv_bfloat16, 64>();
  else
    e = b->dim == 128 ? tma_smem_attr<__half, 128>() : tma_smem_attr<__half, 64>();
  if (e != cudaSuccess) return cuda_status(e);
  b->grid_tma = (int)std::max<int64_t>(1, std::min<int64_t>(sms, ceil_div64(b->n_items, kTmaWarps)));
  b->tma = true;
  return 0;
}

template <typename KT>
int launch_fast_dims(grm_b200_gqa_bank* b, const RouteParams& p, int nt) {
  if (b->dim == 128) {
    if (nt == 1) launch_fast<KT, 128, 1>(b, p);
    else if (nt == 2) launch_fast<KT, 128, 2>(b, p);
    else launch_fast<KT, 128, 4>(b, p);
  } else {
    if (nt == 1) launch_fast<KT, 64, 1>(b, p);
    else if (nt == 2) launch_fast<KT, 64, 2>(b, p);
    else launch_fast<KT, 64, 4>(b, p);
  }
  return cuda_status(cudaGetLastError());
}

// Query prep for banks outside the fast path: only the finite flag and norms.
__global__ void query_info_kernel(RouteParams p) {
  __shared__ int s_bad;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  const int nq = p.heads * p.qt * p.dim;
  for (int i = threadIdx.x; i < nq; i += blockDim.x)
    if (!isfinite(p.query[i])) s_bad = 1;
  for (int h = threadIdx.x; h < p.heads; h += blockDim.x) p.qnorm_h[h] = 0.0f;
  if (p.qT)
    for (int kh = 0; kh < p.kh_n; ++kh) write_qT(p, kh);
  __syncthreads();
  if (threadIdx.x == 0) {
    p.qinfo->finite = !s_bad;
    p.qinfo->fast_ok = 0;
  }
}

constexpr int kRefineSmemMax = 96 * 1024;
constexpr int kRefineSmemCopy = 16 * 1024;  // largest query staged in shared memory

template <typename KT>
cudaError_t launch_refine(grm_b200_gqa_bank* b, const RouteParams& p) {
  if constexpr (sizeof(KT) == 2) {
    if (p.qT) {  // staged keys (the TMA scan's tensor map): one CTA per SM
      const dim3 grid(std::max(1, b->sms)), block(kRefWarps * 32);
      // filtered when the scan ran with fragments of nt tiles
      const int nt = p.amax ? nt_for(p.nv) : 0;
      auto go = [&](auto kernel, size_t smem) {
        return launch_chained(kernel, grid, block, smem, b->stream, b->tmap, p);
      };
      if (b->dim == 128) {
        constexpr size_t sm = RefLayout<128>::kSmem;
        if (nt == 1) return go(refine_tma_kernel<KT, 128, 1>, sm);
        if (nt == 2) return go(refine_tma_kernel<KT, 128, 2>, sm);
        if (nt == 4) return go(refine_tma_kernel<KT, 128, 4>, sm);
        return go(refine_tma_kernel<KT, 128, 0>, sm);
      }
      constexpr size_t sm = RefLayout<64>::kSmem;
      if (nt == 1) return go(refine_tma_kernel<KT, 64, 1>, sm);
      if (nt == 2) return go(refine_tma_kernel<KT, 64, 2>, sm);
      if (nt == 4) return go(refine_tma_kernel<KT, 64, 4>, sm);
      return go(refine_tma_kernel<KT, 64, 0>, sm);
    }
  }
  // one wave: as many blocks as are resident together (measured once)
  static int per_sm[2][64] = {};
  const bool smem_q = sizeof(float) * (size_t)p.heads * p.qt * p.dim <= (size_t)kRefineSmemCopy;
  int& occ = per_sm[smem_q ? 1 : 0][b->device & 63];
  if (occ == 0) {
    const size_t qb = smem_q ? sizeof(float) * (size_t)p.heads * p.qt * p.dim : 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &occ, smem_q ? refine_kernel<KT, true> : refine_kernel<KT, false>, kRefineChunk,
            qb) != cudaSuccess || occ < 1)
      occ = 1;
  }
  dim3 grid(std::max(1, b->sms) * occ);
  const size_t qbytes = sizeof(float) * (size_t)p.heads * p.qt * p.dim;
  // A block takes about one 32-token chunk per kv head of a candidate, so
  // copying a large query into shared memory costs more than it saves: large
  // queries are read through L1 instead.
  if (qbytes <= (size_t)kRefineSmemCopy) {
    static bool attr_set[64] = {};
    if (!attr_set[b->device]) {
      cudaFuncSetAttribute(refine_kernel<KT, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kRefineSmemMax);
      attr_set[b->device] = true;
    }
    return launch_chained(refine_kernel<KT, true>, grid, dim3(kRefineChunk), qbytes, b->stream, p);
  }
  return launch_chained(refine_kernel<KT, false>, grid, dim3(kRefineChunk), 0, b->stream, p);
}

int ensure_heads(grm_b200_gqa_bank* b, int heads, int nt) {
  if (heads > b->headmax_heads) {
    if (b->d_headmax) cudaFree(b->d_headmax);
    if (b->d_amax) cudaFree(b->d_amax);
    b->d_headmax = nullptr;
    b->d_amax = nullptr;
    b->headmax_heads = 0;
    const size_t n = (size_t)b->nodes * heads;
    cudaError_t e = cudaMalloc(&b->d_headmax, n * sizeof(unsigned));
    if (e == cudaSuccess && b->tma) e = cudaMalloc(&b->d_amax, n * sizeof(float));
    if (e == cudaSuccess) e = cudaMemsetAsync(b->d_headmax, 0, n * sizeof(unsigned), b->stream);
    // later launches may use another stream: finish the zero fill now (first use only)
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    if (e != cudaSuccess) return b->err.set(cuda_status(e), "GQA scratch allocation failed");
    b->headmax_heads = heads;
  }
  if (heads > b->qnorm_cap) {
    if (b->d_qnorm) cudaFree(b->d_qnorm);
    b->d_qnorm = nullptr;
    b->qnorm_cap = 0;
    cudaError_t e = cudaMalloc(&b->d_qnorm, sizeof(float) * heads);
    if (e != cudaSuccess) return b->err.set(cuda_status(e), "GQA scratch allocation failed");
    b->qnorm_cap = heads;
  }
  const size_t frag = (size_t)b->kh_n * std::max(nt, 1) * 32 * 16;
  if (frag > b->frag_cap) {
    if (b->d_frag) cudaFree(b->d_frag);
    b->d_frag = nullptr;
    b->frag_cap = 0;
    cudaError_t e = cudaMalloc(&b->d_frag, frag * sizeof(uint32_t));
    if (e != cudaSuccess) return b->err.set(cuda_status(e), "GQA scratch allocation failed");
    b->frag_cap = frag;
  }
  return 0;
}

// The transposed query of refine_tma_kernel: KH x ceil(nv / 4) x D x 4 floats.
int ensure_qT(grm_b200_gqa_bank* b, int nv) {
  const size_t n = (size_t)b->kh_n * (size_t)((nv + 3) / 4) * (size_t)b->dim * 4;
  if (n > b->qT_cap) {
    if (b->d_qT) cudaFree(b->d_qT);
    b->d_qT = nullptr;
    b->qT_cap = 0;
    cudaError_t e = cudaMalloc(&b->d_qT, n * sizeof(float));
    if (e != cudaSuccess) return b->err.set(cuda_status(e), "GQA scratch allocation failed");
    b->qT_cap = n;
  }
  return 0;
}

// `use_bank_stream`: launch on the bank's private stream (synchronous entry
// points); otherwise on `stream`, where 0 is the legacy default stream.
// `allow`, `hits`, `lex_m`: route policy inputs (see RouteParams).
int route_one(grm_b200_gqa_bank* b, const float* dq, int heads, int qt, int topk,
              bool use_bank_stream = true, cudaStream_t stream = nullptr,
              uint64_t* out_ids = nullptr, float* out_scores = nullptr,
              uint64_t id_offset = 0, const uint32_t* allow = nullptr,
              const uint32_t* hits = nullptr, int lex_m = 0) {
  if (use_bank_stream) stream = b->stream;
  const int group = heads / b->kh_n;
  const int nv = group * qt;
  const int nt = nt_for(nv);
  const bool fast = fast_bank(b) && nt > 0;
  int rc = ensure_heads(b, heads, nt);
  if (rc == 0 && b->tma) rc = ensure_qT(b, nv);
  if (rc) return rc;
  RouteParams p;
  p.keys = b->d_keys;
  p.off = b->d_off;
  p.nodes = b->nodes;
  p.kh_n = b->kh_n;
  p.dim = b->dim;
  p.heads = heads;
  p.qt = qt;
  p.group = group;
  p.nv = nv;
  p.inv_denom = 1.0f / std::sqrt(static_cast<float>(b->dim));  // cpp/grm_runtime.cpp:3639-3640
  p.query = dq;
  p.items = b->d_items;
  p.n_items = b->n_items;
  p.kmax = b->d_kmax;
  p.key_bad = b->d_key_bad;
  p.headmax = b->d_headmax;
  p.lo = b->d_lo;
  p.hi = b->d_hi;
  p.cand = b->d_cand;
  p.cand_count = b->d_cand_count;
  p.frag = b->d_frag;
  p.qnorm_h = b->d_qnorm;
  p.qinfo = b->d_qinfo;
  p.qparts = b->d_qparts;
  p.qcount = b->d_qcount;
  p.topk = topk;
  p.fast = fast ? 1 : 0;
  p.result = b->d_result;
  p.refined_total = b->d_refined;
  p.qt4 = (qt == 4) ? 1 : 0;
  p.out_ids = out_ids;
  p.out_scores = out_scores;
  p.id_offset = id_offset;
  p.allow = allow;
  p.hits = hits;
  p.lex_m = lex_m;
  p.qT = b->tma ? b->d_qT : nullptr;
  // the filtered refine (approximate dots on tensor cores, exact dots only for
  // tokens the scan's maxima cannot rule out) needs the scan's fragments
  p.amax = (b->tma && fast) ? b->d_amax : nullptr;
  // absolute query-representation error of an f16 split (subnormal lo parts)
  p.eps_abs = (b->dtype == GRM_B200_F16) ? 2.0e-7f * std::sqrt((float)b->dim) : 1.0e-30f;
  cudaStream_t saved = b->stream;
  b->stream = stream;  // every launch below goes to the caller's stream
  struct Restore {
    grm_b200_gqa_bank* b;
    cudaStream_t s;
    ~Restore() { b->stream = s; }
  } restore{b, saved};
  if (fast) {
    rc = (b->dtype == GRM_B200_BF16) ? launch_fast_dims<__nv_bfloat16>(b, p, nt)
                                     : launch_fast_dims<__half>(b, p, nt);
  } else {
    query_info_kernel<<<1, 256, 0, b->stream>>>(p);
    rc = cuda_status(cudaGetLastError());
  }
  if (rc) return b->err.set(rc, "GQA scan launch failed");
  const float eps_abs = p.eps_abs;
  const int nb_grid = (int)std::min<int64_t>(ceil_div64(b->nodes, kWarps), (int64_t)b->sms * 8);
  cudaError_t le =
      launch_chained(node_bounds_kernel, dim3(nb_grid), dim3(kThreads), 0, b->stream, p, eps_abs);
  if (le == cudaSuccess) le = launch_chained(select_kernel, dim3(1), dim3(1024), 0, b->stream, p);
  if (le == cudaSuccess) {
    switch (b->dtype) {
      case GRM_B200_BF16: le = launch_refine<__nv_bfloat16>(b, p); break;
      case GRM_B200_F16: le = launch_refine<__half>(b, p); break;
      default: le = launch_refine<float>(b, p); break;
    }
  }
  if (le == cudaSuccess) le = launch_chained(finalize_kernel, dim3(1), dim3(32), 0, b->stream, p);
  if (le == cudaSuccess) le = cudaGetLastError();
  rc = cuda_status(le);
  if (rc) return b->err.set(rc, "GQA route launch failed: %s", cudaGetErrorString(le));
  return 0;
}

int route_device_queries(grm_b200_gqa_bank* b, const float* dq, int qc, int heads, int qt,
                         int warmup, int topk, uint64_t* out_ids, float* out_scores,
                         float* elapsed) {
  if (!dq || !out_ids || qc <= 0 || heads <= 0 || qt <= 0 || heads % b->kh_n != 0 || warmup < 0 ||
      warmup >= qc || topk <= 0 || topk > GRM_B200_MAX_TOPK)
    return b->err.set(GRM_B200_EINVAL,
                      "invalid GQA route arguments (queries=%d heads=%d qt=%d kv_heads=%d topk=%d)",
                      qc, heads, qt, b->kh_n, topk);
  cudaError_t e = cudaSetDevice(b->device);
  if (e != cudaSuccess) return b->err.set(cuda_status(e), "cudaSetDevice failed");
  const int64_t qsize = (int64_t)heads * qt * b->dim;
  for (int i = 0; i < qc; ++i) {
    if (i == warmup) cudaEventRecord(b->ev0, b->stream);
    int rc = route_one(b, dq + i * qsize, heads, qt, topk);
    if (rc) return rc;
    e = cudaMemcpyAsync(b->h_result, b->d_result, sizeof(Result), cudaMemcpyDeviceToHost, b->stream);
    // the end event goes in before the last wait, so timing costs no extra round trip
    if (e == cudaSuccess && i == qc - 1) e = cudaEventRecord(b->ev1, b->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    if (e != cudaSuccess) return b->err.set(cuda_status(e), "GQA route failed: %s", cudaGetErrorString(e));
    if (b->h_result->count < 0)
      return b->err.set(GRM_B200_KERNEL_BASE + 1, "GQA scan: a bounded device wait gave up (query %d)", i);
    for (int j = 0; j < topk; ++j) {
      out_ids[(int64_t)i * topk + j] = b->h_result->ids[j];
      if (out_scores) out_scores[(int64_t)i * topk + j] = b->h_result->scores[j];
    }
  }
  e = cudaEventSynchronize(b->ev1);
  float ms = 0.0f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, b->ev0, b->ev1);
  if (e != cudaSuccess) return b->err.set(cuda_status(e), "GQA route timing failed");
  if (elapsed) *elapsed = ms;
  b->routes += (uint64_t)qc;
  return 0;
}

void bank_free(grm_b200_gqa_bank* b) {
  if (!b) return;
  cudaSetDevice(b->device);
  if (b->stream) cudaStreamSynchronize(b->stream);
  if (b->owns_keys && b->d_keys) cudaFree(b->d_keys);
  void* ptrs[] = {b->d_off, b->d_items, b->d_kmax, b->d_key_bad, b->d_headmax, b->d_amax, b->d_lo, b->d_hi,
                  b->d_cand, b->d_cand_count, b->d_frag, b->d_qnorm, b->d_qinfo, b->d_result,
                  b->d_queries, b->d_qparts, b->d_qcount, b->d_refined, b->d_qT};
  for (void* q : ptrs)
    if (q) cudaFree(q);
  if (b->h_result) cudaFreeHost(b->h_result);
  grm_b200::policy::policy_free(b->pol);
  if (b->ev0) cudaEventDestroy(b->ev0);
  if (b->ev1) cudaEventDestroy(b->ev1);
  if (b->stream) cudaStreamDestroy(b->stream);
  delete b;
}

int finish_create(grm_b200_gqa_bank* b) {
  cudaError_t e = cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreate(&b->ev0);
  if (e == cudaSuccess) e = cudaEventCreate(&b->ev1);
  const size_t N = (size_t)b->nodes;
  if (e == cudaSuccess) e = cudaMalloc(&b->d_off, sizeof(uint64_t) * (N + 1));
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(b->d_off, b->h_off.data(), sizeof(uint64_t) * (N + 1),
                        cudaMemcpyHostToDevice, b->stream);
  if (e == cudaSuccess) e = cudaMalloc(&b->d_kmax, sizeof(float) * N * b->kh_n);
  if (e == cudaSuccess) e = cudaMalloc(&b->d_key_bad, N);
  if (e == cudaSuccess) e = cudaMemsetAsync(b->d_key_bad, 0, N, b->stream);
  if (e == cudaSuccess) e = cudaMalloc(&b->d_lo, sizeof(float) * N);
  if (e == cudaSuccess) e = cudaMalloc(&b->d_hi, sizeof(float) * N);
  if (e == cudaSuccess) e = cudaMalloc(&b->d_cand, sizeof(uint32_t) * N);
  if (e == cudaSuccess) e = cudaMalloc(&b->d_cand_count, sizeof(int));
  if (e == cudaSuccess) e = cudaMemsetAsync(b->d_cand_count, 0, sizeof(int), b->stream);
  if (e == cudaSuccess) e = cudaMalloc(&b->d_qinfo, sizeof(QueryInfo));
  if (e == cudaSuccess) e = cudaMalloc(&b->d_qparts, sizeof(int) * b->kh_n);
  if (e == cudaSuccess) e = cudaMalloc(&b->d_qcount, sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemsetAsync(b->d_qcount, 0, sizeof(unsigned), b->stream);
  if (e == cudaSuccess) e = cudaMalloc(&b->d_result, sizeof(Result));
  if (e == cudaSuccess) e = cudaMallocHost(&b->h_result, sizeof(Result));
  if (e == cudaSuccess) e = cudaMalloc(&b->d_refined, sizeof(unsigned long long));
  if (e == cudaSuccess)
    e = cudaMemsetAsync(b->d_refined, 0, sizeof(unsigned long long), b->stream);
  if (e != cudaSuccess) return cuda_status(e);
  DeviceInfo info;
  int rc = device_info(b->device, &info);
  if (rc) return rc;
  b->sms = info.sms;
  // work items (node, kv head, chunk of up to kChunk tokens) for nodes with key tokens
  std::vector<Item> items;
  for (int64_t n = 0; n < b->nodes; ++n) {
    const uint64_t T = b->h_off[n + 1] - b->h_off[n];
    const uint64_t chunks = (T + kChunk - 1) / kChunk;
    for (int kh = 0; kh < b->kh_n; ++kh)
      for (uint64_t c = 0; c < chunks; ++c) {
        Item it;
        it.base = (b->h_off[n] * (uint64_t)b->kh_n + (uint64_t)kh * T + c * kChunk) * (uint64_t)b->dim;
        it.node = (uint32_t)n;
        it.kh = (uint16_t)kh;
        it.ntok = (uint16_t)std::min<uint64_t>(kChunk, T - c * kChunk);
        items.push_back(it);
      }
  }
  b->n_items = (int64_t)items.size();
  if (!items.empty()) {
    e = cudaMalloc(&b->d_items, sizeof(Item) * items.size());
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(b->d_items, items.data(), sizeof(Item) * items.size(),
                          cudaMemcpyHostToDevice, b->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    if (e != cudaSuccess) return cuda_status(e);
  }
  const int grid = (int)std::min<int64_t>(ceil_div64(b->nodes * b->kh_n * 32, 256), (int64_t)info.sms * 16);
  switch (b->dtype) {
    case GRM_B200_BF16:
      attach_stats_kernel<__nv_bfloat16><<<std::max(grid, 1), 256, 0, b->stream>>>(
          static_cast<const __nv_bfloat16*>(b->d_keys), b->d_off, b->nodes, b->kh_n, b->dim,
          b->d_kmax, b->d_key_bad);
      break;
    case GRM_B200_F16:
      attach_stats_kernel<__half><<<std::max(grid, 1), 256, 0, b->stream>>>(
          static_cast<const __half*>(b->d_keys), b->d_off, b->nodes, b->kh_n, b->dim, b->d_kmax,
          b->d_key_bad);
      break;
    default:
      attach_stats_kernel<float><<<std::max(grid, 1), 256, 0, b->stream>>>(
          static_cast<const float*>(b->d_keys), b->d_off, b->nodes, b->kh_n, b->dim, b->d_kmax,
          b->d_key_bad);
  }
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
  if (e != cudaSuccess) return cuda_status(e);
  int occ = 1;
  if (fast_bank(b)) {
    if (b->dtype == GRM_B200_BF16)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
          &occ, b->dim == 128 ? gqa_scan_kernel<__nv_bfloat16, 128, 1> : gqa_scan_kernel<__nv_bfloat16, 64, 1>,
          kThreads, 0);
    else
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
          &occ, b->dim == 128 ? gqa_scan_kernel<__half, 128, 1> : gqa_scan_kernel<__half, 64, 1>,
          kThreads, 0);
    if (e != cudaSuccess) return cuda_status(e);
  }
  const int64_t want = ceil_div64(std::max<int64_t>(b->n_items, 1), kWarps);
  b->grid_scan = (int)std::max<int64_t>(1, std::min<int64_t>((int64_t)info.sms * std::max(occ, 1), want));
  return setup_tma(b, info.sms);
}

int create_common(const void* keys, bool host, int dtype, const uint64_t* off, int64_t nodes,
                  int kh_n, int dim, int device, grm_b200_gqa_bank** out) {
  if (!out) {
    set_thread_error("out_bank is NULL");
    return GRM_B200_EINVAL;
  }
  *out = nullptr;
  if (!keys || !off || nodes <= 0 || nodes >= (int64_t)0x7FFFFFFF || kh_n <= 0 || kh_n > 255 ||
      dim <= 0 || dim > 4096 ||
      !(dtype == GRM_B200_BF16 || dtype == GRM_B200_F16 || dtype == GRM_B200_F32)) {
    set_thread_error("invalid GQA bank arguments (nodes=%lld kv_heads=%d dim=%d dtype=%d)",
                     (long long)nodes, kh_n, dim, dtype);
    return GRM_B200_EINVAL;
  }
  if (off[0] != 0) {
    set_thread_error("token_offsets must start at 0");
    return GRM_B200_EINVAL;
  }
  if ((dim * (dtype == GRM_B200_F32 ? 4 : 2)) % 16 != 0) {
    // key rows are read with 16-byte loads
    set_thread_error("head_dim * element size must be a multiple of 16 bytes (head_dim=%d)", dim);
    return GRM_B200_EINVAL;
  }
  for (int64_t i = 0; i < nodes; ++i) {
    if (off[i + 1] < off[i] || off[i + 1] - off[i] > (uint64_t)(kChunk * (int64_t)0xFFFFFF)) {
      set_thread_error("token_offsets must be non-decreasing (node %lld)", (long long)i);
      return GRM_B200_EINVAL;
    }
  }
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) {
    set_thread_error("cudaSetDevice(%d) failed: %s", device, cudaGetErrorString(e));
    return cuda_status(e);
  }
  auto* b = new grm_b200_gqa_bank();
  b->device = device;
  b->dtype = dtype;
  b->nodes = nodes;
  b->kh_n = kh_n;
  b->dim = dim;
  b->h_off.assign(off, off + nodes + 1);
  const size_t esz = dtype == GRM_B200_F32 ? 4 : 2;
  const size_t bytes = (size_t)off[nodes] * kh_n * dim * esz;
  int rc = 0;
  if (host) {
    b->owns_keys = true;
    e = cudaMalloc(&b->d_keys, std::max<size_t>(bytes, 16));
    if (e == cudaSuccess && bytes) e = cudaMemcpy(b->d_keys, keys, bytes, cudaMemcpyHostToDevice);
    rc = cuda_status(e);
  } else {
    b->owns_keys = false;
    b->d_keys = const_cast<void*>(keys);
  }
  if (!rc) rc = finish_create(b);
  if (rc) {
    set_thread_error("GQA bank create failed (%d): %s", rc, cudaGetErrorString(cudaGetLastError()));
    bank_free(b);
    return rc;
  }
  *out = b;
  return 0;
}

}  // namespace

extern "C" {

int grm_b200_gqa_bank_create(const void* keys_host, int dtype, const uint64_t* token_offsets,
                             int64_t nodes, int kv_heads, int head_dim, int device,
                             grm_b200_gqa_bank** out_bank) {
  return create_common(keys_host, true, dtype, token_offsets, nodes, kv_heads, head_dim, device,
                       out_bank);
}

int grm_b200_gqa_bank_create_device(const void* keys_device, int dtype,
                                    const uint64_t* token_offsets, int64_t nodes, int kv_heads,
                                    int head_dim, grm_b200_gqa_bank** out_bank) {
  int device = 0;
  cudaGetDevice(&device);
  return create_common(keys_device, false, dtype, token_offsets, nodes, kv_heads, head_dim, device,
                       out_bank);
}

int grm_b200_gqa_route(grm_b200_gqa_bank* bank, const float* queries_host, int query_count,
                       int query_heads, int query_tokens, int warmup, int topk,
                       uint64_t* out_ids_host, float* out_scores_host, float* elapsed_ms) {
  if (!bank) return GRM_B200_EINVAL;
  std::lock_guard<std::mutex> lock(bank->mu);
  if (!queries_host || query_count <= 0 || query_heads <= 0 || query_tokens <= 0)
    return bank->err.set(GRM_B200_EINVAL, "invalid GQA route arguments");
  cudaError_t e = cudaSetDevice(bank->device);
  const size_t need = (size_t)query_count * query_heads * query_tokens * bank->dim;
  if (e == cudaSuccess && need > bank->dq_cap) {
    if (bank->d_queries) cudaFree(bank->d_queries);
    bank->d_queries = nullptr;
    bank->dq_cap = 0;
    e = cudaMalloc(&bank->d_queries, need * sizeof(float));
    if (e == cudaSuccess) bank->dq_cap = need;
  }
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(bank->d_queries, queries_host, need * sizeof(float), cudaMemcpyHostToDevice,
                        bank->stream);
  if (e != cudaSuccess)
    return bank->err.set(cuda_status(e), "GQA query upload failed: %s", cudaGetErrorString(e));
  return route_device_queries(bank, bank->d_queries, query_count, query_heads, query_tokens, warmup,
                              topk, out_ids_host, out_scores_host, elapsed_ms);
}

int grm_b200_gqa_route_device(grm_b200_gqa_bank* bank, const float* queries_device,
                              int query_count, int query_heads, int query_tokens, int warmup,
                              int topk, uint64_t* out_ids_host, float* out_scores_host,
                              float* elapsed_ms) {
  if (!bank) return GRM_B200_EINVAL;
  std::lock_guard<std::mutex> lock(bank->mu);
  return route_device_queries(bank, queries_device, query_count, query_heads, query_tokens, warmup,
                              topk, out_ids_host, out_scores_host, elapsed_ms);
}

int grm_b200_gqa_route_async(grm_b200_gqa_bank* bank, const float* queries_device,
                             int query_count, int query_heads, int query_tokens, int topk,
                             uint64_t id_offset, uint64_t* out_ids_device,
                             float* out_scores_device, void* stream) {
  if (!bank) return GRM_B200_EINVAL;
  std::lock_guard<std::mutex> lock(bank->mu);
  if (!queries_device || query_count <= 0 || query_heads <= 0 || query_tokens <= 0 ||
      query_heads % bank->kh_n != 0 || topk <= 0 || topk > GRM_B200_MAX_TOPK ||
      !out_ids_device || !out_scores_device)
    return bank->err.set(GRM_B200_EINVAL, "invalid GQA async route arguments");
  cudaError_t e = cudaSetDevice(bank->device);
  if (e != cudaSuccess) return bank->err.set(cuda_status(e), "cudaSetDevice failed");
  const int64_t qsize = (int64_t)query_heads * query_tokens * bank->dim;
  for (int i = 0; i < query_count; ++i) {
    const int rc = route_one(bank, queries_device + i * qsize, query_heads, query_tokens, topk,
                             false, static_cast<cudaStream_t>(stream),
                             out_ids_device + (int64_t)i * topk,
                             out_scores_device + (int64_t)i * topk, id_offset);
    if (rc) return rc;
  }
  bank->routes += (uint64_t)query_count;
  return 0;
}

int grm_b200_gqa_bank_set_policy(grm_b200_gqa_bank* bank, const char* const* lexical_keys,
                                 const char* const* kinds, const char* const* scopes,
                                 const char* const* durabilities,
                                 const char* const* mutabilities, const uint8_t* active) {
  if (!bank) return GRM_B200_EINVAL;
  std::lock_guard<std::mutex> lock(bank->mu);
  cudaError_t e = cudaSetDevice(bank->device);
  if (e != cudaSuccess) return bank->err.set(cuda_status(e), "cudaSetDevice failed");
  cudaStreamSynchronize(bank->stream);
  const char* const* cats[policy::kCats] = {kinds, scopes, durabilities, mutabilities};
  return policy::policy_set(bank->pol, bank->nodes, lexical_keys, cats, active, bank->err);
}

int grm_b200_gqa_route_policy(grm_b200_gqa_bank* bank, const float* queries_host, int query_count,
                              int query_heads, int query_tokens, int topk,
                              const char* const* lexical_keys, const char* kind_filters,
                              const char* scope_filters, const char* durability_filters,
                              const char* mutability_filters, uint64_t* out_ids_host,
                              float* out_scores_host, float* elapsed_ms) {
  if (!bank) return GRM_B200_EINVAL;
  std::lock_guard<std::mutex> lock(bank->mu);
  if (!queries_host || query_count <= 0 || query_heads <= 0 || query_tokens <= 0 ||
      query_heads % bank->kh_n != 0 || !out_ids_host || topk <= 0 || topk > GRM_B200_MAX_TOPK)
    return bank->err.set(GRM_B200_EINVAL, "invalid GQA policy route arguments");
  cudaError_t e = cudaSetDevice(bank->device);
  if (e != cudaSuccess) return bank->err.set(cuda_status(e), "cudaSetDevice failed");
  int rc = 0;
  if (!bank->pol.set) {  // every node keeps the reference's defaults: no keys, active
    const char* const* cats[policy::kCats] = {nullptr, nullptr, nullptr, nullptr};
    cudaStreamSynchronize(bank->stream);
    if ((rc = policy::policy_set(bank->pol, bank->nodes, nullptr, cats, nullptr, bank->err)))
      return rc;
  }
  const size_t qsize = (size_t)query_heads * query_tokens * bank->dim;
  const size_t need = (size_t)query_count * qsize;
  if (need > bank->dq_cap) {
    if (bank->d_queries) cudaFree(bank->d_queries);
    bank->d_queries = nullptr;
    bank->dq_cap = 0;
    e = cudaMalloc(&bank->d_queries, need * sizeof(float));
    if (e != cudaSuccess) return bank->err.set(cuda_status(e), "GQA query buffer allocation failed");
    bank->dq_cap = need;
  }
  e = cudaMemcpyAsync(bank->d_queries, queries_host, need * sizeof(float), cudaMemcpyHostToDevice,
                      bank->stream);
  if (e != cudaSuccess) return bank->err.set(cuda_status(e), "GQA query upload failed");
  cudaEventRecord(bank->ev0, bank->stream);
  const char* const filters[policy::kCats] = {kind_filters, scope_filters, durability_filters,
                                              mutability_filters};
  const uint32_t* allow = nullptr;
  if ((rc = policy::policy_allow(bank->pol, filters, bank->sms, bank->stream, &allow, bank->err)))
    return rc;
  for (int q = 0; q < query_count; ++q) {
    int m = 0;
    const policy::Ranges ranges =
        policy::policy_ranges(bank->pol, lexical_keys ? lexical_keys[q] : nullptr, &m);
    if (m && (rc = policy::policy_pass(bank->pol, ranges, 0, bank->sms, bank->stream, bank->err)))
      return rc;
    rc = route_one(bank, bank->d_queries + q * qsize, query_heads, query_tokens, topk, true,
                   nullptr, nullptr, nullptr, 0, allow, bank->pol.d_hits, m);
    if (rc) return rc;
    if (m && (rc = policy::policy_pass(bank->pol, ranges, 1, bank->sms, bank->stream, bank->err)))
      return rc;  // leaves hits zero for the next query
    e = cudaMemcpyAsync(bank->h_result, bank->d_result, sizeof(Result), cudaMemcpyDeviceToHost,
                        bank->stream);
    if (e == cudaSuccess && q == query_count - 1) e = cudaEventRecord(bank->ev1, bank->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(bank->stream);
    if (e != cudaSuccess) return bank->err.set(cuda_status(e), "GQA policy route failed: %s", cudaGetErrorString(e));
    if (bank->h_result->count < 0)
      return bank->err.set(GRM_B200_KERNEL_BASE + 1, "GQA scan: a bounded device wait gave up (query %d)", q);
    for (int j = 0; j < topk; ++j) {
      out_ids_host[(int64_t)q * topk + j] = bank->h_result->ids[j];
      if (out_scores_host) out_scores_host[(int64_t)q * topk + j] = bank->h_result->scores[j];
    }
  }
  e = cudaEventSynchronize(bank->ev1);
  float ms = 0.0f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, bank->ev0, bank->ev1);
  if (e != cudaSuccess) return bank->err.set(cuda_status(e), "GQA route timing failed");
  if (elapsed_ms) *elapsed_ms = ms;
  bank->routes += (uint64_t)query_count;
  return 0;
}

int grm_b200_gqa_bank_destroy(grm_b200_gqa_bank* bank) {
  bank_free(bank);
  return 0;
}

const char* grm_b200_gqa_last_error(grm_b200_gqa_bank* bank) {
  return bank ? bank->err.text.c_str() : grm_b200_last_error();
}

int grm_b200_gqa_paths(grm_b200_gqa_bank* bank, int* flags) {
  if (!bank || !flags) return GRM_B200_EINVAL;
  *flags = (fast_bank(bank) ? GRM_B200_GQA_PATH_FAST : 0) | (bank->tma ? GRM_B200_GQA_PATH_TMA : 0);
  return 0;
}

int grm_b200_gqa_stats(grm_b200_gqa_bank* bank, uint64_t* routes, uint64_t* refined_nodes) {
  if (!bank) return GRM_B200_EINVAL;
  std::lock_guard<std::mutex> lock(bank->mu);
  if (routes) *routes = bank->routes;
  if (refined_nodes) {
    unsigned long long n = 0;
    cudaError_t e = cudaSetDevice(bank->device);
    if (e == cudaSuccess) e = cudaMemcpy(&n, bank->d_refined, sizeof(n), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return bank->err.set(cuda_status(e), "GQA stats read failed");
    *refined_nodes = n;
  }
  return 0;
}

}  // extern "C"
