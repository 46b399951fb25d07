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
// [KH, T_i, D] at token offset off[i].  Work items are (node, kv head, 64-token
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

#include "common.cuh"

namespace grm_b200 {
namespace gqa {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kChunk = 64;       // key tokens per work item
constexpr float kEps = 2.44140625e-4f;  // 2^-12 relative to |q||k|: >= 5x the proven bound
constexpr float kHuge = 1.0e30f;
constexpr int kRefineY = 32;     // candidates refined concurrently

struct Result {
  int count;
  int cands;     // nodes recomputed exactly for this route
  uint64_t ids[GRM_B200_MAX_TOPK];
  float scores[GRM_B200_MAX_TOPK];
};

struct QueryInfo {
  int finite;      // every query value finite
  int fast_ok;     // the query fits the fast path (|q| range)
  float pad[2];
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
  const uint64_t* items;       // work items
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
  int topk;
  int fast;                    // 1 = approximate pass available for this bank
  Result* result;
  int qt4;                     // reference query_tokens == 4 path
};

// Query preparation: hi/lo fragments in mma B layout, per-head norms, finite flag.
// One block; K permutation: k-step s, slot (c, j) <-> dim 32*c + 4*s + j for
// D == 128 (16*c + 4*s + j for D == 64).
template <typename KT, int D, int NT>
__global__ void query_prep_kernel(RouteParams p) {
  constexpr int KSTEPS = D / 16;
  constexpr int NVP = NT * 4;  // padded vector count: hi cols [0, NVP), lo cols [NVP, 2 NVP)
  __shared__ int s_bad, s_big;
  if (threadIdx.x == 0) {
    s_bad = 0;
    s_big = 0;
  }
  __syncthreads();
  const int nq = p.heads * p.qt * D;
  for (int i = threadIdx.x; i < nq; i += blockDim.x) {
    const float v = p.query[i];
    if (!isfinite(v)) s_bad = 1;
    if (fabsf(v) > (sizeof(KT) == 2 && !std::is_same<KT, __nv_bfloat16>::value ? 6.0e4f : kHuge))
      s_big = 1;
  }
  // per-head norm (max over query tokens)
  for (int h = threadIdx.x; h < p.heads; h += blockDim.x) {
    float mx = 0.0f;
    for (int qi = 0; qi < p.qt; ++qi) {
      const float* q = p.query + ((int64_t)h * p.qt + qi) * D;
      float ss = 0.0f;
      for (int d = 0; d < D; ++d) ss = fmaf(q[d], q[d], ss);
      mx = fmaxf(mx, sqrtf(ss));
    }
    p.qnorm_h[h] = mx * (1.0f + 9.765625e-4f);
  }
  __syncthreads();
  if constexpr (D == 128 || D == 64) {
    // fragments: [kh][t][lane][2*s + r]
    const int total = p.kh_n * NT * 32 * KSTEPS;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
      const int s = i % KSTEPS;
      const int lane = (i / KSTEPS) % 32;
      const int t = (i / (KSTEPS * 32)) % NT;
      const int kh = i / (KSTEPS * 32 * NT);
      const int g = lane >> 2, c = lane & 3;
      const int col = t * 8 + g;
      const bool is_lo = col >= NVP;
      const int vi = is_lo ? col - NVP : col;
      float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (vi < p.nv) {
        const int lh = vi / p.qt, qi = vi % p.qt;
        const int h = kh * p.group + lh;
        const float* q = p.query + ((int64_t)h * p.qt + qi) * D;
        const int d0 = (D / 4) * c + 4 * s;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float x = q[d0 + j];
          const float xh = round_kt<KT>(x);
          v[j] = is_lo ? (x - xh) : xh;
        }
      }
      uint32_t* dst = p.frag + ((((int64_t)kh * NT + t) * 32 + lane) * (2 * KSTEPS));
      dst[2 * s] = pack2<KT>(v[0], v[1]);
      dst[2 * s + 1] = pack2<KT>(v[2], v[3]);
    }
  }
  if (threadIdx.x == 0) {
    p.qinfo->finite = !s_bad;
    p.qinfo->fast_ok = !s_bad && !s_big;
  }
}

// Approximate pass: one warp per work item (node, kv head, 64-token chunk).
template <typename KT, int D, int NT>
__global__ void __launch_bounds__(kThreads) gqa_scan_kernel(RouteParams p) {
  constexpr int KSTEPS = D / 16;
  constexpr int W = D / 32;         // 16-byte loads per key row per thread (D/4 dims)
  constexpr int NVP = NT * 4;
  const int lane = threadIdx.x & 31;
  if (!p.qinfo->fast_ok) return;
  const int g = lane >> 2, c = lane & 3;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const KT* keys = static_cast<const KT*>(p.keys);
  for (int64_t it = wid; it < p.n_items; it += nw) {
    const uint64_t item = p.items[it];
    const int64_t node = (int64_t)(item >> 32);
    const int kh = (int)((item >> 24) & 0xFF);
    const int chunk = (int)(item & 0xFFFFFF);
    const int64_t T = (int64_t)(p.off[node + 1] - p.off[node]);
    const int64_t t0 = (int64_t)chunk * kChunk;
    const int64_t tend = min(T, t0 + kChunk);
    const KT* base = keys + ((int64_t)p.off[node] * p.kh_n + (int64_t)kh * T) * D;
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
    for (int64_t tt = t0; tt < tend; tt += 16) {
      // this thread's 2 rows x (D/4) contiguous dims
      uint32_t ra[2 * KSTEPS], rb[2 * KSTEPS];
      const int64_t r0 = tt + g, r1 = tt + g + 8;
#pragma unroll
      for (int w = 0; w < W; ++w) {
        uint4 va = make_uint4(0, 0, 0, 0), vb = make_uint4(0, 0, 0, 0);
        if (r0 < tend) va = ld_stream(base + r0 * D + (D / 4) * c + 8 * w);
        if (r1 < tend) vb = ld_stream(base + r1 * D + (D / 4) * c + 8 * w);
        ra[4 * w + 0] = va.x; ra[4 * w + 1] = va.y; ra[4 * w + 2] = va.z; ra[4 * w + 3] = va.w;
        rb[4 * w + 0] = vb.x; rb[4 * w + 1] = vb.y; rb[4 * w + 2] = vb.z; rb[4 * w + 3] = vb.w;
      }
      float acc[NT][4];
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
#pragma unroll
      for (int s = 0; s < KSTEPS; ++s) {
        const uint32_t a[4] = {ra[2 * s], rb[2 * s], ra[2 * s + 1], rb[2 * s + 1]};
#pragma unroll
        for (int t = 0; t < NT; ++t) mma16816<KT>(acc[t], a, bq[t][2 * s], bq[t][2 * s + 1]);
      }
      // combine hi + lo and take |.| max over the two rows
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

// Per node: approximate score interval [lo, hi]; resets headmax.  One warp per node.
__global__ void node_bounds_kernel(RouteParams p, float eps_abs) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const bool qfinite = p.qinfo->finite != 0;
  const bool fast = p.fast && p.qinfo->fast_ok;
  for (int64_t node = wid; node < p.nodes; node += nw) {
    const int64_t T = (int64_t)(p.off[node + 1] - p.off[node]);
    float sum = 0.0f, err = 0.0f;
    bool forced = !fast;
    for (int h = lane; h < p.heads; h += 32) {
      unsigned* slot = p.headmax + node * p.heads + h;
      const float b = __uint_as_float(*slot);
      *slot = 0u;
      const float km = p.kmax[node * p.kh_n + h / p.group];
      const float qn = p.qnorm_h[h];
      const float mag = qn * km;
      if (!(mag < kHuge)) forced = true;
      sum += b;
      err = fmaf(kEps * p.inv_denom, mag, err);
      err = fmaf(eps_abs * p.inv_denom, km, err);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      sum += __shfl_xor_sync(kFull, sum, o);
      err += __shfl_xor_sync(kFull, err, o);
    }
    forced = __any_sync(kFull, forced);
    if (lane == 0) {
      float l, u;
      if (T == 0) {
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
    list.offer(v, (uint32_t)n, lane);
  }
  sh_s[warp * 32 + lane] = list.s;
  sh_id[warp * 32 + lane] = list.id;
  __syncthreads();
  if (warp == 0) {
    for (int w = 1; w < 32; ++w) list.offer(sh_s[w * 32 + lane], sh_id[w * 32 + lane], lane);
    const float L = __shfl_sync(kFull, list.s, p.topk - 1);
    if (lane == 0) sh_L = L;
  }
  __syncthreads();
  const float L = sh_L;
  for (int64_t n = threadIdx.x; n < p.nodes; n += blockDim.x) {
    const float u = p.hi[n];
    if (u == u && u >= L) {  // not NaN
      const int slot = atomicAdd(p.cand_count, 1);
      p.cand[slot] = (uint32_t)n;
    }
  }
}

// Exact refine: grid.y strides candidates, grid.x x threads stride the
// (head, key token) units of one candidate.  Per unit the reference's
// sequential fp32 dot; the per-head max goes through atomicMax on the bits of
// a non-negative float (NaN candidates skipped, exactly as std::max does).
template <typename KT>
__global__ void refine_kernel(RouteParams p) {
  const int count = *p.cand_count;
  const KT* keys = static_cast<const KT*>(p.keys);
  for (int ci = blockIdx.y; ci < count; ci += gridDim.y) {
    const int64_t node = p.cand[ci];
    const int64_t T = (int64_t)(p.off[node + 1] - p.off[node]);
    if (T == 0 || p.key_bad[node] || !p.qinfo->finite) continue;
    const KT* base = keys + (int64_t)p.off[node] * p.kh_n * p.dim;
    unsigned* best_out = p.headmax + (int64_t)ci * p.heads;
    const int64_t units = (int64_t)p.heads * T * (p.qt4 ? 1 : p.qt);
    for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < units;
         u += (int64_t)gridDim.x * blockDim.x) {
      const int64_t t = u % T;
      const int64_t hq = u / T;
      float v;
      int h;
      if (p.qt4) {
        h = (int)hq;
        const int kh = h / p.group;
        const KT* k = base + ((int64_t)kh * T + t) * p.dim;
        const float* q0 = p.query + (int64_t)h * 4 * p.dim;
        float d0 = 0.0f, d1 = 0.0f, d2 = 0.0f, d3 = 0.0f;
        for (int d = 0; d < p.dim; ++d) {
          const float kv = key_to_f(k[d]);
          d0 = __fadd_rn(d0, __fmul_rn(q0[d], kv));
          d1 = __fadd_rn(d1, __fmul_rn(q0[p.dim + d], kv));
          d2 = __fadd_rn(d2, __fmul_rn(q0[2 * p.dim + d], kv));
          d3 = __fadd_rn(d3, __fmul_rn(q0[3 * p.dim + d], kv));
        }
        const float rb = std_max(std_max(fabsf(d0), fabsf(d1)), std_max(fabsf(d2), fabsf(d3)));
        v = __fmul_rn(rb, p.inv_denom);
      } else {
        h = (int)(hq / p.qt);
        const int qi = (int)(hq % p.qt);
        const int kh = h / p.group;
        const KT* k = base + ((int64_t)kh * T + t) * p.dim;
        const float* q = p.query + ((int64_t)h * p.qt + qi) * p.dim;
        float dot = 0.0f;
        for (int d = 0; d < p.dim; ++d) dot = __fadd_rn(dot, __fmul_rn(q[d], key_to_f(k[d])));
        v = __fmul_rn(fabsf(dot), p.inv_denom);
      }
      if (v > 0.0f) atomicMax(best_out + h, __float_as_uint(v));  // NaN and 0 never raise best
    }
  }
}

// Final scores of the candidates (sequential fp32 head sum, as the reference)
// and the exact top-k.  One warp.
__global__ void finalize_kernel(RouteParams p) {
  const int lane = threadIdx.x;
  const int count = *p.cand_count;
  WarpList list;
  list.init();
  for (int base = 0; base < count; base += 32) {
    const int ci = base + lane;
    float score = -INFINITY;
    uint32_t node = kNoRow;
    if (ci < count) {
      node = p.cand[ci];
      const int64_t T = (int64_t)(p.off[node + 1] - p.off[node]);
      unsigned* best = p.headmax + (int64_t)ci * p.heads;
      if (T == 0) {
        score = 0.0f;
      } else if (p.key_bad[node] || !p.qinfo->finite) {
        score = __int_as_float(0x7FC00000);
      } else {
        float total = 0.0f;
        for (int h = 0; h < p.heads; ++h) total = __fadd_rn(total, __uint_as_float(best[h]));
        score = __fdiv_rn(total, (float)p.heads);
      }
      for (int h = 0; h < p.heads; ++h) best[h] = 0u;
    }
    list.offer(score, node, lane);
  }
  const bool ok = lane < p.topk && isfinite(list.s) && list.id != kNoRow;
  const unsigned m = __ballot_sync(kFull, ok);
  if (lane < p.topk) {
    p.result->ids[lane] = ok ? (uint64_t)list.id : UINT64_MAX;
    p.result->scores[lane] = ok ? list.s : __int_as_float(0x7FC00000);
  }
  if (lane == 0) {
    p.result->count = __popc(m);
    p.result->cands = count;
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
  uint64_t* d_items = nullptr;
  int64_t n_items = 0;
  float* d_kmax = nullptr;
  unsigned char* d_key_bad = nullptr;
  unsigned* d_headmax = nullptr;
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
  Result* d_result = nullptr;
  Result* h_result = nullptr;
  float* d_queries = nullptr;
  size_t dq_cap = 0;
  int grid_scan = 1;
  int sms = 1;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  std::mutex mu;
  ErrorSlot err;
  uint64_t routes = 0, refined = 0;
};

namespace {

bool fast_bank(const grm_b200_gqa_bank* b) {
  return (b->dtype == GRM_B200_BF16 || b->dtype == GRM_B200_F16) && (b->dim == 128 || b->dim == 64);
}

int nt_for(int nv) { return nv <= 4 ? 1 : (nv <= 8 ? 2 : (nv <= 16 ? 4 : 0)); }

template <typename KT, int D, int NT>
void launch_fast(grm_b200_gqa_bank* b, const RouteParams& p) {
  query_prep_kernel<KT, D, NT><<<1, 256, 0, b->stream>>>(p);
  if (b->n_items > 0)
    gqa_scan_kernel<KT, D, NT><<<b->grid_scan, kThreads, 0, b->stream>>>(p);
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
  __syncthreads();
  if (threadIdx.x == 0) {
    p.qinfo->finite = !s_bad;
    p.qinfo->fast_ok = 0;
  }
}

template <typename KT>
void launch_refine(grm_b200_gqa_bank* b, const RouteParams& p) {
  dim3 grid(std::max(1, b->sms / 4), kRefineY);
  refine_kernel<KT><<<grid, 256, 0, b->stream>>>(p);
}

int ensure_heads(grm_b200_gqa_bank* b, int heads, int nt) {
  if (heads > b->headmax_heads) {
    if (b->d_headmax) cudaFree(b->d_headmax);
    b->d_headmax = nullptr;
    b->headmax_heads = 0;
    const size_t n = (size_t)b->nodes * heads;
    cudaError_t e = cudaMalloc(&b->d_headmax, n * sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemsetAsync(b->d_headmax, 0, n * sizeof(unsigned), b->stream);
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

int route_one(grm_b200_gqa_bank* b, const float* dq, int heads, int qt, int topk) {
  const int group = heads / b->kh_n;
  const int nv = group * qt;
  const int nt = nt_for(nv);
  const bool fast = fast_bank(b) && nt > 0;
  int rc = ensure_heads(b, heads, nt);
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
  p.topk = topk;
  p.fast = fast ? 1 : 0;
  p.result = b->d_result;
  p.qt4 = (qt == 4) ? 1 : 0;
  if (fast) {
    rc = (b->dtype == GRM_B200_BF16) ? launch_fast_dims<__nv_bfloat16>(b, p, nt)
                                     : launch_fast_dims<__half>(b, p, nt);
  } else {
    query_info_kernel<<<1, 256, 0, b->stream>>>(p);
    rc = cuda_status(cudaGetLastError());
  }
  if (rc) return b->err.set(rc, "GQA scan launch failed");
  // eps_abs: absolute query-representation error of an f16 split (subnormal lo parts)
  const float eps_abs = (b->dtype == GRM_B200_F16) ? 2.0e-7f * std::sqrt((float)b->dim) : 1.0e-30f;
  const int nb_grid = (int)std::min<int64_t>(ceil_div64(b->nodes, kWarps), (int64_t)b->sms * 8);
  node_bounds_kernel<<<nb_grid, kThreads, 0, b->stream>>>(p, eps_abs);
  select_kernel<<<1, 1024, 0, b->stream>>>(p);
  switch (b->dtype) {
    case GRM_B200_BF16: launch_refine<__nv_bfloat16>(b, p); break;
    case GRM_B200_F16: launch_refine<__half>(b, p); break;
    default: launch_refine<float>(b, p); break;
  }
  finalize_kernel<<<1, 32, 0, b->stream>>>(p);
  rc = cuda_status(cudaGetLastError());
  if (rc) return b->err.set(rc, "GQA route launch failed: %s", cudaGetErrorString(cudaGetLastError()));
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
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    if (e != cudaSuccess) return b->err.set(cuda_status(e), "GQA route failed: %s", cudaGetErrorString(e));
    b->refined += (uint64_t)b->h_result->cands;
    for (int j = 0; j < topk; ++j) {
      out_ids[(int64_t)i * topk + j] = b->h_result->ids[j];
      if (out_scores) out_scores[(int64_t)i * topk + j] = b->h_result->scores[j];
    }
  }
  cudaEventRecord(b->ev1, b->stream);
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
  void* ptrs[] = {b->d_off, b->d_items, b->d_kmax, b->d_key_bad, b->d_headmax, b->d_lo, b->d_hi,
                  b->d_cand, b->d_cand_count, b->d_frag, b->d_qnorm, b->d_qinfo, b->d_result,
                  b->d_queries};
  for (void* q : ptrs)
    if (q) cudaFree(q);
  if (b->h_result) cudaFreeHost(b->h_result);
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
  if (e == cudaSuccess) e = cudaMalloc(&b->d_result, sizeof(Result));
  if (e == cudaSuccess) e = cudaMallocHost(&b->h_result, sizeof(Result));
  if (e != cudaSuccess) return cuda_status(e);
  DeviceInfo info;
  int rc = device_info(b->device, &info);
  if (rc) return rc;
  b->sms = info.sms;
  // work items (node, kv head, chunk) for nodes with key tokens
  std::vector<uint64_t> items;
  for (int64_t n = 0; n < b->nodes; ++n) {
    const uint64_t T = b->h_off[n + 1] - b->h_off[n];
    const uint64_t chunks = (T + kChunk - 1) / kChunk;
    for (int kh = 0; kh < b->kh_n; ++kh)
      for (uint64_t c = 0; c < chunks; ++c)
        items.push_back(((uint64_t)n << 32) | ((uint64_t)kh << 24) | c);
  }
  b->n_items = (int64_t)items.size();
  if (!items.empty()) {
    e = cudaMalloc(&b->d_items, sizeof(uint64_t) * items.size());
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(b->d_items, items.data(), sizeof(uint64_t) * items.size(),
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
  return 0;
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

int grm_b200_gqa_bank_destroy(grm_b200_gqa_bank* bank) {
  bank_free(bank);
  return 0;
}

const char* grm_b200_gqa_last_error(grm_b200_gqa_bank* bank) {
  return bank ? bank->err.text.c_str() : grm_b200_last_error();
}

int grm_b200_gqa_stats(grm_b200_gqa_bank* bank, uint64_t* routes, uint64_t* refined_nodes) {
  if (!bank) return GRM_B200_EINVAL;
  if (routes) *routes = bank->routes;
  if (refined_nodes) *refined_nodes = bank->refined;
  return 0;
}

}  // extern "C"
