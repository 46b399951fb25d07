// mla_route.cu -- MLA latent-centroid route on sm_100a.
//
// Law (GraftRepository cpp/grm_runtime.cpp): row norm = float(sqrt(sum_d
// double(c_d)^2)) (:3240-3249); qnorm = sqrt(sum_d double(q_d)^2) (:4311-4315);
// score = float(dot_fp64(q, c) / (qnorm * double(norm) + 1e-8)) with the dot
// accumulated in fp64 in element order (:3518-3545); non-finite scores are
// dropped and the rest ordered by score desc, node id asc (:75-82, :4352-4360).
//
// Design.  One streaming pass reads the bank once from HBM with coalesced
// 16-byte loads: a warp takes 32 rows at a time, each lane dots its 16-byte
// slice of every row with its slice of the unit-normalised query in fp32, and
// a butterfly reduce-scatter leaves one row's approximate cosine per lane.
// Each warp keeps a sorted top-32 of approximate scores in registers (one
// entry per lane), blocks merge their warps, publish only entries within the
// margin of the best block k-th score seen so far, and the last block to
// finish merges those, picks every row whose approximate score is within
// 2*kMargin of the approximate k-th best, and recomputes those rows with the
// reference's exact fp64 arithmetic.  The fp32 approximation is within 21 ulp
// of 1.0 of the reference score (|q'|=1, |s|<=1, <=13 rounding steps per dot);
// kMargin = 2^-16 is >= 12x that bound, so every row that can be in the
// exact top-k is recomputed.  If the approximate lists were saturated inside
// the margin (near-ties, duplicate rows) or the query is outside the safe
// range (zero, non-finite, |q| outside [1e-20, 1e20]), a second kernel
// computes exact scores for every row above the threshold (or for all rows),
// so the result is exact in every case.
#include <algorithm>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "route_policy.cuh"

namespace grm_b200 {
namespace mla {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr float kMargin = 1.52587890625e-05f;  // 2^-16
constexpr double kSafeLo = 1.0e-20, kSafeHi = 1.0e20;
constexpr int kInlineMax = 512;  // largest dim a query can travel inline
constexpr int kBatchMin = 2;     // batches from this size on (top-k <= 16) take the tensor-core route

enum Status : int { kOk = 0, kOverflow = 1, kUnsafe = 2, kError = 3 };

struct Result {
  int status;
  int count;
  float thr;
  int pad;
  uint64_t ids[GRM_B200_MAX_TOPK];
  float scores[GRM_B200_MAX_TOPK];
};

struct Header {
  int lb;          // ordered float: best block k-th approximate score so far
  unsigned done;   // blocks finished in this launch
  int err;         // a bounded device wait gave up in this launch
  unsigned nent;   // entries appended to the published list in this launch
  int floor;       // ordered float: largest score a block dropped for lack of room
  unsigned next;   // next group of the bulk scan's dynamic tail
  int qsafe;       // batched route: the query is inside the batch path's safe range
  int pad[9];
};

struct Entry {
  float s;
  uint32_t id;
};

struct Scratch {
  unsigned char* base;
  size_t stride;  // bytes per query
  int blocks;
  // pointer arithmetic only: the host uses it to pass a query's header to kernels
  __host__ __device__ Header* hdr(int q) const { return reinterpret_cast<Header*>(base + stride * q); }
  __device__ Entry* entries(int q) const {
    return reinterpret_cast<Entry*>(base + stride * q + sizeof(Header));
  }
  __device__ int* counts(int q) const {
    return reinterpret_cast<int*>(base + stride * q + sizeof(Header) + sizeof(Entry) * 32 * blocks);
  }
  // exact (reference-arithmetic) score of each appended entry, written by the
  // single-probe scans before they publish
  __device__ float* exact(int q) const {
    return reinterpret_cast<float*>(base + stride * q + sizeof(Header) +
                                    sizeof(Entry) * 32 * blocks + 8 * (size_t)blocks);
  }
};

// Back to the state a launch starts from (err is cleared by whoever reports it).
__device__ __forceinline__ void reset_header(Header* h) {
  h->lb = kOrderedNegInf;
  h->done = 0;
  h->nent = 0;
  h->floor = kOrderedNegInf;
  h->next = 0;
}

inline size_t scratch_stride(int blocks) {
  size_t b = sizeof(Header) + sizeof(Entry) * 32 * (size_t)blocks + 8 * (size_t)blocks +
             sizeof(float) * 32 * (size_t)blocks;
  return (b + 255) & ~(size_t)255;
}

template <typename T>
struct Params {
  const T* rows;
  const float* norms;
  int64_t nodes;
  int dim;
  const float* queries;  // [Q, dim]
  int topk;
  Scratch scratch;
  Result* results;       // [Q]
  uint64_t* out_ids;     // optional device outputs [Q, topk]
  float* out_scores;
  uint64_t id_offset;
  int force_all;         // exact kernel: score every row (bank outside the fast path)
  int nq;                // exact kernel: queries in this launch
  unsigned long long* fallback_count;  // queries that took the exact pass (optional)
  const uint32_t* allow;  // route filters: bitmap of the rows that may be routed (nullptr: all)
  // multi-row entries (entry score = max over its rows): the scan folds row
  // scores into entry_best[entry_of_row[row]] instead of keeping row lists
  const uint32_t* entry_of_row;
  int* entry_best;        // [entries] ordered float, reset to -inf by the collect step
  int* multi_unsafe;      // [Q] the query is outside the approximate pass's safe range
  double* multi_qnorm;    // the query's reference norm, for the entry refine
  unsigned wait_limit;    // probes per bounded wait of the bulk scan (scan_wait_limit())
  // A single query may travel inside the launch parameters (queries == nullptr):
  // the synchronous host entry then needs no host-to-device copy.
  float qinline[kInlineMax];
};

template <typename T>
__device__ __forceinline__ const float* query_ptr(const Params<T>& p, int q, int dim) {
  return p.queries ? p.queries + (int64_t)q * dim : p.qinline;
}

__device__ __forceinline__ float to_f(__half h) { return __half2float(h); }
__device__ __forceinline__ float to_f(float f) { return f; }

// The reference's exact score for one row (cpp/grm_runtime.cpp:3518-3545).
// Products of two floats are exact in fp64, so fma(q, c, dot) == dot + q*c.
template <typename T>
__device__ float exact_score(const T* row, int dim, const float* q, double qnorm, float norm) {
  double dot = 0.0;
#pragma unroll 8
  for (int d = 0; d < dim; ++d) dot = fma((double)q[d], (double)to_f(row[d]), dot);
  return (float)(dot / (qnorm * (double)norm + 1.0e-8));
}

// Same score with the row norm computed from the row itself in the same pass
// (rebuild_mla_arena's norm, cpp/grm_runtime.cpp:3240-3249: fp64 sum of squares
// in element order, cast to float).  Used where no precomputed norms exist.
template <typename T>
__device__ float exact_score_inline_norm(const T* row, int dim, const float* q, double qnorm) {
  double dot = 0.0, n2 = 0.0;
#pragma unroll 8
  for (int d = 0; d < dim; ++d) {
    const double c = (double)to_f(row[d]);
    dot = fma((double)q[d], c, dot);
    n2 = fma(c, c, n2);
  }
  const float norm = (float)sqrt(n2);
  return (float)(dot / (qnorm * (double)norm + 1.0e-8));
}

// Sum of squares of one 16-byte slice (approximate row norm, fp32).
template <typename T>
__device__ __forceinline__ float sq16(const uint4& v, float acc) {
  if constexpr (sizeof(T) == 2) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(h[k]);
      acc = fmaf(f.x, f.x, acc);
      acc = fmaf(f.y, f.y, acc);
    }
  } else {
    acc = fmaf(__uint_as_float(v.x), __uint_as_float(v.x), acc);
    acc = fmaf(__uint_as_float(v.y), __uint_as_float(v.y), acc);
    acc = fmaf(__uint_as_float(v.z), __uint_as_float(v.z), acc);
    acc = fmaf(__uint_as_float(v.w), __uint_as_float(v.w), acc);
  }
  return acc;
}

// Reference query norm, element order (cpp/grm_runtime.cpp:4311-4315).
__device__ double query_norm_seq(const float* q, int dim) {
  double acc = 0.0;
  for (int d = 0; d < dim; ++d) {
    const double v = (double)q[d];
    acc = fma(v, v, acc);
  }
  return sqrt(acc);
}

// Butterfly reduce-scatter of N partial sums over N lanes: afterwards v[0]
// holds the total of slot (lane & (N-1)) across the N lanes.
template <int N>
__device__ __forceinline__ float reduce_scatter(float (&v)[N], int lane) {
#pragma unroll
  for (int o = N / 2; o >= 1; o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = upper ? v[i] : v[i + o];
      const float keep = upper ? v[i + o] : v[i];
      v[i] = keep + __shfl_xor_sync(kFull, send, o);
    }
  }
  return v[0];
}

template <typename T>
__device__ __forceinline__ float dot16(const uint4& v, const float* qr, float acc) {
  if constexpr (sizeof(T) == 2) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(h[k]);
      acc = fmaf(f.x, qr[2 * k], acc);
      acc = fmaf(f.y, qr[2 * k + 1], acc);
    }
  } else {
    acc = fmaf(__uint_as_float(v.x), qr[0], acc);
    acc = fmaf(__uint_as_float(v.y), qr[1], acc);
    acc = fmaf(__uint_as_float(v.z), qr[2], acc);
    acc = fmaf(__uint_as_float(v.w), qr[3], acc);
  }
  return acc;
}

// Merge the NW warp lists of this block into warp 0's list.
template <int NW = kWarps>
__device__ __forceinline__ void block_merge(WarpList& list, int lane, int warp, float* sh_s,
                                            uint32_t* sh_id) {
  sh_s[warp * 32 + lane] = list.s;
  sh_id[warp * 32 + lane] = list.id;
  __syncthreads();
  if (warp == 0) {
    for (int w = 1; w < NW; ++w) list.offer(sh_s[w * 32 + lane], sh_id[w * 32 + lane], lane);
  }
}

// Write the final top-k (warp 0 of the finishing block; `ex` sorted exact).
template <typename T>
__device__ void write_result(const Params<T>& p, int q, const WarpList& ex, int lane) {
  Result* r = p.results + q;
  const bool ok = lane < p.topk && isfinite(ex.s) && ex.id != kNoRow;
  const unsigned m = __ballot_sync(kFull, ok);
  if (lane < p.topk) {
    const uint64_t id = ok ? (uint64_t)ex.id + p.id_offset : UINT64_MAX;
    const float s = ok ? ex.s : __int_as_float(0x7FC00000);
    r->ids[lane] = id;
    r->scores[lane] = s;
    if (p.out_ids) p.out_ids[(int64_t)q * p.topk + lane] = id;
    if (p.out_scores) p.out_scores[(int64_t)q * p.topk + lane] = s;
  }
  if (lane == 0) {
    r->count = __popc(m);
    r->status = kOk;
  }
}

// Shared memory of the merge/refine epilogue.  qraw holds the query as given
// (the exact refine reads it many times); s/id double as the candidate list
// of the final merge.
template <int NW, int D>
struct FinishSmem {
  float s[NW * 32];
  uint32_t id[NW * 32];
  float ex[NW * 32];  // exact scores of the list (pre-refined entries)
  float kth[NW];
  float floor[NW];
  float qraw[D];
  double qd[D];  // qraw as double, for the exact refine
  double qn;
  int last;
  int ncand;
};

// The reference query norm (query_norm_seq's order) for a compile-time dim.
template <int D>
__device__ __forceinline__ double query_norm_seq_t(const float* q) {
  double acc = 0.0;
#pragma unroll 8
  for (int d = 0; d < D; ++d) {
    const double v = (double)q[d];
    acc = fma(v, v, acc);
  }
  return sqrt(acc);
}

// exact_score / exact_score_inline_norm for the final refine: the row is read
// in rounds of up to 16 vectors (256 bytes) issued together, so a 512-byte
// row costs two memory round trips.  The final merge runs in a single block
// right after the bank stream, so its code is fetched cold: the loop over
// rounds is kept rolled on purpose.
__device__ __forceinline__ double to_d(__half h) {
  double d;
  asm("cvt.f64.f16 %0, %1;" : "=d"(d) : "h"(__half_as_ushort(h)));
  return d;
}
__device__ __forceinline__ double to_d(float f) { return (double)f; }

template <int D, typename T, bool INL>
__device__ float exact_score_tail(const T* row, const double* q, double qnorm, float norm) {
  constexpr int E = 16 / (int)sizeof(T);
  constexpr int NV = D / E;
  constexpr int CH = NV < 16 ? NV : 16;
  static_assert(NV % CH == 0, "a row splits into whole rounds");
  const uint4* rv = reinterpret_cast<const uint4*>(row);
  double dot = 0.0, n2 = 0.0;
#pragma unroll 1
  for (int c0 = 0; c0 < NV; c0 += CH) {
    uint4 v[CH];
#pragma unroll
    for (int i = 0; i < CH; ++i) v[i] = ld_nc16(rv + c0 + i);
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const T* e = reinterpret_cast<const T*>(&v[i]);
#pragma unroll
      for (int k = 0; k < E; ++k) {
        const double c = to_d(e[k]);
        dot = fma(q[(c0 + i) * E + k], c, dot);
        if constexpr (INL) n2 = fma(c, c, n2);
      }
    }
  }
  if constexpr (INL) norm = (float)sqrt(n2);
  return (float)(dot / (qnorm * (double)norm + 1.0e-8));
}

// Largest entry (score desc, id asc) among the R values each lane holds, over
// the warp; returns it in every lane.
template <int R>
__device__ __forceinline__ void warp_best(const float (&v)[R], const uint32_t (&id)[R], float& bs,
                                          uint32_t& bid) {
  bs = v[0];
  bid = id[0];
#pragma unroll
  for (int r = 1; r < R; ++r)
    if (better(v[r], id[r], bs, bid)) {
      bs = v[r];
      bid = id[r];
    }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float os = __shfl_xor_sync(kFull, bs, o);
    const uint32_t oid = __shfl_xor_sync(kFull, bid, o);
    if (better(os, oid, bs, bid)) {
      bs = os;
      bid = oid;
    }
  }
}

constexpr int kSelR = 4;  // candidates per lane in the final selection (128 per warp)

// Final merge of query q (one block, NW warps), after every block published.
// hdr->lb is by now the best block k-th score, a lower bound of the
// approximate k-th best T_k, so entries below lb - 2*margin are skipped: no
// candidate is among them.  Warps 0..NW-2 filter the appended entries into a
// shared list (one load each; candidate rows are prefetched) while warp
// NW-1 computes the reference query norm.  Warp 0 then takes the best 128
// (all of them, or the first 128 after a rank sort when more passed), finds
// T_k by k rounds of warp arg-max, and recomputes every entry >= T_k -
// 2*margin with the reference arithmetic.  When 32 or more entries, or a
// block's dropped rows (hdr->floor), reach that threshold, the exact
// fallback kernel is flagged instead.  QREADY: the caller already filled
// sm.qd and sm.qn (warp NW-1 then only waits at the barriers).  PRE: every
// appended entry already carries its exact score (p.scratch.exact), computed
// by the block that published it, so no row is read here.  KLB: the filter
// threshold is raised to the k-th best of the first NW * 32 * kSelR entries
// (each warp takes 32 * kSelR of them; the k-th best of any subset is no
// higher than the k-th best of all) minus 2*margin, for publishers whose lb
// is far below the final k-th.  XALL: warps 1.. compute the exact scores of
// the filtered entries (one per lane) while warp 0 selects, so the refine's
// sequential fp64 dots run beside the selection; the selection then goes as
// under PRE.
template <int D, typename T, bool INL, int NW, bool QREADY = false, bool PRE = false,
          bool KLB = false, bool XALL = false>
__device__ __forceinline__ void final_merge(const Params<T>& p, int q, float margin, bool safe,
                                            int lane, int warp, FinishSmem<NW, D>& sm) {
  static_assert(NW >= 2, "final_merge needs two warps");
  Header* hdr = p.scratch.hdr(q);
  if (threadIdx.x == 0) sm.ncand = 0;
  __syncthreads();
  const int lb = __ldcg(&hdr->lb);
  float fthr = lb == kOrderedNegInf ? -INFINITY : ordered_to_float(lb) - 2.0f * margin;
  const int nent = min((int)__ldcg(&hdr->nent), p.scratch.blocks * 32);
  const int fl = __ldcg(&hdr->floor);
  const bool failed = __ldcg(&hdr->err) != 0;
  const uint2* ents = reinterpret_cast<const uint2*>(p.scratch.entries(q));
  const float* exs = p.scratch.exact(q);
  // one filtered entry: into the shared list, its row prefetched
  auto keep = [&](float es, uint32_t id, int i) {
    const int slot = atomicAdd(&sm.ncand, 1);
    if (slot < NW * 32) {
      sm.s[slot] = es;
      sm.id[slot] = id;
      if constexpr (PRE) sm.ex[slot] = __ldcg(exs + i);
    }
    if constexpr (!PRE) {
      const char* rb = reinterpret_cast<const char*>(p.rows + (int64_t)id * D);
#pragma unroll 1
      for (int o = 0; o < D * (int)sizeof(T); o += 128)
        asm volatile("prefetch.global.L1 [%0];" ::"l"(rb + o));
    }
  };
  // KLB: the first NW * 32 * kSelR entries are filtered from the registers
  // that found the bound; the strided loop below takes the rest
  int first = 0;
  if constexpr (KLB) {
    float w[kSelR], e0[kSelR];
    uint32_t wid[kSelR];
#pragma unroll
    for (int r = 0; r < kSelR; ++r) {
      const int i = (warp * kSelR + r) * 32 + lane;
      const uint2 e = i < nent ? __ldcg(ents + i) : make_uint2(__float_as_uint(-INFINITY), kNoRow);
      w[r] = e0[r] = __uint_as_float(e.x);
      wid[r] = e.y;
    }
    float kth = -INFINITY;
#pragma unroll 1
    for (int t = 0; t < p.topk; ++t) {
      float bs;
      uint32_t bid;
      warp_best<kSelR>(w, wid, bs, bid);
      kth = bs;
#pragma unroll
      for (int r = 0; r < kSelR; ++r)
        if (wid[r] == bid && w[r] == bs) w[r] = -INFINITY;
    }
    if (lane == 0) sm.kth[warp] = kth;
    __syncthreads();
    float kb = -INFINITY;
#pragma unroll 1
    for (int j = 0; j < NW; ++j) kb = fmaxf(kb, sm.kth[j]);
    if (kb > -INFINITY) fthr = fmaxf(fthr, kb - 2.0f * margin);
#pragma unroll
    for (int r = 0; r < kSelR; ++r) {
      const int i = (warp * kSelR + r) * 32 + lane;
      if (i < nent && e0[r] >= fthr) keep(e0[r], wid[r], i);
    }
    first = NW * 32 * kSelR;
  }
  if (warp == NW - 1 && !PRE) {
    if constexpr (!QREADY && !PRE) {
      for (int d = lane; d < D; d += 32) sm.qd[d] = (double)sm.qraw[d];
      if (lane == 0) sm.qn = query_norm_seq_t<D>(sm.qraw);
    }
  } else {
    constexpr int FW = PRE ? NW : NW - 1;  // filtering warps
#pragma unroll 2
    for (int i = first + threadIdx.x; i < nent; i += FW * 32) {
      const uint2 e = __ldcg(ents + i);
      const float es = __uint_as_float(e.x);
      if (es >= fthr) keep(es, e.y, i);
    }
  }
  __syncthreads();
  const int ncand = sm.ncand;
  const int n = min(ncand, NW * 32);
  if (n > 32 * kSelR) {  // rare: rank sort so the best 32*kSelR come first
    float cs = -INFINITY, cx = -INFINITY;
    uint32_t ci = kNoRow;
    int rank = 0;
    if ((int)threadIdx.x < n) {
      cs = sm.s[threadIdx.x];
      ci = sm.id[threadIdx.x];
      if constexpr (PRE) cx = sm.ex[threadIdx.x];
#pragma unroll 1
      for (int j = 0; j < n; ++j) rank += better(sm.s[j], sm.id[j], cs, ci) ? 1 : 0;
    }
    __syncthreads();
    if ((int)threadIdx.x < n) {
      sm.s[rank] = cs;  // the ranks are a permutation of [0, n)
      sm.id[rank] = ci;
      if constexpr (PRE) sm.ex[rank] = cx;
    }
    __syncthreads();
  }
  constexpr bool HAVE_EX = PRE || XALL;
  // XALL: the exact scores are handed to warp 0 through named barrier 1
  // (every warp arrives once: warps 1.. after their dots, warp 0 after its
  // selection)
  if (warp != 0) {
    if constexpr (XALL) {
      static_assert(!PRE && NW >= 2, "XALL computes what PRE reads");
      if (safe && !failed)
        for (int i = (warp - 1) * 32 + lane; i < n; i += (NW - 1) * 32) {
          const uint32_t id = sm.id[i];
          sm.ex[i] = exact_score_tail<D, T, INL>(p.rows + (int64_t)id * D, sm.qd, sm.qn,
                                                 INL ? 0.0f : __ldg(p.norms + id));
        }
      asm volatile("bar.sync 1, %0;" ::"r"(NW * 32) : "memory");
    }
    return;
  }
  const int m = min(n, 32 * kSelR);
  float v[kSelR], w[kSelR], xr[kSelR];
  uint32_t vid[kSelR];
#pragma unroll
  for (int r = 0; r < kSelR; ++r) {
    const int i = r * 32 + lane;
    v[r] = i < m ? sm.s[i] : -INFINITY;
    vid[r] = i < m ? sm.id[i] : kNoRow;
    xr[r] = (PRE && i < m) ? sm.ex[i] : -INFINITY;
    w[r] = v[r];
  }
  // T_k: remove the best entry k-1 times, then take the best.
  float T_k = -INFINITY;
#pragma unroll 1
  for (int t = 0; t < p.topk; ++t) {
    float bs;
    uint32_t bid;
    warp_best<kSelR>(w, vid, bs, bid);
    T_k = bs;
#pragma unroll
    for (int r = 0; r < kSelR; ++r)
      if (vid[r] == bid && w[r] == bs) w[r] = -INFINITY;
  }
  if constexpr (XALL) {  // the other warps' exact scores are in sm.ex
    asm volatile("bar.sync 1, %0;" ::"r"(NW * 32) : "memory");
#pragma unroll
    for (int r = 0; r < kSelR; ++r) {
      const int i = r * 32 + lane;
      xr[r] = i < m ? sm.ex[i] : -INFINITY;
    }
  }
  float thr = isfinite(T_k) ? T_k - 2.0f * margin : -INFINITY;
  int above = 0;
#pragma unroll
  for (int r = 0; r < kSelR; ++r) above += __popc(__ballot_sync(kFull, isfinite(v[r]) && v[r] >= thr));
  const float floor_max = fl == kOrderedNegInf ? -INFINITY : ordered_to_float(fl);
  bool overflow = above >= 32 || (isfinite(floor_max) && floor_max >= thr);
  if (ncand > NW * 32) {  // more entries inside the margin than the shared list holds
    overflow = true;
    thr = fthr;
  }
  Result* r = p.results + q;
  if (failed) {
    if (lane == 0) {
      r->status = kError;
      r->count = 0;
      reset_header(hdr);
      hdr->err = 0;
    }
    return;
  }
  if (!safe || overflow) {
    if (lane == 0) {
      r->status = safe ? kOverflow : kUnsafe;
      r->thr = thr;
      r->count = 0;
      reset_header(hdr);
    }
    return;
  }
  // Candidates (fewer than 32): compacted through shared memory, one per
  // lane, and recomputed exactly.
  __syncwarp();
  int base = 0;
#pragma unroll
  for (int r = 0; r < kSelR; ++r) {
    const bool c = isfinite(v[r]) && v[r] >= thr;
    const unsigned bal = __ballot_sync(kFull, c);
    if (c) {
      const int pos = base + __popc(bal & ((1u << lane) - 1u));
      sm.s[pos] = v[r];
      sm.id[pos] = vid[r];
      if constexpr (HAVE_EX) sm.ex[pos] = xr[r];
    }
    base += __popc(bal);
  }
  __syncwarp();
  const float cs = lane < base ? sm.s[lane] : -INFINITY;
  const uint32_t ci = lane < base ? sm.id[lane] : kNoRow;
  float es = -INFINITY;
  if (isfinite(cs)) {
    if constexpr (HAVE_EX) {
      es = sm.ex[lane];
    } else {
      es = exact_score_tail<D, T, INL>(p.rows + (int64_t)ci * D, sm.qd, sm.qn,
                                       INL ? 0.0f : __ldg(p.norms + ci));
    }
  }
  WarpList ex;
  ex.init();
  ex.offer(es, ci, lane);
  write_result(p, q, ex, lane);
  if (lane == 0) reset_header(hdr);
}

}  // namespace mla
}  // namespace grm_b200

#include "mla_batch.cuh"
#include "mla_int4.cuh"

namespace grm_b200 {
namespace mla {

// Everything after the streaming loop.  The block list is seeded with the
// warp list whose k-th score is the largest (a copy: lists are sorted) and
// the other warps' entries are merged with offer_margin, so the block's k-th
// approximate score is exact while entries that cannot reach a candidate are
// skipped.  The block raises hdr->lb to its k-th score (atomicMax returns the
// best k-th published before it), raises hdr->floor to the largest score a
// row it dropped for lack of room can have, and appends only its entries
// within 2*kMargin of the larger of the two: hdr->lb only grows and stays a
// lower bound of the final approximate k-th T_k, so no entry below it can be
// a final candidate, and blocks that finish late usually append nothing.
// Before appending, the block recomputes its entries with the reference
// arithmetic (one entry per lane of warp 0; the reference query norm was
// computed by warp 1 while the block streamed), so the last block to finish
// only selects (final_merge<..., PRE>) and reads no row.
template <int D, typename T, bool INL, int NW>
__device__ __forceinline__ void scan_finish(const Params<T>& p, WarpList& list, bool safe, int q,
                                            int lane, int warp, FinishSmem<NW, D>& sm) {
  sm.s[warp * 32 + lane] = list.s;
  sm.id[warp * 32 + lane] = list.id;
  const float kth_w = __shfl_sync(kFull, list.s, p.topk - 1);
  const float last_w = __shfl_sync(kFull, list.s, 31);
  if (lane == 0) {
    sm.kth[warp] = kth_w;
    sm.floor[warp] = last_w;
  }
  __syncthreads();
  Header* hdr = p.scratch.hdr(q);
  if (warp == 0) {
    float kbest = -INFINITY, floor = -INFINITY;
    int wbest = 0;
#pragma unroll 1
    for (int w = 0; w < NW; ++w) {
      const float kw = sm.kth[w];
      if (kw > kbest) {
        kbest = kw;
        wbest = w;
      }
      floor = fmaxf(floor, sm.floor[w]);
    }
    WarpList m;
    m.s = sm.s[wbest * 32 + lane];
    m.id = sm.id[wbest * 32 + lane];
#pragma unroll 1
    for (int w = 0; w < NW; ++w)
      if (w != wbest)
        m.offer_margin(sm.s[w * 32 + lane], sm.id[w * 32 + lane], lane, p.topk, 2.0f * kMargin);
    const float kth = __shfl_sync(kFull, m.s, p.topk - 1);
    floor = fmaxf(floor, __shfl_sync(kFull, m.s, 31));
    int lbv = kOrderedNegInf;
    if (lane == 0) {
      lbv = isfinite(kth) ? max(atomicMax(&hdr->lb, float_to_ordered(kth)), float_to_ordered(kth))
                          : __ldcg(&hdr->lb);
      if (isfinite(floor)) atomicMax(&hdr->floor, float_to_ordered(floor));
    }
    lbv = __shfl_sync(kFull, lbv, 0);
    const float pthr = lbv == kOrderedNegInf ? -INFINITY : ordered_to_float(lbv) - 2.0f * kMargin;
    const bool pub = isfinite(m.s) && m.s >= pthr;
    const int cnt = __popc(__ballot_sync(kFull, pub));
    if (cnt) {
      // lanes 0..cnt-1 hold the published entries (the list is sorted)
      float es = -INFINITY;
      if (pub) {
        es = exact_score_tail<D, T, INL>(p.rows + (int64_t)m.id * D, sm.qd, sm.qn,
                                         INL ? 0.0f : __ldg(p.norms + m.id));
      }
      unsigned at = 0;
      if (lane == 0) at = atomicAdd(&hdr->nent, (unsigned)cnt);
      at = __shfl_sync(kFull, at, 0);
      if (pub) {
        p.scratch.entries(q)[at + lane] = Entry{m.s, m.id};
        p.scratch.exact(q)[at + lane] = es;
      }
    }
    __syncwarp();
    if (lane == 0) {
      // acq_rel: releases this warp's entries (ordered before by __syncwarp)
      // to the block that draws the last ticket, and acquires every other
      // block's when this one does; __syncthreads passes that on to the block.
      unsigned ticket;
      asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;"
                   : "=r"(ticket)
                   : "l"(&hdr->done)
                   : "memory");
      sm.last = (ticket == gridDim.x - 1);
    }
  }
  __syncthreads();
  if (!sm.last) return;
  final_merge<D, T, INL, NW, false, true>(p, q, kMargin, safe, lane, warp, sm);
}

// The reference query (as doubles) and its reference norm for the blocks'
// exact refine, by one warp while the others stream.
template <int D, int NW>
__device__ __forceinline__ void prep_exact_query(FinishSmem<NW, D>& sm, int lane) {
  for (int d = lane; d < D; d += 32) sm.qd[d] = (double)sm.qraw[d];
  if (lane == 0) sm.qn = query_norm_seq_t<D>(sm.qraw);
}

// Approximate streaming pass (one launch per batch of queries: grid.y = query).
// INL: no precomputed norms -- the approximate row norm is accumulated from
// the same loads (fp32, <= 8 ulp relative, inside the margin) and the exact
// refine recomputes the reference norm.
template <int D, typename T, bool INL = false, bool MULTI = false>
__global__ void __launch_bounds__(kThreads) mla_scan_kernel(const __grid_constant__ Params<T> p) {
  constexpr int E = 16 / (int)sizeof(T);
  constexpr int CPR = D / E;
  constexpr int L = CPR >= 32 ? 32 : CPR;
  constexpr int R = 32 / L;
  constexpr int CPL = CPR >= 32 ? CPR / 32 : 1;
  constexpr int SLOTS = L;

  __shared__ FinishSmem<kWarps, D> fsm;
  __shared__ float sh_q[D];
  __shared__ float sh_eq;
  __shared__ int sh_safe;
  __shared__ int sh_next;

  // May be launched as a programmatic dependent of the previous route's
  // resolve kernel: wait for it (and for the query's producer) first.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int q = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* query = query_ptr(p, q, D);

  // Prologue: unit-normalised query (any accurate norm will do for the
  // approximate pass; the exact refine recomputes the reference norm).
  if (warp == 0) {
    double acc = 0.0;
    for (int d = lane; d < D; d += 32) {
      const double v = (double)query[d];
      acc = fma(v, v, acc);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(kFull, acc, o);
    const double qn = sqrt(acc);
    const bool safe = isfinite(qn) && qn > kSafeLo && qn < kSafeHi;
    const float inv = safe ? (float)(1.0 / qn) : 0.0f;
    for (int d = lane; d < D; d += 32) {
      const float v = query[d];
      fsm.qraw[d] = v;
      sh_q[d] = v * inv;
    }
    if (lane == 0) {
      sh_safe = safe;
      sh_eq = safe ? (float)(1.0e-8 / qn) : 0.0f;
    }
  }
  __syncthreads();
  const bool safe = sh_safe != 0;
  const float e_q = sh_eq;
  if constexpr (!MULTI) {
    if (warp == 1 && safe) prep_exact_query<D, kWarps>(fsm, lane);
  }

  float qr[CPL * E];
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = (CPR >= 32) ? lane + 32 * i : lane % L;
#pragma unroll
    for (int e = 0; e < E; ++e) qr[i * E + e] = sh_q[c * E + e];
  }

  WarpList list;
  list.init();
  const int64_t groups = ceil_div64(p.nodes, 32);
  // Each block streams one contiguous range of 32-row groups (equal to +-1
  // group per block, so every SM moves the same bytes); its warps take groups
  // from that range through a shared-memory counter.
  const int64_t g_begin = groups * blockIdx.x / gridDim.x;
  const int64_t g_end = groups * (blockIdx.x + 1) / gridDim.x;
  if (threadIdx.x == 0) sh_next = kWarps;
  __syncthreads();
  if (safe) {
    constexpr int B = 8;  // 16-byte loads in flight per lane per batch
    for (int64_t g = g_begin + warp; g < g_end;) {
      const int64_t row0 = g * 32;
      const int64_t my_row = row0 + (lane % L) * R + lane / L;
      const float nrm_pre = (!INL && my_row < p.nodes) ? __ldg(p.norms + my_row) : 0.0f;
      float part[SLOTS];
      float sq[INL ? SLOTS : 1];
      if (row0 + 32 <= p.nodes) {
        // full group: unchecked, batched loads
        const T* base = p.rows + (row0 + lane / L) * D;
#pragma unroll
        for (int jb = 0; jb < SLOTS; jb += B) {
          uint4 v[B][CPL];
#pragma unroll
          for (int b = 0; b < B; ++b)
#pragma unroll
            for (int i = 0; i < CPL; ++i) {
              const int c = (CPR >= 32) ? lane + 32 * i : lane % L;
              v[b][i] = ld_nc16(base + (int64_t)(jb + b) * R * D + c * E);
            }
#pragma unroll
          for (int b = 0; b < B; ++b) {
            float acc = 0.0f, sacc = 0.0f;
#pragma unroll
            for (int i = 0; i < CPL; ++i) {
              acc = dot16<T>(v[b][i], qr + i * E, acc);
              if constexpr (INL) sacc = sq16<T>(v[b][i], sacc);
            }
            part[jb + b] = acc;
            if constexpr (INL) sq[jb + b] = sacc;
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < SLOTS; ++j) {
          const int64_t row = row0 + j * R + lane / L;
          float acc = 0.0f, sacc = 0.0f;
          if (row < p.nodes) {
            const T* rp = p.rows + row * D;
#pragma unroll
            for (int i = 0; i < CPL; ++i) {
              const int c = (CPR >= 32) ? lane + 32 * i : lane % L;
              const uint4 v = ld_nc16(rp + c * E);
              acc = dot16<T>(v, qr + i * E, acc);
              if constexpr (INL) sacc = sq16<T>(v, sacc);
            }
          }
          part[j] = acc;
          if constexpr (INL) sq[j] = sacc;
        }
      }
      const float dot = reduce_scatter<SLOTS>(part, lane);
      float n2 = 0.0f;
      if constexpr (INL) n2 = reduce_scatter<SLOTS>(sq, lane);
      if constexpr (MULTI) {
        if (my_row < p.nodes) {
          const uint32_t ent = __ldg(p.entry_of_row + my_row);
          if (policy::row_allowed(p.allow, ent) && isfinite(nrm_pre)) {
            const float s = dot * __frcp_rn(nrm_pre + e_q);
            if (isfinite(s)) atomicMax(p.entry_best + ent, float_to_ordered(s));
          }
        }
      } else {
        float s = -INFINITY;
        if (my_row < p.nodes && policy::row_allowed(p.allow, my_row)) {
          const float nrm = INL ? sqrtf(n2) : nrm_pre;
          if (isfinite(nrm)) s = dot * __frcp_rn(nrm + e_q);
        }
        list.offer_margin(s, (uint32_t)my_row, lane, p.topk, 2.0f * kMargin);
      }
      int nxt = 0;
      if (lane == 0) nxt = atomicAdd(&sh_next, 1);
      g = g_begin + __shfl_sync(kFull, nxt, 0);
    }
  }
  if constexpr (MULTI) {  // block 0 streams early groups: its tail hides the norm's chain
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      p.multi_unsafe[q] = safe ? 0 : 1;
      *p.multi_qnorm = query_norm_seq(query, D);
    }
    return;
  }
  // The resolve kernel may be scheduled as blocks leave the streaming loop;
  // it waits for this whole grid before reading anything (griddepcontrol.wait).
  asm volatile("griddepcontrol.launch_dependents;");
  scan_finish<D, T, INL, kWarps>(p, list, safe, q, lane, warp, fsm);
}

// ------------------------------------------------------ multi-row entries
// RouterIndex::exact_mla_entry_score over several rows
// (cpp/grm_runtime.cpp:3518-3545): an entry scores the max of its finite row
// scores, NaN (dropped) if none.  After the streaming pass has folded the
// approximate row scores into entry_best, the entries are selected like the
// single rows: L = the k-th best approximate entry score, candidates = the
// entries within 2*kMargin of it (every row score is within kMargin of its
// exact value, so is their max), refined exactly, top-k by (score, entry).

constexpr int kEntryWarps = 8;

// Per block: the approximate top-32 entries of a strided share.
__global__ void __launch_bounds__(kEntryWarps * 32) entry_top_kernel(
    const int* __restrict__ entry_best, int64_t entries, int topk, float* __restrict__ blk_s,
    uint32_t* __restrict__ blk_id) {
  __shared__ float sh_s[kEntryWarps * 32];
  __shared__ uint32_t sh_id[kEntryWarps * 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  WarpList list;
  list.init();
  // chunks of 32 entries, kPre loaded at once so their latencies overlap
  constexpr int kPre = 8;
  const int64_t step = (int64_t)gridDim.x * kEntryWarps * 32;
  for (int64_t e0 = ((int64_t)blockIdx.x * kEntryWarps + warp) * 32; e0 < entries;
       e0 += kPre * step) {
    float v[kPre];
#pragma unroll
    for (int j = 0; j < kPre; ++j) {
      const int64_t e = e0 + j * step + lane;
      v[j] = e < entries ? ordered_to_float(__ldcg(entry_best + e)) : -INFINITY;
    }
#pragma unroll
    for (int j = 0; j < kPre; ++j)  // only the top k must be exact
      list.offer_margin(v[j], (uint32_t)(e0 + j * step + lane), lane, topk, 0.0f);
  }
  sh_s[warp * 32 + lane] = list.s;
  sh_id[warp * 32 + lane] = list.id;
  __syncthreads();
  if (warp == 0) {
    for (int w = 1; w < kEntryWarps; ++w)
      list.offer_margin(sh_s[w * 32 + lane], sh_id[w * 32 + lane], lane, topk, 0.0f);
    blk_s[blockIdx.x * 32 + lane] = list.s;
    blk_id[blockIdx.x * 32 + lane] = list.id;
  }
}

// One warp: the k-th best over the block lists -> the candidate threshold.
// The k-th best over the block lists -> the candidate threshold.  One block
// of 32 warps: warp w merges lists w, w+32, ... (their loads overlap across
// warps), then warp 0 merges the 32 warp lists from shared memory.  The bulk
// pass's ticket counter is re-armed here for the next query.
constexpr int kThrWarps = 32;

__global__ void __launch_bounds__(kThrWarps * 32) entry_threshold_kernel(
    const float* __restrict__ blk_s, const uint32_t* __restrict__ blk_id, int nblk, int topk,
    float* __restrict__ thr, Header* hdr) {
  __shared__ float sh_s[kThrWarps * 32];
  __shared__ uint32_t sh_id[kThrWarps * 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  WarpList list;
  list.init();
  for (int b = warp; b < nblk; b += kThrWarps)
    list.offer_margin(blk_s[b * 32 + lane], blk_id[b * 32 + lane], lane, topk, 0.0f);
  sh_s[warp * 32 + lane] = list.s;
  sh_id[warp * 32 + lane] = list.id;
  __syncthreads();
  if (warp == 0) {
    for (int w = 1; w < kThrWarps; ++w)
      list.offer_margin(sh_s[w * 32 + lane], sh_id[w * 32 + lane], lane, topk, 0.0f);
    const float kth = __shfl_sync(kFull, list.s, topk - 1);
    if (lane == 0) {
      *thr = isfinite(kth) ? kth - 2.0f * kMargin : -INFINITY;
      hdr->next = 0;
    }
  }
}

// Candidates: entries at or above the threshold (every entry with rows when
// the query is outside the safe range or the bank outside the fast path);
// entry_best is reset for the next query on the way.
__global__ void entry_collect_kernel(int* __restrict__ entry_best, const uint64_t* __restrict__ off,
                                     int64_t entries, const float* __restrict__ thr,
                                     const int* __restrict__ unsafe, int force_all,
                                     uint32_t* __restrict__ cand, unsigned* __restrict__ count) {
  const float t = *thr;
  const bool all = force_all || *unsafe;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < entries;
       e += (int64_t)gridDim.x * blockDim.x) {
    const float v = ordered_to_float(entry_best[e]);
    entry_best[e] = kOrderedNegInf;
    const bool pick = all ? off[e + 1] > off[e] : (v >= t && v > -INFINITY);
    if (pick) cand[atomicAdd(count, 1u)] = (uint32_t)e;
  }
}

// Exact entry scores of the candidates: a warp per entry.  The entry's rows
// are staged in shared memory with coalesced loads, kRows at a time, and
// lane j runs row j's sequential fp64 dot (the reference's order) from there;
// the entry scores the max of its finite rows.
template <typename T>
struct RefineShape {
  static constexpr int kRows = sizeof(T) == 2 ? 8 : 4;   // rows staged per warp
  static constexpr int kMaxDim = 256;
};

// qnorm_in: the query's reference norm computed by an earlier kernel, or
// nullptr (computed here).  Rows go to shared memory with 16-byte loads when
// a row is a whole number of 16-byte chunks.
template <typename T>
__global__ void __launch_bounds__(kEntryWarps * 32) entry_refine_kernel(
    const T* __restrict__ rows, const float* __restrict__ norms, int dim,
    const float* __restrict__ query, const uint64_t* __restrict__ off,
    const uint32_t* __restrict__ cand, const unsigned* __restrict__ count,
    const uint32_t* __restrict__ allow, float* __restrict__ cand_s,
    const double* __restrict__ qnorm_in) {
  constexpr int NR = RefineShape<T>::kRows;
  constexpr int MD = RefineShape<T>::kMaxDim;
  constexpr int EV = 16 / (int)sizeof(T);  // elements per 16-byte chunk
  __shared__ float qs[MD];
  __shared__ __align__(16) T rbuf[kEntryWarps][NR][MD];
  __shared__ double qn;
  for (int d = threadIdx.x; d < dim; d += blockDim.x) qs[d] = query[d];
  __syncthreads();
  if (threadIdx.x == 0) {
    if (qnorm_in) {
      qn = *qnorm_in;
    } else {
      double acc = 0.0;
#pragma unroll 8
      for (int d = 0; d < dim; ++d) acc += (double)qs[d] * (double)qs[d];
      qn = sqrt(acc);
    }
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool vec = dim % EV == 0;
  const unsigned n = *count;
  for (unsigned i = blockIdx.x * kEntryWarps + warp; i < n; i += gridDim.x * kEntryWarps) {
    const uint32_t e = cand[i];
    float best = -INFINITY;
    if (policy::row_allowed(allow, e)) {
      for (uint64_t r0 = off[e]; r0 < off[e + 1]; r0 += NR) {
        const int nr = (int)min((uint64_t)NR, off[e + 1] - r0);
        const T* src = rows + r0 * dim;  // nr consecutive rows
        if (vec) {  // rbuf rows are MD elements apart, source rows dim apart
          const int cpr = dim / EV;
#pragma unroll 4
          for (int x = lane; x < nr * cpr; x += 32) {
            const int j = x / cpr, c = x - j * cpr;
            *reinterpret_cast<uint4*>(&rbuf[warp][j][c * EV]) =
                __ldg(reinterpret_cast<const uint4*>(src + (int64_t)j * dim) + c);
          }
        } else {
#pragma unroll 8
          for (int x = lane; x < nr * dim; x += 32) rbuf[warp][x / dim][x % dim] = src[x];
        }
        __syncwarp();
        if (lane < nr) {
          const float nrm = __ldg(norms + r0 + lane);
          if (isfinite(nrm)) {
            double dot = 0.0;
#pragma unroll 8
            for (int d = 0; d < dim; ++d)
              dot = fma((double)qs[d], (double)to_f(rbuf[warp][lane][d]), dot);
            const float sc = (float)(dot / (qn * (double)nrm + 1.0e-8));
            if (isfinite(sc)) best = fmaxf(best, sc);
          }
        }
        __syncwarp();
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) best = fmaxf(best, __shfl_xor_sync(kFull, best, o));
    if (lane == 0) cand_s[i] = best;  // -inf: no finite row (dropped)
  }
}

// Banks wider than the staging buffer: a lane per row reading global memory.
template <typename T>
__global__ void __launch_bounds__(kEntryWarps * 32) entry_refine_wide_kernel(
    const T* __restrict__ rows, const float* __restrict__ norms, int dim,
    const float* __restrict__ query, const uint64_t* __restrict__ off,
    const uint32_t* __restrict__ cand, const unsigned* __restrict__ count,
    const uint32_t* __restrict__ allow, float* __restrict__ cand_s) {
  __shared__ double qn;
  if (threadIdx.x == 0) qn = query_norm_seq(query, dim);
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned n = *count;
  for (unsigned i = blockIdx.x * kEntryWarps + warp; i < n; i += gridDim.x * kEntryWarps) {
    const uint32_t e = cand[i];
    float best = -INFINITY;
    if (policy::row_allowed(allow, e)) {
      for (uint64_t r = off[e] + lane; r < off[e + 1]; r += 32) {
        const float nrm = __ldg(norms + r);
        if (!isfinite(nrm)) continue;
        const float sc = exact_score<T>(rows + r * dim, dim, query, qn, nrm);
        if (isfinite(sc)) best = fmaxf(best, sc);
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) best = fmaxf(best, __shfl_xor_sync(kFull, best, o));
    if (lane == 0) cand_s[i] = best;
  }
}

// Top-k of the scored candidates into the query's Result.
__global__ void __launch_bounds__(kEntryWarps * 32) entry_finalize_kernel(
    const uint32_t* __restrict__ cand, const float* __restrict__ cand_s,
    unsigned* __restrict__ count, int topk, uint64_t id_offset, Result* __restrict__ r,
    uint64_t* out_ids, float* out_scores, Header* hdr) {
  __shared__ float sh_s[kEntryWarps * 32];
  __shared__ uint32_t sh_id[kEntryWarps * 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned n = *count;
  WarpList list;
  list.init();
  for (unsigned i0 = warp * 32; i0 < n; i0 += blockDim.x) {
    const unsigned i = i0 + lane;
    list.offer_margin(i < n ? cand_s[i] : -INFINITY, i < n ? cand[i] : kNoRow, lane, topk, 0.0f);
  }
  sh_s[warp * 32 + lane] = list.s;
  sh_id[warp * 32 + lane] = list.id;
  __syncthreads();
  if (warp == 0) {
    for (int w = 1; w < kEntryWarps; ++w)
      list.offer_margin(sh_s[w * 32 + lane], sh_id[w * 32 + lane], lane, topk, 0.0f);
    const bool ok = lane < topk && isfinite(list.s) && list.id != kNoRow;
    const unsigned m = __ballot_sync(kFull, ok);
    if (lane < topk) {
      const uint64_t id = ok ? (uint64_t)list.id + id_offset : UINT64_MAX;
      const float sc = ok ? list.s : __int_as_float(0x7FC00000);
      r->ids[lane] = id;
      r->scores[lane] = sc;
      if (out_ids) out_ids[lane] = id;
      if (out_scores) out_scores[lane] = sc;
    }
    if (lane == 0) {
      r->count = __popc(m);
      r->status = hdr->err ? kError : kOk;  // a bounded wait of the pass gave up
      hdr->err = 0;
      *count = 0u;
    }
  }
}

// Packed fp32x2 FMA (sm_100 FFMA2): d = a * b + c on both lanes of a float2.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// One 16-byte slice dotted with its 16/sizeof(T) query values, two partial
// sums (even / odd elements) in a float2.
template <typename T>
__device__ __forceinline__ float2 dot16x2(const uint4& v, const float2* q2, float2 acc) {
  if constexpr (sizeof(T) == 2) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int k = 0; k < 4; ++k) acc = ffma2(__half22float2(h[k]), q2[k], acc);
  } else {
    acc = ffma2(make_float2(__uint_as_float(v.x), __uint_as_float(v.y)), q2[0], acc);
    acc = ffma2(make_float2(__uint_as_float(v.z), __uint_as_float(v.w)), q2[1], acc);
  }
  return acc;
}

// Bulk-copy streaming pass: the same law and epilogue as mla_scan_kernel.
// Each of the kBulkWarps warps streams its 32-row groups as two 16-row halves
// through two shared-memory buffers filled by cp.async.bulk (the next group's
// half is in flight while the current one is consumed), so the bytes in
// flight per SM no longer depend on registers, and 12 warps hide the
// arithmetic latency.  Used when a 16-row half is at most 8 KB (fp16
// D <= 256, fp32 D <= 128).  The dot products use packed f32x2 FMAs (two
// partial sums per slot): the approximation bound gains one rounding step.
constexpr int kBulkWarps = 12;
constexpr int kHalfBytes = 8192;
constexpr int kBulkSmem = kBulkWarps * 2 * kHalfBytes;

template <int D, typename T, bool MULTI = false>
__global__ void __launch_bounds__(kBulkWarps * 32, 1)
    mla_scan_bulk_kernel(const __grid_constant__ Params<T> p) {
  constexpr int NW = kBulkWarps;
  constexpr int E = 16 / (int)sizeof(T);
  constexpr int CPR = D / E;
  constexpr int L = CPR >= 32 ? 32 : CPR;
  constexpr int R = 32 / L;
  constexpr int SLOTS = L;
  constexpr int HS = SLOTS / 2;  // slots per 16-row half
  static_assert(CPR <= 32 && 16 * D * (int)sizeof(T) <= kHalfBytes, "half group must fit");

  extern __shared__ __align__(128) unsigned char dsmem[];
  __shared__ __align__(8) uint64_t sh_bar[NW][2];
  __shared__ FinishSmem<NW, D> fsm;
  __shared__ float sh_q[D];
  __shared__ float sh_eq;
  __shared__ int sh_safe;

  const int q = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned char* const buf0 = dsmem + (warp * 2) * kHalfBytes;
  const int64_t groups = ceil_div64(p.nodes, 32);
  const uint64_t l2_stream = l2_evict_first_policy();
  // half h of group g -> buffer h (lane 0 only)
  auto issue = [&](int64_t g, int h) {
    const int64_t r0 = g * 32 + 16 * h;
    const int64_t rows = max((int64_t)0, min((int64_t)16, p.nodes - r0));
    const unsigned bytes = (unsigned)(rows * D * (int64_t)sizeof(T));
    if (bytes == 0) {
      mbar_arrive_expect_tx(&sh_bar[warp][h], 0);  // completes the phase at once
      return;
    }
    mbar_arrive_expect_tx(&sh_bar[warp][h], bytes);
    bulk_g2s_hint(buf0 + h * kHalfBytes, p.rows + r0 * D, bytes, &sh_bar[warp][h], l2_stream);
  };
  // The bank is written only when it is created, so each warp starts its
  // first group's two copies before waiting for the kernel this launch may
  // depend on (the previous route's resolve kernel, or the query's
  // producer): the first bytes land while that kernel ends and the query is
  // normalised.  Scratch and queries are touched only after the wait.
  const int64_t g_first = (int64_t)blockIdx.x * NW + warp;
  if (lane == 0) {
    mbar_init(&sh_bar[warp][0], 1);
    mbar_init(&sh_bar[warp][1], 1);
    mbar_fence_init();
    if (g_first < groups) {
      issue(g_first, 0);
      issue(g_first, 1);
    }
  }
  unsigned pending_bits = g_first < groups ? 3u : 0u;  // bit h: a copy into buffer h is in flight
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const float* query = query_ptr(p, q, D);

  if (warp == 0) {
    double acc = 0.0;
    for (int d = lane; d < D; d += 32) {
      const double v = (double)query[d];
      acc = fma(v, v, acc);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(kFull, acc, o);
    const double qn = sqrt(acc);
    const bool safe = isfinite(qn) && qn > kSafeLo && qn < kSafeHi;
    const float inv = safe ? (float)(1.0 / qn) : 0.0f;
    for (int d = lane; d < D; d += 32) {
      const float v = query[d];
      fsm.qraw[d] = v;
      sh_q[d] = v * inv;
    }
    if (lane == 0) {
      sh_safe = safe;
      sh_eq = safe ? (float)(1.0e-8 / qn) : 0.0f;
    }
  }
  __syncthreads();
  const bool safe = sh_safe != 0;
  const float e_q = sh_eq;
  if constexpr (!MULTI) {
    if (warp == 1 && safe) prep_exact_query<D, NW>(fsm, lane);
  }
  const int c = lane % L;
  float2 q2[E / 2];
#pragma unroll
  for (int e = 0; e < E / 2; ++e) q2[e] = make_float2(sh_q[c * E + 2 * e], sh_q[c * E + 2 * e + 1]);

  // Static interleaved assignment: warp w of block b takes groups
  // b*NW + w, then every gridDim.x*NW-th group after it, so the warps of the
  // whole grid sweep the bank front to back together.  The last two rounds
  // (dyn0 onwards) are handed out one group at a time through hdr->next, so
  // SMs that stream faster take more of the tail; each ticket is requested a
  // full group ahead of its use.
  const int64_t gstride = (int64_t)gridDim.x * NW;
  const int64_t dyn0 = groups >= 4 * gstride ? (groups / gstride - 2) * gstride : groups;
  unsigned* const next = &p.scratch.hdr(q)->next;

  WarpList list;
  list.init();
  bool failed = false;
  unsigned phase_bits = 0u;    // bit h: parity of the next phase to wait for on buffer h
  if (!safe && pending_bits) {
    // nothing is streamed for this query: drain the copies started above
    for (int k = 0; k < 2; ++k) mbar_wait(&sh_bar[warp][k], 0u, kWaitLimit);
    pending_bits = 0u;
  }
  if (safe) {
    int64_t g = g_first;
    int64_t gn = g + gstride;
    while (g < groups) {
      // the group after gn: static, or a ticket whose atomic completes while
      // this group is processed
      const bool ticket = gn < groups && (gn >= dyn0 || gn + gstride >= dyn0);
      unsigned tk = 0;
      if (ticket && lane == 0) tk = atomicAdd(next, 1u);
      const int64_t row0 = g * 32;
      const int64_t my_row = row0 + (lane % L) * R + lane / L;
      const float nrm_pre = my_row < p.nodes ? __ldg(p.norms + my_row) : 0.0f;
      const int valid = (int)min((int64_t)32, p.nodes - row0);
      float part[SLOTS];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (!mbar_wait(&sh_bar[warp][h], (phase_bits >> h) & 1u, p.wait_limit)) {
          failed = true;
          break;
        }
        phase_bits ^= 1u << h;
        pending_bits &= ~(1u << h);
        const T* sb = reinterpret_cast<const T*>(buf0 + h * kHalfBytes);
        if (valid == 32) {  // every group but possibly the bank's last one
#pragma unroll
          for (int jj = 0; jj < HS; ++jj) {
            const int r = jj * R + lane / L;  // row within the half
            const uint4 v = *reinterpret_cast<const uint4*>(sb + r * D + c * E);
            const float2 a2 = dot16x2<T>(v, q2, make_float2(0.0f, 0.0f));
            part[h * HS + jj] = a2.x + a2.y;
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < HS; ++jj) {
            const int r = jj * R + lane / L;
            const uint4 v = (16 * h + r) < valid
                                ? *reinterpret_cast<const uint4*>(sb + r * D + c * E)
                                : make_uint4(0, 0, 0, 0);
            const float2 a2 = dot16x2<T>(v, q2, make_float2(0.0f, 0.0f));
            part[h * HS + jj] = a2.x + a2.y;
          }
        }
        // this half's buffer is free again: start the next group's half
        __syncwarp();
        fence_proxy_async_smem();
        if (gn < groups) {
          if (lane == 0) issue(gn, h);
          pending_bits |= 1u << h;
        }
      }
      if (failed) break;
      const float dot = reduce_scatter<SLOTS>(part, lane);
      if constexpr (MULTI) {  // fold into the row's entry (see mla_scan_kernel)
        if (my_row < p.nodes && isfinite(nrm_pre)) {
          const uint32_t ent = __ldg(p.entry_of_row + my_row);
          if (policy::row_allowed(p.allow, ent)) {
            const float s = dot * __frcp_rn(nrm_pre + e_q);
            if (isfinite(s)) atomicMax(p.entry_best + ent, float_to_ordered(s));
          }
        }
      } else {
        float s = -INFINITY;
        if (my_row < p.nodes && isfinite(nrm_pre) && policy::row_allowed(p.allow, my_row))
          s = dot * __frcp_rn(nrm_pre + e_q);
        list.offer_margin(s, (uint32_t)my_row, lane, p.topk, 2.0f * kMargin);
      }
      g = gn;
      gn = ticket ? dyn0 + (int64_t)__shfl_sync(kFull, tk, 0) : gn + gstride;
    }
    if (failed) {
      // drain this warp's copies still in flight before the block can exit
      for (int k = 0; k < 2; ++k)
        if ((pending_bits >> k) & 1u)
          mbar_wait(&sh_bar[warp][k], (phase_bits >> k) & 1u, kWaitLimit);
      if (lane == 0) atomicOr(&p.scratch.hdr(q)->err, 1);
    }
  }
  if constexpr (MULTI) {  // the entry kernels reset hdr->next and read hdr->err
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      p.multi_unsafe[q] = safe ? 0 : 1;
      *p.multi_qnorm = query_norm_seq(query, D);
    }
    return;
  }
  asm volatile("griddepcontrol.launch_dependents;");
  scan_finish<D, T, false, NW>(p, list, safe, q, lane, warp, fsm);
}

constexpr int kExactQ = 64;  // queries per block row of the exact kernel

// Shared memory of the exact pass.
template <int D>
struct ExactSmem {
  float s[kWarps * 32];
  uint32_t id[kWarps * 32];
  float q[D > 0 ? D : 1];
  double qnorm;
  float eq;
  int last;
  int work[kExactQ];
  int nwork;
};

// The exact pass of one query (every thread of the block calls it).  kOverflow:
// exact scores for every row whose approximate score reaches the threshold;
// kUnsafe (or force_all): exact scores for every row.
template <int D, typename T, bool INL>
__device__ __forceinline__ void exact_one(const Params<T>& p, int q, int lane, int warp,
                                          ExactSmem<D>& sm) {
  const int dim = D > 0 ? D : p.dim;
  const float* query = query_ptr(p, q, dim);
  Result* r = p.results + q;
  __syncthreads();  // sm is reused from the previous query
  if (threadIdx.x == 0) {
    const double qn = query_norm_seq(query, dim);
    sm.qnorm = qn;
    sm.eq = (float)(1.0e-8 / qn);
    if (blockIdx.x == 0 && p.fallback_count) atomicAdd(p.fallback_count, 1ull);
  }
  __syncthreads();
  const int mode = p.force_all ? (int)kUnsafe : __ldcg(&r->status);
  const double qnorm = sm.qnorm;

  WarpList list;
  list.init();
  if (mode == kUnsafe || D == 0) {
    // Every row, one row per lane, in reference arithmetic.
    for (int64_t row0 = ((int64_t)blockIdx.x * kWarps + warp) * 32; row0 < p.nodes;
         row0 += (int64_t)gridDim.x * kWarps * 32) {
      const int64_t row = row0 + lane;
      float es = -INFINITY;
      if (row < p.nodes && policy::row_allowed(p.allow, row)) {
        if constexpr (INL) {
          es = exact_score_inline_norm<T>(p.rows + row * dim, dim, query, qnorm);
        } else {
          const float nrm = __ldg(p.norms + row);
          if (isfinite(nrm)) es = exact_score<T>(p.rows + row * dim, dim, query, qnorm, nrm);
        }
      }
      list.offer(es, (uint32_t)row, lane);
    }
  } else if constexpr (D > 0) {
    constexpr int E = 16 / (int)sizeof(T);
    constexpr int CPR = D / E;
    constexpr int L = CPR >= 32 ? 32 : CPR;
    constexpr int R = 32 / L;
    constexpr int CPL = CPR >= 32 ? CPR / 32 : 1;
    constexpr int SLOTS = L;
    const float thr = __ldcg(&r->thr);
    const float e_q = sm.eq;
    if (warp == 0) {
      const float inv = (float)(1.0 / qnorm);
      for (int d = lane; d < D; d += 32) sm.q[d] = query[d] * inv;
    }
    __syncthreads();
    float qr[CPL * E];
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int c = (CPR >= 32) ? lane + 32 * i : lane % L;
#pragma unroll
      for (int e = 0; e < E; ++e) qr[i * E + e] = sm.q[c * E + e];
    }
    const int64_t groups = ceil_div64(p.nodes, 32);
    for (int64_t g = (int64_t)blockIdx.x * kWarps + warp; g < groups;
         g += (int64_t)gridDim.x * kWarps) {
      const int64_t row0 = g * 32;
      float part[SLOTS];
      float sq[INL ? SLOTS : 1];
#pragma unroll
      for (int j = 0; j < SLOTS; ++j) {
        const int64_t row = row0 + j * R + lane / L;
        float acc = 0.0f, sacc = 0.0f;
        if (row < p.nodes) {
          const T* rp = p.rows + row * D;
#pragma unroll
          for (int i = 0; i < CPL; ++i) {
            const int c = (CPR >= 32) ? lane + 32 * i : lane % L;
            const uint4 v = *reinterpret_cast<const uint4*>(rp + c * E);
            acc = dot16<T>(v, qr + i * E, acc);
            if constexpr (INL) sacc = sq16<T>(v, sacc);
          }
        }
        part[j] = acc;
        if constexpr (INL) sq[j] = sacc;
      }
      const float dot = reduce_scatter<SLOTS>(part, lane);
      float n2 = 0.0f;
      if constexpr (INL) n2 = reduce_scatter<SLOTS>(sq, lane);
      const int64_t row = row0 + (lane % L) * R + lane / L;
      float es = -INFINITY;
      if (row < p.nodes && policy::row_allowed(p.allow, row)) {
        const float nrm = INL ? sqrtf(n2) : __ldg(p.norms + row);
        if (isfinite(nrm)) {
          const float s = dot * __frcp_rn(nrm + e_q);
          if (s >= thr) {
            if constexpr (INL)
              es = exact_score_inline_norm<T>(p.rows + row * D, D, query, qnorm);
            else
              es = exact_score<T>(p.rows + row * D, D, query, qnorm, nrm);
          }
        }
      }
      list.offer(es, (uint32_t)row, lane);
    }
  }

  block_merge(list, lane, warp, sm.s, sm.id);
  Header* hdr = p.scratch.hdr(q);
  if (warp == 0) {
    const bool keep = lane < p.topk && isfinite(list.s);
    const int cnt = __popc(__ballot_sync(kFull, keep));
    Entry* ent = p.scratch.entries(q) + (int64_t)blockIdx.x * 32;
    if (lane < cnt) ent[lane] = Entry{list.s, list.id};
    if (lane == 0) {
      p.scratch.counts(q)[blockIdx.x] = cnt;
      __threadfence();
      const unsigned ticket = atomicAdd(&hdr->done, 1u);
      sm.last = (ticket == gridDim.x - 1);
    }
  }
  __syncthreads();
  if (!sm.last) return;
  __threadfence();
  list.init();
  for (int b = warp; b < (int)gridDim.x; b += kWarps) {
    const int cnt = __ldcg(p.scratch.counts(q) + b);
    const Entry* ent = p.scratch.entries(q) + (int64_t)b * 32;
    float s = -INFINITY;
    uint32_t id = kNoRow;
    if (lane < cnt) {
      s = __ldcg(&ent[lane].s);
      id = __ldcg(&ent[lane].id);
    }
    list.offer(s, id, lane);
  }
  block_merge(list, lane, warp, sm.s, sm.id);
  if (warp == 0) {
    write_result(p, q, list, lane);
    if (lane == 0) {  // the scan's final merge already reset the rest of the header
      hdr->lb = kOrderedNegInf;
      hdr->done = 0;
    }
  }
}

// Exact fallback (the resolve phase after every scan).  Block row y covers
// queries [64y, 64y + 64): the block reads their statuses in one pass and
// runs exact_one for those whose approximate pass reported kOverflow or
// kUnsafe (all of them under force_all); queries with kOk (or kError) cost
// nothing more.  D == 0 means runtime dim (force_all only).  INL: row norms
// computed inline (see mla_scan_kernel).
//
// At most 64 registers a thread (16K a block): the resolve blocks of one
// route wait, resident, beside the per-query merge blocks of a batched route
// while the next route's scan CTAs start on the same SMs as the previous
// scan's CTAs exit, and the three must fit one register file (a scan CTA
// 33K, a merge block 12K).  The exact pass itself is the rare path.
template <int D, typename T, bool INL = false>
__global__ void __launch_bounds__(kThreads, 4) mla_exact_kernel(const __grid_constant__ Params<T> p) {
  __shared__ ExactSmem<D> sm;
  // Launched with programmatic dependent launch after the scan.  Every block
  // of this grid is resident once it reaches the trigger, so the next route's
  // scan may be scheduled at once: until its own wait on this grid it only
  // starts copies of the read-only bank, overlapping the scan's last block.
  // Then wait until the scan grid has completed and its writes are visible.
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int q0 = (int)blockIdx.y * kExactQ;
  const int nq = min(kExactQ, p.nq - q0);
  if (threadIdx.x == 0) sm.nwork = 0;
  __syncthreads();
  for (int t = threadIdx.x; t < nq; t += blockDim.x) {
    const int st = p.force_all ? (int)kUnsafe : __ldcg(&p.results[q0 + t].status);
    if (st == kOverflow || st == kUnsafe) sm.work[atomicAdd(&sm.nwork, 1)] = q0 + t;
  }
  __syncthreads();
  const int nwork = sm.nwork;
  for (int w = 0; w < nwork; ++w) exact_one<D, T, INL>(p, sm.work[w], lane, warp, sm);
}

template <typename T>
__global__ void row_norms_kernel(const T* rows, int64_t n, int dim, float* norms,
                                 unsigned* special) {
  for (int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; row < n;
       row += (int64_t)gridDim.x * blockDim.x) {
    const T* rp = rows + row * dim;
    double acc = 0.0;
    bool finite = true;
    float maxabs = 0.0f;
    for (int d = 0; d < dim; ++d) {
      const float v = to_f(rp[d]);
      finite = finite && isfinite(v);
      maxabs = fmaxf(maxabs, fabsf(v));
      acc = fma((double)v, (double)v, acc);
    }
    float nrm = (float)sqrt(acc);
    if (!finite) {
      nrm = __int_as_float(0x7FC00000);  // any non-finite value: the reference score is NaN
    } else if (!isfinite(nrm) || maxabs > 1.0e30f) {
      atomicAdd(special, 1u);            // outside the fast path's proven range
    } else if (nrm < kBMinNorm) {
      atomicAdd(special + 1, 1u);        // outside the batched path's proven range
    }
    norms[row] = nrm;
  }
}

// Lexical channel of route_mla_arena (cpp/grm_runtime.cpp:4339-4350): every
// allowed node with lexical hits gets S = exact score + hits / m (fp32 divide,
// fp32 add); non-finite S is dropped by the merge.  A warp per hit node: the
// lanes load the row with independent strided loads into shared memory, then
// lane 0 runs the reference's sequential fp64 dot over it (one memory round
// trip per node instead of one per unrolled slice of the chain).
constexpr int kLexWarps = 4;
constexpr int kLexMaxDim = 1024;

template <typename T>
__global__ void __launch_bounds__(kLexWarps * 32) mla_lex_score_kernel(
    const T* __restrict__ rows, const float* __restrict__ norms, int dim,
    const float* __restrict__ query, const uint2* __restrict__ list,
    const uint32_t* __restrict__ counter, const uint32_t* __restrict__ allow, int m,
    const uint64_t* __restrict__ entry_off, float* __restrict__ cand_s,
    uint32_t* __restrict__ cand_id) {
  __shared__ float qs[kLexMaxDim];
  __shared__ float rowbuf[kLexWarps][kLexMaxDim];
  __shared__ double qn;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int d = threadIdx.x; d < dim; d += blockDim.x) qs[d] = query[d];
  __syncthreads();
  if (threadIdx.x == 0) {  // the reference's query norm (sequential fp64)
    double acc = 0.0;
#pragma unroll 8
    for (int d = 0; d < dim; ++d) acc += (double)qs[d] * (double)qs[d];
    qn = sqrt(acc);
  }
  __syncthreads();
  const uint32_t n = *counter;
  const uint32_t nw = gridDim.x * kLexWarps;
  for (uint32_t i = blockIdx.x * kLexWarps + warp; i < n; i += nw) {
    const uint2 h = list[i];
    const bool ok = policy::row_allowed(allow, h.x);
    // a node's rows: itself, or its entry's rows in a multi-row bank (max)
    const uint64_t r0 = entry_off ? entry_off[h.x] : h.x;
    const uint64_t r1 = entry_off ? entry_off[h.x + 1] : (uint64_t)h.x + 1;
    float best = -INFINITY;
    for (uint64_t r = r0; ok && r < r1; ++r) {
      const T* row = rows + (int64_t)r * dim;
      for (int d = lane; d < dim; d += 32) rowbuf[warp][d] = to_f(__ldg(row + d));
      const float nrm = __ldg(norms + r);
      __syncwarp();
      if (lane == 0 && isfinite(nrm)) {
        double dot = 0.0;
#pragma unroll 8
        for (int d = 0; d < dim; ++d) dot = fma((double)qs[d], (double)rowbuf[warp][d], dot);
        const float es = (float)(dot / (qn * (double)nrm + 1.0e-8));
        if (isfinite(es)) best = fmaxf(best, es);
      }
      __syncwarp();
    }
    if (lane == 0) {
      cand_s[i] = best > -INFINITY ? best + __fdiv_rn((float)h.y, (float)m) : -INFINITY;
      cand_id[i] = h.x;
    }
  }
}

__global__ void scratch_init_kernel(unsigned char* base, size_t stride, int queries) {
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q < queries) {
    Header* h = reinterpret_cast<Header*>(base + stride * q);
    reset_header(h);
    h->err = 0;
  }
}

}  // namespace mla
}  // namespace grm_b200

using namespace grm_b200;
using namespace grm_b200::mla;

struct grm_b200_mla_bank {
  int device = 0;
  int dtype = GRM_B200_F16;
  int64_t nodes = 0;
  int dim = 0;
  void* d_rows = nullptr;
  float* d_norms = nullptr;
  bool exact_only = false;
  bool bulk = false;         // scan with the bulk-copy kernel
  bool batch = false;        // batches of queries go to the tensor-core route
  float* d_rnorms = nullptr;        // its 2^-8 / row norm table
  CUtensorMap tmap;                 // its bank tensor map
  int grid_x = 1;
  int scratch_queries = 0;
  int scratch_set = 0;  // the scratch set of the last route launched (see scratch_base)
  size_t stride = 0;
  unsigned char* d_scratch = nullptr;
  Result* d_results = nullptr;         // async entries
  Result* h_results = nullptr;         // mapped pinned host memory (synchronous entries)
  Result* d_results_mapped = nullptr;  // its device alias
  float* d_queries = nullptr;
  size_t dq_cap = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  std::mutex mu;
  ErrorSlot err;
  uint64_t routes = 0;
  unsigned long long* d_fallbacks = nullptr;  // counted by the exact kernel
  grm_b200::policy::Policy pol;               // lexical keys, filter codes, active flags
  const uint32_t* cur_allow = nullptr;        // filter bitmap of the route in progress
  cudaStream_t lex_stream = nullptr;          // single-query lexical pass beside the scan
  cudaEvent_t ev_fork = nullptr, ev_lex = nullptr;
  // multi-row entries: `nodes` counts rows, `entries` the routed entries
  bool multi = false;
  bool multi_bulk = false;             // stream the rows with the bulk-copy pass
  int64_t entries = 0;
  uint64_t* d_entry_off = nullptr;     // [entries + 1] row offsets
  uint32_t* d_entry_of_row = nullptr;  // [rows]
  int* d_entry_best = nullptr;         // [entries] ordered approximate maxima
  float* d_blk_s = nullptr;            // [entry_blocks * 32]
  uint32_t* d_blk_id = nullptr;
  float* d_thr = nullptr;
  double* d_qn = nullptr;              // the query's reference norm (entry refine)
  int* d_unsafe = nullptr;
  uint32_t* d_cand = nullptr;          // [entries]
  float* d_cand_s = nullptr;
  unsigned* d_cand_count = nullptr;
  int entry_blocks = 1;
  // INT4 bulk/refine mode (route_mla_int4), built by the bank's first INT4 route
  bool q4_ready = false;
  uint32_t* d_q4 = nullptr;      // biased nibbles, 64-row tiles [tiles][dim / 8][64]
  float* d_q4ns = nullptr;       // [nodes] norm scales
  uint32_t* d_q4key = nullptr;   // [nodes] ordered bulk keys of the route in progress
  uint32_t* d_q4cand = nullptr;  // [nodes] candidate rows
  uint2* d_q4bnd = nullptr;      // [nodes] boundary (key, row) pairs
  uint32_t* d_q4tie = nullptr;   // [nodes / 32] tie bitmap (kept zero between routes)
  float* d_q4slot_s = nullptr;   // [refine blocks * 32] per-block top entries
  uint32_t* d_q4slot_id = nullptr;
  int q4_slots = 0;              // refine blocks the slots hold
  grm_b200::mla::Q4Hdr* d_q4hdr = nullptr;
};

namespace {

bool fast_dim(int dim) { return dim == 64 || dim == 128 || dim == 256 || dim == 512; }

template <typename T>
using ScanFn = void (*)(const Params<T>);

bool bulk_ok(int dtype, int dim) {
  return (dtype == GRM_B200_F16 && (dim == 64 || dim == 128 || dim == 256)) ||
         (dtype == GRM_B200_F32 && (dim == 64 || dim == 128));
}

template <typename T>
ScanFn<T> scan_bulk_fn(int dim) {
  if constexpr (sizeof(T) == 2) {
    switch (dim) {
      case 64: return mla_scan_bulk_kernel<64, T>;
      case 128: return mla_scan_bulk_kernel<128, T>;
      case 256: return mla_scan_bulk_kernel<256, T>;
    }
  } else {
    switch (dim) {
      case 64: return mla_scan_bulk_kernel<64, T>;
      case 128: return mla_scan_bulk_kernel<128, T>;
    }
  }
  return nullptr;
}

template <typename T>
ScanFn<T> scan_fn(int dim) {
  switch (dim) {
    case 64: return mla_scan_kernel<64, T>;
    case 128: return mla_scan_kernel<128, T>;
    case 256: return mla_scan_kernel<256, T>;
    case 512: return mla_scan_kernel<512, T>;
  }
  return nullptr;
}

template <typename T>
ScanFn<T> scan_multi_fn(int dim) {
  switch (dim) {
    case 64: return mla_scan_kernel<64, T, false, true>;
    case 128: return mla_scan_kernel<128, T, false, true>;
    case 256: return mla_scan_kernel<256, T, false, true>;
    case 512: return mla_scan_kernel<512, T, false, true>;
  }
  return nullptr;
}

template <typename T>
ScanFn<T> scan_bulk_multi_fn(int dim) {
  if constexpr (sizeof(T) == 2) {
    switch (dim) {
      case 64: return mla_scan_bulk_kernel<64, T, true>;
      case 128: return mla_scan_bulk_kernel<128, T, true>;
      case 256: return mla_scan_bulk_kernel<256, T, true>;
    }
  } else {
    switch (dim) {
      case 64: return mla_scan_bulk_kernel<64, T, true>;
      case 128: return mla_scan_bulk_kernel<128, T, true>;
    }
  }
  return nullptr;
}

template <typename T>
ScanFn<T> exact_fn(int dim) {
  switch (dim) {
    case 64: return mla_exact_kernel<64, T>;
    case 128: return mla_exact_kernel<128, T>;
    case 256: return mla_exact_kernel<256, T>;
    case 512: return mla_exact_kernel<512, T>;
  }
  return mla_exact_kernel<0, T>;
}

int pick_grid(grm_b200_mla_bank* b) {
  DeviceInfo info;
  int rc = device_info(b->device, &info);
  if (rc) return rc;
  int occ = 1;
  cudaError_t e;
  b->bulk = !b->exact_only && bulk_ok(b->dtype, b->dim);
  if (b->bulk) {
    const void* fn = b->dtype == GRM_B200_F16 ? (const void*)scan_bulk_fn<__half>(b->dim)
                                              : (const void*)scan_bulk_fn<float>(b->dim);
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kBulkSmem);
    // The resolve kernel follows every scan: give both the same shared-memory
    // carveout so the SMs need no reconfiguration between them.
    const void* xfn = b->dtype == GRM_B200_F16 ? (const void*)exact_fn<__half>(b->dim)
                                               : (const void*)exact_fn<float>(b->dim);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(xfn, cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared);
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, kBulkWarps * 32, kBulkSmem);
  } else if (b->dtype == GRM_B200_F16) {
    auto fn = fast_dim(b->dim) ? scan_fn<__half>(b->dim) : exact_fn<__half>(b->dim);
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, kThreads, 0);
  } else {
    auto fn = fast_dim(b->dim) ? scan_fn<float>(b->dim) : exact_fn<float>(b->dim);
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, kThreads, 0);
  }
  if (e != cudaSuccess) return cuda_status(e);
  occ = std::max(1, occ);
  const int64_t groups = ceil_div64(b->nodes, 32);
  const int64_t want = ceil_div64(groups, b->bulk ? kBulkWarps : kWarps);
  b->grid_x = (int)std::max<int64_t>(1, std::min<int64_t>((int64_t)info.sms * occ, want));
  return 0;
}

int reserve(grm_b200_mla_bank* b, int queries) {
  if (queries <= b->scratch_queries) return 0;
  const int n = std::max(queries, 8);
  if (b->d_scratch) cudaFree(b->d_scratch);
  if (b->d_results) cudaFree(b->d_results);
  if (b->h_results) cudaFreeHost(b->h_results);
  b->d_scratch = nullptr;
  b->d_results = nullptr;
  b->h_results = nullptr;
  b->d_results_mapped = nullptr;
  b->scratch_queries = 0;
  b->stride = scratch_stride(b->grid_x);
  // two scratch sets (see scratch_base)
  cudaError_t e = cudaMalloc(&b->d_scratch, b->stride * n * 2);
  if (e == cudaSuccess) e = cudaMalloc(&b->d_results, sizeof(Result) * n);
  if (e == cudaSuccess)
    e = cudaHostAlloc(reinterpret_cast<void**>(&b->h_results), sizeof(Result) * n,
                      cudaHostAllocMapped);
  if (e == cudaSuccess)
    e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&b->d_results_mapped), b->h_results, 0);
  if (e != cudaSuccess) return b->err.set(cuda_status(e), "scratch allocation failed: %s", cudaGetErrorString(e));
  scratch_init_kernel<<<(2 * n + 127) / 128, 128, 0, b->stream>>>(b->d_scratch, b->stride, 2 * n);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
  if (e != cudaSuccess) return b->err.set(cuda_status(e), "scratch init failed: %s", cudaGetErrorString(e));
  b->scratch_queries = n;
  return 0;
}

// Two scratch sets of scratch_queries rows each.  A batched route takes the
// set the previous route did not use and touches its rows before its
// programmatic-launch wait (mla_batch_kernel, p.overlap); every other launch
// uses the current set and touches scratch only after its wait.  A set a
// batch takes was last used two routes back, whose merge completed before
// the previous route passed its own wait.
unsigned char* scratch_base(const grm_b200_mla_bank* b) {
  return b->d_scratch + (size_t)b->scratch_set * b->stride * (size_t)b->scratch_queries;
}

template <typename T>
Params<T> make_params(grm_b200_mla_bank* b, const float* dq, int topk) {
  Params<T> p;
  p.rows = static_cast<const T*>(b->d_rows);
  p.norms = b->d_norms;
  p.nodes = b->nodes;
  p.dim = b->dim;
  p.queries = dq;
  p.topk = topk;
  p.scratch = Scratch{scratch_base(b), b->stride, b->grid_x};
  p.results = b->d_results;
  p.out_ids = nullptr;
  p.out_scores = nullptr;
  p.id_offset = 0;
  p.force_all = b->exact_only ? 1 : 0;
  p.nq = 0;
  p.fallback_count = b->d_fallbacks;
  p.allow = b->cur_allow;
  p.entry_of_row = b->d_entry_of_row;
  p.entry_best = b->d_entry_best;
  p.multi_unsafe = b->d_unsafe;
  p.multi_qnorm = b->d_qn;
  p.wait_limit = scan_wait_limit();
  return p;
}

// pdl: launch as a programmatic dependent of the preceding kernel on `s` (the
// previous route's resolve kernel), so this launch overlaps its tail; the scan
// waits for it (griddepcontrol.wait) before reading anything.
template <typename T>
int launch_scan(grm_b200_mla_bank* b, const Params<T>& p, int nq, cudaStream_t s,
                bool pdl = false) {
  dim3 grid(b->grid_x, nq);
  if (b->bulk) {
    auto fn = scan_bulk_fn<T>(b->dim);
    if (!pdl) {
      fn<<<grid, kBulkWarps * 32, kBulkSmem, s>>>(p);
      return cuda_status(cudaGetLastError());
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kBulkWarps * 32);
    cfg.dynamicSmemBytes = kBulkSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, fn, p));
  }
  if (!b->exact_only) {
    scan_fn<T>(b->dim)<<<grid, kThreads, 0, s>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e);
  }
  return 0;
}

// pdl: launch as a programmatic dependent of the preceding scan on `s`, so the
// launch overlaps the scan's tail instead of following it.
template <typename T>
int launch_exact(grm_b200_mla_bank* b, const Params<T>& p0, int nq, cudaStream_t s,
                 bool pdl = false) {
  Params<T> p = p0;
  p.nq = nq;
  dim3 grid(b->grid_x, (unsigned)ceil_div64(nq, kExactQ));
  auto fn = exact_fn<T>(b->exact_only ? 0 : b->dim);
  if (!pdl || b->exact_only) {
    fn<<<grid, kThreads, 0, s>>>(p);
    return cuda_status(cudaGetLastError());
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, fn, p));
}

// ---- batched route (tensor cores) ---------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled from the driver, looked up once (no libcuda link).
EncodeTiledFn encode_tiled() {
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

template <int D>
int batch_smem_attr() {
  cudaError_t e = cudaFuncSetAttribute(mla_batch_kernel<D, 8>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       BLayout<D>::kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(mla_batch_kernel<D, kBList>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, BLayout<D>::kSmem);
  return cuda_status(e);
}

// Enables the batched route for fp16 banks of dim 64/128/256 whose rows all
// have norm >= kBMinNorm (or are non-finite); other banks batch by looping the
// single-query scan.
int setup_batch(grm_b200_mla_bank* b) {
  b->batch = false;
  if (b->dtype != GRM_B200_F16 || !(b->dim == 64 || b->dim == 128 || b->dim == 256) ||
      b->nodes >= ((int64_t)1 << 31) || (reinterpret_cast<uintptr_t>(b->d_rows) & 15) != 0)
    return 0;
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return 0;
  const cuuint64_t dims[2] = {(cuuint64_t)b->dim, (cuuint64_t)b->nodes};
  const cuuint64_t strides[1] = {(cuuint64_t)b->dim * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)kBM};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&b->tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, b->d_rows, dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return 0;
  int rc = b->dim == 64 ? batch_smem_attr<64>() : b->dim == 128 ? batch_smem_attr<128>()
                                                                 : batch_smem_attr<256>();
  if (rc) return b->err.set(rc, "batched route setup failed");
  cudaError_t e = cudaMalloc(&b->d_rnorms, sizeof(float) * (size_t)b->nodes);
  if (e == cudaSuccess) {
    const int grid = (int)std::min<int64_t>(ceil_div64(b->nodes, 256), 148 * 8);
    batch_rnorm_kernel<<<grid, 256, 0, b->stream>>>(b->d_norms, b->nodes, b->d_rnorms);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
  if (e != cudaSuccess) return b->err.set(cuda_status(e), "batched route setup failed");
  b->batch = true;
  return 0;
}

cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// Prep, scan and per-query merge of up to kBQ queries (p.queries / p.results /
// p.out_* / p.scratch already offset to the chunk).  Statuses other than kOk
// are resolved by the exact kernel launched after it.
template <int D>
int launch_batch_chunk(grm_b200_mla_bank* b, const Params<__half>& p, int nq, cudaStream_t s) {
  BatchParams bp;
  bp.tmap = b->tmap;
  bp.queries = p.queries;
  bp.overlap = 1;
  bp.rnorms = b->d_rnorms;
  bp.allow = p.allow;
  bp.nodes = b->nodes;
  bp.tiles = ceil_div64(b->nodes, kBM);
  bp.nq = nq;
  bp.topk = p.topk;
  bp.scratch = p.scratch;
  const int grid = (int)std::min<int64_t>(b->grid_x, bp.tiles);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(dim3(grid), dim3(kBThreads), BLayout<D>::kSmem, s, attr);
  cudaError_t e = p.topk <= 4 ? cudaLaunchKernelEx(&cfg, mla_batch_kernel<D, 8>, bp)
                  : cudaLaunchKernelEx(&cfg, mla_batch_kernel<D, kBList>, bp);
  if (e != cudaSuccess) return cuda_status(e);
  cfg = pdl_config(dim3(nq), dim3(kBMergeWarps * 32), 0, s, attr);
  e = cudaLaunchKernelEx(&cfg, mla_batch_merge_kernel<D>, p);
  return cuda_status(e);
}

// Switches the bank to the other scratch set and points p0 (the caller's
// params, which its resolve launch reuses) at it.
int launch_batch(grm_b200_mla_bank* b, Params<__half>& p0, int nq, cudaStream_t s) {
  b->scratch_set ^= 1;
  p0.scratch.base = scratch_base(b);
  for (int c0 = 0; c0 < nq; c0 += kBQ) {
    const int n = std::min(kBQ, nq - c0);
    Params<__half> p = p0;
    p.queries = p0.queries + (int64_t)c0 * b->dim;
    p.results = p0.results + c0;
    p.scratch.base = p0.scratch.base + p0.scratch.stride * (size_t)c0;
    if (p0.out_ids) p.out_ids = p0.out_ids + (int64_t)c0 * p0.topk;
    if (p0.out_scores) p.out_scores = p0.out_scores + (int64_t)c0 * p0.topk;
    const int rc = b->dim == 64    ? launch_batch_chunk<64>(b, p, n, s)
                   : b->dim == 128 ? launch_batch_chunk<128>(b, p, n, s)
                                   : launch_batch_chunk<256>(b, p, n, s);
    if (rc) return rc;
  }
  return 0;
}

// Route `nq` queries synchronously into b->h_results[0..nq).  The queries are
// device memory (dq), or one host query carried inline in the launch
// parameters (dq == nullptr, q_host != nullptr).  Results are written by the
// kernels straight into mapped pinned host memory (no copy-back call).
// `done` (optional) is recorded after the chunk's last launch, before the
// host waits, so the caller's elapsed time needs no second round trip.
template <typename T>
int run_chunk(grm_b200_mla_bank* b, const float* dq, const float* q_host, int nq, int topk,
              cudaEvent_t done);

// Multi-row bank, stream-ordered: per query the folding scan, the entry
// threshold and candidates, their exact scores and the top-k into
// results[q] (and the optional device outputs).
template <typename T>
int launch_multi(grm_b200_mla_bank* b, const float* dq, int nq, int topk, Result* results,
                 cudaStream_t s, uint64_t* out_ids = nullptr, float* out_scores = nullptr,
                 uint64_t id_offset = 0) {
  DeviceInfo info;
  if (device_info(b->device, &info) != 0) info.sms = 148;
  for (int q = 0; q < nq; ++q) {
    const float* qp = dq + (int64_t)q * b->dim;
    Params<T> p = make_params<T>(b, qp, topk);
    if (!b->exact_only) {
      if (b->multi_bulk)
        scan_bulk_multi_fn<T>(b->dim)<<<dim3(b->grid_x, 1), kBulkWarps * 32, kBulkSmem, s>>>(p);
      else
        scan_multi_fn<T>(b->dim)<<<dim3(b->grid_x, 1), kThreads, 0, s>>>(p);
      entry_top_kernel<<<b->entry_blocks, kEntryWarps * 32, 0, s>>>(b->d_entry_best, b->entries,
                                                                     topk, b->d_blk_s, b->d_blk_id);
      entry_threshold_kernel<<<1, kThrWarps * 32, 0, s>>>(b->d_blk_s, b->d_blk_id,
                                                          b->entry_blocks, topk, b->d_thr,
                                                          p.scratch.hdr(0));
    }
    const int cg = (int)std::max<int64_t>(1, std::min<int64_t>((int64_t)info.sms * 4,
                                                                ceil_div64(b->entries, 256)));
    entry_collect_kernel<<<cg, 256, 0, s>>>(b->d_entry_best, b->d_entry_off, b->entries, b->d_thr,
                                            b->d_unsafe, b->exact_only ? 1 : 0, b->d_cand,
                                            b->d_cand_count);
    if (b->dim <= RefineShape<T>::kMaxDim)
      entry_refine_kernel<T><<<info.sms * 2, kEntryWarps * 32, 0, s>>>(
          static_cast<const T*>(b->d_rows), b->d_norms, b->dim, qp, b->d_entry_off, b->d_cand,
          b->d_cand_count, b->cur_allow, b->d_cand_s, b->exact_only ? nullptr : b->d_qn);
    else
      entry_refine_wide_kernel<T><<<info.sms * 2, kEntryWarps * 32, 0, s>>>(
          static_cast<const T*>(b->d_rows), b->d_norms, b->dim, qp, b->d_entry_off, b->d_cand,
          b->d_cand_count, b->cur_allow, b->d_cand_s);
    entry_finalize_kernel<<<1, kEntryWarps * 32, 0, s>>>(
        b->d_cand, b->d_cand_s, b->d_cand_count, topk, id_offset, results + q,
        out_ids ? out_ids + (int64_t)q * topk : nullptr,
        out_scores ? out_scores + (int64_t)q * topk : nullptr, p.scratch.hdr(0));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e);
  }
  return 0;
}

template <typename T>
int run_chunk(grm_b200_mla_bank* b, const float* dq, const float* q_host, int nq, int topk,
              cudaEvent_t done) {
  if (b->multi) {
    int rc = launch_multi<T>(b, dq, nq, topk, b->d_results_mapped, b->stream);
    if (rc) return b->err.set(rc, "MLA multi-row route launch failed");
    if (done) cudaEventRecord(done, b->stream);
    cudaError_t e = cudaStreamSynchronize(b->stream);
    if (e != cudaSuccess) return b->err.set(cuda_status(e), "MLA multi-row route failed: %s", cudaGetErrorString(e));
    for (int i = 0; i < nq; ++i)
      if (((volatile Result*)b->h_results)[i].status == kError)
        return b->err.set(GRM_B200_KERNEL_BASE + 1,
                          "MLA scan: a bounded device wait gave up (query %d)", i);
    return 0;
  }
  Params<T> p = make_params<T>(b, dq, topk);
  p.results = b->d_results_mapped;
  if (!dq) std::memcpy(p.qinline, q_host, sizeof(float) * (size_t)b->dim);
  int rc;
  if constexpr (sizeof(T) == 2) {
    rc = (b->batch && dq && nq >= kBatchMin && topk <= kBMaxTopk)
             ? launch_batch(b, p, nq, b->stream)
             : launch_scan<T>(b, p, nq, b->stream);
  } else {
    rc = launch_scan<T>(b, p, nq, b->stream);
  }
  if (rc) return b->err.set(rc, "MLA scan launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  bool need_exact = b->exact_only;
  if (!b->exact_only) {
    if (done) cudaEventRecord(done, b->stream);
    cudaError_t e = cudaStreamSynchronize(b->stream);
    if (e != cudaSuccess) return b->err.set(cuda_status(e), "MLA route failed: %s", cudaGetErrorString(e));
    for (int i = 0; i < nq; ++i) {
      const int st = ((volatile Result*)b->h_results)[i].status;
      if (st == kError)
        return b->err.set(GRM_B200_KERNEL_BASE + 1,
                          "MLA scan: a bounded device wait gave up (query %d)", i);
      need_exact = need_exact || st != kOk;
    }
  }
  if (need_exact) {
    rc = launch_exact<T>(b, p, nq, b->stream);
    if (rc) return b->err.set(rc, "MLA exact pass launch failed");
    if (done) cudaEventRecord(done, b->stream);
    cudaError_t e = cudaStreamSynchronize(b->stream);
    if (e != cudaSuccess) return b->err.set(cuda_status(e), "MLA exact pass failed: %s", cudaGetErrorString(e));
  }
  return 0;
}

int route_device_queries(grm_b200_mla_bank* b, const float* dq, int query_count, int warmup,
                         int topk, uint64_t* out_ids, float* out_scores, float* elapsed,
                         const float* q_host = nullptr) {
  if ((!dq && !q_host) || !out_ids || query_count <= 0 || warmup < 0 || warmup >= query_count || topk <= 0 ||
      topk > GRM_B200_MAX_TOPK)
    return b->err.set(GRM_B200_EINVAL, "invalid MLA route arguments (queries=%d warmup=%d topk=%d)",
                      query_count, warmup, topk);
  cudaError_t e = cudaSetDevice(b->device);
  if (e != cudaSuccess) return b->err.set(cuda_status(e), "cudaSetDevice failed");
  int rc = reserve(b, query_count);
  if (rc) return rc;
  auto chunk = [&](int q0, int nq, cudaEvent_t done) -> int {
    const float* qd = dq ? dq + (int64_t)q0 * b->dim : nullptr;
    rc = (b->dtype == GRM_B200_F16) ? run_chunk<__half>(b, qd, q_host, nq, topk, done)
                                    : run_chunk<float>(b, qd, q_host, nq, topk, done);
    if (rc) return rc;
    for (int i = 0; i < nq; ++i) {
      const Result& r = b->h_results[i];
      for (int j = 0; j < topk; ++j) {
        out_ids[(int64_t)(q0 + i) * topk + j] = r.ids[j];
        if (out_scores) out_scores[(int64_t)(q0 + i) * topk + j] = r.scores[j];
      }
    }
    return 0;
  };
  if (warmup > 0 && (rc = chunk(0, warmup, nullptr))) return rc;
  cudaEventRecord(b->ev0, b->stream);
  if ((rc = chunk(warmup, query_count - warmup, b->ev1))) return rc;
  e = cudaEventSynchronize(b->ev1);  // recorded before the chunk's last wait: already done
  float ms = 0.0f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, b->ev0, b->ev1);
  if (e != cudaSuccess) return b->err.set(cuda_status(e), "MLA route timing failed");
  if (elapsed) *elapsed = ms;
  b->routes += (uint64_t)query_count;
  return 0;
}

// ---- INT4 bulk/refine mode ---------------------------------------------------

// The INT4 arena and the route buffers, built once per bank on its stream.
int int4_prepare(grm_b200_mla_bank* b) {
  if (b->q4_ready) return 0;
  if (b->multi)
    return b->err.set(GRM_B200_EINVAL, "the INT4 route mode takes banks of single-row entries");
  if (b->dim % 8 != 0)
    return b->err.set(GRM_B200_EINVAL, "the INT4 route mode needs dim %% 8 == 0 (dim %d)", b->dim);
  const int64_t n = b->nodes;
  const size_t words = (size_t)ceil_div64(n, kQ4Tile) * kQ4Tile * 4 * (size_t)q4_quads(b->dim);
  const size_t tie_words = (size_t)ceil_div64(n, 32);
  DeviceInfo dinfo;
  if (int drc = device_info(b->device, &dinfo)) return b->err.set(drc, "device query failed");
  b->q4_slots = dinfo.sms * 2;
  cudaError_t e = cudaMalloc(&b->d_q4, words * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMalloc(&b->d_q4slot_s, sizeof(float) * 32 * (size_t)b->q4_slots);
  if (e == cudaSuccess)
    e = cudaMalloc(&b->d_q4slot_id, sizeof(uint32_t) * 32 * (size_t)b->q4_slots);
  if (e == cudaSuccess) e = cudaMalloc(&b->d_q4ns, (size_t)n * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&b->d_q4key, (size_t)n * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMalloc(&b->d_q4cand, (size_t)n * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMalloc(&b->d_q4bnd, (size_t)n * sizeof(uint2));
  if (e == cudaSuccess) e = cudaMalloc(&b->d_q4tie, tie_words * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMalloc(&b->d_q4hdr, sizeof(Q4Hdr));
  if (e == cudaSuccess) e = cudaMemsetAsync(b->d_q4tie, 0, tie_words * sizeof(uint32_t), b->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(b->d_q4hdr, 0, sizeof(Q4Hdr), b->stream);
  if (e != cudaSuccess)
    return b->err.set(cuda_status(e), "INT4 arena allocation failed: %s", cudaGetErrorString(e));
  DeviceInfo info;
  int rc = device_info(b->device, &info);
  if (rc) return b->err.set(rc, "device query failed");
  const int grid = info.sms * 8;
  // the bulk kernel holds the query (quads x 128 B) beside its 16 KB histogram
  e = cudaFuncSetAttribute(int4_bulk_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)(sizeof(float) * 32 * q4_quads(4096)));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(int4_refine_kernel<__half>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(sizeof(double) * 4096) + kQ4StageMax);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(int4_refine_kernel<float>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(sizeof(double) * 4096) + kQ4StageMax);
  if (e != cudaSuccess)
    return b->err.set(cuda_status(e), "INT4 kernel set-up failed: %s", cudaGetErrorString(e));
  if (b->dtype == GRM_B200_F16)
    int4_arena_kernel<__half><<<grid, 256, 0, b->stream>>>(
        static_cast<const __half*>(b->d_rows), b->d_norms, n, b->dim, b->d_q4, b->d_q4ns);
  else
    int4_arena_kernel<float><<<grid, 256, 0, b->stream>>>(
        static_cast<const float*>(b->d_rows), b->d_norms, n, b->dim, b->d_q4, b->d_q4ns);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
  if (e != cudaSuccess)
    return b->err.set(cuda_status(e), "INT4 arena build failed: %s", cudaGetErrorString(e));
  b->q4_ready = true;
  return 0;
}

// Route queries dq[nq, dim] (device) in the INT4 mode on `s`: four kernels
// per query, each after the first a programmatic dependent of the one before
// (the first waits for whatever precedes it, including the previous query's
// refine, which resets the shared header).
template <typename T>
int int4_launch(grm_b200_mla_bank* b, const float* dq, int nq, int topk, int64_t refine_m,
                uint64_t id_offset, Result* results, uint64_t* out_ids, float* out_scores,
                cudaStream_t s) {
  DeviceInfo info;
  int rc = device_info(b->device, &info);
  if (rc) return rc;
  const int64_t n = b->nodes;
  const unsigned M = (unsigned)std::min<int64_t>(std::max<int64_t>(topk, refine_m), n);
  const int64_t tiles = ceil_div64(n, kQ4Tile);
  const int bulk_grid = (int)std::max<int64_t>(
      1, std::min<int64_t>((int64_t)info.sms * 6, ceil_div64(tiles, kQ4BulkWarps)));
  const int coll_grid = (int)std::max<int64_t>(
      1, std::min<int64_t>((int64_t)info.sms * 2, ceil_div64(n, kQ4Chunk)));
  const int ref_grid = (int)std::max<int64_t>(
      1, std::min<int64_t>((int64_t)b->q4_slots, ceil_div64(M, kQ4RefThreads)));
  // candidate rows staged in shared memory when 32 padded rows per warp fit
  const size_t row_vecs = (size_t)b->dim * (b->dtype == GRM_B200_F16 ? 2 : 4) / 16 + 1;
  const size_t stage_bytes = (size_t)(kQ4RefThreads / 32) * 32 * row_vecs * 16;
  // (staged by bulk copies: rows 16-byte aligned)
  const int stage =
      stage_bytes <= (size_t)kQ4StageMax && (reinterpret_cast<uintptr_t>(b->d_rows) & 15) == 0
          ? 1 : 0;
  const size_t ref_smem = (((size_t)8 * b->dim + 15) & ~(size_t)15) + (stage ? stage_bytes : 0);
  cudaLaunchAttribute attr[1];
  for (int q = 0; q < nq; ++q) {
    const float* qp = dq + (int64_t)q * b->dim;
    cudaLaunchConfig_t cfg = pdl_config(dim3(bulk_grid), dim3(kQ4BulkWarps * 32),
                                        sizeof(float) * 32 * (size_t)q4_quads(b->dim), s, attr);
    const uint4* q4 = reinterpret_cast<const uint4*>(b->d_q4);
    const float* ns = b->d_q4ns;
    const int qc = q4_quads(b->dim);
    cudaError_t e =
        qc == 8   ? cudaLaunchKernelEx(&cfg, int4_bulk_kernel<8>, q4, ns, n, b->dim, qp,
                                       b->d_q4key, b->d_q4hdr, M)
        : qc == 4 ? cudaLaunchKernelEx(&cfg, int4_bulk_kernel<4>, q4, ns, n, b->dim, qp,
                                       b->d_q4key, b->d_q4hdr, M)
        : qc == 2 ? cudaLaunchKernelEx(&cfg, int4_bulk_kernel<2>, q4, ns, n, b->dim, qp,
                                       b->d_q4key, b->d_q4hdr, M)
                  : cudaLaunchKernelEx(&cfg, int4_bulk_kernel<0>, q4, ns, n, b->dim, qp,
                                       b->d_q4key, b->d_q4hdr, M);
    if (e == cudaSuccess) {
      cfg = pdl_config(dim3(coll_grid), dim3(kQ4CollThreads), 0, s, attr);
      e = cudaLaunchKernelEx(&cfg, int4_collect_kernel, (const uint32_t*)b->d_q4key, n,
                             b->d_q4hdr, b->d_q4cand, b->d_q4bnd);
    }
    if (e == cudaSuccess) {
      cfg = pdl_config(dim3(1), dim3(kQ4SelThreads), 0, s, attr);
      e = cudaLaunchKernelEx(&cfg, int4_select_kernel, (const uint2*)b->d_q4bnd, n, M,
                             b->d_q4hdr, b->d_q4cand, b->d_q4tie);
    }
    if (e == cudaSuccess) {
      cfg = pdl_config(dim3(ref_grid), dim3(kQ4RefThreads), ref_smem, s, attr);
      e = cudaLaunchKernelEx(&cfg, int4_refine_kernel<T>, static_cast<const T*>(b->d_rows),
                             (const float*)b->d_norms, b->dim, qp, (const uint32_t*)b->d_q4cand,
                             b->d_q4hdr, b->d_q4slot_s, b->d_q4slot_id, topk, id_offset,
                             results ? results + q : nullptr,
                             out_ids ? out_ids + (int64_t)q * topk : nullptr,
                             out_scores ? out_scores + (int64_t)q * topk : nullptr, stage);
    }
    if (e != cudaSuccess) return cuda_status(e);
  }
  return 0;
}

int int4_launch_any(grm_b200_mla_bank* b, const float* dq, int nq, int topk, int64_t refine_m,
                    uint64_t id_offset, Result* results, uint64_t* out_ids, float* out_scores,
                    cudaStream_t s) {
  return b->dtype == GRM_B200_F16
             ? int4_launch<__half>(b, dq, nq, topk, refine_m, id_offset, results, out_ids,
                                   out_scores, s)
             : int4_launch<float>(b, dq, nq, topk, refine_m, id_offset, results, out_ids,
                                  out_scores, s);
}

int bank_finish_create(grm_b200_mla_bank* b) {
  cudaError_t e = cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreate(&b->ev0);
  if (e == cudaSuccess) e = cudaEventCreate(&b->ev1);
  if (e == cudaSuccess) e = cudaMalloc(&b->d_norms, sizeof(float) * (size_t)b->nodes);
  if (e == cudaSuccess) e = cudaMalloc(&b->d_fallbacks, sizeof(unsigned long long));
  if (e == cudaSuccess)
    e = cudaMemsetAsync(b->d_fallbacks, 0, sizeof(unsigned long long), b->stream);
  if (e != cudaSuccess) return cuda_status(e);
  unsigned* d_special = nullptr;  // [0] rows outside the fast path, [1] outside the batch path
  e = cudaMalloc(&d_special, 2 * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemsetAsync(d_special, 0, 2 * sizeof(unsigned), b->stream);
  if (e != cudaSuccess) return cuda_status(e);
  DeviceInfo info;
  int rc = device_info(b->device, &info);
  if (rc) return rc;
  const int grid = (int)std::min<int64_t>(ceil_div64(b->nodes, 256), (int64_t)info.sms * 8);
  if (b->dtype == GRM_B200_F16)
    row_norms_kernel<__half><<<grid, 256, 0, b->stream>>>(static_cast<const __half*>(b->d_rows),
                                                          b->nodes, b->dim, b->d_norms, d_special);
  else
    row_norms_kernel<float><<<grid, 256, 0, b->stream>>>(static_cast<const float*>(b->d_rows),
                                                         b->nodes, b->dim, b->d_norms, d_special);
  unsigned special[2] = {0, 0};
  e = cudaGetLastError();
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(special, d_special, 2 * sizeof(unsigned), cudaMemcpyDeviceToHost, b->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
  cudaFree(d_special);
  if (e != cudaSuccess) return cuda_status(e);
  b->exact_only = !fast_dim(b->dim) || special[0] > 0;
  rc = pick_grid(b);
  if (rc) return rc;
  if (!b->exact_only && special[1] == 0 && (rc = setup_batch(b))) return rc;
  return reserve(b, 8);
}

void bank_free(grm_b200_mla_bank* b) {
  if (!b) return;
  cudaSetDevice(b->device);
  if (b->stream) cudaStreamSynchronize(b->stream);
  if (b->d_rows) cudaFree(b->d_rows);
  if (b->d_norms) cudaFree(b->d_norms);
  if (b->d_fallbacks) cudaFree(b->d_fallbacks);
  if (b->d_rnorms) cudaFree(b->d_rnorms);
  if (b->d_scratch) cudaFree(b->d_scratch);
  if (b->d_results) cudaFree(b->d_results);
  if (b->h_results) cudaFreeHost(b->h_results);
  if (b->d_queries) cudaFree(b->d_queries);
  grm_b200::policy::policy_free(b->pol);
  if (b->lex_stream) cudaStreamSynchronize(b->lex_stream);
  void* mptrs[] = {b->d_entry_off, b->d_entry_of_row, b->d_entry_best, b->d_blk_s, b->d_blk_id,
                   b->d_thr, b->d_qn, b->d_unsafe, b->d_cand, b->d_cand_s, b->d_cand_count,
                   b->d_q4, b->d_q4ns, b->d_q4key, b->d_q4cand, b->d_q4bnd,
                   b->d_q4tie, b->d_q4slot_s, b->d_q4slot_id, b->d_q4hdr};
  for (void* m : mptrs)
    if (m) cudaFree(m);
  if (b->ev_fork) cudaEventDestroy(b->ev_fork);
  if (b->ev_lex) cudaEventDestroy(b->ev_lex);
  if (b->lex_stream) cudaStreamDestroy(b->lex_stream);
  if (b->ev0) cudaEventDestroy(b->ev0);
  if (b->ev1) cudaEventDestroy(b->ev1);
  if (b->stream) cudaStreamDestroy(b->stream);
  delete b;
}

int create_common(const void* rows, bool host, int dtype, int64_t nodes, int dim, int device,
                  grm_b200_mla_bank** out) {
  if (!out) {
    set_thread_error("out_bank is NULL");
    return GRM_B200_EINVAL;
  }
  *out = nullptr;
  if (!rows || nodes <= 0 || nodes >= (int64_t)0xFFFFFFFF || dim <= 0 || dim > 4096 ||
      !(dtype == GRM_B200_F16 || dtype == GRM_B200_F32)) {
    set_thread_error("invalid MLA bank arguments (nodes=%lld dim=%d dtype=%d)", (long long)nodes,
                     dim, dtype);
    return GRM_B200_EINVAL;
  }
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) {
    set_thread_error("cudaSetDevice(%d) failed: %s", device, cudaGetErrorString(e));
    return cuda_status(e);
  }
  auto* b = new grm_b200_mla_bank();
  b->device = device;
  b->dtype = dtype;
  b->nodes = nodes;
  b->dim = dim;
  const size_t bytes = (size_t)nodes * dim * (dtype == GRM_B200_F16 ? 2 : 4);
  e = cudaMalloc(&b->d_rows, bytes);
  if (e == cudaSuccess)
    e = cudaMemcpy(b->d_rows, rows, bytes, host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice);
  int rc = cuda_status(e);
  if (!rc) rc = bank_finish_create(b);
  if (rc) {
    set_thread_error("MLA bank create failed (%d): %s", rc, cudaGetErrorString(cudaGetLastError()));
    bank_free(b);
    return rc;
  }
  *out = b;
  return 0;
}

__global__ void fill_int_kernel(int* p, int64_t n, int v) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

// Turn a row bank into a bank of multi-row entries: entry e owns rows
// off[e] .. off[e+1]-1 (RouterIndex's entry_row_offsets, cpp/grm_runtime.cpp:3219-3260).
int make_multi(grm_b200_mla_bank* b, const uint64_t* off, int64_t entries) {
  b->multi = true;
  b->batch = false;
  b->bulk = false;
  b->entries = entries;
  DeviceInfo info;
  int rc = device_info(b->device, &info);
  if (rc) return rc;
  int occ = 1;
  cudaError_t e = cudaSuccess;
  b->multi_bulk = !b->exact_only && bulk_ok(b->dtype, b->dim);
  if (b->multi_bulk) {
    const void* fn = b->dtype == GRM_B200_F16 ? (const void*)scan_bulk_multi_fn<__half>(b->dim)
                                              : (const void*)scan_bulk_multi_fn<float>(b->dim);
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kBulkSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared);
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, kBulkWarps * 32, kBulkSmem);
    if (e != cudaSuccess) return cuda_status(e);
  } else if (!b->exact_only) {
    const void* fn = b->dtype == GRM_B200_F16 ? (const void*)scan_multi_fn<__half>(b->dim)
                                              : (const void*)scan_multi_fn<float>(b->dim);
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, kThreads, 0);
    if (e != cudaSuccess) return cuda_status(e);
  }
  b->grid_x = (int)std::max<int64_t>(
      1, std::min<int64_t>((int64_t)info.sms * std::max(occ, 1),
                           ceil_div64(ceil_div64(b->nodes, 32), b->multi_bulk ? kBulkWarps : kWarps)));
  b->entry_blocks = (int)std::max<int64_t>(
      1, std::min<int64_t>((int64_t)info.sms * 2, ceil_div64(entries, kEntryWarps * 32)));
  std::vector<uint32_t> eor((size_t)b->nodes);
  for (int64_t en = 0; en < entries; ++en)
    for (uint64_t r = off[en]; r < off[en + 1]; ++r) eor[(size_t)r] = (uint32_t)en;
  auto alloc = [&](void** ptr, size_t bytes) {
    if (e == cudaSuccess) e = cudaMalloc(ptr, std::max<size_t>(bytes, 16));
  };
  alloc((void**)&b->d_entry_off, sizeof(uint64_t) * (size_t)(entries + 1));
  alloc((void**)&b->d_entry_of_row, sizeof(uint32_t) * (size_t)b->nodes);
  alloc((void**)&b->d_entry_best, sizeof(int) * (size_t)entries);
  alloc((void**)&b->d_blk_s, sizeof(float) * 32 * (size_t)b->entry_blocks);
  alloc((void**)&b->d_blk_id, sizeof(uint32_t) * 32 * (size_t)b->entry_blocks);
  alloc((void**)&b->d_thr, sizeof(float));
  alloc((void**)&b->d_qn, sizeof(double));
  alloc((void**)&b->d_unsafe, sizeof(int) * 64);
  alloc((void**)&b->d_cand, sizeof(uint32_t) * (size_t)entries);
  alloc((void**)&b->d_cand_s, sizeof(float) * (size_t)entries);
  alloc((void**)&b->d_cand_count, sizeof(unsigned));
  if (e == cudaSuccess)
    e = cudaMemcpy(b->d_entry_off, off, sizeof(uint64_t) * (size_t)(entries + 1),
                   cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(b->d_entry_of_row, eor.data(), sizeof(uint32_t) * eor.size(),
                   cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(b->d_cand_count, 0, sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(b->d_unsafe, 0, sizeof(int) * 64);
  if (e == cudaSuccess) {
    fill_int_kernel<<<info.sms * 4, 256, 0, b->stream>>>(b->d_entry_best, entries, kOrderedNegInf);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
  return cuda_status(e);
}

}  // namespace

extern "C" {

int grm_b200_mla_bank_create_multi(const void* rows_host, int dtype, int64_t rows, int dim,
                                   const uint64_t* entry_row_offsets, int64_t entries, int device,
                                   grm_b200_mla_bank** out_bank) {
  if (!out_bank) return GRM_B200_EINVAL;
  *out_bank = nullptr;
  if (!entry_row_offsets || entries <= 0 || entries >= (int64_t)0xFFFFFFFF ||
      entry_row_offsets[0] != 0 || entry_row_offsets[entries] != (uint64_t)rows) {
    set_thread_error("invalid entry_row_offsets (entries=%lld rows=%lld)", (long long)entries,
                     (long long)rows);
    return GRM_B200_EINVAL;
  }
  for (int64_t i = 0; i < entries; ++i)
    if (entry_row_offsets[i + 1] < entry_row_offsets[i]) {
      set_thread_error("entry_row_offsets must be non-decreasing (entry %lld)", (long long)i);
      return GRM_B200_EINVAL;
    }
  grm_b200_mla_bank* b = nullptr;
  int rc = create_common(rows_host, true, dtype, rows, dim, device, &b);
  if (rc) return rc;
  if ((rc = make_multi(b, entry_row_offsets, entries))) {
    set_thread_error("MLA multi-row bank setup failed (%d)", rc);
    bank_free(b);
    return rc;
  }
  *out_bank = b;
  return 0;
}

int grm_b200_mla_bank_create(const void* rows_host, int dtype, int64_t nodes, int dim, int device,
                             grm_b200_mla_bank** out_bank) {
  return create_common(rows_host, true, dtype, nodes, dim, device, out_bank);
}

int grm_b200_mla_bank_create_device(const void* rows_device, int dtype, int64_t nodes, int dim,
                                    grm_b200_mla_bank** out_bank) {
  int device = 0;
  cudaGetDevice(&device);
  return create_common(rows_device, false, dtype, nodes, dim, device, out_bank);
}

int grm_b200_mla_route(grm_b200_mla_bank* bank, const float* queries_host, int query_count, int dim,
                       int warmup, int topk, uint64_t* out_ids_host, float* out_scores_host,
                       float* elapsed_ms) {
  if (!bank) return GRM_B200_EINVAL;
  std::lock_guard<std::mutex> lock(bank->mu);
  if (!queries_host || query_count <= 0 || dim != bank->dim)
    return bank->err.set(GRM_B200_EINVAL, "invalid MLA route arguments (dim=%d, bank dim=%d)", dim,
                         bank->dim);
  cudaError_t e = cudaSetDevice(bank->device);
  if (e == cudaSuccess && query_count == 1 && dim <= kInlineMax && !bank->multi)
    return route_device_queries(bank, nullptr, 1, warmup, topk, out_ids_host, out_scores_host,
                                elapsed_ms, queries_host);
  const size_t need = (size_t)query_count * dim;
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
    return bank->err.set(cuda_status(e), "MLA query upload failed: %s", cudaGetErrorString(e));
  return route_device_queries(bank, bank->d_queries, query_count, warmup, topk, out_ids_host,
                              out_scores_host, elapsed_ms);
}

int grm_b200_mla_route_device(grm_b200_mla_bank* bank, const float* queries_device, int query_count,
                              int dim, int warmup, int topk, uint64_t* out_ids_host,
                              float* out_scores_host, float* elapsed_ms) {
  if (!bank) return GRM_B200_EINVAL;
  std::lock_guard<std::mutex> lock(bank->mu);
  if (dim != bank->dim)
    return bank->err.set(GRM_B200_EINVAL, "query dim %d does not match bank dim %d", dim, bank->dim);
  return route_device_queries(bank, queries_device, query_count, warmup, topk, out_ids_host,
                              out_scores_host, elapsed_ms);
}

int grm_b200_mla_route_int4(grm_b200_mla_bank* bank, const float* queries_host, int query_count,
                            int dim, int topk, int64_t refine_m, uint64_t* out_ids_host,
                            float* out_scores_host, float* elapsed_ms) {
  if (!bank) return GRM_B200_EINVAL;
  std::lock_guard<std::mutex> lock(bank->mu);
  if (!queries_host || query_count <= 0 || dim != bank->dim || !out_ids_host || topk <= 0 ||
      topk > GRM_B200_MAX_TOPK || refine_m < 0)
    return bank->err.set(GRM_B200_EINVAL,
                         "invalid MLA INT4 route arguments (queries=%d dim=%d topk=%d refine_m=%lld)",
                         query_count, dim, topk, (long long)refine_m);
  cudaError_t e = cudaSetDevice(bank->device);
  if (e != cudaSuccess) return bank->err.set(cuda_status(e), "cudaSetDevice failed");
  int rc = int4_prepare(bank);
  if (rc) return rc;
  if ((rc = reserve(bank, query_count))) return rc;
  const size_t need = (size_t)query_count * dim;
  if (need > bank->dq_cap) {
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
    return bank->err.set(cuda_status(e), "MLA query upload failed: %s", cudaGetErrorString(e));
  cudaEventRecord(bank->ev0, bank->stream);
  rc = int4_launch_any(bank, bank->d_queries, query_count, topk, refine_m, 0,
                       bank->d_results_mapped, nullptr, nullptr, bank->stream);
  if (rc) return bank->err.set(rc, "MLA INT4 route launch failed");
  cudaEventRecord(bank->ev1, bank->stream);
  e = cudaStreamSynchronize(bank->stream);
  if (e != cudaSuccess)
    return bank->err.set(cuda_status(e), "MLA INT4 route failed: %s", cudaGetErrorString(e));
  for (int i = 0; i < query_count; ++i) {
    const Result& r = bank->h_results[i];
    for (int j = 0; j < topk; ++j) {
      out_ids_host[(int64_t)i * topk + j] = r.ids[j];
      if (out_scores_host) out_scores_host[(int64_t)i * topk + j] = r.scores[j];
    }
  }
  float ms = 0.0f;
  e = cudaEventElapsedTime(&ms, bank->ev0, bank->ev1);
  if (e != cudaSuccess) return bank->err.set(cuda_status(e), "MLA INT4 route timing failed");
  if (elapsed_ms) *elapsed_ms = ms;
  bank->routes += (uint64_t)query_count;
  return 0;
}

int grm_b200_mla_route_int4_async(grm_b200_mla_bank* bank, const float* queries_device,
                                  int query_count, int topk, int64_t refine_m, uint64_t id_offset,
                                  uint64_t* out_ids_device, float* out_scores_device,
                                  void* stream) {
  if (!bank) return GRM_B200_EINVAL;
  std::lock_guard<std::mutex> lock(bank->mu);
  if (!queries_device || query_count <= 0 || topk <= 0 || topk > GRM_B200_MAX_TOPK ||
      refine_m < 0 || (!out_ids_device && !out_scores_device))
    return bank->err.set(GRM_B200_EINVAL, "invalid MLA INT4 async route arguments");
  cudaError_t e = cudaSetDevice(bank->device);
  if (e != cudaSuccess) return bank->err.set(cuda_status(e), "cudaSetDevice failed");
  int rc = int4_prepare(bank);
  if (rc) return rc;
  rc = int4_launch_any(bank, queries_device, query_count, topk, refine_m, id_offset, nullptr,
                       out_ids_device, out_scores_device, static_cast<cudaStream_t>(stream));
  if (rc) return bank->err.set(rc, "MLA INT4 async route launch failed");
  return 0;
}

}  // extern "C"

namespace {

// phase: 1 = scan only, 2 = resolve only, 3 = both.
int route_async_phases(grm_b200_mla_bank* bank, const float* queries_device, int query_count,
                       int topk, uint64_t id_offset, uint64_t* out_ids_device,
                       float* out_scores_device, void* stream, int phase) {
  if (!bank) return GRM_B200_EINVAL;
  std::lock_guard<std::mutex> lock(bank->mu);
  if (!queries_device || query_count <= 0 || topk <= 0 || topk > GRM_B200_MAX_TOPK ||
      (!out_ids_device && !out_scores_device))
    return bank->err.set(GRM_B200_EINVAL, "invalid MLA async route arguments");
  if (query_count > bank->scratch_queries)
    return bank->err.set(GRM_B200_EINVAL,
                         "query_count %d exceeds reserved scratch (%d): call grm_b200_mla_reserve",
                         query_count, bank->scratch_queries);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = 0;
  if (bank->multi) {  // one stream-ordered pipeline: both phases at once
    if (phase & 1) {
      rc = (bank->dtype == GRM_B200_F16)
               ? launch_multi<__half>(bank, queries_device, query_count, topk, bank->d_results, s,
                                      out_ids_device, out_scores_device, id_offset)
               : launch_multi<float>(bank, queries_device, query_count, topk, bank->d_results, s,
                                     out_ids_device, out_scores_device, id_offset);
      if (rc) return bank->err.set(rc, "MLA multi-row async route launch failed");
      bank->routes += (uint64_t)query_count;
    }
    return 0;
  }
  if (bank->dtype == GRM_B200_F16) {
    Params<__half> p = make_params<__half>(bank, queries_device, topk);
    p.out_ids = out_ids_device;
    p.out_scores = out_scores_device;
    p.id_offset = id_offset;
    if (phase & 1)
      rc = (bank->batch && query_count >= kBatchMin && topk <= kBMaxTopk)
               ? launch_batch(bank, p, query_count, s)
               : launch_scan<__half>(bank, p, query_count, s, true);
    if (!rc && (phase & 2)) rc = launch_exact<__half>(bank, p, query_count, s, true);
  } else {
    Params<float> p = make_params<float>(bank, queries_device, topk);
    p.out_ids = out_ids_device;
    p.out_scores = out_scores_device;
    p.id_offset = id_offset;
    if (phase & 1) rc = launch_scan<float>(bank, p, query_count, s, true);
    if (!rc && (phase & 2)) rc = launch_exact<float>(bank, p, query_count, s, true);
  }
  if (rc) return bank->err.set(rc, "MLA async route launch failed");
  if (phase & 1) bank->routes += (uint64_t)query_count;
  return 0;
}

}  // namespace

extern "C" {

int grm_b200_mla_route_async(grm_b200_mla_bank* bank, const float* queries_device, int query_count,
                             int topk, uint64_t id_offset, uint64_t* out_ids_device,
                             float* out_scores_device, void* stream) {
  return route_async_phases(bank, queries_device, query_count, topk, id_offset, out_ids_device,
                            out_scores_device, stream, 3);
}

int grm_b200_mla_scan_async(grm_b200_mla_bank* bank, const float* queries_device, int query_count,
                            int topk, uint64_t id_offset, uint64_t* out_ids_device,
                            float* out_scores_device, void* stream) {
  return route_async_phases(bank, queries_device, query_count, topk, id_offset, out_ids_device,
                            out_scores_device, stream, 1);
}

int grm_b200_mla_resolve_async(grm_b200_mla_bank* bank, const float* queries_device,
                               int query_count, int topk, uint64_t id_offset,
                               uint64_t* out_ids_device, float* out_scores_device, void* stream) {
  return route_async_phases(bank, queries_device, query_count, topk, id_offset, out_ids_device,
                            out_scores_device, stream, 2);
}

int grm_b200_mla_reserve(grm_b200_mla_bank* bank, int max_queries) {
  if (!bank || max_queries <= 0) return GRM_B200_EINVAL;
  std::lock_guard<std::mutex> lock(bank->mu);
  cudaSetDevice(bank->device);
  return reserve(bank, max_queries);
}

int grm_b200_mla_bank_destroy(grm_b200_mla_bank* bank) {
  bank_free(bank);
  return 0;
}

const char* grm_b200_mla_last_error(grm_b200_mla_bank* bank) {
  return bank ? bank->err.text.c_str() : grm_b200_last_error();
}

const float* grm_b200_mla_row_norms_device(grm_b200_mla_bank* bank) {
  return bank ? bank->d_norms : nullptr;
}

int grm_b200_mla_bank_set_policy(grm_b200_mla_bank* bank, const char* const* lexical_keys,
                                 const char* const* kinds, const char* const* scopes,
                                 const char* const* durabilities,
                                 const char* const* mutabilities, const uint8_t* active) {
  if (!bank) return GRM_B200_EINVAL;
  std::lock_guard<std::mutex> lock(bank->mu);
  cudaError_t e = cudaSetDevice(bank->device);
  if (e != cudaSuccess) return bank->err.set(cuda_status(e), "cudaSetDevice failed");
  cudaStreamSynchronize(bank->stream);
  const char* const* cats[policy::kCats] = {kinds, scopes, durabilities, mutabilities};
  return policy::policy_set(bank->pol, bank->multi ? bank->entries : bank->nodes, lexical_keys,
                            cats, active, bank->err);
}

int grm_b200_mla_route_policy(grm_b200_mla_bank* bank, const float* queries_host, int query_count,
                              int dim, int topk, const char* const* lexical_keys,
                              const char* kind_filters, const char* scope_filters,
                              const char* durability_filters, const char* mutability_filters,
                              uint64_t* out_ids_host, float* out_scores_host, float* elapsed_ms) {
  if (!bank) return GRM_B200_EINVAL;
  std::lock_guard<std::mutex> lock(bank->mu);
  if (!queries_host || query_count <= 0 || dim != bank->dim || !out_ids_host || topk <= 0 ||
      topk > GRM_B200_MAX_TOPK)
    return bank->err.set(GRM_B200_EINVAL, "invalid MLA policy route arguments (queries=%d dim=%d topk=%d)",
                         query_count, dim, topk);
  bool any_lex = false;
  for (int i = 0; lexical_keys && i < query_count; ++i)
    any_lex = any_lex || !policy::split_keys(lexical_keys[i]).empty();
  if (any_lex && dim > kLexMaxDim)
    return bank->err.set(GRM_B200_EINVAL, "lexical keys on banks of dim > %d are not supported",
                         kLexMaxDim);
  cudaError_t e = cudaSetDevice(bank->device);
  if (e != cudaSuccess) return bank->err.set(cuda_status(e), "cudaSetDevice failed");
  int rc = reserve(bank, query_count);
  if (rc) return rc;
  if (!bank->pol.set) {  // every node keeps the reference's defaults: no keys, active
    const char* const* cats[policy::kCats] = {nullptr, nullptr, nullptr, nullptr};
    cudaStreamSynchronize(bank->stream);
    if ((rc = policy::policy_set(bank->pol, bank->multi ? bank->entries : bank->nodes, nullptr,
                                 cats, nullptr, bank->err)))
      return rc;
  }
  const size_t need = (size_t)query_count * dim;
  if (need > bank->dq_cap) {
    if (bank->d_queries) cudaFree(bank->d_queries);
    bank->d_queries = nullptr;
    bank->dq_cap = 0;
    e = cudaMalloc(&bank->d_queries, need * sizeof(float));
    if (e != cudaSuccess) return bank->err.set(cuda_status(e), "MLA query buffer allocation failed");
    bank->dq_cap = need;
  }
  e = cudaMemcpyAsync(bank->d_queries, queries_host, need * sizeof(float), cudaMemcpyHostToDevice,
                      bank->stream);
  if (e != cudaSuccess) return bank->err.set(cuda_status(e), "MLA query upload failed");
  DeviceInfo info;
  if (device_info(bank->device, &info) != 0) info.sms = 148;
  cudaEventRecord(bank->ev0, bank->stream);
  const char* const filters[policy::kCats] = {kind_filters, scope_filters, durability_filters,
                                              mutability_filters};
  const uint32_t* allow = nullptr;
  if ((rc = policy::policy_allow(bank->pol, filters, info.sms, bank->stream, &allow, bank->err)))
    return rc;
  // Stream-ordered from here to the final event: scan and exact pass chained
  // as in the async route (the exact kernel reads the statuses on the
  // device), the lexical kernels per query, one host wait at the end.  A
  // single query's lexical pass (postings, hit scores) does not depend on the
  // scan: it runs on a side stream launched first, and only the merge waits
  // for both.
  auto lex_pass = [&](int q, cudaStream_t st, int* m) -> int {
    uint64_t postings = 0;  // bounds the hit nodes: one warp each at most
    int r = policy::policy_collect(bank->pol, lexical_keys[q], info.sms, st, m, bank->err,
                                   &postings);
    if (r || *m == 0) return r;
    const float* dq = bank->d_queries + (int64_t)q * dim;
    const int grid = (int)std::max<uint64_t>(
        1, std::min<uint64_t>((uint64_t)info.sms * 2, (postings + kLexWarps - 1) / kLexWarps));
    if (bank->dtype == GRM_B200_F16)
      mla_lex_score_kernel<__half><<<grid, kLexWarps * 32, 0, st>>>(
          static_cast<const __half*>(bank->d_rows), bank->d_norms, dim, dq, bank->pol.d_hitlist,
          bank->pol.d_counter, allow, *m, bank->d_entry_off, bank->pol.d_cand_s,
          bank->pol.d_cand_id);
    else
      mla_lex_score_kernel<float><<<grid, kLexWarps * 32, 0, st>>>(
          static_cast<const float*>(bank->d_rows), bank->d_norms, dim, dq, bank->pol.d_hitlist,
          bank->pol.d_counter, allow, *m, bank->d_entry_off, bank->pol.d_cand_s,
          bank->pol.d_cand_id);
    cudaError_t le = cudaGetLastError();
    return le == cudaSuccess ? 0 : bank->err.set(cuda_status(le), "MLA lexical kernels launch failed");
  };
  auto merge = [&](int q, cudaStream_t st) -> int {
    Result* r = bank->d_results + q;
    policy::lex_merge_kernel<<<1, policy::kMergeWarps * 32, 0, st>>>(
        r->ids, r->scores, &r->count, topk, 0, bank->pol.d_cand_s, bank->pol.d_cand_id,
        bank->pol.d_counter);
    cudaError_t le = cudaGetLastError();
    return le == cudaSuccess ? 0 : bank->err.set(cuda_status(le), "MLA lexical merge launch failed");
  };
  int m0 = 0;
  const bool side = any_lex && query_count == 1;
  if (side) {
    if (!bank->lex_stream) {
      e = cudaStreamCreateWithFlags(&bank->lex_stream, cudaStreamNonBlocking);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&bank->ev_fork, cudaEventDisableTiming);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&bank->ev_lex, cudaEventDisableTiming);
      if (e != cudaSuccess) return bank->err.set(cuda_status(e), "lexical stream setup failed");
    }
    cudaEventRecord(bank->ev_fork, bank->stream);  // queries uploaded, allow built
    cudaStreamWaitEvent(bank->lex_stream, bank->ev_fork, 0);
    if ((rc = lex_pass(0, bank->lex_stream, &m0))) return rc;
    cudaEventRecord(bank->ev_lex, bank->lex_stream);
  }
  bank->cur_allow = allow;
  if (bank->multi) {
    rc = (bank->dtype == GRM_B200_F16)
             ? launch_multi<__half>(bank, bank->d_queries, query_count, topk, bank->d_results,
                                    bank->stream)
             : launch_multi<float>(bank, bank->d_queries, query_count, topk, bank->d_results,
                                   bank->stream);
  } else if (bank->dtype == GRM_B200_F16) {
    Params<__half> p = make_params<__half>(bank, bank->d_queries, topk);  // device results
    rc = (bank->batch && query_count >= kBatchMin && topk <= kBMaxTopk)
             ? launch_batch(bank, p, query_count, bank->stream)
             : launch_scan<__half>(bank, p, query_count, bank->stream, true);
    if (!rc) rc = launch_exact<__half>(bank, p, query_count, bank->stream, true);
  } else {
    Params<float> p = make_params<float>(bank, bank->d_queries, topk);
    rc = launch_scan<float>(bank, p, query_count, bank->stream, true);
    if (!rc) rc = launch_exact<float>(bank, p, query_count, bank->stream, true);
  }
  bank->cur_allow = nullptr;
  if (rc) return bank->err.set(rc, "MLA policy route launch failed");
  if (side) {
    cudaStreamWaitEvent(bank->stream, bank->ev_lex, 0);
    if (m0 && (rc = merge(0, bank->stream))) return rc;
  } else {
    for (int q = 0; any_lex && q < query_count; ++q) {
      int m = 0;
      if ((rc = lex_pass(q, bank->stream, &m))) return rc;
      if (m && (rc = merge(q, bank->stream))) return rc;
    }
  }
  e = cudaMemcpyAsync(bank->h_results, bank->d_results, sizeof(Result) * query_count,
                      cudaMemcpyDeviceToHost, bank->stream);
  if (e != cudaSuccess) return bank->err.set(cuda_status(e), "MLA policy result copy failed");
  cudaEventRecord(bank->ev1, bank->stream);
  e = cudaEventSynchronize(bank->ev1);
  float ms = 0.0f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, bank->ev0, bank->ev1);
  if (e != cudaSuccess) return bank->err.set(cuda_status(e), "MLA policy route failed: %s", cudaGetErrorString(e));
  for (int q = 0; q < query_count; ++q)
    if (((volatile Result*)bank->h_results)[q].status == kError)
      return bank->err.set(GRM_B200_KERNEL_BASE + 1,
                           "MLA scan: a bounded device wait gave up (query %d)", q);
  for (int q = 0; q < query_count; ++q) {
    const Result& r = bank->h_results[q];
    for (int j = 0; j < topk; ++j) {
      out_ids_host[(int64_t)q * topk + j] = r.ids[j];
      if (out_scores_host) out_scores_host[(int64_t)q * topk + j] = r.scores[j];
    }
  }
  if (elapsed_ms) *elapsed_ms = ms;
  bank->routes += (uint64_t)query_count;
  return 0;
}

int grm_b200_mla_paths(grm_b200_mla_bank* bank, int* flags) {
  if (!bank || !flags) return GRM_B200_EINVAL;
  *flags = (bank->bulk ? GRM_B200_PATH_BULK : 0) | (bank->batch ? GRM_B200_PATH_BATCH : 0) |
           (bank->exact_only ? GRM_B200_PATH_EXACT : 0);
  return 0;
}

int grm_b200_mla_stats(grm_b200_mla_bank* bank, uint64_t* routes, uint64_t* fallbacks) {
  if (!bank) return GRM_B200_EINVAL;
  std::lock_guard<std::mutex> lock(bank->mu);
  if (routes) *routes = bank->routes;
  if (fallbacks) {
    unsigned long long n = 0;
    cudaError_t e = cudaSetDevice(bank->device);
    if (e == cudaSuccess) e = cudaMemcpy(&n, bank->d_fallbacks, sizeof(n), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return bank->err.set(cuda_status(e), "MLA stats read failed");
    *fallbacks = n;
  }
  return 0;
}

}  // extern "C"

// ----------------------------------------------------------------------------
// Allocation-free route.
//
// Some callers cannot call cudaMalloc on the route path: a serving engine that
// reserves all of HBM for its KV cache and hands out memory only through its
// own pool, code that routes while a CUDA graph is being captured (cudaMalloc
// is not a capturable operation), or a latency-critical decode loop that must
// never hit the implicit device synchronisation of an allocation.  Such
// callers own their centroid rows and output buffers already; this entry point
// routes over them using only a fixed scratch array compiled into the library.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes (2 MiB).
// Every GPU that loads this library holds it until the process exits.  All
// calls on a device share it and it keeps the last call's contents, so each
// call first clears the per-query counters it relies on; calls whose kernels
// overlap on the GPU (different streams, or concurrent host threads) race on
// it and must be serialised by the caller.  Host code only ever passes the
// address returned by cudaGetSymbolAddress, fetched once per device on the
// first call made with that device current; that first call should therefore
// come before any stream capture.

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(2) << 20;
constexpr int kNoAllocMaxQueries = 16;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
unsigned char* g_noalloc_ptr[64] = {};
int g_noalloc_occ[64][4] = {};

int dim_slot(int dim) {
  switch (dim) {
    case 64: return 0;
    case 128: return 1;
    case 256: return 2;
    case 512: return 3;
  }
  return -1;
}

ScanFn<__half> scan_fn_inline(int dim) {
  switch (dim) {
    case 64: return mla_scan_kernel<64, __half, true>;
    case 128: return mla_scan_kernel<128, __half, true>;
    case 256: return mla_scan_kernel<256, __half, true>;
    case 512: return mla_scan_kernel<512, __half, true>;
  }
  return nullptr;
}

ScanFn<__half> exact_fn_inline(int dim) {
  switch (dim) {
    case 64: return mla_exact_kernel<64, __half, true>;
    case 128: return mla_exact_kernel<128, __half, true>;
    case 256: return mla_exact_kernel<256, __half, true>;
    case 512: return mla_exact_kernel<512, __half, true>;
  }
  return nullptr;
}

// Per-device set-up: the device address of the scratch array and the
// occupancy of the inline scan kernels.  Runs under g_noalloc_mu.
int noalloc_setup(int dev, int slot, unsigned char** base, int* occ) {
  if (dev < 0 || dev >= 64) return GRM_B200_EINVAL;
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) {
      set_thread_error("cudaGetSymbolAddress(scratch) failed on device %d: %s", dev,
                       cudaGetErrorString(e));
      return cuda_status(e);
    }
    g_noalloc_ptr[dev] = static_cast<unsigned char*>(ptr);
  }
  if (!g_noalloc_occ[dev][slot]) {
    int o = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &o, scan_fn_inline(64 << slot), kThreads, 0);
    if (e != cudaSuccess) {
      set_thread_error("occupancy query failed: %s", cudaGetErrorString(e));
      return cuda_status(e);
    }
    g_noalloc_occ[dev][slot] = std::max(1, o);
  }
  *base = g_noalloc_ptr[dev];
  *occ = g_noalloc_occ[dev][slot];
  return 0;
}

}  // namespace

extern "C" int grm_b200_mla_route_noalloc(const void* rows_device, int64_t nodes, int dim,
                                          const float* queries_device, int query_count, int topk,
                                          uint64_t* out_ids_device, float* out_scores_device,
                                          void* stream) {
  const int slot = dim_slot(dim);
  if (!rows_device || !queries_device || !out_ids_device || !out_scores_device || nodes <= 0 ||
      nodes >= (int64_t)0xFFFFFFFF || slot < 0 || topk <= 0 || topk > GRM_B200_MAX_TOPK ||
      query_count <= 0) {
    set_thread_error("invalid allocation-free MLA route arguments (nodes=%lld dim=%d topk=%d "
                     "queries=%d; dim must be 64, 128, 256 or 512)",
                     (long long)nodes, dim, topk, query_count);
    return GRM_B200_EINVAL;
  }
  if (query_count > kNoAllocMaxQueries) {
    set_thread_error("allocation-free MLA route takes at most %d queries per call (got %d)",
                     kNoAllocMaxQueries, query_count);
    return GRM_B200_EINVAL;
  }
  // The scans read rows with 16-byte vector loads, queries as floats, and
  // store whole uint64 / float result words: a misaligned view (an offset into
  // a caller's pool) is rejected here instead of faulting on the device.
  const uintptr_t rows_a = reinterpret_cast<uintptr_t>(rows_device);
  const uintptr_t q_a = reinterpret_cast<uintptr_t>(queries_device);
  if ((rows_a & 15) || (q_a & 3) || (reinterpret_cast<uintptr_t>(out_ids_device) & 7) ||
      (reinterpret_cast<uintptr_t>(out_scores_device) & 3)) {
    set_thread_error("allocation-free MLA route needs rows 16-byte, queries 4-byte, ids 8-byte "
                     "and scores 4-byte aligned device pointers (rows %% 16 = %d)",
                     (int)(rows_a & 15));
    return GRM_B200_EINVAL;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_thread_error("cudaGetDevice failed: %s", cudaGetErrorString(e));
    return cuda_status(e);
  }
  DeviceInfo info;
  int rc = device_info(dev, &info);
  if (rc) {
    set_thread_error("device query failed");
    return rc;
  }
  unsigned char* base = nullptr;
  int occ = 1;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    rc = noalloc_setup(dev, slot, &base, &occ);
  }
  if (rc) return rc;
  const int64_t groups = ceil_div64(nodes, 32);
  int grid_x = (int)std::max<int64_t>(
      1, std::min<int64_t>((int64_t)info.sms * occ, ceil_div64(groups, kWarps)));
  const size_t results_bytes = (sizeof(Result) * (size_t)query_count + 255) & ~(size_t)255;
  // The per-query scratch grows with the grid; shrink the grid until every
  // query's slice fits (the scan's block ranges and the exact pass accept any
  // grid width), so a full batch of queries always routes.
  while (grid_x > 1 &&
         results_bytes + scratch_stride(grid_x) * (size_t)query_count > kNoAllocScratchBytes)
    --grid_x;
  const size_t stride = scratch_stride(grid_x);
  const size_t need = results_bytes + stride * (size_t)query_count;
  if (need > kNoAllocScratchBytes) {
    set_thread_error("allocation-free MLA route needs %zu scratch bytes, the fixed array holds %zu",
                     need, kNoAllocScratchBytes);
    return GRM_B200_EINVAL;
  }
  Params<__half> p;
  p.rows = static_cast<const __half*>(rows_device);
  p.norms = nullptr;
  p.nodes = nodes;
  p.dim = dim;
  p.queries = queries_device;
  p.topk = topk;
  p.scratch = Scratch{base + results_bytes, stride, grid_x};
  p.results = reinterpret_cast<Result*>(base);
  p.out_ids = out_ids_device;
  p.out_scores = out_scores_device;
  p.id_offset = 0;
  p.force_all = 0;
  p.nq = query_count;
  p.fallback_count = nullptr;
  p.allow = nullptr;
  p.entry_of_row = nullptr;
  p.entry_best = nullptr;
  p.multi_unsafe = nullptr;
  p.multi_qnorm = nullptr;
  p.wait_limit = scan_wait_limit();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  scratch_init_kernel<<<(query_count + 127) / 128, 128, 0, s>>>(base + results_bytes, stride,
                                                                 query_count);
  dim3 grid(grid_x, query_count);
  scan_fn_inline(dim)<<<grid, kThreads, 0, s>>>(p);
  exact_fn_inline(dim)<<<dim3(grid_x, (unsigned)ceil_div64(query_count, kExactQ)), kThreads, 0,
                         s>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_thread_error("allocation-free MLA route launch failed: %s", cudaGetErrorString(e));
    return cuda_status(e);
  }
  return 0;
}
