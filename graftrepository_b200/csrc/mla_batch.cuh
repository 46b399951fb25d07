// mla_batch.cuh -- batched MLA route on the 5th-generation tensor cores.
//
// Included by mla_route.cu inside namespace grm_b200::mla.  A batch of up to
// kBQ queries reads the bank once: the approximate scores are the product
// Qs x bank^T, computed with tcgen05.mma (M = 128 query rows: the kBQ queries
// twice, N = 128 bank rows, K = 16 per instruction, fp16 operands, fp32
// accumulators in tensor memory), so a 64-query batch costs one pass over HBM
// instead of 64.  Queries on the M side put one query in each tensor-memory
// lane: an epilogue thread reads its query's scores for consecutive bank rows
// and filters them against its own threshold in registers.  The second copy
// of the queries fills tensor-memory lanes 64..127, so all four lane quarters
// -- and the warps of all four scheduler partitions -- share the epilogue.
//
// Operands.  The bank tile is loaded by TMA (2D tensor map, 128-byte swizzle,
// box 64 elements x 128 rows, one box per 128-byte K atom) into a ring of
// shared-memory stages (as many as fit).  The query matrix is built by every
// CTA in its own shared memory (build_query_image): q' = q / |q| (fp64 norm),
// scaled by 2^8 (no fp16 subnormals) and rounded to fp16, in the same K-major
// swizzled layout; no separate prep kernel stands between two batches.
//
// Roles (one CTA per SM, persistent over the 128-row tiles it claims):
//   warps 0..7         epilogue: warp w reads tensor-memory lanes 32*(w % 4)..
//                      (32 queries, one per thread) and one quarter (32) of
//                      the tile's 128 bank rows; each thread keeps its query's
//                      sorted top-16 in registers (inserts are per thread: no
//                      warp traffic).  Batches ask for top-k <= 16.
//   warp 8, one lane   TMA producer (bounded waits on the stage ring)
//   warp 9             tensor-memory allocation; one lane issues the MMAs
// Two 128-column accumulator buffers let the MMAs of tile i+1 run while the
// epilogue reads tile i.
//
// Error bound of the approximate score s~ = acc * 2^-8 / norm against the
// reference score s (|q'| = 1):
//   fp16 rounding of 256 q'_d: |sum_d c_d (q'_d - h_d)| <= 2^-11 sum |c_d q'_d|
//                               <= 2^-11 |c|;
//   products c_d h_d are exact in fp32 (11 x 11 significant bits); fp32
//   accumulation of <= 512 terms: <= 2^-14 |c| even with truncation;
//   fp16 bank subnormals, should the tensor core flush them: <= 16 * 2^-14 / |c|
//   relative, <= 2^-9 for rows with |c| >= 1/2 (banks with smaller rows are not
//   batched);
//   dropping the reference's 1e-8 / |q| term: <= 2^-16 for |q| >= 2^-8 (smaller
//   queries take the exact path).
// Total < 2^-8.5; kBMargin = 2^-8.  Candidates within 2 * kBMargin of the
// approximate k-th best are recomputed with the reference arithmetic by the
// per-query merge (final_merge); saturated lists flag the exact fallback.
#pragma once

#include <cuda.h>

namespace grm_b200 {
namespace mla {

constexpr int kBQ = 64;                    // queries per launch
constexpr int kBMq = 128;                  // MMA M: the kBQ queries, twice
constexpr int kBM = 128;                   // bank rows per tile (MMA N)
constexpr int kBSmemMax = 232448;          // dynamic shared memory a CTA may use (227 KB)
constexpr int kBCoResident = 32 * 1024;    // left free for other kernels' blocks
constexpr int kBEpi = 8;                   // epilogue warps 0..7
constexpr int kBThreads = 10 * 32;
constexpr int kBProducerWarp = 8;
constexpr int kBMmaWarp = 9;
constexpr int kBList = 16;                 // per-thread list capacity: top-k <= 16
constexpr int kBMaxTopk = kBList;
constexpr int kBMergeWarps = 12;           // warps of the per-query merge kernel
constexpr float kBMargin = 0.00390625f;    // 2^-8
constexpr float kBQScale = 256.0f;         // 2^8
constexpr float kBMinNorm = 0.5f;          // smallest bank row norm the batch path accepts
constexpr double kBSafeLo = 0.00390625;    // 2^-8: smaller query norms take the exact path
constexpr uint32_t kBTmemCols = 2 * kBM;   // two accumulator buffers
constexpr int kBSched = 4;                 // tile-id ring between the producer and the consumers
constexpr int kBTail = 4;                  // last rounds of tiles claimed, not assigned
constexpr int kBPub = 8;                   // entries a thread publishes per query at most

template <int D>
struct BLayout {
  static constexpr int KA = D / 64;                    // 128-byte swizzle atoms along K
  static constexpr int SA = KA >= 2 ? 2 : 1;           // atoms per stage
  static constexpr int SPT = KA / SA;                  // stages per tile
  static constexpr int kAtomT = kBM * 128;             // 16 KB: 128 bank rows x 64 halves
  static constexpr int kAtomQ = kBMq * 128;            // 16 KB: 128 query rows x 64 halves
  static constexpr int kStage = SA * kAtomT;
  static constexpr int kQ = KA * kAtomQ;
  // As many stages as fit beside the query image (1 KB alignment slack, 1 KB
  // for the static shared variables), leaving kBCoResident bytes so that the
  // previous batch's merge and resolve blocks fit on the SM beside this CTA
  // (the next batch starts while they run).  D = 256: 4 stages (2 tiles),
  // 128: 5 (5 tiles), 64: 11.
  static constexpr int kStages = (kBSmemMax - 2048 - kBCoResident - kQ) / kStage;
  static constexpr int kSmem = 1024 + kQ + kStages * kStage;  // + alignment slack
  static_assert(D % 64 == 0 && D <= 256, "batched dims: 64, 128, 256");
  static_assert(kStages >= 2 * SPT && kStages <= 16, "stage ring: two tiles at least");
};

struct BatchParams {
  CUtensorMap tmap;              // bank [nodes, D] fp16, box 64 x 128, 128-byte swizzle
  const float* queries;          // [nq, D] fp32 probes of this batch
  int overlap;                   // 1: the scratch rows are this launch's own (see the kernel)
  const float* rnorms;           // 2^-8 / row norm (NaN for non-finite rows)
  const uint32_t* allow;         // route filters: routable rows (nullptr: all)
  int64_t nodes;
  int64_t tiles;
  int nq;
  int topk;
  Scratch scratch;
};

// ---- PTX wrappers ------------------------------------------------------------

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] x B[smem]^T, both K-major fp16.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every MMA issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 consecutive fp32 columns of this warp's 32 tensor-memory lanes; the
// registers are valid after tmem_wait_ld().
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms
// 1024 bytes apart (stride byte offset 64 x 16 B), descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(const void* smem) {
  const uint32_t a = smem_u32(smem);
  return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)64 << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: fp32 accumulator, fp16 A and B, both K-major,
// M = kBMq query rows, N = kBM bank rows.
constexpr uint32_t kBIdesc =
    (1u << 4) | ((uint32_t)(kBM >> 3) << 17) | ((uint32_t)(kBMq >> 4) << 24);

// Byte offset of element (query row j, dim d) in the swizzled query image.
__host__ __device__ constexpr int qmat_offset(int j, int d) {
  return (d / 64) * (kBMq * 128) + j * 128 + ((((d % 64) / 8) ^ (j % 8)) * 16) + (d % 8) * 2;
}

// A thread's sorted top-C (score desc, id asc) in registers.  Inserting is
// an unrolled compare-and-shift (no dynamic indexing, no warp traffic).
template <int C>
struct LaneList {
  float s[C];
  uint32_t id[C];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int i = 0; i < C; ++i) {
      s[i] = -INFINITY;
      id[i] = kNoRow;
    }
  }
  // Insert (cs, cid) when it beats the last entry.
  __device__ __forceinline__ void insert(float cs, uint32_t cid) {
    if (!better(cs, cid, s[C - 1], id[C - 1])) return;
#pragma unroll
    for (int i = C - 1; i >= 1; --i) {
      if (better(cs, cid, s[i - 1], id[i - 1])) {
        s[i] = s[i - 1];
        id[i] = id[i - 1];
      } else if (better(cs, cid, s[i], id[i])) {
        s[i] = cs;
        id[i] = cid;
      }
    }
    if (better(cs, cid, s[0], id[0])) {
      s[0] = cs;
      id[0] = cid;
    }
  }
  // Score of entry k-1 (runtime 1 <= k <= C): the list is sorted, so it is
  // the minimum of the first k scores -- a tree reduction, which keeps the
  // list in registers (an indexed read would move it to local memory).
  __device__ __forceinline__ float kth(int k) const {
    float t[C / 2];
#pragma unroll
    for (int i = 0; i < C / 2; ++i)
      t[i] = fminf(2 * i < k ? s[2 * i] : INFINITY, 2 * i + 1 < k ? s[2 * i + 1] : INFINITY);
#pragma unroll
    for (int w = C / 4; w >= 1; w >>= 1)
#pragma unroll
      for (int i = 0; i < w; ++i) t[i] = fminf(t[i], t[i + w]);
    return t[0];
  }
};

// v[c] for a runtime c in [0, 32), by a 5-level select tree over its bits.
__device__ __forceinline__ float pick32(const float (&v)[32], int c) {
  float t[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) t[i] = (c & 1) ? v[2 * i + 1] : v[2 * i];
#pragma unroll
  for (int lvl = 1, w = 8; w >= 1; ++lvl, w >>= 1)
#pragma unroll
    for (int i = 0; i < w; ++i) t[i] = ((c >> lvl) & 1) ? t[2 * i + 1] : t[2 * i];
  return t[0];
}

// ---- kernels -----------------------------------------------------------------

// The batch's query image in this CTA's shared memory, in the swizzled
// K-major layout of the MMA's A operand, the queries at rows j and kBQ + j:
// q' = q / |q| (fp64 sum of squares, lane-strided then a butterfly, so every
// CTA builds the same bits), scaled by 2^8 (no fp16 subnormals) and rounded to
// fp16.  Rows of queries outside the safe range, and rows past the batch, are
// zero.  Builder warp w of nw takes queries w, w + nw, ...; the loads of
// kGroup of them are issued together, so the build costs about one memory
// latency instead of one per query (the stage ring covers only a few
// microseconds of streaming).  qsafe[j] records whether query j is inside the
// batched path's safe range.
template <int D>
__device__ __forceinline__ void build_query_image(const float* queries, int nq, unsigned char* img,
                                                  int* qsafe, int w, int nw, int lane) {
  constexpr int kPer = D / 32;
  constexpr int kGroup = kPer >= 8 ? 4 : 8;  // at most 32 values a lane in flight
  for (int j0 = w; j0 < kBQ; j0 += nw * kGroup) {
    float v[kGroup][kPer];
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
      const int j = j0 + g * nw;
#pragma unroll
      for (int i = 0; i < kPer; ++i)
        v[g][i] = j < nq ? __ldg(queries + (int64_t)j * D + lane + 32 * i) : 0.0f;
    }
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
      const int j = j0 + g * nw;
      if (j >= kBQ) break;
      bool safe = false;
      float inv = 0.0f;
      if (j < nq) {
        double acc = 0.0;
#pragma unroll
        for (int i = 0; i < kPer; ++i) acc = fma((double)v[g][i], (double)v[g][i], acc);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(kFull, acc, o);
        const double qn = sqrt(acc);
        safe = isfinite(qn) && qn >= kBSafeLo && qn < kSafeHi;
        inv = safe ? (float)(1.0 / qn) : 0.0f;
      }
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int d = lane + 32 * i;
        const __half h = __float2half_rn(safe ? v[g][i] * inv * kBQScale : 0.0f);
        *reinterpret_cast<__half*>(img + qmat_offset(j, d)) = h;
        *reinterpret_cast<__half*>(img + qmat_offset(kBQ + j, d)) = h;  // second copy
      }
      if (lane == 0) qsafe[j] = safe ? 1 : 0;
    }
  }
}

// 2^-8 / row norm for the batch epilogue (NaN for non-finite rows).
__global__ void batch_rnorm_kernel(const float* norms, int64_t n, float* rnorms) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float nrm = norms[i];
    rnorms[i] = isfinite(nrm) ? (1.0f / nrm) * (1.0f / kBQScale) : __int_as_float(0x7FC00000);
  }
}

// C: per-thread list capacity (>= top-k; 8 serves top-k <= 4 with a quarter
// of the insert cost of 16).
template <int D, int C>
__global__ void __launch_bounds__(kBThreads, 1)
    mla_batch_kernel(const __grid_constant__ BatchParams p) {
  using LY = BLayout<D>;
  extern __shared__ unsigned char bsm_raw[];
  unsigned char* const sm = bsm_raw + ((1024u - (smem_u32(bsm_raw) & 1023u)) & 1023u);
  unsigned char* const smQ = sm;
  unsigned char* const smT = sm + LY::kQ;
  __shared__ __align__(8) uint64_t full[LY::kStages], empty[LY::kStages], tfull[2], tempty[2], bq_bar,
      mma_done, sfull[kBSched], sempty[kBSched];
  __shared__ int sh_tile[kBSched];
  __shared__ uint32_t sh_tmem;
  __shared__ int sh_fail;
  __shared__ unsigned sh_issued, sh_consumed;
  __shared__ int sh_qsafe[kBQ];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Tiles: the CTA's first n_static tiles are its own (b, b + grid, ...);
  // the last kBTail rounds and the remainder (from dyn0 on) are claimed: the
  // producer takes the next one from the launch's counter (the chunk's first
  // query header, next; the per-query merge of that query resets it once the
  // scan has completed) as it needs one and passes its index (-1: none left)
  // to the MMA issuer and the epilogue warps through the sh_tile ring.  A CTA
  // that streams slowly or started late takes fewer of them, and the CTAs end
  // their streams together.
  Header* const sched = p.scratch.hdr(0);
  const int64_t rounds = p.tiles / gridDim.x;
  const int64_t n_static = rounds > kBTail ? rounds - kBTail : 0;
  const int64_t dyn0 = n_static * gridDim.x;
  // epilogue warps 0..7: tensor-memory lane quarter lq holds queries
  // 32*(lq & 1) + lane (quarters 2, 3: the second copy); the warp takes the
  // tile's bank rows 32*cq .. 32*cq + 31
  static_assert(C == 8 || C == kBList, "list capacity");
  const bool epi = warp < kBEpi;
  const int lq = warp & 3;
  const int cq = (warp >> 2) * 2 + (lq >> 1);
  const int qi = (lq & 1) * 32 + lane;  // this thread's query

  // Programmatic dependent launch: nothing before this grid's wait reads
  // memory the preceding kernel writes.  The bank and its norms are written
  // only at attach; the queries are the caller's input (none of this
  // library's kernels that let their dependents start early writes them), so
  // the producer streams the bank and the other warps build the query image
  // at once.  The scratch rows are read before the wait only when this
  // launch owns them (p.overlap: consecutive batches alternate between two
  // scratch sets, and the set was released by a merge that completed before
  // the previous batch passed its own wait); otherwise the epilogue waits
  // first.  Every thread waits before the publish, so this grid completes
  // after its predecessor.
  if (threadIdx.x == 0) {
    for (int s = 0; s < LY::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&tfull[0], 1);
    mbar_init(&tfull[1], 1);
    mbar_init(&tempty[0], kBEpi);
    mbar_init(&tempty[1], kBEpi);
    mbar_init(&bq_bar, kBEpi + 1);  // the image builders: warps 0..7 and the MMA warp
    mbar_init(&mma_done, 1);
    for (int s = 0; s < kBSched; ++s) {
      mbar_init(&sfull[s], 1);
      mbar_init(&sempty[s], kBEpi + 1);  // the MMA issuer and the 8 epilogue warps
    }
    sh_fail = 0;
    sh_issued = 0;
    sh_consumed = 0;
    mbar_fence_init();
  }
  if (warp == kBMmaWarp) {
    tmem_alloc(&sh_tmem, kBTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh_tmem;
  if (warp != kBProducerWarp) {
    build_query_image<D>(p.queries, p.nq, smQ, sh_qsafe, warp < kBEpi ? warp : kBEpi, kBEpi + 1,
                         lane);
    fence_proxy_async_smem();  // generic-proxy writes, read by the tensor cores
    __syncwarp();
    if (lane == 0) mbar_arrive(&bq_bar);
    if (epi && !p.overlap) asm volatile("griddepcontrol.wait;" ::: "memory");
  }

  if (warp == kBProducerWarp) {
    if (lane == 0) {  // TMA producer
      const uint64_t pol = l2_evict_first_policy();
      int st = 0;
      unsigned ph = 0, issued = 0;
      bool ok = true;
      // each claim is made one tile ahead, so its round trip to L2 overlaps
      // the waits for the stages of the tile before
      auto claim = [&]() { return atomicAdd(&sched->next, 1u); };
      unsigned c_next = n_static == 0 ? claim() : 0u;
      for (int64_t i = 0; ok; ++i) {
        int64_t t;
        if (i < n_static) {
          t = blockIdx.x + i * (int64_t)gridDim.x;
          if (i + 1 == n_static) c_next = claim();
        } else {
          const int64_t j = i - n_static;
          const int slot = (int)(j % kBSched);
          if (!mbar_wait(&sempty[slot], ((unsigned)(j / kBSched) & 1u) ^ 1u, kWaitLimit)) {
            ok = false;
            break;
          }
          t = dyn0 + c_next;
          const bool last = t >= p.tiles;
          sh_tile[slot] = last ? -1 : (int)t;
          mbar_arrive(&sfull[slot]);  // releases sh_tile[slot]
          if (last) break;
          c_next = claim();
        }
        const int y = (int)t * kBM;
        for (int sp = 0; sp < LY::SPT; ++sp) {
          if (!mbar_wait(&empty[st], ph ^ 1u, kWaitLimit)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[st], LY::kStage);
#pragma unroll
          for (int a = 0; a < LY::SA; ++a)
            tma_load_2d(smT + st * LY::kStage + a * LY::kAtomT, &p.tmap, (sp * LY::SA + a) * 64,
                        y, &full[st], pol);
          ++issued;
          if (++st == LY::kStages) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
      sh_issued = issued;
      if (!ok) atomicOr(&sh_fail, 1);
    }
  } else if (warp == kBMmaWarp) {
    if (lane == 0) {  // MMA issuer: D[query][row] = Q x T^T
      bool ok = mbar_wait(&bq_bar, 0, kWaitLimit);
      int st = 0;
      unsigned ph = 0, consumed = 0;
      for (int64_t i = 0; ok; ++i) {
        if (i >= n_static) {  // a claimed tile, or none left
          const int64_t j = i - n_static;
          const int slot = (int)(j % kBSched);
          if (!mbar_wait(&sfull[slot], (unsigned)(j / kBSched) & 1u, kWaitLimit)) {
            ok = false;
            break;
          }
          const int tile = sh_tile[slot];
          mbar_arrive(&sempty[slot]);
          if (tile < 0) break;
        }
        const int b = (int)(i & 1);
        const unsigned u = (unsigned)(i >> 1);
        if (!mbar_wait(&tempty[b], (u & 1u) ^ 1u, kWaitLimit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * kBM);
        for (int sp = 0; sp < LY::SPT; ++sp) {
          if (!mbar_wait(&full[st], ph, kWaitLimit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          ++consumed;
#pragma unroll
          for (int a = 0; a < LY::SA; ++a)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t qd = sw128_desc(smQ + (sp * LY::SA + a) * LY::kAtomQ + kk * 32);
              const uint64_t td = sw128_desc(smT + st * LY::kStage + a * LY::kAtomT + kk * 32);
              umma_f16(d, qd, td, kBIdesc, (sp | a | kk) != 0 ? 1u : 0u);
            }
          umma_commit(&empty[st]);  // the stage is free once these MMAs completed
          if (++st == LY::kStages) {
            st = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[b]);
      }
      // every MMA this thread issued completes before the teardown
      umma_commit(&mma_done);
      if (!mbar_wait(&mma_done, 0, kWaitLimit)) ok = false;
      sh_consumed = consumed;
      if (!ok) atomicOr(&sh_fail, 1);
    }
  } else if (epi) {
    LaneList<C> L;
    L.init();
    bool done_all = true;
    const float m2 = 2.0f * kBMargin;
    const bool active = qi < p.nq;
    // max(last entry, entry k-1 - 2*margin): rows below never enter
    float thr = active ? -INFINITY : INFINITY;
    // 2^-8 / norm of the warp's 32 rows of a tile, lane l holding row l (NaN
    // past the bank and for rows a route filter excludes: their scores never
    // reach a threshold), loaded one tile ahead.
    auto load_rn = [&](int tile) -> float {
      const int64_t r = (int64_t)tile * kBM + cq * 32 + lane;
      return (tile >= 0 && r < p.nodes && policy::row_allowed(p.allow, r))
                 ? __ldg(p.rnorms + r)
                 : __int_as_float(0x7FC00000);
    };
    // the CTA's i-th tile index (-1: none left), from the producer's ring;
    // false if the wait gave up
    auto next_tile = [&](int64_t i, int& tile) -> bool {
      if (i < n_static) {
        tile = (int)(blockIdx.x + i * (int64_t)gridDim.x);
        return true;
      }
      const int64_t j = i - n_static;
      const int slot = (int)(j % kBSched);
      if (!mbar_wait(&sfull[slot], (unsigned)(j / kBSched) & 1u, kWaitLimit)) return false;
      tile = sh_tile[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty[slot]);
      return true;
    };
    int tile = -1;
    if (!next_tile(0, tile)) {
      if (lane == 0) atomicOr(&sh_fail, 1);
      done_all = false;
    }
    float rn = load_rn(tile);
    // The query's header slot lb collects every CTA's k-th approximate score
    // (a lower bound of the final k-th best); it is read one tile ahead.
    int* const lbq = &p.scratch.hdr(active ? qi : 0)->lb;
    float kpub = -INFINITY;
    for (int64_t i = 0; tile >= 0; ++i) {
      const int b = (int)(i & 1);
      const unsigned u = (unsigned)(i >> 1);
      const int64_t row0 = (int64_t)tile * kBM + cq * 32;
      int tile_next = -1;
      if (!next_tile(i + 1, tile_next)) {
        if (lane == 0) atomicOr(&sh_fail, 1);
        done_all = false;
        break;
      }
      const float rn_next = load_rn(tile_next);
      const int lb_next = active ? __ldcg(lbq) : kOrderedNegInf;
      if (!mbar_wait(&tfull[b], u & 1u, kWaitLimit)) {
        if (lane == 0) atomicOr(&sh_fail, 1);
        done_all = false;
        break;
      }
      tc_fence_after();
      uint32_t v[32];
      tmem_ld32_nowait(tmem + ((uint32_t)(lq * 32) << 16) + (uint32_t)(b * kBM + cq * 32), v);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
      // hot path: scores and a bit per row that reaches the threshold (the
      // shuffles run in every lane; lanes past the batch have thr = +inf)
      float sc[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) sc[c] = __uint_as_float(v[c]) * __shfl_sync(kFull, rn, c);
      if (i == 0 && active) {
        // The first tile finds an empty list: start the threshold at the k-th
        // largest distinct score of this tile (k rows score at least that, so
        // the k-th best is no lower), minus the margin, instead of letting
        // every row through the insert path.
        float vk = INFINITY;
        for (int j = 0; j < p.topk; ++j) {
          float mx = -INFINITY;
#pragma unroll
          for (int c = 0; c < 32; ++c) mx = sc[c] < vk ? fmaxf(mx, sc[c]) : mx;
          vk = mx;
        }
        if (vk > -INFINITY) thr = fmaxf(thr, vk - m2);
      }
      uint32_t mask = 0;
#pragma unroll
      for (int c = 0; c < 32; ++c) mask |= (sc[c] >= thr ? 1u : 0u) << c;
      // rare path, rolled so the insert is inlined once
#pragma unroll 1
      while (mask) {
        const int c = __ffs(mask) - 1;
        mask &= mask - 1;
        const float x = pick32(sc, c);
        if (x >= thr) {
          L.insert(x, (uint32_t)(row0 + c));
          const float kt = L.kth(p.topk);
          thr = fmaxf(thr, fmaxf(L.s[C - 1], kt - m2));
          if (kt > kpub) {  // share this query's k-th score with every CTA
            kpub = kt;
            atomicMax(lbq, float_to_ordered(kt));
          }
        }
      }
      // every CTA's k-th score for this query bounds its final k-th from below
      if (lb_next != kOrderedNegInf) thr = fmaxf(thr, ordered_to_float(lb_next) - m2);
      rn = rn_next;
      tile = tile_next;
    }
    // Publish this thread's list.  hdr->lb holds the best k-th score any
    // thread has reached (each raised it to its own k-th while streaming): a
    // lower bound of the final approximate k-th best, so entries below it
    // minus 2 margins cannot reach the final top-k, and the rest (a prefix of
    // the sorted list, at most kBPub) are appended.  A full list may have
    // dropped rows below its last entry, and the cap drops the entries past
    // kBPub: the largest such score goes to hdr->floor, which flags the exact
    // fallback when it reaches the final threshold.
    if (done_all && active) {
      Header* const hdr = p.scratch.hdr(qi);
      const int lbs = __ldcg(&hdr->lb);
      const float wthr = lbs == kOrderedNegInf ? -INFINITY : ordered_to_float(lbs) - m2;
      int c = 0;
#pragma unroll
      for (int j = 0; j < C; ++j) c += (L.s[j] > -INFINITY && L.s[j] >= wthr) ? 1 : 0;
      float floor = L.s[C - 1];
      if constexpr (C > kBPub) {
        if (c > kBPub) {
          floor = fmaxf(floor, L.s[kBPub]);
          c = kBPub;
        }
      }
      if (floor > -INFINITY) atomicMax(&hdr->floor, float_to_ordered(floor));
      if (c > 0) {
        Entry* const out = p.scratch.entries(qi) + atomicAdd(&hdr->nent, (unsigned)c);
#pragma unroll
        for (int j = 0; j < (C < kBPub ? C : kBPub); ++j)
          if (j < c) out[j] = Entry{L.s[j], L.id[j]};
      }
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");  // every thread, before completing
  __syncwarp();
  __syncthreads();
  if (blockIdx.x == 0)  // the merge kernel reads the safe flags
    for (int j = threadIdx.x; j < p.nq; j += blockDim.x) p.scratch.hdr(j)->qsafe = sh_qsafe[j];
  if (sh_fail)  // the merge reports the batch's queries as failed
    for (int j = threadIdx.x; j < p.nq; j += blockDim.x) atomicOr(&p.scratch.hdr(j)->err, 1);

  // Teardown: every bulk load issued has landed, every MMA has completed.
  if (warp == kBProducerWarp && lane == 0 && sh_fail) {
    for (unsigned k = sh_consumed; k < sh_issued; ++k)
      mbar_wait(&full[k % LY::kStages], (k / LY::kStages) & 1u, kWaitLimit);
  }
  __syncthreads();
  if (warp == kBMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kBTmemCols);
  }
  asm volatile("griddepcontrol.launch_dependents;");
}

// One block per query of the batch: the final merge and exact refine of
// final_merge, with the batch margin.  Launched as a programmatic dependent of
// mla_batch_kernel.
template <int D>
__global__ void __launch_bounds__(kBMergeWarps * 32)
    mla_batch_merge_kernel(const __grid_constant__ Params<__half> p) {
  __shared__ FinishSmem<kBMergeWarps, D> fsm;
  const int q = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // The resolve kernel, and after it the next batch, may be scheduled at once:
  // the resolve waits for this grid; the next batch, until its own wait, reads
  // only the bank, its queries and the scratch set this batch did not use.
  asm volatile("griddepcontrol.launch_dependents;");
  // The query side before the wait on the scan: the queries are the caller's
  // input (read by the scan before its own wait, see mla_batch_kernel), and
  // this grid starts only after every block of the scan passed its wait.  The
  // last warp's reference query norm (a serial fp64 chain) overlaps the
  // scan's tail.
  const float* query = p.queries + (int64_t)q * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    const float v = query[d];
    fsm.qraw[d] = v;
    fsm.qd[d] = (double)v;
  }
  __syncthreads();
  if (warp == kBMergeWarps - 1 && lane == 0) fsm.qn = query_norm_seq_t<D>(fsm.qraw);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const bool safe = __ldcg(&p.scratch.hdr(q)->qsafe) != 0;
  final_merge<D, __half, false, kBMergeWarps, true, false, true, true>(p, q, kBMargin, safe, lane,
                                                                        warp, fsm);
}

}  // namespace mla
}  // namespace grm_b200
