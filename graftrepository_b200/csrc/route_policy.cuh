// route_policy.cuh -- the route policy channels of RouterIndex on the device:
// the lexical bonus and the kind/scope/durability/mutability filters plus the
// entry's active flag (GraftRepository cpp/grm_runtime.cpp:3056-3105
// entry_allowed / filter_allows_bits, :3107-3167 lexical_hit_count /
// lexical_bonus, :4299-4361 route_mla_arena, :4840-4867 the GQA lexical law).
//
// Layout.  Strings never reach the device.  At attach the host keeps one
// dictionary per category (string -> code 0..254) and one dictionary of
// lexical keys (string -> id).  The device holds
//   codes[N]      the node's four category codes, one byte each;
//   active[N/32]  bitmap of active nodes;
//   post_off/post the inverted index: lexical id -> the nodes that carry it
//                 (each node once per id).
// A filtered route turns each filter list into a 256-bit set of codes (values
// absent from the dictionary match no node, as a string compare would) and
// builds allow[N/32] with one warp ballot per 32 nodes.  The scans then treat
// a row outside `allow` as absent.  The lexical channel of a query: every
// query key (with multiplicity, as lexical_hit_count counts) adds 1 to the
// nodes of its posting list; the nodes with hits are collected into a list
// of (node, hits), scored exactly by the route's own law plus hits / m, and
// merged with the route's top-k: a node without hits has bonus 0 and is in
// that top-k whenever it belongs to the final one.
#pragma once

#include <algorithm>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"

namespace grm_b200 {
namespace policy {

constexpr int kCats = 4;           // kind, scope, durability, mutability
constexpr int kMaxCodes = 255;     // codes per category; 255 = more values than that
constexpr int kItemsPerLaunch = 64;

// RouterIndex::Entry defaults (cpp/grm_runtime.hpp:488-492); set_route_metadata
// ignores empty values (:2922-2946), so "" or NULL keeps the default.
inline const char* category_default(int k) {
  static const char* const d[kCats] = {"turn", "conversation", "session", "ephemeral"};
  return d[k];
}

// split_lexical_keys (cpp/grm_runtime.cpp:5196-5208): '\n'-separated, empty
// items dropped.
inline std::vector<std::string> split_keys(const char* blob) {
  std::vector<std::string> out;
  if (!blob) return out;
  const char* s = blob;
  while (*s) {
    const char* e = s;
    while (*e && *e != '\n') ++e;
    if (e > s) out.emplace_back(s, (size_t)(e - s));
    s = *e ? e + 1 : e;
  }
  return out;
}

struct AllowSets {
  uint32_t bits[kCats][8];  // code c allowed: bit c of category's 256-bit set
  int on[kCats];            // category constrained (non-empty filter list)
};

// Posting ranges of up to kItemsPerLaunch query keys.
struct ItemRanges {
  uint32_t off[kItemsPerLaunch];
  uint32_t len[kItemsPerLaunch];
  uint32_t start[kItemsPerLaunch + 1];  // prefix sums of len
  int n;
};

struct Policy {
  bool set = false;
  int64_t nodes = 0;
  bool any_inactive = false;
  bool cat_overflow[kCats] = {false, false, false, false};
  std::unordered_map<std::string, int> cat_dict[kCats];
  std::unordered_map<std::string, uint32_t> lex_dict;
  std::vector<uint32_t> h_post_off;  // host copy of the index offsets
  uint32_t* d_codes = nullptr;
  uint32_t* d_active = nullptr;
  uint32_t* d_post = nullptr;
  uint32_t* d_allow = nullptr;
  uint32_t* d_hits = nullptr;       // [N], zero between routes
  uint2* d_hitlist = nullptr;       // [N] (node, hits)
  float* d_cand_s = nullptr;        // [N] scored hit nodes
  uint32_t* d_cand_id = nullptr;
  uint32_t* d_counter = nullptr;    // [1] hit nodes collected
};

inline void policy_free(Policy& P) {
  cudaFree(P.d_codes);
  cudaFree(P.d_active);
  cudaFree(P.d_post);
  cudaFree(P.d_allow);
  cudaFree(P.d_hits);
  cudaFree(P.d_hitlist);
  cudaFree(P.d_cand_s);
  cudaFree(P.d_cand_id);
  cudaFree(P.d_counter);
  P = Policy();
}

__device__ __forceinline__ bool row_allowed(const uint32_t* allow, int64_t row) {
  return !allow || ((__ldg(allow + (row >> 5)) >> (row & 31)) & 1u);
}

// allow word w covers rows 32w .. 32w+31: lane l tests row 32w + l.
static __global__ void allow_kernel(const uint32_t* __restrict__ codes, const uint32_t* __restrict__ active,
                             int64_t nodes, AllowSets sets, uint32_t* __restrict__ allow) {
  const int lane = threadIdx.x & 31;
  const int64_t words = (nodes + 31) / 32;
  for (int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32; w < words;
       w += (int64_t)gridDim.x * blockDim.x / 32) {
    const int64_t row = w * 32 + lane;
    bool ok = row < nodes && ((__ldg(active + w) >> lane) & 1u);
    if (ok) {
      const uint32_t c = __ldg(codes + row);
#pragma unroll
      for (int k = 0; k < kCats; ++k) {
        const uint32_t code = (c >> (8 * k)) & 0xFFu;
        if (sets.on[k] && !((sets.bits[k][code >> 5] >> (code & 31)) & 1u)) ok = false;
      }
    }
    const unsigned m = __ballot_sync(kFull, ok);
    if (lane == 0) allow[w] = m;
  }
}

__device__ __forceinline__ uint32_t posting_node(const ItemRanges& r, const uint32_t* post,
                                                 uint32_t j) {
  int it = 0;
  while (it + 1 < r.n && r.start[it + 1] <= j) ++it;
  return __ldg(post + r.off[it] + (j - r.start[it]));
}

// Every posting of every query key: hits[node] += 1.
static __global__ void lex_count_kernel(ItemRanges r, const uint32_t* __restrict__ post,
                                 uint32_t* __restrict__ hits) {
  const uint32_t total = r.start[r.n];
  for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < total; j += gridDim.x * blockDim.x)
    atomicAdd(hits + posting_node(r, post, j), 1u);
}

// The first posting thread to reach a node takes its count (and leaves 0
// behind for the next route) and appends (node, hits).
static __global__ void lex_collect_kernel(ItemRanges r, const uint32_t* __restrict__ post,
                                   uint32_t* __restrict__ hits, uint2* __restrict__ list,
                                   uint32_t* __restrict__ counter) {
  const uint32_t total = r.start[r.n];
  for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < total; j += gridDim.x * blockDim.x) {
    const uint32_t node = posting_node(r, post, j);
    const uint32_t c = atomicExch(hits + node, 0u);
    if (c) list[atomicAdd(counter, 1u)] = make_uint2(node, c);
  }
}

// Final top-k of one query: the route's own top-k (`base`, S = score + 0 for
// nodes without hits, the reference's `best + lexical_bonus` with bonus 0)
// merged with the scored hit nodes (S already final); a base entry whose
// node has hits is replaced by its scored hit entry.  Ties: lower node
// first; non-finite S dropped.  One block of kMergeWarps warps.
constexpr int kMergeWarps = 8;

static __global__ void __launch_bounds__(kMergeWarps * 32) lex_merge_kernel(
    uint64_t* ids, float* scores, int* count, int topk, uint64_t id_offset,
    const float* __restrict__ cand_s, const uint32_t* __restrict__ cand_id,
    const uint32_t* __restrict__ counter) {
  __shared__ uint32_t base_id[GRM_B200_MAX_TOPK];
  __shared__ float base_s[GRM_B200_MAX_TOPK];
  __shared__ unsigned superseded;
  __shared__ float sh_s[kMergeWarps * 32];
  __shared__ uint32_t sh_id[kMergeWarps * 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t n = *counter;
  const int bc = *count;
  if (threadIdx.x < GRM_B200_MAX_TOPK) {
    const bool v = (int)threadIdx.x < bc;
    base_id[threadIdx.x] = v ? (uint32_t)(ids[threadIdx.x] - id_offset) : kNoRow;
    base_s[threadIdx.x] = v ? scores[threadIdx.x] + 0.0f : -INFINITY;
  }
  if (threadIdx.x == 0) superseded = 0u;
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    const uint32_t node = cand_id[i];
    for (int b = 0; b < bc; ++b)
      if (base_id[b] == node) atomicOr(&superseded, 1u << b);
  }
  __syncthreads();
  WarpList list;
  list.init();
  // only the first topk entries of each list matter: candidates below the
  // list's k-th are skipped (that k-th only grows)
  for (uint32_t i0 = (uint32_t)warp * 32; i0 < n; i0 += blockDim.x) {
    const uint32_t i = i0 + lane;
    const float s = i < n ? cand_s[i] : -INFINITY;
    const uint32_t id = i < n ? cand_id[i] : kNoRow;
    list.offer_margin(s, id, lane, topk, 0.0f);
  }
  if (warp == 0) {
    const bool keep = lane < bc && !((superseded >> lane) & 1u);
    list.offer_margin(keep ? base_s[lane] : -INFINITY, keep ? base_id[lane] : kNoRow, lane, topk,
                      0.0f);
  }
  sh_s[warp * 32 + lane] = list.s;
  sh_id[warp * 32 + lane] = list.id;
  __syncthreads();
  if (warp == 0) {
    for (int w = 1; w < kMergeWarps; ++w)
      list.offer_margin(sh_s[w * 32 + lane], sh_id[w * 32 + lane], lane, topk, 0.0f);
    const bool ok = lane < topk && isfinite(list.s) && list.id != kNoRow;
    const unsigned m = __ballot_sync(kFull, ok);
    if (lane < topk) {
      ids[lane] = ok ? (uint64_t)list.id + id_offset : UINT64_MAX;
      scores[lane] = ok ? list.s : __int_as_float(0x7FC00000);
    }
    if (lane == 0) *count = __popc(m);
  }
}

// ---------------------------------------------------------------- host side

// Attach the per-node policy data.  lexical[i]: node i's '\n'-separated keys
// (NULL: none); cats[k][i]: node i's kind / scope / durability / mutability
// (cats[k] NULL: "" for every node); active: NULL = all active.
inline int policy_set(Policy& P, int64_t nodes, const char* const* lexical,
                      const char* const* const cats[kCats], const uint8_t* active,
                      ErrorSlot& err) {
  policy_free(P);
  P.nodes = nodes;
  std::vector<uint32_t> codes((size_t)nodes, 0u);
  for (int k = 0; k < kCats; ++k) {
    for (int64_t i = 0; i < nodes; ++i) {
      const std::string v = (cats[k] && cats[k][i] && cats[k][i][0]) ? cats[k][i]
                                                                       : category_default(k);
      auto it = P.cat_dict[k].find(v);
      int code;
      if (it != P.cat_dict[k].end()) {
        code = it->second;
      } else if ((int)P.cat_dict[k].size() < kMaxCodes) {
        code = (int)P.cat_dict[k].size();
        P.cat_dict[k].emplace(v, code);
      } else {
        code = kMaxCodes;
        P.cat_overflow[k] = true;
      }
      codes[(size_t)i] |= (uint32_t)code << (8 * k);
    }
  }
  const int64_t words = (nodes + 31) / 32;
  std::vector<uint32_t> act((size_t)words, 0u);
  for (int64_t i = 0; i < nodes; ++i) {
    const bool a = !active || active[i];
    if (a) act[(size_t)(i >> 5)] |= 1u << (i & 31);
    else P.any_inactive = true;
  }
  // inverted lexical index, each node once per key
  std::vector<std::vector<uint32_t>> lists;
  if (lexical) {
    std::vector<uint32_t> ids;
    for (int64_t i = 0; i < nodes; ++i) {
      if (!lexical[i]) continue;
      ids.clear();
      for (const auto& key : split_keys(lexical[i])) {
        auto it = P.lex_dict.find(key);
        uint32_t id;
        if (it == P.lex_dict.end()) {
          id = (uint32_t)P.lex_dict.size();
          P.lex_dict.emplace(key, id);
          lists.emplace_back();
        } else {
          id = it->second;
        }
        ids.push_back(id);
      }
      std::sort(ids.begin(), ids.end());
      ids.erase(std::unique(ids.begin(), ids.end()), ids.end());
      for (uint32_t id : ids) lists[id].push_back((uint32_t)i);
    }
  }
  P.h_post_off.assign(lists.size() + 1, 0u);
  uint64_t total = 0;
  for (size_t v = 0; v < lists.size(); ++v) {
    total += lists[v].size();
    if (total > 0xFFFFFFFFull) return err.set(GRM_B200_EINVAL, "lexical index exceeds 2^32 postings");
    P.h_post_off[v + 1] = (uint32_t)total;
  }
  std::vector<uint32_t> post;
  post.reserve((size_t)total);
  for (auto& l : lists) post.insert(post.end(), l.begin(), l.end());

  cudaError_t e = cudaSuccess;
  auto alloc = [&](void** p, size_t bytes) {
    if (e == cudaSuccess) e = cudaMalloc(p, bytes ? bytes : 16);
  };
  alloc((void**)&P.d_codes, sizeof(uint32_t) * (size_t)nodes);
  alloc((void**)&P.d_active, sizeof(uint32_t) * (size_t)words);
  alloc((void**)&P.d_post, sizeof(uint32_t) * post.size());
  alloc((void**)&P.d_allow, sizeof(uint32_t) * (size_t)words);
  alloc((void**)&P.d_hits, sizeof(uint32_t) * (size_t)nodes);
  alloc((void**)&P.d_hitlist, sizeof(uint2) * (size_t)nodes);
  alloc((void**)&P.d_cand_s, sizeof(float) * (size_t)nodes);
  alloc((void**)&P.d_cand_id, sizeof(uint32_t) * (size_t)nodes);
  alloc((void**)&P.d_counter, sizeof(uint32_t));
  if (e == cudaSuccess)
    e = cudaMemcpy(P.d_codes, codes.data(), sizeof(uint32_t) * codes.size(), cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(P.d_active, act.data(), sizeof(uint32_t) * act.size(), cudaMemcpyHostToDevice);
  if (e == cudaSuccess && !post.empty())
    e = cudaMemcpy(P.d_post, post.data(), sizeof(uint32_t) * post.size(), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(P.d_hits, 0, sizeof(uint32_t) * (size_t)nodes);
  if (e != cudaSuccess) {
    policy_free(P);
    return err.set(cuda_status(e), "route policy upload failed: %s", cudaGetErrorString(e));
  }
  P.set = true;
  return 0;
}

// The allow bitmap for one call's filters (kind, scope, durability,
// mutability blobs), or nullptr when every active node is allowed and none
// is inactive.
inline int policy_allow(Policy& P, const char* const filters[kCats], int sms, cudaStream_t s,
                        const uint32_t** allow_out, ErrorSlot& err) {
  *allow_out = nullptr;
  AllowSets sets;
  std::memset(&sets, 0, sizeof(sets));
  bool any = false;
  for (int k = 0; k < kCats; ++k) {
    const auto vals = split_keys(filters ? filters[k] : nullptr);
    if (vals.empty()) continue;
    if (P.cat_overflow[k])
      return err.set(GRM_B200_EINVAL,
                     "filter category %d has more than %d distinct values in this bank", k,
                     kMaxCodes);
    sets.on[k] = 1;
    any = true;
    for (const auto& v : vals) {
      auto it = P.cat_dict[k].find(v);
      if (it != P.cat_dict[k].end()) sets.bits[k][it->second >> 5] |= 1u << (it->second & 31);
    }
  }
  if (!any && !P.any_inactive) return 0;
  const int64_t words = (P.nodes + 31) / 32;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((int64_t)sms * 8, (words + 7) / 8));
  allow_kernel<<<grid, 256, 0, s>>>(P.d_codes, P.d_active, P.nodes, sets, P.d_allow);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return err.set(cuda_status(e), "allow kernel launch failed");
  *allow_out = P.d_allow;
  return 0;
}

// The posting ranges of one query's lexical keys (keys absent from the
// bank's dictionary have none).  *m_out = the number of query keys, the
// bonus denominator (unknown keys included).
using Ranges = std::vector<std::pair<uint32_t, uint32_t>>;

inline Ranges policy_ranges(const Policy& P, const char* blob, int* m_out) {
  const auto keys = split_keys(blob);
  *m_out = (int)keys.size();
  Ranges ranges;
  for (const auto& k : keys) {
    auto it = P.lex_dict.find(k);
    if (it == P.lex_dict.end()) continue;
    const uint32_t off = P.h_post_off[it->second], end = P.h_post_off[it->second + 1];
    if (end > off) ranges.emplace_back(off, end - off);
  }
  return ranges;
}

// pass 0: hits[node] += 1 over every posting; pass 1: take the counts into
// the hit list (and leave hits zero).
inline int policy_pass(Policy& P, const Ranges& ranges, int pass, int sms, cudaStream_t s,
                       ErrorSlot& err) {
  for (size_t c0 = 0; c0 < ranges.size(); c0 += kItemsPerLaunch) {
    ItemRanges r;
    std::memset(&r, 0, sizeof(r));
    r.n = (int)std::min<size_t>(kItemsPerLaunch, ranges.size() - c0);
    uint64_t acc = 0;
    for (int i = 0; i < r.n; ++i) {
      r.off[i] = ranges[c0 + i].first;
      r.len[i] = ranges[c0 + i].second;
      r.start[i] = (uint32_t)acc;
      acc += r.len[i];
    }
    if (acc > 0xFFFFFFFFull) return err.set(GRM_B200_EINVAL, "lexical postings exceed 2^32");
    r.start[r.n] = (uint32_t)acc;
    const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((uint64_t)sms * 8, (acc + 255) / 256));
    if (pass == 0)
      lex_count_kernel<<<grid, 256, 0, s>>>(r, P.d_post, P.d_hits);
    else
      lex_collect_kernel<<<grid, 256, 0, s>>>(r, P.d_post, P.d_hits, P.d_hitlist, P.d_counter);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return err.set(cuda_status(e), "lexical kernels launch failed");
  return 0;
}

// Count + collect for one query: the hit list (node, hits) in d_hitlist,
// its length in d_counter.  Returns 0 with *m_out == 0 when the query has no
// keys.
inline int policy_collect(Policy& P, const char* blob, int sms, cudaStream_t s, int* m_out,
                          ErrorSlot& err, uint64_t* postings = nullptr) {
  const Ranges ranges = policy_ranges(P, blob, m_out);
  if (postings) {
    *postings = 0;
    for (const auto& r : ranges) *postings += r.second;
  }
  if (*m_out == 0) return 0;
  cudaError_t e = cudaMemsetAsync(P.d_counter, 0, sizeof(uint32_t), s);
  if (e != cudaSuccess) return err.set(cuda_status(e), "lexical counter reset failed");
  int rc = policy_pass(P, ranges, 0, sms, s, err);
  if (!rc) rc = policy_pass(P, ranges, 1, sms, s, err);
  return rc;
}

}  // namespace policy
}  // namespace grm_b200
