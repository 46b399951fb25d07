/*
 * grm_oracle.c -- CPU restatement of GraftRepository's graft-route and
 * graft-mount arithmetic.  TEST INFRASTRUCTURE ONLY: this file is the parity
 * checker for the sm_100a kernels in graftrepository_b200/csrc.  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it; the
 * product path never does.
 *
 * Every function cites the reference code it restates (paths relative to the
 * GraftRepository checkout).  The arithmetic is written so that the C compiler
 * reproduces the reference's rounding exactly: build with -ffp-contract=off and
 * without -ffast-math (the recipe in oracle/Makefile does).
 *
 * Laws restated here:
 *   MLA route   cpp/grm_runtime.cpp:3193-3282 (rebuild_mla_arena: fp64 row
 *               norms cast to float), :3518-3545 (exact_mla_entry_score: fp64
 *               sequential dot, score = float(dot / (qnorm*norm + 1e-8))),
 *               :4299-4361 (route_mla_arena: drop non-finite, sort),
 *               :75-82 (score_node_better: score desc, node id asc).
 *   MLA INT4    cpp/grm_runtime.cpp:3241-3266 (INT4 arena: per-row max-abs
 *               scale, values clamped to [-7, 7]), :3568-3585
 *               (int4_mla_row_score, default non-OpenMP build: sequential fp32),
 *               :4363-4482 (route_mla_int4: top-M bulk, exact refine).
 *   GQA route   cpp/grm_runtime.cpp:3588-3671 (gqa_arena_key_score, general
 *               path: fp32 sequential dot, best = std::max(best, |dot|*inv),
 *               total += best over heads, total / H), :3673-3739 (the
 *               query_tokens == 4 path), :4498-4838 (route_gqa_raw ordering).
 *   Quant       core/graft_quant.py:93-144 (symmetric group-32 quantise /
 *               dequantise, fp32 scales, int8 container, fp16 output); the
 *               upload to bf16 at core/graft_arena.py:3490.
 *   Packed      the build's packed mount format (group 64, fp16 scales, 8/6/4
 *               bit little-endian bit packing): same math as graft_quant with
 *               the scale rounded to fp16 before the codes are taken.
 *   Splice      cpp/grm_runtime.cpp:4941-5064 (DeviceArena::apply_swap_tensor:
 *               sink | mount | live tail per outer row).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ floats */

static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* fp32 -> fp16, round to nearest even (IEEE 754 convertFormat). */
ORC_API uint16_t orc_f32_to_f16(float f) {
  const uint32_t x = f32_bits(f);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t ax = x & 0x7FFFFFFFu;
  if (ax > 0x7F800000u) return (uint16_t)(sign | 0x7E00u);       /* NaN */
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);      /* >= 65520 -> inf */
  if (ax >= 0x38800000u) {                                        /* normal half */
    const uint32_t r = ax - (112u << 23) + 0xFFFu + ((ax >> 13) & 1u);
    return (uint16_t)(sign | (r >> 13));
  }
  /* subnormal half: value = m * 2^-24; the scaling by 2^24 is exact */
  const float m = nearbyintf(bits_f32(ax) * 16777216.0f);
  return (uint16_t)(sign | (uint16_t)m);
}

ORC_API float orc_f16_to_f32(uint16_t h) {
  const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1Fu;
  const uint32_t m = h & 0x3FFu;
  if (e == 0) {
    const float v = (float)m * (1.0f / 16777216.0f);              /* exact */
    return sign ? -v : v;
  }
  if (e == 31) return bits_f32(sign | 0x7F800000u | (m << 13));
  return bits_f32(sign | ((e + 112u) << 23) | (m << 13));
}

/* bf16 -> fp32 (exact). */
ORC_API float orc_bf16_to_f32(uint16_t b) { return bits_f32((uint32_t)b << 16); }

/* fp32 -> bf16, round to nearest even. */
ORC_API uint16_t orc_f32_to_bf16(float f) {
  const uint32_t u = f32_bits(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)(((u >> 16) & 0x8000u) | 0x7FC0u);
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

static inline float bf16_to_f32(uint16_t b) { return bits_f32((uint32_t)b << 16); }

/* ------------------------------------------------------------------- top-k */

/* score_node_better (cpp/grm_runtime.cpp:75-82): score desc, id asc.  Float
 * comparison semantics (so -0 == +0). */
static inline int better(float sa, uint64_t ia, float sb, uint64_t ib) {
  if (sa != sb) return sa > sb;
  return ia < ib;
}

typedef struct { float s; uint64_t id; } orc_pair;

/* Keep the best `k` finite (score, id) pairs, sorted best first. */
static int64_t topk_select(const float* scores, const uint64_t* ids, int64_t n,
                           int64_t k, uint64_t* out_ids, float* out_scores) {
  orc_pair* best = (orc_pair*)malloc(sizeof(orc_pair) * (size_t)(k > 0 ? k : 1));
  int64_t have = 0;
  for (int64_t i = 0; i < n; ++i) {
    const float s = scores[i];
    if (!isfinite(s)) continue;                       /* M6: non-finite dropped */
    const uint64_t id = ids ? ids[i] : (uint64_t)i;
    if (have == k && !better(s, id, best[k - 1].s, best[k - 1].id)) continue;
    int64_t pos = have < k ? have : k - 1;
    while (pos > 0 && better(s, id, best[pos - 1].s, best[pos - 1].id)) {
      best[pos] = best[pos - 1];
      --pos;
    }
    best[pos].s = s;
    best[pos].id = id;
    if (have < k) ++have;
  }
  for (int64_t i = 0; i < k; ++i) {
    if (i < have) {
      out_ids[i] = best[i].id;
      if (out_scores) out_scores[i] = best[i].s;
    } else {
      out_ids[i] = UINT64_MAX;
      if (out_scores) out_scores[i] = NAN;
    }
  }
  free(best);
  return have;
}

ORC_API int64_t orc_topk(const float* scores, const uint64_t* ids, int64_t n, int64_t k,
                         uint64_t* out_ids, float* out_scores) {
  if (k <= 0) return 0;
  return topk_select(scores, ids, n, k, out_ids, out_scores);
}

/* --------------------------------------------------------------------- MLA */

/* rebuild_mla_arena (cpp/grm_runtime.cpp:3240-3249): norm_sq accumulated in
 * fp64 in element order, norm = float(sqrt(norm_sq)). */
ORC_API void orc_mla_row_norms(const float* rows, int64_t n, int64_t dim, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float* r = rows + i * dim;
    double acc = 0.0;
    for (int64_t d = 0; d < dim; ++d) acc += (double)r[d] * (double)r[d];
    out[i] = (float)sqrt(acc);
  }
}

/* route_mla_arena qnorm (cpp/grm_runtime.cpp:4311-4315). */
ORC_API double orc_mla_query_norm(const float* q, int64_t dim) {
  double acc = 0.0;
  for (int64_t d = 0; d < dim; ++d) acc += (double)q[d] * (double)q[d];
  return sqrt(acc);
}

/* exact_mla_entry_score for single-row entries (cpp/grm_runtime.cpp:3518-3545). */
ORC_API void orc_mla_scores(const float* rows, const float* norms, int64_t n, int64_t dim,
                            const float* q, float* out_scores) {
  const double qnorm = orc_mla_query_norm(q, dim);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float* r = rows + i * dim;
    double dot = 0.0;
    for (int64_t d = 0; d < dim; ++d) dot += (double)q[d] * (double)r[d];
    out_scores[i] = (float)(dot / ((qnorm * (double)norms[i]) + 1.0e-8));
  }
}

/* route_mla_arena (cpp/grm_runtime.cpp:4299-4361) without lexical/filter
 * policy: returns the number of finite scores placed (<= topk); unfilled id
 * slots are UINT64_MAX. */
ORC_API int64_t orc_mla_route(const float* rows, const float* norms, int64_t n, int64_t dim,
                              const float* q, int64_t topk, uint64_t* out_ids,
                              float* out_scores) {
  float* scores = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
  orc_mla_scores(rows, norms, n, dim, q, scores);
  const int64_t got = orc_topk(scores, NULL, n, topk, out_ids, out_scores);
  free(scores);
  return got;
}

/* ------------------------------------------------------------ MLA, INT4 mode */

static inline float std_min_f(float a, float b) { return (b < a) ? b : a; }  /* std::min */
static inline float std_max_f(float a, float b) { return (a < b) ? b : a; }  /* std::max */

/* The INT4 part of rebuild_mla_arena (cpp/grm_runtime.cpp:3241-3266), per
 * row: max |v| over the row (std::max, so NaN values are skipped), scale =
 * max_abs > 0 ? max_abs / 7 : 1, value_d = int8(clamp(round(v_d / scale),
 * -7, 7)) with std::round (half away from zero) and std::min / std::max
 * (a NaN quotient becomes 7), norm_scale = scale * (norm > 0 ? 1 / norm : 0)
 * with the row's fp32 norm. */
ORC_API void orc_mla_int4_arena(const float* rows, const float* norms, int64_t n, int64_t dim,
                                int8_t* values, float* norm_scales) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float* r = rows + i * dim;
    float max_abs = 0.0f;
    for (int64_t d = 0; d < dim; ++d) max_abs = std_max_f(max_abs, fabsf(r[d]));
    const float norm = norms[i];
    const float inv_norm = norm > 0.0f ? 1.0f / norm : 0.0f;
    const float scale = max_abs > 0.0f ? max_abs / 7.0f : 1.0f;
    norm_scales[i] = scale * inv_norm;
    for (int64_t d = 0; d < dim; ++d)
      values[i * dim + d] = (int8_t)std_max_f(-7.0f, std_min_f(7.0f, roundf(r[d] / scale)));
  }
}

/* int4_mla_row_score (cpp/grm_runtime.cpp:3568-3585) as the default build
 * (no OpenMP) computes it: dot_i4 += q_d * float(value_d) in fp32, element
 * order; score = dot_i4 * norm_scale * float(1 / (qnorm + 1e-8)); then the
 * route's `score += lexical_bonus` (0 without lexical keys, :4401-4402). */
ORC_API void orc_mla_int4_scores(const int8_t* values, const float* norm_scales, int64_t n,
                                 int64_t dim, const float* q, float* out) {
  const double qnorm = orc_mla_query_norm(q, dim);
  const float qinv = (float)(1.0 / (qnorm + 1.0e-8));
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const int8_t* v = values + i * dim;
    float dot = 0.0f;
    for (int64_t d = 0; d < dim; ++d) dot += q[d] * (float)v[d];
    float s = dot * norm_scales[i] * qinv;
    s += 0.0f;
    out[i] = s;
  }
}

static int pair_better(const void* a, const void* b) {
  const orc_pair* x = (const orc_pair*)a;
  const orc_pair* y = (const orc_pair*)b;
  if (better(x->s, x->id, y->s, y->id)) return -1;
  if (better(y->s, y->id, x->s, x->id)) return 1;
  return 0;
}

/* route_mla_int4 (cpp/grm_runtime.cpp:4363-4482) for single-row entries
 * without lexical keys or filters: the M = max(topk, refine_m) best finite
 * bulk scores by (score desc, node id asc) -- every finite one when M >= n --
 * are rescored with exact_mla_entry_score; the top-k of those finite exact
 * scores, ordered by score_node_better.  Returns the number placed. */
ORC_API int64_t orc_mla_int4_route(const float* rows, const float* norms, int64_t n, int64_t dim,
                                   const float* q, int64_t topk, int64_t refine_m,
                                   uint64_t* out_ids, float* out_scores) {
  int8_t* values = (int8_t*)malloc((size_t)(n > 0 ? n : 1) * (size_t)dim);
  float* ns = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
  float* bulk = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
  orc_pair* cand = (orc_pair*)malloc(sizeof(orc_pair) * (size_t)(n > 0 ? n : 1));
  orc_mla_int4_arena(rows, norms, n, dim, values, ns);
  orc_mla_int4_scores(values, ns, n, dim, q, bulk);
  int64_t nc = 0;
  for (int64_t i = 0; i < n; ++i)
    if (isfinite(bulk[i])) {
      cand[nc].s = bulk[i];
      cand[nc].id = (uint64_t)i;
      ++nc;
    }
  const int64_t m = refine_m > topk ? refine_m : topk;
  if (m < nc) {
    qsort(cand, (size_t)nc, sizeof(orc_pair), pair_better);
    nc = m;
  }
  const double qnorm = orc_mla_query_norm(q, dim);
  float* ex = (float*)malloc(sizeof(float) * (size_t)(nc > 0 ? nc : 1));
  uint64_t* ids = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)(nc > 0 ? nc : 1));
  for (int64_t c = 0; c < nc; ++c) {
    const int64_t i = (int64_t)cand[c].id;
    const float* r = rows + i * dim;
    double dot = 0.0;
    for (int64_t d = 0; d < dim; ++d) dot += (double)q[d] * (double)r[d];
    ex[c] = (float)(dot / ((qnorm * (double)norms[i]) + 1.0e-8));
    ids[c] = (uint64_t)i;
  }
  const int64_t got = topk_select(ex, ids, nc, topk, out_ids, out_scores);
  free(values);
  free(ns);
  free(bulk);
  free(cand);
  free(ex);
  free(ids);
  return got;
}

/* --------------------------------------------------------------------- GQA */

static inline float std_max(float a, float b) { return (a < b) ? b : a; }  /* std::max */

/* gqa_arena_key_score for one ragged key block laid out [kv_heads, T, dim]
 * (cpp/grm_runtime.cpp:3588-3671, and the query_tokens == 4 path at
 * :3673-3739).  `key_finite` mirrors arena.key_finite (:3369-3372). */
static float gqa_node_score(const uint16_t* key, int64_t T, int key_finite,
                            int64_t kv_heads, int64_t dim, const float* q,
                            int query_finite, int64_t q_heads, int64_t q_tokens) {
  if (T == 0) return 0.0f;
  if (!query_finite || !key_finite) return NAN;
  const int64_t repeat = q_heads / kv_heads;
  const float inv_denom = 1.0f / sqrtf((float)dim);
  float total = 0.0f;
  for (int64_t h = 0; h < q_heads; ++h) {
    const int64_t kh = h / repeat;
    float best = 0.0f;
    if (q_tokens == 4) {
      const float* q0 = q + (h * 4) * dim;
      for (int64_t ki = 0; ki < T; ++ki) {
        const uint16_t* k = key + (kh * T + ki) * dim;
        float dots[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int64_t d = 0; d < dim; ++d) {
          const float kv = bf16_to_f32(k[d]);
          for (int j = 0; j < 4; ++j) {
            const float p = q0[j * dim + d] * kv;
            dots[j] = dots[j] + p;
          }
        }
        const float row_best = std_max(std_max(fabsf(dots[0]), fabsf(dots[1])),
                                       std_max(fabsf(dots[2]), fabsf(dots[3])));
        best = std_max(best, row_best * inv_denom);
      }
    } else {
      for (int64_t qi = 0; qi < q_tokens; ++qi) {
        const float* qv = q + (h * q_tokens + qi) * dim;
        for (int64_t ki = 0; ki < T; ++ki) {
          const uint16_t* k = key + (kh * T + ki) * dim;
          float dot = 0.0f;
          for (int64_t d = 0; d < dim; ++d) {
            const float p = qv[d] * bf16_to_f32(k[d]);
            dot = dot + p;
          }
          best = std_max(best, fabsf(dot) * inv_denom);
        }
      }
    }
    total += best;
  }
  return total / (float)q_heads;
}

/* Per-node scores over a CSR bank: node i owns tokens [off[i], off[i+1]) and
 * its keys are the contiguous block keys[off[i]*kv_heads*dim ...] laid out
 * [kv_heads, T_i, dim] (bf16 bit patterns). */
ORC_API void orc_gqa_scores(const uint16_t* keys, const uint64_t* tok_off, int64_t n_nodes,
                            int64_t kv_heads, int64_t dim, const float* q, int64_t q_heads,
                            int64_t q_tokens, float* out_scores) {
  int query_finite = 1;
  const int64_t qn = q_heads * q_tokens * dim;
  for (int64_t i = 0; i < qn; ++i) query_finite = query_finite && isfinite(q[i]);
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t i = 0; i < n_nodes; ++i) {
    const int64_t T = (int64_t)(tok_off[i + 1] - tok_off[i]);
    const uint16_t* key = keys + (int64_t)tok_off[i] * kv_heads * dim;
    int key_finite = 1;
    const int64_t nv = kv_heads * T * dim;
    for (int64_t v = 0; v < nv && key_finite; ++v)
      key_finite = ((key[v] & 0x7F80u) != 0x7F80u);
    out_scores[i] = gqa_node_score(key, T, key_finite, kv_heads, dim, q, query_finite,
                                   q_heads, q_tokens);
  }
}

ORC_API int64_t orc_gqa_route(const uint16_t* keys, const uint64_t* tok_off, int64_t n_nodes,
                              int64_t kv_heads, int64_t dim, const float* q, int64_t q_heads,
                              int64_t q_tokens, int64_t topk, uint64_t* out_ids,
                              float* out_scores) {
  float* scores = (float*)malloc(sizeof(float) * (size_t)(n_nodes > 0 ? n_nodes : 1));
  orc_gqa_scores(keys, tok_off, n_nodes, kv_heads, dim, q, q_heads, q_tokens, scores);
  const int64_t got = orc_topk(scores, NULL, n_nodes, topk, out_ids, out_scores);
  free(scores);
  return got;
}

/* ------------------------------------------------------------------- quant */

static inline int qmax_signed(int bits) { return (1 << (bits - 1)) - 1; }  /* graft_quant.py:79 */

/* quantize_symmetric_group32 (core/graft_quant.py:93-133) over a flat stream
 * of n_groups groups of `group` values: scale = max|x|/qmax (fp32, 0 -> 1),
 * code = clip(round_half_even(x / scale), -qmax-1, qmax). */
ORC_API void orc_quant_ref(const float* x, int64_t n_groups, int group, int bits,
                           int8_t* codes, float* scales) {
  const int qmax = qmax_signed(bits);
#pragma omp parallel for schedule(static)
  for (int64_t g = 0; g < n_groups; ++g) {
    const float* xg = x + g * group;
    float m = 0.0f;
    for (int j = 0; j < group; ++j) { const float a = fabsf(xg[j]); m = (a > m) ? a : m; }
    float s = m / (float)qmax;
    if (s == 0.0f) s = 1.0f;
    scales[g] = s;
    for (int j = 0; j < group; ++j) {
      float c = nearbyintf(xg[j] / s);
      if (c < (float)(-qmax - 1)) c = (float)(-qmax - 1);
      if (c > (float)qmax) c = (float)qmax;
      codes[g * group + j] = (int8_t)c;
    }
  }
}

/* dequantize_symmetric_group32 (core/graft_quant.py:136-144): fp32(code)*scale
 * -> fp16; `out_bf16` additionally applies the fp16 -> bf16 upload cast
 * (core/graft_arena.py:3490).  Either output may be NULL. */
ORC_API void orc_dequant_ref(const int8_t* codes, const float* scales, int64_t n_groups,
                             int group, uint16_t* out_f16, uint16_t* out_bf16) {
#pragma omp parallel for schedule(static)
  for (int64_t g = 0; g < n_groups; ++g) {
    const float s = scales[g];
    for (int j = 0; j < group; ++j) {
      const int64_t i = g * group + j;
      const uint16_t h = orc_f32_to_f16((float)codes[i] * s);
      if (out_f16) out_f16[i] = h;
      if (out_bf16) out_bf16[i] = orc_f32_to_bf16(orc_f16_to_f32(h));
    }
  }
}

/* Packed mount format: bytes per group of `group` codes at `bits` bits. */
ORC_API int64_t orc_packed_group_bytes(int bits, int group) { return (int64_t)group * bits / 8; }

static void pack_codes(const int* c, int group, int bits, uint8_t* out) {
  if (bits == 8) {
    for (int j = 0; j < group; ++j) out[j] = (uint8_t)(c[j] & 0xFF);
  } else if (bits == 4) {
    for (int j = 0; j < group; j += 2)
      out[j / 2] = (uint8_t)((c[j] & 0xF) | ((c[j + 1] & 0xF) << 4));
  } else { /* bits == 6: 4 codes -> 3 bytes, little-endian 24-bit word */
    for (int j = 0; j < group; j += 4) {
      const uint32_t w = (uint32_t)(c[j] & 0x3F) | ((uint32_t)(c[j + 1] & 0x3F) << 6) |
                         ((uint32_t)(c[j + 2] & 0x3F) << 12) | ((uint32_t)(c[j + 3] & 0x3F) << 18);
      out[(j / 4) * 3 + 0] = (uint8_t)(w & 0xFF);
      out[(j / 4) * 3 + 1] = (uint8_t)((w >> 8) & 0xFF);
      out[(j / 4) * 3 + 2] = (uint8_t)((w >> 16) & 0xFF);
    }
  }
}

static inline int sext(uint32_t v, int bits) {
  const uint32_t m = 1u << (bits - 1);
  return (int)((v ^ m) - m);
}

static void unpack_codes(const uint8_t* in, int group, int bits, int* c) {
  if (bits == 8) {
    for (int j = 0; j < group; ++j) c[j] = (int)(int8_t)in[j];
  } else if (bits == 4) {
    for (int j = 0; j < group; j += 2) {
      c[j] = sext(in[j / 2] & 0xFu, 4);
      c[j + 1] = sext((in[j / 2] >> 4) & 0xFu, 4);
    }
  } else {
    for (int j = 0; j < group; j += 4) {
      const uint32_t w = (uint32_t)in[(j / 4) * 3] | ((uint32_t)in[(j / 4) * 3 + 1] << 8) |
                         ((uint32_t)in[(j / 4) * 3 + 2] << 16);
      for (int t = 0; t < 4; ++t) c[j + t] = sext((w >> (6 * t)) & 0x3Fu, 6);
    }
  }
}

/* Packed-format quantiser: the graft_quant law with the group scale rounded
 * to fp16 first (0 -> 1, capped at the largest finite fp16), codes taken
 * against that fp16 scale, then bit-packed.  Returns -1 on bad arguments. */
ORC_API int orc_quant_packed(const float* x, int64_t n_groups, int group, int bits,
                             uint8_t* codes, uint16_t* scales_f16) {
  if (!(bits == 8 || bits == 6 || bits == 4) || group <= 0 || group > 1024 || group % 4) return -1;
  const int qmax = qmax_signed(bits);
  const int64_t gb = orc_packed_group_bytes(bits, group);
#pragma omp parallel for schedule(static)
  for (int64_t g = 0; g < n_groups; ++g) {
    const float* xg = x + g * group;
    int c[1024];
    float m = 0.0f;
    for (int j = 0; j < group; ++j) { const float a = fabsf(xg[j]); m = (a > m) ? a : m; }
    uint16_t s16 = orc_f32_to_f16(m / (float)qmax);
    if ((s16 & 0x7FFFu) == 0) s16 = 0x3C00u;                 /* 0 -> 1.0 */
    if ((s16 & 0x7FFFu) >= 0x7C00u) s16 = 0x7BFFu;           /* cap at 65504 */
    const float s = orc_f16_to_f32(s16);
    scales_f16[g] = s16;
    for (int j = 0; j < group; ++j) {
      float v = nearbyintf(xg[j] / s);
      if (v < (float)(-qmax - 1)) v = (float)(-qmax - 1);
      if (v > (float)qmax) v = (float)qmax;
      c[j] = (int)v;
    }
    pack_codes(c, group, bits, codes + g * gb);
  }
  return 0;
}

/* Packed-format dequant: bf16_rn(fp32(code) * fp32(scale_f16)). */
ORC_API int orc_dequant_packed(const uint8_t* codes, const uint16_t* scales_f16, int64_t n_groups,
                               int group, int bits, uint16_t* out_bf16) {
  if (!(bits == 8 || bits == 6 || bits == 4) || group <= 0 || group > 1024 || group % 4) return -1;
  const int64_t gb = orc_packed_group_bytes(bits, group);
#pragma omp parallel for schedule(static)
  for (int64_t g = 0; g < n_groups; ++g) {
    int c[1024];
    unpack_codes(codes + g * gb, group, bits, c);
    const float s = orc_f16_to_f32(scales_f16[g]);
    for (int j = 0; j < group; ++j)
      out_bf16[g * group + j] = orc_f32_to_bf16((float)c[j] * s);
  }
  return 0;
}

/* ------------------------------------------------------------------- mount */

/* Scatter dequantised graft slices into the arena: graft g's layer l block of
 * `tokens` rows x `width` values lands at arena[l, seat[g] .. seat[g]+tokens).
 * `values` holds the grafts as [grafts, layers, tokens, width] bf16. */
ORC_API int orc_mount_scatter(const uint16_t* values, int64_t grafts, int64_t layers,
                              int64_t tokens, int64_t width, const int64_t* seats,
                              uint16_t* arena, int64_t arena_seats) {
  for (int64_t g = 0; g < grafts; ++g)
    if (seats[g] < 0 || seats[g] + tokens > arena_seats) return -1;
  for (int64_t g = 0; g < grafts; ++g)
    for (int64_t l = 0; l < layers; ++l)
      memcpy(arena + (l * arena_seats + seats[g]) * width,
             values + ((g * layers + l) * tokens) * width,
             (size_t)(tokens * width) * sizeof(uint16_t));
  return 0;
}

/* Re-RoPE of the positional part of mounted rows, at their arena seats
 * (core/graft_arena.py:344-367 `_rope_tensor` / `_rope_block_at`, called from
 * `_graft_block` :1848-1859 with pos0 = the first mounted seat).  For graft
 * g, layer l, token t at arena row p = seat[g] + t, every rope head (columns
 * offset + h*dim .. +dim, h = 0 .. (width-offset)/dim - 1) of the stored bf16
 * row becomes apply_rotary at position p, as the reference's fallback path
 * computes it on the uploaded tensor: x' = pair_swap ? [x0 x2 x4 ... x1 x3 ...]
 * (`_pair_swap_last`) : x; out_j = x'_j*cos[p][j] + r_j*sin[p][j] with
 * r_j = -x'_{j+dim/2} for j < dim/2 and x'_{j-dim/2} otherwise (rotate_half;
 * the tables hold cat([pos*inv, pos*inv])).  fp32 arithmetic: two products,
 * then one add (no fused multiply-add), one rounding to bf16.  tensor_cuda's
 * rope_apply, which the reference prefers, is not vendored: parity of this
 * step is unpinned. */
ORC_API int orc_mount_rope(uint16_t* arena, int64_t grafts, int64_t layers, int64_t tokens,
                           int64_t width, const int64_t* seats, int64_t arena_seats,
                           const float* cos_t, const float* sin_t, int64_t rows, int64_t offset,
                           int64_t dim, int pair_swap) {
  if (dim <= 0 || dim % 2 || dim > 1024 || offset < 0 || offset > width ||
      (width - offset) % dim)
    return -1;
  for (int64_t g = 0; g < grafts; ++g)
    if (seats[g] < 0 || seats[g] + tokens > arena_seats || seats[g] + tokens > rows) return -1;
  const int64_t heads = (width - offset) / dim, half = dim / 2;
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t g = 0; g < grafts; ++g)
    for (int64_t l = 0; l < layers; ++l) {
      float x[1024], xp[1024];
      for (int64_t t = 0; t < tokens; ++t) {
        const int64_t pos = seats[g] + t;
        uint16_t* row = arena + (l * arena_seats + pos) * width;
        for (int64_t h = 0; h < heads; ++h) {
          uint16_t* hp = row + offset + h * dim;
          for (int64_t j = 0; j < dim; ++j) x[j] = orc_bf16_to_f32(hp[j]);
          for (int64_t j = 0; j < dim; ++j)
            xp[j] = pair_swap ? (j < half ? x[2 * j] : x[2 * (j - half) + 1]) : x[j];
          for (int64_t j = 0; j < dim; ++j) {
            const float r = j < half ? -xp[j + half] : xp[j - half];
            const float a = xp[j] * cos_t[pos * dim + j];
            const float b = r * sin_t[pos * dim + j];
            hp[j] = orc_f32_to_bf16(a + b);
          }
        }
      }
    }
  return 0;
}

/* DeviceArena::apply_swap_tensor byte splice (cpp/grm_runtime.cpp:4941-5064):
 * per outer row, out = old[0:sink] | mount[0:n_mount] | old[tail_start:]. */
ORC_API int orc_swap_splice(const uint8_t* old_payload, int64_t outer, int64_t input_tokens,
                            const uint8_t* mount_payload, int64_t mount_tokens,
                            int64_t row_bytes, int64_t sink_tokens, int64_t old_mount_tokens,
                            uint8_t* out, int64_t* out_tokens) {
  if (input_tokens < sink_tokens) return -1;
  int64_t old_end = sink_tokens + old_mount_tokens;
  const int64_t tail_start = old_end < input_tokens ? old_end : input_tokens;
  const int64_t tail = input_tokens - tail_start;
  const int64_t out_t = sink_tokens + mount_tokens + tail;
  *out_tokens = out_t;
  for (int64_t o = 0; o < outer; ++o) {
    uint8_t* dst = out + o * out_t * row_bytes;
    const uint8_t* src = old_payload + o * input_tokens * row_bytes;
    memcpy(dst, src, (size_t)(sink_tokens * row_bytes));
    memcpy(dst + sink_tokens * row_bytes, mount_payload + o * mount_tokens * row_bytes,
           (size_t)(mount_tokens * row_bytes));
    memcpy(dst + (sink_tokens + mount_tokens) * row_bytes, src + tail_start * row_bytes,
           (size_t)(tail * row_bytes));
  }
  return 0;
}
