/*
 * grm_b200.h -- C ABI of the B200 (sm_100a) graft route + mount library
 * (graftrepository_b200/libgrm_b200.so).
 *
 * This is the drop-in replacement for the CUDA route sidecars of
 * GraftRepository and for the device mount of routed grafts.  Each entry point
 * names the reference interface it replaces (paths are relative to the
 * GraftRepository checkout).  Conventions follow cpp/grm_runtime_c.h and the
 * sidecar ABI in scripts/grm_mla_cuda_probe.py:60-66:
 *
 *   - every function returns an int status: 0 ok, -1 invalid argument,
 *     1000 + cudaError_t for a CUDA runtime failure, 3000 + n for an error
 *     detected inside a kernel (3001 = a bounded device wait gave up);
 *   - a human-readable message is kept per handle (grm_b200_*_last_error) and
 *     per thread for handle-less calls (grm_b200_last_error);
 *   - a handle owns all the device memory it allocates (bank copy, row norms,
 *     route scratch); the caller owns every host buffer it passes;
 *   - route outputs are host arrays ids[query_count * topk] (uint64) and,
 *     optionally, scores[query_count * topk] (float); slots past the number of
 *     finite scores hold UINT64_MAX / NaN (the UINT64_MAX sentinel law of
 *     core/grm_cuda_router.py:465-475);
 *   - ids are bank row indices 0..nodes-1; callers map them to node ids;
 *   - calls on one handle are serialised by a mutex inside the handle; use one
 *     handle per stream for concurrency.
 *
 * Results are bit-exact against the reference's CPU route laws: the MLA
 * cosine of cpp/grm_runtime.cpp:3518-3545 (fp64 dot, fp64 query norm, fp32 row
 * norm) and the GQA raw |q.k| law of cpp/grm_runtime.cpp:3588-3671 (sequential
 * fp32), ordered by score desc then row asc (score_node_better, :75-82), with
 * non-finite scores dropped.
 */
#ifndef GRM_B200_H
#define GRM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* Element types of a bank or a query buffer. */
#define GRM_B200_F32 0
#define GRM_B200_F16 1
#define GRM_B200_BF16 2

#define GRM_B200_OK 0
#define GRM_B200_EINVAL (-1)
#define GRM_B200_CUDA_BASE 1000
#define GRM_B200_KERNEL_BASE 3000
/* Largest top-k a route call accepts (the reference caps at 16:
 * scripts/grm_mla_cuda_probe.py:357). */
#define GRM_B200_MAX_TOPK 32

typedef struct grm_b200_mla_bank grm_b200_mla_bank;
typedef struct grm_b200_gqa_bank grm_b200_gqa_bank;

/* ---------------------------------------------------------------- MLA route */

/* Upload a dense MLA centroid bank rows[nodes, dim] (row-major, element type
 * GRM_B200_F32 or GRM_B200_F16) to `device` and compute the fp32 row norms
 * (fp64 accumulate, cpp/grm_runtime.cpp:3240-3249).
 * Replaces grm_mla_cuda_arena_create (scripts/grm_mla_cuda_probe.py:286-336). */
int grm_b200_mla_bank_create(const void* rows_host, int dtype, int64_t nodes, int dim,
                             int device, grm_b200_mla_bank** out_bank);

/* A bank of multi-row entries (a digest node with its child centroids,
 * core/graft_arena.py:1670-1684): entry e owns rows entry_row_offsets[e] ..
 * entry_row_offsets[e+1]-1 of rows_host[rows, dim] and scores the max of its
 * finite row scores (RouterIndex::exact_mla_entry_score over
 * entry_row_offsets, cpp/grm_runtime.cpp:3219-3260, :3518-3545); routes
 * return entry indices.  The reference's CUDA sidecar takes single-row
 * entries only (core/graft_arena.py:1125-1143); this replaces the CPU route
 * those banks fall back to.  Every route entry point accepts such a bank
 * (the batched tensor-core path is not used for it). */
int grm_b200_mla_bank_create_multi(const void* rows_host, int dtype, int64_t rows, int dim,
                                   const uint64_t* entry_row_offsets, int64_t entries,
                                   int device, grm_b200_mla_bank** out_bank);

/* Same, from rows already resident on the current device; the bank copies
 * them (the caller may free its buffer afterwards). */
int grm_b200_mla_bank_create_device(const void* rows_device, int dtype, int64_t nodes,
                                    int dim, grm_b200_mla_bank** out_bank);

/* Route host queries[query_count, dim] (fp32).  Queries [0, warmup) are routed
 * but not timed; *elapsed_ms (may be NULL) is the device time of the rest.
 * out_scores may be NULL.
 * Replaces grm_mla_cuda_arena_route (scripts/grm_mla_cuda_probe.py:437-467). */
int grm_b200_mla_route(grm_b200_mla_bank* bank, const float* queries_host, int query_count,
                       int dim, int warmup, int topk, uint64_t* out_ids_host,
                       float* out_scores_host, float* elapsed_ms);

/* Route device-resident queries (no H2D copy).
 * Replaces grm_mla_cuda_arena_route_device (scripts/grm_mla_cuda_probe.py:473-488). */
int grm_b200_mla_route_device(grm_b200_mla_bank* bank, const float* queries_device,
                              int query_count, int dim, int warmup, int topk,
                              uint64_t* out_ids_host, float* out_scores_host,
                              float* elapsed_ms);

/* Stream-ordered route with device outputs and no host synchronisation (for
 * CUDA-graph capture and the node-sharded multi-GPU route): writes
 * out_ids_device[query_count * topk] and out_scores_device[...] on `stream`
 * (a cudaStream_t, NULL = legacy default stream).  `id_offset` is added to
 * every returned row id (the first global row of this shard).  query_count
 * must not exceed the capacity reserved by an earlier synchronous call or by
 * grm_b200_mla_reserve.  No reference counterpart (the reference is
 * single-GPU and always synchronises). */
int grm_b200_mla_route_async(grm_b200_mla_bank* bank, const float* queries_device,
                             int query_count, int topk, uint64_t id_offset,
                             uint64_t* out_ids_device, float* out_scores_device,
                             void* stream);

/* The two phases of grm_b200_mla_route_async, for callers that overlap or
 * time them separately (same arguments; call scan then resolve on one
 * stream).  Scan streams the bank once and resolves every query whose
 * candidates it can prove; resolve runs the exact fallback for the rest and
 * exits at once when there is none. */
int grm_b200_mla_scan_async(grm_b200_mla_bank* bank, const float* queries_device,
                            int query_count, int topk, uint64_t id_offset,
                            uint64_t* out_ids_device, float* out_scores_device, void* stream);
int grm_b200_mla_resolve_async(grm_b200_mla_bank* bank, const float* queries_device,
                               int query_count, int topk, uint64_t id_offset,
                               uint64_t* out_ids_device, float* out_scores_device,
                               void* stream);

/* Pre-size the per-query route scratch for up to `max_queries` queries per call. */
int grm_b200_mla_reserve(grm_b200_mla_bank* bank, int max_queries);

/* Replaces grm_mla_cuda_arena_destroy (scripts/grm_mla_cuda_probe.py:522-525). */
int grm_b200_mla_bank_destroy(grm_b200_mla_bank* bank);
const char* grm_b200_mla_last_error(grm_b200_mla_bank* bank);

/* Device pointer to the bank's fp32 row norms (nodes floats), for callers
 * that keep their own bank copy. */
const float* grm_b200_mla_row_norms_device(grm_b200_mla_bank* bank);

/* Counters of the exactness machinery since bank creation: queries routed,
 * and queries that took the exact fallback pass (margin saturated by
 * near-ties, a query outside the fast path's safe range, or a bank outside it),
 * counted on the device and read here with a blocking copy, so queries still
 * in flight on other streams may not be counted yet. */
int grm_b200_mla_stats(grm_b200_mla_bank* bank, uint64_t* routes, uint64_t* fallbacks);

/* Route policy data of the bank's nodes (RouterIndex::Entry lexical_keys,
 * kind, scope, durability, mutability, active; set through
 * grm_store_set_route_list's lexical blob, grm_store_set_route_metadata and
 * grm_store_set_active, cpp/grm_runtime_c.h:162-184, :394-400).
 * lexical_keys[i]: node i's '\n'-separated keys (NULL array or entry: none);
 * kinds/scopes/durabilities/mutabilities[i]: node i's values (NULL array or
 * entry, or "": the reference's defaults "turn" / "conversation" / "session" /
 * "ephemeral", cpp/grm_runtime.hpp:488-492); active[i] != 0 (NULL: all
 * active).  Replaces the previous policy data; at most 255 distinct values
 * per category are filterable. */
int grm_b200_mla_bank_set_policy(grm_b200_mla_bank* bank, const char* const* lexical_keys,
                                 const char* const* kinds, const char* const* scopes,
                                 const char* const* durabilities,
                                 const char* const* mutabilities, const uint8_t* active);

/* route_mla_arena with its policy channels (cpp/grm_runtime.cpp:4299-4361),
 * replacing grm_store_route / grm_store_route_filtered
 * (cpp/grm_runtime_c.h:403-422) for an MLA store: only active nodes whose
 * values pass every non-empty filter list are routed; a node's score is its
 * exact MLA score plus hits / m, where m is the number of the query's lexical
 * keys and hits how many of them the node carries (lexical_hit_count /
 * lexical_bonus, :3107-3167).  lexical_keys[q]: query q's '\n'-separated keys
 * (NULL array or entry: none); filters: '\n'-separated value lists, NULL or
 * "" = no constraint (split as split_lexical_keys, :5196-5208).  Output as
 * grm_b200_mla_route (scores are the policy scores). */
int grm_b200_mla_route_policy(grm_b200_mla_bank* bank, const float* queries_host,
                              int query_count, int dim, int topk,
                              const char* const* lexical_keys, const char* kind_filters,
                              const char* scope_filters, const char* durability_filters,
                              const char* mutability_filters, uint64_t* out_ids_host,
                              float* out_scores_host, float* elapsed_ms);

/* The reference's INT4 bulk/refine route mode: RouterIndex::route_mla_int4
 * (cpp/grm_runtime.cpp:4363-4482), which RouterIndex::route selects when
 * GRM_ROUTER_INT4 is set (:4486-4494); replaces grm_store_route in that mode
 * for a store of single-row entries routed without lexical keys or filters.
 * Each row is quantised to INT4 as rebuild_mla_arena does (:3241-3266:
 * per-row max-abs scale / 7, values in [-7, 7], norm scale = scale / norm),
 * every row gets the bulk score of int4_mla_row_score (:3568-3585, the default
 * build's sequential fp32 dot), the refine_m best bulk scores (score desc, row
 * asc; GRM_ROUTER_INT4_REFINE_M, default 4096; values below topk act as
 * topk) are rescored with the exact MLA law, and their top-k is returned
 * (exact scores), bit-exact with the reference's mode.  The INT4 arena (4
 * bits per value plus ~24 bytes per row of route buffers: ~152 MB at
 * 1M x 256) is built on the device by the bank's first INT4 call and kept
 * with the bank.  dim must be a multiple of 8; multi-row banks are refused.
 * Outputs as grm_b200_mla_route. */
int grm_b200_mla_route_int4(grm_b200_mla_bank* bank, const float* queries_host, int query_count,
                            int dim, int topk, int64_t refine_m, uint64_t* out_ids_host,
                            float* out_scores_host, float* elapsed_ms);

/* The same, stream-ordered with device queries and device outputs (as
 * grm_b200_mla_route_async; no scratch reservation is needed).  Calls on one
 * bank must not overlap on the GPU.  No reference counterpart beyond the
 * mode itself. */
int grm_b200_mla_route_int4_async(grm_b200_mla_bank* bank, const float* queries_device,
                                  int query_count, int topk, int64_t refine_m,
                                  uint64_t id_offset, uint64_t* out_ids_device,
                                  float* out_scores_device, void* stream);

/* Which kernels serve this bank (no reference counterpart; for tests and
 * diagnostics): GRM_B200_PATH_* bits. */
#define GRM_B200_PATH_BULK 1   /* single queries: bulk-copy streaming scan */
#define GRM_B200_PATH_BATCH 2  /* batches of >= 2 queries: tensor-core route */
#define GRM_B200_PATH_EXACT 4  /* bank outside the fast path: exact kernel only */
int grm_b200_mla_paths(grm_b200_mla_bank* bank, int* flags);

/* Allocation-free MLA route.  No counterpart in the reference.  For callers
 * that must not allocate device memory on the route path -- an engine that owns
 * all of HBM through its own pool, a route issued during CUDA-graph capture, a
 * decode loop that cannot afford an allocation's implicit synchronisation.
 * The caller passes fp16 rows[nodes, dim] (dim 64, 128, 256 or 512) and fp32
 * queries[query_count, dim] (query_count <= 16) in device memory and receives
 * ids/scores[query_count, topk] in its own device buffers on `stream`; row
 * norms are computed inline, results are bit-exact with the bank entry
 * points.  rows_device must be 16-byte aligned (rows are read with 16-byte
 * vector loads), queries_device and out_scores_device 4-byte and
 * out_ids_device 8-byte aligned; a misaligned pointer (e.g. an odd offset into
 * a pool) returns -1 before anything is launched.  Large banks with many
 * queries route on a narrower grid so that every query's scratch fits.
 * Scratch is a fixed 2 MiB __device__ array inside the library (held
 * by every GPU that loads it until exit), shared by all calls: calls that
 * overlap on the GPU race and must be serialised by the caller.  The first
 * call on each device looks up the array's device address; make it before any
 * stream capture.  Oversized requests return -1 with a message in
 * grm_b200_last_error(). */
int grm_b200_mla_route_noalloc(const void* rows_device, int64_t nodes, int dim,
                               const float* queries_device, int query_count, int topk,
                               uint64_t* out_ids_device, float* out_scores_device,
                               void* stream);

/* ---------------------------------------------------------------- GQA route */

/* Ragged (CSR) GQA key bank.  Node i owns tokens [token_offsets[i],
 * token_offsets[i+1]); its keys are the contiguous block
 * keys + token_offsets[i] * kv_heads * head_dim laid out [kv_heads, T_i,
 * head_dim] (layers concatenated on the head axis).  dtype GRM_B200_BF16,
 * GRM_B200_F16 or GRM_B200_F32; token_offsets has nodes + 1 entries starting
 * at 0.  Replaces grm_gqa_cuda_arena_create (scripts/grm_gqa_cuda_probe.py:
 * 297-365), whose dense zero-padded bank is dropped for CSR. */
int grm_b200_gqa_bank_create(const void* keys_host, int dtype, const uint64_t* token_offsets,
                             int64_t nodes, int kv_heads, int head_dim, int device,
                             grm_b200_gqa_bank** out_bank);

/* Same over keys already resident on the current device.  The bank BORROWS
 * keys_device (no copy: a 100k-node bank is ~216 GB); the caller keeps it
 * alive until grm_b200_gqa_bank_destroy. */
int grm_b200_gqa_bank_create_device(const void* keys_device, int dtype,
                                    const uint64_t* token_offsets, int64_t nodes,
                                    int kv_heads, int head_dim,
                                    grm_b200_gqa_bank** out_bank);

/* Route host queries[query_count, query_heads, query_tokens, head_dim] (fp32).
 * query_heads must be a multiple of kv_heads (GQA group = query_heads /
 * kv_heads).  Replaces grm_gqa_cuda_arena_route
 * (scripts/grm_gqa_cuda_probe.py:484-516). */
int grm_b200_gqa_route(grm_b200_gqa_bank* bank, const float* queries_host, int query_count,
                       int query_heads, int query_tokens, int warmup, int topk,
                       uint64_t* out_ids_host, float* out_scores_host, float* elapsed_ms);

/* Replaces grm_gqa_cuda_arena_route_device (scripts/grm_gqa_cuda_probe.py:524-537). */
int grm_b200_gqa_route_device(grm_b200_gqa_bank* bank, const float* queries_device,
                              int query_count, int query_heads, int query_tokens,
                              int warmup, int topk, uint64_t* out_ids_host,
                              float* out_scores_host, float* elapsed_ms);

/* Stream-ordered GQA route with device outputs (no host synchronisation):
 * out_ids_device / out_scores_device [query_count * topk] on `stream`;
 * `id_offset` is added to every returned node row (the first row of this
 * shard).  Calls on one bank must not overlap on the GPU (shared scratch).
 * No reference counterpart (the reference GQA route always synchronises). */
int grm_b200_gqa_route_async(grm_b200_gqa_bank* bank, const float* queries_device,
                             int query_count, int query_heads, int query_tokens, int topk,
                             uint64_t id_offset, uint64_t* out_ids_device,
                             float* out_scores_device, void* stream);

/* Replaces grm_gqa_cuda_arena_destroy (scripts/grm_gqa_cuda_probe.py:584-587). */
int grm_b200_gqa_bank_destroy(grm_b200_gqa_bank* bank);
const char* grm_b200_gqa_last_error(grm_b200_gqa_bank* bank);
int grm_b200_gqa_stats(grm_b200_gqa_bank* bank, uint64_t* routes, uint64_t* refined_nodes);

/* Which scan serves this bank (no reference counterpart; for tests and
 * diagnostics): GRM_B200_GQA_PATH_* bits. */
#define GRM_B200_GQA_PATH_FAST 1  /* tensor-core approximate pass + exact refine */
#define GRM_B200_GQA_PATH_TMA 2   /* ... with TMA-staged key tiles */
int grm_b200_gqa_paths(grm_b200_gqa_bank* bank, int* flags);

/* Route policy data of the GQA bank's nodes: as grm_b200_mla_bank_set_policy. */
int grm_b200_gqa_bank_set_policy(grm_b200_gqa_bank* bank, const char* const* lexical_keys,
                                 const char* const* kinds, const char* const* scopes,
                                 const char* const* durabilities,
                                 const char* const* mutabilities, const uint8_t* active);

/* route_gqa_raw with its policy channels (cpp/grm_runtime.cpp:4498-4867),
 * replacing grm_store_route_gqa with lexical keys or filters
 * (cpp/grm_runtime_c.h:423-436): filters as grm_b200_mla_route_policy; with
 * lexical keys the order is S = raw / (max raw + 1e-8) + hits / m over the
 * allowed nodes (the normalised law of :4840-4867), without them the raw
 * order.  Scores returned are S (lexical) or raw. */
int grm_b200_gqa_route_policy(grm_b200_gqa_bank* bank, const float* queries_host,
                              int query_count, int query_heads, int query_tokens, int topk,
                              const char* const* lexical_keys, const char* kind_filters,
                              const char* scope_filters, const char* durability_filters,
                              const char* mutability_filters, uint64_t* out_ids_host,
                              float* out_scores_host, float* elapsed_ms);

/* ------------------------------------------------------------------- mount */

/* Fused dequantise + scatter of routed grafts into a preallocated bf16 arena
 * arena[layers, arena_seats, width] (device).  Graft g's layer l block of
 * `tokens` rows lands at arena[l, seats[g] .. seats[g] + tokens).  seats is a
 * host array of n_grafts (<= 64) non-negative offsets with
 * seats[g] + tokens <= arena_seats.  Runs on `stream` without synchronising.
 *
 * grm_b200_mount_ref: the reference storage format of core/graft_quant.py
 * (:93-144, pack_kv_arrays :177-217): int8 codes (one byte per code at every
 * bit depth) in groups of 32 along the value stream, fp32 scales; output
 * bf16(fp16(fp32(code) * scale)) -- the fp16 dequant of
 * dequantize_symmetric_group32 followed by the bf16 upload cast of
 * core/graft_arena.py:3490.  codes[n_grafts, layers, tokens * width],
 * scales[n_grafts, layers, tokens * width / 32].
 * Replaces unpack_node's host dequant + upload (core/graft_arena.py:3479-3492)
 * and the splice of core/graft_arena.py:1933-1995. */
int grm_b200_mount_ref(const int8_t* codes_device, const float* scales_device,
                       int64_t n_grafts, int64_t layers, int64_t tokens, int64_t width,
                       const int64_t* seats_host, uint16_t* arena_device,
                       int64_t arena_seats, void* stream);

/* grm_b200_mount_packed: the packed format -- codes bit-packed little-endian at
 * `bits` in {8, 6, 4} in groups of `group` (64) values along the flattened
 * (token, value) stream of each (graft, layer), one fp16 scale per group;
 * output bf16(fp32(code) * fp32(scale)).  codes[n_grafts, layers,
 * tokens * width * bits / 8], scales[n_grafts, layers, tokens * width / group].
 * No reference counterpart (graft_quant keeps one byte per code and fp32
 * scales); same quantisation law with the scale rounded to fp16. */
int grm_b200_mount_packed(const uint8_t* codes_device, const uint16_t* scales_device,
                          int bits, int group, int64_t n_grafts, int64_t layers,
                          int64_t tokens, int64_t width, const int64_t* seats_host,
                          uint16_t* arena_device, int64_t arena_seats, void* stream);

/* Re-RoPE of the positional part of the mounted rows, fused into the mount
 * (core/graft_arena.py:344-367 `_rope_tensor`, applied by `_graft_block`
 * :1848-1859 at the mount seats; the reference runs it through tensor_cuda's
 * rope_apply, which is not vendored).  Columns [offset, width) of every
 * mounted row are heads of `dim` values (MLA: the 32-d k_pe after the 256-d
 * latent, offset 256; GQA: offset 0, dim = head_dim).  Head element j of the
 * row at arena seat p becomes x'_j * cos[p][j] + r_j * sin[p][j] with x' the
 * stored bf16 values (pair-swapped [x0 x2 .. x1 x3 ..] when pair_swap, the
 * `ROPE_PAIR_SWAP` layout), r = rotate_half(x'); fp32 products and add, one
 * bf16 rounding.  cos/sin: device fp32 [rows, dim], rows > every seat + tokens - 1;
 * offset % 8 == 0, dim % 16 == 0.  With dim a power of two <= 256, offset a
 * multiple of dim and 16-byte aligned tables (every MLA k_pe and GQA head
 * layout) the partner values come from the same warp's registers; other
 * layouts re-read them from the codes. */
typedef struct grm_b200_rope_spec {
  const float* cos_device;
  const float* sin_device;
  int64_t rows;
  int64_t offset;
  int64_t dim;
  int pair_swap;
} grm_b200_rope_spec;

int grm_b200_mount_packed_rope(const uint8_t* codes_device, const uint16_t* scales_device,
                               int bits, int group, int64_t n_grafts, int64_t layers,
                               int64_t tokens, int64_t width, const int64_t* seats_host,
                               uint16_t* arena_device, int64_t arena_seats,
                               const grm_b200_rope_spec* rope, void* stream);

/* The reference format with the same fused re-RoPE (on the bf16(fp16(code *
 * scale)) values the plain mount stores). */
int grm_b200_mount_ref_rope(const int8_t* codes_device, const float* scales_device,
                            int64_t n_grafts, int64_t layers, int64_t tokens, int64_t width,
                            const int64_t* seats_host, uint16_t* arena_device,
                            int64_t arena_seats, const grm_b200_rope_spec* rope, void* stream);

/* Device byte splice out = old[:sink] | mount | old[tail_start:] per outer row,
 * tail_start = min(sink + old_mount_tokens, input_tokens).  old[outer,
 * input_tokens, row_bytes], mount[outer, mount_tokens, row_bytes], out[outer,
 * sink + mount_tokens + (input_tokens - tail_start), row_bytes]; row_bytes a
 * multiple of 16.  *out_tokens receives the output sequence length.  Replaces
 * the host byte splice DeviceArena::apply_swap_tensor
 * (cpp/grm_runtime.cpp:4941-5064) / tc.arena_row_pair_transaction. */
int grm_b200_arena_splice(const void* old_device, int64_t outer, int64_t input_tokens,
                          const void* mount_device, int64_t mount_tokens, int64_t row_bytes,
                          int64_t sink_tokens, int64_t old_mount_tokens, void* out_device,
                          int64_t* out_tokens, void* stream);

/* Host -> device upload of a packed payload's per-row parts, interleaved:
 * device row r (dst_row_bytes) = part 0 row r | part 1 row r | ..., where
 * part p is rows x part_row_bytes[p] contiguous bytes at parts_host[p].  This
 * puts an MLA node's separately packed {"c", "kpe"} codes (or scales) side
 * by side as the arena row [latent | k_pe] the mount writes, without a host
 * copy (pack_kv_arrays fields, core/graft_quant.py:177-217; node payload
 * core/graft_arena.py:464-477).  Stream-ordered on `stream`. */
int grm_b200_upload_rows(const void* const* parts_host, const int64_t* part_row_bytes,
                         int n_parts, int64_t rows, void* dst_device, int64_t dst_row_bytes,
                         void* stream);

/* ----------------------------------------------------- multi-GPU top-k merge */

/* Merge `lists` candidate lists of `per_list` (score, id) entries each (device
 * arrays scores[lists * per_list], ids[...], UINT64_MAX = empty) into the best
 * `topk` by score desc then id asc, dropping non-finite scores.  Used after an
 * NCCL all-gather of per-shard route results.  No reference counterpart (the
 * reference is single-GPU). */
int grm_b200_merge_topk(const float* scores_device, const uint64_t* ids_device, int queries,
                        int lists, int per_list, int topk, float* out_scores_device,
                        uint64_t* out_ids_device, void* stream);

/* The same merge with list l's entries at scores_device + l * scores_list_stride
 * and ids_device + l * ids_list_stride (elements; each stride >= queries *
 * per_list), so the scores and ids of every rank can travel in one all-gather
 * of a packed per-rank block.  No reference counterpart. */
int grm_b200_merge_topk_strided(const float* scores_device, int64_t scores_list_stride,
                                const uint64_t* ids_device, int64_t ids_list_stride, int queries,
                                int lists, int per_list, int topk, float* out_scores_device,
                                uint64_t* out_ids_device, void* stream);

/* ----------------------------------------------------------------- helpers */

/* Upload a host buffer to a fresh device allocation on the current device.
 * Replaces grm_{mla,gqa}_cuda_upload_queries (scripts/grm_mla_cuda_probe.py:493-513). */
int grm_b200_upload(const void* host, size_t bytes, void** out_device);
/* Replaces grm_{mla,gqa}_cuda_free_device_ptr (scripts/grm_mla_cuda_probe.py:515-520). */
int grm_b200_free_device_ptr(void* device);
/* Message of the last failed handle-less call on this thread. */
const char* grm_b200_last_error(void);
/* Library version string. */
const char* grm_b200_version(void);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* GRM_B200_H */
