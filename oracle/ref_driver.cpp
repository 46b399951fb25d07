// ref_driver.cpp -- thin C driver over the REFERENCE's own native runtime
// (GraftRepository cpp/grm_runtime.cpp, compiled from its sources by
// oracle/Makefile into oracle/_ref/).  TEST INFRASTRUCTURE ONLY: it loads
// whole route banks into a reference grm_store_handle through the reference's
// C ABI (cpp/grm_runtime_c.h) in one native call, so the Python tests and the
// CPU baseline avoid one ctypes call per node.  Nothing here computes a score:
// every number comes from the reference's RouterIndex / DeviceArena.
#include <cstdint>
#include <cstring>
#include <vector>

#include "grm_runtime_c.h"

extern "C" {

// MLA store (cpp/grm_runtime_c.h:70-76) with one single-row route key per node
// (grm_store_set_route_list, :394-400).  Node ids are 0..n-1 (add_node order).
grm_store_handle* refd_mla_create(const float* rows, uint64_t n, uint64_t dim) {
  grm_store_handle* h = grm_store_create_mla("RefDriverMLA", 1, 2048, 576, 0, 512, 64);
  if (!h) return nullptr;
  const uint64_t offs[2] = {0, dim};
  for (uint64_t i = 0; i < n; ++i) {
    uint64_t id = 0;
    if (grm_store_add_node(h, "", 1, nullptr, 0, &id) != 0 || id != i) {
      grm_store_destroy(h);
      return nullptr;
    }
    if (grm_store_set_route_list(h, id, rows + i * dim, dim, offs, 1, "") != 0) {
      grm_store_destroy(h);
      return nullptr;
    }
  }
  return h;
}

// MLA store with route policy data per node: lexical keys through
// grm_store_set_route_list's blob, kind/scope/durability/mutability through
// grm_store_set_route_metadata and the active flag through grm_store_set_active
// (cpp/grm_runtime_c.h:162-184, :394-400).  NULL arrays or entries leave the
// reference's defaults.
grm_store_handle* refd_mla_create_policy(const float* rows, uint64_t n, uint64_t dim,
                                         const char* const* lexical, const char* const* kinds,
                                         const char* const* scopes,
                                         const char* const* durabilities,
                                         const char* const* mutabilities,
                                         const uint8_t* active) {
  grm_store_handle* h = grm_store_create_mla("RefDriverMLA", 1, 2048, 576, 0, 512, 64);
  if (!h) return nullptr;
  const uint64_t offs[2] = {0, dim};
  auto at = [](const char* const* a, uint64_t i) -> const char* { return a ? a[i] : nullptr; };
  for (uint64_t i = 0; i < n; ++i) {
    uint64_t id = 0;
    const char* lex = at(lexical, i);
    int rc = grm_store_add_node(h, "", 1, nullptr, 0, &id);
    if (rc == 0 && id != i) rc = -1;
    if (rc == 0) rc = grm_store_set_route_list(h, id, rows + i * dim, dim, offs, 1, lex ? lex : "");
    if (rc == 0 && (kinds || scopes || durabilities || mutabilities))
      rc = grm_store_set_route_metadata(h, id, at(kinds, i), at(scopes, i), at(durabilities, i),
                                        at(mutabilities, i));
    if (rc == 0 && active && !active[i]) rc = grm_store_set_active(h, id, 0);
    if (rc != 0) {
      grm_store_destroy(h);
      return nullptr;
    }
  }
  return h;
}

// grm_store_route_filtered (cpp/grm_runtime_c.h:411-422).
int refd_mla_route_policy(grm_store_handle* h, const float* q, uint64_t dim, const char* lexical,
                          const char* kinds, const char* scopes, const char* durabilities,
                          const char* mutabilities, uint64_t topk, uint64_t* out,
                          uint64_t* out_count) {
  return grm_store_route_filtered(h, q, dim, lexical ? lexical : "", kinds ? kinds : "",
                                  scopes ? scopes : "", durabilities ? durabilities : "",
                                  mutabilities ? mutabilities : "", topk, out, topk, out_count);
}

// MLA store of multi-row entries: node e's route keys are rows off[e] ..
// off[e+1]-1 (grm_store_set_route_list with key_count > 1).
grm_store_handle* refd_mla_create_multi(const float* rows, uint64_t n_rows, uint64_t dim,
                                        const uint64_t* off, uint64_t entries) {
  grm_store_handle* h = grm_store_create_mla("RefDriverMLA", 1, 2048, 576, 0, 512, 64);
  if (!h) return nullptr;
  std::vector<uint64_t> offs;
  for (uint64_t e = 0; e < entries; ++e) {
    uint64_t id = 0;
    int rc = grm_store_add_node(h, "", 1, nullptr, 0, &id);
    if (rc == 0 && id != e) rc = -1;
    const uint64_t k = off[e + 1] - off[e];
    offs.resize(k + 1);
    for (uint64_t j = 0; j <= k; ++j) offs[j] = j * dim;
    if (rc == 0 && k > 0)
      rc = grm_store_set_route_list(h, id, rows + off[e] * dim, k * dim, offs.data(), k, "");
    if (rc != 0 || off[e + 1] > n_rows) {
      grm_store_destroy(h);
      return nullptr;
    }
  }
  return h;
}

// grm_store_route (cpp/grm_runtime_c.h:403-410).
int refd_mla_route(grm_store_handle* h, const float* q, uint64_t dim, uint64_t topk,
                   uint64_t* out, uint64_t* out_count) {
  return grm_store_route(h, q, dim, "", topk, out, topk, out_count);
}

// GQA store (cpp/grm_runtime_c.h:89-95) over a CSR bank of bf16 keys: node i's
// key block is [kv_heads, T_i, head_dim] at keys + tok_off[i]*kv_heads*head_dim.
// The reference stores fp32, so each bf16 value is widened exactly.
grm_store_handle* refd_gqa_create(const uint16_t* keys_bf16, const uint64_t* tok_off,
                                  uint64_t n, uint64_t kv_heads, uint64_t head_dim) {
  grm_store_handle* h = grm_store_create_gqa(
      "RefDriverGQA", 36, 2560, 2048, 0, static_cast<int>(kv_heads),
      static_cast<int>(head_dim));
  if (!h) return nullptr;
  std::vector<float> buf;
  for (uint64_t i = 0; i < n; ++i) {
    uint64_t id = 0;
    if (grm_store_add_node(h, "", 1, nullptr, 0, &id) != 0 || id != i) {
      grm_store_destroy(h);
      return nullptr;
    }
    const uint64_t T = tok_off[i + 1] - tok_off[i];
    const uint64_t nv = kv_heads * T * head_dim;
    buf.resize(nv);
    const uint16_t* src = keys_bf16 + tok_off[i] * kv_heads * head_dim;
    for (uint64_t v = 0; v < nv; ++v) {
      const uint32_t u = static_cast<uint32_t>(src[v]) << 16;
      std::memcpy(&buf[v], &u, 4);
    }
    const uint64_t offs[2] = {0, nv};
    if (grm_store_set_route_list(h, id, buf.data(), nv, offs, 1, "") != 0) {
      grm_store_destroy(h);
      return nullptr;
    }
  }
  return h;
}

// GQA store with route policy data per node (as refd_mla_create_policy).
grm_store_handle* refd_gqa_create_policy(const uint16_t* keys_bf16, const uint64_t* tok_off,
                                         uint64_t n, uint64_t kv_heads, uint64_t head_dim,
                                         const char* const* lexical, const char* const* kinds,
                                         const char* const* scopes,
                                         const char* const* durabilities,
                                         const char* const* mutabilities,
                                         const uint8_t* active) {
  grm_store_handle* h = grm_store_create_gqa(
      "RefDriverGQA", 36, 2560, 2048, 0, static_cast<int>(kv_heads),
      static_cast<int>(head_dim));
  if (!h) return nullptr;
  auto at = [](const char* const* a, uint64_t i) -> const char* { return a ? a[i] : nullptr; };
  std::vector<float> buf;
  for (uint64_t i = 0; i < n; ++i) {
    uint64_t id = 0;
    int rc = grm_store_add_node(h, "", 1, nullptr, 0, &id);
    if (rc == 0 && id != i) rc = -1;
    const uint64_t T = tok_off[i + 1] - tok_off[i];
    const uint64_t nv = kv_heads * T * head_dim;
    buf.resize(nv);
    const uint16_t* src = keys_bf16 + tok_off[i] * kv_heads * head_dim;
    for (uint64_t v = 0; v < nv; ++v) {
      const uint32_t u = static_cast<uint32_t>(src[v]) << 16;
      std::memcpy(&buf[v], &u, 4);
    }
    const uint64_t offs[2] = {0, nv};
    const char* lex = at(lexical, i);
    if (rc == 0) rc = grm_store_set_route_list(h, id, buf.data(), nv, offs, 1, lex ? lex : "");
    if (rc == 0 && (kinds || scopes || durabilities || mutabilities))
      rc = grm_store_set_route_metadata(h, id, at(kinds, i), at(scopes, i), at(durabilities, i),
                                        at(mutabilities, i));
    if (rc == 0 && active && !active[i]) rc = grm_store_set_active(h, id, 0);
    if (rc != 0) {
      grm_store_destroy(h);
      return nullptr;
    }
  }
  return h;
}

int refd_gqa_route_policy(grm_store_handle* h, const float* q, uint64_t q_heads, uint64_t q_tokens,
                          uint64_t head_dim, const char* lexical, const char* kinds,
                          const char* scopes, const char* durabilities, const char* mutabilities,
                          uint64_t topk, uint64_t* out, uint64_t* out_count) {
  return grm_store_route_gqa(h, q, q_heads, q_tokens, head_dim, lexical ? lexical : "",
                             kinds ? kinds : "", scopes ? scopes : "",
                             durabilities ? durabilities : "", mutabilities ? mutabilities : "",
                             topk, out, topk, out_count);
}

// grm_store_route_gqa (cpp/grm_runtime_c.h:423-436), no lexical/filter policy.
int refd_gqa_route(grm_store_handle* h, const float* q, uint64_t q_heads, uint64_t q_tokens,
                   uint64_t head_dim, uint64_t topk, uint64_t* out, uint64_t* out_count) {
  return grm_store_route_gqa(h, q, q_heads, q_tokens, head_dim, "", "", "", "", "", topk, out,
                             topk, out_count);
}

// DeviceArena byte splice through the reference ABI (cpp/grm_runtime_c.h:437-466):
// configure the arena, record `old_mount_tokens` as the current mount, then
// apply_swap_tensor.  Shapes are rank-3 [outer, tokens, inner] with seq_dim 1.
int refd_swap(uint64_t sink, uint64_t width, uint64_t old_mount_tokens,
              const uint8_t* old_payload, uint64_t outer, uint64_t input_tokens,
              const uint8_t* mount_payload, uint64_t mount_tokens, uint64_t inner,
              uint64_t elem_size, uint8_t* out, uint64_t out_cap, uint64_t* out_len,
              uint64_t* out_tokens) {
  grm_store_handle* h = grm_store_create_mla("RefDriverArena", 1, 2048, 576, 0, 512, 64);
  if (!h) return -1;
  int rc = grm_store_configure_arena(h, sink, width);
  if (rc == 0) {
    std::vector<uint64_t> ids;
    rc = grm_store_commit_mount(h, ids.data(), 0, old_mount_tokens);
  }
  if (rc == 0) {
    const uint64_t old_shape[3] = {outer, input_tokens, inner};
    const uint64_t mount_shape[3] = {outer, mount_tokens, inner};
    uint64_t out_shape[3] = {0, 0, 0};
    grm_arena_swap_plan_c plan;
    rc = grm_store_apply_swap_tensor(
        h, mount_tokens, input_tokens, old_shape, 3, 1, elem_size, old_payload,
        outer * input_tokens * inner * elem_size, mount_shape, 3, mount_payload,
        outer * mount_tokens * inner * elem_size, out_shape, 3, out, out_cap, out_len, &plan);
    *out_tokens = out_shape[1];
  }
  grm_store_destroy(h);
  return rc;
}

const char* refd_last_error(grm_store_handle* h) { return grm_store_last_error(h); }

void refd_destroy(grm_store_handle* h) { grm_store_destroy(h); }

}  // extern "C"
