// One layer's complete compression step behind a single entry point
// (replaces COREMemoryPress.compress, core/kvpress_adapter.py:968-1210):
// QK features -> coverage -> auxiliary + indexer MLP -> Top-B -> memory write
// -> retained-KV gather, all enqueued on one stream.
#include "common.cuh"
#include "host_util.h"

namespace core {
int qk_features_impl(const core_dims_t* d, const void* q, const void* k, int32_t topk_qk,
                     int32_t n_recent_queries, const float* lse_in, float* lse_out,
                     float* features, int32_t feature_stride, void* workspace,
                     size_t workspace_bytes, void* stream, void* ev0, void* ev1,
                     uint32_t* summary = nullptr);
int indexer_scores_split(const core_dims_t* d, const void* v, const int64_t* positions,
                         const uint8_t* special, int32_t original_length, int32_t is_prefill,
                         int32_t n_sink, float* features, const float* mlp, float* scores,
                         void* workspace, size_t workspace_bytes, void* stream);
}

using namespace core;

static core_dims_t kv_dims(const core_dims_t* d) {
  core_dims_t e = *d;
  e.n_queries = 0;
  return e;
}

extern "C" size_t core_compress_layer_workspace_bytes(const core_dims_t* d, int32_t n_kept,
                                                      int32_t d_mem) {
  if (check_dims(d, "core_compress_layer_workspace_bytes", true) != CORE_OK) return 0;
  size_t ws = core_qk_features_workspace_bytes(d);
  core_dims_t e = kv_dims(d);
  size_t c = core_coverage_workspace_bytes(&e);
  if (c > ws) ws = c;
  const size_t hs = sizeof(float) * (size_t)d->batch * d->seq_len * d->n_kv_heads + 256;
  if (hs > ws) ws = hs;  // per-head value sums of the indexer
  const int n_evict = d->seq_len - n_kept;
  if (d_mem > 0 && n_evict > 0) {
    size_t m = core_memory_write_workspace_bytes(&e, n_evict, d_mem);
    if (m > ws) ws = m;
  }
  return ws;
}

extern "C" int core_compress_layer(const core_dims_t* d, const void* q, const void* k,
                                   const void* v, const int64_t* positions, const uint8_t* special,
                                   const float* lse_in, const core_layer_weights_t* w,
                                   const core_compress_args_t* a, float* features, float* scores,
                                   int32_t* keep_idx, int32_t* evict_idx, float* M, float* b_state,
                                   float* Z, void* out_k, void* out_v, void* workspace,
                                   size_t workspace_bytes, void* stream, void* ev_begin,
                                   void* ev_end) {
  int rc = check_dims(d, "core_compress_layer", true);
  if (rc != CORE_OK) return rc;
  if (w == nullptr || a == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_compress_layer: NULL weights or args");
  const int L = d->seq_len;
  if (a->n_kept <= 0 || a->n_kept > L)
    return set_error(CORE_ERR_INVALID_ARG, "core_compress_layer: bad n_kept");
  core_dims_t e = kv_dims(d);
  if ((rc = qk_features_impl(d, q, k, a->topk_qk, a->n_recent_queries, lse_in, nullptr, features,
                             14, workspace, workspace_bytes, stream, ev_begin, ev_end)) != CORE_OK)
    return rc;
  if ((rc = core_coverage_features(&e, k, w->geometry_ext, w->prototypes, a->shrinkage_rho,
                                   features, 14, 6, workspace, workspace_bytes, stream)) != CORE_OK)
    return rc;
  if ((rc = indexer_scores_split(&e, v, positions, special, a->original_length, a->is_prefill,
                                 a->n_sink, features, w->mlp, scores, workspace, workspace_bytes,
                                 stream)) != CORE_OK)
    return rc;
  if (a->n_kept >= L) return CORE_OK;  // nothing to evict: the caller keeps the cache
  if ((rc = core_topb_select(scores, d->batch, L, a->n_kept, a->n_sink, keep_idx, evict_idx,
                             nullptr, 0, stream)) != CORE_OK)
    return rc;
  if (w->theta_split != nullptr && M != nullptr) {
    if ((rc = core_memory_write(&e, k, v, scores, evict_idx, L - a->n_kept, w->theta_split,
                                w->d_mem, a->gamma, a->eta, a->student_temp, M, b_state, Z,
                                workspace, workspace_bytes, stream)) != CORE_OK)
      return rc;
  }
  return core_compact_kv(&e, k, v, keep_idx, a->n_kept, out_k, out_v, stream);
}
