/*
 * core_b200.h -- C ABI of the B200 (sm_100a) implementation of CORE's
 * KV-compression step (the `core_full` press) and its latent-memory readout.
 *
 * Every entry point:
 *   - takes plain device pointers, sizes and a cudaStream_t (passed as void*);
 *   - is asynchronous on that stream and allocates nothing: scratch memory is
 *     a caller-provided workspace whose size the matching *_workspace_bytes
 *     query returns;
 *   - returns an int status (CORE_OK = 0, negative on error).  A readable
 *     message for the last error of the calling thread is available from
 *     core_last_error().  Device-side failures (a bounded wait that gave up, a
 *     non-finite feature) are recorded in a device status word that
 *     core_check_device_status() reads back (it synchronises the stream).
 *
 * Tensor layouts are those of the reference press (HF DynamicCache layers):
 *   Q  : (B, Hq, nq, d)    post-RoPE queries of the query buffer
 *   K,V: (B, Hkv, L, d)    cached keys / values
 * with d = 128 and Hq = G * Hkv, G <= 4.  dims.dtype names the element type
 * of Q, K and V.  CORE_DTYPE_BF16 runs the contractions on tcgen05 and rounds
 * where the reference's bf16 tensor ops round (logits, the a_value steps, the
 * readout residual).  CORE_DTYPE_F32 (the reference's fp32 path) runs them on
 * CUDA cores in f32 without those roundings.
 *
 * The reference is pure Python; each entry point below names the reference
 * function (file:line in the reference project) whose behaviour it replaces.
 */
#ifndef CORE_B200_H_
#define CORE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define CORE_OK 0
#define CORE_ERR_INVALID_ARG (-1)
#define CORE_ERR_UNSUPPORTED (-2)
#define CORE_ERR_NONFINITE (-3)
#define CORE_ERR_TIMEOUT (-4)
#define CORE_ERR_CUDA (-5)
#define CORE_ERR_WORKSPACE (-6)

/* ---- dtypes ---- */
#define CORE_DTYPE_BF16 1
#define CORE_DTYPE_F32 2
#define CORE_DTYPE_F16 3 /* core_rope_queries and core_compact_kv only */

typedef struct core_dims {
  int32_t batch;      /* B   */
  int32_t n_q_heads;  /* Hq  */
  int32_t n_kv_heads; /* Hkv */
  int32_t head_dim;   /* d (must be 128) */
  int32_t n_queries;  /* nq: buffered queries, the last nq cache positions */
  int32_t seq_len;    /* L: cached tokens */
  int32_t dtype;      /* CORE_DTYPE_* of Q, K, V */
} core_dims_t;

/* Library version (major*10000 + minor*100 + patch). */
int core_version(void);

/* Caps the number of SMs the persistent grids plan for (0: all SMs), so that
 * kernels of another stream can run beside them; process-wide, read when a
 * call plans its launch (workspace sizes depend on it: query them under the
 * same budget).  A scheduling setting with no counterpart in the reference. */
int core_set_sm_budget(int32_t n_sms);

/* Copies the last error message of the calling host thread into buf. */
int core_last_error(char* buf, size_t buf_len);

/* Reads and clears the device status word written by the kernels; returns
 * CORE_OK or the first recorded CORE_ERR_* code.  Synchronises `stream`. */
int core_check_device_status(void* stream);

/* ---------------------------------------------------------------------------
 * QK relation features f1..f6 and causal row LSE.
 * Replaces strict_causal_qk_features (core/fused_qk.py:373-587) including its
 * kernels _causal_row_lse_kernel (:26-107), _grouped_relation_tile_kernel
 * (:110-230), _basic_relation_stats_kernel (:233-292) and the top-k
 * reductions (:527-582).
 *   q          : (B, Hq, nq, d)
 *   k          : (B, Hkv, L, d)
 *   lse_in     : optional (B, Hq, nq) f32 external row LSE (FlashAttention's
 *                softmax_lse); when non-NULL the LSE pass is skipped (:444-456)
 *   lse_out    : optional (B, Hq, nq) f32
 *   features   : (B, L, feature_stride) f32, columns 0..5 receive f1..f6
 * ------------------------------------------------------------------------- */
size_t core_qk_features_workspace_bytes(const core_dims_t* dims);
int core_qk_features(const core_dims_t* dims, const void* q, const void* k,
                     int32_t topk_qk, int32_t n_recent_queries, const float* lse_in,
                     float* lse_out, float* features, int32_t feature_stride,
                     void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Coverage features o, d_proto, delta_proto, g.
 * Replaces COREFeatureExtractor.compute_coverage_features
 * (core/features.py:790-858) with LayerwiseKeyGeometryProjector.forward
 * (:53-77), PrototypeBank.get_coverage_features (:146-213) and
 * HadamardProjector.rotate (:259-261).
 *   geometry_ext : (3, 128, Hkv*d) bf16 from core_prepare_geometry
 *   prototypes   : (64, P) f32 unit rows, 16-byte aligned
 *   features     : (B, L, feature_stride) f32, columns col0..col0+3
 * P (proto_dim) must be 64 and the prototype count 64.
 * ------------------------------------------------------------------------- */
size_t core_coverage_workspace_bytes(const core_dims_t* dims);
int core_coverage_features(const core_dims_t* dims, const void* k, const void* geometry_ext,
                           const float* prototypes, float shrinkage_rho, float* features,
                           int32_t feature_stride, int32_t col0, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Once per layer: geometry_ext = three bf16 terms of [W ; R W], where W is the
 * layer's (64, in_dim) f32 Gaussian projection (core/features.py:29-50) and R
 * the (64, 64) Hadamard rotation (:216-236), so that one tensor-core pass
 * yields both the projected key and its rotation.  No reference counterpart
 * (the reference multiplies by W and R separately in f32). */
int core_prepare_geometry(const float* geometry, const float* hadamard, int32_t in_dim,
                          void* geometry_ext, void* stream);

/* ---------------------------------------------------------------------------
 * Auxiliary features + indexer MLP -> per-token scores.
 * Replaces compute_auxiliary_features (core/features.py:861-921), the
 * feature concatenation (core/kvpress_adapter.py:536) and COREIndexerMLP
 * (core/indexer.py:88-108, 14 -> 128 -> 128 -> 1, exact GELU).
 *   v          : (B, Hkv, L, d)
 *   positions  : (B, L) int64 original token positions of the cache slots
 *   special    : optional (B, L) uint8, 1 where the token id is a special id
 *   features   : (B, L, 14) f32; columns 0..9 already hold f1..f6 and the
 *                coverage features; columns 10..13 are written here
 *   mlp        : a prepared indexer MLP (core_prepare_indexer_mlp), 16-byte
 *                aligned; an unprepared buffer fails with CORE_ERR_INVALID_ARG
 *                (device status site 612) and leaves scores unwritten
 *   scores     : (B, L) f32
 * ------------------------------------------------------------------------- */
/* Bytes of a prepared indexer MLP buffer (173056). */
size_t core_indexer_mlp_bytes(void);
/* Prepare an indexer MLP in place.  `mlp` (16-byte aligned, device memory,
 * core_indexer_mlp_bytes() bytes) holds in its first 18561 floats
 *   [w1 (128 out,14 in) | b1 (128) | w2 transposed (128 in,128 out) | b2 (128) |
 *    w3 (128) | b3 (1)];
 * this writes, behind them at byte 74752, layer 2's weights split into three
 * bf16 terms (w = t0 + t1 + t2 to f32 precision) in the swizzled K-major
 * layout of a tensor-core operand, and a tag the scoring kernels check.  Done
 * once per set of weights (the reference's COREIndexerMLP parameters,
 * core/indexer.py:88-108); no reference counterpart as a call. */
int core_prepare_indexer_mlp(float* mlp, void* stream);
int core_indexer_scores(const core_dims_t* dims, const void* v, const int64_t* positions,
                        const uint8_t* special, int32_t original_length, int32_t is_prefill,
                        int32_t n_sink, float* features, const float* mlp, float* scores,
                        void* stream);

/* ---------------------------------------------------------------------------
 * Top-B selection with sink protection.
 * Replaces the sink saturation of COREScorerPress.score
 * (core/kvpress_adapter.py:773-778) and the pooled stable descending argsort,
 * truncation and chronological re-sort of COREMemoryPress.compress (:1017-1025).
 *   scores    : (B, L) f32 calibrated scores
 *   keep_idx  : (B, n_kept) int32, ascending
 *   evict_idx : (B, L - n_kept) int32, ascending
 * Ties are broken toward the lower index (stable sort).
 * ------------------------------------------------------------------------- */
size_t core_topb_workspace_bytes(int32_t batch, int32_t seq_len);
int core_topb_select(const float* scores, int32_t batch, int32_t seq_len, int32_t n_kept,
                     int32_t n_sink, int32_t* keep_idx, int32_t* evict_idx, void* workspace,
                     size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Latent-memory write and decayed recurrence (pre_o_proj value space).
 * Replaces core/kvpress_adapter.py:1041-1202 (student_distribution,
 * conditional_evicted_weights, phi = K Theta_f^T, M_bar, b_bar, and the
 * Z/M/b recurrence).
 *   scores_cal  : (B, L) f32 calibrated (unsaturated) scores
 *   evict_idx   : (B, n_evict) int32 from core_topb_select
 *   theta_split : bf16 caches: (2, d_mem, Hkv*d) bf16 hi/lo of the
 *                 group-folded Theta; f32 caches: that Theta itself,
 *                 (d_mem, Hkv*d) f32
 *   M           : (B, d_mem, Hkv*d) f32, updated in place
 *   b_state     : (B, d_mem) f32, updated in place
 *   Z           : (B,) f32, updated in place (0 for a fresh layer)
 * d_mem must be a multiple of 128 (<= 512).
 * ------------------------------------------------------------------------- */
size_t core_memory_write_workspace_bytes(const core_dims_t* dims, int32_t n_evict, int32_t d_mem);
int core_memory_write(const core_dims_t* dims, const void* k, const void* v,
                      const float* scores_cal, const int32_t* evict_idx, int32_t n_evict,
                      const void* theta_split, int32_t d_mem, float gamma, float eta,
                      float student_temp, float* M, float* b_state, float* Z, void* workspace,
                      size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Retained-KV gather.  Replaces keys.gather / values.gather
 * (core/kvpress_adapter.py:1204-1210).  out_k / out_v: (B, Hkv, n_kept, d).
 * ------------------------------------------------------------------------- */
int core_compact_kv(const core_dims_t* dims, const void* k, const void* v,
                    const int32_t* keep_idx, int32_t n_kept, void* out_k, void* out_v,
                    void* stream);

/* ---------------------------------------------------------------------------
 * Gated latent-memory readout added to the attention output.
 * Replaces MemoryModule.readout (core/indexer.py:165-207) and the folded
 * o_proj projection of COREMemoryPress.apply_memory_readout
 * (core/kvpress_adapter.py:1302-1352).
 *   q        : (B, Hq, q_len, d) post-RoPE queries (dims.dtype: CORE_DTYPE_BF16,
 *              _F16 or _F32)
 *   theta    : (d_mem, Hq*d) f32;  gate_w1 : (gh, Hq*d) f32; gate_b1 : (gh)
 *   gate_w2  : (gh) f32; gate_b2 : scalar f32 (pointer)
 *   M, b     : layer fast state (B, d_mem, Hkv*d), (B, d_mem) f32
 *   o_fold   : (hidden, Hkv*d) f32 group-folded o_proj
 *   attn_out : (B, q_len, hidden) of dims.dtype, updated in place (bf16 and
 *              fp16: the residual and the o_proj product are rounded to that
 *              dtype before the sum, as the reference's .to(dtype) casts)
 * gate_override NaN uses the learned gate; any finite value is the constant
 * gate (MemoryModule.readout's gate_override, negative values included);
 * infinities are rejected.
 * Any alignment is accepted; 16-byte aligned theta, gate_w1, M and o_fold
 * (and q aligned to 8 bytes for 16-bit types, 16 for f32) take the faster kernels.
 * ------------------------------------------------------------------------- */
size_t core_memory_readout_workspace_bytes(const core_dims_t* dims, int32_t q_len,
                                           int32_t d_mem, int32_t gate_hidden);
int core_memory_readout(const core_dims_t* dims, int32_t q_len, const void* q, const float* theta,
                        const float* gate_w1, const float* gate_b1, const float* gate_w2,
                        const float* gate_b2, int32_t d_mem, int32_t gate_hidden,
                        float gate_override, const float* M, const float* b_state,
                        const float* o_fold, int32_t hidden, void* attn_out, void* workspace,
                        size_t workspace_bytes, void* stream);

/* core_memory_readout without a caller workspace: no counterpart in the
 * reference.  Same arguments and result as core_memory_readout; its scratch is
 * a 256 KB static device array (no cudaMalloc or other allocation), so
 * B * q_len * (d_mem + gate_hidden + Hkv*d) floats, each of the three parts
 * rounded up to 256 bytes, must fit in 256 KB; larger calls return
 * CORE_ERR_INVALID_ARG.  The first call on a device, with that device current,
 * resolves the scratch address (cudaGetSymbolAddress) and should precede any
 * stream capture.  The resolved address is kept for the life of the process:
 * it does not survive cudaDeviceReset or a re-created primary context.  Nothing in the scratch needs to start at zero.  There is one
 * scratch per device: calls that overlap on one device (other streams or host
 * threads) race on it and must be serialised by the caller. */
int core_memory_readout_noalloc(const core_dims_t* dims, int32_t q_len, const void* q,
                                const float* theta, const float* gate_w1, const float* gate_b1,
                                const float* gate_w2, const float* gate_b2, int32_t d_mem,
                                int32_t gate_hidden, float gate_override, const float* M,
                                const float* b_state, const float* o_fold, int32_t hidden,
                                void* attn_out, void* stream);

/* ---------------------------------------------------------------------------
 * One layer's complete compression step.
 * Replaces COREMemoryPress.compress (core/kvpress_adapter.py:968-1210) with
 * the scores of COREScorerPress.score (:690-797): the QK, coverage and
 * auxiliary features, the indexer MLP, Top-B with sinks, the memory write
 * (when theta_split and M are non-NULL) and the retained-KV gather.
 *   features  : (B, L, 14) f32 out;  scores : (B, L) f32 out (calibrated)
 *   keep_idx  : (B, n_kept) int32 out;  evict_idx : (B, L - n_kept) int32 out
 *   out_k/v   : (B, Hkv, n_kept, d) out
 * When n_kept >= L only features and scores are produced.  ev_begin/ev_end,
 * when non-NULL, are cudaEvent_t recorded around the QK relation kernel.
 * ------------------------------------------------------------------------- */
typedef struct core_layer_weights {
  const void* geometry_ext;   /* (3, 128, Hkv*d) bf16 from core_prepare_geometry */
  const float* prototypes;    /* (64, 64) f32 */
  const float* mlp;           /* prepared indexer MLP (core_prepare_indexer_mlp) */
  const void* theta_split;    /* as core_memory_write's (by dims.dtype), or NULL: no write */
  int32_t d_mem;
} core_layer_weights_t;

typedef struct core_compress_args {
  int32_t n_kept;
  int32_t n_sink;
  int32_t topk_qk;
  int32_t n_recent_queries;
  float shrinkage_rho;
  int32_t original_length;
  int32_t is_prefill;
  float gamma;
  float eta;
  float student_temp;
} core_compress_args_t;

size_t core_compress_layer_workspace_bytes(const core_dims_t* dims, int32_t n_kept, int32_t d_mem);
int core_compress_layer(const core_dims_t* dims, const void* q, const void* k, const void* v,
                        const int64_t* positions, const uint8_t* special, const float* lse_in,
                        const core_layer_weights_t* weights, const core_compress_args_t* args,
                        float* features, float* scores, int32_t* keep_idx, int32_t* evict_idx,
                        float* M, float* b_state, float* Z, void* out_k, void* out_v,
                        void* workspace, size_t workspace_bytes, void* stream, void* ev_begin,
                        void* ev_end);

/* ---------------------------------------------------------------------------
 * Weight preparation: split an f32 array into `terms` (2 or 3) bf16 arrays
 * whose sum reproduces it (hi = bf16(x), mid = bf16(x - hi), lo = ...).
 * Used once per layer for the geometry projection and the folded Theta.
 * No reference counterpart (the reference multiplies in f32 directly).
 * ------------------------------------------------------------------------- */
int core_split_bf16(const float* src, int64_t n, int32_t terms, void* dst, void* stream);

/* ---------------------------------------------------------------------------
 * Self-test of the device-side bounded wait (no reference counterpart): one
 * warp waits, for limit_us microseconds (1 us .. 1 s), on an mbarrier that
 * nothing completes, using the wait every pipelined kernel uses; the wait
 * gives up and records CORE_ERR_TIMEOUT, which core_check_device_status then
 * returns (and clears).  The kernel itself ends normally.
 * ------------------------------------------------------------------------- */
int core_selftest_wait_timeout(int32_t limit_us, void* stream);

/* ===========================================================================
 * Head-sharded caches: one sequence whose KV heads are split across ranks
 * (one process per GPU).  The reference runs one process with all heads; these
 * entry points are its per-layer functions split at their cross-head
 * reductions, which the caller performs between the calls with NCCL:
 *   rank r holds KV heads [r*Hkv/N, (r+1)*Hkv/N) and their query heads, and
 *   finishes the features and scores of keys [r*Lc, min(L, (r+1)*Lc)),
 *   Lc = ceil(L/N).  All are bf16-only and take dims with batch 1 and the
 *   rank's own head counts, unless noted.
 * ======================================================================== */

/* Words per per-key QK summary for n_queries buffered queries (a multiple
 * of 4). */
int32_t core_qk_summary_words(int32_t n_queries);

/* strict_causal_qk_features (core/fused_qk.py:373-587) over this rank's heads,
 * stopped before the cross-head reduction: per key, the top-4 and recent top-4
 * relation values, positive sum and count, the count of heads whose f6 test
 * is positive, and the positive-query bits (OR over the heads).
 *   summary : (L, core_qk_summary_words(nq)) uint32, 16-byte aligned
 *   lse_out : optional (Hq_rank, nq) f32
 * Workspace: core_qk_features_workspace_bytes(dims). */
int core_qk_head_summary(const core_dims_t* dims, const void* q, const void* k, int32_t topk_qk,
                         int32_t n_recent_queries, float* lse_out, uint32_t* summary,
                         void* workspace, size_t workspace_bytes, void* stream);

/* The cross-head reduction of core/fused_qk.py:505-582 for keys
 * key0 .. key0 + n_keys - 1: parts = (n_parts, part_rows, words) summaries
 * of those keys from every rank (row i = key key0 + i), n_kv_heads the total
 * head count; writes f1..f6 to features[i * feature_stride + 0..5]. */
int core_qk_merge_summaries(const uint32_t* parts, int32_t n_parts, int64_t part_rows,
                            int32_t key0, int32_t n_keys, int32_t seq_len, int32_t n_queries,
                            int32_t n_kv_heads, int32_t topk_qk, int32_t n_recent_queries,
                            float* features, int32_t feature_stride, void* stream);

/* LayerwiseKeyGeometryProjector.forward (core/features.py:53-77) before the
 * head concatenation is complete: y = sum over this rank's heads of
 * W_h k_h / (|k_h| + eps), (L, 64) f32, 16-byte aligned.  geometry_ext holds
 * only this rank's columns, (3, 128, Hkv_rank*d) from core_prepare_geometry.
 * Workspace: core_coverage_workspace_bytes(dims). */
int core_coverage_partial_projection(const core_dims_t* dims, const void* k,
                                     const void* geometry_ext, float* y, void* workspace,
                                     size_t workspace_bytes, void* stream);

/* The rest of compute_coverage_features (core/features.py:790-858) for the
 * n_keys keys of a range, in three calls with two sums across ranks between
 * them.  range_totals: z = y / (|y| + eps) for the summed y, zt = R z
 * (HadamardProjector.rotate, :259-261; hadamard (64, 64) f32), and this
 * range's column sums of z, zt, zt^2 as totals (192) f64.  range_assign:
 * the statistics of the summed totals over all seq_len keys (mean z, mu,
 * sigma2_eff), prototype assignment, d_proto, delta_proto and g, and this
 * range's assignment histogram hist (64) int32.  range_occupancy: o from the
 * summed histogram.  Workspace: core_coverage_range_workspace_bytes(n_keys). */
size_t core_coverage_range_workspace_bytes(int32_t n_keys);
int core_coverage_range_totals(const float* y, int32_t n_keys, const float* hadamard, float* z,
                               float* zt, double* totals, void* workspace,
                               size_t workspace_bytes, void* stream);
int core_coverage_range_assign(const double* totals, int32_t seq_len, float shrinkage_rho,
                               const float* z, const float* zt, int32_t n_keys,
                               const float* prototypes, int32_t* assign, int32_t* hist,
                               float* features, int32_t feature_stride, int32_t col0,
                               void* workspace, size_t workspace_bytes, void* stream);
int core_coverage_range_occupancy(const int32_t* assign, const int32_t* hist, int32_t n_keys,
                                  float* features, int32_t feature_stride, int32_t col0,
                                  void* stream);

/* The per-head sums of compute_auxiliary_features' a_value
 * (core/features.py:914-915) in the bf16 arithmetic of core_indexer_scores:
 * out[h * out_stride + token] for this rank's heads. */
int core_value_head_sums(const core_dims_t* dims, const void* v, float* out, int64_t out_stride,
                         void* stream);

/* core_indexer_scores for n_keys keys of one sequence, with the values'
 * per-head sums (all n_kv_heads heads, head_sums[h * hs_stride + i] for key
 * i of the range) in place of V; positions, special, features (n_keys, 14)
 * and scores (n_keys) start at the range's first key. */
int core_indexer_scores_from_sums(int32_t n_kv_heads, int32_t n_keys, const float* head_sums,
                                  int64_t hs_stride, const int64_t* positions,
                                  const uint8_t* special, int32_t original_length,
                                  int32_t is_prefill, int32_t n_sink, float* features,
                                  const float* mlp, float* scores, void* stream);

/* core_memory_write on rows already gathered: k_ev, v_ev = (B, Hkv, n_evict,
 * d) hold the evicted rows in evict_idx order (all heads, e.g. collected on
 * the rank that owns the layer's memory state); evict_idx still indexes
 * scores_cal (B, seq_len).  Same workspace as core_memory_write. */
int core_memory_write_gathered(const core_dims_t* dims, const void* k_ev, const void* v_ev,
                               const float* scores_cal, const int32_t* evict_idx, int32_t n_evict,
                               const void* theta_split, int32_t d_mem, float gamma, float eta,
                               float student_temp, float* M, float* b_state, float* Z,
                               void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Post-RoPE queries of buffered hidden states.
 * Replaces the rotary part of BackboneStatsCollector._recompute_post_rope_queries
 * (core/collector.py:163-192): transformers' LlamaRotaryEmbedding.forward and
 * apply_rotary_pos_emb, fused with the transpose to the QK kernels' layout.
 * The q_proj GEMM before it is the caller's (a library GEMM).
 *   q_proj    : (B, T, Hq*head_dim) rows of `dtype` (CORE_DTYPE_BF16, _F16 or
 *               _F32), row r at q_proj + r * row_stride elements
 *   positions : (B, T) int64 absolute positions   } used when cos/sin are NULL:
 *   inv_freq  : (head_dim/2) f32                  } angle = inv_freq[j] * pos,
 *               c = dtype(cosf(angle) * attention_scaling), likewise s
 *   cos, sin  : (cos_batch, T, head_dim) of `dtype`, a model's precomputed
 *               position embeddings (cos_batch 1 or B), or NULL
 *   q_out     : (B, Hq, T, head_dim) of `dtype`
 * Every product and sum rounds to `dtype` as the torch ops do.
 * ------------------------------------------------------------------------- */
int core_rope_queries(int32_t batch, int32_t n_tokens, int32_t n_q_heads, int32_t head_dim,
                      int32_t dtype, const void* q_proj, int64_t row_stride,
                      const int64_t* positions, const float* inv_freq, float attention_scaling,
                      const void* cos, const void* sin, int32_t cos_batch, void* q_out,
                      void* stream);

/* ---------------------------------------------------------------------------
 * Causal prefill attention that also returns the row log-sum-exp.
 * Replaces the flash_attn_func call of _core_flash_attention_forward
 * (core/kvpress_pipeline.py:24-91: causal, no dropout, return_attn_probs for
 * softmax_lse only), whose LSE the press reuses as the QK relation pass's row
 * normaliser (core/kvpress_adapter.py:400-438; core/fused_qk.py:444-456):
 * pass `lse` to core_qk_features as lse_in.
 *   dims      : batch, n_q_heads, n_kv_heads, head_dim = 128,
 *               n_queries = Lq, seq_len = Lk (Lq <= Lk), dtype CORE_DTYPE_BF16
 *               or CORE_DTYPE_F16
 *   q         : (B, Hq, Lq, d) with element strides q_strides = {b, h, t};
 *   k, v      : (B, Hkv, Lk, d) likewise; d contiguous, every stride a
 *               multiple of 8 elements, base pointers 16-byte aligned
 *   out       : (B, Lq, Hq, d) contiguous, dims.dtype (the layout
 *               flash_attn_func returns)
 *   lse       : (B, Hq, Lq) f32, natural log of sum_k exp(scale * q.k) over
 *               the keys the row sees (FlashAttention's softmax_lse)
 * Query row i sees keys 0 .. i + Lk - Lq (the bottom-right causal mask of
 * FlashAttention 2).  Scores in f32 from 16-bit inputs, P rounded to dims.dtype
 * for the P V product, f32 accumulation, as FlashAttention computes.
 * ------------------------------------------------------------------------- */
int core_attention_prefill(const core_dims_t* dims, const void* q, const int64_t* q_strides,
                           const void* k, const int64_t* k_strides, const void* v,
                           const int64_t* v_strides, void* out, float* lse, float softmax_scale,
                           void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CORE_B200_H_ */
