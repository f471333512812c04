// Auxiliary features and the indexer MLP (replaces core/features.py:861-921,
// the feature concatenation at core/kvpress_adapter.py:536 and
// COREIndexerMLP, core/indexer.py:88-108).
//
// Four threads per cached token, persistent blocks.  The auxiliary features
// follow the reference's dtype: for bf16 caches a_value is computed with the
// same bf16 roundings as the reference's torch ops (squares, per-head sums,
// the head mean, /d and log1p each round to bf16).  The MLP runs in f32 with
// its weights staged once per block into shared memory (cp.async) and read as
// broadcasts: hidden unit k of layer 1 is computed, GELU'd, and immediately
// accumulated into the 128 layer-2 outputs held in registers, a quarter per
// thread (an outer-product form, so layer-2 sums run over k in ascending order).
#include <cmath>

#include "common.cuh"
#include "host_util.h"

namespace core {
namespace idx {

constexpr int kIn = 14;
constexpr int kHid = 128;
constexpr int kThreads = 256;  // 64 tokens x 4 threads
// packed global layout (floats): [w1 (128,14) | b1 | w2^T (in 128, out 128) | b2 | w3 | b3]
constexpr int kGW1 = 0;
constexpr int kGB1 = kGW1 + kHid * kIn;    // 1792
constexpr int kGW2T = kGB1 + kHid;         // 1920 (16-byte aligned)
constexpr int kGB3 = kGW2T + kHid * kHid + 2 * kHid;
// shared layout (floats): w1 rows padded to 16 | b1 | w2^T | b2 | w3 | b3
constexpr int kW1Stride = 16;
constexpr int kOffW1 = 0;
constexpr int kOffB1 = kOffW1 + kHid * kW1Stride;  // 2048
constexpr int kOffW2T = kOffB1 + kHid;             // 2176 (16-byte aligned)
constexpr int kOffB2 = kOffW2T + kHid * kHid;
constexpr int kOffW3 = kOffB2 + kHid;
constexpr int kOffB3 = kOffW3 + kHid;
constexpr int kSmemFloats = kOffB3 + 4;
constexpr int kMaxHkv = 16;
static_assert(kGW2T % 4 == 0 && kOffW2T % 4 == 0, "cp.async chunks need 16-byte alignment");

__device__ __forceinline__ float gelu(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

struct Params {
  int B, Hkv, L, original_length, is_prefill, n_sink;
  const __nv_bfloat16* v;
  const int64_t* positions;
  const uint8_t* special;
  float* features;
  const float* mlp;
  float* scores;
  DeviceStatus* status;
};

__global__ void __launch_bounds__(kThreads, 2)
    indexer_scores_kernel(const Params p) {
  extern __shared__ __align__(16) float sm[];
  // w2^T | b2 | w3 are contiguous in both layouts: one asynchronous copy
  cp_async_block(sm + kOffW2T, p.mlp + kGW2T, (kHid * kHid + 2 * kHid) / 4);
  {
    static_assert(kHid * kIn % kThreads == 0 && kHid <= kThreads, "staging layout");
    float r[kHid * kIn / kThreads + 1];
#pragma unroll
    for (int j = 0; j < kHid * kIn / kThreads; ++j) r[j] = p.mlp[kGW1 + threadIdx.x + j * kThreads];
    if (threadIdx.x < kHid) r[kHid * kIn / kThreads] = p.mlp[kGB1 + threadIdx.x];
#pragma unroll
    for (int j = 0; j < kHid * kIn / kThreads; ++j) {
      const int i = threadIdx.x + j * kThreads;
      sm[kOffW1 + (i / kIn) * kW1Stride + (i % kIn)] = r[j];
    }
    if (threadIdx.x < kHid) sm[kOffB1 + threadIdx.x] = r[kHid * kIn / kThreads];
    if (threadIdx.x == 0) sm[kOffB3] = p.mlp[kGB3];
  }
  cp_async_wait_all();
  __syncthreads();

  const long long n = (long long)p.B * p.L;
  const float age_den = log1pf((float)(p.original_length - 1 > 1 ? p.original_length - 1 : 1));
  const int part = threadIdx.x & 3;       // this thread's quarter of the token's work
  const int lane = threadIdx.x & 31;
  const int qbase = lane & ~3;            // lane of part 0 of this token
  for (long long gi = ((long long)blockIdx.x * kThreads + threadIdx.x) >> 2; ;
       gi += (long long)gridDim.x * (kThreads / 4)) {
    const long long g0 = gi - (threadIdx.x >> 2);  // first token of this block's group
    if (g0 >= n) break;
    const bool active = gi < n;
    float x[kIn];
    // ---- a_value: heads part, part + 4, ... summed here, combined in head order ----
    float hs[kMaxHkv / 4];
    const int b = active ? (int)(gi / p.L) : 0;
    const int i = active ? (int)(gi % p.L) : 0;
#pragma unroll
    for (int r = 0; r < kMaxHkv / 4; ++r) {
      hs[r] = 0.f;
      const int h = 4 * r + part;
      if (active && h < p.Hkv) {
        const uint4* row =
            reinterpret_cast<const uint4*>(p.v + (((long long)b * p.Hkv + h) * p.L + i) * 128);
        float s = 0.f;
#pragma unroll 4
        for (int c = 0; c < 16; ++c) {
          const uint4 w = __ldg(row + c);
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 t = __bfloat1622float2(h2[e]);
            s += bf16_round(t.x * t.x);
            s += bf16_round(t.y * t.y);
          }
        }
        hs[r] = bf16_round(s);
      }
    }
    float hsum = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxHkv / 4; ++r) {
#pragma unroll
      for (int pp = 0; pp < 4; ++pp) {
        const float t = __shfl_sync(0xffffffffu, hs[r], qbase | pp);
        if (4 * r + pp < p.Hkv) hsum += t;
      }
    }
    if (active) {
      // ---- auxiliary features (features.py:886-921) ----
      const long long pos = p.positions[gi];
      const int T = p.original_length;
      if (part == 0 && (pos < 0 || pos >= T)) record_error(p.status, CORE_ERR_INVALID_ARG, 601, i);
      const float a_age = log1pf((float)(T - 1 - pos)) / age_den;
      bool sink = pos < p.n_sink;
      if (p.special != nullptr && p.special[gi]) sink = true;
      const float vmean = bf16_round(hsum / (float)p.Hkv);
      const float a_value = bf16_round(log1pf(bf16_round(vmean / 128.0f)));
      float* f = p.features + gi * kIn;
#pragma unroll
      for (int k = 0; k < 10; ++k) x[k] = f[k];
      x[10] = a_age;
      x[11] = sink ? 1.0f : 0.0f;
      x[12] = a_value;
      x[13] = p.is_prefill ? 0.0f : 1.0f;
      if (part == 0) {
#pragma unroll
        for (int k = 10; k < kIn; ++k) f[k] = x[k];
        bool finite = true;
#pragma unroll
        for (int k = 0; k < kIn; ++k) finite &= isfinite(x[k]);
        if (!finite) record_error(p.status, CORE_ERR_NONFINITE, 602, i);
      }
    } else {
#pragma unroll
      for (int k = 0; k < kIn; ++k) x[k] = 0.f;
    }
    // ---- MLP.  Hidden unit k = 4 j + pp is computed by part pp and shared by
    // shuffle; this thread accumulates outputs o = 16 c + 4 part + e (c < 8,
    // e < 4) over k in ascending order. ----
    float acc[kHid / 4];
#pragma unroll
    for (int o = 0; o < kHid / 4; ++o) acc[o] = 0.f;
#pragma unroll 1
    for (int j = 0; j < kHid / 4; ++j) {
      const int kown = 4 * j + part;
      const float4* w1 = reinterpret_cast<const float4*>(sm + kOffW1 + kown * kW1Stride);
      const float4 a0 = w1[0], a1 = w1[1], a2 = w1[2], a3 = w1[3];
      float t = 0.f;
      t = fmaf(a0.x, x[0], t);
      t = fmaf(a0.y, x[1], t);
      t = fmaf(a0.z, x[2], t);
      t = fmaf(a0.w, x[3], t);
      t = fmaf(a1.x, x[4], t);
      t = fmaf(a1.y, x[5], t);
      t = fmaf(a1.z, x[6], t);
      t = fmaf(a1.w, x[7], t);
      t = fmaf(a2.x, x[8], t);
      t = fmaf(a2.y, x[9], t);
      t = fmaf(a2.z, x[10], t);
      t = fmaf(a2.w, x[11], t);
      t = fmaf(a3.x, x[12], t);
      t = fmaf(a3.y, x[13], t);
      const float hown = gelu(t + sm[kOffB1 + kown]);
#pragma unroll
      for (int pp = 0; pp < 4; ++pp) {
        const float hk = __shfl_sync(0xffffffffu, hown, qbase | pp);
        const float4* w2 = reinterpret_cast<const float4*>(sm + kOffW2T + (4 * j + pp) * kHid) + part;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 w = w2[4 * c];
          acc[4 * c] = fmaf(w.x, hk, acc[4 * c]);
          acc[4 * c + 1] = fmaf(w.y, hk, acc[4 * c + 1]);
          acc[4 * c + 2] = fmaf(w.z, hk, acc[4 * c + 2]);
          acc[4 * c + 3] = fmaf(w.w, hk, acc[4 * c + 3]);
        }
      }
    }
    float out = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int o = 16 * c + 4 * part + e;
        out = fmaf(sm[kOffW3 + o], gelu(acc[4 * c + e] + sm[kOffB2 + o]), out);
      }
    }
    out += __shfl_xor_sync(0xffffffffu, out, 1);
    out += __shfl_xor_sync(0xffffffffu, out, 2);
    if (active && part == 0) p.scores[gi] = out + sm[kOffB3];
  }
}

}  // namespace idx
}  // namespace core

using namespace core;
using namespace core::idx;

extern "C" int core_indexer_scores(const core_dims_t* d, const void* v, const int64_t* positions,
                                   const uint8_t* special, int32_t original_length,
                                   int32_t is_prefill, int32_t n_sink, float* features,
                                   const float* mlp, float* scores, void* stream) {
  int rc = check_dims(d, "core_indexer_scores");
  if (rc != CORE_OK) return rc;
  if (v == nullptr || positions == nullptr || features == nullptr || mlp == nullptr ||
      scores == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_indexer_scores: NULL tensor");
  if (reinterpret_cast<uintptr_t>(mlp) % 16 != 0)
    return set_error(CORE_ERR_INVALID_ARG, "core_indexer_scores: mlp must be 16-byte aligned");
  if (original_length < d->seq_len)
    return set_error(CORE_ERR_INVALID_ARG, "core_indexer_scores: original_length < seq_len");
  if (d->n_kv_heads > kMaxHkv)
    return set_error(CORE_ERR_UNSUPPORTED, "core_indexer_scores: at most 16 KV heads");
  Params p{};
  p.B = d->batch;
  p.Hkv = d->n_kv_heads;
  p.L = d->seq_len;
  p.original_length = original_length;
  p.is_prefill = is_prefill;
  p.n_sink = n_sink;
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.positions = positions;
  p.special = special;
  p.features = features;
  p.mlp = mlp;
  p.scores = scores;
  p.status = device_status();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t smem = sizeof(float) * kSmemFloats;
  cudaError_t e =
      cudaFuncSetAttribute(indexer_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_error(e, "indexer_scores_kernel attribute");
  const long long n = (long long)p.B * p.L;
  long long blocks = (n + kThreads / 4 - 1) / (kThreads / 4);
  if (blocks > 2LL * sm_count()) blocks = 2LL * sm_count();
  indexer_scores_kernel<<<(unsigned)blocks, kThreads, smem, s>>>(p);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "indexer_scores_kernel launch");
  return CORE_OK;
}
