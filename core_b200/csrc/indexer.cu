// Auxiliary features and the indexer MLP (replaces core/features.py:861-921,
// the feature concatenation at core/kvpress_adapter.py:536 and
// COREIndexerMLP, core/indexer.py:88-108).
//
// One thread per cached token.  The auxiliary features follow the
// reference's dtype: for bf16 caches a_value is computed with the same
// bf16 roundings as the reference's torch ops (squares, per-head sums, the
// head mean, /d and log1p each round to bf16).  The MLP runs in f32 with its
// weights in shared memory (exact erf GELU).
#include <cmath>

#include "common.cuh"
#include "host_util.h"

namespace core {
namespace idx {

constexpr int kIn = 14;
constexpr int kHid = 128;
constexpr int kThreads = 128;
constexpr int kMlpFloats = kHid * kIn + kHid + kHid * kHid + kHid + kHid + 1;

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

__global__ void __launch_bounds__(kThreads)
    indexer_scores_kernel(const Params p) {
  extern __shared__ float sw[];
  for (int i = threadIdx.x; i < kMlpFloats; i += blockDim.x) sw[i] = p.mlp[i];
  __syncthreads();
  const float* w1 = sw;
  const float* b1 = w1 + kHid * kIn;
  const float* w2 = b1 + kHid;
  const float* b2 = w2 + kHid * kHid;
  const float* w3 = b2 + kHid;
  const float b3 = w3[kHid];

  const long long gi = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (gi >= (long long)p.B * p.L) return;
  const int b = (int)(gi / p.L);
  const int i = (int)(gi % p.L);
  float* f = p.features + gi * kIn;

  // ---- auxiliary features (features.py:886-921) ----
  const long long pos = p.positions[gi];
  const int T = p.original_length;
  if (pos < 0 || pos >= T) record_error(p.status, CORE_ERR_INVALID_ARG, 601, i);
  const float age_den = log1pf((float)(T - 1 > 1 ? T - 1 : 1));
  const float a_age = log1pf((float)(T - 1 - pos)) / age_den;
  bool sink = pos < p.n_sink;
  if (p.special != nullptr && p.special[gi]) sink = true;
  // a_value = log1p(mean_h |v_h|^2 / d) with bf16 rounding at each torch op
  float hsum = 0.f;
  for (int h = 0; h < p.Hkv; ++h) {
    const uint4* row = reinterpret_cast<const uint4*>(p.v + (((long long)b * p.Hkv + h) * p.L + i) * 128);
    float s = 0.f;
#pragma unroll 4
    for (int c = 0; c < 16; ++c) {
      const uint4 w = row[c];
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 x = __bfloat1622float2(h2[e]);
        s += bf16_round(x.x * x.x);
        s += bf16_round(x.y * x.y);
      }
    }
    hsum += bf16_round(s);
  }
  const float vmean = bf16_round(hsum / (float)p.Hkv);
  const float a_value = bf16_round(log1pf(bf16_round(vmean / 128.0f)));
  f[10] = a_age;
  f[11] = sink ? 1.0f : 0.0f;
  f[12] = a_value;
  f[13] = p.is_prefill ? 0.0f : 1.0f;

  float x[kIn];
#pragma unroll
  for (int k = 0; k < kIn; ++k) x[k] = f[k];
  bool finite = true;
#pragma unroll
  for (int k = 0; k < kIn; ++k) finite &= isfinite(x[k]);
  if (!finite) record_error(p.status, CORE_ERR_NONFINITE, 602, i);

  // ---- MLP 14 -> 128 -> 128 -> 1 ----
  float h1[kHid];
#pragma unroll
  for (int o = 0; o < kHid; ++o) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < kIn; ++k) acc = fmaf(w1[o * kIn + k], x[k], acc);
    h1[o] = gelu(acc + b1[o]);
  }
  float out = 0.f;
  for (int o = 0; o < kHid; ++o) {
    const float4* wr = reinterpret_cast<const float4*>(w2 + o * kHid);
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < kHid / 4; ++k) {
      const float4 w = wr[k];
      acc = fmaf(w.x, h1[4 * k], acc);
      acc = fmaf(w.y, h1[4 * k + 1], acc);
      acc = fmaf(w.z, h1[4 * k + 2], acc);
      acc = fmaf(w.w, h1[4 * k + 3], acc);
    }
    out = fmaf(w3[o], gelu(acc + b2[o]), out);
  }
  p.scores[gi] = out + b3;
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
  if (original_length < d->seq_len)
    return set_error(CORE_ERR_INVALID_ARG, "core_indexer_scores: original_length < seq_len");
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
  const size_t smem = sizeof(float) * kMlpFloats;
  cudaError_t e =
      cudaFuncSetAttribute(indexer_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_error(e, "indexer_scores_kernel attribute");
  const long long n = (long long)p.B * p.L;
  indexer_scores_kernel<<<(unsigned)((n + kThreads - 1) / kThreads), kThreads, smem, s>>>(p);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "indexer_scores_kernel launch");
  return CORE_OK;
}
