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
constexpr int kThreads = 128;          // 32 tokens x 4 threads
constexpr int kTok = kThreads / 4;
constexpr int kMlpFloats = kHid * kIn + kHid + kHid * kHid + kHid + kHid + 1;
// shared-memory layout (floats): padded rows keep the four threads of a token
// on distinct banks
constexpr int kW1Stride = 16;
constexpr int kW2Stride = 132;
constexpr int kH1Stride = 132;
constexpr int kOffW1 = 0;
constexpr int kOffB1 = kOffW1 + kHid * kW1Stride;
constexpr int kOffW2 = kOffB1 + kHid;
constexpr int kOffB2 = kOffW2 + kHid * kW2Stride;
constexpr int kOffW3 = kOffB2 + kHid;
constexpr int kOffB3 = kOffW3 + kHid;
constexpr int kOffH1 = kOffB3 + 4;
constexpr int kOffX = kOffH1 + kTok * kH1Stride;
constexpr int kOffHs = kOffX + kTok * 16;
constexpr int kMaxHkv = 16;
constexpr int kSmemFloats = kOffHs + kTok * kMaxHkv;

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
  extern __shared__ float sm[];
  {
    const float* w1 = p.mlp;
    const float* b1 = w1 + kHid * kIn;
    const float* w2 = b1 + kHid;
    const float* b2 = w2 + kHid * kHid;
    const float* w3 = b2 + kHid;
    for (int i = threadIdx.x; i < kHid * kIn; i += blockDim.x)
      sm[kOffW1 + (i / kIn) * kW1Stride + (i % kIn)] = w1[i];
    for (int i = threadIdx.x; i < kHid * kHid; i += blockDim.x)
      sm[kOffW2 + (i / kHid) * kW2Stride + (i % kHid)] = w2[i];
    for (int i = threadIdx.x; i < kHid; i += blockDim.x) {
      sm[kOffB1 + i] = b1[i];
      sm[kOffB2 + i] = b2[i];
      sm[kOffW3 + i] = w3[i];
    }
    if (threadIdx.x == 0) sm[kOffB3] = w3[kHid];
  }
  __syncthreads();
  const int tl = threadIdx.x >> 2;  // token within the group
  const int part = threadIdx.x & 3;
  const long long ngroups = ((long long)p.B * p.L + kTok - 1) / kTok;
  for (long long grp = blockIdx.x; grp < ngroups; grp += gridDim.x) {
  const long long gi = grp * kTok + tl;
  const bool active = gi < (long long)p.B * p.L;
  const int b = active ? (int)(gi / p.L) : 0;
  const int i = active ? (int)(gi % p.L) : 0;
  float* hs = sm + kOffHs + tl * kMaxHkv;
  float* xs = sm + kOffX + tl * 16;

  // ---- a_value: bf16-rounded |v_h|^2 per head, heads split over the 4 threads ----
  if (active) {
    for (int h = part; h < p.Hkv; h += 4) {
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
      hs[h] = bf16_round(s);
    }
  }
  __syncwarp();
  if (active && part == 0) {
    // auxiliary features (features.py:886-921), heads summed in order
    const long long pos = p.positions[gi];
    const int T = p.original_length;
    if (pos < 0 || pos >= T) record_error(p.status, CORE_ERR_INVALID_ARG, 601, i);
    const float age_den = log1pf((float)(T - 1 > 1 ? T - 1 : 1));
    const float a_age = log1pf((float)(T - 1 - pos)) / age_den;
    bool sink = pos < p.n_sink;
    if (p.special != nullptr && p.special[gi]) sink = true;
    float hsum = 0.f;
    for (int h = 0; h < p.Hkv; ++h) hsum += hs[h];
    const float vmean = bf16_round(hsum / (float)p.Hkv);
    const float a_value = bf16_round(log1pf(bf16_round(vmean / 128.0f)));
    float* f = p.features + gi * kIn;
    f[10] = a_age;
    f[11] = sink ? 1.0f : 0.0f;
    f[12] = a_value;
    f[13] = p.is_prefill ? 0.0f : 1.0f;
    bool finite = true;
    for (int k = 0; k < kIn; ++k) {
      xs[k] = f[k];
      finite &= isfinite(xs[k]);
    }
    if (!finite) record_error(p.status, CORE_ERR_NONFINITE, 602, i);
  }
  __syncwarp();
  // ---- layer 1: this thread's hidden units o = 4 j + part ----
  float x[kIn];
#pragma unroll
  for (int k = 0; k < kIn; ++k) x[k] = xs[k];
  float* h1 = sm + kOffH1 + tl * kH1Stride;
  for (int j = 0; j < kHid / 4; ++j) {
    const int o = 4 * j + part;
    const float* w = sm + kOffW1 + o * kW1Stride;
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < kIn; ++k) acc = fmaf(w[k], x[k], acc);
    h1[o] = gelu(acc + sm[kOffB1 + o]);
  }
  __syncwarp();
  // ---- layer 2 (four outputs at a time) and the output unit ----
  float out = 0.f;
  const float4* h4 = reinterpret_cast<const float4*>(h1);
  for (int j = 0; j < kHid / 4; j += 4) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int k = 0; k < kHid / 4; ++k) {
      const float4 hv = h4[k];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int o = 4 * (j + u) + part;
        const float4 w = reinterpret_cast<const float4*>(sm + kOffW2 + o * kW2Stride)[k];
        acc[u] = fmaf(w.x, hv.x, acc[u]);
        acc[u] = fmaf(w.y, hv.y, acc[u]);
        acc[u] = fmaf(w.z, hv.z, acc[u]);
        acc[u] = fmaf(w.w, hv.w, acc[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int o = 4 * (j + u) + part;
      out = fmaf(sm[kOffW3 + o], gelu(acc[u] + sm[kOffB2 + o]), out);
    }
  }
  out += __shfl_xor_sync(0xffffffffu, out, 1);
  out += __shfl_xor_sync(0xffffffffu, out, 2);
  if (active && part == 0) p.scores[gi] = out + sm[kOffB3];
  __syncwarp();
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
  long long blocks = (n + kTok - 1) / kTok;
  if (blocks > 2LL * sm_count()) blocks = 2LL * sm_count();
  indexer_scores_kernel<<<(unsigned)blocks, kThreads, smem, s>>>(p);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "indexer_scores_kernel launch");
  return CORE_OK;
}
