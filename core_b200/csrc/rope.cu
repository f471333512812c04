// Post-RoPE query reconstruction for the decode-time compression and the
// memory readout (replaces the tail of
// BackboneStatsCollector._recompute_post_rope_queries, core/collector.py:163-192:
// transformers' LlamaRotaryEmbedding.forward followed by apply_rotary_pos_emb).
//
// The q_proj GEMM stays a library call (cuBLAS through torch); this kernel
// takes its output, rotates every head and writes the (B, Hq, T, d) layout the
// QK kernels read, in one pass.  Roundings follow the torch ops it replaces:
//   angle = f32(inv_freq[j] * f32(pos))            (a K = 1 matmul: one rounding)
//   c = T(cosf(angle) * scaling), s = T(sinf(angle) * scaling)
//   out[j]      = T( T(x1 * c) + T(-x2 * s) )      (rotate_half = cat(-x2, x1))
//   out[j + d/2] = T( T(x2 * c) + T( x1 * s) )
// where T() rounds to the query dtype (bf16, fp16, or none for f32), and
// every product and sum is a separately rounded f32 operation (no FMA).
// When the caller passes the cos / sin tensors a model computed (the
// position_embeddings of its forward), they are used instead.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "common.cuh"
#include "host_util.h"

namespace core {
namespace rope {

template <typename T>
struct Round;
template <>
struct Round<__nv_bfloat16> {
  static __device__ __forceinline__ float f(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
  static __device__ __forceinline__ float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float x) { *p = __float2bfloat16_rn(x); }
};
template <>
struct Round<__half> {
  static __device__ __forceinline__ float f(float x) { return __half2float(__float2half_rn(x)); }
  static __device__ __forceinline__ float load(const __half* p) { return __half2float(*p); }
  static __device__ __forceinline__ void store(__half* p, float x) { *p = __float2half_rn(x); }
};
template <>
struct Round<float> {
  static __device__ __forceinline__ float f(float x) { return x; }
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ void store(float* p, float x) { *p = x; }
};

// One thread per rotation pair (j, j + d/2) of one (b, t): it computes (or
// reads) that pair's cos / sin once and rotates the pair in every head.
constexpr int kThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kThreads)
    rope_queries_kernel(int B, int Tn, int Hq, int d, const T* __restrict__ qp, long long row_stride,
                        const int64_t* __restrict__ pos, const float* __restrict__ inv_freq,
                        float scaling, const T* __restrict__ cosv, const T* __restrict__ sinv,
                        int cs_batch, T* __restrict__ out) {
  const int half = d >> 1;
  const long long n_pairs = (long long)B * Tn * half;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n_pairs;
       i += (long long)gridDim.x * blockDim.x) {
    const int j = (int)(i % half);
    const long long bt = i / half;
    const int t = (int)(bt % Tn);
    const int b = (int)(bt / Tn);
    float c, s;
    if (cosv != nullptr) {
      const long long cb = (cs_batch == 1) ? 0 : b;
      const long long ci = (cb * Tn + t) * d + j;
      c = Round<T>::load(cosv + ci);
      s = Round<T>::load(sinv + ci);
    } else {
      const float angle = __fmul_rn(inv_freq[j], (float)pos[bt]);
      c = Round<T>::f(__fmul_rn(cosf(angle), scaling));
      s = Round<T>::f(__fmul_rn(sinf(angle), scaling));
    }
    const T* src = qp + bt * row_stride;
    for (int h = 0; h < Hq; ++h) {
      const float x1 = Round<T>::load(src + (long long)h * d + j);
      const float x2 = Round<T>::load(src + (long long)h * d + j + half);
      const float lo = Round<T>::f(__fadd_rn(Round<T>::f(__fmul_rn(x1, c)),
                                             Round<T>::f(__fmul_rn(-x2, s))));
      const float hi = Round<T>::f(__fadd_rn(Round<T>::f(__fmul_rn(x2, c)),
                                             Round<T>::f(__fmul_rn(x1, s))));
      T* dst = out + (((long long)b * Hq + h) * Tn + t) * d;
      Round<T>::store(dst + j, lo);
      Round<T>::store(dst + j + half, hi);
    }
  }
}

template <typename T>
int launch(int B, int Tn, int Hq, int d, const void* qp, long long row_stride, const int64_t* pos,
           const float* inv_freq, float scaling, const void* cosv, const void* sinv, int cs_batch,
           void* out, cudaStream_t st) {
  const long long n_pairs = (long long)B * Tn * (d / 2);
  const int blocks = (int)((n_pairs + kThreads - 1) / kThreads);
  rope_queries_kernel<T><<<blocks, kThreads, 0, st>>>(
      B, Tn, Hq, d, static_cast<const T*>(qp), row_stride, pos, inv_freq, scaling,
      static_cast<const T*>(cosv), static_cast<const T*>(sinv), cs_batch, static_cast<T*>(out));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CORE_OK : cuda_error(e, "rope_queries_kernel launch");
}

}  // namespace rope
}  // namespace core

extern "C" int core_rope_queries(int32_t batch, int32_t n_tokens, int32_t n_q_heads,
                                 int32_t head_dim, int32_t dtype, const void* q_proj,
                                 int64_t row_stride, const int64_t* positions,
                                 const float* inv_freq, float attention_scaling, const void* cos,
                                 const void* sin, int32_t cos_batch, void* q_out, void* stream) {
  using namespace core;
  if (batch < 1 || n_tokens < 0 || n_q_heads < 1 || head_dim < 2 || (head_dim & 1))
    return set_error(CORE_ERR_INVALID_ARG, "core_rope_queries: bad shape");
  if (n_tokens == 0) return CORE_OK;
  if (row_stride < (int64_t)n_q_heads * head_dim)
    return set_error(CORE_ERR_INVALID_ARG, "core_rope_queries: row_stride below Hq*head_dim");
  if (q_proj == nullptr || q_out == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_rope_queries: NULL tensor");
  const bool given = cos != nullptr || sin != nullptr;
  if (given) {
    if (cos == nullptr || sin == nullptr || (cos_batch != 1 && cos_batch != batch))
      return set_error(CORE_ERR_INVALID_ARG,
                       "core_rope_queries: cos and sin must both be given, batch 1 or B");
  } else if (positions == nullptr || inv_freq == nullptr) {
    return set_error(CORE_ERR_INVALID_ARG,
                     "core_rope_queries: positions and inv_freq are required without cos/sin");
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case CORE_DTYPE_BF16:
      return rope::launch<__nv_bfloat16>(batch, n_tokens, n_q_heads, head_dim, q_proj, row_stride,
                                         positions, inv_freq, attention_scaling, cos, sin,
                                         cos_batch, q_out, st);
    case CORE_DTYPE_F16:
      return rope::launch<__half>(batch, n_tokens, n_q_heads, head_dim, q_proj, row_stride,
                                  positions, inv_freq, attention_scaling, cos, sin, cos_batch,
                                  q_out, st);
    case CORE_DTYPE_F32:
      return rope::launch<float>(batch, n_tokens, n_q_heads, head_dim, q_proj, row_stride,
                                 positions, inv_freq, attention_scaling, cos, sin, cos_batch,
                                 q_out, st);
    default:
      return set_error(CORE_ERR_INVALID_ARG, "core_rope_queries: dtype must be bf16, f16 or f32");
  }
}
