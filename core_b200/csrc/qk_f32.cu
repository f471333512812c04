// QK features of f32 caches on CUDA cores (the reference's fp32 path:
// core/features.py:425-632 and core/fused_qk.py with logits left unrounded).
//
//   lse_f32_kernel      : causal row log-sum-exp per (q-head, query), online over
//                         64-key tiles, 4 x 4 register-blocked f32 FMAs.
//   relation_f32_kernel : the relation values R of 64 keys x one 128-query
//                         block, summed over the KV group's q-heads, reduced to
//                         the same 64-byte per-key records as the bf16
//                         tensor-core kernels, so qk_merge_kernel and
//                         qk_f6_resolve_kernel finish f1..f6 unchanged.
// Dot products run over d in ascending order with fmaf; exp and log are the
// accurate library functions.
#include <cmath>

#include "common.cuh"
#include "host_util.h"
#include "qk_common.cuh"

namespace core {
namespace qkf {

using qk::kLogFloor;
using qk::kRecWords;
using qk::logaddexp_floor;
using qk::relation_offset;

constexpr int kD = 128;
constexpr int kThreads = 256;
constexpr int kPad = kD + 1;  // padded row stride (floats): column reads hit distinct banks

// ---------------------------------------------------------------------------
// LSE: block = (64 queries, q-head, batch row); thread (rq = tid / 16, rk = tid % 16)
// owns queries 4 rq + i and keys rk + 16 j (i, j < 4) of every 64-key tile.
// ---------------------------------------------------------------------------
constexpr int kLseQ = 64;
constexpr int kLseK = 64;
constexpr size_t kLseSmem = sizeof(float) * (size_t)(kLseQ + kLseK) * kPad;

__global__ void __launch_bounds__(kThreads)
    lse_f32_kernel(const float* __restrict__ q, const float* __restrict__ k, int Hq, int Hkv,
                   int nq, int L, int q_start, float scale, float* __restrict__ lse) {
  extern __shared__ float sm[];
  float* sQ = sm;                   // [64][kPad]
  float* sK = sm + kLseQ * kPad;    // [64][kPad]
  const int qh = blockIdx.y, b = blockIdx.z;
  const int h = qh / (Hq / Hkv);
  const int t0 = blockIdx.x * kLseQ;
  const int tid = threadIdx.x, rq = tid >> 4, rk = tid & 15;
  const float* qb = q + (long long)(b * Hq + qh) * nq * kD;
  const float* kb = k + (long long)(b * Hkv + h) * L * kD;
  for (int i = tid; i < kLseQ * kD; i += kThreads) {
    const int r = i / kD, e = i % kD;
    sQ[r * kPad + e] = (t0 + r < nq) ? qb[(long long)(t0 + r) * kD + e] : 0.f;
  }
  // keys any query of the block can see: [0, min(L, q_start + last query + 1))
  const long long last_q = (long long)q_start + min(t0 + kLseQ, nq) - 1;
  const int kend = (int)min((long long)L, last_q + 1);
  float m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
  }
  for (int k0 = 0; k0 < kend; k0 += kLseK) {
    __syncthreads();
    for (int i = tid; i < kLseK * kD; i += kThreads) {
      const int r = i / kD, e = i % kD;
      sK[r * kPad + e] = (k0 + r < L) ? kb[(long long)(k0 + r) * kD + e] : 0.f;
    }
    __syncthreads();
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
#pragma unroll 4
    for (int e = 0; e < kD; ++e) {
      float qv[4], kv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qv[i] = sQ[(4 * rq + i) * kPad + e];
#pragma unroll
      for (int j = 0; j < 4; ++j) kv[j] = sK[(rk + 16 * j) * kPad + e];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(qv[i], kv[j], acc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = t0 + 4 * rq + i;
      const long long qpos = (long long)q_start + t;
      float tmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = k0 + rk + 16 * j;
        const bool vis = t < nq && key < L && key <= qpos;
        acc[i][j] = vis ? acc[i][j] * scale : -INFINITY;
        tmax = fmaxf(tmax, acc[i][j]);
      }
      // the 16 threads holding this query's keys are lanes 16 (rq & 1) + [0, 16)
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      const float nm = fmaxf(m[i], tmax);
      const float base = (nm == -INFINITY) ? 0.f : nm;
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) s += expf(acc[i][j] - base);
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (nm != -INFINITY) {
        l[i] = l[i] * expf(m[i] - nm) + s;
        m[i] = nm;
      }
    }
  }
  if (rk == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = t0 + 4 * rq + i;
      if (t < nq)
        lse[(long long)(b * Hq + qh) * nq + t] = (m[i] == -INFINITY) ? -INFINITY : m[i] + logf(l[i]);
    }
  }
}

// ---------------------------------------------------------------------------
// Relation: block = (64 keys, KV head, 128-query block, batch row); thread
// (key kk = tid / 4, quarter qq = tid % 4) owns queries 32 qq .. 32 qq + 31 of
// the block: the 32 relation values of one record word.
// ---------------------------------------------------------------------------
constexpr int kRelK = 64;
constexpr int kRelQ = 128;
constexpr int kQuarter = 36;  // padded quarter of a transposed query row: quarters on distinct banks
constexpr size_t kRelSmem =
    sizeof(float) * ((size_t)kRelK * kPad + (size_t)kD * 4 * kQuarter + 2 * kRelQ);

struct RelParams {
  int B, Hq, Hkv, G, nq, L, q_start, n_qb, head_topk, n_recent;
  float scale;
  const float* q;    // (B, Hq, nq, d)
  const float* k;    // (B, Hkv, L, d)
  const float* lse;  // (B, Hq, nq)
  uint32_t* rec;     // (B, L, Hkv, n_qb, 16)
};

__device__ __forceinline__ void merge_top4(float (&t)[4], int off) {
  float o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = __shfl_xor_sync(0xffffffffu, t[i], off);
#pragma unroll
  for (int i = 0; i < 4; ++i) top4_insert(t, o[i]);
}

__global__ void __launch_bounds__(kThreads)
    relation_f32_kernel(const RelParams p) {
  extern __shared__ float sm[];
  float* sK = sm;                               // [64][kPad]
  float* sQT = sK + kRelK * kPad;               // [d][4][kQuarter]: q of the head, transposed
  float* s_nc = sQT + kD * 4 * kQuarter;        // [128] -lse + log|C_t| of the head's queries
  const int k0 = blockIdx.x * kRelK;
  const int h = blockIdx.y % p.Hkv, qb = blockIdx.y / p.Hkv;
  const int b = blockIdx.z;
  const int tid = threadIdx.x, kk = tid >> 2, qq = tid & 3;
  const int key = k0 + kk;
  const float* kb = p.k + (long long)(b * p.Hkv + h) * p.L * kD;
  for (int i = tid; i < kRelK * kD; i += kThreads) {
    const int r = i / kD, e = i % kD;
    sK[r * kPad + e] = (k0 + r < p.L) ? kb[(long long)(k0 + r) * kD + e] : 0.f;
  }
  const int tq0 = qb * kRelQ;               // first query of the block
  const int qvalid = min(kRelQ, p.nq - tq0);
  const float single_val = log1pf(expf(kLogFloor));
  float acc[32], mn[32];
  for (int g = 0; g < p.G; ++g) {
    const int qh = h * p.G + g;
    __syncthreads();  // the previous head's readers of sQT are done
    const float* qsrc = p.q + ((long long)(b * p.Hq + qh) * p.nq + tq0) * kD;
    for (int i = tid; i < kRelQ * kD; i += kThreads) {
      const int t = i / kD, e = i % kD;
      sQT[(e * 4 + (t >> 5)) * kQuarter + (t & 31)] = (t < qvalid) ? qsrc[(long long)t * kD + e] : 0.f;
    }
    for (int t = tid; t < kRelQ; t += kThreads) {
      const long long qpos = (long long)p.q_start + tq0 + t;
      const long long cc = (qpos + 1 < p.L) ? qpos + 1 : p.L;
      s_nc[t] = (t < qvalid) ? relation_offset(p.lse[(long long)(b * p.Hq + qh) * p.nq + tq0 + t], cc)
                             : 0.f;
    }
    __syncthreads();
    float dot[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) dot[j] = 0.f;
#pragma unroll 2
    for (int e = 0; e < kD; ++e) {
      const float kv = sK[kk * kPad + e];
      const float4* qr = reinterpret_cast<const float4*>(sQT + (e * 4 + qq) * kQuarter);
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const float4 v = qr[w];
        dot[4 * w] = fmaf(kv, v.x, dot[4 * w]);
        dot[4 * w + 1] = fmaf(kv, v.y, dot[4 * w + 1]);
        dot[4 * w + 2] = fmaf(kv, v.z, dot[4 * w + 2]);
        dot[4 * w + 3] = fmaf(kv, v.w, dot[4 * w + 3]);
      }
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int t = qq * 32 + j;
      const long long qpos = (long long)p.q_start + tq0 + t;
      const float r = fmaf(dot[j], p.scale, s_nc[t]);
      float rel = logaddexp_floor(r);
      if (key > qpos) rel = kLogFloor;
      else if (qpos == 0) rel = single_val;
      acc[j] = (g == 0) ? rel : acc[j] + rel;
      mn[j] = (g == 0) ? rel : fminf(mn[j], rel);
    }
  }
  // ---- per-key statistics over this thread's 32 queries ----
  float top[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  float rtop[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  float psum = 0.f, mxnp = -INFINITY, nsum = 0.f;
  uint32_t word = 0;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int t = qq * 32 + j;
    const long long qpos = (long long)p.q_start + tq0 + t;
    float R = (p.head_topk < p.G) ? __fdiv_rn(acc[j] - mn[j], (float)p.head_topk)
                                  : __fdiv_rn(acc[j], (float)p.head_topk);
    if (t >= qvalid || key > qpos) R = -INFINITY;
    top4_insert(top, R);
    if (tq0 + t >= p.nq - p.n_recent) top4_insert(rtop, R);
    const bool pz = R > 0.f;
    psum += fmaxf(R, 0.f);
    if (R > -INFINITY) nsum += fminf(R, 0.f);  // masked entries are not queries
    word |= (pz ? 1u : 0u) << j;
    mxnp = fmaxf(mxnp, pz ? -INFINITY : R);
  }
  // ---- the key's four quarters: lanes 4 kk + [0, 4) ----
  merge_top4(top, 1);
  merge_top4(top, 2);
  merge_top4(rtop, 1);
  merge_top4(rtop, 2);
  psum += __shfl_xor_sync(0xffffffffu, psum, 1);
  psum += __shfl_xor_sync(0xffffffffu, psum, 2);
  nsum += __shfl_xor_sync(0xffffffffu, nsum, 1);
  nsum += __shfl_xor_sync(0xffffffffu, nsum, 2);
  mxnp = fmaxf(mxnp, __shfl_xor_sync(0xffffffffu, mxnp, 1));
  mxnp = fmaxf(mxnp, __shfl_xor_sync(0xffffffffu, mxnp, 2));
  uint32_t cnt = __popc(word);
  cnt += __shfl_xor_sync(0xffffffffu, cnt, 1);
  cnt += __shfl_xor_sync(0xffffffffu, cnt, 2);
  if (key < p.L) {
    uint32_t* dst = p.rec + ((((long long)b * p.L + key) * p.Hkv + h) * p.n_qb + qb) * kRecWords;
    dst[10 + qq] = word;
    if (qq == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        dst[i] = __float_as_uint(top[i]);
        dst[4 + i] = __float_as_uint(rtop[i]);
      }
      dst[8] = __float_as_uint(psum);
      dst[9] = cnt;
      dst[14] = __float_as_uint(mxnp);
      dst[15] = __float_as_uint(nsum);
    }
  }
}

}  // namespace qkf
}  // namespace core

namespace core {

// LSE (unless the caller supplied it) and the per-key records of f32 caches;
// the caller runs qk_merge_kernel and qk_f6_resolve_kernel on the records.
int qk_f32_records(const core_dims_t* d, int q_start, int n_qb, int head_topk, int n_recent,
                   float scale, const float* q, const float* k, bool run_lse, float* lse,
                   uint32_t* rec, cudaStream_t s) {
  using namespace qkf;
  const int B = d->batch, Hq = d->n_q_heads, Hkv = d->n_kv_heads, nq = d->n_queries,
            L = d->seq_len;
  cudaError_t e;
  if (run_lse) {
    e = cudaFuncSetAttribute(lse_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kLseSmem);
    if (e != cudaSuccess) return cuda_error(e, "lse_f32_kernel attribute");
    lse_f32_kernel<<<dim3((nq + kLseQ - 1) / kLseQ, Hq, B), kThreads, kLseSmem, s>>>(
        q, k, Hq, Hkv, nq, L, q_start, scale, lse);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "lse_f32_kernel launch");
  }
  RelParams p{};
  p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.G = Hq / Hkv; p.nq = nq; p.L = L; p.q_start = q_start;
  p.n_qb = n_qb; p.head_topk = head_topk; p.n_recent = n_recent; p.scale = scale;
  p.q = q; p.k = k; p.lse = lse; p.rec = rec;
  e = cudaFuncSetAttribute(relation_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kRelSmem);
  if (e != cudaSuccess) return cuda_error(e, "relation_f32_kernel attribute");
  relation_f32_kernel<<<dim3((L + kRelK - 1) / kRelK, Hkv * n_qb, B), kThreads, kRelSmem, s>>>(p);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "relation_f32_kernel launch");
  return CORE_OK;
}

}  // namespace core
