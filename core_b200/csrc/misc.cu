// Retained-KV gather (replaces core/kvpress_adapter.py:1204-1210) and the
// gated latent-memory readout (replaces core/indexer.py:165-207 and
// core/kvpress_adapter.py:1302-1352).
#include <cmath>
#include <cstdint>
#include <type_traits>
#include <cuda_fp16.h>

#include <cooperative_groups.h>

#include "common.cuh"
#include "host_util.h"

namespace core {
namespace misc {

namespace cg = cooperative_groups;
constexpr int kD = 128;

// out[b, h, j, :] = in[b, h, keep[b, j], :]; kVec lanes move one row with
// 16-byte accesses (16 for a 256-byte bf16 row, 32 for a 512-byte f32 row).
template <int kVec>
__global__ void compact_kernel(const uint4* __restrict__ k, const uint4* __restrict__ v,
                               const int* __restrict__ keep, int Hkv, int L, int n_kept,
                               uint4* __restrict__ ok, uint4* __restrict__ ov) {
  const int b = blockIdx.y;  // gridDim.y = B
  const long long per_b = (long long)Hkv * n_kept;
  for (long long r = (long long)blockIdx.x * (blockDim.x / kVec) + (threadIdx.x / kVec); r < per_b;
       r += (long long)gridDim.x * (blockDim.x / kVec)) {
    const int h = (int)(r / n_kept), j = (int)(r % n_kept);
    const int src = keep[(long long)b * n_kept + j];
    const int q = threadIdx.x % kVec;
    const long long si = (((long long)b * Hkv + h) * L + src) * kVec + q;
    const long long di = (((long long)b * Hkv + h) * n_kept + j) * kVec + q;
    ok[di] = k[si];
    ov[di] = v[si];
  }
}

__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float f16_round(float x) { return __half2float(__float2half_rn(x)); }
// out += residual product, in the attention output's dtype: the product is
// rounded to that dtype first, then the sum (reference: .to(dtype) then +)
__device__ __forceinline__ __nv_bfloat16 add_out(__nv_bfloat16 a, float r) {
  return __float2bfloat16_rn(__bfloat162float(a) + bf16_round(r));
}
__device__ __forceinline__ __half add_out(__half a, float r) {
  return __float2half_rn(__half2float(a) + f16_round(r));
}
__device__ __forceinline__ float add_out(float a, float r) { return a + r; }

// Rounding of the gated residual to the attention output's dtype before the
// o_proj product (kvpress_adapter.py:1320: residual.to(output[0].dtype)).
enum RoundMode { kRoundNone = 0, kRoundBf16 = 1, kRoundF16 = 2 };
__device__ __forceinline__ float round_to(float x, int mode) {
  return mode == kRoundBf16 ? bf16_round(x) : mode == kRoundF16 ? f16_round(x) : x;
}
// A gate_override that is NaN selects the learned gate; any other value is
// the fixed gate, as MemoryModule.readout's torch.full_like(denom, override).
__device__ __forceinline__ bool learned_gate(float gate_override) { return gate_override != gate_override; }

__device__ __forceinline__ float gelu(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

// Stage 1: proj = Theta q (d_mem rows) and gate pre-activations W1 q + c1 (gh
// rows).  Two warps per weight row (each half of the row, all of its loads in
// flight at once), the halves added in order; all q_len queries per row.
constexpr int kProjWarps = 8;  // 4 rows per block

template <typename T>
__global__ void __launch_bounds__(kProjWarps * 32)
    readout_proj_kernel(const T* __restrict__ q, int Hq, int q_len,
                        const float* __restrict__ theta, const float* __restrict__ gw1,
                        const float* __restrict__ gb1, int d_mem, int gh,
                        float* __restrict__ proj, float* __restrict__ gpre) {
  extern __shared__ float sq[];  // (q_len, Hq*d) f32 of this batch row
  __shared__ float s_half[kProjWarps];
  const int b = blockIdx.y;
  const int dm = Hq * kD;
  for (int i = threadIdx.x; i < q_len * dm; i += blockDim.x) {
    const int t = i / dm, c = i % dm;
    const int qh = c / kD, e = c % kD;
    sq[i] = to_f32(q[(((long long)b * Hq + qh) * q_len + t) * kD + e]);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = warp & 1;
  const int half_len = dm / 2;  // a multiple of 128 (dm = Hq * 128, Hq even)
  for (int r0 = blockIdx.x * (kProjWarps / 2); r0 < d_mem + gh; r0 += gridDim.x * (kProjWarps / 2)) {
    const int r = r0 + (warp >> 1);
    const bool live = r < d_mem + gh;
    const float* w = !live ? theta
                     : (r < d_mem) ? theta + (long long)r * dm : gw1 + (long long)(r - d_mem) * dm;
    for (int t = 0; t < q_len; ++t) {
      const float* x = sq + t * dm + half * half_len;
      const float* wh = w + half * half_len;
      float acc = 0.f;
      if (live) {
#pragma unroll 16
        for (int c = lane * 4; c < half_len; c += 128) {
          const float4 ww = *reinterpret_cast<const float4*>(wh + c);
          acc = fmaf(ww.x, x[c], acc);
          acc = fmaf(ww.y, x[c + 1], acc);
          acc = fmaf(ww.z, x[c + 2], acc);
          acc = fmaf(ww.w, x[c + 3], acc);
        }
      }
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) s_half[warp] = acc;
      __syncthreads();
      if (live && half == 0 && lane == 0) {
        const float v = acc + s_half[warp + 1];
        if (r < d_mem) proj[((long long)b * q_len + t) * d_mem + r] = v;
        else gpre[((long long)b * q_len + t) * gh + (r - d_mem)] = v + gb1[r - d_mem];
      }
      __syncthreads();
    }
  }
}

// Stage 1 for rows that fit in registers (Hq a multiple of 4, Hq/4 <= kMaxV):
// four warps split each weight row; a lane loads its whole weight segment and
// the q elements of the same columns straight from global memory, so one
// round trip to HBM covers the block.  The four parts are added in order.
constexpr int kProjSplit = 4;          // warps per weight row
constexpr int kProjRowsPerBlock = 2;   // 8 warps

__device__ __forceinline__ float4 ldg4(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}
__device__ __forceinline__ float4 ldq4(const float* p) { return ldg4(p); }
__device__ __forceinline__ float4 ldq4(const __nv_bfloat16* p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
  const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
  return make_float4(__low2float(lo), __high2float(lo), __low2float(hi), __high2float(hi));
}
__device__ __forceinline__ float4 ldq4(const __half* p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const __half2 lo = *reinterpret_cast<const __half2*>(&u.x);
  const __half2 hi = *reinterpret_cast<const __half2*>(&u.y);
  return make_float4(__low2float(lo), __high2float(lo), __low2float(hi), __high2float(hi));
}
__device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
  acc = fmaf(a.x, b.x, acc);
  acc = fmaf(a.y, b.y, acc);
  acc = fmaf(a.z, b.z, acc);
  return fmaf(a.w, b.w, acc);
}

template <typename T, int kMaxV>
__global__ void __launch_bounds__(kProjSplit * kProjRowsPerBlock * 32)
    readout_proj_reg_kernel(const T* __restrict__ q, int Hq, int q_len,
                            const float* __restrict__ theta, const float* __restrict__ gw1,
                            const float* __restrict__ gb1, int d_mem, int gh,
                            float* __restrict__ proj, float* __restrict__ gpre) {
  __shared__ float s_part[kProjSplit * kProjRowsPerBlock];
  const int b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dm = Hq * kD, rows = d_mem + gh;
  const int r = blockIdx.x * kProjRowsPerBlock + warp / kProjSplit;
  const int part = warp % kProjSplit;
  const bool live = r < rows;
  const int nv = Hq / kProjSplit;  // float4 per lane: column part*seg + i*128 + lane*4
  const float* w = !live ? theta
                   : (r < d_mem ? theta + (long long)r * dm : gw1 + (long long)(r - d_mem) * dm);
  w += part * nv * 128 + lane * 4;
  // q head part*nv + i holds the columns of float4 i; element lane*4 of that head
  const T* qb = q + (((long long)b * Hq + part * nv) * q_len) * kD + lane * 4;
  float4 wv[kMaxV], xv[kMaxV];
#pragma unroll
  for (int i = 0; i < kMaxV; ++i) {
    const bool on = live && i < nv;
    wv[i] = on ? ldg4(w + i * 128) : make_float4(0.f, 0.f, 0.f, 0.f);
    xv[i] = on ? ldq4(qb + (long long)i * q_len * kD) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int t = 0; t < q_len; ++t) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxV; ++i) acc = dot4(wv[i], xv[i], acc);
    if (t + 1 < q_len) {
#pragma unroll
      for (int i = 0; i < kMaxV; ++i)
        if (live && i < nv) xv[i] = ldq4(qb + ((long long)i * q_len + t + 1) * kD);
    }
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    __syncthreads();  // the previous t's parts are consumed
    if (lane == 0) s_part[warp] = acc;
    __syncthreads();
    if (threadIdx.x < kProjRowsPerBlock) {
      const int rr = blockIdx.x * kProjRowsPerBlock + threadIdx.x;
      if (rr < rows) {
        float v = 0.f;
        for (int pp = 0; pp < kProjSplit; ++pp) v += s_part[threadIdx.x * kProjSplit + pp];
        if (rr < d_mem) proj[((long long)b * q_len + t) * d_mem + rr] = v;
        else gpre[((long long)b * q_len + t) * gh + (rr - d_mem)] = v + gb1[rr - d_mem];
      }
    }
  }
}

// Stage 2: m = proj M / sqrt(proj^2 . b + eps), gate, residual (rounded to
// bf16 when the attention output is bf16).
// A block covers 32 value columns (one per lane); its 8 warps split the d_mem
// rows of M and their partial sums are added in warp order.
constexpr int kMemWarps = 16;

__global__ void __launch_bounds__(kMemWarps * 32)
    readout_mem_kernel(const float* __restrict__ proj, const float* __restrict__ gpre,
                       const float* __restrict__ gw2, const float* __restrict__ gb2,
                       float gate_override, const float* __restrict__ M,
                       const float* __restrict__ bst, int q_len, int d_mem, int gh, int kvw,
                       int round_mode, float* __restrict__ res) {
  extern __shared__ float sp[];  // proj (d_mem) of this (b, t)
  __shared__ float s_den, s_g;
  __shared__ float s_part[kMemWarps][32];
  const int b = blockIdx.y, t = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* pr = proj + ((long long)b * q_len + t) * d_mem;
  for (int j = threadIdx.x; j < d_mem; j += blockDim.x) sp[j] = pr[j];
  __syncthreads();
  if (warp == 0) {
    float den = 0.f;
    for (int j = lane; j < d_mem; j += 32) den = fmaf(sp[j] * sp[j], bst[(long long)b * d_mem + j], den);
    for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    float gl = 0.f;
    for (int o = lane; o < gh; o += 32)
      gl = fmaf(gw2[o], gelu(gpre[((long long)b * q_len + t) * gh + o]), gl);
    for (int o = 16; o > 0; o >>= 1) gl += __shfl_xor_sync(0xffffffffu, gl, o);
    if (lane == 0) {
      s_den = den + 1e-8f;
      s_g = learned_gate(gate_override) ? 1.0f / (1.0f + expf(-(gl + gb2[0]))) : gate_override;
    }
  }
  const int c = blockIdx.x * 32 + lane;
  const float* Mb = M + (long long)b * d_mem * kvw;
  const int j0 = (int)((long long)warp * d_mem / kMemWarps);
  const int j1 = (int)((long long)(warp + 1) * d_mem / kMemWarps);
  float acc = 0.f;
  if (c < kvw) {
#pragma unroll 32
    for (int j = j0; j < j1; ++j) acc = fmaf(sp[j], Mb[(long long)j * kvw + c], acc);
  }
  s_part[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && c < kvw) {
    float m = 0.f;
#pragma unroll
    for (int w = 0; w < kMemWarps; ++w) m += s_part[w][lane];
    m = __fdiv_rn(m, sqrtf(s_den));
    const float r = s_g * m;
    res[((long long)b * q_len + t) * kvw + c] = round_to(r, round_mode);
  }
}

// Stage 2 as an 8-CTA cluster per 128 columns of M (d_mem <= 64 * kMaxR): CTA
// rank c of the cluster takes rows [c*d_mem/8, (c+1)*d_mem/8), each of its 8
// warps a slice of those rows with every row's float4 loaded at once; the
// warps' sums, then the CTAs' sums, are added in rank order, the second
// through distributed shared memory on rank 0, which applies the norm and
// gate.  The norm's 8 partial sums are formed the same way.
constexpr int kMemCluster = 8;
constexpr int kMemCWarps = 8;

template <int kMaxR>
__global__ void __cluster_dims__(1, kMemCluster, 1) __launch_bounds__(kMemCWarps * 32)
    readout_mem_cluster_kernel(const float* __restrict__ proj, const float* __restrict__ gpre,
                               const float* __restrict__ gw2, const float* __restrict__ gb2,
                               float gate_override, const float* __restrict__ M,
                               const float* __restrict__ bst, int q_len, int d_mem, int gh,
                               int kvw, int round_mode, float* __restrict__ res) {
  __shared__ float4 s_w[kMemCWarps][32];
  __shared__ float s_wden[kMemCWarps];
  __shared__ float4 s_cta[32];  // this CTA's sum over its rows, read by rank 0
  __shared__ float s_den;
  __shared__ float s_g;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int z = blockIdx.z, b = z / q_len;  // z = b * q_len + t
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x * 128 + lane * 4;
  const int r0 = (int)((long long)rank * d_mem / kMemCluster);
  const int r1 = (int)((long long)(rank + 1) * d_mem / kMemCluster);
  const int j0 = r0 + (int)((long long)warp * (r1 - r0) / kMemCWarps);
  const int j1 = r0 + (int)((long long)(warp + 1) * (r1 - r0) / kMemCWarps);
  const float* pr = proj + (long long)z * d_mem;
  const float* Mb = M + (long long)b * d_mem * kvw + c;
  const float* bb = bst + (long long)b * d_mem;
  float4 mv[kMaxR];
  float pv[kMaxR], bv[kMaxR];
#pragma unroll
  for (int i = 0; i < kMaxR; ++i) {
    const bool on = j0 + i < j1;
    mv[i] = on ? ldg4(Mb + (long long)(j0 + i) * kvw) : make_float4(0.f, 0.f, 0.f, 0.f);
    pv[i] = on ? __ldg(pr + j0 + i) : 0.f;
    bv[i] = on ? __ldg(bb + j0 + i) : 0.f;
  }
  float gl = 0.f;
  if (rank == 0 && warp == kMemCWarps - 1) {
    for (int o = lane; o < gh; o += 32) gl = fmaf(gw2[o], gelu(gpre[(long long)z * gh + o]), gl);
    for (int o = 16; o > 0; o >>= 1) gl += __shfl_xor_sync(0xffffffffu, gl, o);
  }
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float den = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxR; ++i) {
    acc.x = fmaf(pv[i], mv[i].x, acc.x);
    acc.y = fmaf(pv[i], mv[i].y, acc.y);
    acc.z = fmaf(pv[i], mv[i].z, acc.z);
    acc.w = fmaf(pv[i], mv[i].w, acc.w);
    den = fmaf(pv[i] * pv[i], bv[i], den);
  }
  s_w[warp][lane] = acc;
  if (lane == 0) s_wden[warp] = den;
  if (rank == 0 && warp == kMemCWarps - 1 && lane == 0)
    s_g = learned_gate(gate_override) ? 1.0f / (1.0f + expf(-(gl + gb2[0]))) : gate_override;
  __syncthreads();
  if (warp == 0) {
    float4 v = s_w[0][lane];
    for (int w2 = 1; w2 < kMemCWarps; ++w2) {
      const float4 u = s_w[w2][lane];
      v.x += u.x; v.y += u.y; v.z += u.z; v.w += u.w;
    }
    s_cta[lane] = v;
    if (lane == 0) {
      float dd = 0.f;
      for (int w2 = 0; w2 < kMemCWarps; ++w2) dd += s_wden[w2];
      s_den = dd;
    }
  }
  cluster.sync();
  if (rank == 0 && warp == 0) {
    // all remote reads first, then the sums in rank order
    float4 u[kMemCluster];
    float dv[kMemCluster];
#pragma unroll
    for (int k = 0; k < kMemCluster; ++k) {
      u[k] = *cluster.map_shared_rank(&s_cta[lane], k);
      dv[k] = *cluster.map_shared_rank(&s_den, k);
    }
    float4 m = make_float4(0.f, 0.f, 0.f, 0.f);
    float dd = 0.f;
#pragma unroll
    for (int k = 0; k < kMemCluster; ++k) {
      m.x += u[k].x; m.y += u[k].y; m.z += u[k].z; m.w += u[k].w;
      dd += dv[k];
    }
    const float sq = sqrtf(dd + 1e-8f), g = s_g;
    float4 o;
    o.x = round_to(g * __fdiv_rn(m.x, sq), round_mode);
    o.y = round_to(g * __fdiv_rn(m.y, sq), round_mode);
    o.z = round_to(g * __fdiv_rn(m.z, sq), round_mode);
    o.w = round_to(g * __fdiv_rn(m.w, sq), round_mode);
    *reinterpret_cast<float4*>(res + (long long)z * kvw + c) = o;
  }
  cluster.sync();  // rank 0 has read every CTA's shared memory
}

// Stage 3 for rows that fit in registers (kvw <= 128 * kMaxV): kRows output
// rows per warp, each lane loading its float4 of every row and of the
// residual straight from global memory; the block needs no shared memory.
constexpr int kOutWarps = 8;

template <typename T, int kRows, int kMaxV>
__global__ void __launch_bounds__(kOutWarps * 32)
    readout_out_reg_kernel(const float* __restrict__ res, const float* __restrict__ ofold,
                           int q_len, int kvw, int hidden, T* __restrict__ out) {
  const int b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o0 = (blockIdx.x * kOutWarps + warp) * kRows;
  const int nv = kvw / 128;
  const float* rb = res + (long long)b * q_len * kvw + lane * 4;
  float4 wv[kRows][kMaxV], xv[kMaxV];
#pragma unroll
  for (int k = 0; k < kRows; ++k) {
    const bool live = o0 + k < hidden;
    const float* w = ofold + (long long)(live ? o0 + k : 0) * kvw + lane * 4;
#pragma unroll
    for (int i = 0; i < kMaxV; ++i)
      wv[k][i] = (live && i < nv) ? ldg4(w + i * 128) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int i = 0; i < kMaxV; ++i) xv[i] = i < nv ? ldg4(rb + i * 128) : make_float4(0.f, 0.f, 0.f, 0.f);
  for (int t = 0; t < q_len; ++t) {
    float acc[kRows];
#pragma unroll
    for (int k = 0; k < kRows; ++k) {
      acc[k] = 0.f;
#pragma unroll
      for (int i = 0; i < kMaxV; ++i) acc[k] = dot4(wv[k][i], xv[i], acc[k]);
    }
    if (t + 1 < q_len) {
#pragma unroll
      for (int i = 0; i < kMaxV; ++i)
        if (i < nv) xv[i] = ldg4(rb + (long long)(t + 1) * kvw + i * 128);
    }
#pragma unroll
    for (int k = 0; k < kRows; ++k)
      for (int sft = 16; sft > 0; sft >>= 1) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], sft);
    if (lane == 0) {
      T* row = out + ((long long)b * q_len + t) * hidden;
#pragma unroll
      for (int k = 0; k < kRows; ++k)
        if (o0 + k < hidden) row[o0 + k] = add_out(row[o0 + k], acc[k]);
    }
  }
}

// Stage 3: out += o_fold res (bf16 outputs: the product rounded to bf16, then
// the sum); one warp per output row.
template <typename T>
__global__ void readout_out_kernel(const float* __restrict__ res, const float* __restrict__ ofold,
                                   int q_len, int kvw, int hidden, T* __restrict__ out) {
  extern __shared__ float sr[];  // (q_len, kvw)
  const int b = blockIdx.y;
  for (int i = threadIdx.x; i < q_len * kvw; i += blockDim.x)
    sr[i] = res[(long long)b * q_len * kvw + i];
  __syncthreads();
  const int warps = blockDim.x / 32, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int stride = gridDim.x * warps;
  // two output rows per iteration, so that both rows' loads are in flight together
  for (int o0 = blockIdx.x * warps + warp; o0 < hidden; o0 += 2 * stride) {
    const int o1 = o0 + stride;
    const bool has1 = o1 < hidden;
    const float* w0 = ofold + (long long)o0 * kvw;
    const float* w1 = ofold + (long long)(has1 ? o1 : o0) * kvw;
    for (int t = 0; t < q_len; ++t) {
      const float* x = sr + t * kvw;
      float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 8
      for (int c = lane * 4; c < kvw; c += 128) {
        const float4 a = *reinterpret_cast<const float4*>(w0 + c);
        const float4 bb = *reinterpret_cast<const float4*>(w1 + c);
        acc0 = fmaf(a.x, x[c], acc0);
        acc0 = fmaf(a.y, x[c + 1], acc0);
        acc0 = fmaf(a.z, x[c + 2], acc0);
        acc0 = fmaf(a.w, x[c + 3], acc0);
        acc1 = fmaf(bb.x, x[c], acc1);
        acc1 = fmaf(bb.y, x[c + 1], acc1);
        acc1 = fmaf(bb.z, x[c + 2], acc1);
        acc1 = fmaf(bb.w, x[c + 3], acc1);
      }
      for (int s = 16; s > 0; s >>= 1) {
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, s);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, s);
      }
      if (lane == 0) {
        T* row = out + ((long long)b * q_len + t) * hidden;
        row[o0] = add_out(row[o0], acc0);
        if (has1) row[o1] = add_out(row[o1], acc1);
      }
    }
  }
}

}  // namespace misc
}  // namespace core

using namespace core;
using namespace core::misc;

extern "C" int core_compact_kv(const core_dims_t* d, const void* k, const void* v,
                               const int32_t* keep_idx, int32_t n_kept, void* out_k, void* out_v,
                               void* stream) {
  // the gather moves raw 16-byte pieces: fp16 rows travel like bf16 ones
  core_dims_t dd;
  if (d != nullptr) {
    dd = *d;
    if (dd.dtype == CORE_DTYPE_F16) dd.dtype = CORE_DTYPE_BF16;
    d = &dd;
  }
  int rc = check_dims(d, "core_compact_kv", true);
  if (rc != CORE_OK) return rc;
  if (k == nullptr || v == nullptr || keep_idx == nullptr || out_k == nullptr || out_v == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_compact_kv: NULL tensor");
  if (n_kept <= 0 || n_kept > d->seq_len)
    return set_error(CORE_ERR_INVALID_ARG, "core_compact_kv: bad n_kept");
  if (!aligned16(k) || !aligned16(v) || !aligned16(out_k) || !aligned16(out_v))
    return set_error(CORE_ERR_INVALID_ARG, "core_compact_kv: tensors must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long rows = (long long)d->n_kv_heads * n_kept;
  const int threads = 256;
  const int vec = d->dtype == CORE_DTYPE_F32 ? 32 : 16;  // 16-byte pieces of a row
  long long blocks = (rows + (threads / vec) - 1) / (threads / vec);
  const long long cap = (long long)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  dim3 grid((unsigned)blocks, (unsigned)d->batch);
  const uint4* kk = static_cast<const uint4*>(k);
  const uint4* vv = static_cast<const uint4*>(v);
  uint4* okk = static_cast<uint4*>(out_k);
  uint4* ovv = static_cast<uint4*>(out_v);
  if (vec == 32)
    compact_kernel<32><<<grid, threads, 0, s>>>(kk, vv, keep_idx, d->n_kv_heads, d->seq_len, n_kept,
                                                okk, ovv);
  else
    compact_kernel<16><<<grid, threads, 0, s>>>(kk, vv, keep_idx, d->n_kv_heads, d->seq_len, n_kept,
                                                okk, ovv);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CORE_OK : cuda_error(e, "compact_kernel launch");
}

extern "C" size_t core_memory_readout_workspace_bytes(const core_dims_t* d, int32_t q_len,
                                                      int32_t d_mem, int32_t gate_hidden) {
  if (d == nullptr || q_len <= 0) return 0;
  Sizer z;
  z.take<float>((size_t)d->batch * q_len * d_mem);
  z.take<float>((size_t)d->batch * q_len * (gate_hidden > 0 ? gate_hidden : 1));
  z.take<float>((size_t)d->batch * q_len * d->n_kv_heads * kD);
  return z.used;
}

namespace {

// The three readout stages for queries and attention output of type T
// (bf16, fp16 or f32); proj / gpre / res are the workspace carves.
template <typename T>
int readout_launch(const core_dims_t* d, int32_t q_len, const T* q, const float* theta,
                   const float* gate_w1, const float* gate_b1, const float* gate_w2,
                   const float* gate_b2, int32_t d_mem, int gh, float gate_override,
                   const float* M, const float* b_state, const float* o_fold, int32_t hidden,
                   T* attn_out, float* proj, float* gpre, float* res, cudaStream_t s) {
  using namespace core::misc;
  constexpr bool kF32 = std::is_same<T, float>::value;
  const int round_mode = kF32 ? kRoundNone
                         : std::is_same<T, __half>::value ? kRoundF16 : kRoundBf16;
  const int dm = d->n_q_heads * kD, kvw = d->n_kv_heads * kD;
  cudaError_t e;
  const int sms = sm_count();
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  // register paths: 16-byte weight rows and 8-byte (16-bit types) or 16-byte (f32) q groups
  const bool q_al = (reinterpret_cast<uintptr_t>(q) & (kF32 ? 15 : 7)) == 0;
  const int pv = d->n_q_heads / kProjSplit;
  const bool proj_reg = d->n_q_heads % kProjSplit == 0 && pv <= 16 && q_al && al16(theta) &&
                        (gh == 0 || al16(gate_w1));
  if (proj_reg) {
    const dim3 grid((d_mem + gh + kProjRowsPerBlock - 1) / kProjRowsPerBlock, d->batch);
    const int threads = kProjSplit * kProjRowsPerBlock * 32;
    if (pv <= 8)
      readout_proj_reg_kernel<T, 8><<<grid, threads, 0, s>>>(q, d->n_q_heads, q_len, theta,
                                                              gate_w1, gate_b1, d_mem, gh, proj,
                                                              gpre);
    else
      readout_proj_reg_kernel<T, 16><<<grid, threads, 0, s>>>(q, d->n_q_heads, q_len, theta,
                                                               gate_w1, gate_b1, d_mem, gh, proj,
                                                               gpre);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "readout_proj launch");
  } else {
    const size_t smem = (size_t)q_len * dm * 4;
    e = cudaFuncSetAttribute(readout_proj_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
    if (e != cudaSuccess) return cuda_error(e, "readout_proj attribute");
    const int rows = d_mem + gh;
    int bx = (rows + kProjWarps / 2 - 1) / (kProjWarps / 2);  // two warps per weight row
    if (bx > sms) bx = sms;
    readout_proj_kernel<T><<<dim3(bx, d->batch), kProjWarps * 32, smem, s>>>(
        q, d->n_q_heads, q_len, theta, gate_w1, gate_b1, d_mem, gh, proj, gpre);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "readout_proj launch");
  }
  if (d_mem <= 64 * 16 && al16(M) && (long long)d->batch * q_len <= 65535) {
    const dim3 grid(kvw / 128, kMemCluster, d->batch * q_len);
    if (d_mem <= 64 * 8)
      readout_mem_cluster_kernel<8><<<grid, kMemCWarps * 32, 0, s>>>(
          proj, gpre, gate_w2, gate_b2, gate_override, M, b_state, q_len, d_mem, gh, kvw,
          round_mode, res);
    else
      readout_mem_cluster_kernel<16><<<grid, kMemCWarps * 32, 0, s>>>(
          proj, gpre, gate_w2, gate_b2, gate_override, M, b_state, q_len, d_mem, gh, kvw,
          round_mode, res);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "readout_mem launch");
  } else {
    const size_t smem = (size_t)d_mem * 4;
    readout_mem_kernel<<<dim3((kvw + 31) / 32, d->batch, q_len), kMemWarps * 32, smem, s>>>(
        proj, gpre, gate_w2, gate_b2, gate_override, M, b_state, q_len, d_mem, gh, kvw,
        round_mode, res);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "readout_mem launch");
  }
  if (kvw <= 128 * 16 && al16(o_fold)) {
    const int rpw = kvw <= 128 * 8 ? 2 : 1;  // rows per warp
    const dim3 grid((hidden + kOutWarps * rpw - 1) / (kOutWarps * rpw), d->batch);
    if (rpw == 2)
      readout_out_reg_kernel<T, 2, 8><<<grid, kOutWarps * 32, 0, s>>>(res, o_fold, q_len, kvw,
                                                                      hidden, attn_out);
    else
      readout_out_reg_kernel<T, 1, 16><<<grid, kOutWarps * 32, 0, s>>>(res, o_fold, q_len, kvw,
                                                                       hidden, attn_out);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "readout_out launch");
  } else {
    const size_t smem = (size_t)q_len * kvw * 4;
    e = cudaFuncSetAttribute(readout_out_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
    if (e != cudaSuccess) return cuda_error(e, "readout_out attribute");
    int bx = (hidden + 7) / 8;
    if (bx > sms) bx = sms;
    readout_out_kernel<T><<<dim3(bx, d->batch), 256, smem, s>>>(res, o_fold, q_len, kvw, hidden,
                                                                attn_out);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "readout_out launch");
  }
  return CORE_OK;
}

}  // namespace

extern "C" int core_memory_readout(const core_dims_t* d, int32_t q_len, const void* q,
                                   const float* theta, const float* gate_w1, const float* gate_b1,
                                   const float* gate_w2, const float* gate_b2, int32_t d_mem,
                                   int32_t gate_hidden, float gate_override, const float* M,
                                   const float* b_state, const float* o_fold, int32_t hidden,
                                   void* attn_out, void* workspace, size_t workspace_bytes,
                                   void* stream) {
  if (d == nullptr || d->batch <= 0 || d->n_q_heads <= 0 || d->n_kv_heads <= 0 || d->head_dim != kD)
    return set_error(CORE_ERR_INVALID_ARG, "core_memory_readout: bad dims");
  const bool learned = gate_override != gate_override;  // NaN: the learned gate
  if (q == nullptr || theta == nullptr || M == nullptr || b_state == nullptr || o_fold == nullptr ||
      attn_out == nullptr || (learned && (gate_w1 == nullptr || gate_b1 == nullptr ||
                                          gate_w2 == nullptr || gate_b2 == nullptr)))
    return set_error(CORE_ERR_INVALID_ARG, "core_memory_readout: NULL tensor");
  if (!learned && !std::isfinite(gate_override))
    return set_error(CORE_ERR_INVALID_ARG, "core_memory_readout: gate_override must be finite or NaN");
  if (q_len <= 0 || d_mem <= 0 || hidden <= 0 || gate_hidden < 0)
    return set_error(CORE_ERR_INVALID_ARG, "core_memory_readout: bad sizes");
  if (d->dtype != CORE_DTYPE_BF16 && d->dtype != CORE_DTYPE_F32 && d->dtype != CORE_DTYPE_F16)
    return set_error(CORE_ERR_UNSUPPORTED, "core_memory_readout: dtype must be bf16, f16 or f32");
  const int dm = d->n_q_heads * kD, kvw = d->n_kv_heads * kD;
  if ((size_t)q_len * dm * 4 > 200 * 1024 || (size_t)q_len * kvw * 4 > 200 * 1024)
    return set_error(CORE_ERR_UNSUPPORTED, "core_memory_readout: q_len too large for one call");
  Carver cv(workspace, workspace_bytes);
  float* proj = cv.take<float>((size_t)d->batch * q_len * d_mem);
  float* gpre = cv.take<float>((size_t)d->batch * q_len * (gate_hidden > 0 ? gate_hidden : 1));
  float* res = cv.take<float>((size_t)d->batch * q_len * kvw);
  if (cv.overflow) return set_error(CORE_ERR_WORKSPACE, "core_memory_readout: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int gh = learned ? gate_hidden : 0;
  switch (d->dtype) {
    case CORE_DTYPE_F32:
      return readout_launch<float>(d, q_len, static_cast<const float*>(q), theta, gate_w1, gate_b1,
                                   gate_w2, gate_b2, d_mem, gh, gate_override, M, b_state, o_fold,
                                   hidden, static_cast<float*>(attn_out), proj, gpre, res, s);
    case CORE_DTYPE_F16:
      return readout_launch<__half>(d, q_len, static_cast<const __half*>(q), theta, gate_w1,
                                    gate_b1, gate_w2, gate_b2, d_mem, gh, gate_override, M,
                                    b_state, o_fold, hidden, static_cast<__half*>(attn_out), proj,
                                    gpre, res, s);
    default:
      return readout_launch<__nv_bfloat16>(d, q_len, static_cast<const __nv_bfloat16*>(q), theta,
                                           gate_w1, gate_b1, gate_w2, gate_b2, d_mem, gh,
                                           gate_override, M, b_state, o_fold, hidden,
                                           static_cast<__nv_bfloat16*>(attn_out), proj, gpre, res,
                                           s);
  }
}

// ---------------------------------------------------------------------------
// Readout without a caller workspace: the same three kernels, their scratch in
// a file-scope device array.  Every scratch element a kernel reads is written
// earlier in the same call, so nothing has to start at zero.  The array is one
// per device: overlapping calls on one device race on it.
// ---------------------------------------------------------------------------
#include <mutex>

namespace {
constexpr size_t kReadoutScratchFloats = 65536;  // 256 KB
__device__ __align__(256) float g_readout_scratch[kReadoutScratchFloats];

constexpr int kMaxDevices = 64;
float* g_readout_scratch_ptr[kMaxDevices] = {};
std::mutex g_readout_scratch_mu;

// Resolves the scratch address of the current device once (the first call on
// a device does this set-up; later calls only read the cached pointer).
int readout_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "core_memory_readout_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(CORE_ERR_UNSUPPORTED, "core_memory_readout_noalloc: device index above 63");
  std::lock_guard<std::mutex> lock(g_readout_scratch_mu);
  if (g_readout_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_readout_scratch);
    if (e != cudaSuccess) return cuda_error(e, "core_memory_readout_noalloc: cudaGetSymbolAddress");
    g_readout_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_readout_scratch_ptr[dev];
  return CORE_OK;
}
}  // namespace

extern "C" int core_memory_readout_noalloc(const core_dims_t* d, int32_t q_len, const void* q,
                                           const float* theta, const float* gate_w1,
                                           const float* gate_b1, const float* gate_w2,
                                           const float* gate_b2, int32_t d_mem,
                                           int32_t gate_hidden, float gate_override,
                                           const float* M, const float* b_state,
                                           const float* o_fold, int32_t hidden, void* attn_out,
                                           void* stream) {
  if (d == nullptr || d->batch <= 0 || d->n_q_heads <= 0 || d->n_kv_heads <= 0 || d->head_dim != kD)
    return set_error(CORE_ERR_INVALID_ARG, "core_memory_readout_noalloc: bad dims");
  if (q_len <= 0 || d_mem <= 0 || hidden <= 0 || gate_hidden < 0)
    return set_error(CORE_ERR_INVALID_ARG, "core_memory_readout_noalloc: bad sizes");
  // the carves core_memory_readout makes from its workspace, 256-byte aligned
  Sizer need;
  need.take<float>((size_t)d->batch * q_len * d_mem);
  need.take<float>((size_t)d->batch * q_len * (gate_hidden > 0 ? gate_hidden : 1));
  need.take<float>((size_t)d->batch * q_len * d->n_kv_heads * kD);
  if (need.used > kReadoutScratchFloats * sizeof(float))
    return set_error(CORE_ERR_INVALID_ARG,
                     "core_memory_readout_noalloc: B*q_len*(d_mem + gate_hidden + Hkv*d) floats "
                     "exceed the 256 KB static scratch; use core_memory_readout");
  float* scratch = nullptr;
  int rc = readout_scratch(&scratch);
  if (rc != CORE_OK) return rc;
  return core_memory_readout(d, q_len, q, theta, gate_w1, gate_b1, gate_w2, gate_b2, d_mem,
                             gate_hidden, gate_override, M, b_state, o_fold, hidden, attn_out,
                             scratch, kReadoutScratchFloats * sizeof(float), stream);
}
