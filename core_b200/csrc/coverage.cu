// Coverage features o, d_proto, delta_proto, g
// (replaces core/features.py:790-858 with :53-77, :146-213, :259-261).
//
//   cov_project_kernel : z = normalize(sum_h (W_h k_h) / (|k_h| + eps)) for a
//                        128-token tile.  W_h k_h runs on tcgen05 with the fp32
//                        geometry split into three bf16 terms (K is exact in
//                        bf16, so the product is f32-accurate); the per-head
//                        norms come from the same K tile in shared memory.
//                        Also accumulates sum z, sum zt, sum zt^2 (zt = R z).
//   cov_stats_kernel   : reduces those sums to mean z, mu, sigma2_eff.
//   cov_assign_kernel  : centred prototype cosines, first-max assignment,
//                        second best, occupancy histogram, d, delta and g.
//   cov_occupancy_kernel : o = log1p(count of the token's prototype).
#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "host_util.h"

namespace core {
namespace cov {

constexpr int kD = 128;
constexpr int kTile = 128;
constexpr int kP = 64;           // proto_dim
constexpr int kNP = 64;          // number of prototypes
constexpr int kThreads = 256;    // warp 0 TMA, warp 1 MMA, warps 4..7 epilogue
constexpr int kStages = 2;
constexpr uint32_t kABytes = kTile * kD * 2;      // 32 KB: one head's K tile
constexpr uint32_t kBBytes = 3u * kP * kD * 2;    // 48 KB: three terms of W_h
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr int kNStats = 3 * kP;  // sum z, sum zt, sum zt^2

struct Params {
  int B, Hkv, L, n_tiles;
  long long U;
  float* z;              // (B, L, 64)
  double* part;          // (grid, B, 192) per-CTA sums
  const float* hadamard; // (64, 64)
  DeviceStatus* status;
};

__device__ __forceinline__ long long unit_begin(int c, long long U, int P) {
  return (long long)c * U / P;
}

struct Smem {
  static constexpr uint32_t kStageOff = 0;
  static constexpr uint32_t kROff = kStages * kStageBytes;         // hadamard f32 64x64
  static constexpr uint32_t kRedOff = kROff + kP * kP * 4;          // double [4 warps][192]
  static constexpr uint32_t kBarOff = kRedOff + 4 * kNStats * 8;
  static constexpr uint32_t kTotal = kBarOff + 256;
};

__global__ void __launch_bounds__(kThreads, 1)
    cov_project_kernel(const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmW, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  float* sR = reinterpret_cast<float*>(sgen + Smem::kROff);
  double* sRed = reinterpret_cast<double*>(sgen + Smem::kRedOff);
  const uint32_t bar = sbase + Smem::kBarOff;
  auto bar_full = [&](int s) { return bar + 8u * s; };
  auto bar_empty = [&](int s) { return bar + 8u * (kStages + s); };
  auto bar_tfull = [&](int h) { return bar + 8u * (2 * kStages + h); };    // 8 slots
  auto bar_tempty = [&](int h) { return bar + 8u * (2 * kStages + 8 + h); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + Smem::kBarOff + 224);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sgen + Smem::kBarOff + 232);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = gridDim.x;
  const long long u0 = unit_begin(blockIdx.x, p.U, P), u1 = unit_begin(blockIdx.x + 1, p.U, P);

  for (int i = threadIdx.x; i < kP * kP; i += kThreads) sR[i] = p.hadamard[i];
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar_full(s), 1);
      mbar_init(bar_empty(s), 1 + 4);  // MMA commit + 4 epilogue warps (norms read)
    }
    for (int h = 0; h < 8; ++h) {
      mbar_init(bar_tfull(h), 1);
      mbar_init(bar_tempty(h), 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmW);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto wait = [&](uint32_t b, uint32_t parity, int where) -> bool {
    return bounded_wait(b, parity, abort_flag, p.status, where);
  };

  // Each unit = (b, tile); it streams Hkv stages (one per KV head).  TMEM holds
  // eight 64-column slots; head h of every unit uses slot h % 8.
  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (long long u = u0; u < u1 && ok; ++u) {
        const int b = (int)(u / p.n_tiles), tile = (int)(u % p.n_tiles);
        for (int h = 0; h < p.Hkv; ++h) {
          const int st = it % kStages;
          if (it >= kStages && !(ok = wait(bar_empty(st), ((it / kStages) - 1) & 1, 301))) break;
          const uint32_t base = sbase + st * kStageBytes;
          mbar_arrive_expect_tx(bar_full(st), kStageBytes);
          for (int ka = 0; ka < 2; ++ka)
            tma_load_3d(base + ka * (kTile * 128u), &tmK, bar_full(st), ka * 64, tile * kTile,
                        b * p.Hkv + h);
          // W terms: rows (term*64 + j), columns h*128 + [0, 128)
          for (int ka = 0; ka < 2; ++ka)
            tma_load_2d(base + kABytes + ka * (3u * kP * 128u), &tmW, bar_full(st),
                        h * kD + ka * 64, 0);
          ++it;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(128, kP, 0, 0);
      int it = 0;
      long long nslot = 0;
      bool ok = true;
      for (long long u = u0; u < u1 && ok; ++u) {
        for (int h = 0; h < p.Hkv; ++h, ++nslot) {
          const int st = it % kStages;
          if (!(ok = wait(bar_full(st), (it / kStages) & 1, 302))) break;
          const int slot = (int)(nslot & 7);
          const long long use = nslot >> 3;
          if (use > 0 && !(ok = wait(bar_tempty(slot), (uint32_t)((use - 1) & 1), 303))) break;
          tc_fence_after();
          const uint32_t base = sbase + st * kStageBytes;
          const uint32_t d = tmem + (uint32_t)(slot * kP);
          for (int term = 0; term < 3; ++term) {
            for (int ks = 0; ks < 8; ++ks) {
              const uint64_t a = sdesc_kmajor(base + (uint32_t)(ks >> 2) * kTile * 128u +
                                              (uint32_t)(ks & 3) * 32u);
              const uint64_t bd = sdesc_kmajor(base + kABytes + (uint32_t)(ks >> 2) * 3u * kP * 128u +
                                               (uint32_t)term * kP * 128u + (uint32_t)(ks & 3) * 32u);
              mma_bf16(d, a, bd, idesc, (term > 0 || ks > 0) ? 1u : 0u);
            }
          }
          mma_commit(bar_tfull(slot));
          mma_commit(bar_empty(st));
          ++it;
        }
      }
    }
  } else if (warp >= 4) {
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    // per-CTA running sums, accumulated in shared memory by warp 4..7 partials
    for (int i = threadIdx.x - 128; i < 4 * kNStats; i += 128) sRed[i] = 0.0;
    named_barrier(1, 128);
    long long nslot = 0;
    int it = 0;
    bool ok = true;
    int cur_b = -1;
    for (long long u = u0; u < u1 && ok; ++u) {
      const int b = (int)(u / p.n_tiles), tile = (int)(u % p.n_tiles);
      if (b != cur_b) {
        if (cur_b >= 0) {
          // flush the previous batch row's sums
          named_barrier(1, 128);
          for (int i = threadIdx.x - 128; i < kNStats; i += 128) {
            double s = sRed[i] + sRed[kNStats + i] + sRed[2 * kNStats + i] + sRed[3 * kNStats + i];
            p.part[((long long)blockIdx.x * p.B + cur_b) * kNStats + i] = s;
          }
          named_barrier(1, 128);
          for (int i = threadIdx.x - 128; i < 4 * kNStats; i += 128) sRed[i] = 0.0;
          named_barrier(1, 128);
        }
        cur_b = b;
      }
      const int tok = tile * kTile + row;
      float z[kP];
#pragma unroll
      for (int j = 0; j < kP; ++j) z[j] = 0.f;
      for (int h = 0; h < p.Hkv; ++h, ++nslot) {
        const int st = it % kStages;
        const int slot = (int)(nslot & 7);
        const long long use = nslot >> 3;
        if (!(ok = wait(bar_tfull(slot), (uint32_t)(use & 1), 304))) break;
        tc_fence_after();
        // |k_h| of this token from the swizzled K tile (two 128-byte atoms)
        const uint8_t* kt = sgen + st * kStageBytes;
        float ss = 0.f;
        for (int ka = 0; ka < 2; ++ka) {
          const uint8_t* rowp = kt + ka * (kTile * 128) + row * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 w = *reinterpret_cast<const uint4*>(rowp + ((c ^ (row & 7)) * 16));
            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f2 = __bfloat1622float2(h2[e]);
              ss = fmaf(f2.x, f2.x, ss);
              ss = fmaf(f2.y, f2.y, ss);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_empty(st));
        const float inv = 1.0f / (sqrtf(ss) + 1e-8f);
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(wq * 32) << 16) + (uint32_t)(slot * kP), v);
#pragma unroll
        for (int j = 0; j < 32; ++j) z[j] = fmaf(v[j], inv, z[j]);
        tmem_ld32(tmem + ((uint32_t)(wq * 32) << 16) + (uint32_t)(slot * kP + 32), v);
#pragma unroll
        for (int j = 0; j < 32; ++j) z[32 + j] = fmaf(v[j], inv, z[32 + j]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_tempty(slot));
        ++it;
      }
      if (!ok) break;
      float nn = 0.f;
#pragma unroll
      for (int j = 0; j < kP; ++j) nn = fmaf(z[j], z[j], nn);
      const float inv = 1.0f / (sqrtf(nn) + 1e-8f);
#pragma unroll
      for (int j = 0; j < kP; ++j) z[j] *= inv;
      const bool valid = tok < p.L;
      if (valid) {
        float4* dst = reinterpret_cast<float4*>(p.z + ((long long)b * p.L + tok) * kP);
#pragma unroll
        for (int j = 0; j < kP / 4; ++j) dst[j] = make_float4(z[4 * j], z[4 * j + 1], z[4 * j + 2], z[4 * j + 3]);
      }
      // Sums over the tile: warp reduce each statistic, lane 0 accumulates.
      for (int j = 0; j < kP; ++j) {
        float zt = 0.f;
#pragma unroll 8
        for (int i = 0; i < kP; ++i) zt = fmaf(sR[j * kP + i], z[i], zt);
        float a = valid ? z[j] : 0.f;
        float bz = valid ? zt : 0.f;
        float c = valid ? zt * zt : 0.f;
        double da = a, db = bz, dc = c;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          da += __shfl_xor_sync(0xffffffffu, da, o);
          db += __shfl_xor_sync(0xffffffffu, db, o);
          dc += __shfl_xor_sync(0xffffffffu, dc, o);
        }
        if (lane == 0) {
          sRed[wq * kNStats + j] += da;
          sRed[wq * kNStats + kP + j] += db;
          sRed[wq * kNStats + 2 * kP + j] += dc;
        }
      }
    }
    if (ok && cur_b >= 0) {
      named_barrier(1, 128);
      for (int i = threadIdx.x - 128; i < kNStats; i += 128) {
        double s = sRed[i] + sRed[kNStats + i] + sRed[2 * kNStats + i] + sRed[3 * kNStats + i];
        p.part[((long long)blockIdx.x * p.B + cur_b) * kNStats + i] = s;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Per batch row: mean z (64), mu (64), sigma2_eff (64).
__global__ void cov_stats_kernel(const double* __restrict__ part, int grid_ctas, int B, int L,
                                 int n_tiles, float rho, float* __restrict__ stats) {
  const int b = blockIdx.x;
  __shared__ double s[kNStats];
  __shared__ float sig[kP];
  const int i = threadIdx.x;  // 192 threads
  double acc = 0.0;
  const long long U = (long long)B * n_tiles;
  const long long lo = (long long)b * n_tiles, hi = lo + n_tiles;
  for (int c = 0; c < grid_ctas; ++c) {
    // CTA c covers units [c*U/P, (c+1)*U/P) of the static partition
    const long long a = (long long)c * U / grid_ctas, e = (long long)(c + 1) * U / grid_ctas;
    if (a < hi && e > lo) acc += part[((long long)c * B + b) * kNStats + i];
  }
  s[i] = acc;
  __syncthreads();
  float* out = stats + (long long)b * kNStats;
  if (i < kP) {
    out[i] = (float)(s[i] / L);  // mean z
    const double mu = s[kP + i] / L;
    const double ez2 = s[2 * kP + i] / L;
    out[kP + i] = (float)mu;
    float v = (float)(ez2 - mu * mu);
    sig[i] = v > 0.f ? v : 0.f;  // clamp_min(0) (features.py:840)
  }
  __syncthreads();
  if (i < kP) {
    double a = 0.0;
    for (int j = 0; j < kP; ++j) a += sig[j];
    const float avg = (float)(a / kP);
    out[2 * kP + i] = ((1.0f - rho) * sig[i] + rho * avg) + 1e-8f;
  }
}

__global__ void __launch_bounds__(128)
    cov_assign_kernel(const float* __restrict__ z, const float* __restrict__ stats,
                      const float* __restrict__ protos, const float* __restrict__ hadamard,
                      int B, int L, int* __restrict__ assign, int* __restrict__ hist,
                      float* __restrict__ features, int stride, int col0, DeviceStatus* status) {
  __shared__ float sP[kNP * kP];
  __shared__ float sR[kP * kP];
  __shared__ int sh[kNP];
  for (int i = threadIdx.x; i < kNP * kP; i += blockDim.x) {
    sP[i] = protos[i];
    sR[i] = hadamard[i];
  }
  for (int i = threadIdx.x; i < kNP; i += blockDim.x) sh[i] = 0;
  __syncthreads();
  const long long gi = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const bool active = gi < (long long)B * L;
  int b = 0;
  if (active) {
    b = (int)(gi / L);
    const float* st = stats + (long long)b * kNStats;
    float zv[kP], zc[kP];
    const float4* src = reinterpret_cast<const float4*>(z + gi * kP);
#pragma unroll
    for (int j = 0; j < kP / 4; ++j) {
      float4 t = src[j];
      zv[4 * j] = t.x; zv[4 * j + 1] = t.y; zv[4 * j + 2] = t.z; zv[4 * j + 3] = t.w;
    }
    float cn2 = 0.f;
#pragma unroll
    for (int j = 0; j < kP; ++j) {
      zc[j] = zv[j] - st[j];
      cn2 = fmaf(zc[j], zc[j], cn2);
    }
    const float cn = sqrtf(cn2);
    const bool reliable = cn > 1e-6f;
    const float inv = 1.0f / fmaxf(cn, 1e-6f);
#pragma unroll
    for (int j = 0; j < kP; ++j) zc[j] = zc[j] * inv;
    float c1 = -INFINITY, c2 = -INFINITY;
    int m1 = 0;
    for (int m = 0; m < kNP; ++m) {
      float c = 0.f;
#pragma unroll 16
      for (int j = 0; j < kP; ++j) c = fmaf(zc[j], sP[m * kP + j], c);
      if (c > c1) {  // strict: first maximum wins (features.py:177)
        c2 = c1;
        c1 = c;
        m1 = m;
      } else if (c > c2) {
        c2 = c;
      }
    }
    // g: standardised squared deviation of the rotated z (features.py:826-853)
    float gs = 0.f;
    for (int j = 0; j < kP; ++j) {
      float zt = 0.f;
#pragma unroll 16
      for (int i = 0; i < kP; ++i) zt = fmaf(sR[j * kP + i], zv[i], zt);
      const float dv = zt - st[kP + j];
      gs += (dv * dv) / st[2 * kP + j];
    }
    const float g = log1pf(gs / (float)kP);
    float* out = features + gi * stride + col0;
    out[1] = reliable ? 1.0f - c1 : 1.0f;
    out[2] = reliable ? c1 - c2 : 0.0f;
    out[3] = g;
    assign[gi] = reliable ? m1 : -1;
    if (reliable) {
      if (b == (int)(((long long)blockIdx.x * blockDim.x) / L)) atomicAdd(&sh[m1], 1);
      else atomicAdd(&hist[b * kNP + m1], 1);
    }
    if (!isfinite(c1) || !isfinite(g)) record_error(status, CORE_ERR_NONFINITE, 501, (int)gi);
  }
  __syncthreads();
  // Tokens of the block's first batch row were counted in shared memory
  // (above); a block that reaches into later rows counts those tokens with
  // global atomics.
  const long long first = (long long)blockIdx.x * blockDim.x;
  const int row0 = (int)(first / L);
  for (int m = threadIdx.x; m < kNP; m += blockDim.x)
    if (sh[m]) atomicAdd(&hist[row0 * kNP + m], sh[m]);
}

__global__ void cov_occupancy_kernel(const int* __restrict__ assign, const int* __restrict__ hist,
                                     int B, int L, float* __restrict__ features, int stride,
                                     int col0) {
  const long long gi = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (gi >= (long long)B * L) return;
  const int b = (int)(gi / L);
  const int m = assign[gi];
  features[gi * stride + col0] = (m >= 0) ? log1pf((float)hist[b * kNP + m]) : 0.0f;
}

}  // namespace cov
}  // namespace core

using namespace core;
using namespace core::cov;

namespace {
struct CovPlan {
  Params p;
  int grid;
};
void plan_cov(const core_dims_t* d, CovPlan* c) {
  c->p = Params{};
  c->p.B = d->batch;
  c->p.Hkv = d->n_kv_heads;
  c->p.L = d->seq_len;
  c->p.n_tiles = (d->seq_len + kTile - 1) / kTile;
  c->p.U = (long long)c->p.B * c->p.n_tiles;
  const int sms = sm_count();
  c->grid = (int)(c->p.U < sms ? c->p.U : sms);
}
}  // namespace

extern "C" size_t core_coverage_workspace_bytes(const core_dims_t* d) {
  if (check_dims(d, "core_coverage_workspace_bytes") != CORE_OK) return 0;
  CovPlan c;
  plan_cov(d, &c);
  Sizer z;
  z.take<float>((size_t)d->batch * d->seq_len * kP);                 // z
  z.take<double>((size_t)c.grid * d->batch * kNStats);               // per-CTA sums
  z.take<float>((size_t)d->batch * kNStats);                         // stats
  z.take<int>((size_t)d->batch * d->seq_len);                        // assignment
  z.take<int>((size_t)d->batch * kNP);                               // histogram
  return z.used;
}

extern "C" int core_coverage_features(const core_dims_t* d, const void* k,
                                      const void* geometry_split, const float* prototypes,
                                      const float* hadamard, float shrinkage_rho,
                                      float* features, int32_t feature_stride, int32_t col0,
                                      void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_dims(d, "core_coverage_features");
  if (rc != CORE_OK) return rc;
  if (k == nullptr || geometry_split == nullptr || prototypes == nullptr || hadamard == nullptr ||
      features == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_coverage_features: NULL tensor");
  if (col0 < 0 || col0 + 4 > feature_stride)
    return set_error(CORE_ERR_INVALID_ARG, "core_coverage_features: bad feature columns");
  CovPlan c;
  plan_cov(d, &c);
  Params& p = c.p;
  Carver cv(workspace, workspace_bytes);
  p.z = cv.take<float>((size_t)p.B * p.L * kP);
  p.part = cv.take<double>((size_t)c.grid * p.B * kNStats);
  float* stats = cv.take<float>((size_t)p.B * kNStats);
  int* assign = cv.take<int>((size_t)p.B * p.L);
  int* hist = cv.take<int>((size_t)p.B * kNP);
  if (cv.overflow) return set_error(CORE_ERR_WORKSPACE, "core_coverage_features: workspace too small");
  p.hadamard = hadamard;
  p.status = device_status();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;

  e = cudaMemsetAsync(hist, 0, sizeof(int) * (size_t)p.B * kNP, s);
  if (e != cudaSuccess) return cuda_error(e, "coverage histogram clear");

  CUtensorMap tmK, tmW;
  {
    uint64_t dims[3] = {128, (uint64_t)p.L, (uint64_t)p.B * p.Hkv};
    uint64_t str[2] = {256, (uint64_t)p.L * 256};
    uint32_t box[3] = {64, 128, 1};
    if ((rc = make_tmap_bf16(&tmK, k, 3, dims, str, box, true)) != CORE_OK) return rc;
  }
  {
    const uint64_t in = (uint64_t)p.Hkv * kD;
    uint64_t dims[2] = {in, 3u * kP};
    uint64_t str[1] = {in * 2};
    uint32_t box[2] = {64, 3u * kP};
    if ((rc = make_tmap_bf16(&tmW, geometry_split, 2, dims, str, box, true)) != CORE_OK) return rc;
  }
  const uint32_t smem = Smem::kTotal + 1024;
  e = cudaFuncSetAttribute(cov_project_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_error(e, "cov_project_kernel attribute");
  cov_project_kernel<<<c.grid, kThreads, smem, s>>>(tmK, tmW, p);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "cov_project_kernel launch");
  cov_stats_kernel<<<p.B, kNStats, 0, s>>>(p.part, c.grid, p.B, p.L, p.n_tiles, shrinkage_rho, stats);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "cov_stats_kernel launch");
  const long long n = (long long)p.B * p.L;
  const unsigned blocks = (unsigned)((n + 127) / 128);
  cov_assign_kernel<<<blocks, 128, 0, s>>>(p.z, stats, prototypes, hadamard, p.B, p.L, assign, hist,
                                           features, feature_stride, col0, p.status);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "cov_assign_kernel launch");
  cov_occupancy_kernel<<<blocks, 128, 0, s>>>(assign, hist, p.B, p.L, features, feature_stride, col0);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "cov_occupancy_kernel launch");
  return CORE_OK;
}
