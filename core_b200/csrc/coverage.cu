// Coverage features o, d_proto, delta_proto, g
// (replaces core/features.py:790-858 with :53-77, :146-213, :259-261).
//
//   geometry_prepare_kernel : once per layer, W_ext = [W ; R W] (128 x Hkv*d)
//                             split into three bf16 terms, so one MMA yields both
//                             the projection and its Hadamard rotation.
//   cov_project_kernel      : per 128-token tile, y = sum_h W_ext,h k_h / (|k_h| + eps)
//                             on tcgen05 (K is exact in bf16 and W_ext carries three
//                             bf16 terms, so the product is f32-accurate);
//                             z = y[:64] / (|y[:64]| + eps), zt = y[64:] / (same), and
//                             per-CTA column sums of z, zt, zt^2.
//   cov_stats_kernel        : reduces the per-CTA sums (double) and finalises the row
//                             statistics.
//   cov_assign_kernel       : four threads per token: centred prototype cosines,
//                             first-max assignment, second best, occupancy
//                             histogram, d, delta and g.
//   cov_occupancy_kernel    : o = log1p(count of the token's prototype).
#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "host_util.h"

namespace core {
namespace cov {

constexpr int kD = 128;
constexpr int kTile = 128;
constexpr int kP = 64;            // proto_dim
constexpr int kNP = 64;           // number of prototypes
constexpr int kNExt = 2 * kP;     // MMA N: projection rows + rotated rows
constexpr int kThreads = 384;     // warp 0 TMA, warp 1 MMA, warps 4..7 / 8..11 epilogue (z / zt)
constexpr int kStages = 3;
// one stage = one 64-column K atom of one head: A 128 x 128 B, B 3 terms x 128 x 128 B
constexpr uint32_t kABytes = kTile * 128u;           // 16 KB
constexpr uint32_t kBBytes = 3u * kNExt * 128u;      // 48 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;  // 64 KB
constexpr int kSlots = 4;                            // TMEM slots of 128 columns
constexpr int kNStats = 3 * kP;                      // sum z, sum zt, sum zt^2

struct Params {
  int B, Hkv, L, n_tiles;
  long long U;
  int partial;           // 1: write the raw projection of this rank's heads (head-sharded caches)
  float* z;              // (B, L, 64)
  float* zt;             // (B, L, 64)
  double* part;          // (grid, B, 192) per-CTA sums
  DeviceStatus* status;
};

__device__ __forceinline__ long long unit_begin(int c, long long U, int P) {
  return (long long)c * U / P;
}

struct Smem {
  static constexpr uint32_t kStageOff = 0;
  static constexpr uint32_t kTileSumOff = kStages * kStageBytes;        // float [4 warps][192]
  static constexpr uint32_t kRedOff = kTileSumOff + 4 * kNStats * 4;    // double [192]
  static constexpr uint32_t kNormOff = kRedOff + kNStats * 8;           // float [128]
  static constexpr uint32_t kBarOff = kNormOff + kTile * 4;
  static constexpr uint32_t kTotal = kBarOff + 256;
};

// Column sums of a 32-token x 32-column block held one row per lane: on
// return, lane j holds the sum of column j (31 shuffles).
__device__ __forceinline__ float warp_column_sums(float (&w)[32], int lane) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
    for (int j = 0; j < off; ++j) {
      const bool upper = (lane & off) != 0;
      const float send = upper ? w[j] : w[j + off];
      const float keep = upper ? w[j + off] : w[j];
      w[j] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return w[0];
}

__global__ void __launch_bounds__(kThreads, 1)
    cov_project_kernel(const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmW, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  float* sTile = reinterpret_cast<float*>(sgen + Smem::kTileSumOff);
  double* sRed = reinterpret_cast<double*>(sgen + Smem::kRedOff);
  const uint32_t bar = sbase + Smem::kBarOff;
  auto bar_full = [&](int s) { return bar + 8u * s; };
  auto bar_empty = [&](int s) { return bar + 8u * (kStages + s); };
  auto bar_tfull = [&](int h) { return bar + 8u * (2 * kStages + h); };
  auto bar_tempty = [&](int h) { return bar + 8u * (2 * kStages + kSlots + h); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + Smem::kBarOff + 224);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sgen + Smem::kBarOff + 232);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = gridDim.x;
  const long long u0 = unit_begin(blockIdx.x, p.U, P), u1 = unit_begin(blockIdx.x + 1, p.U, P);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar_full(s), 1);
      mbar_init(bar_empty(s), 1 + 8);  // MMA commit + 8 epilogue warps (norm rows read)
    }
    for (int h = 0; h < kSlots; ++h) {
      mbar_init(bar_tfull(h), 1);
      mbar_init(bar_tempty(h), 8);
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

  // Each unit = (b, tile) streams 2 * Hkv stages (head h, K atom ka); the n-th
  // head processed by this CTA uses TMEM slot n % kSlots.
  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (long long u = u0; u < u1 && ok; ++u) {
        const int b = (int)(u / p.n_tiles), tile = (int)(u % p.n_tiles);
        for (int hi = 0; hi < p.Hkv && ok; ++hi) {
          // each token tile starts at its own head, so that the CTAs stream
          // different W_ext tiles at any moment rather than the same lines of
          // L2 (the order depends on the tile only, not on the grid)
          const int h = (hi + tile) % p.Hkv;
          for (int ka = 0; ka < 2; ++ka, ++it) {
            const int st = it % kStages;
            if (it >= kStages && !(ok = wait(bar_empty(st), ((it / kStages) - 1) & 1, 301))) break;
            const uint32_t base = sbase + st * kStageBytes;
            mbar_arrive_expect_tx(bar_full(st), kStageBytes);
            tma_load_3d(base, &tmK, bar_full(st), ka * 64, tile * kTile, b * p.Hkv + h);
            // W_ext terms: rows (term * 128 + j), columns h*128 + ka*64 + [0, 64)
            for (int term = 0; term < 3; ++term)
              tma_load_2d(base + kABytes + (uint32_t)term * kNExt * 128u, &tmW, bar_full(st),
                          h * kD + ka * 64, term * kNExt);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(128, kNExt, 0, 0);
      int it = 0;
      long long nhead = 0;
      bool ok = true;
      for (long long u = u0; u < u1 && ok; ++u) {
        for (int h = 0; h < p.Hkv && ok; ++h, ++nhead) {
          const int slot = (int)(nhead % kSlots);
          const long long use = nhead / kSlots;
          if (use > 0 && !(ok = wait(bar_tempty(slot), (uint32_t)((use - 1) & 1), 303))) break;
          tc_fence_after();
          const uint32_t d = tmem + (uint32_t)(slot * kNExt);
          for (int ka = 0; ka < 2 && ok; ++ka, ++it) {
            const int st = it % kStages;
            if (!(ok = wait(bar_full(st), (it / kStages) & 1, 302))) break;
            tc_fence_after();
            const uint32_t base = sbase + st * kStageBytes;
            for (int term = 0; term < 3; ++term) {
              for (int ks = 0; ks < 4; ++ks) {
                const uint64_t a = sdesc_kmajor(base + (uint32_t)ks * 32u);
                const uint64_t bd = sdesc_kmajor(base + kABytes + (uint32_t)term * kNExt * 128u +
                                                 (uint32_t)ks * 32u);
                mma_bf16(d, a, bd, idesc, (ka > 0 || term > 0 || ks > 0) ? 1u : 0u);
              }
            }
            mma_commit(bar_empty(st));
          }
          if (ok) mma_commit(bar_tfull(slot));
        }
      }
    }
  } else if (warp >= 4) {
    // team 0 (warps 4..7) accumulates the projection z, team 1 (warps 8..11)
    // the rotated zt; both need |k_h|, and team 1 needs |y| from team 0.
    float* sNorm = reinterpret_cast<float*>(sgen + Smem::kNormOff);
    const int wq = warp & 3;
    const int team = (warp - 4) >> 2;
    const int row = wq * 32 + lane;
    const int etid = threadIdx.x - 128;  // 0..255
    for (int i = etid; i < kNStats; i += 256) sRed[i] = 0.0;
    named_barrier(1, 256);
    long long nhead = 0;
    int it = 0;
    bool ok = true;
    int cur_b = -1;
    auto flush = [&](int b) {
      named_barrier(1, 256);
      for (int i = etid; i < kNStats; i += 256) {
        p.part[((long long)blockIdx.x * p.B + b) * kNStats + i] = sRed[i];
        sRed[i] = 0.0;
      }
      named_barrier(1, 256);
    };
    for (long long u = u0; u < u1 && ok; ++u) {
      const int b = (int)(u / p.n_tiles), tile = (int)(u % p.n_tiles);
      if (b != cur_b) {
        if (cur_b >= 0) flush(cur_b);
        cur_b = b;
      }
      const int tok = tile * kTile + row;
      float y[kP];
#pragma unroll
      for (int j = 0; j < kP; ++j) y[j] = 0.f;
      for (int h = 0; h < p.Hkv && ok; ++h, ++nhead) {
        // |k_h| of this token from the two swizzled K atoms of head h
        float ss = 0.f;
        for (int ka = 0; ka < 2; ++ka, ++it) {
          const int st = it % kStages;
          if (!(ok = wait(bar_full(st), (it / kStages) & 1, 305))) break;
          const uint8_t* rowp = sgen + st * kStageBytes + row * 128;
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
          // order these generic-proxy reads before the TMA (async proxy) refill of the stage
          fence_proxy_async_shared();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_empty(st));
        }
        if (!ok) break;
        const int slot = (int)(nhead % kSlots);
        const long long use = nhead / kSlots;
        if (!(ok = wait(bar_tfull(slot), (uint32_t)(use & 1), 304))) break;
        tc_fence_after();
        const float inv = 1.0f / (sqrtf(ss) + 1e-8f);
        const uint32_t ta = tmem + ((uint32_t)(wq * 32) << 16) + (uint32_t)(slot * kNExt + team * kP);
        float v[32];
        tmem_ld32(ta, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) y[j] = fmaf(v[j], inv, y[j]);
        tmem_ld32(ta + 32, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) y[32 + j] = fmaf(v[j], inv, y[32 + j]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_tempty(slot));
      }
      if (!ok) break;
      if (p.partial) {  // uniform: y[:64] = sum over this rank's heads, reduced across ranks later
        if (team == 0 && tok < p.L) {
          float4* dst = reinterpret_cast<float4*>(p.z + ((long long)b * p.L + tok) * kP);
#pragma unroll
          for (int j = 0; j < kP / 4; ++j)
            dst[j] = make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
        }
        continue;
      }
      if (team == 0) {
        float nn = 0.f;
#pragma unroll
        for (int j = 0; j < kP; ++j) nn = fmaf(y[j], y[j], nn);
        sNorm[row] = 1.0f / (sqrtf(nn) + 1e-8f);
      }
      named_barrier(2, 256);
      const float inv = sNorm[row];
#pragma unroll
      for (int j = 0; j < kP; ++j) y[j] *= inv;  // team 0: z; team 1: zt = R z
      const bool valid = tok < p.L;
      if (valid) {
        float4* dst = reinterpret_cast<float4*>((team == 0 ? p.z : p.zt) + ((long long)b * p.L + tok) * kP);
#pragma unroll
        for (int j = 0; j < kP / 4; ++j) dst[j] = make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
      }
      // column sums over this warp's 32 tokens: team 0 -> z; team 1 -> zt, zt^2
#pragma unroll
      for (int blk = 0; blk < 4; ++blk) {
        if (team == 0 && blk >= 2) break;
        float w[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float x = y[(blk & 1) * 32 + j];
          if (blk >= 2) x = x * x;
          w[j] = valid ? x : 0.f;
        }
        const int col = team == 0 ? blk * 32 : kP + blk * 32;
        sTile[wq * kNStats + col + lane] = warp_column_sums(w, lane);
      }
      named_barrier(1, 256);
      for (int i = etid; i < kNStats; i += 256)
        sRed[i] += (double)(((sTile[i] + sTile[kNStats + i]) + sTile[2 * kNStats + i]) +
                            sTile[3 * kNStats + i]);
      named_barrier(1, 256);
    }
    if (ok && cur_b >= 0) flush(cur_b);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Per batch row: the column sums over the CTAs that covered the row (double),
// then mean z, mu and sigma2_eff (features.py:812, :830-845) as floats:
// stats[b] = [mean z (64) | mu (64) | sigma2_eff (64)].
// ---------------------------------------------------------------------------
// f32 keys: the same projection on CUDA cores, with the unit partition,
// outputs and per-CTA partial sums of cov_project_kernel, so cov_stats_kernel
// and the assignment kernels run unchanged.  W_ext is rebuilt in f32 from its
// three bf16 terms ((hi + mid) is exact; + lo restores the 24-bit significand).
// Thread (tr = tid / 16, tc = tid % 16) owns tokens tr + 16 i and output
// columns tc + 16 j (i, j < 8): columns j < 4 are z, j >= 4 the rotated zt.
// ---------------------------------------------------------------------------
constexpr int kF32Threads = 256;
constexpr int kF32Pad = kD + 1;  // padded rows: a warp's 16 column owners hit distinct banks
constexpr size_t kF32Smem =
    sizeof(double) * kNStats + sizeof(float) * (2 * (size_t)kTile * kF32Pad + kTile);

__global__ void __launch_bounds__(kF32Threads, 1)
    cov_project_f32_kernel(const float* __restrict__ k, const __nv_bfloat16* __restrict__ wext,
                           const Params p) {
  extern __shared__ __align__(16) uint8_t sraw[];
  double* sRed = reinterpret_cast<double*>(sraw);            // [192] column sums of the row
  float* sK = reinterpret_cast<float*>(sraw + kNStats * 8);  // [128][kF32Pad] keys of a head; then y
  float* sW = sK + kTile * kF32Pad;                          // [128][kF32Pad] W_ext columns of a head
  float* sInv = sW + kTile * kF32Pad;                        // [128] 1 / (|k_h| + eps)
  const int tid = threadIdx.x, tr = tid >> 4, tc = tid & 15;
  const long long in = (long long)p.Hkv * kD;
  const long long term = (long long)kNExt * in;
  const long long u0 = unit_begin(blockIdx.x, p.U, gridDim.x);
  const long long u1 = unit_begin(blockIdx.x + 1, p.U, gridDim.x);
  for (int i = tid; i < kNStats; i += kF32Threads) sRed[i] = 0.0;
  auto flush = [&](int bb) {
    __syncthreads();
    for (int i = tid; i < kNStats; i += kF32Threads) {
      p.part[((long long)blockIdx.x * p.B + bb) * kNStats + i] = sRed[i];
      sRed[i] = 0.0;
    }
    __syncthreads();
  };
  int cur_b = -1;
  for (long long u = u0; u < u1; ++u) {
    const int b = (int)(u / p.n_tiles), tile = (int)(u % p.n_tiles);
    if (b != cur_b) {
      if (cur_b >= 0) flush(cur_b);
      cur_b = b;
    }
    float y[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) y[i][j] = 0.f;
    for (int h = 0; h < p.Hkv; ++h) {
      __syncthreads();  // the previous head's (or unit's) readers of sK, sW, sInv are done
      const float* kb = k + ((long long)b * p.Hkv + h) * p.L * kD;
      for (int i = tid; i < kTile * (kD / 4); i += kF32Threads) {
        const int r = i / (kD / 4), c4 = i % (kD / 4);
        const int tok = tile * kTile + r;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (tok < p.L) x = __ldg(reinterpret_cast<const float4*>(kb + (long long)tok * kD) + c4);
        float* dst = sK + r * kF32Pad + 4 * c4;
        dst[0] = x.x;
        dst[1] = x.y;
        dst[2] = x.z;
        dst[3] = x.w;
      }
      for (int i = tid; i < kNExt * kD; i += kF32Threads) {
        const int o = i / kD, e = i % kD;
        const long long g = (long long)o * in + (long long)h * kD + e;
        sW[o * kF32Pad + e] = (__bfloat162float(wext[g]) + __bfloat162float(wext[term + g])) +
                              __bfloat162float(wext[2 * term + g]);
      }
      __syncthreads();
      if (tid < kTile) {
        float ss = 0.f;
        for (int e = 0; e < kD; ++e) {
          const float x = sK[tid * kF32Pad + e];
          ss = fmaf(x, x, ss);
        }
        sInv[tid] = 1.0f / (sqrtf(ss) + 1e-8f);
      }
      float acc[8][8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
#pragma unroll 2
      for (int e = 0; e < kD; ++e) {
        float kv[8], wv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) kv[i] = sK[(tr + 16 * i) * kF32Pad + e];
#pragma unroll
        for (int j = 0; j < 8; ++j) wv[j] = sW[(tc + 16 * j) * kF32Pad + e];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(kv[i], wv[j], acc[i][j]);
      }
      __syncthreads();  // sInv is complete
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float inv = sInv[tr + 16 * i];
#pragma unroll
        for (int j = 0; j < 8; ++j) y[i][j] = fmaf(acc[i][j], inv, y[i][j]);
      }
    }
    // z = y[:64] / (|y[:64]| + eps); zt = y[64:] / (same) = R z
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float nn = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) nn = fmaf(y[i][j], y[i][j], nn);
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) nn += __shfl_xor_sync(0xffffffffu, nn, o);
      const float inv = 1.0f / (sqrtf(nn) + 1e-8f);
#pragma unroll
      for (int j = 0; j < 8; ++j) y[i][j] *= inv;
    }
    __syncthreads();  // the last head's readers of sK are done: sK now holds y
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = tr + 16 * i;
      const int tok = tile * kTile + r;
      const bool valid = tok < p.L;
#pragma unroll
      for (int j = 0; j < 8; ++j) sK[r * kF32Pad + tc + 16 * j] = valid ? y[i][j] : 0.f;
      if (valid) {
        float* zr = p.z + ((long long)b * p.L + tok) * kP;
        float* ztr = p.zt + ((long long)b * p.L + tok) * kP;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          zr[tc + 16 * j] = y[i][j];
          ztr[tc + 16 * j] = y[i][4 + j];
        }
      }
    }
    __syncthreads();
    if (tid < kNStats) {  // columns: sum z (0..63), sum zt (64..127), sum zt^2 (128..191)
      const int c = tid < 2 * kP ? tid : tid - kP;
      float sum = 0.f;
      for (int r = 0; r < kTile; ++r) {
        const float x = sK[r * kF32Pad + c];
        sum += tid < 2 * kP ? x : x * x;
      }
      sRed[tid] += (double)sum;
    }
  }
  if (cur_b >= 0) flush(cur_b);
}

// ---------------------------------------------------------------------------
// Head-sharded caches, one sequence: after the ranks' raw projections are
// summed, each rank finishes the keys of its range.  cov_range_finalize_kernel:
// 128 keys per block, z = y / (|y| + eps), zt = R z (CUDA cores, the rotation
// in f32), and per-block column sums of z, zt, zt^2 in key order;
// cov_range_totals_kernel adds the blocks in order (f64).  Across ranks the
// totals are summed and cov_stats_kernel finishes them as for one GPU.
// ---------------------------------------------------------------------------
constexpr int kRangeKeys = 128;
constexpr int kRangePad = kP + 1;
constexpr size_t kRangeSmem = sizeof(float) * ((size_t)kP * kP + 2 * (size_t)kRangeKeys * kRangePad);

__global__ void __launch_bounds__(kRangeKeys)
    cov_range_finalize_kernel(const float* __restrict__ y, int n, const float* __restrict__ R,
                              float* __restrict__ z, float* __restrict__ zt,
                              float* __restrict__ block_sums) {
  extern __shared__ float sm_range[];
  float* sR = sm_range;                      // [64][64] rotation
  float* sZ = sR + kP * kP;                  // [128][kRangePad] y, then z
  float* sT = sZ + kRangeKeys * kRangePad;   // [128][kRangePad] zt
  const int tid = threadIdx.x;
  const int k0 = blockIdx.x * kRangeKeys;
  for (int i = tid; i < kP * kP; i += kRangeKeys) sR[i] = R[i];
  for (int i = tid; i < kRangeKeys * kP; i += kRangeKeys) {
    const int r = i / kP, c = i % kP;
    sZ[r * kRangePad + c] = (k0 + r < n) ? y[(long long)(k0 + r) * kP + c] : 0.f;
  }
  __syncthreads();
  {
    const int r = tid;
    float nn = 0.f;
    for (int c = 0; c < kP; ++c) nn = fmaf(sZ[r * kRangePad + c], sZ[r * kRangePad + c], nn);
    const float inv = 1.0f / (sqrtf(nn) + 1e-8f);
    for (int c = 0; c < kP; ++c) sZ[r * kRangePad + c] *= inv;
    for (int i = 0; i < kP; ++i) {  // zt_i = sum_j R_ij z_j (features.py:259-261)
      float a = 0.f;
      for (int j = 0; j < kP; ++j) a = fmaf(sR[i * kP + j], sZ[r * kRangePad + j], a);
      sT[r * kRangePad + i] = (k0 + r < n) ? a : 0.f;
    }
    if (k0 + r >= n)
      for (int c = 0; c < kP; ++c) sZ[r * kRangePad + c] = 0.f;
  }
  __syncthreads();
  for (int i = tid; i < kRangeKeys * kP; i += kRangeKeys) {
    const int r = i / kP, c = i % kP;
    if (k0 + r < n) {
      z[(long long)(k0 + r) * kP + c] = sZ[r * kRangePad + c];
      zt[(long long)(k0 + r) * kP + c] = sT[r * kRangePad + c];
    }
  }
  for (int col = tid; col < kNStats; col += kRangeKeys) {
    const float* src = col < kP ? sZ : sT;
    const int c = col < kP ? col : (col < 2 * kP ? col - kP : col - 2 * kP);
    float a = 0.f;
    for (int r = 0; r < kRangeKeys; ++r) {
      const float x = src[r * kRangePad + c];
      a += col < 2 * kP ? x : x * x;
    }
    block_sums[(long long)blockIdx.x * kNStats + col] = a;
  }
}

__global__ void cov_range_totals_kernel(const float* __restrict__ block_sums, int n_blocks,
                                        double* __restrict__ totals) {
  const int col = threadIdx.x;
  if (col >= kNStats) return;
  double a = 0.0;
  for (int i = 0; i < n_blocks; ++i) a += (double)block_sums[(long long)i * kNStats + col];
  totals[col] = a;
}

constexpr int kStatsThreads = 1024;
constexpr int kMaxPartCtas = 256;
constexpr int kStatsChunk = 64;  // CTA partials staged in shared memory per pass (96 KB)

// CTA owning unit u under the contiguous static partition of unit_begin.
__device__ __forceinline__ int cta_of_unit(long long u, long long U, int P) {
  return (int)(((u + 1) * P + U - 1) / U) - 1;
}

// Per batch row: the column sums of the CTAs that covered the row (a
// contiguous CTA range), staged into shared memory with cp.async and summed
// in CTA order (double), then mean z, mu and sigma2_eff (features.py:812,
// :830-845) as floats: stats[b] = [mean z (64) | mu (64) | sigma2_eff (64)].
__global__ void __launch_bounds__(kStatsThreads)
    cov_stats_kernel(const double* __restrict__ part, int grid_ctas, int B, int n_tiles, int L,
                     float rho, float* __restrict__ stats) {
  extern __shared__ __align__(16) double sp[];  // [kStatsChunk][kNStats]
  __shared__ double s[kNStats];
  __shared__ float var[kP];
  const int b = blockIdx.x;
  const int tid = threadIdx.x;
  const long long U = (long long)B * n_tiles;
  const int c_lo = cta_of_unit((long long)b * n_tiles, U, grid_ctas);
  const int c_hi = cta_of_unit((long long)(b + 1) * n_tiles - 1, U, grid_ctas);
  constexpr int kPieces = kNStats * 8 / 16;  // 16-byte pieces of one CTA's partial row
  double acc = 0.0;
  for (int c0 = c_lo; c0 <= c_hi; c0 += kStatsChunk) {
    const int n = min(kStatsChunk, c_hi - c0 + 1);
    const uint32_t d = smem_u32(sp);
    for (int j = tid; j < n * kPieces; j += kStatsThreads) {
      const int cc = j / kPieces, q = j % kPieces;
      cp_async16(d + (uint32_t)(cc * kNStats) * 8u + 16u * q,
                 part + ((long long)(c0 + cc) * B + b) * kNStats + 2 * q);
    }
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
    if (tid < kNStats)
      for (int cc = 0; cc < n; ++cc) acc += sp[cc * kNStats + tid];
    __syncthreads();
  }
  if (tid < kNStats) s[tid] = acc;
  __syncthreads();
  float* out = stats + (long long)b * kNStats;
  if (threadIdx.x < kP) {
    const int i = threadIdx.x;
    out[i] = (float)(s[i] / L);
    const double mu = s[kP + i] / L;
    out[kP + i] = (float)mu;
    const float v = (float)(s[2 * kP + i] / L - mu * mu);
    var[i] = v > 0.f ? v : 0.f;  // clamp_min(0) (features.py:840)
  }
  __syncthreads();
  if (threadIdx.x < kP) {
    double a = 0.0;
    for (int j = 0; j < kP; ++j) a += var[j];
    const float avg = (float)(a / kP);
    out[2 * kP + threadIdx.x] = ((1.0f - rho) * var[threadIdx.x] + rho * avg) + 1e-8f;
  }
}

constexpr int kAssignThreads = 128;  // 32 tokens x 4 threads
constexpr int kProtoStride = 68;     // padded prototype rows: the 4 threads of a token hit distinct banks

// Prototype assignment and g.  Thread `part` of a token scores prototypes
// m = 4 mm + part (mm ascending); ties resolve to the lowest index, as the
// first maximum of argmax does (features.py:177).
__global__ void __launch_bounds__(kAssignThreads)
    cov_assign_kernel(const float* __restrict__ z, const float* __restrict__ zt,
                      const float* __restrict__ stats, const float* __restrict__ protos,
                      int B, int L, int* __restrict__ assign, int* __restrict__ hist,
                      float* __restrict__ features, int stride, int col0, DeviceStatus* status) {
  __shared__ __align__(16) float sP[kNP * kProtoStride];
  __shared__ int sh[kNP];
  const int tid = threadIdx.x;
  {
    const uint32_t d = smem_u32(sP);
    for (int i = tid; i < kNP * kP / 4; i += blockDim.x) {
      const int m = i / (kP / 4), c = i % (kP / 4);
      cp_async16(d + (uint32_t)(m * kProtoStride + 4 * c) * 4u, protos + 4 * i);
    }
    cp_async_commit();
    cp_async_wait_all();
  }
  const long long n = (long long)B * L;
  const long long ngroups = (n + kAssignThreads / 4 - 1) / (kAssignThreads / 4);
  for (long long grp = blockIdx.x; grp < ngroups; grp += gridDim.x) {
    for (int i = tid; i < kNP; i += blockDim.x) sh[i] = 0;
    __syncthreads();
    const long long tok0 = grp * (kAssignThreads / 4);
    const int row0 = (int)(tok0 / L);
    const long long gi = tok0 + (tid >> 2);
    const int part = tid & 3;  // prototypes 4 mm + part; zt dims [16 part, 16 part + 16)
    const bool active = gi < n;
    const int b = active ? (int)(gi / L) : row0;
    const float* st = stats + (long long)b * kNStats;
    float zc[kP];
    float cn2 = 0.f;
    if (active) {
      const float4* src = reinterpret_cast<const float4*>(z + gi * kP);
#pragma unroll
      for (int j = 0; j < kP / 4; ++j) {
        const float4 t = src[j];
        zc[4 * j] = t.x - st[4 * j];
        zc[4 * j + 1] = t.y - st[4 * j + 1];
        zc[4 * j + 2] = t.z - st[4 * j + 2];
        zc[4 * j + 3] = t.w - st[4 * j + 3];
      }
#pragma unroll
      for (int j = 0; j < kP; ++j) cn2 = fmaf(zc[j], zc[j], cn2);
    } else {
#pragma unroll
      for (int j = 0; j < kP; ++j) zc[j] = 0.f;
    }
    const float cn = sqrtf(cn2);
    const bool reliable = cn > 1e-6f;
    const float inv = 1.0f / fmaxf(cn, 1e-6f);
#pragma unroll
    for (int j = 0; j < kP; ++j) zc[j] *= inv;
    // top-2 of this thread's 16 prototypes, ascending index (first maximum
    // wins).  Four prototypes at a time, each cosine its own chain of 64 FMAs
    // in column order (the same sums as one at a time), so the chains overlap.
    float c1 = -INFINITY, c2 = -INFINITY;
    int m1 = part;
#pragma unroll 1
    for (int mg = 0; mg < kNP / 16; ++mg) {
      float c[4] = {0.f, 0.f, 0.f, 0.f};
      const float4* pr[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        pr[q] = reinterpret_cast<const float4*>(sP + (16 * mg + 4 * q + part) * kProtoStride);
#pragma unroll
      for (int j = 0; j < kP / 4; ++j) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 w = pr[q][j];
          c[q] = fmaf(zc[4 * j], w.x, c[q]);
          c[q] = fmaf(zc[4 * j + 1], w.y, c[q]);
          c[q] = fmaf(zc[4 * j + 2], w.z, c[q]);
          c[q] = fmaf(zc[4 * j + 3], w.w, c[q]);
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int m = 16 * mg + 4 * q + part;
        if (c[q] > c1) {
          c2 = c1;
          c1 = c[q];
          m1 = m;
        } else if (c[q] > c2) {
          c2 = c[q];
        }
      }
    }
    // merge across the 4 threads of the token; equal cosines go to the lower index
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      const float oc1 = __shfl_xor_sync(0xffffffffu, c1, off);
      const float oc2 = __shfl_xor_sync(0xffffffffu, c2, off);
      const int om1 = __shfl_xor_sync(0xffffffffu, m1, off);
      if (oc1 > c1 || (oc1 == c1 && om1 < m1)) {
        c2 = fmaxf(c1, oc2);
        c1 = oc1;
        m1 = om1;
      } else {
        c2 = fmaxf(c2, oc1);
      }
    }
    // g over this thread's 16 rotated dims, then summed across the 4 threads
    float gs = 0.f;
    if (active) {
      const float4* src = reinterpret_cast<const float4*>(zt + gi * kP + part * 16);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 t = src[j];
        const float x[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int dd = part * 16 + 4 * j + e;
          const float dv = x[e] - st[kP + dd];
          gs += (dv * dv) / st[2 * kP + dd];
        }
      }
    }
    gs += __shfl_xor_sync(0xffffffffu, gs, 1);
    gs += __shfl_xor_sync(0xffffffffu, gs, 2);
    if (active && part == 0) {
      const float g = log1pf(gs / (float)kP);
      float* out = features + gi * stride + col0;
      out[1] = reliable ? 1.0f - c1 : 1.0f;
      out[2] = reliable ? c1 - c2 : 0.0f;
      out[3] = g;
      assign[gi] = reliable ? m1 : -1;
      if (reliable) {
        if (b == row0) atomicAdd(&sh[m1], 1);
        else atomicAdd(&hist[b * kNP + m1], 1);
      }
      if (!isfinite(c1) || !isfinite(g)) record_error(status, CORE_ERR_NONFINITE, 501, (int)gi);
    }
    __syncthreads();
    for (int m = tid; m < kNP; m += blockDim.x)
      if (sh[m]) atomicAdd(&hist[row0 * kNP + m], sh[m]);
  }
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

// W_ext term t (t = 0..2): bf16 terms of [W ; R W] (128 x C), R W accumulated in double.
__global__ void geometry_prepare_kernel(const float* __restrict__ W, const float* __restrict__ R,
                                        int C, __nv_bfloat16* __restrict__ out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)kNExt * C) return;
  const int r = (int)(i / C), c = (int)(i % C);
  float x;
  if (r < kP) {
    x = W[(long long)r * C + c];
  } else {
    double acc = 0.0;
    for (int k = 0; k < kP; ++k) acc += (double)R[(r - kP) * kP + k] * (double)W[(long long)k * C + c];
    x = (float)acc;
  }
  for (int t = 0; t < 3; ++t) {
    const __nv_bfloat16 h = __float2bfloat16_rn(x);
    out[(long long)t * kNExt * C + i] = h;
    x -= __bfloat162float(h);
  }
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
  const int sms = sm_count() < kMaxPartCtas ? sm_count() : kMaxPartCtas;
  c->grid = (int)(c->p.U < sms ? c->p.U : sms);
}
}  // namespace

extern "C" int core_prepare_geometry(const float* geometry, const float* hadamard, int32_t in_dim,
                                     void* geometry_ext, void* stream) {
  if (geometry == nullptr || hadamard == nullptr || geometry_ext == nullptr || in_dim <= 0)
    return set_error(CORE_ERR_INVALID_ARG, "core_prepare_geometry: bad arguments");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long n = (long long)kNExt * in_dim;
  geometry_prepare_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
      geometry, hadamard, in_dim, static_cast<__nv_bfloat16*>(geometry_ext));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CORE_OK : cuda_error(e, "geometry_prepare_kernel launch");
}

extern "C" size_t core_coverage_workspace_bytes(const core_dims_t* d) {
  if (check_dims(d, "core_coverage_workspace_bytes", true) != CORE_OK) return 0;
  CovPlan c;
  plan_cov(d, &c);
  Sizer z;
  z.take<float>((size_t)d->batch * d->seq_len * kP);       // z
  z.take<float>((size_t)d->batch * d->seq_len * kP);       // zt
  z.take<double>((size_t)c.grid * d->batch * kNStats);     // per-CTA sums
  z.take<float>((size_t)d->batch * kNStats);               // row statistics
  z.take<int>((size_t)d->batch * d->seq_len);              // assignment
  z.take<int>((size_t)d->batch * kNP);                     // histogram
  return z.used;
}

extern "C" int core_coverage_features(const core_dims_t* d, const void* k,
                                      const void* geometry_ext, const float* prototypes,
                                      float shrinkage_rho, float* features, int32_t feature_stride,
                                      int32_t col0, void* workspace, size_t workspace_bytes,
                                      void* stream) {
  int rc = check_dims(d, "core_coverage_features", true);
  if (rc != CORE_OK) return rc;
  if (k == nullptr || geometry_ext == nullptr || prototypes == nullptr || features == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_coverage_features: NULL tensor");
  if (col0 < 0 || col0 + 4 > feature_stride)
    return set_error(CORE_ERR_INVALID_ARG, "core_coverage_features: bad feature columns");
  if (reinterpret_cast<uintptr_t>(prototypes) % 16 != 0)
    return set_error(CORE_ERR_INVALID_ARG, "core_coverage_features: prototypes must be 16-byte aligned");
  CovPlan c;
  plan_cov(d, &c);
  Params& p = c.p;
  Carver cv(workspace, workspace_bytes);
  p.z = cv.take<float>((size_t)p.B * p.L * kP);
  p.zt = cv.take<float>((size_t)p.B * p.L * kP);
  p.part = cv.take<double>((size_t)c.grid * p.B * kNStats);
  float* stats = cv.take<float>((size_t)p.B * kNStats);
  int* assign = cv.take<int>((size_t)p.B * p.L);
  int* hist = cv.take<int>((size_t)p.B * kNP);
  if (cv.overflow) return set_error(CORE_ERR_WORKSPACE, "core_coverage_features: workspace too small");
  p.status = device_status();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(hist, 0, sizeof(int) * (size_t)p.B * kNP, s);
  if (e != cudaSuccess) return cuda_error(e, "coverage histogram clear");

  if (d->dtype == CORE_DTYPE_F32) {
    e = cudaFuncSetAttribute(cov_project_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kF32Smem);
    if (e != cudaSuccess) return cuda_error(e, "cov_project_f32_kernel attribute");
    cov_project_f32_kernel<<<c.grid, kF32Threads, kF32Smem, s>>>(
        static_cast<const float*>(k), static_cast<const __nv_bfloat16*>(geometry_ext), p);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "cov_project_f32_kernel launch");
  } else {
  CUtensorMap tmK, tmW;
  {
    uint64_t dims[3] = {128, (uint64_t)p.L, (uint64_t)p.B * p.Hkv};
    uint64_t str[2] = {256, (uint64_t)p.L * 256};
    uint32_t box[3] = {64, 128, 1};
    if ((rc = make_tmap_bf16(&tmK, k, 3, dims, str, box, true)) != CORE_OK) return rc;
  }
  {
    const uint64_t in = (uint64_t)p.Hkv * kD;
    uint64_t dims[2] = {in, 3u * kNExt};
    uint64_t str[1] = {in * 2};
    uint32_t box[2] = {64, (uint32_t)kNExt};
    if ((rc = make_tmap_bf16(&tmW, geometry_ext, 2, dims, str, box, true)) != CORE_OK) return rc;
  }
  const uint32_t smem = Smem::kTotal + 1024;
  e = cudaFuncSetAttribute(cov_project_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_error(e, "cov_project_kernel attribute");
  cov_project_kernel<<<c.grid, kThreads, smem, s>>>(tmK, tmW, p);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "cov_project_kernel launch");
  }
  {
    const size_t smem = sizeof(double) * kStatsChunk * kNStats;
    e = cudaFuncSetAttribute(cov_stats_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_error(e, "cov_stats_kernel attribute");
    cov_stats_kernel<<<p.B, kStatsThreads, smem, s>>>(p.part, c.grid, p.B, p.n_tiles, p.L,
                                                      shrinkage_rho, stats);
  }
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "cov_stats_kernel launch");
  const long long n = (long long)p.B * p.L;
  long long ablocks = (n + kAssignThreads / 4 - 1) / (kAssignThreads / 4);
  if (ablocks > 4LL * sm_count()) ablocks = 4LL * sm_count();
  cov_assign_kernel<<<(unsigned)ablocks, kAssignThreads, 0, s>>>(p.z, p.zt, stats, prototypes, p.B,
                                                                 p.L, assign, hist, features,
                                                                 feature_stride, col0, p.status);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "cov_assign_kernel launch");
  cov_occupancy_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(assign, hist, p.B, p.L, features,
                                                                  feature_stride, col0);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "cov_occupancy_kernel launch");
  return CORE_OK;
}

// ---------------------------------------------------------------------------
// Head-sharded caches (one sequence; each rank holds some KV heads).
// ---------------------------------------------------------------------------
extern "C" int core_coverage_partial_projection(const core_dims_t* d, const void* k,
                                                const void* geometry_ext, float* y,
                                                void* workspace, size_t workspace_bytes,
                                                void* stream) {
  int rc = check_dims(d, "core_coverage_partial_projection");
  if (rc != CORE_OK) return rc;
  if (k == nullptr || geometry_ext == nullptr || y == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_coverage_partial_projection: NULL tensor");
  if (reinterpret_cast<uintptr_t>(y) % 16 != 0)
    return set_error(CORE_ERR_INVALID_ARG, "core_coverage_partial_projection: y must be 16-byte aligned");
  CovPlan c;
  plan_cov(d, &c);
  Params& p = c.p;
  p.partial = 1;
  Carver cv(workspace, workspace_bytes);
  p.part = cv.take<double>((size_t)c.grid * p.B * kNStats);
  if (cv.overflow)
    return set_error(CORE_ERR_WORKSPACE, "core_coverage_partial_projection: workspace too small");
  p.z = y;
  p.zt = nullptr;
  p.status = device_status();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap tmK, tmW;
  {
    uint64_t dims[3] = {128, (uint64_t)p.L, (uint64_t)p.B * p.Hkv};
    uint64_t str[2] = {256, (uint64_t)p.L * 256};
    uint32_t box[3] = {64, 128, 1};
    if ((rc = make_tmap_bf16(&tmK, k, 3, dims, str, box, true)) != CORE_OK) return rc;
  }
  {
    const uint64_t in = (uint64_t)p.Hkv * kD;
    uint64_t dims[2] = {in, 3u * kNExt};
    uint64_t str[1] = {in * 2};
    uint32_t box[2] = {64, (uint32_t)kNExt};
    if ((rc = make_tmap_bf16(&tmW, geometry_ext, 2, dims, str, box, true)) != CORE_OK) return rc;
  }
  const uint32_t smem = Smem::kTotal + 1024;
  cudaError_t e = cudaFuncSetAttribute(cov_project_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_error(e, "cov_project_kernel attribute");
  cov_project_kernel<<<c.grid, kThreads, smem, s>>>(tmK, tmW, p);
  e = cudaGetLastError();
  return e == cudaSuccess ? CORE_OK : cuda_error(e, "cov_project_kernel launch");
}

extern "C" size_t core_coverage_range_workspace_bytes(int32_t n_keys) {
  Sizer z;
  z.take<float>((size_t)((n_keys + kRangeKeys - 1) / kRangeKeys) * kNStats);  // block sums
  z.take<float>((size_t)kNStats);                                            // statistics
  return z.used;
}

extern "C" int core_coverage_range_totals(const float* y, int32_t n_keys, const float* hadamard,
                                          float* z, float* zt, double* totals, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  if (y == nullptr || hadamard == nullptr || z == nullptr || zt == nullptr || totals == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_coverage_range_totals: NULL tensor");
  if (n_keys < 0) return set_error(CORE_ERR_INVALID_ARG, "core_coverage_range_totals: n_keys < 0");
  Carver cv(workspace, workspace_bytes);
  const int n_blocks = (n_keys + kRangeKeys - 1) / kRangeKeys;
  float* bs = cv.take<float>((size_t)(n_blocks > 0 ? n_blocks : 1) * kNStats);
  if (cv.overflow) return set_error(CORE_ERR_WORKSPACE, "core_coverage_range_totals: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (n_blocks > 0) {
    e = cudaFuncSetAttribute(cov_range_finalize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kRangeSmem);
    if (e != cudaSuccess) return cuda_error(e, "cov_range_finalize_kernel attribute");
    cov_range_finalize_kernel<<<n_blocks, kRangeKeys, kRangeSmem, s>>>(y, n_keys, hadamard, z, zt, bs);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "cov_range_finalize_kernel launch");
  }
  cov_range_totals_kernel<<<1, 256, 0, s>>>(bs, n_blocks, totals);
  e = cudaGetLastError();
  return e == cudaSuccess ? CORE_OK : cuda_error(e, "cov_range_totals_kernel launch");
}

extern "C" int core_coverage_range_assign(const double* totals, int32_t seq_len, float shrinkage_rho,
                                          const float* z, const float* zt, int32_t n_keys,
                                          const float* prototypes, int32_t* assign, int32_t* hist,
                                          float* features, int32_t feature_stride, int32_t col0,
                                          void* workspace, size_t workspace_bytes, void* stream) {
  if (totals == nullptr || z == nullptr || zt == nullptr || prototypes == nullptr ||
      assign == nullptr || hist == nullptr || features == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_coverage_range_assign: NULL tensor");
  if (seq_len <= 0 || n_keys < 0 || n_keys > seq_len || col0 < 0 || col0 + 4 > feature_stride)
    return set_error(CORE_ERR_INVALID_ARG, "core_coverage_range_assign: bad sizes");
  if (reinterpret_cast<uintptr_t>(totals) % 16 != 0 || reinterpret_cast<uintptr_t>(prototypes) % 16 != 0)
    return set_error(CORE_ERR_INVALID_ARG, "core_coverage_range_assign: totals and prototypes must be 16-byte aligned");
  Carver cv(workspace, workspace_bytes);
  const int n_blocks = (n_keys + kRangeKeys - 1) / kRangeKeys;
  cv.take<float>((size_t)(n_blocks > 0 ? n_blocks : 1) * kNStats);
  float* stats = cv.take<float>((size_t)kNStats);
  if (cv.overflow) return set_error(CORE_ERR_WORKSPACE, "core_coverage_range_assign: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(hist, 0, sizeof(int) * kNP, s);
  if (e != cudaSuccess) return cuda_error(e, "coverage histogram clear");
  {
    // the summed totals are one "CTA" covering the whole sequence
    const size_t smem = sizeof(double) * kStatsChunk * kNStats;
    e = cudaFuncSetAttribute(cov_stats_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_error(e, "cov_stats_kernel attribute");
    cov_stats_kernel<<<1, kStatsThreads, smem, s>>>(totals, 1, 1, 1, seq_len, shrinkage_rho, stats);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "cov_stats_kernel launch");
  }
  if (n_keys == 0) return CORE_OK;
  long long ablocks = ((long long)n_keys + kAssignThreads / 4 - 1) / (kAssignThreads / 4);
  if (ablocks > 4LL * sm_count()) ablocks = 4LL * sm_count();
  cov_assign_kernel<<<(unsigned)ablocks, kAssignThreads, 0, s>>>(z, zt, stats, prototypes, 1, n_keys,
                                                                 assign, hist, features,
                                                                 feature_stride, col0, device_status());
  e = cudaGetLastError();
  return e == cudaSuccess ? CORE_OK : cuda_error(e, "cov_assign_kernel launch");
}

extern "C" int core_coverage_range_occupancy(const int32_t* assign, const int32_t* hist,
                                             int32_t n_keys, float* features,
                                             int32_t feature_stride, int32_t col0, void* stream) {
  if (assign == nullptr || hist == nullptr || features == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_coverage_range_occupancy: NULL tensor");
  if (n_keys < 0 || col0 < 0 || col0 + 4 > feature_stride)
    return set_error(CORE_ERR_INVALID_ARG, "core_coverage_range_occupancy: bad sizes");
  if (n_keys == 0) return CORE_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cov_occupancy_kernel<<<(unsigned)((n_keys + 127) / 128), 128, 0, s>>>(assign, hist, 1, n_keys,
                                                                        features, feature_stride, col0);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CORE_OK : cuda_error(e, "cov_occupancy_kernel launch");
}
