// Latent-memory write and decayed recurrence
// (replaces core/kvpress_adapter.py:1041-1202, pre_o_proj value space).
//
//   mw_mass_kernel   : p = softmax(s / tau) over the whole cache, pi_E = sum of
//                      p over evicted tokens, p_bar = p / pi_E on the evicted
//                      list (core/indexer.py:55-72, :247-273); Z <- gamma Z + pi_E.
//   mw_phi_kernel    : phi^T = Theta_f K_ev^T for 128 memory rows x 128 gathered
//                      evicted tokens on tcgen05 (Theta_f as two bf16 terms by
//                      TMA, K rows gathered with cp.async into swizzled shared
//                      memory, K exact in bf16, four stages), epilogue
//                      W^T = p_bar * phi^T written as bf16 hi/lo in (d_mem,
//                      token) order and per-row sums of p_bar * phi^2 (b_bar
//                      partials).
//   mw_mbar_kernel   : M_bar partial = W^T V_ev on tcgen05 (A = W tiles by TMA,
//                      B = gathered V rows, MN-major), split over token chunks.
//   mw_update_kernel : M, b <- (gamma Z M + pi_E eta M_bar) / (Z' + eps).
#include <cooperative_groups.h>

#include <cmath>

#include "common.cuh"
#include "host_util.h"

namespace cg = cooperative_groups;

namespace core {
namespace mw {

constexpr int kD = 128;
constexpr int kTok = 128;         // evicted tokens per phi unit (MMA N)
constexpr int kProdThreads = 128; // 4 gathering warps
constexpr int kMbarChunk = 64;    // tokens per M_bar K chunk


// ===========================================================================
// softmax mass
// ===========================================================================
constexpr int kMassMaxSmem = 49152;  // exp terms of rows up to this length stay in shared memory

template <bool kSmem>
__global__ void __launch_bounds__(1024)
    mw_mass_kernel(const float* __restrict__ scores, int L, const int* __restrict__ evict,
                   int n_evict, int n_ev_pad, float tau, float gamma, float* __restrict__ Z,
                   float* __restrict__ pbar, float* __restrict__ coef, DeviceStatus* status) {
  extern __shared__ float se[];  // x_i = s_i / tau, then exp(x_i - max)  (kSmem only)
  const int b = blockIdx.x;
  const float* s = scores + (long long)b * L;
  __shared__ float red[32];
  __shared__ double redd[32];
  __shared__ float s_max, s_sum;
  __shared__ double s_pie;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool unit_tau = tau == 1.0f;  // s / 1 is exact: skip the division
  auto scaled = [&](int i) { return unit_tau ? s[i] : s[i] / tau; };
  float m = -INFINITY;
#pragma unroll 8
  for (int i = threadIdx.x; i < L; i += blockDim.x) {
    const float x = scaled(i);
    if constexpr (kSmem) se[i] = x;
    m = fmaxf(m, x);
  }
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = red[0];
    for (int w = 1; w < (int)(blockDim.x / 32); ++w) mm = fmaxf(mm, red[w]);
    s_max = mm;
  }
  __syncthreads();
  const float mx = s_max;
  double sum = 0.0;
#pragma unroll 8
  for (int i = threadIdx.x; i < L; i += blockDim.x) {
    float e;
    if constexpr (kSmem) {
      e = expf(se[i] - mx);
      se[i] = e;
    } else {
      e = expf(scaled(i) - mx);
    }
    sum += (double)e;
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) redd[warp] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x / 32); ++w) t += redd[w];
    s_sum = (float)t;
  }
  __syncthreads();
  const float tot = s_sum;
  const int* ev = evict + (long long)b * n_evict;
  auto ex = [&](int i) -> float {
    if ((unsigned)i >= (unsigned)L) {  // evicted index outside the cache
      record_error(status, CORE_ERR_INVALID_ARG, 802, i);
      return 0.f;
    }
    if constexpr (kSmem) return se[i];
    else return expf(scaled(i) - mx);
  };
  double pe = 0.0;
#pragma unroll 8
  for (int k = threadIdx.x; k < n_evict; k += blockDim.x) pe += (double)(ex(ev[k]) / tot);
  for (int o = 16; o > 0; o >>= 1) pe += __shfl_xor_sync(0xffffffffu, pe, o);
  if (lane == 0) redd[warp] = pe;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x / 32); ++w) t += redd[w];
    s_pie = t;
  }
  __syncthreads();
  const float pie = (float)s_pie;
  const float mass = pie > 0.f ? pie : 1.0f;
  float* pb = pbar + (long long)b * n_ev_pad;
#pragma unroll 8
  for (int k = threadIdx.x; k < n_ev_pad; k += blockDim.x) {
    float v = 0.f;
    if (k < n_evict) v = (ex(ev[k]) / tot) / mass;
    pb[k] = v;
  }
  if (threadIdx.x == 0) {
    const float gz = gamma * Z[b];
    const float zt = gz + pie;
    coef[b * 3 + 0] = gz;
    coef[b * 3 + 1] = pie;
    coef[b * 3 + 2] = zt + 1e-8f;
    Z[b] = zt;
    if (!isfinite(pie) || !isfinite(tot)) record_error(status, CORE_ERR_NONFINITE, 801, b);
  }
}

// Long rows: the same softmax mass on one cluster of kMassCluster CTAs per
// batch row.  CTA c caches exp(x_i - max) of tokens [c Lc, (c + 1) Lc) in its
// shared memory; the maximum, the f64 sums and pi_E are combined across the
// cluster in CTA order, and the evicted list (split evenly over the CTAs)
// reads each term from the CTA that holds it through distributed shared
// memory.  Same arithmetic per term as mw_mass_kernel; only the order of the
// f64 partial sums differs.
constexpr int kMassCluster = 8;
constexpr int kMassClusterMinLen = 8192;  // shorter rows: one CTA

__device__ __forceinline__ double block_sum_f64(double v, double* red, int lane, int warp) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < (int)(blockDim.x / 32); ++w) t += red[w];
  return t;
}

__global__ void __cluster_dims__(kMassCluster, 1, 1) __launch_bounds__(1024)
    mw_mass_cluster_kernel(const float* __restrict__ scores, int L, const int* __restrict__ evict,
                           int n_evict, int n_ev_pad, float tau, float gamma,
                           float* __restrict__ Z, float* __restrict__ pbar,
                           float* __restrict__ coef, DeviceStatus* status) {
  extern __shared__ float se[];  // exp(x_i - max) of this CTA's tokens
  cg::cluster_group cluster = cg::this_cluster();
  const int cr = (int)cluster.block_rank();
  const int b = blockIdx.x / kMassCluster;
  const float* s = scores + (long long)b * L;
  const int Lc = (L + kMassCluster - 1) / kMassCluster;
  const int lo = min(L, cr * Lc), hi = min(L, lo + Lc);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __shared__ float redf[32];
  __shared__ double redd[32];
  __shared__ float s_part_max;
  __shared__ double s_part_sum, s_part_pe;
  const bool unit_tau = tau == 1.0f;
  // ---- maximum ----
  float m = -INFINITY;
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float x = unit_tau ? s[i] : s[i] / tau;
    se[i - lo] = x;
    m = fmaxf(m, x);
  }
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) redf[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = redf[0];
    for (int w = 1; w < (int)(blockDim.x / 32); ++w) mm = fmaxf(mm, redf[w]);
    s_part_max = mm;
  }
  cluster.sync();
  float mx = -INFINITY;
  for (int c = 0; c < kMassCluster; ++c) mx = fmaxf(mx, *cluster.map_shared_rank(&s_part_max, c));
  // ---- sum of the exps ----
  double sum = 0.0;
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float e = expf(se[i - lo] - mx);
    se[i - lo] = e;
    sum += (double)e;
  }
  sum = block_sum_f64(sum, redd, lane, warp);
  if (threadIdx.x == 0) s_part_sum = sum;
  cluster.sync();
  double tot_d = 0.0;
  for (int c = 0; c < kMassCluster; ++c) tot_d += *cluster.map_shared_rank(&s_part_sum, c);
  const float tot = (float)tot_d;
  // ---- evicted mass: CTA c takes evicted entries [c Kc, (c + 1) Kc) ----
  const int* ev = evict + (long long)b * n_evict;
  float* pb = pbar + (long long)b * n_ev_pad;
  const int Kc = (n_evict + kMassCluster - 1) / kMassCluster;
  const int k_lo = min(n_evict, cr * Kc), k_hi = min(n_evict, k_lo + Kc);
  double pe = 0.0;
  for (int k = k_lo + threadIdx.x; k < k_hi; k += blockDim.x) {
    const int i = ev[k];
    float p = 0.f;
    if ((unsigned)i >= (unsigned)L) {  // evicted index outside the cache
      record_error(status, CORE_ERR_INVALID_ARG, 802, i);
    } else {
      const float e = cluster.map_shared_rank(se, i / Lc)[i % Lc];
      p = e / tot;
    }
    pb[k] = p;
    pe += (double)p;
  }
  pe = block_sum_f64(pe, redd, lane, warp);
  if (threadIdx.x == 0) s_part_pe = pe;
  cluster.sync();
  double pie_d = 0.0;
  for (int c = 0; c < kMassCluster; ++c) pie_d += *cluster.map_shared_rank(&s_part_pe, c);
  const float pie = (float)pie_d;
  const float mass = pie > 0.f ? pie : 1.0f;
  for (int k = k_lo + threadIdx.x; k < k_hi; k += blockDim.x) pb[k] = pb[k] / mass;
  if (cr == kMassCluster - 1)
    for (int k = n_evict + threadIdx.x; k < n_ev_pad; k += blockDim.x) pb[k] = 0.f;
  if (cr == 0 && threadIdx.x == 0) {
    const float gz = gamma * Z[b];
    const float zt = gz + pie;
    coef[b * 3 + 0] = gz;
    coef[b * 3 + 1] = pie;
    coef[b * 3 + 2] = zt + 1e-8f;
    Z[b] = zt;
    if (!isfinite(pie) || !isfinite(tot)) record_error(status, CORE_ERR_NONFINITE, 801, b);
  }
  cluster.sync();  // no CTA leaves while another may still read its shared memory
}

// ===========================================================================
// phi tile: W = p_bar * (K_ev Theta_f^T), b_bar partials
// ===========================================================================
struct PhiParams {
  int B, Hkv, L, n_evict, n_ev_pad, n_et, d_mem, d_pad, n_dh;
  long long U;
  const __nv_bfloat16* k;
  const int* evict;
  const float* pbar;
  __nv_bfloat16* wt;   // (2, d_pad, n_ev_pad)
  float* bpart;        // (B, n_et, d_pad)
  DeviceStatus* status;
};

// phi^T tile: M = 128 memory rows of Theta_f (A, two bf16 terms, TMA) x N = 128
// gathered evicted tokens (B, cp.async), K = the 1024-wide key row in 64-column
// chunks, two chunks per pipeline stage.  TMEM lanes are memory rows, columns
// are tokens, so the epilogue writes W^T rows with contiguous token runs and
// sums b_bar along its own row.  A stage carries 96 KB: a stage ring pays a
// fixed synchronisation cost per stage, so fewer, larger stages stream faster.
constexpr int kPhiRows = 128;                    // memory rows per unit (MMA M)
constexpr int kPhiCps = 2;                       // 64-column K chunks per stage
constexpr uint32_t kPhiA = 2u * kPhiRows * 128;  // 32 KB: two Theta terms x 128 rows x 64 columns
constexpr uint32_t kPhiB = kTok * 128;           // 16 KB: 128 tokens x 64 columns
constexpr uint32_t kPhiStage = kPhiCps * (kPhiA + kPhiB);  // [A c0][A c1][B c0][B c1]
constexpr int kPhiStages = 2;
constexpr int kPhiThreads = 512;         // warps 0-3 gather, 4 MMA, 8-15 epilogue
constexpr uint32_t kPhiSmem = kPhiStages * kPhiStage + 2 * kTok * 4 + 256 + 1024;

// K chunk pair processed at step ci of a unit of token tile et: each token
// tile starts at its own pair, so that the CTAs stream different Theta tiles
// at any moment instead of all reading the same lines of L2.  The order
// depends on the tile only, not on the grid.
__device__ __forceinline__ int phi_pair(int ci, int et, int n) {
  const int c = ci + et % n;
  return c < n ? c : c - n;
}

__global__ void __launch_bounds__(kPhiThreads, 1)
    mw_phi_kernel(const __grid_constant__ CUtensorMap tmT, const PhiParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  const uint32_t aux_off = kPhiStages * kPhiStage;
  float* s_pbar = reinterpret_cast<float*>(sgen + aux_off);  // [128] p_bar of the unit's tokens
  float* s_bh = s_pbar + kTok;                                // [128] team-1 b_bar halves
  const uint32_t bar = sbase + aux_off + 2 * kTok * 4;
  auto bar_full = [&](int s) { return bar + 8u * s; };
  auto bar_empty = [&](int s) { return bar + 8u * (kPhiStages + s); };
  auto bar_tfull = [&](int s) { return bar + 8u * (2 * kPhiStages + s); };
  auto bar_tempty = [&](int s) { return bar + 8u * (2 * kPhiStages + 2 + s); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + aux_off + 2 * kTok * 4 + 200);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sgen + aux_off + 2 * kTok * 4 + 208);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = gridDim.x;
  const long long u0 = (long long)blockIdx.x * p.U / P, u1 = (long long)(blockIdx.x + 1) * p.U / P;
  const int n_pairs = p.Hkv;  // pairs of 64-column K chunks = heads of the 1024-wide key row

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPhiStages; ++s) {
      mbar_init(bar_full(s), 1 + kProdThreads);  // TMA expect_tx + every gathering thread
      mbar_init(bar_empty(s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar_tfull(s), 1);
      mbar_init(bar_tempty(s), 8);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 4) {
    tmem_alloc(smem_u32(tmem_slot), 2 * kTok);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto wait = [&](uint32_t b, uint32_t parity, int where) -> bool {
    return bounded_wait(b, parity, abort_flag, p.status, where);
  };
  if (warp < 4) {
    // ---- producers: Theta by TMA (thread 0), token rows gathered with cp.async ----
    const int tid = threadIdx.x;
    int it = 0;
    bool ok = true;
    for (long long u = u0; u < u1 && ok; ++u) {
      const int dt = (int)(u % p.n_dh);
      const long long rest = u / p.n_dh;
      const int et = (int)(rest % p.n_et), b = (int)(rest / p.n_et);
      // the unit's 128 token rows serve all its K chunks: indices loaded once
      // (8 rows per thread: r = tid / 8 + 16 i)
      constexpr int kPer = kTok * 8 / kProdThreads;
      int toks[kPer];
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int kidx = et * kTok + ((tid + i * kProdThreads) >> 3);
        // an index outside the cache (error 802 of the mass kernel) gathers a zero row
        // evict NULL: the rows are already gathered (row kidx is evicted token kidx)
        const int ix = kidx < p.n_evict
                           ? (p.evict != nullptr ? p.evict[(long long)b * p.n_evict + kidx] : kidx)
                           : -1;
        toks[i] = (unsigned)ix < (unsigned)p.L ? ix : -1;
      }
      for (int ci = 0; ci < n_pairs && ok; ++ci, ++it) {
        const int h = phi_pair(ci, et, n_pairs);  // this stage: head h, both 64-column halves
        const int st = it % kPhiStages;
        if (it >= kPhiStages && !(ok = wait(bar_empty(st), ((it / kPhiStages) - 1) & 1, 901))) break;
        const uint32_t s_base = sbase + st * kPhiStage;
        if (tid == 0) {
          mbar_arrive_expect_tx(bar_full(st), kPhiCps * kPhiA);
          for (int half = 0; half < kPhiCps; ++half)
            for (int t = 0; t < 2; ++t)
              tma_load_3d(s_base + half * kPhiA + t * (kPhiRows * 128u), &tmT, bar_full(st),
                          (2 * h + half) * 64, dt * kPhiRows, t);
        }
        // 2 halves x 128 rows x 8 sixteen-byte pieces = 2048 copies, 16 per
        // thread; rows outside the cache are zero-filled by the same copies
#pragma unroll
        for (int half = 0; half < kPhiCps; ++half) {
#pragma unroll
          for (int i = 0; i < kPer; ++i) {
            const int j = tid + i * kProdThreads;
            const int r = j >> 3, q = j & 7;
            const uint32_t dst = s_base + kPhiCps * kPhiA + half * kPhiB + (uint32_t)r * 128u +
                                 (uint32_t)((q ^ (r & 7)) << 4);
            const __nv_bfloat16* src =
                toks[i] >= 0 ? p.k + (((long long)b * p.Hkv + h) * p.L + toks[i]) * kD + half * 64 + q * 8
                             : p.k;
            cp_async16_zfill(dst, src, toks[i] >= 0);
          }
        }
        // the stage fills when every producer's copies have landed; the thread
        // goes on to the next stage without waiting for them
        cp_async_mbar_arrive(bar_full(st));
      }
    }
    cp_async_wait_all();
  } else if (warp == 4) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(kPhiRows, kTok, 0, 0);
      int it = 0, sub = 0;
      bool ok = true;
      for (long long u = u0; u < u1 && ok; ++u, ++sub) {
        const int buf = sub & 1, n = sub >> 1;
        if (sub >= 2 && !(ok = wait(bar_tempty(buf), (n - 1) & 1, 902))) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * kTok);
        for (int ci = 0; ci < n_pairs && ok; ++ci, ++it) {
          const int st = it % kPhiStages;
          if (!(ok = wait(bar_full(st), (it / kPhiStages) & 1, 903))) break;
          fence_proxy_async_shared();  // gathered rows (cp.async) before the MMA reads them
          tc_fence_after();
          const uint32_t s_base = sbase + st * kPhiStage;
          for (int half = 0; half < kPhiCps; ++half) {
            for (int ks = 0; ks < 4; ++ks) {
              const uint64_t bd = sdesc_kmajor(s_base + kPhiCps * kPhiA + half * kPhiB + (uint32_t)ks * 32u);
              for (int t = 0; t < 2; ++t) {
                const uint64_t a = sdesc_kmajor(s_base + half * kPhiA + (uint32_t)t * kPhiRows * 128u +
                                                (uint32_t)ks * 32u);
                mma_bf16(d, a, bd, idesc, (ci > 0 || half > 0 || ks > 0 || t > 0) ? 1u : 0u);
              }
            }
          }
          mma_commit(bar_empty(st));
        }
        if (ok) mma_commit(bar_tfull(buf));
      }
    }
  } else if (warp >= 8) {
    // ---- epilogue: lanes are memory rows, columns tokens ----
    const int team = (warp - 8) >> 2;  // token half [64 team, 64 team + 64)
    const int wq = warp & 3;
    const int row = wq * 32 + lane;    // memory row inside the unit
    const int etid = threadIdx.x - 256;
    int sub = 0;
    for (long long u = u0; u < u1; ++u, ++sub) {
      const int dt = (int)(u % p.n_dh);
      const long long rest = u / p.n_dh;
      const int et = (int)(rest % p.n_et), b = (int)(rest / p.n_et);
      named_barrier(1, 256);  // the previous unit's readers of s_pbar / s_bh are done
      if (etid < kTok) s_pbar[etid] = p.pbar[(long long)b * p.n_ev_pad + et * kTok + etid];
      const int buf = sub & 1, n = sub >> 1;
      const bool got = wait(bar_tfull(buf), n & 1, 904);
      if (!named_barrier_and(1, 256, got)) break;  // uniform: every epilogue warp stops together
      tc_fence_after();
      const int drow = dt * kPhiRows + row;  // row of W^T and b_bar (< d_pad)
      float bsum = 0.f;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int t0 = team * 64 + q * 32;  // first token column of the chunk
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(wq * 32) << 16) + (uint32_t)(buf * kTok + t0), v);
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float pb0 = s_pbar[t0 + j], pb1 = s_pbar[t0 + j + 1];
          const float w0 = v[j] * pb0, w1 = v[j + 1] * pb1;  // phi * w (kvpress_adapter.py:1155)
          bsum += (v[j] * v[j]) * pb0;                        // (phi*phi) * w (:1157)
          bsum += (v[j + 1] * v[j + 1]) * pb1;
          __nv_bfloat162 hh = __floats2bfloat162_rn(w0, w1);
          const uint32_t hw = *reinterpret_cast<uint32_t*>(&hh);
          __nv_bfloat162 ll = __floats2bfloat162_rn(w0 - __uint_as_float(hw << 16),
                                                    w1 - __uint_as_float(hw & 0xFFFF0000u));
          hi[j >> 1] = hw;
          lo[j >> 1] = *reinterpret_cast<uint32_t*>(&ll);
        }
        // 32 tokens of one W^T row: 64 contiguous bytes per term
        __nv_bfloat16* dst = p.wt + (long long)drow * p.n_ev_pad + et * kTok + t0;
        uint4* d0 = reinterpret_cast<uint4*>(dst);
        uint4* d1 = reinterpret_cast<uint4*>(dst + (long long)p.d_pad * p.n_ev_pad);
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          d0[w] = make_uint4(hi[4 * w], hi[4 * w + 1], hi[4 * w + 2], hi[4 * w + 3]);
          d1[w] = make_uint4(lo[4 * w], lo[4 * w + 1], lo[4 * w + 2], lo[4 * w + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_tempty(buf));
      // b_bar partial of this row over the unit's tokens: the two halves in a fixed order
      if (team == 1) s_bh[row] = bsum;
      named_barrier(1, 256);
      if (team == 0) p.bpart[((long long)b * p.n_et + et) * p.d_pad + drow] = bsum + s_bh[row];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kTok);
  }
}

// ===========================================================================
// M_bar partial = W^T V_ev over one token range, one (128 x 256) output tile
// ===========================================================================
struct MbarParams {
  int Hkv, L, n_evict, n_ev_pad, d_pad, kvw, n_jt, n_ct, splits;
  long long split_stride;  // elements between consecutive splits of mpart
  const __nv_bfloat16* v;  // this batch row's values (Hkv, L, d)
  const int* evict;        // this batch row's evicted indices
  float* mpart;            // this batch row's (d_pad, kvw) slice of split 0
  DeviceStatus* status;
};

constexpr uint32_t kMbA = 2u * 128 * 128;           // two terms x 128 rows x 64 tokens
constexpr uint32_t kMbBMax = 4u * kMbarChunk * 128; // up to 4 MN atoms x 64 token rows x 128 B
constexpr uint32_t kMbStage = kMbA + kMbBMax;       // 64 KB
constexpr int kMbStages = 3;
constexpr int kMbThreads = 384;  // warps 0-3 gather, 4 MMA, 8-11 epilogue

// CT = value columns per output tile (256, or 128 when Hkv*d is an odd
// multiple of 128).
template <int CT>
__global__ void __launch_bounds__(kMbThreads, 1)
    mw_mbar_kernel(const __grid_constant__ CUtensorMap tmW, const MbarParams p) {
  constexpr int kAtoms = CT / 64;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  const uint32_t bar = sbase + kMbStages * kMbStage;
  auto bar_full = [&](int s) { return bar + 8u * s; };
  auto bar_empty = [&](int s) { return bar + 8u * (kMbStages + s); };
  const uint32_t bar_done = bar + 8u * (2 * kMbStages);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + kMbStages * kMbStage + 200);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sgen + kMbStages * kMbStage + 208);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // unit = (split, jt, ct), one per CTA
  long long u = blockIdx.x;
  const int ct = (int)(u % p.n_ct); u /= p.n_ct;
  const int jt = (int)(u % p.n_jt);
  const int split = (int)(u / p.n_jt);
  const int n_kc = p.n_ev_pad / kMbarChunk;
  const int kc0 = (int)((long long)split * n_kc / p.splits);
  const int kc1 = (int)((long long)(split + 1) * n_kc / p.splits);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kMbStages; ++s) {
      mbar_init(bar_full(s), 1 + kProdThreads);  // TMA expect_tx + every gathering thread
      mbar_init(bar_empty(s), 1);
    }
    mbar_init(bar_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 4) {
    tmem_alloc(smem_u32(tmem_slot), 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  static_assert(CT == 128 || CT == 256, "tile width");
  auto wait = [&](uint32_t bb, uint32_t parity, int where) -> bool {
    return bounded_wait(bb, parity, abort_flag, p.status, where);
  };

  if (warp < 4) {
    const int tid = threadIdx.x;
    bool ok = true;
    constexpr int kPer = kMbarChunk * kAtoms * 8 / kProdThreads;
    // token indices of chunk kc (the rows this thread gathers); the loads of
    // the next chunk's indices are issued one chunk ahead, so their latency
    // overlaps the current chunk instead of stalling every chunk
    auto load_idx = [&](int kc, int (&dst)[kPer]) {
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int kidx = kc * kMbarChunk + (tid + i * kProdThreads) / (kAtoms * 8);
        dst[i] = kidx < p.n_evict ? (p.evict != nullptr ? p.evict[kidx] : kidx) : -1;
      }
    };
    int nxt[kPer];
    if (kc0 < kc1) load_idx(kc0, nxt);
    for (int kc = kc0, it = 0; kc < kc1 && ok; ++kc, ++it) {
      const int st = it % kMbStages;
      int toks[kPer];
#pragma unroll
      for (int i = 0; i < kPer; ++i)
        toks[i] = (unsigned)nxt[i] < (unsigned)p.L ? nxt[i] : -1;  // outside the cache: zero row
      if (kc + 1 < kc1) load_idx(kc + 1, nxt);
      if (it >= kMbStages && !(ok = wait(bar_empty(st), ((it / kMbStages) - 1) & 1, 911))) break;
      const uint32_t base = sbase + st * kMbStage;
      if (tid == 0) {
        mbar_arrive_expect_tx(bar_full(st), kMbA);
        for (int t = 0; t < 2; ++t)
          tma_load_2d(base + t * (128u * 128u), &tmW, bar_full(st), kc * kMbarChunk,
                      t * p.d_pad + jt * 128);
      }
      // 64 token rows x kAtoms MN atoms x 8 pieces (rows outside the cache zero-filled)
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int j = tid + i * kProdThreads;
        const int r = j / (kAtoms * 8), a = (j >> 3) % kAtoms, q = j & 7;
        const uint32_t dst = base + kMbA + (uint32_t)a * (kMbarChunk * 128u) + (uint32_t)r * 128u +
                             (uint32_t)((q ^ (r & 7)) << 4);
        const int col = ct * CT + a * 64 + q * 8;  // column of the (Hkv*d) value row
        const int h = col >> 7, e = col & 127;
        const __nv_bfloat16* src = toks[i] >= 0 ? p.v + ((long long)h * p.L + toks[i]) * kD + e : p.v;
        cp_async16_zfill(dst, src, toks[i] >= 0);
      }
      // the stage fills when every producer's copies have landed (no wait here)
      cp_async_mbar_arrive(bar_full(st));
    }
    cp_async_wait_all();
  } else if (warp == 4) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(128, CT, 0, 1);
      bool ok = true;
      for (int kc = kc0, it = 0; kc < kc1 && ok; ++kc, ++it) {
        const int st = it % kMbStages;
        if (!(ok = wait(bar_full(st), (it / kMbStages) & 1, 912))) break;
        fence_proxy_async_shared();  // gathered rows (cp.async) before the MMA reads them
        tc_fence_after();
        const uint32_t base = sbase + st * kMbStage;
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t bd = sdesc_sw128(base + kMbA + (uint32_t)ks * (16u * 128u),
                                          kMbarChunk * 128u, 1024u);
          for (int t = 0; t < 2; ++t) {
            const uint64_t a = sdesc_kmajor(base + (uint32_t)t * (128u * 128u) + (uint32_t)ks * 32u);
            mma_bf16(tmem, a, bd, idesc, (it > 0 || ks > 0 || t > 0) ? 1u : 0u);
          }
        }
        mma_commit(bar_empty(st));
      }
      mma_commit(bar_done);
    }
  } else if (warp >= 8) {
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const bool has_work = kc1 > kc0;
    bool ok = true;
    if (has_work) ok = wait(bar_done, 0, 913);
    tc_fence_after();
    float* dst = p.mpart + (long long)split * p.split_stride + ((long long)jt * 128 + row) * p.kvw + ct * CT;
    for (int q = 0; q < CT / 32 && ok; ++q) {
      float v[32];
      if (has_work) {
        tmem_ld32(tmem + ((uint32_t)(wq * 32) << 16) + (uint32_t)(q * 32), v);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
      }
      float4* d4 = reinterpret_cast<float4*>(dst + q * 32);
#pragma unroll
      for (int j = 0; j < 8; ++j) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ===========================================================================
// f32 caches on CUDA cores: phi/W/b_bar and M_bar with the workspace layouts
// of the tensor-core kernels (W^T as f32 (d_pad, n_ev_pad) in the bytes of the
// two bf16 terms), so mw_update_kernel is shared.  Theta_f is the folded f32
// projection (d_mem, Hkv*d); evicted indices outside the cache gather zero rows.
// ===========================================================================
constexpr int kF32Rows = 64;   // memory rows per block
constexpr int kF32Chunk = 32;  // reduction chunk
constexpr int kF32Pad = kF32Chunk + 1;

// W^T[m, e] = p_bar_e * (Theta_f K_ev^T)[m, e] for 64 rows x 128 tokens and
// the b_bar partial sum over those tokens.  Thread (tm = tid % 16, tt = tid / 16)
// owns rows tm + 16 i (i < 4) and tokens tt + 16 j (j < 8).
__global__ void __launch_bounds__(256)
    mw_phi_f32_kernel(const float* __restrict__ theta, const float* __restrict__ k,
                      const int* __restrict__ evict, const float* __restrict__ pbar, int Hkv, int L,
                      int n_evict, int n_ev_pad, int d_mem, int d_pad, float* __restrict__ wt,
                      float* __restrict__ bpart) {
  __shared__ float sT[kF32Rows][kF32Pad];
  __shared__ float sK[kTok][kF32Pad];
  __shared__ float sB[16][kF32Rows];
  __shared__ int sTok[kTok];
  const int tid = threadIdx.x, tm = tid & 15, tt = tid >> 4;
  const int et = blockIdx.x, m0 = blockIdx.y * kF32Rows;
  const int kvw = Hkv * kD;
  if (tid < kTok) {
    const int e = et * kTok + tid;
    const int ix = e < n_evict ? (evict != nullptr ? evict[e] : e) : -1;
    sTok[tid] = (unsigned)ix < (unsigned)L ? ix : -1;
  }
  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  for (int c0 = 0; c0 < kvw; c0 += kF32Chunk) {
    __syncthreads();  // sTok ready; the previous chunk's readers are done
    const int h = c0 / kD, e0 = c0 % kD;
    for (int i = tid; i < kF32Rows * kF32Chunk; i += 256) {
      const int r = i / kF32Chunk, cc = i % kF32Chunk;
      sT[r][cc] = (m0 + r < d_mem) ? theta[(long long)(m0 + r) * kvw + c0 + cc] : 0.f;
    }
    for (int i = tid; i < kTok * kF32Chunk; i += 256) {
      const int r = i / kF32Chunk, cc = i % kF32Chunk;
      const int tok = sTok[r];
      sK[r][cc] = tok >= 0 ? k[((long long)h * L + tok) * kD + e0 + cc] : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int cc = 0; cc < kF32Chunk; ++cc) {
      float tv[4], kv[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) tv[i] = sT[tm + 16 * i][cc];
#pragma unroll
      for (int j = 0; j < 8; ++j) kv[j] = sK[tt + 16 * j][cc];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(tv[i], kv[j], acc[i][j]);
    }
  }
  float bsum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int e = et * kTok + tt + 16 * j;
    const float w = pbar[e];  // zero on the padding
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float phi = acc[i][j];
      const float wphi = w * phi;
      wt[(long long)(m0 + tm + 16 * i) * n_ev_pad + e] = wphi;
      bsum[i] = fmaf(wphi, phi, bsum[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) sB[tt][tm + 16 * i] = bsum[i];
  __syncthreads();
  if (tid < kF32Rows) {
    float t = 0.f;
    for (int g = 0; g < 16; ++g) t += sB[g][tid];
    bpart[(long long)et * d_pad + m0 + tid] = t;
  }
}

// M_bar partial of one token split: (W^T V_ev)[m, c] for 64 rows x 64 value
// columns.  Thread (tm = tid % 16, tc = tid / 16) owns rows tm + 16 i and
// columns tc + 16 j (i, j < 4).
__global__ void __launch_bounds__(256)
    mw_mbar_f32_kernel(const float* __restrict__ wt, const float* __restrict__ v,
                       const int* __restrict__ evict, int Hkv, int L, int n_evict, int n_ev_pad,
                       int d_pad, int splits, long long split_stride, float* __restrict__ mpart) {
  __shared__ float sW[kF32Rows][kF32Pad];
  __shared__ float sV[kF32Chunk][kF32Rows + 1];
  __shared__ int sTok[kF32Chunk];
  const int tid = threadIdx.x, tm = tid & 15, tc = tid >> 4;
  const int c0 = blockIdx.x * 64, m0 = blockIdx.y * kF32Rows, sp = blockIdx.z;
  const int kvw = Hkv * kD;
  const int h = c0 / kD, col0 = c0 % kD;
  const int n_chunks = n_ev_pad / kF32Chunk;
  const int per = (n_chunks + splits - 1) / splits;
  const int ch0 = sp * per, ch1 = min(n_chunks, ch0 + per);
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int ch = ch0; ch < ch1; ++ch) {
    const int e0 = ch * kF32Chunk;
    __syncthreads();  // the previous chunk's readers are done
    if (tid < kF32Chunk) {
      const int e = e0 + tid;
      const int ix = e < n_evict ? (evict != nullptr ? evict[e] : e) : -1;
      sTok[tid] = (unsigned)ix < (unsigned)L ? ix : -1;
    }
    for (int i = tid; i < kF32Rows * kF32Chunk; i += 256) {
      const int r = i / kF32Chunk, cc = i % kF32Chunk;
      sW[r][cc] = wt[(long long)(m0 + r) * n_ev_pad + e0 + cc];
    }
    __syncthreads();
    for (int i = tid; i < kF32Chunk * 64; i += 256) {
      const int r = i / 64, cc = i % 64;
      const int tok = sTok[r];
      sV[r][cc] = tok >= 0 ? v[((long long)h * L + tok) * kD + col0 + cc] : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int e = 0; e < kF32Chunk; ++e) {
      float wv[4], vv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) wv[i] = sW[tm + 16 * i][e];
#pragma unroll
      for (int j = 0; j < 4; ++j) vv[j] = sV[e][tc + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(wv[i], vv[j], acc[i][j]);
    }
  }
  float* out = mpart + (long long)sp * split_stride;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
      out[(long long)(m0 + tm + 16 * i) * kvw + c0 + tc + 16 * j] = acc[i][j];
}

// ===========================================================================
// recurrence
// ===========================================================================
// Blocks [0, m_blocks) update M, one element per thread; the blocks after
// them update b, one warp per row (lane l sums tiles l, l + 32, ..., then the
// warp adds the 32 lane sums as a tree), so that no thread walks all the
// b_bar partials of a row alone.
__global__ void mw_update_kernel(const float* __restrict__ mpart, int splits, int B, int d_mem,
                                 int d_pad, int kvw, const float* __restrict__ bpart, int n_et,
                                 const float* __restrict__ coef, float eta, float* __restrict__ M,
                                 float* __restrict__ bst, int m_blocks) {
  if ((int)blockIdx.x < m_blocks) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long nM = (long long)B * d_mem * kvw;
    if (i >= nM) return;
    const int c = (int)(i % kvw);
    const long long bj = i / kvw;
    const int j = (int)(bj % d_mem);
    const int b = (int)(bj / d_mem);
    float s = 0.f;
    for (int sp = 0; sp < splits; ++sp)
      s += mpart[(((long long)sp * B + b) * d_pad + j) * kvw + c];
    const float mbar = s * eta;
    const float gz = coef[b * 3], pie = coef[b * 3 + 1], den = coef[b * 3 + 2];
    M[i] = (gz * M[i] + pie * mbar) / den;
    return;
  }
  const long long row = ((long long)(blockIdx.x - m_blocks) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= (long long)B * d_mem) return;  // whole warps: row is uniform in the warp
  const int j = (int)(row % d_mem);
  const int b = (int)(row / d_mem);
  float s = 0.f;
  for (int t = lane; t < n_et; t += 32) s += bpart[((long long)b * n_et + t) * d_pad + j];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) {
    const float bbar = s * eta;
    const float gz = coef[b * 3], pie = coef[b * 3 + 1], den = coef[b * 3 + 2];
    bst[row] = (gz * bst[row] + pie * bbar) / den;
  }
}

// The same update with four columns of M per thread: block (x, y) with
// y < B d_mem takes float4 groups [256 x, 256 x + 256) of row y of M, so the
// row is a block index and no thread divides; blocks y >= B d_mem (x = 0)
// update b as above, one warp per row.  Every element is computed with the
// same expressions, in the same split order, as mw_update_kernel.
__global__ void mw_update4_kernel(const float4* __restrict__ mpart, int splits, int B, int d_mem,
                                  int d_pad, int kvw4, const float* __restrict__ bpart, int n_et,
                                  const float* __restrict__ coef, float eta, float4* __restrict__ M,
                                  float* __restrict__ bst) {
  const int rows = B * d_mem;
  const int y = blockIdx.y;
  if (y < rows) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= kvw4) return;
    const int b = y / d_mem, j = y - b * d_mem;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < splits; ++sp) {
      const float4 t = mpart[(((long long)sp * B + b) * d_pad + j) * kvw4 + c];
      s.x += t.x;
      s.y += t.y;
      s.z += t.z;
      s.w += t.w;
    }
    const float gz = coef[b * 3], pie = coef[b * 3 + 1], den = coef[b * 3 + 2];
    float4* mp = M + (long long)y * kvw4 + c;
    float4 m = *mp;
    float mbar = s.x * eta;
    m.x = (gz * m.x + pie * mbar) / den;
    mbar = s.y * eta;
    m.y = (gz * m.y + pie * mbar) / den;
    mbar = s.z * eta;
    m.z = (gz * m.z + pie * mbar) / den;
    mbar = s.w * eta;
    m.w = (gz * m.w + pie * mbar) / den;
    *mp = m;
    return;
  }
  if (blockIdx.x != 0) return;
  const int row = (y - rows) * (int)(blockDim.x >> 5) + (int)(threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;  // whole warps: row is uniform in the warp
  const int b = row / d_mem, j = row - b * d_mem;
  float sb = 0.f;
  for (int t = lane; t < n_et; t += 32) sb += bpart[((long long)b * n_et + t) * d_pad + j];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sb += __shfl_xor_sync(0xffffffffu, sb, o);
  if (lane == 0) {
    const float bbar = sb * eta;
    const float gz = coef[b * 3], pie = coef[b * 3 + 1], den = coef[b * 3 + 2];
    bst[row] = (gz * bst[row] + pie * bbar) / den;
  }
}

}  // namespace mw
}  // namespace core

using namespace core;
using namespace core::mw;

namespace {
struct MwPlan {
  int n_ev_pad, n_et, d_pad, n_dh, kvw, splits, n_jt, n_ct, ct, phi_grid;
  long long phi_units;
};
void plan_mw(const core_dims_t* d, int n_evict, int d_mem, MwPlan* m) {
  m->n_et = (n_evict + kTok - 1) / kTok;
  m->n_ev_pad = m->n_et * kTok;
  m->d_pad = ((d_mem + 127) / 128) * 128;
  m->n_dh = m->d_pad / kPhiRows;
  m->kvw = d->n_kv_heads * kD;
  m->phi_units = (long long)d->batch * m->n_et * m->n_dh;
  const int sms = sm_count();
  m->phi_grid = (int)(m->phi_units < sms ? m->phi_units : sms);
  m->n_jt = m->d_pad / 128;
  m->ct = (m->kvw % 256 == 0) ? 256 : 128;
  m->n_ct = m->kvw / m->ct;
  const long long tiles = (long long)m->n_jt * m->n_ct;
  const int n_kc = m->n_ev_pad / kMbarChunk;
  int splits = (int)(sms / tiles);  // one wave: one CTA per SM (the stages fill shared memory)
  if (splits > n_kc) splits = n_kc;
  if (splits < 1) splits = 1;
  m->splits = splits;
}
}  // namespace

extern "C" size_t core_memory_write_workspace_bytes(const core_dims_t* d, int32_t n_evict,
                                                    int32_t d_mem) {
  if (check_dims(d, "core_memory_write_workspace_bytes", true) != CORE_OK || n_evict <= 0 || d_mem <= 0)
    return 0;
  MwPlan m;
  plan_mw(d, n_evict, d_mem, &m);
  Sizer z;
  z.take<float>((size_t)d->batch * m.n_ev_pad);                         // p_bar
  z.take<float>((size_t)d->batch * 3);                                  // coefficients
  z.take<__nv_bfloat16>((size_t)2 * m.d_pad * m.n_ev_pad);              // W^T (one batch row at a time)
  z.take<float>((size_t)d->batch * m.n_et * m.d_pad);                   // b_bar partials
  z.take<float>((size_t)m.splits * d->batch * m.d_pad * m.kvw);         // M_bar partials
  return z.used;
}

// gathered: k, v hold only the evicted rows, (B, Hkv, n_evict, d) in evict_idx
// order; evict_idx still indexes scores_cal (the softmax runs over the cache).
static int memory_write_impl(const core_dims_t* d, const void* k, const void* v,
                             const float* scores_cal, const int32_t* evict_idx, int32_t n_evict,
                             const void* theta_split, int32_t d_mem, float gamma, float eta,
                             float student_temp, float* M, float* b_state, float* Z,
                             void* workspace, size_t workspace_bytes, void* stream, bool gathered) {
  int rc = check_dims(d, "core_memory_write", true);
  if (rc != CORE_OK) return rc;
  if (k == nullptr || v == nullptr || scores_cal == nullptr || evict_idx == nullptr ||
      theta_split == nullptr || M == nullptr || b_state == nullptr || Z == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_memory_write: NULL tensor");
  if (n_evict <= 0 || n_evict > d->seq_len)
    return set_error(CORE_ERR_INVALID_ARG, "core_memory_write: bad n_evict");
  if (d_mem <= 0 || d_mem > 4096 || (d_mem % 8) != 0)
    return set_error(CORE_ERR_UNSUPPORTED, "core_memory_write: d_mem must be a positive multiple of 8");
  if (!(student_temp > 0.f)) return set_error(CORE_ERR_INVALID_ARG, "student_temp must be > 0");
  MwPlan m;
  plan_mw(d, n_evict, d_mem, &m);
  const int kv_rows = gathered ? n_evict : d->seq_len;  // rows per (batch, head) of k and v
  Carver cv(workspace, workspace_bytes);
  float* pbar = cv.take<float>((size_t)d->batch * m.n_ev_pad);
  float* coef = cv.take<float>((size_t)d->batch * 3);
  __nv_bfloat16* wt = cv.take<__nv_bfloat16>((size_t)2 * m.d_pad * m.n_ev_pad);
  float* bpart = cv.take<float>((size_t)d->batch * m.n_et * m.d_pad);
  float* mpart = cv.take<float>((size_t)m.splits * d->batch * m.d_pad * m.kvw);
  if (cv.overflow) return set_error(CORE_ERR_WORKSPACE, "core_memory_write: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceStatus* st = device_status();
  cudaError_t e;

  if (d->seq_len >= kMassClusterMinLen && d->seq_len <= kMassCluster * kMassMaxSmem) {
    const int Lc = (d->seq_len + kMassCluster - 1) / kMassCluster;
    e = cudaFuncSetAttribute(mw_mass_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(sizeof(float) * kMassMaxSmem));
    if (e != cudaSuccess) return cuda_error(e, "mw_mass_cluster_kernel attribute");
    mw_mass_cluster_kernel<<<d->batch * kMassCluster, 1024, sizeof(float) * (size_t)Lc, s>>>(
        scores_cal, d->seq_len, evict_idx, n_evict, m.n_ev_pad, student_temp, gamma, Z, pbar, coef,
        st);
  } else if (d->seq_len <= kMassMaxSmem) {
    e = cudaFuncSetAttribute(mw_mass_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(sizeof(float) * kMassMaxSmem));
    if (e != cudaSuccess) return cuda_error(e, "mw_mass_kernel attribute");
    mw_mass_kernel<true><<<d->batch, 1024, sizeof(float) * (size_t)d->seq_len, s>>>(
        scores_cal, d->seq_len, evict_idx, n_evict, m.n_ev_pad, student_temp, gamma, Z, pbar, coef,
        st);
  } else {
    mw_mass_kernel<false><<<d->batch, 1024, 0, s>>>(scores_cal, d->seq_len, evict_idx, n_evict,
                                                   m.n_ev_pad, student_temp, gamma, Z, pbar, coef,
                                                   st);
  }
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "mw_mass_kernel launch");

  if (d->dtype == CORE_DTYPE_F32) {
    float* wtf = reinterpret_cast<float*>(wt);  // (d_pad, n_ev_pad) f32 in the bytes of the two terms
    for (int b = 0; b < d->batch; ++b) {
      const long long kv_off = (long long)b * d->n_kv_heads * kv_rows * kD;
      mw_phi_f32_kernel<<<dim3(m.n_et, m.d_pad / kF32Rows), 256, 0, s>>>(
          static_cast<const float*>(theta_split), static_cast<const float*>(k) + kv_off,
          gathered ? nullptr : evict_idx + (long long)b * n_evict, pbar + (long long)b * m.n_ev_pad,
          d->n_kv_heads, kv_rows, n_evict, m.n_ev_pad, d_mem, m.d_pad, wtf,
          bpart + (long long)b * m.n_et * m.d_pad);
      if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "mw_phi_f32_kernel launch");
      mw_mbar_f32_kernel<<<dim3(m.kvw / 64, m.d_pad / kF32Rows, m.splits), 256, 0, s>>>(
          wtf, static_cast<const float*>(v) + kv_off,
          gathered ? nullptr : evict_idx + (long long)b * n_evict, d->n_kv_heads, kv_rows, n_evict,
          m.n_ev_pad, m.d_pad, m.splits,
          (long long)d->batch * m.d_pad * m.kvw, mpart + (long long)b * m.d_pad * m.kvw);
      if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "mw_mbar_f32_kernel launch");
    }
  } else {
  CUtensorMap tmT;
  {
    const uint64_t kvw = (uint64_t)m.kvw;
    uint64_t dims[3] = {kvw, (uint64_t)d_mem, 2};
    uint64_t str[2] = {kvw * 2, kvw * 2 * (uint64_t)d_mem};
    uint32_t box[3] = {64, (uint32_t)kPhiRows, 1};
    if ((rc = make_tmap_bf16(&tmT, theta_split, 3, dims, str, box, true)) != CORE_OK) return rc;
  }
  // W^T is (2, d_pad, n_ev_pad); each batch row reuses the same buffer, so
  // rows run one after another (phi of row b, then M_bar of row b).
  CUtensorMap tmW;
  {
    uint64_t dims[2] = {(uint64_t)m.n_ev_pad, (uint64_t)2 * m.d_pad};
    uint64_t str[1] = {(uint64_t)m.n_ev_pad * 2};
    uint32_t box[2] = {64, 128};
    if ((rc = make_tmap_bf16(&tmW, wt, 2, dims, str, box, true)) != CORE_OK) return rc;
  }
  const uint32_t phi_smem = kPhiSmem;
  e = cudaFuncSetAttribute(mw_phi_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, phi_smem);
  if (e != cudaSuccess) return cuda_error(e, "mw_phi_kernel attribute");
  const uint32_t mb_smem = kMbStages * kMbStage + 256 + 1024;
  e = cudaFuncSetAttribute(mw_mbar_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, mb_smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(mw_mbar_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, mb_smem);
  if (e != cudaSuccess) return cuda_error(e, "mw_mbar_kernel attribute");

  for (int b = 0; b < d->batch; ++b) {
    PhiParams pp{};
    pp.B = 1; pp.Hkv = d->n_kv_heads; pp.L = kv_rows; pp.n_evict = n_evict;
    pp.n_ev_pad = m.n_ev_pad; pp.n_et = m.n_et; pp.d_mem = d_mem; pp.d_pad = m.d_pad;
    pp.n_dh = m.n_dh;
    pp.U = (long long)m.n_et * m.n_dh;
    pp.k = static_cast<const __nv_bfloat16*>(k) + (long long)b * d->n_kv_heads * kv_rows * kD;
    pp.evict = gathered ? nullptr : evict_idx + (long long)b * n_evict;
    pp.pbar = pbar + (long long)b * m.n_ev_pad;
    pp.wt = wt;
    pp.bpart = bpart + (long long)b * m.n_et * m.d_pad;
    pp.status = st;
    const int sms = sm_count();
    const int grid = (int)(pp.U < sms ? pp.U : sms);
    mw_phi_kernel<<<grid, kPhiThreads, phi_smem, s>>>(tmT, pp);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "mw_phi_kernel launch");

    MbarParams mq{};
    mq.Hkv = d->n_kv_heads; mq.L = kv_rows; mq.n_evict = n_evict;
    mq.n_ev_pad = m.n_ev_pad; mq.d_pad = m.d_pad; mq.kvw = m.kvw; mq.n_jt = m.n_jt;
    mq.n_ct = m.n_ct; mq.splits = m.splits;
    mq.split_stride = (long long)d->batch * m.d_pad * m.kvw;
    mq.v = static_cast<const __nv_bfloat16*>(v) + (long long)b * d->n_kv_heads * kv_rows * kD;
    mq.evict = gathered ? nullptr : evict_idx + (long long)b * n_evict;
    mq.mpart = mpart + (long long)b * m.d_pad * m.kvw;
    mq.status = st;
    if (m.ct == 256)
      mw_mbar_kernel<256><<<(unsigned)(m.splits * m.n_jt * m.n_ct), kMbThreads, mb_smem, s>>>(tmW, mq);
    else
      mw_mbar_kernel<128><<<(unsigned)(m.splits * m.n_jt * m.n_ct), kMbThreads, mb_smem, s>>>(tmW, mq);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "mw_mbar_kernel launch");
  }
  }
  const long long n = (long long)d->batch * d_mem * m.kvw;
  const long long rows = (long long)d->batch * d_mem;
  const long long b_rows = (rows + 7) / 8;  // 8 warps, one row of b each, per block
  if (m.kvw % 4 == 0 && reinterpret_cast<uintptr_t>(M) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(mpart) % 16 == 0 && rows + b_rows <= 65535) {
    const int kvw4 = m.kvw / 4;
    const dim3 grid((unsigned)((kvw4 + 255) / 256), (unsigned)(rows + b_rows));
    mw_update4_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const float4*>(mpart), m.splits,
                                           d->batch, d_mem, m.d_pad, kvw4, bpart, m.n_et, coef, eta,
                                           reinterpret_cast<float4*>(M), b_state);
  } else {
    const int m_blocks = (int)((n + 255) / 256);
    const int b_blocks = (int)(((long long)d->batch * d_mem * 32 + 255) / 256);  // a warp per row of b
    mw_update_kernel<<<(unsigned)(m_blocks + b_blocks), 256, 0, s>>>(
        mpart, m.splits, d->batch, d_mem, m.d_pad, m.kvw, bpart, m.n_et, coef, eta, M, b_state,
        m_blocks);
  }
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "mw_update_kernel launch");
  return CORE_OK;
}

extern "C" int core_memory_write(const core_dims_t* d, const void* k, const void* v,
                                 const float* scores_cal, const int32_t* evict_idx,
                                 int32_t n_evict, const void* theta_split, int32_t d_mem,
                                 float gamma, float eta, float student_temp, float* M,
                                 float* b_state, float* Z, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  return memory_write_impl(d, k, v, scores_cal, evict_idx, n_evict, theta_split, d_mem, gamma, eta,
                           student_temp, M, b_state, Z, workspace, workspace_bytes, stream, false);
}

extern "C" int core_memory_write_gathered(const core_dims_t* d, const void* k_ev, const void* v_ev,
                                          const float* scores_cal, const int32_t* evict_idx,
                                          int32_t n_evict, const void* theta_split, int32_t d_mem,
                                          float gamma, float eta, float student_temp, float* M,
                                          float* b_state, float* Z, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  return memory_write_impl(d, k_ev, v_ev, scores_cal, evict_idx, n_evict, theta_split, d_mem, gamma,
                           eta, student_temp, M, b_state, Z, workspace, workspace_bytes, stream, true);
}
