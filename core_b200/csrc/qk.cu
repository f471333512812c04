// QK relation features f1..f6 (replaces core/fused_qk.py:373-587).
//
// Three kernels run per call:
//   1. qk_lse_kernel       : causal row log-sum-exp partials.  tcgen05 MMA,
//                            queries on the 128 TMEM lanes (A = Q block,
//                            B = 64-key sub-tiles), online max/sum per lane.
//   2. lse_combine_kernel  : merges the partials into LSE (B, Hq, nq).
//   3. qk_relation_kernel  : second MMA pass with keys on the TMEM lanes
//                            (A = 128-key tile, B = the GQA group's queries),
//                            the attention advantage, its GQA mean and the
//                            per-key running statistics; one 64-byte record
//                            per (key, KV head, query block).
//   4. qk_merge_kernel     : per key, merges the records over KV heads and
//                            query blocks into f1..f6, resolving the rare
//                            f6 cases the running statistics cannot decide by
//                            an exact recomputation.
//
// Work is split into units (batch b, KV head h, query block qb, key tile kt);
// a persistent grid of one CTA per SM takes a contiguous range of units.
#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "qk_common.cuh"
#include "host_util.h"

namespace core {
namespace qk {

constexpr int kD = 128;          // head dim
constexpr int kTile = 128;       // keys per tile == queries per block
constexpr int kRelTeams = 4;                 // relation epilogue: 16-query quarters of each half
constexpr int kRelQ = 64 / kRelTeams;        // queries per thread per half (one chunk of 16)
constexpr int kEpiThreads = 128 * kRelTeams;
constexpr int kThreads = 64 + kEpiThreads;   // warp 0 TMA, warp 1 MMA, 16 epilogue warps
static_assert(kRelTeams == 4, "the team merge packs two 16-query masks per record word");
static_assert(kRelQ == 16, "one 16-query chunk per thread and half");
constexpr int kLseTeams = 4;                       // LSE epilogue: 16-key quarters of a sub-tile
constexpr int kLseEpiThreads = 128 * kLseTeams;
constexpr int kLseThreads = 64 + kLseEpiThreads;  // warp 0 TMA, warp 1 MMA, 16 epilogue warps
constexpr int kKStages = 2;
constexpr uint32_t kKTileBytes = kTile * kD * 2;  // 32 KB
constexpr uint32_t kAtom = 1024;                  // 8 rows x 128 B

struct Params {
  int B, Hq, Hkv, G, nq, L, q_start, n_qb, n_kt;
  long long U;          // number of units
  float scale;          // d^-0.5
  float scale_log2;     // d^-0.5 * log2(e)
  int slot_stride;      // LSE partial slots per (b, qh, t)
  int head_topk;        // min(topk_qk, G)
  int n_recent;         // min(n_recent_queries, nq)
  float2* part;         // LSE partials (log2 units)
  const float* lse;     // (B, Hq, nq) natural-log LSE
  uint32_t* rec;        // (B, L, Hkv, n_qb, 16) records
  DeviceStatus* status;
};

__device__ __forceinline__ long long unit_begin(int c, long long U, int P) {
  return (long long)c * U / P;
}
__device__ __host__ __forceinline__ int cta_of_unit(long long u, long long U, int P) {
  return (int)(((u + 1) * P + U - 1) / U) - 1;
}

struct Unit {
  int b, h, qb, kt;
  long long grp;
};
// Last key tile holding a key that some query of block qb sees; the units of
// later tiles (above the causal diagonal: every key after every query of the
// block) are skipped by all roles and produce no LSE terms and no records.
__device__ __host__ __forceinline__ int kt_last(const Params& p, int qb) {
  const long long last_q = (long long)p.q_start + (long long)qb * kTile + kTile - 1;
  const long long kt = last_q / kTile;
  return (int)(kt < p.n_kt - 1 ? kt : p.n_kt - 1);
}

__device__ __forceinline__ Unit decode(long long u, const Params& p) {
  Unit r;
  r.kt = (int)(u % p.n_kt);
  r.grp = u / p.n_kt;
  r.qb = (int)(r.grp % p.n_qb);
  long long bh = r.grp / p.n_qb;
  r.h = (int)(bh % p.Hkv);
  r.b = (int)(bh / p.Hkv);
  return r;
}


// The unit after t, for walking a CTA's contiguous range (key tile fastest,
// then query block, KV head, batch row) without decode()'s 64-bit divisions.
__device__ __forceinline__ void advance(Unit& t, const Params& p) {
  if (++t.kt == p.n_kt) {
    t.kt = 0;
    ++t.grp;
    if (++t.qb == p.n_qb) {
      t.qb = 0;
      if (++t.h == p.Hkv) {
        t.h = 0;
        ++t.b;
      }
    }
  }
}


// ===========================================================================
// 1. LSE partial kernel
// ===========================================================================
template <int G>
struct LseSmem {
  static constexpr uint32_t kQBytes = 2u * G * kTile * 128u;  // [katom][g][128 rows][128 B]
  static constexpr uint32_t kQOff = 0;
  static constexpr uint32_t kKOff = kQOff + kQBytes;
  static constexpr uint32_t kBarOff = kKOff + kKStages * kKTileBytes;
  static constexpr uint32_t kTotal = kBarOff + 256;
};

template <int G>
__global__ void __launch_bounds__(kLseThreads, 1)
    qk_lse_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const Params p) {
  using S = LseSmem<G>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  const uint32_t sQ = sbase + S::kQOff;
  const uint32_t sK = sbase + S::kKOff;
  const uint32_t bar = sbase + S::kBarOff;
  // barrier slots (8 bytes each)
  const uint32_t bar_q_full = bar + 0, bar_q_empty = bar + 8;
  auto bar_k_full = [&](int s) { return bar + 16 + 8u * s; };
  auto bar_k_empty = [&](int s) { return bar + 16 + 8u * (kKStages + s); };
  auto bar_t_full = [&](int s) { return bar + 16 + 8u * (2 * kKStages + s); };
  auto bar_t_empty = [&](int s) { return bar + 16 + 8u * (2 * kKStages + 2 + s); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + S::kBarOff + 200);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sgen + S::kBarOff + 208);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = gridDim.x;
  const long long u0 = unit_begin(blockIdx.x, p.U, P), u1 = unit_begin(blockIdx.x + 1, p.U, P);

  if (threadIdx.x == 0) {
    mbar_init(bar_q_full, 1);
    mbar_init(bar_q_empty, 1);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(bar_k_full(s), 1);
      mbar_init(bar_k_empty(s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar_t_full(s), 1);
      mbar_init(bar_t_empty(s), kLseEpiThreads / 32);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto wait = [&](uint32_t b, uint32_t parity, int where) -> bool {
    return bounded_wait(b, parity, abort_flag, p.status, where);
  };

  if (warp == 0) {
    if (lane == 0) {
      long long cur = -1;
      int gcount = 0, it = 0;
      Unit t = decode(u0, p);
      for (long long u = u0; u < u1; ++u, advance(t, p)) {
        if (t.kt > kt_last(p, t.qb)) continue;  // above the causal diagonal
        if (t.grp != cur) {
          if (gcount > 0 && !wait(bar_q_empty, (gcount - 1) & 1, 101)) break;
          mbar_arrive_expect_tx(bar_q_full, S::kQBytes);
          for (int ka = 0; ka < 2; ++ka)
            for (int g = 0; g < G; ++g)
              tma_load_3d(sQ + (uint32_t)(ka * G + g) * kTile * 128u, &tmQ, bar_q_full, ka * 64,
                          t.qb * kTile, (t.b * p.Hq + t.h * G + g));
          cur = t.grp;
          ++gcount;
        }
        const int st = it % kKStages;
        if (it >= kKStages && !wait(bar_k_empty(st), ((it / kKStages) - 1) & 1, 102)) break;
        mbar_arrive_expect_tx(bar_k_full(st), kKTileBytes);
        for (int ka = 0; ka < 2; ++ka)
          tma_load_3d(sK + st * kKTileBytes + ka * (kTile * 128u), &tmK, bar_k_full(st), ka * 64,
                      t.kt * kTile, t.b * p.Hkv + t.h);
        ++it;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(128, 64, 0, 0);
      long long cur = -1;
      int gcount = 0, it = 0, sub = 0;
      bool ok = true;
      Unit t = decode(u0, p);
      for (long long u = u0; u < u1 && ok; ++u, advance(t, p)) {
        if (t.kt > kt_last(p, t.qb)) continue;  // above the causal diagonal
        if (t.grp != cur) {
          if (!(ok = wait(bar_q_full, gcount & 1, 103))) break;
          cur = t.grp;
          ++gcount;
        }
        const int st = it % kKStages;
        if (!(ok = wait(bar_k_full(st), (it / kKStages) & 1, 104))) break;
        tc_fence_after();
        for (int ss = 0; ss < 2 && ok; ++ss) {
          const int buf = sub & 1, n = sub >> 1;
          if (sub >= 2) {
            if (!(ok = wait(bar_t_empty(buf), (n - 1) & 1, 105))) break;
            tc_fence_after();
          }
          for (int g = 0; g < G; ++g) {
            const uint32_t d = tmem + (uint32_t)(buf * G * 64 + g * 64);
            for (int ks = 0; ks < 8; ++ks) {
              // A: rows of q-head g inside K atom ks/4: sQ + ((ks/4)*G + g) * 16 KB
              const uint64_t a = sdesc_kmajor(sQ + (uint32_t)((ks >> 2) * G + g) * kTile * 128u + (uint32_t)(ks & 3) * 32u);
              const uint64_t bdesc =
                  sdesc_kmajor(sK + st * kKTileBytes + (uint32_t)(ks >> 2) * kTile * 128u +
                               (uint32_t)ss * 64u * 128u + (uint32_t)(ks & 3) * 32u);
              mma_bf16(d, a, bdesc, idesc, ks > 0 ? 1u : 0u);
            }
          }
          mma_commit(bar_t_full(buf));
          ++sub;
        }
        if (!ok) break;
        mma_commit(bar_k_empty(st));
        ++it;
        // the group's units after this one are in another CTA or above the diagonal
        const bool last_of_group = (u + 1 >= u1) || (t.kt == kt_last(p, t.qb));
        if (last_of_group) mma_commit(bar_q_empty);
      }
    }
  } else {
    // ---------------- epilogue: online max / sum per (q-head, query) ----------------
    const int ew = warp - 2;
    const int team = ew >> 2;      // 16-key quarter of each 64-key sub-tile
    const int wq = warp & 3;       // TMEM lane quarter
    const int row = wq * 32 + lane;
    float m[G], l[G];
    long long cur = -1;
    Unit cu{};
    int sub = 0;
    bool ok = true;
    auto flush = [&](const Unit& t) {
      const int tq = t.qb * kTile + row;
      if (tq < p.nq) {
        const int c_lo = cta_of_unit(t.grp * (long long)p.n_kt, p.U, P);
        const int slot = (blockIdx.x - c_lo) * kLseTeams + team;
        for (int g = 0; g < G; ++g) {
          const long long r = ((long long)(t.b * p.Hq + t.h * G + g) * p.nq + tq);
          p.part[r * p.slot_stride + slot] = make_float2(m[g], l[g]);
        }
      }
    };
    const unsigned long long sc2 = f2_pack(p.scale_log2, p.scale_log2);
    Unit t = decode(u0, p);
    for (long long u = u0; u < u1 && ok; ++u, advance(t, p)) {
      if (t.kt > kt_last(p, t.qb)) continue;  // above the causal diagonal
      if (t.grp != cur) {
        if (cur >= 0) flush(cu);
        for (int g = 0; g < G; ++g) {
          m[g] = -INFINITY;
          l[g] = 0.f;
        }
        cur = t.grp;
        cu = t;
      }
      const int qpos = p.q_start + t.qb * kTile + row;  // absolute query position
      for (int ss = 0; ss < 2; ++ss) {
        const int buf = sub & 1, n = sub >> 1;
        if (!(ok = wait(bar_t_full(buf), n & 1, 106))) break;
        tc_fence_after();
        const int k0 = t.kt * kTile + ss * 64 + team * 16;
        const bool need_mask = (k0 + 15 > p.q_start + t.qb * kTile) || (k0 + 16 > p.L);
        for (int g = 0; g < G; ++g) {
          float v[16];
          tmem_ld16(tmem + ((uint32_t)(wq * 32) << 16) + (uint32_t)(buf * G * 64 + g * 64 + team * 16), v);
#pragma unroll
          for (int j = 0; j < 16; j += 2) bf16_round2(v[j], v[j + 1]);  // bf16 logits (fused_qk.py:83-87)
          if (need_mask) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int kk = k0 + j;
              if (kk > qpos || kk >= p.L) v[j] = -INFINITY;
            }
          }
          float cmax = v[0];
#pragma unroll
          for (int j = 1; j < 15; j += 2) cmax = fmax3(cmax, v[j], v[j + 1]);
          cmax = fmaxf(cmax, v[15]);
          // scale > 0: the scaled maximum is the scaled raw maximum
          const float nm = fmaxf(m[g], cmax * p.scale_log2);
          if (nm != -INFINITY) {
            const unsigned long long neg2 = f2_pack(-nm, -nm);
            unsigned long long acc = 0ull;
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
              const unsigned long long y = f2_fma(f2_pack(v[j], v[j + 1]), sc2, neg2);
              acc = f2_add(acc, f2_pack(ex2_approx(f2_lo(y)), ex2_approx(f2_hi(y))));
            }
            l[g] = l[g] * ex2_approx(m[g] - nm) + (f2_lo(acc) + f2_hi(acc));
            m[g] = nm;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_t_empty(buf));
        ++sub;
      }
    }
    if (ok && cur >= 0) flush(cu);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ===========================================================================
// 2. LSE combine
// ===========================================================================
// Eight lanes per (b, q-head, query) row: lane j takes slots j, j + 8, ...;
// the maximum and then the rescaled sums are combined by shuffles.
__global__ void lse_combine_kernel2(const Params p, int grid_ctas, float* __restrict__ lse_out) {
  const long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 3;
  const int sl = threadIdx.x & 7;
  const long long n = (long long)p.B * p.Hq * p.nq;
  int nslots = 0;
  const float2* s = p.part;
  if (i < n) {
    const int t = (int)(i % p.nq);
    const long long bq = i / p.nq;
    const int qh = (int)(bq % p.Hq);
    const int b = (int)(bq / p.Hq);
    const int h = qh / p.G;
    const int qb = t / kTile;
    const long long grp = ((long long)b * p.Hkv + h) * p.n_qb + qb;
    const int c_lo = cta_of_unit(grp * (long long)p.n_kt, p.U, grid_ctas);
    const int c_hi = cta_of_unit(grp * (long long)p.n_kt + kt_last(p, qb), p.U, grid_ctas);
    nslots = (c_hi - c_lo + 1) * kLseTeams;
    s = p.part + i * p.slot_stride;
  }
  float mm = -INFINITY;
  for (int k = sl; k < nslots; k += 8) mm = fmaxf(mm, s[k].x);
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
  float ll = 0.f;
  if (mm != -INFINITY) {
    for (int k = sl; k < nslots; k += 8) {
      const float2 v = s[k];
      if (v.y > 0.f) ll += v.y * ex2_approx(v.x - mm);
    }
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) ll += __shfl_xor_sync(0xffffffffu, ll, o);
  if (i < n && sl == 0)
    lse_out[i] = (mm == -INFINITY || ll <= 0.f) ? -INFINITY : (mm + log2f(ll)) * kLn2;
}

// ===========================================================================
// 3. Relation kernel
// ===========================================================================
template <int G>
struct RelSmem {
  static constexpr uint32_t kQBytes = 2u * 2u * G * 64u * 128u;  // [katom][half][g][64][128 B]
  static constexpr uint32_t kQOff = 0;
  static constexpr uint32_t kKOff = kQOff + kQBytes;
  static constexpr uint32_t kLseOff = kKOff + kKStages * kKTileBytes;  // float2 [G][128]: (-lse, log|C|)
  static constexpr uint32_t kCcOff = kLseOff + G * kTile * 8;          // unused
  static constexpr uint32_t kXchOff = kCcOff + kTile * 4;  // uint32 [3 slots][16 words][128 rows]
  static constexpr uint32_t kBarOff = kXchOff + (kRelTeams - 1) * kTile * 16 * 4;
  static constexpr uint32_t kTotal = kBarOff + 256;
};

// Running statistics of one key over one thread's queries of a unit.
struct KeyStats {
  float top[4], rtop[4];
  float psum, mxnp, nsum;  // sum of the positive R, max and sum of the non-positive R
  uint32_t pcnt;
  uint32_t mask0, mask1;   // positive-R bits of the thread's queries, per half
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int i = 0; i < 4; ++i) top[i] = rtop[i] = -INFINITY;
    psum = 0.f;
    mxnp = -INFINITY;
    nsum = 0.f;
    pcnt = 0;
    mask0 = mask1 = 0;
  }
};

// Team exchange slot (word-major: word i of key row r at x[i * kTile + r]).
__device__ __forceinline__ void xch_put(uint32_t* x, const KeyStats& st, uint32_t w0,
                                        uint32_t w1) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[i * kTile] = __float_as_uint(st.top[i]);
    x[(4 + i) * kTile] = __float_as_uint(st.rtop[i]);
  }
  x[8 * kTile] = __float_as_uint(st.psum);
  x[9 * kTile] = st.pcnt;
  x[10 * kTile] = w0;
  x[11 * kTile] = w1;
  x[12 * kTile] = __float_as_uint(st.mxnp);
  x[13 * kTile] = __float_as_uint(st.nsum);
}
__device__ __forceinline__ void xch_take(const uint32_t* x, KeyStats& st, uint32_t& w0,
                                         uint32_t& w1) {
  float o[4], ro[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[i] = __uint_as_float(x[i * kTile]);
    ro[i] = __uint_as_float(x[(4 + i) * kTile]);
  }
  top4_merge(st.top, o);
  top4_merge(st.rtop, ro);
  st.psum += __uint_as_float(x[8 * kTile]);
  st.pcnt += x[9 * kTile];
  w0 = x[10 * kTile];
  w1 = x[11 * kTile];
  st.mxnp = fmaxf(st.mxnp, __uint_as_float(x[12 * kTile]));
  st.nsum += __uint_as_float(x[13 * kTile]);
}

// 18 warps: five share one scheduler's 16K registers, so 96 registers a thread
template <int G, bool kLoo>
__global__ void __launch_bounds__(kThreads, 1)
    qk_relation_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK, const Params p) {
  using S = RelSmem<G>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  const uint32_t sQ = sbase + S::kQOff;
  const uint32_t sK = sbase + S::kKOff;
  float* s_nc = reinterpret_cast<float*>(sgen + S::kLseOff);  // [G][128] -lse + log|C_t|
  uint32_t* s_xch = reinterpret_cast<uint32_t*>(sgen + S::kXchOff);
  const uint32_t bar = sbase + S::kBarOff;
  const uint32_t bar_q_full = bar + 0, bar_q_empty = bar + 8;
  auto bar_k_full = [&](int s) { return bar + 16 + 8u * s; };
  auto bar_k_empty = [&](int s) { return bar + 16 + 8u * (kKStages + s); };
  auto bar_t_full = [&](int s) { return bar + 16 + 8u * (2 * kKStages + s); };
  auto bar_t_empty = [&](int s) { return bar + 16 + 8u * (2 * kKStages + 2 + s); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + S::kBarOff + 200);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sgen + S::kBarOff + 208);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = gridDim.x;
  const long long u0 = unit_begin(blockIdx.x, p.U, P), u1 = unit_begin(blockIdx.x + 1, p.U, P);
  constexpr int kN = G * 64;  // MMA N: G query heads x 64 queries
  constexpr uint32_t kQHalf = (uint32_t)G * 64u * 128u;  // bytes of one query half in one atom

  if (threadIdx.x == 0) {
    mbar_init(bar_q_full, 1);
    mbar_init(bar_q_empty, 1);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(bar_k_full(s), 1);
      mbar_init(bar_k_empty(s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar_t_full(s), 1);
      mbar_init(bar_t_empty(s), kEpiThreads / 32);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto wait = [&](uint32_t b, uint32_t parity, int where) -> bool {
    return bounded_wait(b, parity, abort_flag, p.status, where);
  };

  if (warp == 0) {
    if (lane == 0) {
      long long cur = -1;
      int gcount = 0, it = 0;
      Unit t = decode(u0, p);
      for (long long u = u0; u < u1; ++u, advance(t, p)) {
        if (t.kt > kt_last(p, t.qb)) continue;  // above the causal diagonal
        if (t.grp != cur) {
          if (gcount > 0 && !wait(bar_q_empty, (gcount - 1) & 1, 201)) break;
          mbar_arrive_expect_tx(bar_q_full, S::kQBytes);
          // rows of a half ordered [team][head][16 queries], so that one
          // epilogue thread's queries of all G heads are G*16 adjacent TMEM columns
          for (int ka = 0; ka < 2; ++ka)
            for (int hf = 0; hf < 2; ++hf)
              for (int tm = 0; tm < kRelTeams; ++tm)
                for (int g = 0; g < G; ++g)
                  tma_load_3d(sQ + (uint32_t)ka * 2u * kQHalf + (uint32_t)hf * kQHalf +
                                  (uint32_t)(tm * G + g) * 16u * 128u,
                              &tmQ, bar_q_full, ka * 64, t.qb * kTile + hf * 64 + tm * kRelQ,
                              t.b * p.Hq + t.h * G + g);
          cur = t.grp;
          ++gcount;
        }
        const int st = it % kKStages;
        if (it >= kKStages && !wait(bar_k_empty(st), ((it / kKStages) - 1) & 1, 202)) break;
        mbar_arrive_expect_tx(bar_k_full(st), kKTileBytes);
        for (int ka = 0; ka < 2; ++ka)
          tma_load_3d(sK + st * kKTileBytes + ka * (kTile * 128u), &tmK, bar_k_full(st), ka * 64,
                      t.kt * kTile, t.b * p.Hkv + t.h);
        ++it;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(128, kN, 0, 0);
      long long cur = -1;
      int gcount = 0, it = 0, sub = 0;
      bool ok = true;
      Unit t = decode(u0, p);
      for (long long u = u0; u < u1 && ok; ++u, advance(t, p)) {
        if (t.kt > kt_last(p, t.qb)) continue;  // above the causal diagonal
        if (t.grp != cur) {
          if (!(ok = wait(bar_q_full, gcount & 1, 203))) break;
          cur = t.grp;
          ++gcount;
        }
        const int st = it % kKStages;
        if (!(ok = wait(bar_k_full(st), (it / kKStages) & 1, 204))) break;
        tc_fence_after();
        for (int hf = 0; hf < 2 && ok; ++hf) {
          const int buf = sub & 1, n = sub >> 1;
          if (sub >= 2) {
            if (!(ok = wait(bar_t_empty(buf), (n - 1) & 1, 205))) break;
            tc_fence_after();
          }
          const uint32_t d = tmem + (uint32_t)(buf * kN);
          for (int ks = 0; ks < 8; ++ks) {
            const uint64_t a = sdesc_kmajor(sK + st * kKTileBytes + (uint32_t)(ks >> 2) * kTile * 128u +
                                            (uint32_t)(ks & 3) * 32u);
            const uint64_t bdesc = sdesc_kmajor(sQ + (uint32_t)(ks >> 2) * 2u * kQHalf +
                                                (uint32_t)hf * kQHalf + (uint32_t)(ks & 3) * 32u);
            mma_bf16(d, a, bdesc, idesc, ks > 0 ? 1u : 0u);
          }
          mma_commit(bar_t_full(buf));
          ++sub;
        }
        if (!ok) break;
        mma_commit(bar_k_empty(st));
        ++it;
        // the group's units after this one are in another CTA or above the diagonal
        const bool last_of_group = (u + 1 >= u1) || (t.kt == kt_last(p, t.qb));
        if (last_of_group) mma_commit(bar_q_empty);
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int ew = warp - 2;
    const int team = ew >> 2;  // which 16 of each 64-query half
    const int wq = warp & 3;
    const int krow = wq * 32 + lane;  // key row inside the tile
    const float inv_ht = 1.0f / (float)p.head_topk;
    const unsigned long long sc2 = f2_pack(p.scale, p.scale);
    const bool exact_div = (p.head_topk != 1 && p.head_topk != 2 && p.head_topk != 4);
    const float single_val = log1pf(expf(kLogFloor));
    long long cur = -1;
    int sub = 0;
    bool ok = true;
    Unit t = decode(u0, p);
    for (long long u = u0; u < u1 && ok; ++u, advance(t, p)) {
      if (t.kt > kt_last(p, t.qb)) continue;  // above the causal diagonal
      if (t.grp != cur) {
        // (re)load (-lse, log|C_t|) of this query block
        named_barrier(1, kEpiThreads);
        const int tid = threadIdx.x - 64;
        for (int i = tid; i < G * kTile; i += kEpiThreads) {
          const int g = i / kTile, tq = i % kTile;
          const int tt = t.qb * kTile + tq;
          const long long qpos = (long long)p.q_start + tt;
          const long long cc = (qpos + 1 < p.L) ? qpos + 1 : p.L;
          s_nc[i] = (tt < p.nq)
                        ? relation_offset(p.lse[(long long)(t.b * p.Hq + t.h * G + g) * p.nq + tt], cc)
                        : 0.f;
        }
        named_barrier(1, kEpiThreads);
        cur = t.grp;
      }
      const int key = t.kt * kTile + krow;
      KeyStats st;
      st.init();
      const int qb_first_pos = p.q_start + t.qb * kTile;
      const int qb_valid = min(kTile, p.nq - t.qb * kTile);
      // every key of the tile visible to every query of the block, and in range
      const bool keys_full = (t.kt * kTile + kTile - 1 <= qb_first_pos) && (t.kt * kTile + kTile <= p.L);
      // Full units keep their statistics on the unscaled head sum S = head_topk * R:
      // 1/head_topk is a power of two here, so scaling the finished statistics
      // (maxima, top-4, positive sum) is exact and the signs are unchanged.
      const bool sspace = !kLoo && !exact_div && keys_full && qb_valid == kTile;
      for (int hf = 0; hf < 2; ++hf) {
        const int buf = sub & 1, n = sub >> 1;
        if (!(ok = wait(bar_t_full(buf), n & 1, 206))) break;
        tc_fence_after();
        const int tl0 = hf * 64 + team * kRelQ;  // query index within the block of j = 0
        const bool full = keys_full && (tl0 + kRelQ <= qb_valid);
        // this thread's G * 16 columns: head g's 16 queries at tcol + 16 g
        const uint32_t tcol = tmem + ((uint32_t)(wq * 32) << 16) + (uint32_t)(buf * kN + team * G * kRelQ);
        // kRelQ queries per thread, in chunks of 16 to bound registers
        uint32_t msk = 0;
#pragma unroll 1
        for (int ch = 0; ch < kRelQ / 16; ++ch) {
          const int c0 = tl0 + ch * 16;  // query index within the block of element 0
          const int tabs0 = t.qb * kTile + c0;  // absolute query index of element 0
          const bool recent_chunk = tabs0 + 15 >= p.nq - p.n_recent;
          bool done = false;
          if (sspace) {
            // S = sum over the group's heads of fma(s, bf16(x), -lse + log|C|) in
            // f32x2, with the floor clamp left out: exact when every r of the
            // chunk lies at least 16 above the floor (then logaddexp(r, floor)
            // is r); otherwise the chunk is redone below
            unsigned long long S2[8];
            float rmin = INFINITY;
#pragma unroll
            for (int g = 0; g < G; ++g) {
              float v[16];
              tmem_ld16(tcol + (uint32_t)(g * 16), v);
              const float4* nc4 = reinterpret_cast<const float4*>(s_nc + g * kTile + c0);
#pragma unroll
              for (int q4 = 0; q4 < 4; ++q4) {
                const float4 c = nc4[q4];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  const int j = q4 * 4 + e * 2;
                  bf16_round2(v[j], v[j + 1]);
                  const unsigned long long r2 =
                      f2_fma(f2_pack(v[j], v[j + 1]), sc2, e ? f2_pack(c.z, c.w) : f2_pack(c.x, c.y));
                  rmin = fmin3(rmin, f2_lo(r2), f2_hi(r2));
                  S2[j >> 1] = (g == 0) ? r2 : f2_add(S2[j >> 1], r2);
                }
              }
            }
            if (!__any_sync(0xffffffffu, rmin < kLogFloor + 16.0f)) {
              done = true;
#pragma unroll
              for (int jj = 0; jj < 8; ++jj) {
                const float a = f2_lo(S2[jj]), b = f2_hi(S2[jj]);
                top4_insert2(st.top, a, b);
                const bool pa = a > 0.f, pb = b > 0.f;
                if (pa) {
                  st.psum += a;
                } else {
                  st.mxnp = fmaxf(st.mxnp, a);
                  st.nsum += a;
                }
                if (pb) {
                  st.psum += b;
                } else {
                  st.mxnp = fmaxf(st.mxnp, b);
                  st.nsum += b;
                }
                msk |= ((pa ? 1u : 0u) | (pb ? 2u : 0u)) << (ch * 16 + 2 * jj);
              }
              if (recent_chunk) {
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                  const int r0 = p.nq - p.n_recent - tabs0;  // first recent element
                  if (2 * jj >= r0) top4_insert(st.rtop, f2_lo(S2[jj]));
                  if (2 * jj + 1 >= r0) top4_insert(st.rtop, f2_hi(S2[jj]));
                }
              }
            }
          }
          if (done) continue;
          // general path: exact logaddexp with the floor where needed, causal and
          // ragged masks, leave-one-out TopMean
          float acc[16];
          float mn[kLoo ? 16 : 1];
#pragma unroll 1
          for (int g = 0; g < G; ++g) {
            float v[16];
            tmem_ld16(tcol + (uint32_t)(g * 16), v);
            const float* ncp = s_nc + g * kTile + c0;
            float rmin = INFINITY;
            // r for pairs of queries in packed f32x2 arithmetic (each lane rounds as the
            // scalar form), kept in v
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
              bf16_round2(v[j], v[j + 1]);
              const unsigned long long nc2 = *reinterpret_cast<const unsigned long long*>(ncp + j);
              const unsigned long long r2 = f2_fma(f2_pack(v[j], v[j + 1]), sc2, nc2);
              v[j] = f2_lo(r2);
              v[j + 1] = f2_hi(r2);
              rmin = fmin3(rmin, v[j], v[j + 1]);
            }
            // v = logaddexp_floor_fast(r): max(r, floor) unless some r of the chunk lies
            // within 16 of the floor (rare): then the exact form (warp-uniform branch)
            if (__any_sync(0xffffffffu, rmin < kLogFloor + 16.0f)) {
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = logaddexp_floor_fast(v[j]);
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = fmaxf(v[j], kLogFloor);
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float rel = v[j];
              if (!full) {
                const int qpos = qb_first_pos + c0 + j;
                if (key > qpos) rel = kLogFloor;
                else if (qpos == 0) rel = single_val;
              }
              if (g == 0) {
                acc[j] = rel;
                if (kLoo) mn[kLoo ? j : 0] = rel;
              } else {
                acc[j] += rel;
                if (kLoo) mn[kLoo ? j : 0] = fminf(mn[kLoo ? j : 0], rel);
              }
            }
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float R;
            if (kLoo) {
              R = __fdiv_rn(acc[j] - mn[kLoo ? j : 0], (float)p.head_topk);
            } else if (sspace) {
              R = acc[j];
            } else {
              R = exact_div ? __fdiv_rn(acc[j], (float)p.head_topk) : acc[j] * inv_ht;
            }
            if (!full) {
              const int qpos = qb_first_pos + c0 + j;
              if (c0 + j >= qb_valid || key > qpos) R = -INFINITY;
            }
            top4_insert(st.top, R);
            if (recent_chunk && tabs0 + j >= p.nq - p.n_recent) top4_insert(st.rtop, R);
            const bool pz = R > 0.f;
            st.psum += fmaxf(R, 0.f);  // adds R when positive, +0 otherwise (NaN: +0)
            if (R > -INFINITY) st.nsum += fminf(R, 0.f);  // masked entries are not queries
            msk |= (pz ? 1u : 0u) << (ch * 16 + j);
            st.mxnp = fmaxf(st.mxnp, pz ? -INFINITY : R);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_t_empty(buf));
        ++sub;
        if (hf == 0) st.mask0 = msk; else st.mask1 = msk;
      }
      if (!ok) break;
      if (sspace) {  // back to R = S / head_topk (exact)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          st.top[i] *= inv_ht;
          st.rtop[i] *= inv_ht;
        }
        st.psum *= inv_ht;
        st.mxnp *= inv_ht;
        st.nsum *= inv_ht;
      }
      st.pcnt = (uint32_t)(__popc(st.mask0) + __popc(st.mask1));  // positive relations
      // Merge the four teams (same key, different query quarters) as a tree:
      // 1 -> 0 and 3 -> 2, then 2 -> 0, which stores the record.  Exchange
      // slots are word-major (word i of key row r at [i * kTile + r]), so a
      // warp's 32 rows fall in 32 banks.  Slot 0 and 1 are written before the
      // first barrier and read before the second; slot 2 between them and read
      // after the second, so two barriers per unit suffice.
      // query bits: record word 2 hf + (team >> 1) holds teams 2 (team >> 1) and
      // 2 (team >> 1) + 1 of half hf, the odd team in the upper 16 bits
      uint32_t* xrow = s_xch + krow;
      if (team & 1) xch_put(xrow + (team >> 1) * 16 * kTile, st, st.mask0, st.mask1);
      named_barrier(2, kEpiThreads);
      uint32_t wa = 0, wb = 0;
      if (!(team & 1)) {
        uint32_t o0, o1;
        xch_take(xrow + (team >> 1) * 16 * kTile, st, o0, o1);
        wa = st.mask0 | (o0 << kRelQ);
        wb = st.mask1 | (o1 << kRelQ);
        if (team == 2) xch_put(xrow + 2 * 16 * kTile, st, wa, wb);
      }
      named_barrier(2, kEpiThreads);
      if (team == 0) {
        uint32_t w1, w3;
        xch_take(xrow + 2 * 16 * kTile, st, w1, w3);
        if (key < p.L) {
          uint4* dst = reinterpret_cast<uint4*>(
              p.rec + ((((long long)t.b * p.L + key) * p.Hkv + t.h) * p.n_qb + t.qb) * kRecWords);
          dst[0] = make_uint4(__float_as_uint(st.top[0]), __float_as_uint(st.top[1]),
                              __float_as_uint(st.top[2]), __float_as_uint(st.top[3]));
          dst[1] = make_uint4(__float_as_uint(st.rtop[0]), __float_as_uint(st.rtop[1]),
                              __float_as_uint(st.rtop[2]), __float_as_uint(st.rtop[3]));
          dst[2] = make_uint4(__float_as_uint(st.psum), st.pcnt, wa, w1);
          dst[3] = make_uint4(wb, w3, __float_as_uint(st.mxnp), __float_as_uint(st.nsum));
        }
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

// ===========================================================================
// 4. Merge records into f1..f6
// ===========================================================================
struct MergeParams {
  int B, Hq, Hkv, G, nq, L, q_start, n_qb, topk, n_recent, head_topk;
  float scale;
  const uint32_t* rec;
  const __nv_bfloat16* q;  // (B, Hq, nq, d), bf16 caches
  const __nv_bfloat16* k;  // (B, Hkv, L, d), bf16 caches
  const float* qf;         // the same for f32 caches (then q, k are NULL)
  const float* kf;
  const float* lse;        // (B, Hq, nq)
  float* features;
  int stride;
  uint32_t* summary;     // summary mode (head-sharded caches): per-key summaries instead of features
  int sum_words;         // words per summary: kSumHead + 4 n_qb
  float* f6_target;      // where qk_f6_resolve_kernel adds a positive head: features[:, 5] or summary word 10
  int f6_stride;
  float f6_inc;          // 1 / Hkv (features) or 1 (summary count)
  int* queue_count;      // undecided f6 (key, head) pairs, resolved by qk_f6_resolve_kernel
  int2* queue;
  int queue_cap;
  DeviceStatus* status;
};

constexpr int kMergeThreads = 256;
constexpr int kMaxSlowNq = 2048;

__device__ __forceinline__ float sum_top_desc(const float (&t)[4], int k) {
  // cumsum of the descending values, read at k-1 (fused_qk.py:541-543)
  float s = t[0];
  if (k > 1) s += t[1];
  if (k > 2) s += t[2];
  if (k > 3) s += t[3];
  return s;
}

// Exact relation value R[h, t, key] (one query), as the relation kernel
// computes it; the key row is in shared memory as f32, the G query rows are
// read 8 bf16 at a time and the dot products run over d in ascending order.
__device__ float relation_exact(const MergeParams& p, int b, int h, int key, int t,
                                const float* __restrict__ s_k) {
  const long long qpos = (long long)p.q_start + t;
  if (key > qpos) return kLogFloor;
  const long long cc = (qpos + 1 < p.L) ? qpos + 1 : p.L;
  float dot[4] = {0.f, 0.f, 0.f, 0.f};
  if (p.qf != nullptr) {  // f32 caches: unrounded logits (fp32 reference path)
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      if (g < p.G) {
        const float4* qr4 = reinterpret_cast<const float4*>(
            p.qf + (((long long)b * p.Hq + h * p.G + g) * p.nq + t) * kD);
        for (int c = 0; c < kD / 4; ++c) {
          const float4 w = __ldg(qr4 + c);
          const float4 kv = reinterpret_cast<const float4*>(s_k)[c];
          dot[g] = fmaf(w.x, kv.x, dot[g]);
          dot[g] = fmaf(w.y, kv.y, dot[g]);
          dot[g] = fmaf(w.z, kv.z, dot[g]);
          dot[g] = fmaf(w.w, kv.w, dot[g]);
        }
      }
    }
  } else {
  const uint4* qr[4];
#pragma unroll
  for (int g = 0; g < 4; ++g)
    qr[g] = reinterpret_cast<const uint4*>(
        p.q + (((long long)b * p.Hq + h * p.G + (g < p.G ? g : 0)) * p.nq + t) * kD);
#pragma unroll 4
  for (int c = 0; c < kD / 8; ++c) {
    const float4 k0 = reinterpret_cast<const float4*>(s_k)[2 * c];
    const float4 k1 = reinterpret_cast<const float4*>(s_k)[2 * c + 1];
    const float kv[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      if (g < p.G) {
        const uint4 w = __ldg(qr[g] + c);
        const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 qf = __bfloat1622float2(q2[e]);
          dot[g] = fmaf(qf.x, kv[2 * e], dot[g]);
          dot[g] = fmaf(qf.y, kv[2 * e + 1], dot[g]);
        }
      }
    }
  }
  }
  float acc = 0.f, mn = INFINITY;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    if (g < p.G) {
      const int qh = h * p.G + g;
      const bool f32 = p.qf != nullptr;
      const float x = f32 ? dot[g] : bf16_round(dot[g]);
      const float r = fmaf(x, p.scale, relation_offset(p.lse[((long long)b * p.Hq + qh) * p.nq + t], cc));
      float rel = f32 ? logaddexp_floor(r) : logaddexp_floor_fast(r);
      if (qpos == 0) rel = log1pf(expf(kLogFloor));
      acc = (g == 0) ? rel : acc + rel;
      mn = fminf(mn, rel);
    }
  }
  if (p.head_topk < p.G) return __fdiv_rn(acc - mn, (float)p.head_topk);
  return __fdiv_rn(acc, (float)p.head_topk);
}

// One lane per KV head, Hkv lanes per key (Hkv a power of two, at most 16):
// each lane walks its head's records of the key (contiguous, n_qb x 64 B),
// keeps that head's f6 test to itself, and the key's lanes combine the rest
// with shuffles: the top-4 lists (order-free), the positive sums and counts,
// and the OR of the positive-query bits of every query block.
template <int kLanes>
__device__ __forceinline__ void merge_top4_lanes(float (&t)[4]) {
#pragma unroll
  for (int off = 1; off < kLanes; off <<= 1) {
    float o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = __shfl_xor_sync(0xffffffffu, t[i], off);
#pragma unroll
    for (int i = 0; i < 4; ++i) top4_insert(t, o[i]);
  }
}

template <int kLanes, typename T>
__device__ __forceinline__ T lanes_sum(T v) {
#pragma unroll
  for (int off = 1; off < kLanes; off <<= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

template <int kLanes>
__device__ __forceinline__ uint32_t lanes_or(uint32_t v) {
#pragma unroll
  for (int off = 1; off < kLanes; off <<= 1) v |= __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

template <int kLanes>
__global__ void __launch_bounds__(kMergeThreads)
    qk_merge_kernel(const MergeParams p) {
  const long long tid = (long long)blockIdx.x * kMergeThreads + threadIdx.x;
  const long long gi_raw = tid / kLanes;
  const int h = (int)(tid % kLanes);  // this lane's KV head
  // whole key groups stay in the grid (kLanes divides the block), so the
  // shuffles below always see all lanes of the key; lanes past the last key
  // compute on a clamped key and store nothing
  const bool live = gi_raw < (long long)p.B * p.L;
  const long long gi = live ? gi_raw : 0;
  const int b = (int)(gi / p.L);
  const int key = (int)(gi % p.L);
  int valid = p.nq - max(key - p.q_start, 0);
  valid = min(max(valid, 1), p.nq);
  const int k2max = min(p.topk, p.nq * p.Hkv);
  const int k2 = min(max(valid * p.Hkv, 1), k2max);
  const int nrec = p.n_recent;
  const int rstart = p.q_start + p.nq - nrec;
  int rvalid = p.q_start + p.nq - max(key, rstart);
  rvalid = min(max(rvalid, 1), nrec);
  const int k4max = min(p.topk, nrec * p.Hkv);
  const int k4 = min(max(rvalid * p.Hkv, 1), k4max);
  const int kf = max((valid + 3) / 4, 1);

  float top[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  float rtop[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  float hs = 0.f, mx = -INFINITY, ns = 0.f;
  unsigned int hc = 0;
  int f5cnt = 0;
  uint32_t* sum_out = (p.summary != nullptr && live) ? p.summary + gi * p.sum_words : nullptr;
  const uint32_t* base = p.rec + (gi * p.Hkv + h) * (long long)p.n_qb * kRecWords;
  // Blocks before qb_min hold no query that sees this key (their units may
  // have been skipped, leaving no record).  The lanes of a warp loop from the
  // smallest qb_min among them, so that their shuffles stay together, and
  // take empty statistics for the blocks before their own.
  const int qb_min = max(key - p.q_start, 0) / kTile;
  const int qb_lo = __reduce_min_sync(0xffffffffu, qb_min);
  if (sum_out != nullptr && h == 0)
    for (int qb = 0; qb < qb_lo; ++qb)
      reinterpret_cast<uint4*>(sum_out + kSumHead)[qb] = make_uint4(0u, 0u, 0u, 0u);
  for (int qb = qb_lo; qb < p.n_qb; ++qb) {
    uint4 r0 = make_uint4(__float_as_uint(-INFINITY), __float_as_uint(-INFINITY),
                          __float_as_uint(-INFINITY), __float_as_uint(-INFINITY));
    uint4 r1 = r0, r2 = make_uint4(0u, 0u, 0u, 0u), r3 = make_uint4(0u, 0u, __float_as_uint(-INFINITY), 0u);
    if (qb >= qb_min) {
      const uint4* r = reinterpret_cast<const uint4*>(base + (long long)qb * kRecWords);
      r0 = r[0]; r1 = r[1]; r2 = r[2]; r3 = r[3];
    }
    top4_insert(top, __uint_as_float(r0.x));
    top4_insert(top, __uint_as_float(r0.y));
    top4_insert(top, __uint_as_float(r0.z));
    top4_insert(top, __uint_as_float(r0.w));
    top4_insert(rtop, __uint_as_float(r1.x));
    top4_insert(rtop, __uint_as_float(r1.y));
    top4_insert(rtop, __uint_as_float(r1.z));
    top4_insert(rtop, __uint_as_float(r1.w));
    hs += __uint_as_float(r2.x);
    hc += r2.y;
    mx = fmaxf(mx, __uint_as_float(r3.z));
    ns += __uint_as_float(r3.w);
    // f5: OR over the heads of the positive-query bits of this block
    const uint32_t w0 = lanes_or<kLanes>(r2.z), w1 = lanes_or<kLanes>(r2.w);
    const uint32_t w2 = lanes_or<kLanes>(r3.x), w3 = lanes_or<kLanes>(r3.y);
    f5cnt += __popc(w0) + __popc(w1) + __popc(w2) + __popc(w3);
    if (sum_out != nullptr && h == 0)
      reinterpret_cast<uint4*>(sum_out + kSumHead)[qb] = make_uint4(w0, w1, w2, w3);
  }
  // f6 for this lane's head: sign of the mean of the top-kf relations over queries
  int f6pos = 0;
  if ((int)hc >= kf) {
    f6pos = 1;
  } else if (hc > 0) {
    // the top kf are the hc positive values and the largest rem non-positive
    // ones: those lie at or below mx, and their mean is at least the mean of
    // all valid - hc non-positive values (ns / (valid - hc)), as rem <= valid - hc
    const float rem = (float)(kf - (int)hc);
    const float mean_np = ns / (float)(valid - (int)hc);
    const float hi = hs + rem * mx;
    const float lo = hs + rem * fmaxf(mean_np, kLogFloor * 1.0001f);
    const float tol = 1e-5f * (fabsf(hs) + rem * fabsf(kLogFloor));
    if (hi < -tol) {
      // definitely not positive
    } else if (lo > tol) {
      f6pos = 1;
    } else if (live) {
      const int slot = atomicAdd(p.queue_count, 1);
      if (slot < p.queue_cap) p.queue[slot] = make_int2((int)gi, h);
      else record_error(p.status, CORE_ERR_UNSUPPORTED, 401, key);
    }
  }
  merge_top4_lanes<kLanes>(top);
  merge_top4_lanes<kLanes>(rtop);
  const float psum = lanes_sum<kLanes>(hs);
  const unsigned int pcnt = lanes_sum<kLanes>(hc);
  f6pos = lanes_sum<kLanes>(f6pos);
  if (!live || h != 0) return;
  if (sum_out != nullptr) {  // this rank's heads only: the cross-rank merge finishes f1..f6
    uint4* o = reinterpret_cast<uint4*>(sum_out);
    o[0] = make_uint4(__float_as_uint(top[0]), __float_as_uint(top[1]), __float_as_uint(top[2]),
                      __float_as_uint(top[3]));
    o[1] = make_uint4(__float_as_uint(rtop[0]), __float_as_uint(rtop[1]), __float_as_uint(rtop[2]),
                      __float_as_uint(rtop[3]));
    o[2] = make_uint4(__float_as_uint(psum), pcnt, __float_as_uint((float)f6pos), 0u);
    return;
  }
  float f[6];
  f[0] = top[0];
  f[1] = sum_top_desc(top, k2) / (float)k2;
  f[2] = psum / (float)(pcnt > 0 ? pcnt : 1);
  f[3] = sum_top_desc(rtop, k4) / (float)k4;
  f[4] = (float)f5cnt / (float)p.nq;
  f[5] = (float)f6pos / (float)p.Hkv;  // undecided heads are added by qk_f6_resolve_kernel
  float* out = p.features + gi * p.stride;
  bool finite = true;
  for (int i = 0; i < 6; ++i) {
    out[i] = f[i];
    finite &= isfinite(f[i]);
  }
  if (!finite) record_error(p.status, CORE_ERR_NONFINITE, 402, key);
}

// Exact resolution of the f6 heads the running statistics could not decide:
// one block per queued (key, head) pair recomputes its relation values over
// all queries, ranks them (descending, ties by query index, i.e. the order of
// a stable descending sort) and tests the mean of the top ceil(valid / 4)
// summed in that order (fused_qk.py:571-578).  A positive head adds 1/Hkv to
// f6; Hkv is a power of two here, so the additions are exact in any order.
constexpr int kResolveThreads = 128;

__global__ void __launch_bounds__(kResolveThreads)
    qk_f6_resolve_kernel(const MergeParams p) {
  __shared__ __align__(16) float s_k[kD];
  __shared__ float s_rel[kMaxSlowNq];
  __shared__ float s_sorted[kMaxSlowNq];
  const int count = min(*p.queue_count, p.queue_cap);
  for (int it = blockIdx.x; it < count; it += gridDim.x) {
    const int2 item = p.queue[it];
    const int bb = (int)(item.x / p.L), kk = (int)(item.x % p.L), h = item.y;
    const long long krow = (((long long)bb * p.Hkv + h) * p.L + kk) * kD;
    for (int e = threadIdx.x; e < kD; e += kResolveThreads)
      s_k[e] = (p.kf != nullptr) ? p.kf[krow + e] : __bfloat162float(p.k[krow + e]);
    __syncthreads();
    for (int t = threadIdx.x; t < p.nq; t += kResolveThreads)
      s_rel[t] = relation_exact(p, bb, h, kk, t, s_k);
    __syncthreads();
    for (int t = threadIdx.x; t < p.nq; t += kResolveThreads) {
      const float v = s_rel[t];
      int r = 0;
      for (int j = 0; j < p.nq; ++j) {
        const float u = s_rel[j];
        r += (u > v || (u == v && j < t)) ? 1 : 0;
      }
      s_sorted[r] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int vld = p.nq - max(kk - p.q_start, 0);
      vld = min(max(vld, 1), p.nq);
      const int kfr = max((vld + 3) / 4, 1);
      float sum = 0.f;
      for (int i = 0; i < kfr; ++i) sum += s_sorted[i];
      if (sum / (float)kfr > 0.f) atomicAdd(p.f6_target + (long long)item.x * p.f6_stride, p.f6_inc);
    }
    __syncthreads();
  }
}


// The same resolution for query buffers longer than kMaxSlowNq (full-scope
// prefill): the pair's relation values over its visible queries go to a
// per-block global scratch row, the ceil(valid / 4)-th largest is found by a
// four-pass radix select on order-preserving 32-bit keys (8-bit digits, block
// histograms), and the sum of the top values is the sum of those above it
// plus the tied copies of it.  Ties change nothing: equal values add equally.
constexpr int kResolveLargeThreads = 256;

__device__ __forceinline__ uint32_t float_order_key(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // ascending keys for ascending floats
}

__global__ void __launch_bounds__(kResolveLargeThreads)
    qk_f6_resolve_large_kernel(const MergeParams p, float* __restrict__ scratch) {
  __shared__ __align__(16) float s_k[kD];
  __shared__ int s_hist[256];
  __shared__ uint32_t s_prefix;
  __shared__ int s_remaining;
  __shared__ float s_red[kResolveLargeThreads / 32];
  float* vals = scratch + (long long)blockIdx.x * p.nq;
  const int count = min(*p.queue_count, p.queue_cap);
  for (int it = blockIdx.x; it < count; it += gridDim.x) {
    const int2 item = p.queue[it];
    const int bb = (int)(item.x / p.L), kk = (int)(item.x % p.L), h = item.y;
    const long long krow = (((long long)bb * p.Hkv + h) * p.L + kk) * kD;
    for (int e = threadIdx.x; e < kD; e += kResolveLargeThreads)
      s_k[e] = (p.kf != nullptr) ? p.kf[krow + e] : __bfloat162float(p.k[krow + e]);
    __syncthreads();
    const int t0 = max(kk - p.q_start, 0);  // first query that sees the key
    const int n = p.nq - t0;                 // the key's valid count (>= 1)
    for (int i = threadIdx.x; i < n; i += kResolveLargeThreads)
      vals[i] = relation_exact(p, bb, h, kk, t0 + i, s_k);
    __syncthreads();
    const int kf = max((n + 3) / 4, 1);
    if (threadIdx.x == 0) {
      s_prefix = 0u;
      s_remaining = kf;  // rank of the threshold among the values still matching the prefix
    }
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = threadIdx.x; i < 256; i += kResolveLargeThreads) s_hist[i] = 0;
      __syncthreads();
      const uint32_t hi_mask = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
      const uint32_t prefix = s_prefix;
      for (int i = threadIdx.x; i < n; i += kResolveLargeThreads) {
        const uint32_t key = float_order_key(vals[i]);
        if ((key & hi_mask) == prefix) atomicAdd(&s_hist[(key >> shift) & 255], 1);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        int rem = s_remaining, dgt = 255;
        for (; dgt > 0; --dgt) {  // largest digits first
          if (s_hist[dgt] >= rem) break;
          rem -= s_hist[dgt];
        }
        s_prefix = prefix | ((uint32_t)dgt << shift);
        s_remaining = rem;  // copies of the threshold among the top kf
      }
      __syncthreads();
    }
    const uint32_t thr = s_prefix;
    float part = 0.f;
    for (int i = threadIdx.x; i < n; i += kResolveLargeThreads) {
      const float v = vals[i];
      if (float_order_key(v) > thr) part += v;
    }
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = part;
    __syncthreads();
    if (threadIdx.x == 0) {
      float sum = 0.f;
      for (int w = 0; w < kResolveLargeThreads / 32; ++w) sum += s_red[w];
      const uint32_t tu = (thr & 0x80000000u) ? (thr & 0x7FFFFFFFu) : ~thr;  // back to float bits
      sum += (float)s_remaining * __uint_as_float(tu);
      if (sum / (float)kf > 0.f) atomicAdd(p.f6_target + (long long)item.x * p.f6_stride, p.f6_inc);
    }
    __syncthreads();
  }
}

// Cross-rank merge of head-sharded summaries (one sequence): for keys key0 +
// [0, n) the n_parts summaries of the ranks' KV heads (each written by
// qk_merge_kernel in summary mode over that rank's heads) combine into f1..f6
// exactly as qk_merge_kernel combines heads: the union's top 4 (order-free),
// summed positive mass and counts, the OR of the positive-query bits, and the
// positive-head count over all Hkv heads.
struct SumMergeParams {
  const uint32_t* parts;   // (n_parts, part_rows, sum_words)
  long long part_rows;
  int n_parts, n, key0, L, nq, q_start, n_qb, Hkv, topk, n_recent, sum_words;
  float* features;         // rows key0 .. key0 + n - 1 at features + i * stride
  int stride;
  DeviceStatus* status;
};

__global__ void __launch_bounds__(kMergeThreads)
    qk_summary_merge_kernel(const SumMergeParams p) {
  const int i = blockIdx.x * kMergeThreads + threadIdx.x;
  if (i >= p.n) return;
  const int key = p.key0 + i;
  int valid = p.nq - max(key - p.q_start, 0);
  valid = min(max(valid, 1), p.nq);
  const int k2max = min(p.topk, p.nq * p.Hkv);
  const int k2 = min(max(valid * p.Hkv, 1), k2max);
  const int nrec = p.n_recent;
  const int rstart = p.q_start + p.nq - nrec;
  int rvalid = p.q_start + p.nq - max(key, rstart);
  rvalid = min(max(rvalid, 1), nrec);
  const int k4max = min(p.topk, nrec * p.Hkv);
  const int k4 = min(max(rvalid * p.Hkv, 1), k4max);
  float top[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  float rtop[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  float psum = 0.f, f6pos = 0.f;
  unsigned long long pcnt = 0;
  for (int part = 0; part < p.n_parts; ++part) {
    const uint4* r = reinterpret_cast<const uint4*>(
        p.parts + ((long long)part * p.part_rows + i) * p.sum_words);
    const uint4 r0 = r[0], r1 = r[1], r2 = r[2];
    top4_insert(top, __uint_as_float(r0.x));
    top4_insert(top, __uint_as_float(r0.y));
    top4_insert(top, __uint_as_float(r0.z));
    top4_insert(top, __uint_as_float(r0.w));
    top4_insert(rtop, __uint_as_float(r1.x));
    top4_insert(rtop, __uint_as_float(r1.y));
    top4_insert(rtop, __uint_as_float(r1.z));
    top4_insert(rtop, __uint_as_float(r1.w));
    psum += __uint_as_float(r2.x);
    pcnt += r2.y;
    f6pos += __uint_as_float(r2.z);
  }
  int f5cnt = 0;
  for (int qb = 0; qb < p.n_qb; ++qb) {
    uint4 w = make_uint4(0u, 0u, 0u, 0u);
    for (int part = 0; part < p.n_parts; ++part) {
      const uint4 x = reinterpret_cast<const uint4*>(
          p.parts + ((long long)part * p.part_rows + i) * p.sum_words + kSumHead)[qb];
      w.x |= x.x;
      w.y |= x.y;
      w.z |= x.z;
      w.w |= x.w;
    }
    f5cnt += __popc(w.x) + __popc(w.y) + __popc(w.z) + __popc(w.w);
  }
  float f[6];
  f[0] = top[0];
  f[1] = sum_top_desc(top, k2) / (float)k2;
  f[2] = psum / (float)(pcnt > 0 ? pcnt : 1);
  f[3] = sum_top_desc(rtop, k4) / (float)k4;
  f[4] = (float)f5cnt / (float)p.nq;
  f[5] = f6pos / (float)p.Hkv;
  float* out = p.features + (long long)i * p.stride;
  bool finite = true;
  for (int j = 0; j < 6; ++j) {
    out[j] = f[j];
    finite &= isfinite(f[j]);
  }
  if (!finite) record_error(p.status, CORE_ERR_NONFINITE, 403, key);
}

}  // namespace qk
}  // namespace core

using namespace core;
using namespace core::qk;

namespace {

struct QKPlan {
  Params p;
  int grid;
  size_t part_elems, rec_words;
};

int plan_qk(const core_dims_t* d, int topk, int n_recent, QKPlan* out) {
  Params& p = out->p;
  p = Params{};
  p.B = d->batch;
  p.Hq = d->n_q_heads;
  p.Hkv = d->n_kv_heads;
  p.G = p.Hq / p.Hkv;
  p.nq = d->n_queries;
  p.L = d->seq_len;
  p.q_start = p.L - p.nq;
  p.n_qb = (p.nq + kTile - 1) / kTile;
  p.n_kt = (p.L + kTile - 1) / kTile;
  p.U = (long long)p.B * p.Hkv * p.n_qb * p.n_kt;
  p.scale = 1.0f / sqrtf((float)kD);
  p.scale_log2 = p.scale * kLog2e;
  p.head_topk = topk < p.G ? topk : p.G;
  p.n_recent = n_recent < p.nq ? n_recent : p.nq;
  const int sms = sm_count();
  out->grid = (int)(p.U < sms ? p.U : sms);
  // slots: kLseTeams epilogue teams x CTAs overlapping one group
  int maxc = 1;
  const long long groups = p.U / p.n_kt;
  for (long long g = 0; g < groups; ++g) {
    int lo = cta_of_unit(g * p.n_kt, p.U, out->grid);
    int hi = cta_of_unit(g * p.n_kt + kt_last(p, (int)(g % p.n_qb)), p.U, out->grid);
    if (hi - lo + 1 > maxc) maxc = hi - lo + 1;
  }
  p.slot_stride = kLseTeams * maxc;
  out->part_elems = (size_t)p.B * p.Hq * p.nq * p.slot_stride;
  out->rec_words = (size_t)p.B * p.L * p.Hkv * p.n_qb * kRecWords;
  return CORE_OK;
}

template <int G>
int launch_qk(const QKPlan& plan, const CUtensorMap& tmQ_lse, const CUtensorMap& tmQ_rel,
              const CUtensorMap& tmK, bool run_lse, float* lse_buf, cudaStream_t s,
              cudaEvent_t ev0, cudaEvent_t ev1) {
  const Params& p = plan.p;
  cudaError_t e;
  if (run_lse) {
    const uint32_t smem = LseSmem<G>::kTotal + 1024;
    e = cudaFuncSetAttribute(qk_lse_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_error(e, "qk_lse_kernel attribute");
    qk_lse_kernel<G><<<plan.grid, kLseThreads, smem, s>>>(tmQ_lse, tmK, p);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "qk_lse_kernel launch");
    const long long n = (long long)p.B * p.Hq * p.nq;
    lse_combine_kernel2<<<(unsigned)((8 * n + 255) / 256), 256, 0, s>>>(p, plan.grid, lse_buf);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "lse_combine launch");
  }
  const uint32_t smem = RelSmem<G>::kTotal + 1024;
  const bool loo = p.head_topk < G;
  auto kern = loo ? qk_relation_kernel<G, (G > 1)> : qk_relation_kernel<G, false>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_error(e, "qk_relation_kernel attribute");
  if (ev0 != nullptr) cudaEventRecord(ev0, s);
  kern<<<plan.grid, kThreads, smem, s>>>(tmQ_rel, tmK, p);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "qk_relation_kernel launch");
  if (ev1 != nullptr) cudaEventRecord(ev1, s);
  return CORE_OK;
}

}  // namespace

// Blocks of qk_f6_resolve_large_kernel and their scratch rows (one relation
// value per query of the buffer each).
static int resolve_large_blocks() { return 2 * sm_count(); }
static size_t resolve_scratch_floats(const core_dims_t* d) {
  return (size_t)resolve_large_blocks() * d->n_queries;
}

static size_t queue_cap_for(const core_dims_t* d) {
  // undecided f6 heads: bounded by every (key, head) pair of the cache
  return (size_t)d->batch * d->seq_len * d->n_kv_heads;
}

extern "C" size_t core_qk_features_workspace_bytes(const core_dims_t* d) {
  if (check_dims(d, "core_qk_features_workspace_bytes", true) != CORE_OK) return 0;
  QKPlan plan;
  plan_qk(d, 4, 16, &plan);
  Sizer z;
  z.take<float2>(plan.part_elems);
  z.take<float>((size_t)d->batch * d->n_q_heads * d->n_queries);
  z.take<uint32_t>(plan.rec_words);
  z.take<int>(1);
  z.take<int2>(queue_cap_for(d));
  if (d->n_queries > kMaxSlowNq) z.take<float>(resolve_scratch_floats(d));
  return z.used;
}

namespace core {
int qk_f32_records(const core_dims_t* d, int q_start, int n_qb, int head_topk, int n_recent,
                   float scale, const float* q, const float* k, bool run_lse, float* lse,
                   uint32_t* rec, cudaStream_t s);
int qk_features_impl(const core_dims_t* d, const void* q, const void* k, int32_t topk_qk,
                     int32_t n_recent_queries, const float* lse_in, float* lse_out,
                     float* features, int32_t feature_stride, void* workspace,
                     size_t workspace_bytes, void* stream, void* ev0, void* ev1,
                     uint32_t* summary = nullptr);
}

extern "C" int core_qk_features(const core_dims_t* d, const void* q, const void* k,
                                int32_t topk_qk, int32_t n_recent_queries, const float* lse_in,
                                float* lse_out, float* features, int32_t feature_stride,
                                void* workspace, size_t workspace_bytes, void* stream) {
  return core::qk_features_impl(d, q, k, topk_qk, n_recent_queries, lse_in, lse_out, features,
                                feature_stride, workspace, workspace_bytes, stream, nullptr,
                                nullptr);
}

int core::qk_features_impl(const core_dims_t* d, const void* q, const void* k, int32_t topk_qk,
                           int32_t n_recent_queries, const float* lse_in, float* lse_out,
                           float* features, int32_t feature_stride, void* workspace,
                           size_t workspace_bytes, void* stream, void* ev0_, void* ev1_,
                           uint32_t* summary) {
  cudaEvent_t ev0 = static_cast<cudaEvent_t>(ev0_), ev1 = static_cast<cudaEvent_t>(ev1_);
  int rc = check_dims(d, "core_qk_features", true);
  if (rc != CORE_OK) return rc;
  const bool f32 = d->dtype == CORE_DTYPE_F32;
  if (q == nullptr || k == nullptr || (features == nullptr && summary == nullptr))
    return set_error(CORE_ERR_INVALID_ARG, "core_qk_features: NULL tensor");
  if (d->n_queries <= 0) return set_error(CORE_ERR_INVALID_ARG, "core_qk_features: no queries");
  if (topk_qk <= 0 || topk_qk > 4)
    return set_error(CORE_ERR_UNSUPPORTED, "core_qk_features: topk_qk must be in 1..4");
  const int G = d->n_q_heads / d->n_kv_heads;
  if (topk_qk < G - 1)
    return set_error(CORE_ERR_UNSUPPORTED,
                     "core_qk_features: requires topk_qk >= group size - 1 (fused_qk.py:19-21)");
  if (n_recent_queries <= 0) return set_error(CORE_ERR_INVALID_ARG, "core_qk_features: n_recent <= 0");
  if (summary == nullptr && feature_stride < 6)
    return set_error(CORE_ERR_INVALID_ARG, "core_qk_features: feature_stride < 6");
  QKPlan plan;
  plan_qk(d, topk_qk, n_recent_queries, &plan);
  Params& p = plan.p;
  Carver c(workspace, workspace_bytes);
  p.part = c.take<float2>(plan.part_elems);
  float* lse_buf = c.take<float>((size_t)p.B * p.Hq * p.nq);
  p.rec = c.take<uint32_t>(plan.rec_words);
  int* queue_count = c.take<int>(1);
  int2* queue = c.take<int2>(queue_cap_for(d));
  float* resolve_scratch = p.nq > kMaxSlowNq ? c.take<float>(resolve_scratch_floats(d)) : nullptr;
  if (c.overflow)
    return set_error(CORE_ERR_WORKSPACE, "core_qk_features: workspace too small");
  p.status = device_status();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (lse_in != nullptr) {
    e = cudaMemcpyAsync(lse_buf, lse_in, sizeof(float) * (size_t)p.B * p.Hq * p.nq,
                        cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return cuda_error(e, "core_qk_features lse copy");
  }
  p.lse = lse_buf;

  const bool run_lse = (lse_in == nullptr);
  if (f32) {
    if (ev0 != nullptr) cudaEventRecord(ev0, s);
    rc = qk_f32_records(d, p.q_start, p.n_qb, p.head_topk, p.n_recent, p.scale,
                        static_cast<const float*>(q), static_cast<const float*>(k), run_lse,
                        lse_buf, p.rec, s);
    if (ev1 != nullptr) cudaEventRecord(ev1, s);
    if (rc != CORE_OK) return rc;
  } else {
  // Tensor maps: Q as (B*Hq, nq, 128) and K as (B*Hkv, L, 128), bf16, 128 B swizzle.
  CUtensorMap tmQ_lse, tmQ_rel, tmK;
  {
    uint64_t dims[3] = {128, (uint64_t)p.nq, (uint64_t)p.B * p.Hq};
    uint64_t str[2] = {256, (uint64_t)p.nq * 256};
    uint32_t box_lse[3] = {64, 128, 1};
    uint32_t box_rel[3] = {64, (uint32_t)kRelQ, 1};
    if ((rc = make_tmap_bf16(&tmQ_lse, q, 3, dims, str, box_lse, true)) != CORE_OK) return rc;
    if ((rc = make_tmap_bf16(&tmQ_rel, q, 3, dims, str, box_rel, true)) != CORE_OK) return rc;
  }
  {
    uint64_t dims[3] = {128, (uint64_t)p.L, (uint64_t)p.B * p.Hkv};
    uint64_t str[2] = {256, (uint64_t)p.L * 256};
    uint32_t box[3] = {64, 128, 1};
    if ((rc = make_tmap_bf16(&tmK, k, 3, dims, str, box, true)) != CORE_OK) return rc;
  }
  switch (p.G) {
    case 1: rc = launch_qk<1>(plan, tmQ_lse, tmQ_rel, tmK, run_lse, lse_buf, s, ev0, ev1); break;
    case 2: rc = launch_qk<2>(plan, tmQ_lse, tmQ_rel, tmK, run_lse, lse_buf, s, ev0, ev1); break;
    case 4: rc = launch_qk<4>(plan, tmQ_lse, tmQ_rel, tmK, run_lse, lse_buf, s, ev0, ev1); break;
    default: return set_error(CORE_ERR_UNSUPPORTED, "core_qk_features: group size");
  }
  if (rc != CORE_OK) return rc;
  }

  MergeParams mp{};
  mp.B = p.B; mp.Hq = p.Hq; mp.Hkv = p.Hkv; mp.G = p.G; mp.nq = p.nq; mp.L = p.L;
  mp.q_start = p.q_start; mp.n_qb = p.n_qb; mp.topk = topk_qk; mp.n_recent = p.n_recent;
  mp.head_topk = p.head_topk; mp.scale = p.scale; mp.rec = p.rec;
  mp.q = f32 ? nullptr : static_cast<const __nv_bfloat16*>(q);
  mp.k = f32 ? nullptr : static_cast<const __nv_bfloat16*>(k);
  mp.qf = f32 ? static_cast<const float*>(q) : nullptr;
  mp.kf = f32 ? static_cast<const float*>(k) : nullptr;
  mp.lse = lse_buf; mp.features = features; mp.stride = feature_stride; mp.status = p.status;
  mp.queue_count = queue_count; mp.queue = queue; mp.queue_cap = (int)queue_cap_for(d);
  mp.summary = summary;
  mp.sum_words = kSumHead + 4 * p.n_qb;
  if (summary != nullptr) {
    mp.f6_target = reinterpret_cast<float*>(summary) + 10;
    mp.f6_stride = mp.sum_words;
    mp.f6_inc = 1.0f;
  } else {
    mp.f6_target = features + 5;
    mp.f6_stride = feature_stride;
    mp.f6_inc = 1.0f / (float)p.Hkv;
  }
  if ((p.Hkv & (p.Hkv - 1)) != 0)
    return set_error(CORE_ERR_UNSUPPORTED, "core_qk_features: n_kv_heads must be a power of two");
  e = cudaMemsetAsync(queue_count, 0, sizeof(int), s);
  if (e != cudaSuccess) return cuda_error(e, "core_qk_features queue clear");
  const long long n = (long long)p.B * p.L;
  {
    // Hkv lanes per key (a power of two, checked above)
    const long long threads = n * p.Hkv;
    const unsigned blocks = (unsigned)((threads + kMergeThreads - 1) / kMergeThreads);
    switch (p.Hkv) {
      case 1: qk_merge_kernel<1><<<blocks, kMergeThreads, 0, s>>>(mp); break;
      case 2: qk_merge_kernel<2><<<blocks, kMergeThreads, 0, s>>>(mp); break;
      case 4: qk_merge_kernel<4><<<blocks, kMergeThreads, 0, s>>>(mp); break;
      case 8: qk_merge_kernel<8><<<blocks, kMergeThreads, 0, s>>>(mp); break;
      case 16: qk_merge_kernel<16><<<blocks, kMergeThreads, 0, s>>>(mp); break;
      default: return set_error(CORE_ERR_UNSUPPORTED, "core_qk_features: at most 16 KV heads");
    }
  }
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "qk_merge_kernel launch");
  if (p.nq <= kMaxSlowNq)
    qk_f6_resolve_kernel<<<4 * sm_count(), kResolveThreads, 0, s>>>(mp);
  else
    qk_f6_resolve_large_kernel<<<resolve_large_blocks(), kResolveLargeThreads, 0, s>>>(mp,
                                                                                 resolve_scratch);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "qk_f6_resolve_kernel launch");
  if (lse_out != nullptr) {
    e = cudaMemcpyAsync(lse_out, lse_buf, sizeof(float) * (size_t)p.B * p.Hq * p.nq,
                        cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return cuda_error(e, "core_qk_features lse copy out");
  }
  return CORE_OK;
}

extern "C" int32_t core_qk_summary_words(int32_t n_queries) {
  if (n_queries <= 0) return 0;
  return kSumHead + 4 * ((n_queries + kTile - 1) / kTile);
}

extern "C" int core_qk_head_summary(const core_dims_t* d, const void* q, const void* k,
                                    int32_t topk_qk, int32_t n_recent_queries, float* lse_out,
                                    uint32_t* summary, void* workspace, size_t workspace_bytes,
                                    void* stream) {
  if (summary == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_qk_head_summary: NULL summary");
  if (reinterpret_cast<uintptr_t>(summary) % 16 != 0)
    return set_error(CORE_ERR_INVALID_ARG, "core_qk_head_summary: summary must be 16-byte aligned");
  return core::qk_features_impl(d, q, k, topk_qk, n_recent_queries, nullptr, lse_out, nullptr, 0,
                                workspace, workspace_bytes, stream, nullptr, nullptr, summary);
}

extern "C" int core_qk_merge_summaries(const uint32_t* parts, int32_t n_parts, int64_t part_rows,
                                       int32_t key0, int32_t n_keys, int32_t seq_len,
                                       int32_t n_queries, int32_t n_kv_heads, int32_t topk_qk,
                                       int32_t n_recent_queries, float* features,
                                       int32_t feature_stride, void* stream) {
  if (parts == nullptr || features == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_qk_merge_summaries: NULL tensor");
  if (reinterpret_cast<uintptr_t>(parts) % 16 != 0)
    return set_error(CORE_ERR_INVALID_ARG, "core_qk_merge_summaries: parts must be 16-byte aligned");
  if (n_parts <= 0 || n_keys < 0 || key0 < 0 || key0 + n_keys > seq_len || part_rows < n_keys ||
      n_queries <= 0 || n_queries > seq_len || n_kv_heads <= 0 || feature_stride < 6)
    return set_error(CORE_ERR_INVALID_ARG, "core_qk_merge_summaries: bad sizes");
  if (topk_qk <= 0 || topk_qk > 4 || n_recent_queries <= 0)
    return set_error(CORE_ERR_INVALID_ARG, "core_qk_merge_summaries: bad topk / n_recent");
  if (n_keys == 0) return CORE_OK;
  SumMergeParams p{};
  p.parts = parts;
  p.part_rows = part_rows;
  p.n_parts = n_parts;
  p.n = n_keys;
  p.key0 = key0;
  p.L = seq_len;
  p.nq = n_queries;
  p.q_start = seq_len - n_queries;
  p.n_qb = (n_queries + kTile - 1) / kTile;
  p.Hkv = n_kv_heads;
  p.topk = topk_qk;
  p.n_recent = n_recent_queries < n_queries ? n_recent_queries : n_queries;
  p.sum_words = kSumHead + 4 * p.n_qb;
  p.features = features;
  p.stride = feature_stride;
  p.status = device_status();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  qk_summary_merge_kernel<<<(unsigned)((n_keys + kMergeThreads - 1) / kMergeThreads), kMergeThreads,
                            0, s>>>(p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CORE_OK : cuda_error(e, "qk_summary_merge_kernel launch");
}
