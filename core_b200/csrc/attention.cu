// Causal prefill attention with the row log-sum-exp exported: the
// FlashAttention-2 forward that the reference's attention hook calls
// (core/kvpress_pipeline.py:24-91, _core_flash_attention_forward: causal,
// no dropout, softmax scale d^-0.5, return_attn_probs only for softmax_lse),
// written for tcgen05.  The LSE it exports is what the press reuses as the
// row normaliser of the QK relation pass (core/fused_qk.py:444-456), so a
// prefill that runs this kernel skips the LSE pass of core_qk_features.
//
// One CTA per SM, persistent over units (batch row, query head, 128-query
// tile), heaviest tiles first.  Warp 0 issues TMA loads (Q once per unit, K
// and V tiles of 128 keys double-buffered), warp 1 issues the MMAs, warps 4-7
// run the online softmax, one thread per query row:
//
//   S_j  = Q K_j^T            tcgen05, 128 x 128 x 128 into TMEM (two buffers)
//   P_j  = exp2(S_j s log2e - m)   bf16/f16 into swizzled shared memory
//   O   += P_j V_j            tcgen05, A = P from shared memory, B = V tile
//                             (MN-major), O resident in TMEM
//
// The running maximum m of a row is raised only when a tile's maximum exceeds
// it by more than 2^8 (then O and the row sum are rescaled in TMEM after the
// previous P V product has landed); otherwise P stays below 2^8 and no
// rescale is needed.  O / l and LSE = (m + log2 l) ln 2 are written at the end.
#include <cmath>

#include "common.cuh"
#include "host_util.h"

namespace core {
namespace attn {

constexpr int kD = 128;
constexpr int kTile = 128;
constexpr int kThreads = 384;  // warp 0 TMA, warp 1 MMA, warps 4-7 / 8-11 softmax (key halves)
constexpr uint32_t kTileBytes = kTile * kD * 2;  // 32 KB: a Q, K, V or P tile
constexpr uint32_t kAtomBytes = kTile * 128u;    // 16 KB: 64 columns of 128 rows
constexpr int kStages = 2;
constexpr float kRescaleLog2 = 8.0f;  // P <= 2^8 before the maximum is raised

struct Smem {
  static constexpr uint32_t kQ = 0;
  static constexpr uint32_t kK = kQ + kTileBytes;
  static constexpr uint32_t kV = kK + kStages * kTileBytes;
  static constexpr uint32_t kP = kV + kStages * kTileBytes;
  static constexpr uint32_t kBar = kP + 2 * kTileBytes;
  static constexpr uint32_t kTotal = kBar + 256;
};

struct Params {
  int B, Hq, Hkv, G, Lq, Lk, off, n_qt;
  long long U;       // units = B * Hq * n_qt
  float scale_log2;  // softmax scale * log2(e)
  void* out;         // (B, Lq, Hq, d), 16-bit
  float* lse;        // (B, Hq, Lq), natural log
  DeviceStatus* status;
};

struct Unit {
  int b, qh, qt, n_kt;
};

// Units in order of decreasing work: the last query tile of every (b, head)
// first, so that the static round-robin over CTAs balances the causal rows.
__device__ __forceinline__ Unit decode(long long u, const Params& p) {
  Unit r;
  const long long bh_n = (long long)p.B * p.Hq;
  const int bh = (int)(u % bh_n);
  r.qt = p.n_qt - 1 - (int)(u / bh_n);
  r.qh = bh % p.Hq;
  r.b = bh / p.Hq;
  const int last_row = min(r.qt * kTile + kTile - 1, p.Lq - 1);
  r.n_kt = min((last_row + p.off) / kTile + 1, (p.Lk + kTile - 1) / kTile);
  return r;
}

template <bool kF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (kF16) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

template <bool kF16>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  const uint32_t sQ = sbase + Smem::kQ, sK = sbase + Smem::kK, sV = sbase + Smem::kV,
                 sP = sbase + Smem::kP;
  const uint32_t bar = sbase + Smem::kBar;
  const uint32_t bar_q_full = bar, bar_q_empty = bar + 8, bar_o_empty = bar + 16;
  auto bar_k_full = [&](int s) { return bar + 24 + 8u * s; };
  auto bar_k_empty = [&](int s) { return bar + 40 + 8u * s; };
  auto bar_v_full = [&](int s) { return bar + 56 + 8u * s; };
  auto bar_v_empty = [&](int s) { return bar + 72 + 8u * s; };
  auto bar_s_full = [&](int s) { return bar + 88 + 8u * s; };
  auto bar_s_empty = [&](int s) { return bar + 104 + 8u * s; };
  auto bar_p_full = [&](int s) { return bar + 120 + 8u * s; };
  auto bar_pv_done = [&](int s) { return bar + 136 + 8u * s; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + Smem::kBar + 200);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sgen + Smem::kBar + 208);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long P = gridDim.x;

  if (threadIdx.x == 0) {
    mbar_init(bar_q_full, 1);
    mbar_init(bar_q_empty, 1);
    mbar_init(bar_o_empty, 8);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar_k_full(s), 1);
      mbar_init(bar_k_empty(s), 1);
      mbar_init(bar_v_full(s), 1);
      mbar_init(bar_v_empty(s), 1);
      mbar_init(bar_s_full(s), 1);
      mbar_init(bar_s_empty(s), 8);
      mbar_init(bar_p_full(s), 8);
      mbar_init(bar_pv_done(s), 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    // S0 [0,128), S1 [128,256), O [256,384); columns 384.. carry the softmax
    // groups' exchanges (row maxima by tile parity, then row sums)
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
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
      int g = 0, un = 0;
      bool ok = true;
      for (long long u = blockIdx.x; u < p.U && ok; u += P, ++un) {
        const Unit t = decode(u, p);
        const int kvh = t.qh / p.G;
        if (un > 0 && !(ok = wait(bar_q_empty, (un - 1) & 1, 1301))) break;
        mbar_arrive_expect_tx(bar_q_full, kTileBytes);
        for (int a = 0; a < 2; ++a)
          tma_load_4d(sQ + a * kAtomBytes, &tmQ, bar_q_full, a * 64, t.qt * kTile, t.qh, t.b);
        for (int j = 0; j < t.n_kt; ++j, ++g) {
          const int st = g & 1;
          if (g >= 2 && !(ok = wait(bar_k_empty(st), ((g >> 1) - 1) & 1, 1302))) break;
          mbar_arrive_expect_tx(bar_k_full(st), kTileBytes);
          for (int a = 0; a < 2; ++a)
            tma_load_4d(sK + st * kTileBytes + a * kAtomBytes, &tmK, bar_k_full(st), a * 64,
                        j * kTile, kvh, t.b);
          if (g >= 2 && !(ok = wait(bar_v_empty(st), ((g >> 1) - 1) & 1, 1303))) break;
          mbar_arrive_expect_tx(bar_v_full(st), kTileBytes);
          for (int a = 0; a < 2; ++a)
            tma_load_4d(sV + st * kTileBytes + a * kAtomBytes, &tmV, bar_v_full(st), a * 64,
                        j * kTile, kvh, t.b);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t fmt = kF16 ? 0u : 1u;  // kind::f16 operand format: 0 f16, 1 bf16
      constexpr uint32_t idesc_qk = (1u << 4) | (fmt << 7) | (fmt << 10) |
                                    ((uint32_t)(kTile >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
      constexpr uint32_t idesc_pv = idesc_qk | (1u << 16);  // B (the V tile) MN-major
      int g0 = 0, un = 0;
      bool ok = true;
      for (long long u = blockIdx.x; u < p.U && ok; u += P, ++un) {
        const Unit t = decode(u, p);
        if (!(ok = wait(bar_q_full, un & 1, 1311))) break;
        // QK_0, QK_1, PV_0, QK_2, PV_1, ..., QK_{n-1}, PV_{n-2}, PV_{n-1}
        for (int j = 0; j <= t.n_kt && ok; ++j) {
          if (j < t.n_kt) {
            const int g = g0 + j, sb = g & 1;
            if (!(ok = wait(bar_k_full(sb), (g >> 1) & 1, 1312))) break;
            if (g >= 2 && !(ok = wait(bar_s_empty(sb), ((g >> 1) - 1) & 1, 1313))) break;
            tc_fence_after();
            const uint32_t d = tmem + (uint32_t)(sb * kTile);
            for (int ks = 0; ks < 8; ++ks) {
              const uint32_t off = (uint32_t)(ks >> 2) * kAtomBytes + (uint32_t)(ks & 3) * 32u;
              mma_bf16(d, sdesc_kmajor(sQ + off), sdesc_kmajor(sK + sb * kTileBytes + off), idesc_qk,
                       ks > 0 ? 1u : 0u);
            }
            mma_commit(bar_s_full(sb));
            mma_commit(bar_k_empty(sb));
            if (j == t.n_kt - 1) mma_commit(bar_q_empty);
          }
          if (j >= 1) {
            const int g = g0 + j - 1, pb = g & 1;
            if (!(ok = wait(bar_v_full(pb), (g >> 1) & 1, 1314))) break;
            if (!(ok = wait(bar_p_full(pb), (g >> 1) & 1, 1315))) break;
            if (j == 1 && un > 0 && !(ok = wait(bar_o_empty, (un - 1) & 1, 1316))) break;
            tc_fence_after();
            for (int ks = 0; ks < 8; ++ks) {
              const uint64_t a = sdesc_kmajor(sP + pb * kTileBytes + (uint32_t)(ks >> 2) * kAtomBytes +
                                              (uint32_t)(ks & 3) * 32u);
              const uint64_t b = sdesc_sw128(sV + pb * kTileBytes + (uint32_t)ks * 16u * 128u,
                                             kAtomBytes, 1024u);
              mma_bf16(tmem + 2 * kTile, a, b, idesc_pv, (j > 1 || ks > 0) ? 1u : 0u);
            }
            mma_commit(bar_pv_done(pb));
            mma_commit(bar_v_empty(pb));
          }
        }
        g0 += t.n_kt;
      }
    }
  } else if (warp >= 4) {
    // ---------------- softmax and epilogue ----------------
    // Two warpgroups, one thread per query row in each: group h takes keys
    // [64 h, 64 h + 64) of every tile and columns [64 h, 64 h + 64) of O.  The
    // row maximum of a tile is exchanged through TMEM (warps 4 + w and 8 + w
    // reach the same lanes): column 384 + 2 (tile parity) + h.  Each group
    // keeps its own partial row sum; they meet in columns 388 + h and are added
    // group 0 first.
    const int half = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(wq * 32) << 16);
    const uint32_t x_col = lane_base + 3 * kTile;  // column 384 of this warp's lanes
    const unsigned long long sc2 = f2_pack(p.scale_log2, p.scale_log2);
    int g0 = 0;
    bool ok = true;
    for (long long u = blockIdx.x; u < p.U && ok; u += P) {
      const Unit t = decode(u, p);
      const int i = t.qt * kTile + r;  // query row within Lq
      const int lim = i + p.off;        // last key this row sees
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < t.n_kt; ++j) {
        const int g = g0 + j, sb = g & 1;
        bool got = ok && wait(bar_s_full(sb), (g >> 1) & 1, 1321);
        got = __all_sync(0xffffffffu, got);
        const int key0 = j * kTile + half * 64;  // first key of this group's half
        // some row of the tile masks some key of this half
        const bool masked = key0 + 63 > t.qt * kTile + p.off;
        const uint32_t tS = lane_base + (uint32_t)(sb * kTile + half * 64);
        float mx = -INFINITY;
        if (got) {
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            float v[32];
            tmem_ld32(tS + (uint32_t)(c * 32), v);
            if (!masked) {
#pragma unroll
              for (int e = 0; e < 32; e += 2) mx = fmax3(mx, v[e], v[e + 1]);
            } else {
#pragma unroll
              for (int e = 0; e < 32; ++e) mx = fmaxf(mx, key0 + c * 32 + e <= lim ? v[e] : -INFINITY);
            }
          }
          tmem_st1(x_col + (uint32_t)((g & 1) * 2 + half), mx);
          tc_fence_before();
        }
        // the groups' halves meet here (also a uniform decision after the waits)
        if (!named_barrier_and(1, 256, got)) { ok = false; break; }
        tc_fence_after();
        mx = fmaxf(mx, tmem_ld1(x_col + (uint32_t)((g & 1) * 2 + (half ^ 1))));
        const float mt = mx * p.scale_log2;  // the scale is positive
        const bool raise = mt > m_used + kRescaleLog2;
        // both groups take the same decision for a row (same m_used, same mt);
        // TMEM loads and stores are warp-collective, so a warp rescales
        // together, rows that keep their maximum with a factor of exactly 1
        // A wait that gives up below only clears `ok` (warp-uniform): the
        // groups must reach the same named barriers, so the failure stops them
        // together at the next one.
        if (__any_sync(0xffffffffu, raise)) {
          if (j > 0) {
            // rescale this group's O columns and l once the previous P V product has landed
            const int gp = g - 1;
            ok = __all_sync(0xffffffffu, wait(bar_pv_done(gp & 1), (gp >> 1) & 1, 1322));
          }
          if (j > 0 && ok) {
            tc_fence_after();
            const float f = raise ? ex2_approx(m_used - mt) : 1.0f;
            l *= f;
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
              const uint32_t ta = lane_base + 2 * kTile + (uint32_t)(half * 64 + c * 32);
              float o[32];
              tmem_ld32(ta, o);
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] *= f;
              tmem_st32(ta, o);
            }
          }
          if (raise) m_used = mt;
        }
        const float msub = m_used == -INFINITY ? 0.f : m_used;
        // the P buffer was last read by the P V product of tile g - 2
        if (ok && g >= 2) ok = __all_sync(0xffffffffu, wait(bar_pv_done(sb), ((g >> 1) - 1) & 1, 1323));
        if (!ok) continue;  // the next barrier stops both groups
        // pass 2: P = exp2(s * scale * log2e - m), the partial row sum, P into shared memory
        const unsigned long long neg2 = f2_pack(-msub, -msub);
        unsigned long long acc = 0ull;
        const uint32_t prow = sP + sb * kTileBytes + (uint32_t)half * kAtomBytes + (uint32_t)r * 128u;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          float v[32];
          tmem_ld32(tS + (uint32_t)(c * 32), v);
          if (masked) {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (key0 + c * 32 + e > lim) v[e] = -INFINITY;  // exp2(-inf) = 0
          }
          uint32_t h[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const unsigned long long y = f2_fma(f2_pack(v[e], v[e + 1]), sc2, neg2);
            const float p0 = ex2_approx(f2_lo(y)), p1 = ex2_approx(f2_hi(y));
            acc = f2_add(acc, f2_pack(p0, p1));
            h[e >> 1] = pack2<kF16>(p0, p1);
          }
          // row r, keys [64 half + 32 c, + 32): atom `half`, 16-byte chunks 4 c .. 4 c + 3
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int chunk = c * 4 + q;
            const uint32_t dst = prow + (uint32_t)((chunk ^ (r & 7)) << 4);
            asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(h[4 * q]),
                         "r"(h[4 * q + 1]), "r"(h[4 * q + 2]), "r"(h[4 * q + 3])
                         : "memory");
          }
        }
        l += f2_lo(acc) + f2_hi(acc);
        fence_proxy_async_shared();  // P (generic stores) before the MMA reads it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar_s_empty(sb));
          mbar_arrive(bar_p_full(sb));
        }
      }
      // epilogue: O / l and the row LSE (a failure above arrives here with
      // ok cleared, so both groups take this barrier and stop together)
      const int gl = g0 + t.n_kt - 1;
      bool got = ok && wait(bar_pv_done(gl & 1), (gl >> 1) & 1, 1324);
      got = __all_sync(0xffffffffu, got);
      if (got) {
        tmem_st1(x_col + 4u + (uint32_t)half, l);
        tc_fence_before();
      }
      if (!named_barrier_and(1, 256, got)) { ok = false; break; }
      tc_fence_after();
      const float lo = tmem_ld1(x_col + 4u + (uint32_t)(half ^ 1));
      const float ltot = half == 0 ? l + lo : lo + l;  // group 0's sum first
      const float inv_l = 1.0f / ltot;
      uint16_t* orow = static_cast<uint16_t*>(p.out) + (((long long)t.b * p.Lq + i) * p.Hq + t.qh) * kD + half * 64;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        float o[32];
        tmem_ld32(lane_base + 2 * kTile + (uint32_t)(half * 64 + c * 32), o);
        if (i < p.Lq) {
          uint32_t h[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) h[e >> 1] = pack2<kF16>(o[e] * inv_l, o[e + 1] * inv_l);
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) dst[q] = make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
        }
      }
      if (half == 0 && i < p.Lq)
        p.lse[((long long)t.b * p.Hq + t.qh) * p.Lq + i] = (m_used + log2f(ltot)) * 0.69314718055994531f;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_o_empty);
      // the row sums are read before any group rewrites them: the next unit's
      // write follows its first tile barrier
      g0 += t.n_kt;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace attn
}  // namespace core

using namespace core;

extern "C" int core_attention_prefill(const core_dims_t* d, const void* q, const int64_t* q_strides,
                                      const void* k, const int64_t* k_strides, const void* v,
                                      const int64_t* v_strides, void* out, float* lse,
                                      float softmax_scale, void* stream) {
  if (d == nullptr || q == nullptr || k == nullptr || v == nullptr || out == nullptr ||
      lse == nullptr || q_strides == nullptr || k_strides == nullptr || v_strides == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_attention_prefill: NULL argument");
  if (d->batch <= 0 || d->n_q_heads <= 0 || d->n_kv_heads <= 0 || d->n_queries <= 0 ||
      d->seq_len <= 0)
    return set_error(CORE_ERR_INVALID_ARG, "core_attention_prefill: non-positive dimension");
  if (d->head_dim != attn::kD)
    return set_error(CORE_ERR_UNSUPPORTED, "core_attention_prefill: head_dim must be 128");
  if (d->n_q_heads % d->n_kv_heads != 0)
    return set_error(CORE_ERR_INVALID_ARG, "core_attention_prefill: n_q_heads must be a multiple of n_kv_heads");
  if (d->dtype != CORE_DTYPE_BF16 && d->dtype != CORE_DTYPE_F16)
    return set_error(CORE_ERR_UNSUPPORTED, "core_attention_prefill: dtype must be bf16 or f16");
  if (d->n_queries > d->seq_len)
    return set_error(CORE_ERR_UNSUPPORTED,
                     "core_attention_prefill: more queries than keys (rows without a visible key)");
  if (!(softmax_scale > 0.f) || !std::isfinite(softmax_scale))
    return set_error(CORE_ERR_INVALID_ARG, "core_attention_prefill: softmax_scale must be positive");
  if (!aligned16(out) || (reinterpret_cast<uintptr_t>(lse) & 3u) != 0)
    return set_error(CORE_ERR_INVALID_ARG, "core_attention_prefill: out must be 16-byte aligned");
  const bool f16 = d->dtype == CORE_DTYPE_F16;
  const int B = d->batch, Hq = d->n_q_heads, Hkv = d->n_kv_heads, Lq = d->n_queries, Lk = d->seq_len;
  int rc;
  CUtensorMap tq, tk, tv;
  auto make = [&](CUtensorMap* m, const void* base, const int64_t* s, int H, int L) -> int {
    for (int i = 0; i < 3; ++i)
      if (s[i] <= 0) return set_error(CORE_ERR_INVALID_ARG, "core_attention_prefill: strides must be positive");
    uint64_t dims[4] = {(uint64_t)attn::kD, (uint64_t)L, (uint64_t)H, (uint64_t)B};
    uint64_t str[3] = {(uint64_t)s[2] * 2, (uint64_t)s[1] * 2, (uint64_t)s[0] * 2};
    uint32_t box[4] = {64, (uint32_t)attn::kTile, 1, 1};
    return make_tmap_16bit(m, base, 4, dims, str, box, true, f16);
  };
  if ((rc = make(&tq, q, q_strides, Hq, Lq)) != CORE_OK) return rc;
  if ((rc = make(&tk, k, k_strides, Hkv, Lk)) != CORE_OK) return rc;
  if ((rc = make(&tv, v, v_strides, Hkv, Lk)) != CORE_OK) return rc;

  attn::Params p{};
  p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.G = Hq / Hkv; p.Lq = Lq; p.Lk = Lk; p.off = Lk - Lq;
  p.n_qt = (Lq + attn::kTile - 1) / attn::kTile;
  p.U = (long long)B * Hq * p.n_qt;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.out = out;
  p.lse = lse;
  p.status = device_status();
  const uint32_t smem = attn::Smem::kTotal + 1024;
  cudaError_t e;
  auto kern = f16 ? attn::attn_fwd_kernel<true> : attn::attn_fwd_kernel<false>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return cuda_error(e, "attn_fwd_kernel attribute");
  const int sms = sm_count();
  const int grid = (int)(p.U < sms ? p.U : sms);
  kern<<<grid, attn::kThreads, smem, static_cast<cudaStream_t>(stream)>>>(tq, tk, tv, p);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "attn_fwd_kernel launch");
  return CORE_OK;
}
