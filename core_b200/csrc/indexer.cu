// Auxiliary features and the indexer MLP (replaces core/features.py:861-921,
// the feature concatenation at core/kvpress_adapter.py:536 and
// COREIndexerMLP, core/indexer.py:88-108).
//
// Persistent CTAs of 512 threads over tiles of 128 cached tokens; thread
// (token t = tid % 128, quarter q = tid / 128).
//   0. once per CTA: the three bf16 terms of W2 arrive as one prepared image
//      (core_prepare_indexer_mlp: already split and in the SW128 K-major
//      layout of a tcgen05 B operand) by bulk copies;
//   1. auxiliary features: a_value from V with the reference's bf16 roundings
//      (squares, per-head sums, the head mean, /d and log1p each round to
//      bf16; heads split over the quarters and summed in head order),
//      a_age, a_sink, a_phase;
//   2. layer 1 (14 -> 128, f32 FMAs, exact erf GELU): each quarter computes 32
//      hidden units and stores them as three bf16 terms (hi + mid + lo = the
//      f32 value) in the SW128 K-major layout of a tcgen05 A operand;
//   3. layer 2 (128 -> 128) on tcgen05: A = hidden terms, B = the W2 terms, the
//      six products whose term orders sum to at most 2 accumulated in f32 in
//      TMEM — f32-level accuracy;
//   4. epilogue: TMEM -> registers, + b2, GELU, dot with w3 (32 outputs per
//      quarter), the quarters' parts added, + b3.
#include <cmath>

#include "common.cuh"
#include "host_util.h"

namespace core {
namespace idx {

constexpr int kIn = 14;
constexpr int kHid = 128;
constexpr int kTile = 128;     // tokens per tile (MMA M)
constexpr int kThreads = 512;  // 128 tokens x 4 quarters
constexpr int kMaxHkv = 16;
// packed global layout (floats): [w1 (128,14) | b1 | w2^T (in 128, out 128) | b2 | w3 | b3]
constexpr int kGW1 = 0;
constexpr int kGB1 = kGW1 + kHid * kIn;
constexpr int kGW2T = kGB1 + kHid;
constexpr int kGB2 = kGW2T + kHid * kHid;
constexpr int kGW3 = kGB2 + kHid;
constexpr int kGB3 = kGW3 + kHid;
constexpr int kGFloats = kGB3 + 1;
// after the f32 block, at a 1024-byte boundary: the W2 image (three bf16 terms
// of the (out, in) K-major SW128 operand), written by core_prepare_indexer_mlp
constexpr uint32_t kGImageOff = ((uint32_t)kGFloats * 4u + 1023u) & ~1023u;
// word kGFloats holds this tag once the image is written: a packed buffer
// without it is refused by the kernel instead of read past its end
constexpr uint32_t kImageTag = 0x32574958u;
// shared memory, from a 1024-byte aligned base
constexpr uint32_t kTermBytes = kTile * kHid * 2;  // one bf16 term: two K atoms of 16 KB
constexpr uint32_t kOffW = 0;                      // W2 terms (out, in), B operand
constexpr uint32_t kOffH = 3 * kTermBytes;         // hidden terms (token, hidden), A operand
constexpr uint32_t kOffF = 6 * kTermBytes;         // f32 block below
constexpr int kW1Stride = 16;
constexpr int kFW1 = 0;                            // [128][16]
constexpr int kFB1 = kFW1 + kHid * kW1Stride;
constexpr int kFB2 = kFB1 + kHid;
constexpr int kFW3 = kFB2 + kHid;
constexpr int kFB3 = kFW3 + kHid;                  // 4 floats
constexpr int kFHs = kFB3 + 4;                     // per-head value energies [128][kMaxHkv]
constexpr int kFPart = kFHs + kTile * kMaxHkv;     // quarters 1-3 partial scores [3][128]
constexpr int kFFloats = kFPart + 3 * kTile;
constexpr uint32_t kOffBar = kOffF + 4u * kFFloats;
constexpr uint32_t kSmemBytes = kOffBar + 64 + 1024;  // + barriers, TMEM slot, alignment slack
constexpr uint32_t kImageBytes = 3 * kTermBytes;
constexpr size_t kPackedBytes = (size_t)kGImageOff + kImageBytes;
static_assert(kSmemBytes <= 227u * 1024u, "shared memory budget");

__device__ __forceinline__ float gelu(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

// Byte offset of 16-byte chunk `chunk` (k / 8 inside the atom) of row `row`
// of a 128-row K-major SW128 operand tile made of two 64-element K atoms.
__device__ __forceinline__ uint32_t sw128_chunk(int row, int atom, int chunk) {
  return (uint32_t)atom * 16384u + (uint32_t)row * 128u + (uint32_t)((chunk ^ (row & 7)) << 4);
}

// Split 8 f32 values into three bf16 terms (x = t0 + t1 + t2 to f32 precision)
// packed as three uint4 of 8 bf16 each.
__device__ __forceinline__ void split3(const float (&x)[8], uint4& t0, uint4& t1, uint4& t2) {
  uint32_t w0[4], w1[4], w2[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float a = x[2 * i], b = x[2 * i + 1];
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    w0[i] = *reinterpret_cast<uint32_t*>(&h);
    a -= __uint_as_float(w0[i] << 16);
    b -= __uint_as_float(w0[i] & 0xFFFF0000u);
    h = __floats2bfloat162_rn(a, b);
    w1[i] = *reinterpret_cast<uint32_t*>(&h);
    a -= __uint_as_float(w1[i] << 16);
    b -= __uint_as_float(w1[i] & 0xFFFF0000u);
    h = __floats2bfloat162_rn(a, b);
    w2[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  t0 = make_uint4(w0[0], w0[1], w0[2], w0[3]);
  t1 = make_uint4(w1[0], w1[1], w1[2], w1[3]);
  t2 = make_uint4(w2[0], w2[1], w2[2], w2[3]);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, const uint4& v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

struct Params {
  int B, Hkv, L, original_length, is_prefill, n_sink;
  const __nv_bfloat16* v;   // bf16 values, or
  const float* vf;          // f32 values (then v is NULL and no bf16 roundings apply)
  const float* head_sums;   // or per-head value sums (h, token) from value_head_sums_kernel
  long long hs_stride;      // (head-sharded caches: the heads live on other ranks)
  const int64_t* positions;
  const uint8_t* special;
  float* features;
  const float* mlp;
  float* scores;
  DeviceStatus* status;
};

// The W2 image of core_prepare_indexer_mlp: unit (o, c) = output row o, input
// columns [8 c, 8 c + 8), split into three bf16 terms at the SW128 offset of
// row o, K atom c / 8, chunk c % 8 in each 32 KB term.
__global__ void indexer_w2_image_kernel(const float* __restrict__ packed, uint8_t* __restrict__ image) {
  const int u = blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= kHid * (kHid / 8)) return;
  const int o = u & (kHid - 1), c = u >> 7;
  float x[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = packed[kGW2T + (8 * c + i) * kHid + o];
  uint4 t0, t1, t2;
  split3(x, t0, t1, t2);
  const uint32_t off = sw128_chunk(o, c >> 3, c & 7);
  *reinterpret_cast<uint4*>(image + off) = t0;
  *reinterpret_cast<uint4*>(image + kTermBytes + off) = t1;
  *reinterpret_cast<uint4*>(image + 2 * kTermBytes + off) = t2;
  if (u == 0) reinterpret_cast<uint32_t*>(const_cast<float*>(packed))[kGFloats] = kImageTag;
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    indexer_scores_kernel(const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  float* sf = reinterpret_cast<float*>(sgen + kOffF);
  const uint32_t bar = sbase + kOffBar;        // layer-2 MMA done (one phase per tile)
  const uint32_t bar_w2 = sbase + kOffBar + 8; // W2 image in shared memory
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + kOffBar + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sgen + kOffBar + 24);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int t = tid & (kTile - 1);  // token row of the tile == TMEM lane
  const int quarter = tid >> 7;

  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_init(bar_w2, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 128);
    tmem_relinquish();
  }
  __syncthreads();
  if (tid == 0) {  // the prepared W2 terms: three 32 KB bulk copies
    if (reinterpret_cast<const uint32_t*>(p.mlp)[kGFloats] == kImageTag) {
      mbar_arrive_expect_tx(bar_w2, kImageBytes);
      const uint8_t* img = reinterpret_cast<const uint8_t*>(p.mlp) + kGImageOff;
      for (int tm = 0; tm < 3; ++tm)
        bulk_g2s(sbase + kOffW + tm * kTermBytes, img + tm * kTermBytes, kTermBytes, bar_w2);
    } else {
      *abort_flag = 1;
      if (blockIdx.x == 0) record_error(p.status, CORE_ERR_INVALID_ARG, 612, 0);
    }
  }
  for (int i = tid; i < kHid * kIn; i += kThreads)
    sf[kFW1 + (i / kIn) * kW1Stride + (i % kIn)] = p.mlp[kGW1 + i];
  for (int i = tid; i < kHid; i += kThreads) {
    sf[kFB1 + i] = p.mlp[kGB1 + i];
    sf[kFB2 + i] = p.mlp[kGB2 + i];
    sf[kFW3 + i] = p.mlp[kGW3 + i];
  }
  if (tid == 0) sf[kFB3] = p.mlp[kGB3];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool have_image = *abort_flag == 0;

  const long long n = (long long)p.B * p.L;
  const long long n_tiles = (n + kTile - 1) / kTile;
  const float age_den = log1pf((float)(p.original_length - 1 > 1 ? p.original_length - 1 : 1));
  int iter = 0;
  for (long long tile = blockIdx.x; have_image && tile < n_tiles; tile += gridDim.x, ++iter) {
    const long long gi = tile * kTile + t;
    const bool active = gi < n;
    const int b = active ? (int)(gi / p.L) : 0;
    const int i = active ? (int)(gi % p.L) : 0;
    // ---- 1. auxiliary features (features.py:886-921) ----
    if (active && p.head_sums != nullptr) {
      for (int h = quarter; h < p.Hkv; h += 4)
        sf[kFHs + t * kMaxHkv + h] = p.head_sums[(long long)h * p.hs_stride + gi];
    } else if (active && p.vf != nullptr) {
      for (int h = quarter; h < p.Hkv; h += 4) {
        const float4* row =
            reinterpret_cast<const float4*>(p.vf + (((long long)b * p.Hkv + h) * p.L + i) * 128);
        float s = 0.f;
#pragma unroll
        for (int c0 = 0; c0 < 32; c0 += 16) {
          float4 w[16];  // half the 512-byte row in flight at once
#pragma unroll
          for (int c = 0; c < 16; ++c) w[c] = __ldg(row + c0 + c);
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            s = fmaf(w[c].x, w[c].x, s);
            s = fmaf(w[c].y, w[c].y, s);
            s = fmaf(w[c].z, w[c].z, s);
            s = fmaf(w[c].w, w[c].w, s);
          }
        }
        sf[kFHs + t * kMaxHkv + h] = s;
      }
    } else if (active) {
      for (int h = quarter; h < p.Hkv; h += 4) {
        const uint4* row =
            reinterpret_cast<const uint4*>(p.v + (((long long)b * p.Hkv + h) * p.L + i) * 128);
        uint4 w[16];  // the whole 256-byte row in flight at once
#pragma unroll
        for (int c = 0; c < 16; ++c) w[c] = __ldg(row + c);
        float s = 0.f;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&w[c]);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f2 = __bfloat1622float2(h2[e]);
            s += bf16_round(f2.x * f2.x);
            s += bf16_round(f2.y * f2.y);
          }
        }
        sf[kFHs + t * kMaxHkv + h] = bf16_round(s);
      }
    }
    __syncthreads();
    float x[kIn];
    if (active) {
      float hsum = 0.f;
      for (int h = 0; h < p.Hkv; ++h) hsum += sf[kFHs + t * kMaxHkv + h];
      const long long pos = p.positions[gi];
      const int T = p.original_length;
      if (quarter == 0 && (pos < 0 || pos >= T)) record_error(p.status, CORE_ERR_INVALID_ARG, 601, i);
      const float a_age = log1pf((float)(T - 1 - pos)) / age_den;
      bool sink = pos < p.n_sink;
      if (p.special != nullptr && p.special[gi]) sink = true;
      float a_value;
      if (p.vf != nullptr) {  // f32 arithmetic (features.py:914-915 on f32 values)
        a_value = log1pf((hsum / (float)p.Hkv) / 128.0f);
      } else {                // every step rounded to bf16 like the bf16 tensor ops
        const float vmean = bf16_round(hsum / (float)p.Hkv);
        a_value = bf16_round(log1pf(bf16_round(vmean / 128.0f)));
      }
      float* f = p.features + gi * kIn;
#pragma unroll
      for (int k = 0; k < 10; ++k) x[k] = f[k];
      x[10] = a_age;
      x[11] = sink ? 1.0f : 0.0f;
      x[12] = a_value;
      x[13] = p.is_prefill ? 0.0f : 1.0f;
      if (quarter == 0) {
#pragma unroll
        for (int k = 10; k < kIn; ++k) f[k] = x[k];
        bool finite = true;
#pragma unroll
        for (int k = 0; k < kIn; ++k) finite &= isfinite(x[k]);
        if (!finite) record_error(p.status, CORE_ERR_NONFINITE, 602, i);
      }
    } else {
#pragma unroll
      for (int k = 0; k < kIn; ++k) x[k] = 0.f;
    }
    // ---- 2. layer 1: hidden units [32 q, 32 q + 32) as three bf16 terms ----
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float hv[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int k = 32 * quarter + 8 * c + e;
        const float4* w1 = reinterpret_cast<const float4*>(sf + kFW1 + k * kW1Stride);
        const float4 a0 = w1[0], a1 = w1[1], a2 = w1[2], a3 = w1[3];
        float acc = 0.f;
        acc = fmaf(a0.x, x[0], acc);
        acc = fmaf(a0.y, x[1], acc);
        acc = fmaf(a0.z, x[2], acc);
        acc = fmaf(a0.w, x[3], acc);
        acc = fmaf(a1.x, x[4], acc);
        acc = fmaf(a1.y, x[5], acc);
        acc = fmaf(a1.z, x[6], acc);
        acc = fmaf(a1.w, x[7], acc);
        acc = fmaf(a2.x, x[8], acc);
        acc = fmaf(a2.y, x[9], acc);
        acc = fmaf(a2.z, x[10], acc);
        acc = fmaf(a2.w, x[11], acc);
        acc = fmaf(a3.x, x[12], acc);
        acc = fmaf(a3.y, x[13], acc);
        hv[e] = gelu(acc + sf[kFB1 + k]);
      }
      uint4 t0, t1, t2;
      split3(hv, t0, t1, t2);
      // hidden 32 q + 8 c: K atom q / 2, chunk 4 (q % 2) + c
      const uint32_t off = sw128_chunk(t, quarter >> 1, 4 * (quarter & 1) + c);
      st_shared_v4(sbase + kOffH + off, t0);
      st_shared_v4(sbase + kOffH + kTermBytes + off, t1);
      st_shared_v4(sbase + kOffH + 2 * kTermBytes + off, t2);
    }
    fence_proxy_async_shared();
    tc_fence_before();
    __syncthreads();
    // ---- 3. layer 2 on tcgen05: sum of hidden-term x weight-term products of order <= 2 ----
    bool ok = true;
    if (tid == 0) {
      if (iter == 0) ok = bounded_wait(bar_w2, 0, abort_flag, p.status, 611);
      tc_fence_after();
      constexpr uint32_t idesc = idesc_bf16(kTile, kHid, 0, 0);
      constexpr int kTa[6] = {2, 1, 0, 1, 0, 0};  // small products first
      constexpr int kTb[6] = {0, 1, 2, 0, 1, 0};
      if (ok) {
#pragma unroll
        for (int pi = 0; pi < 6; ++pi) {
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint32_t koff = (uint32_t)(ks >> 2) * 16384u + (uint32_t)(ks & 3) * 32u;
            const uint64_t a = sdesc_kmajor(sbase + kOffH + (uint32_t)kTa[pi] * kTermBytes + koff);
            const uint64_t bd = sdesc_kmajor(sbase + kOffW + (uint32_t)kTb[pi] * kTermBytes + koff);
            mma_bf16(tmem, a, bd, idesc, (pi > 0 || ks > 0) ? 1u : 0u);
          }
        }
        mma_commit(bar);
      }
    }
    ok = __syncthreads_and(ok);
    if (ok) ok = bounded_wait(bar, (uint32_t)(iter & 1), abort_flag, p.status, 610);
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc_fence_after();
    // ---- 4. epilogue: outputs [32 q, 32 q + 32) of token t ----
    float part = 0.f;
    {
      float v[32];
      tmem_ld32(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(32 * quarter), v);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int o = 32 * quarter + j;
        part = fmaf(sf[kFW3 + o], gelu(v[j] + sf[kFB2 + o]), part);
      }
    }
    if (quarter > 0) sf[kFPart + (quarter - 1) * kTile + t] = part;
    tc_fence_before();
    __syncthreads();
    if (quarter == 0 && active)
      p.scores[gi] = ((part + sf[kFPart + t]) + (sf[kFPart + kTile + t] + sf[kFPart + 2 * kTile + t])) +
                     sf[kFB3];
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// Per-(head, token) value sums of squares in the arithmetic of the indexer's
// auxiliary block (squares rounded to bf16 and added in index order, the sum
// rounded to bf16): out[h * out_stride + b * L + token].  One thread per row,
// like the indexer, so the sums agree bit for bit.  Each warp first copies
// its 32 rows (8 KB) into shared memory with coalesced 16-byte cp.async
// pieces, all in flight at once; rows are padded to 17 pieces so that the
// lanes' row reads afterwards hit distinct banks.
constexpr int kVhsWarps = 4;
constexpr int kVhsRowsPerBlock = kVhsWarps * 32;
constexpr int kVhsPad = 17;  // uint4 pieces per staged row (16 + 1)

__global__ void __launch_bounds__(kVhsWarps * 32)
    value_head_sums_kernel(const __nv_bfloat16* __restrict__ v, int B, int Hkv, int L,
                           float* __restrict__ out, long long out_stride) {
  __shared__ __align__(16) uint4 s_rows[kVhsWarps][32 * kVhsPad];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long rows = (long long)B * Hkv * L;
  const long long row0 = (long long)blockIdx.x * kVhsRowsPerBlock + warp * 32;
  if (row0 >= rows) return;  // whole warp
  const int nrows = rows - row0 < 32 ? (int)(rows - row0) : 32;
  const uint4* src = reinterpret_cast<const uint4*>(v) + row0 * 16;
  uint4* stage = s_rows[warp];
  const uint32_t sbase = smem_u32(stage);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int q = lane + 32 * i;  // piece q of the warp's rows: row q / 16, piece q % 16
    if ((q >> 4) < nrows) cp_async16(sbase + (uint32_t)(((q >> 4) * kVhsPad + (q & 15)) * 16), src + q);
  }
  cp_async_commit();
  cp_async_wait_all();
  __syncwarp();
  if (lane >= nrows) return;
  const uint4* rowp = stage + lane * kVhsPad;
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    const uint4 w = rowp[c];
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f2 = __bfloat1622float2(h2[e]);
      s += bf16_round(f2.x * f2.x);
      s += bf16_round(f2.y * f2.y);
    }
  }
  const long long row = row0 + lane;
  const long long bh = row / L;
  const int b = (int)(bh / Hkv), h = (int)(bh % Hkv), t = (int)(row % L);
  out[(long long)h * out_stride + (long long)b * L + t] = bf16_round(s);
}

}  // namespace idx
}  // namespace core

using namespace core;
using namespace core::idx;

extern "C" size_t core_indexer_mlp_bytes(void) { return kPackedBytes; }

extern "C" int core_prepare_indexer_mlp(float* mlp, void* stream) {
  if (mlp == nullptr) return set_error(CORE_ERR_INVALID_ARG, "core_prepare_indexer_mlp: NULL buffer");
  if (reinterpret_cast<uintptr_t>(mlp) % 16 != 0)
    return set_error(CORE_ERR_INVALID_ARG, "core_prepare_indexer_mlp: buffer must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  constexpr int units = kHid * (kHid / 8);
  indexer_w2_image_kernel<<<units / 128, 128, 0, s>>>(mlp, reinterpret_cast<uint8_t*>(mlp) + kGImageOff);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CORE_OK : cuda_error(e, "indexer_w2_image_kernel launch");
}

extern "C" int core_indexer_scores(const core_dims_t* d, const void* v, const int64_t* positions,
                                   const uint8_t* special, int32_t original_length,
                                   int32_t is_prefill, int32_t n_sink, float* features,
                                   const float* mlp, float* scores, void* stream) {
  int rc = check_dims(d, "core_indexer_scores", true);
  if (rc != CORE_OK) return rc;
  if (v == nullptr || positions == nullptr || features == nullptr || mlp == nullptr ||
      scores == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_indexer_scores: NULL tensor");
  if (reinterpret_cast<uintptr_t>(mlp) % 16 != 0)
    return set_error(CORE_ERR_INVALID_ARG, "core_indexer_scores: mlp must be 16-byte aligned");
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
  const bool f32 = d->dtype == CORE_DTYPE_F32;
  p.v = f32 ? nullptr : static_cast<const __nv_bfloat16*>(v);
  p.vf = f32 ? static_cast<const float*>(v) : nullptr;
  p.positions = positions;
  p.special = special;
  p.features = features;
  p.mlp = mlp;
  p.scores = scores;
  p.status = device_status();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t smem = kSmemBytes;
  cudaError_t e =
      cudaFuncSetAttribute(indexer_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_error(e, "indexer_scores_kernel attribute");
  const long long n_tiles = ((long long)p.B * p.L + kTile - 1) / kTile;
  const long long blocks = n_tiles < sm_count() ? n_tiles : sm_count();
  indexer_scores_kernel<<<(unsigned)blocks, kThreads, smem, s>>>(p);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "indexer_scores_kernel launch");
  return CORE_OK;
}

// ---------------------------------------------------------------------------
// Head-sharded caches (one sequence).
// ---------------------------------------------------------------------------
extern "C" int core_value_head_sums(const core_dims_t* d, const void* v, float* out,
                                    int64_t out_stride, void* stream) {
  int rc = check_dims(d, "core_value_head_sums");
  if (rc != CORE_OK) return rc;
  if (v == nullptr || out == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_value_head_sums: NULL tensor");
  if (d->batch != 1) return set_error(CORE_ERR_UNSUPPORTED, "core_value_head_sums: one sequence");
  if (out_stride < d->seq_len)
    return set_error(CORE_ERR_INVALID_ARG, "core_value_head_sums: out_stride < seq_len");
  const long long rows = (long long)d->n_kv_heads * d->seq_len;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  value_head_sums_kernel<<<(unsigned)((rows + kVhsRowsPerBlock - 1) / kVhsRowsPerBlock),
                           kVhsRowsPerBlock, 0, s>>>(
      static_cast<const __nv_bfloat16*>(v), 1, d->n_kv_heads, d->seq_len, out, out_stride);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CORE_OK : cuda_error(e, "value_head_sums_kernel launch");
}

extern "C" int core_indexer_scores_from_sums(int32_t n_kv_heads, int32_t n_keys,
                                             const float* head_sums, int64_t hs_stride,
                                             const int64_t* positions, const uint8_t* special,
                                             int32_t original_length, int32_t is_prefill,
                                             int32_t n_sink, float* features, const float* mlp,
                                             float* scores, void* stream) {
  if (head_sums == nullptr || positions == nullptr || features == nullptr || mlp == nullptr ||
      scores == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_indexer_scores_from_sums: NULL tensor");
  if (reinterpret_cast<uintptr_t>(mlp) % 16 != 0)
    return set_error(CORE_ERR_INVALID_ARG, "core_indexer_scores_from_sums: mlp must be 16-byte aligned");
  if (n_kv_heads <= 0 || n_kv_heads > kMaxHkv)
    return set_error(CORE_ERR_UNSUPPORTED, "core_indexer_scores_from_sums: 1 to 16 KV heads");
  if (n_keys < 0 || hs_stride < n_keys || original_length < n_keys)
    return set_error(CORE_ERR_INVALID_ARG, "core_indexer_scores_from_sums: bad sizes");
  if (n_keys == 0) return CORE_OK;
  Params p{};
  p.B = 1;
  p.Hkv = n_kv_heads;
  p.L = n_keys;
  p.original_length = original_length;
  p.is_prefill = is_prefill;
  p.n_sink = n_sink;
  p.head_sums = head_sums;
  p.hs_stride = hs_stride;
  p.positions = positions;
  p.special = special;
  p.features = features;
  p.mlp = mlp;
  p.scores = scores;
  p.status = device_status();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e =
      cudaFuncSetAttribute(indexer_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return cuda_error(e, "indexer_scores_kernel attribute");
  const long long n_tiles = ((long long)n_keys + kTile - 1) / kTile;
  const long long blocks = n_tiles < sm_count() ? n_tiles : sm_count();
  indexer_scores_kernel<<<(unsigned)blocks, kThreads, kSmemBytes, s>>>(p);
  e = cudaGetLastError();
  return e == cudaSuccess ? CORE_OK : cuda_error(e, "indexer_scores_kernel launch");
}

namespace core {
// core_indexer_scores for bf16 caches in two launches: the per-head value sums
// into the workspace (B * L * Hkv floats), then the indexer reading them.
// Same results, bit for bit, as the one-launch form.
int indexer_scores_split(const core_dims_t* d, const void* v, const int64_t* positions,
                         const uint8_t* special, int32_t original_length, int32_t is_prefill,
                         int32_t n_sink, float* features, const float* mlp, float* scores,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (d == nullptr || d->dtype != CORE_DTYPE_BF16 || workspace == nullptr)
    return core_indexer_scores(d, v, positions, special, original_length, is_prefill, n_sink,
                               features, mlp, scores, stream);
  int rc = check_dims(d, "core_indexer_scores");
  if (rc != CORE_OK) return rc;
  if (v == nullptr || positions == nullptr || features == nullptr || mlp == nullptr ||
      scores == nullptr)
    return set_error(CORE_ERR_INVALID_ARG, "core_indexer_scores: NULL tensor");
  if (reinterpret_cast<uintptr_t>(mlp) % 16 != 0)
    return set_error(CORE_ERR_INVALID_ARG, "core_indexer_scores: mlp must be 16-byte aligned");
  if (original_length < d->seq_len)
    return set_error(CORE_ERR_INVALID_ARG, "core_indexer_scores: original_length < seq_len");
  if (d->n_kv_heads > kMaxHkv)
    return set_error(CORE_ERR_UNSUPPORTED, "core_indexer_scores: at most 16 KV heads");
  const long long BL = (long long)d->batch * d->seq_len;
  Carver cv(workspace, workspace_bytes);
  float* hs = cv.take<float>((size_t)BL * d->n_kv_heads);
  if (cv.overflow) return set_error(CORE_ERR_WORKSPACE, "core_indexer_scores: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long rows = BL * d->n_kv_heads;
  value_head_sums_kernel<<<(unsigned)((rows + kVhsRowsPerBlock - 1) / kVhsRowsPerBlock),
                           kVhsRowsPerBlock, 0, s>>>(
      static_cast<const __nv_bfloat16*>(v), d->batch, d->n_kv_heads, d->seq_len, hs, BL);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "value_head_sums_kernel launch");
  Params p{};
  p.B = d->batch;
  p.Hkv = d->n_kv_heads;
  p.L = d->seq_len;
  p.original_length = original_length;
  p.is_prefill = is_prefill;
  p.n_sink = n_sink;
  p.head_sums = hs;
  p.hs_stride = BL;
  p.positions = positions;
  p.special = special;
  p.features = features;
  p.mlp = mlp;
  p.scores = scores;
  p.status = device_status();
  e = cudaFuncSetAttribute(indexer_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return cuda_error(e, "indexer_scores_kernel attribute");
  const long long n_tiles = (BL + kTile - 1) / kTile;
  const long long blocks = n_tiles < sm_count() ? n_tiles : sm_count();
  indexer_scores_kernel<<<(unsigned)blocks, kThreads, kSmemBytes, s>>>(p);
  e = cudaGetLastError();
  return e == cudaSuccess ? CORE_OK : cuda_error(e, "indexer_scores_kernel launch");
}
}  // namespace core
