// Top-B selection with sink protection (replaces core/kvpress_adapter.py:773-778
// and :1017-1025).
//
// Semantics of the reference: the first n_sink tokens are saturated to
// max(scores) + 1 (so they are always kept), the pooled scores are sorted
// with a stable descending argsort, the first n_kept indices are kept and
// re-sorted ascending.  Equivalently: keep the sinks, then the
// (n_kept - n_sink) best non-sink tokens ordered by (score desc, index asc).
//
// One CTA per batch row: an MSB-first 8-bit radix select over order-preserving
// uint32 keys of the scores finds the threshold key and how many of the tied
// tokens at the threshold to keep (lowest indices first); histograms are
// warp-aggregated (__match_any_sync) and the digit is picked by one warp's
// suffix scan.  Then every thread takes a contiguous run of tokens, one
// block-wide scan of packed (ties, definite keeps) counts gives each run its
// output offsets, and the kept and evicted indices are written in ascending
// order.
#include <cmath>

#include "common.cuh"
#include "host_util.h"

namespace core {
namespace topb {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ uint32_t order_key(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7FFFFFFFu) == 0) u = 0;  // -0 == +0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Block-wide exclusive scan of one 64-bit value per thread.
__device__ __forceinline__ unsigned long long block_exclusive_scan64(unsigned long long v,
                                                                     unsigned long long* s_warp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    unsigned long long w = (lane < kWarps) ? s_warp[lane] : 0ull;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    s_warp[lane] = w;  // inclusive warp prefix
  }
  __syncthreads();
  return (warp > 0 ? s_warp[warp - 1] : 0ull) + x - v;
}

__global__ void __launch_bounds__(kThreads)
    topb_kernel(const float* __restrict__ scores, int L, int n_kept, int n_sink,
                int* __restrict__ keep_idx, int* __restrict__ evict_idx, DeviceStatus* status) {
  const int b = blockIdx.x;
  const float* s = scores + (long long)b * L;
  const int sinks = (n_sink > 0 && n_sink < L) ? n_sink : 0;
  const int need = n_kept - sinks;  // non-sink tokens to keep (>= 0)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __shared__ int hist[256];
  __shared__ unsigned long long s_warp[32];
  __shared__ uint32_t s_prefix, s_mask;
  __shared__ int s_need, s_bad;

  if (threadIdx.x == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_need = need;
    s_bad = 0;
  }
  __syncthreads();
  // ---- radix select: find key T such that #(key > T) < need <= #(key >= T) ----
  bool bad = false;
  for (int shift = 24; shift >= 0 && need > 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += kThreads) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
#pragma unroll 4
    for (int i0 = sinks; i0 < L; i0 += kThreads) {
      const int i = i0 + threadIdx.x;
      int bin = -1;
      if (i < L) {
        const float x = s[i];
        bad |= isnan(x);
        const uint32_t k = order_key(x);
        if ((k & mask) == prefix) bin = (int)((k >> shift) & 255u);
      }
      const unsigned grp = __match_any_sync(0xffffffffu, bin);
      if (bin >= 0 && lane == __ffs(grp) - 1) atomicAdd(&hist[bin], __popc(grp));
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns bins [8 l, 8 l + 8); inclusive suffix sums over lanes
      int own = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) own += hist[8 * lane + j];
      int suf = own;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_down_sync(0xffffffffu, suf, o);
        if (lane + o < 32) suf += y;
      }
      const int rem0 = s_need;
      const int above = suf - own;
      if (above < rem0 && rem0 <= suf) {
        int rem = rem0 - above;
        int d = 8 * lane + 7;
        for (; d > 8 * lane; --d) {
          if (hist[d] >= rem) break;
          rem -= hist[d];
        }
        s_prefix = prefix | ((uint32_t)d << shift);
        s_mask = mask | (255u << shift);
        s_need = rem;
      }
    }
    __syncthreads();
  }
  if (bad) s_bad = 1;
  __syncthreads();
  if (s_bad && threadIdx.x == 0) record_error(status, CORE_ERR_NONFINITE, 701, b);
  const uint32_t T = s_prefix;
  const int ties_keep = s_need;  // tokens equal to T to keep, lowest index first
  // ---- ascending compaction over contiguous runs ----
  const int per = (L + kThreads - 1) / kThreads;
  const int r0 = min(L, threadIdx.x * per), r1 = min(L, r0 + per);
  int n_def = 0, n_tie = 0;
  for (int i = r0; i < r1; ++i) {
    if (i < sinks) {
      ++n_def;
    } else if (need > 0) {
      const uint32_t k = order_key(s[i]);
      n_def += (k > T);
      n_tie += (k == T);
    }
  }
  const unsigned long long pre =
      block_exclusive_scan64(((unsigned long long)n_tie << 32) | (unsigned)n_def, s_warp);
  int tie_before = (int)(pre >> 32);
  int kept_before = (int)(pre & 0xFFFFFFFFull) + min(tie_before, ties_keep);
  int* kout = keep_idx + (long long)b * n_kept;
  int* eout = evict_idx + (long long)b * (L - n_kept);
  for (int i = r0; i < r1; ++i) {
    bool keep;
    if (i < sinks) {
      keep = true;
    } else if (need > 0) {
      const uint32_t k = order_key(s[i]);
      keep = k > T;
      if (k == T) keep = tie_before++ < ties_keep;
    } else {
      keep = false;
    }
    if (keep) {
      if (kept_before < n_kept) kout[kept_before] = i;
      ++kept_before;
    } else {
      const int epos = i - kept_before;  // evicted tokens before i
      if (epos < L - n_kept) eout[epos] = i;
    }
  }
  if (threadIdx.x == kThreads - 1 && kept_before != n_kept)
    record_error(status, CORE_ERR_INVALID_ARG, 702, b);
}

}  // namespace topb
}  // namespace core

using namespace core;

extern "C" size_t core_topb_workspace_bytes(int32_t batch, int32_t seq_len) {
  (void)batch;
  (void)seq_len;
  return 0;
}

extern "C" int core_topb_select(const float* scores, int32_t batch, int32_t seq_len, int32_t n_kept,
                                int32_t n_sink, int32_t* keep_idx, int32_t* evict_idx,
                                void* workspace, size_t workspace_bytes, void* stream) {
  (void)workspace;
  (void)workspace_bytes;
  if (scores == nullptr || keep_idx == nullptr || (evict_idx == nullptr && n_kept < seq_len))
    return set_error(CORE_ERR_INVALID_ARG, "core_topb_select: NULL tensor");
  if (batch <= 0 || seq_len <= 0 || n_kept <= 0 || n_kept > seq_len)
    return set_error(CORE_ERR_INVALID_ARG, "core_topb_select: bad sizes");
  const int sinks = (n_sink > 0 && n_sink < seq_len) ? n_sink : 0;
  if (n_kept < sinks)
    return set_error(CORE_ERR_INVALID_ARG, "core_topb_select: n_kept smaller than the sink count");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  topb::topb_kernel<<<batch, topb::kThreads, 0, s>>>(scores, seq_len, n_kept, n_sink, keep_idx,
                                                    evict_idx, device_status());
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CORE_OK : cuda_error(e, "topb_kernel launch");
}
