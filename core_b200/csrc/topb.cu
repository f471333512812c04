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
// tokens at the threshold to keep (lowest indices first), then a block-wide
// prefix scan writes the kept and evicted indices in ascending order.
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

// Block-wide exclusive scan of one int per thread; returns the exclusive
// prefix and writes the block total to *total.
__device__ __forceinline__ int block_exclusive_scan(int v, int* s_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = (lane < kWarps) ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    s_warp[lane] = w;  // inclusive warp prefix
  }
  __syncthreads();
  const int before = (warp > 0 ? s_warp[warp - 1] : 0) + x - v;
  *total = s_warp[kWarps - 1];
  __syncthreads();
  return before;
}

__global__ void __launch_bounds__(kThreads)
    topb_kernel(const float* __restrict__ scores, int L, int n_kept, int n_sink,
                int* __restrict__ keep_idx, int* __restrict__ evict_idx, DeviceStatus* status) {
  const int b = blockIdx.x;
  const float* s = scores + (long long)b * L;
  const int sinks = (n_sink > 0 && n_sink < L) ? n_sink : 0;
  const int need = n_kept - sinks;  // non-sink tokens to keep (>= 0)
  __shared__ int hist[256];
  __shared__ int s_warp[32];
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
  for (int shift = 24; shift >= 0 && need > 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += kThreads) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    for (int i = sinks + threadIdx.x; i < L; i += kThreads) {
      const float x = s[i];
      if (isnan(x)) s_bad = 1;
      const uint32_t k = order_key(x);
      if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int rem = s_need;
      int d = 255;
      for (; d > 0; --d) {
        if (hist[d] >= rem) break;
        rem -= hist[d];
      }
      s_prefix = prefix | ((uint32_t)d << shift);
      s_mask = mask | (255u << shift);
      s_need = rem;
    }
    __syncthreads();
  }
  if (s_bad && threadIdx.x == 0) record_error(status, CORE_ERR_NONFINITE, 701, b);
  const uint32_t T = s_prefix;
  const int ties_keep = s_need;  // tokens equal to T to keep, lowest index first
  // ---- ascending compaction ----
  int kept_base = 0, ev_base = 0, tie_base = 0;
  int* kout = keep_idx + (long long)b * n_kept;
  int* eout = evict_idx + (long long)b * (L - n_kept);
  for (int c0 = 0; c0 < L; c0 += kThreads) {
    const int i = c0 + threadIdx.x;
    int is_tie = 0, keep = 0;
    if (i < L) {
      if (i < sinks) {
        keep = 1;
      } else if (need > 0) {
        const uint32_t k = order_key(s[i]);
        if (k > T) keep = 1;
        else if (k == T) is_tie = 1;
      }
    }
    int tie_total;
    const int tie_rank = tie_base + block_exclusive_scan(is_tie, s_warp, &tie_total);
    if (is_tie && tie_rank < ties_keep) keep = 1;
    int keep_total;
    const int kpos = kept_base + block_exclusive_scan(keep, s_warp, &keep_total);
    if (i < L) {
      if (keep) {
        if (kpos < n_kept) kout[kpos] = i;
      } else {
        const int epos = i - kpos;  // evicted tokens before i
        if (epos < L - n_kept) eout[epos] = i;
      }
    }
    kept_base += keep_total;
    tie_base += tie_total;
    ev_base += (min(kThreads, L - c0) - keep_total);
  }
  if (threadIdx.x == 0 && kept_base != n_kept) record_error(status, CORE_ERR_INVALID_ARG, 702, b);
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
