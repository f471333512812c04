// Top-B selection with sink protection (replaces core/kvpress_adapter.py:773-778
// and :1017-1025).
//
// Semantics of the reference: the first n_sink tokens are saturated to
// max(scores) + 1 (so they are always kept), the pooled scores are sorted
// with a stable descending argsort, the first n_kept indices are kept and
// re-sorted ascending.  Equivalently: keep the sinks, then the
// (n_kept - n_sink) best non-sink tokens ordered by (score desc, index asc).
//
// One CTA per batch row.  The row's order-preserving uint32 keys are staged
// in shared memory (rows of up to 49152 tokens; longer rows recompute them
// from the scores).  An MSB-first 8-bit radix select finds the threshold
// prefix and how many of the tokens tied on it to keep (lowest indices
// first), stopping early once a whole bin is kept; histograms are
// warp-aggregated (__match_any_sync) and the digit is picked by one warp's
// suffix scan.  Compaction: each warp owns a contiguous chunk, ballots rank
// the tokens inside the warp, one pass of per-warp counts gives the offsets,
// and kept and evicted indices are written in ascending order.
#include <cooperative_groups.h>

#include <cmath>

#include "common.cuh"
#include "host_util.h"

namespace cg = cooperative_groups;

namespace core {
namespace topb {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ uint32_t order_key(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7FFFFFFFu) == 0) u = 0;  // -0 == +0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kMaxSmemKeys = 49152;  // 192 KB of keys in shared memory

// Key of token i (i >= sinks): from shared memory when the row fits, else
// recomputed from the scores.
template <bool kSmem>
__device__ __forceinline__ uint32_t key_at(const uint32_t* sk, const float* s, int i) {
  if constexpr (kSmem) return sk[i];
  else return order_key(s[i]);
}

template <bool kSmem>
__global__ void __launch_bounds__(kThreads)
    topb_kernel(const float* __restrict__ scores, int L, int n_kept, int n_sink,
                int* __restrict__ keep_idx, int* __restrict__ evict_idx, DeviceStatus* status) {
  extern __shared__ uint32_t sk[];  // order keys of the row (kSmem only)
  const int b = blockIdx.x;
  const float* s = scores + (long long)b * L;
  const int sinks = (n_sink > 0 && n_sink < L) ? n_sink : 0;
  const int need = n_kept - sinks;  // non-sink tokens to keep (>= 0)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __shared__ int hist[256];
  __shared__ int s_cnt[kWarps][2];
  __shared__ uint32_t s_prefix, s_mask;
  __shared__ int s_need, s_bad, s_done;

  if (threadIdx.x == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_need = need;
    s_bad = 0;
    s_done = need <= 0;
  }
  bool bad = false;
  if constexpr (kSmem) {
#pragma unroll 4
    for (int i = threadIdx.x; i < L; i += kThreads) {
      const float x = s[i];
      bad |= (i >= sinks) && isnan(x);
      sk[i] = order_key(x);
    }
  }
  __syncthreads();
  // ---- radix select over 8-bit digits, MSB first.  Invariant: the tokens with
  // (key & mask) > prefix are all kept and number need - s_need; s_need of the
  // tokens with (key & mask) == prefix are kept, lowest index first. ----
  for (int shift = 24; shift >= 0; shift -= 8) {
    if (s_done) break;  // uniform: read after a barrier
    for (int i = threadIdx.x; i < 256; i += kThreads) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
#pragma unroll 4
    for (int i0 = sinks; i0 < L; i0 += kThreads) {
      const int i = i0 + threadIdx.x;
      int bin = -1;
      if (i < L) {
        uint32_t k;
        if constexpr (kSmem) {
          k = sk[i];
        } else {
          const float x = s[i];
          bad |= isnan(x);
          k = order_key(x);
        }
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
        if (rem == hist[d]) s_done = 1;  // the whole bin is kept: no tie to break
      }
    }
    __syncthreads();
  }
  if (bad) s_bad = 1;
  __syncthreads();
  if (s_bad && threadIdx.x == 0) record_error(status, CORE_ERR_NONFINITE, 701, b);
  const uint32_t T = s_prefix, TM = s_mask;
  const int ties_keep = s_need;
  // ---- ascending compaction: warp w owns a contiguous chunk; ballots give
  // in-warp ranks, one pass of counts gives the warps' offsets ----
  auto classify = [&](int i, bool& def, bool& tie) {
    def = false;
    tie = false;
    if (i < sinks) {
      def = true;
    } else if (need > 0) {
      const uint32_t km = key_at<kSmem>(sk, s, i) & TM;
      def = km > T;
      tie = km == T;
    }
  };
  const int chunk = ((L + kThreads - 1) / kThreads) * 32;
  const int c0 = min(L, warp * chunk), c1 = min(L, c0 + chunk);
  int ndef = 0, ntie = 0;
  for (int i0 = c0; i0 < c1; i0 += 32) {
    const int i = i0 + lane;
    bool def = false, tie = false;
    if (i < c1) classify(i, def, tie);
    ndef += __popc(__ballot_sync(0xffffffffu, def));
    ntie += __popc(__ballot_sync(0xffffffffu, tie));
  }
  if (lane == 0) {
    s_cnt[warp][0] = ndef;
    s_cnt[warp][1] = ntie;
  }
  __syncthreads();
  const int def_before = __reduce_add_sync(0xffffffffu, lane < warp ? s_cnt[lane][0] : 0);
  int tb = __reduce_add_sync(0xffffffffu, lane < warp ? s_cnt[lane][1] : 0);
  int kept = def_before + min(tb, ties_keep);
  const unsigned lt = (1u << lane) - 1u;
  int* kout = keep_idx + (long long)b * n_kept;
  int* eout = evict_idx + (long long)b * (L - n_kept);
  for (int i0 = c0; i0 < c1; i0 += 32) {
    const int i = i0 + lane;
    bool def = false, tie = false;
    if (i < c1) classify(i, def, tie);
    const unsigned tmask = __ballot_sync(0xffffffffu, tie);
    const bool keep = def || (tie && tb + __popc(tmask & lt) < ties_keep);
    const unsigned kmask = __ballot_sync(0xffffffffu, keep);
    const int kpos = kept + __popc(kmask & lt);
    if (i < c1) {
      if (keep) {
        if (kpos < n_kept) kout[kpos] = i;
      } else {
        const int epos = i - kpos;  // evicted tokens before i
        if (epos < L - n_kept) eout[epos] = i;
      }
    }
    kept += __popc(kmask);
    tb += __popc(tmask);
  }
  if (warp == kWarps - 1 && lane == 0 && kept != n_kept)
    record_error(status, CORE_ERR_INVALID_ARG, 702, b);
}


// ---------------------------------------------------------------------------
// Long rows: one cluster of kCluster CTAs per batch row.  CTA c holds the keys
// of tokens [c Lc, (c + 1) Lc) in its shared memory; every radix pass adds the
// CTAs' histograms in CTA order through distributed shared memory, so all CTAs
// take the same digit decision as the one-CTA kernel above (double-buffered
// histograms: one cluster barrier per pass).  Compaction offsets come from the
// lower CTAs' counts.  Results are those of topb_kernel.
// ---------------------------------------------------------------------------
constexpr int kCluster = 8;
constexpr int kMaxClusterKeys = kCluster * kMaxSmemKeys;
constexpr int kClusterMinKeys = 8192;  // shorter rows: one CTA

__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads)
    topb_cluster_kernel(const float* __restrict__ scores, int L, int n_kept, int n_sink,
                        int* __restrict__ keep_idx, int* __restrict__ evict_idx,
                        DeviceStatus* status) {
  extern __shared__ uint32_t sk[];  // order keys of this CTA's tokens
  cg::cluster_group cluster = cg::this_cluster();
  const int cr = (int)cluster.block_rank();
  const int b = blockIdx.x / kCluster;
  const float* s = scores + (long long)b * L;
  const int sinks = (n_sink > 0 && n_sink < L) ? n_sink : 0;
  const int need = n_kept - sinks;
  const int Lc = (L + kCluster - 1) / kCluster;
  const int lo = min(L, cr * Lc), hi = min(L, lo + Lc);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __shared__ int hist[2][256];
  __shared__ int ghist[256];
  __shared__ int s_cnt[kWarps][2];
  __shared__ int s_tot[2];  // this CTA's (definite, tie) counts, read by the higher CTAs
  __shared__ uint32_t s_prefix, s_mask;
  __shared__ int s_need, s_done;

  if (threadIdx.x == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_need = need;
    s_done = need <= 0;
  }
  bool bad = false;
#pragma unroll 4
  for (int i = lo + threadIdx.x; i < hi; i += kThreads) {
    const float x = s[i];
    bad |= (i >= sinks) && isnan(x);
    sk[i - lo] = order_key(x);
  }
  __syncthreads();
  int pass = 0;
  for (int shift = 24; shift >= 0; shift -= 8, ++pass) {
    if (s_done) break;  // uniform across the cluster: every CTA took the same decisions
    int* h = hist[pass & 1];
    for (int i = threadIdx.x; i < 256; i += kThreads) h[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    const int first = max(lo, sinks);
#pragma unroll 4
    for (int i0 = first; i0 < hi; i0 += kThreads) {
      const int i = i0 + threadIdx.x;
      int bin = -1;
      if (i < hi) {
        const uint32_t k = sk[i - lo];
        if ((k & mask) == prefix) bin = (int)((k >> shift) & 255u);
      }
      const unsigned grp = __match_any_sync(0xffffffffu, bin);
      if (bin >= 0 && lane == __ffs(grp) - 1) atomicAdd(&h[bin], __popc(grp));
    }
    cluster.sync();  // every CTA's histogram of this pass is complete
    for (int i = threadIdx.x; i < 256; i += kThreads) {
      int t = 0;
      for (int c = 0; c < kCluster; ++c) t += cluster.map_shared_rank(h, c)[i];
      ghist[i] = t;
    }
    __syncthreads();
    if (warp == 0) {
      int own = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) own += ghist[8 * lane + j];
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
          if (ghist[d] >= rem) break;
          rem -= ghist[d];
        }
        s_prefix = prefix | ((uint32_t)d << shift);
        s_mask = mask | (255u << shift);
        s_need = rem;
        if (rem == ghist[d]) s_done = 1;
      }
    }
    __syncthreads();
  }
  if (__syncthreads_or(bad) && threadIdx.x == 0) record_error(status, CORE_ERR_NONFINITE, 701, b);
  const uint32_t T = s_prefix, TM = s_mask;
  const int ties_keep = s_need;
  auto classify = [&](int i, bool& def, bool& tie) {
    def = false;
    tie = false;
    if (i < sinks) {
      def = true;
    } else if (need > 0) {
      const uint32_t km = sk[i - lo] & TM;
      def = km > T;
      tie = km == T;
    }
  };
  const int n_here = hi - lo;
  const int chunk = ((n_here + kThreads - 1) / kThreads) * 32;
  const int c0 = min(hi, lo + warp * chunk), c1 = min(hi, c0 + chunk);
  int ndef = 0, ntie = 0;
  for (int i0 = c0; i0 < c1; i0 += 32) {
    const int i = i0 + lane;
    bool def = false, tie = false;
    if (i < c1) classify(i, def, tie);
    ndef += __popc(__ballot_sync(0xffffffffu, def));
    ntie += __popc(__ballot_sync(0xffffffffu, tie));
  }
  if (lane == 0) {
    s_cnt[warp][0] = ndef;
    s_cnt[warp][1] = ntie;
  }
  __syncthreads();
  if (warp == 0) {
    const int d = __reduce_add_sync(0xffffffffu, s_cnt[lane][0]);
    const int t = __reduce_add_sync(0xffffffffu, s_cnt[lane][1]);
    if (lane == 0) {
      s_tot[0] = d;
      s_tot[1] = t;
    }
  }
  cluster.sync();  // every CTA's totals are published
  int def_cta = 0, tie_cta = 0;
  for (int c = 0; c < cr; ++c) {
    const int* r = cluster.map_shared_rank(s_tot, c);
    def_cta += r[0];
    tie_cta += r[1];
  }
  const int def_before = def_cta + __reduce_add_sync(0xffffffffu, lane < warp ? s_cnt[lane][0] : 0);
  int tb = tie_cta + __reduce_add_sync(0xffffffffu, lane < warp ? s_cnt[lane][1] : 0);
  int kept = def_before + min(tb, ties_keep);
  const unsigned lt = (1u << lane) - 1u;
  int* kout = keep_idx + (long long)b * n_kept;
  int* eout = evict_idx + (long long)b * (L - n_kept);
  for (int i0 = c0; i0 < c1; i0 += 32) {
    const int i = i0 + lane;
    bool def = false, tie = false;
    if (i < c1) classify(i, def, tie);
    const unsigned tmask = __ballot_sync(0xffffffffu, tie);
    const bool keep = def || (tie && tb + __popc(tmask & lt) < ties_keep);
    const unsigned kmask = __ballot_sync(0xffffffffu, keep);
    const int kpos = kept + __popc(kmask & lt);
    if (i < c1) {
      if (keep) {
        if (kpos < n_kept) kout[kpos] = i;
      } else {
        const int epos = i - kpos;
        if (epos < L - n_kept) eout[epos] = i;
      }
    }
    kept += __popc(kmask);
    tb += __popc(tmask);
  }
  if (cr == kCluster - 1 && warp == kWarps - 1 && lane == 0 && kept != n_kept)
    record_error(status, CORE_ERR_INVALID_ARG, 702, b);
  cluster.sync();  // no CTA leaves while another may still read its shared memory
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
  cudaError_t e;
  if (seq_len >= topb::kClusterMinKeys && seq_len <= topb::kMaxClusterKeys) {
    const int Lc = (seq_len + topb::kCluster - 1) / topb::kCluster;
    const size_t smem = sizeof(uint32_t) * (size_t)Lc;
    e = cudaFuncSetAttribute(topb::topb_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(sizeof(uint32_t) * topb::kMaxSmemKeys));
    if (e != cudaSuccess) return cuda_error(e, "topb_cluster_kernel attribute");
    topb::topb_cluster_kernel<<<batch * topb::kCluster, topb::kThreads, smem, s>>>(
        scores, seq_len, n_kept, n_sink, keep_idx, evict_idx, device_status());
  } else if (seq_len <= topb::kMaxSmemKeys) {
    const size_t smem = sizeof(uint32_t) * (size_t)seq_len;
    e = cudaFuncSetAttribute(topb::topb_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(sizeof(uint32_t) * topb::kMaxSmemKeys));
    if (e != cudaSuccess) return cuda_error(e, "topb_kernel attribute");
    topb::topb_kernel<true><<<batch, topb::kThreads, smem, s>>>(scores, seq_len, n_kept, n_sink,
                                                              keep_idx, evict_idx, device_status());
  } else {
    topb::topb_kernel<false><<<batch, topb::kThreads, 0, s>>>(scores, seq_len, n_kept, n_sink,
                                                            keep_idx, evict_idx, device_status());
  }
  e = cudaGetLastError();
  return e == cudaSuccess ? CORE_OK : cuda_error(e, "topb_kernel launch");
}
