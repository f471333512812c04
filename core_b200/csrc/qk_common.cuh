// Definitions shared by the bf16 tensor-core and the f32 CUDA-core QK kernels:
// the relation floor, the per-key record layout and the logaddexp with the
// floor (core/fused_qk.py:200-202, :382, :494).
#pragma once

#include "common.cuh"

namespace core {
namespace qk {

// log(1e-8) as the float the reference passes to its kernels (fused_qk.py:382, :494).
constexpr float kLogFloor = -18.420680743952367f;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// One 64-byte record per (key, KV head, 128-query block), 16 words:
//   [0..3]  top-4 R over the block's queries (descending)
//   [4..7]  top-4 R over the block's recent queries
//   [8]     sum of the positive R          [9]  count of the positive R
//   [10..13] positive-R bits, query 32 w + b of the block in word w, bit b
//   [14]    max of the non-positive R      [15] sum of the non-positive R
constexpr int kRecWords = 16;
// Per-key summary of one rank's KV heads (head-sharded caches), sum_words =
// kSumHead + 4 n_qb words: 0-3 top-4 relation values (descending), 4-7 top-4
// of the recent queries, 8 positive sum (f32), 9 positive count, 10 positive-
// head count for f6 (f32), 11 unused, then 4 words of positive-query bits (OR
// over the heads) per 128-query block.
constexpr int kSumHead = 12;

// -LSE + log|C_t| of one (q-head, query): with it r = fmaf(s x, offset).
__device__ __forceinline__ float relation_offset(float lse, long long count) {
  return -lse + logf((float)count);
}

// logaddexp(r, f) without the correction term where it is below 1.2e-7
// (|r - f| >= 16): that term moves the result by at most two f32 ulps.  The
// bf16 relation kernels use this; the f32 kernels keep the exact form below.
__device__ __forceinline__ float logaddexp_floor_fast(float r) {
  const float a = fabsf(r - kLogFloor);
  return a < 16.0f ? fmaxf(r, kLogFloor) + log1pf(expf(-a)) : fmaxf(r, kLogFloor);
}

__device__ __forceinline__ float logaddexp_floor(float r) {
  // max(r, f) + log1p(exp(-|r - f|)), f = log(1e-8)  (fused_qk.py:200-202)
  float a = fabsf(r - kLogFloor);
  float t;
  if (a < 16.0f) {
    t = log1pf(expf(-a));
  } else {
    // exp(-a) < 1.2e-7: log1p(x) equals x to within half an ulp of x.
    t = ex2_approx(-a * kLog2e);
  }
  return fmaxf(r, kLogFloor) + t;
}

}  // namespace qk
}  // namespace core
