// Shared device helpers for the CORE B200 kernels (sm_100a only).
//
// Everything here is thin inline PTX around the Blackwell primitives the
// kernels use: mbarriers with bounded waits, TMA tensor loads (never with
// cluster multicast), tcgen05 MMA / TMEM allocation / TMEM loads, and the
// shared-memory and instruction descriptors those take.  Descriptor bit
// layouts follow the PTX ISA "tcgen05 matrix descriptors" section.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "core_b200.h"

#if !defined(__CUDA_ARCH__) || (__CUDA_ARCH__ >= 1000)
#define CORE_SM100 1
#endif

namespace core {

// ---------------------------------------------------------------------------
// Device-side error word.  Kernels never trap: a bounded wait that gives up,
// or a detected bad value, records a code here and the kernel returns.  The
// host reads it back after the launch sequence (core_check_device_error).
// ---------------------------------------------------------------------------
struct DeviceStatus {
  int code;      // first error code recorded (0 = none)
  int where;     // kernel-specific location tag
  int detail;    // kernel-specific detail (e.g. unit index)
  int count;     // number of errors recorded
};

__device__ __forceinline__ void record_error(DeviceStatus* st, int code, int where, int detail) {
  if (st == nullptr) return;
  if (atomicCAS(&st->code, 0, code) == 0) {
    st->where = where;
    st->detail = detail;
  }
  atomicAdd(&st->count, 1);
}

// Upper bound, in nanoseconds of %globaltimer, for every wait on an mbarrier.
// Every legitimate wait in these kernels lasts micro- to milliseconds; the
// bound is reached only when a producer never arrives, and the kernel then
// records CORE_ERR_TIMEOUT, raises the CTA's abort flag and winds down.
constexpr uint64_t kWaitLimitNs = 4000000000ull;

// ---------------------------------------------------------------------------
// Basic PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Time-bounded wait on an mbarrier phase.  Returns false when the CTA's abort
// flag is raised by another thread or when kWaitLimitNs passes (then records
// CORE_ERR_TIMEOUT and raises the flag); callers then stop issuing work.
__device__ __forceinline__ bool bounded_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                             DeviceStatus* st, int where,
                                             uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        record_error(st, CORE_ERR_TIMEOUT, where, (int)blockIdx.x);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// TMA tiled loads into this CTA's shared memory, completing on an mbarrier.
// No multicast form is used anywhere in this library.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* m, uint32_t bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* m, uint32_t bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* m, uint32_t bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

// Named barrier among a subset of warps (ids 1..15; id 0 is __syncthreads).
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also returns the AND of `pred` over the participating
// threads: lets a group of warps take one uniform decision after a bounded wait.
__device__ __forceinline__ bool named_barrier_and(uint32_t id, uint32_t nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %2, 0;\n\t"
      "bar.red.and.pred q, %1, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(id), "r"((uint32_t)pred), "r"(nthreads)
      : "memory");
  return r != 0;
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 inputs, f32 accumulate).
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// 32 lanes x 32 consecutive columns of 32-bit data: thread t of the warp
// receives row (lane_base + t), columns [col, col + 32).  The load and its
// completion wait are one asm statement so no consumer can be scheduled
// between them.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 16 consecutive columns (load and wait in one asm statement).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 32 consecutive columns stored from registers (store and its
// completion wait in one asm statement).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

// One 32-bit column of 32 lanes: thread t stores / loads lane (lane_base + t).
__device__ __forceinline__ void tmem_st1(uint32_t taddr, float v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr), "r"(__float_as_uint(v))
      : "memory");
}
__device__ __forceinline__ float tmem_ld1(uint32_t taddr) {
  uint32_t r;
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r)
      : "r"(taddr)
      : "memory");
  return __uint_as_float(r);
}

// ---------------------------------------------------------------------------
// Descriptors
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor, 128-byte swizzle.  K-major operands use
// rows of 128 bytes (64 bf16) grouped in 8-row, 1024-byte atoms: SBO = 1024,
// LBO unused (1).  MN-major operands (used for gathered V tiles) use 64-element
// MN atoms 128 bytes wide stacked over 8 K-rows: SBO = 1024 between 8-row K
// groups, LBO = byte distance between consecutive MN atoms.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ uint64_t sdesc_kmajor(uint32_t saddr) {
  return sdesc_sw128(saddr, 16, 1024);
}

// Instruction descriptor for kind::f16 with bf16 A/B and f32 accumulate.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4)                         // D format f32
         | (1u << 7)                       // A format bf16
         | (1u << 10)                      // B format bf16
         | ((uint32_t)a_mn_major << 15)    // A major
         | ((uint32_t)b_mn_major << 16)    // B major
         | ((uint32_t)(N >> 3) << 17)      // N / 8
         | ((uint32_t)(M >> 4) << 24);     // M / 16
}

// ---------------------------------------------------------------------------
// cp.async (16-byte global -> shared copies, L1 bypass)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// 16-byte copy, or 16 zero bytes when !valid (src-size 0: nothing is read).
__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(valid ? 16u : 0u)
               : "memory");
}
// Arrive on an mbarrier once every cp.async this thread issued so far has
// landed; .noinc: the arrival counts against the barrier's expected count, so
// the thread goes on issuing without waiting for its copies.
__device__ __forceinline__ void cp_async_mbar_arrive(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Hint: bring the 128-byte line holding p into L2.
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Copy n16 16-byte chunks global -> shared with all threads of the block
// (both addresses 16-byte aligned); completes with cp_async_wait_all().
__device__ __forceinline__ void cp_async_block(void* dst, const void* src, int n16) {
  const uint32_t d = smem_u32(dst);
  const char* s = static_cast<const char*>(src);
  for (int i = threadIdx.x; i < n16; i += blockDim.x) cp_async16(d + 16u * i, s + 16ll * i);
  cp_async_commit();
}

// ---------------------------------------------------------------------------
// Numerics helpers
// ---------------------------------------------------------------------------
// Round an f32 to bfloat16 precision (nearest-even) and widen back.
__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Round two f32 values to bf16 precision with one packed conversion.
__device__ __forceinline__ void bf16_round2(float& a, float& b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const uint32_t u = *reinterpret_cast<const uint32_t*>(&h);
  a = __uint_as_float(u << 16);
  b = __uint_as_float(u & 0xFFFF0000u);
}

// Packed f32x2 arithmetic (sm_100): two lanes of f32 in one 64-bit register.
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
  return ((unsigned long long)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float f2_lo(unsigned long long v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(unsigned long long v) {
  return __uint_as_float((uint32_t)(v >> 32));
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Three-input f32 maximum (sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Three-input f32 minimum (sm_100).
__device__ __forceinline__ float fmin3(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Insert v into a descending top-4 list (t0 >= t1 >= t2 >= t3).
__device__ __forceinline__ void top4_insert(float (&t)[4], float v) {
  float a = fminf(t[0], v), b = fminf(t[1], v), c = fminf(t[2], v);
  t[3] = fmaxf(t[3], c);
  t[2] = fmaxf(t[2], b);
  t[1] = fmaxf(t[1], a);
  t[0] = fmaxf(t[0], v);
}

// Merge a pair {a, b} into a descending top-4 list: the k-th largest of the
// union is the largest min(t_i, pair_j) with i + j = k (pair sorted).
__device__ __forceinline__ void top4_insert2(float (&t)[4], float a, float b) {
  const float hi = fmaxf(a, b), lo = fminf(a, b);
  t[3] = fmax3(t[3], fminf(t[2], hi), fminf(t[1], lo));
  t[2] = fmax3(t[2], fminf(t[1], hi), fminf(t[0], lo));
  t[1] = fmax3(t[1], fminf(t[0], hi), lo);
  t[0] = fmaxf(t[0], hi);
}

// Top-4 of the union of two descending top-4 lists: max(t_i, o_{3-i}) are the
// four largest (a bitonic sequence), then two compare-exchange stages sort them.
__device__ __forceinline__ void cex_desc(float& a, float& b) {
  const float hi = fmaxf(a, b), lo = fminf(a, b);
  a = hi;
  b = lo;
}
__device__ __forceinline__ void top4_merge(float (&t)[4], const float (&o)[4]) {
  float d0 = fmaxf(t[0], o[3]), d1 = fmaxf(t[1], o[2]), d2 = fmaxf(t[2], o[1]),
        d3 = fmaxf(t[3], o[0]);
  cex_desc(d0, d2);
  cex_desc(d1, d3);
  cex_desc(d0, d1);
  cex_desc(d2, d3);
  t[0] = d0;
  t[1] = d1;
  t[2] = d2;
  t[3] = d3;
}

}  // namespace core
