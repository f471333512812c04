// Host helpers and the small entry points (version, errors, device status,
// weight splitting).
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "host_util.h"

#include <atomic>

namespace core {

static thread_local std::string g_last_error;

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_error(cudaError_t e, const char* what) {
  return set_error(CORE_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// The device status word lives in device global memory of every GPU that
// loads the library (a module-scope variable, so no allocation is needed).
__device__ DeviceStatus g_device_status;

static constexpr int kMaxDevices = 64;
static DeviceStatus* g_status[kMaxDevices] = {nullptr};
static std::mutex g_status_mu;

DeviceStatus* device_status() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_status_mu);
  if (g_status[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
    g_status[dev] = static_cast<DeviceStatus*>(p);
  }
  return g_status[dev];
}

// Process-wide cap on the SMs a launch plans for (0: all of them).
static std::atomic<int> g_sm_budget{0};

int sm_count() {
  static int cache[kMaxDevices] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) dev = 0;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 1;
  }
  const int budget = g_sm_budget.load(std::memory_order_relaxed);
  return (budget > 0 && budget < cache[dev]) ? budget : cache[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

int make_tmap_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128) {
  return make_tmap_16bit(map, base, rank, dims, strides_bytes, box, swizzle128, false);
}

int make_tmap_16bit(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128,
                    bool f16) {
  auto enc = get_encode();
  if (enc == nullptr) return set_error(CORE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (!aligned16(base)) return set_error(CORE_ERR_INVALID_ARG, "TMA base pointer not 16-byte aligned");
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
    if (i > 0) {
      if (strides_bytes[i - 1] % 16 != 0)
        return set_error(CORE_ERR_INVALID_ARG, "TMA stride not a multiple of 16 bytes");
      gstride[i - 1] = strides_bytes[i - 1];
    }
  }
  CUresult r = enc(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                   (cuuint32_t)rank, const_cast<void*>(base),
                   gdim, gstride, bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[128];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return set_error(CORE_ERR_CUDA, buf);
  }
  return CORE_OK;
}

int check_dims(const core_dims_t* d, const char* fn, bool allow_f32) {
  std::string f(fn);
  if (d == nullptr) return set_error(CORE_ERR_INVALID_ARG, f + ": dims is NULL");
  if (d->batch <= 0 || d->n_q_heads <= 0 || d->n_kv_heads <= 0 || d->seq_len <= 0 ||
      d->n_queries < 0)
    return set_error(CORE_ERR_INVALID_ARG, f + ": non-positive dimension");
  if (d->head_dim != 128) return set_error(CORE_ERR_UNSUPPORTED, f + ": head_dim must be 128");
  if (d->n_q_heads % d->n_kv_heads != 0)
    return set_error(CORE_ERR_INVALID_ARG, f + ": n_q_heads must be a multiple of n_kv_heads");
  int g = d->n_q_heads / d->n_kv_heads;
  if (g != 1 && g != 2 && g != 4)
    return set_error(CORE_ERR_UNSUPPORTED, f + ": GQA group size must be 1, 2 or 4");
  if (d->dtype != CORE_DTYPE_BF16 && !(allow_f32 && d->dtype == CORE_DTYPE_F32))
    return set_error(CORE_ERR_UNSUPPORTED,
                     f + (allow_f32 ? ": dtype must be bf16 or f32" : ": this entry point takes bf16 caches only"));
  if (d->n_queries > d->seq_len)
    return set_error(CORE_ERR_INVALID_ARG, f + ": n_queries exceeds seq_len");
  return CORE_OK;
}

// --------------------------------------------------------------------------
// bf16 term splitting of f32 weights
// --------------------------------------------------------------------------
__global__ void split_bf16_kernel(const float* __restrict__ src, int64_t n, int terms,
                                  __nv_bfloat16* __restrict__ dst) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float x = src[i];
  for (int t = 0; t < terms; ++t) {
    __nv_bfloat16 h = __float2bfloat16_rn(x);
    dst[(int64_t)t * n + i] = h;
    x = x - __bfloat162float(h);
  }
}

}  // namespace core

using namespace core;

extern "C" int core_version(void) { return 100; }

extern "C" int core_last_error(char* buf, size_t buf_len) {
  if (buf == nullptr || buf_len == 0) return CORE_ERR_INVALID_ARG;
  size_t n = g_last_error.size() < buf_len - 1 ? g_last_error.size() : buf_len - 1;
  memcpy(buf, g_last_error.data(), n);
  buf[n] = 0;
  return CORE_OK;
}

extern "C" int core_check_device_status(void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceStatus* st = device_status();
  if (st == nullptr) return set_error(CORE_ERR_CUDA, "device status allocation failed");
  DeviceStatus h;
  cudaError_t e = cudaMemcpyAsync(&h, st, sizeof(h), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_error(e, "core_check_device_status");
  if (h.code != 0) {
    cudaMemsetAsync(st, 0, sizeof(DeviceStatus), s);
    cudaStreamSynchronize(s);
    char buf[160];
    snprintf(buf, sizeof(buf), "device status %d (where=%d detail=%d count=%d)", h.code, h.where,
             h.detail, h.count);
    return set_error(h.code, buf);
  }
  return CORE_OK;
}

extern "C" int core_split_bf16(const float* src, int64_t n, int32_t terms, void* dst,
                               void* stream) {
  if (src == nullptr || dst == nullptr || n <= 0 || terms < 1 || terms > 3)
    return set_error(CORE_ERR_INVALID_ARG, "core_split_bf16: bad arguments");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int threads = 256;
  int64_t blocks = (n + threads - 1) / threads;
  split_bf16_kernel<<<(unsigned)blocks, threads, 0, s>>>(src, n, terms,
                                                         static_cast<__nv_bfloat16*>(dst));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CORE_OK : cuda_error(e, "core_split_bf16 launch");
}

extern "C" int core_set_sm_budget(int32_t n_sms) {
  if (n_sms < 0) return set_error(CORE_ERR_INVALID_ARG, "core_set_sm_budget: negative SM count");
  g_sm_budget.store(n_sms, std::memory_order_relaxed);
  return CORE_OK;
}

// ---------------------------------------------------------------------------
// Self-test of the bounded wait: one warp waits on an mbarrier that nothing
// arrives at, with the given limit, through the same bounded_wait the kernels
// use; the wait gives up, records CORE_ERR_TIMEOUT (site 990) in the device
// status and the kernel returns normally, leaving the context usable.
// ---------------------------------------------------------------------------
namespace {
__global__ void selftest_wait_kernel(uint64_t limit_ns, core::DeviceStatus* st) {
  __shared__ __align__(8) uint64_t bar_storage;
  __shared__ int abort_flag;
  const uint32_t bar = core::smem_u32(&bar_storage);
  if (threadIdx.x == 0) {
    core::mbar_init(bar, 1);
    abort_flag = 0;
    core::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) core::bounded_wait(bar, 0, &abort_flag, st, 990, limit_ns);
  __syncthreads();
}
}  // namespace

extern "C" int core_selftest_wait_timeout(int32_t limit_us, void* stream) {
  if (limit_us <= 0 || limit_us > 1000000)
    return set_error(CORE_ERR_INVALID_ARG, "core_selftest_wait_timeout: limit must be 1 us to 1 s");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  selftest_wait_kernel<<<1, 32, 0, s>>>((uint64_t)limit_us * 1000ull, core::device_status());
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CORE_OK : cuda_error(e, "selftest_wait_kernel launch");
}
