// Host-side helpers shared by the entry points: error reporting, argument
// checks, TMA tensor-map encoding and workspace carving.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "core_b200.h"

namespace core {

struct DeviceStatus;

// Records `msg` as the calling thread's last error and returns `code`.
int set_error(int code, const std::string& msg);
int cuda_error(cudaError_t e, const char* what);

// The device status word (one per device), zeroed at first use.
DeviceStatus* device_status();

// Number of SMs of the current device.
int sm_count();

// Encodes a bf16 tiled tensor map of a row-major tensor with 2..5 dims.
// dims / box are innermost-first; strides (bytes) are for dims 1..rank-1.
// swizzle128: 128-byte swizzle (inner box must then be 64 bf16).
int make_tmap_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128);
// The same for bf16 (f16 = false) or f16 elements.
int make_tmap_16bit(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128,
                    bool f16);

// Bump allocator over a caller-provided workspace (256-byte aligned pieces).
struct Carver {
  uint8_t* base;
  size_t size;
  size_t used = 0;
  bool overflow = false;
  Carver(void* b, size_t s) : base(static_cast<uint8_t*>(b)), size(s) {}
  template <class T>
  T* take(size_t count) {
    size_t off = (used + 255) & ~size_t(255);
    size_t bytes = count * sizeof(T);
    if (base == nullptr || off + bytes > size) {
      overflow = true;
      used = off + bytes;
      return nullptr;
    }
    used = off + bytes;
    return reinterpret_cast<T*>(base + off);
  }
};

// Size-only twin of Carver, for the *_workspace_bytes queries.
struct Sizer {
  size_t used = 0;
  template <class T>
  void take(size_t count) {
    used = ((used + 255) & ~size_t(255)) + count * sizeof(T);
  }
};

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Validates the shared dimensions; f32 caches pass only where allow_f32.
int check_dims(const core_dims_t* d, const char* fn, bool allow_f32 = false);

}  // namespace core
