// Host-side helpers: TMA tensor-map encoding through the driver entry point
// (no link-time dependency on libcuda), device properties, error word.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdint>
#include <cstring>

#include "w4a8.h"

namespace w4a8 {

// Per-device values looked up once (device ids 0..63) and shared by every
// host thread. Slots are atomics: threads that race on a first lookup each
// compute the same value and store it, which is well defined; a zero /
// null slot means "not looked up yet".
template <typename T>
struct PerDevice {
  std::atomic<T> slot[64];
  T get(int dev) const { return (dev >= 0 && dev < 64) ? slot[dev].load(std::memory_order_relaxed) : T{}; }
  void set(int dev, T v) {
    if (dev >= 0 && dev < 64) slot[dev].store(v, std::memory_order_relaxed);
  }
};

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::atomic<PFN_cuTensorMapEncodeTiled_v12000> fn{nullptr};
  PFN_cuTensorMapEncodeTiled_v12000 f = fn.load(std::memory_order_relaxed);
  if (!f) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      f = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
      fn.store(f, std::memory_order_relaxed);
    }
  }
  return f;
}

// Encodes a uint8 tiled map. dims/box innermost first; strides (bytes) for
// dims 1..rank-1. Returns W4A8_OK or W4A8_ERR_TENSORMAP.
inline int encode_u8(CUtensorMap* map, const void* ptr, int rank, const uint64_t* dims, const uint64_t* strides,
                     const uint32_t* box, CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return W4A8_ERR_TENSORMAP;
  uint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? W4A8_OK : W4A8_ERR_TENSORMAP;
}

inline int device_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  static PerDevice<int> cached;
  if (const int c = cached.get(dev)) return c;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cached.set(dev, sms);
  return sms;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Address of the device error word on the current device.
unsigned* device_error_word();

}  // namespace w4a8
