// Host-side helpers shared by the entry points: thread-local error text, argument checks,
// TMA tensor-map encoding through the driver entry point, and the device error word.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <climits>
#include <cstdio>
#include <string>

#include "xdna_b200.h"

namespace xdna {

// Sets the thread's last-error text and returns `code`.
int fail(int code, const char* fmt, ...);

#define XDNA_CHECK_ARG(cond, ...)                          \
  do {                                                     \
    if (!(cond)) return ::xdna::fail(XDNA_ERR_INVALID, __VA_ARGS__); \
  } while (0)

#define XDNA_CUDA(call)                                                                              \
  do {                                                                                               \
    cudaError_t e_ = (call);                                                                         \
    if (e_ != cudaSuccess) return ::xdna::fail(XDNA_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

// Checks that the current device is an sm_100 GPU; caches the answer per device.
int check_device(int* sm_count);

// Device address of this library's error word (int[4]) on the current device.
int* device_error_word();

// Kernel launch error check (after <<<>>>).
int check_launch(const char* what);

// Encodes a tiled TMA map (128-byte swizzle unless given) with zero fill for out-of-range loads.
// dims/strides innermost first; strides_bytes has rank-1 entries (dims 1..rank-1).
int encode_tma(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
               const uint64_t* strides_bytes, const uint32_t* box, const char* what,
               CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

inline int dtype_size(int dt) {
  switch (dt) {
    case XDNA_F32:
    case XDNA_I32:
      return 4;
    case XDNA_BF16:
    case XDNA_F16:
      return 2;
    case XDNA_I8:
    case XDNA_U8:
      return 1;
    default:
      return 0;
  }
}

inline bool is_float_dtype(int dt) { return dt == XDNA_F32 || dt == XDNA_BF16 || dt == XDNA_F16; }

}  // namespace xdna
