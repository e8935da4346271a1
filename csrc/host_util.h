// Host-side helpers shared by the kernel translation units (no torch headers,
// so every .cu file compiles quickly and exposes a plain C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdio>
#include <mutex>
#include <string>

namespace lk {

// Last error message of a launcher on this thread (read by the bindings).
inline std::string& last_error() {
  static thread_local std::string msg;
  return msg;
}

inline int fail(const char* what) {
  last_error() = what;
  return -1;
}

#define LK_REQUIRE(cond, msg) \
  do {                        \
    if (!(cond)) return ::lk::fail(msg); \
  } while (0)

// Number of kernels this library has enqueued (all devices, all threads).
inline std::atomic<unsigned long long>& launch_counter() {
  static std::atomic<unsigned long long> n{0};
  return n;
}

inline int check_launch(const char* name) {
  launch_counter().fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    last_error() = std::string(name) + ": " + cudaGetErrorString(e);
    return -1;
  }
  return 0;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D tiled TMA map over a row-major matrix [rows, cols] (cols contiguous),
// row pitch `ld` elements, box [box_rows, box_cols].  Returns false on error.
inline bool make_tmap_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dtype,
                         int elem_bytes, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                         int box_cols, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) {
    last_error() = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0 || (ld * elem_bytes) % 16 != 0 ||
      (box_cols * elem_bytes) % 16 != 0) {
    last_error() = "TMA operand is not 16-byte aligned";
    return false;
  }
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * elem_bytes)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[96];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d)", (int)r);
    last_error() = buf;
    return false;
  }
  return true;
}

// 3-D tiled TMA map over [d2][d1][d0] (d0 contiguous) with byte strides s1
// (between d1 entries) and s2 (between d2 entries), box [b2][b1][b0], no
// swizzle.  Out-of-range boxes read zeros.  Returns false on error.
inline bool make_tmap_3d(CUtensorMap* m, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                         int64_t d0, int64_t d1, int64_t d2, int64_t s1, int64_t s2, int b0, int b1, int b2) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) {
    last_error() = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0 || s1 % 16 != 0 || s2 % 16 != 0 || (b0 * elem_bytes) % 16 != 0) {
    last_error() = "TMA operand is not 16-byte aligned";
    return false;
  }
  cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
  cuuint64_t strides[2] = {(cuuint64_t)s1, (cuuint64_t)s2};
  cuuint32_t box[3] = {(cuuint32_t)b0, (cuuint32_t)b1, (cuuint32_t)b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, dtype, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[96];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
    last_error() = buf;
    return false;
  }
  return true;
}

inline int num_sms() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (n[dev] == 0) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev];
}

inline int cdiv(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

}  // namespace lk
