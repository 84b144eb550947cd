// Host-side helpers shared by every C-ABI entry point: status codes, the
// thread-local last-error string, TMA descriptor encoding and SM-count cache.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include <atomic>
#include <mutex>

#include "../../include/siglip2_b200.h"

namespace sg {

inline thread_local char t_last_error[512] = "";

inline int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

#define SG_CHECK_ARG(cond, ...) \
  do {                           \
    if (!(cond)) return ::sg::set_error(SIGLIP2_ERR_ARG, __VA_ARGS__); \
  } while (0)

#define SG_CUDA(call)                                                                             \
  do {                                                                                            \
    cudaError_t e_ = (call);                                                                      \
    if (e_ != cudaSuccess)                                                                        \
      return ::sg::set_error(SIGLIP2_ERR_CUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                             __FILE__, __LINE__);                                                 \
  } while (0)

#define SG_LAUNCH_CHECK()                                                                          \
  do {                                                                                             \
    ::sg::launch_counter().fetch_add(1, std::memory_order_relaxed);                                \
    cudaError_t e_ = cudaGetLastError();                                                           \
    if (e_ != cudaSuccess)                                                                         \
      return ::sg::set_error(SIGLIP2_ERR_CUDA, "kernel launch failed: %s (%s:%d)", cudaGetErrorString(e_), \
                             __FILE__, __LINE__);                                                  \
  } while (0)

#define SG_TRY(expr)           \
  do {                         \
    int rc_ = (expr);          \
    if (rc_ != SIGLIP2_OK) return rc_; \
  } while (0)

// Kernel launches issued by this library since load (host-side count).
inline std::atomic<unsigned long long>& launch_counter() {
  static std::atomic<unsigned long long> n{0};
  return n;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// TMA descriptors through the driver entry point (no -lcuda link needed)
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

inline CUtensorMapSwizzle swizzle_for_bytes(int inner_box_bytes) {
  switch (inner_box_bytes) {
    case 128: return CU_TENSOR_MAP_SWIZZLE_128B;
    case 64: return CU_TENSOR_MAP_SWIZZLE_64B;
    case 32: return CU_TENSOR_MAP_SWIZZLE_32B;
    default: return CU_TENSOR_MAP_SWIZZLE_NONE;
  }
}

// 2-D row-major tensor [rows, cols] with row pitch `ld` elements; box
// [box_rows, box_cols]; swizzle span = box_cols * elem bytes.
inline int make_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, int64_t rows, int64_t cols, int64_t ld,
                        int box_rows, int box_cols) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return set_error(SIGLIP2_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (!aligned16(base)) return set_error(SIGLIP2_ERR_ALIGN, "TMA base address %p is not 16-byte aligned", base);
  if ((ld * elem_bytes) % 16 != 0)
    return set_error(SIGLIP2_ERR_ALIGN, "row pitch %lld elements is not a multiple of 16 bytes", (long long)ld);
  const CUtensorMapDataType dt = elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;  // 2-byte: bf16 and f16 alike
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * elem_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle_for_bytes(box_cols * elem_bytes), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(SIGLIP2_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) rows=%lld cols=%lld ld=%lld box=%dx%d",
                     (int)r, (long long)rows, (long long)cols, (long long)ld, box_rows, box_cols);
  return SIGLIP2_OK;
}

inline int sm_count() {
  static int n = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  });
  return n;
}

}  // namespace sg
