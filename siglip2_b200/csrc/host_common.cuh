// Host-side helpers shared by every C-ABI entry point: status codes, the
// thread-local last-error string, TMA descriptor encoding and SM-count cache.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include <atomic>
#include <map>
#include <mutex>
#include <utility>

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

// 3-D view [d2][d1][d0] (d0 contiguous) with byte strides for d1 and d2.
// Box elements past d0 (or any other extent) are read as zeros.
inline int make_tmap_3d(CUtensorMap* map, const void* base, int elem_bytes, int64_t d0, int64_t d1, int64_t d2,
                        int64_t stride1_bytes, int64_t stride2_bytes, int box0, int box1, int box2) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return set_error(SIGLIP2_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (!aligned16(base)) return set_error(SIGLIP2_ERR_ALIGN, "TMA base address %p is not 16-byte aligned", base);
  if (stride1_bytes % 16 != 0 || stride2_bytes % 16 != 0)
    return set_error(SIGLIP2_ERR_ALIGN, "TMA strides %lld / %lld bytes are not multiples of 16", (long long)stride1_bytes,
                     (long long)stride2_bytes);
  const CUtensorMapDataType dt = elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1), static_cast<cuuint64_t>(d2)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(stride1_bytes), static_cast<cuuint64_t>(stride2_bytes)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box0), static_cast<cuuint32_t>(box1), static_cast<cuuint32_t>(box2)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle_for_bytes(box0 * elem_bytes), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(SIGLIP2_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d) dims=%lldx%lldx%lld box=%dx%dx%d", (int)r,
                     (long long)d0, (long long)d1, (long long)d2, box0, box1, box2);
  return SIGLIP2_OK;
}

// Per-device host caches: one process may drive several GPUs (one host
// thread per device, or cudaSetDevice between calls), so anything learnt from
// or set on a device is kept per device ordinal.
constexpr int kMaxDevices = 64;

// SM count of the current device (queried once per device).
inline int sm_count() {
  static std::atomic<int> cache[kMaxDevices];  // zero-initialised: not yet queried
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  const bool cached = dev >= 0 && dev < kMaxDevices;
  int n = cached ? cache[dev].load(std::memory_order_relaxed) : 0;
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    if (cached) cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// cudaFuncAttributeMaxDynamicSharedMemorySize holds per kernel and per
// device: raise it on the current device when a launch needs more than was
// set there before (never lowers it, so launches of different sizes can
// interleave).
inline int ensure_dynamic_smem(const void* kern, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> set_bytes;  // (kernel, device) -> attribute value
  int dev = 0;
  SG_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  int& cur = set_bytes[std::make_pair(kern, dev)];
  if (bytes > cur) {
    SG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    cur = bytes;
  }
  return SIGLIP2_OK;
}

}  // namespace sg
