// 8-bit (e4m3) operands for the tensor-core GEMM (gemm_tc2_kernel<..., kF8>).
//
// Per-row quantisation: for row r of x,
//     amax[r]  = max_c |x[r, c]|
//     scale[r] = amax[r] / 448                      (448 = largest finite e4m3)
//     q[r, c]  = e4m3(x[r, c] * (448 / amax[r]))     round to nearest even,
//                                                    saturating at +-448
// (an all-zero row gets scale 0 and zero codes), so x[r, c] ~ q[r, c] * scale[r].
// Applied to activations it gives per-token scales, to a weight [N_out, K]
// per-output-channel scales; the GEMM epilogue multiplies the fp32
// accumulator by a_scale[m] * b_scale[n].
//
// One warp per row, 8 elements (16 bytes of bf16 / f16, 32 of fp32) per lane
// per step: a first pass for the row maximum (warp-shuffle reduction), a
// second pass (the row is then in L1 / L2) that converts pairs with
// cvt.rn.satfinite.e4m3x2.f32 and stores 8 codes per lane as one 8-byte word.
#pragma once

#include "rowops.cuh"

namespace sg {

__device__ __forceinline__ uint16_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

template <typename T>
__device__ __forceinline__ void load8_f32(const T* p, float* f) {
  if constexpr (std::is_same<T, float>::value) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = Pack2<T>::unpack(w[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
}

// x [rows, cols] (row stride ldx elements) -> q [rows, cols] e4m3 codes (row
// stride ldq bytes) and scale [rows]; cols % 8 == 0, 16-byte aligned rows.
template <typename T>
__global__ void __launch_bounds__(256) quantize_e4m3_rows_kernel(const T* __restrict__ x, int ldx, int rows, int cols,
                                                                 uint8_t* __restrict__ q, int ldq,
                                                                 float* __restrict__ scale) {
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const T* xr = x + static_cast<size_t>(r) * ldx;
    float amax = 0.f;
    for (int c = lane * 8; c < cols; c += 256) {
      float f[8];
      load8_f32(xr + c, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float inv = amax > 0.f ? 448.f / amax : 0.f;
    if (lane == 0) scale[r] = amax / 448.f;
    uint8_t* qr = q + static_cast<size_t>(r) * ldq;
    for (int c = lane * 8; c < cols; c += 256) {
      float f[8];
      load8_f32(xr + c, f);
      uint2 w;
      w.x = static_cast<uint32_t>(cvt_e4m3x2(f[0] * inv, f[1] * inv)) |
            (static_cast<uint32_t>(cvt_e4m3x2(f[2] * inv, f[3] * inv)) << 16);
      w.y = static_cast<uint32_t>(cvt_e4m3x2(f[4] * inv, f[5] * inv)) |
            (static_cast<uint32_t>(cvt_e4m3x2(f[6] * inv, f[7] * inv)) << 16);
      *reinterpret_cast<uint2*>(qr + c) = w;
    }
  }
}

}  // namespace sg
