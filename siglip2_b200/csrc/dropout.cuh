// Attention-output dropout of the reference's train mode (model.py:166-169:
// nn.functional.dropout on the per-head attention output before out_proj):
//   y = x * keep / (1 - p),  keep = u >= p,  u uniform in [0, 1).
//
// The mask is a pure function of (seed, offset, element index), so the
// forward (fused into the attention kernel's output store) and the backward
// (siglip2_dropout on the incoming gradient) regenerate the same bits
// without storing them.  u comes from the counter-based generator
// Philox4x32-10 (Salmon, Moraes, Dror and Shaw, "Parallel random numbers:
// as easy as 1, 2, 3", SC 2011): for element e of the logical [rows, width]
// matrix, counter = (e / 4 low, e / 4 high, offset low, offset high), key =
// (seed low, seed high), and word e % 4 of the output gives
// u = (word >> 8) * 2^-24.
#pragma once

#include "rowops.cuh"

namespace sg {

struct DropoutParams {
  float p;            // drop probability in [0, 1); 0 = off
  float scale;        // 1 / (1 - p)
  uint32_t seed_lo, seed_hi;
  uint32_t off_lo, off_hi;
};

__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
  constexpr uint32_t kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u;  // round multipliers
  constexpr uint32_t kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;  // key schedule (Weyl) increments
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = kM0 * c.x, hi0 = __umulhi(kM0, c.x);
    const uint32_t lo1 = kM1 * c.z, hi1 = __umulhi(kM1, c.z);
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
    k0 += kW0;
    k1 += kW1;
  }
  return c;
}

// keep/scale factors of the 8 consecutive elements e0 .. e0+7 (e0 % 8 == 0)
__device__ __forceinline__ void dropout_factors8(const DropoutParams& d, unsigned long long e0, float* f) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const unsigned long long q = (e0 >> 2) + h;
    const uint4 w = philox4x32_10(make_uint4(static_cast<uint32_t>(q), static_cast<uint32_t>(q >> 32), d.off_lo,
                                             d.off_hi),
                                  d.seed_lo, d.seed_hi);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float u = static_cast<float>(ws[i] >> 8) * (1.0f / 16777216.0f);
      f[4 * h + i] = u >= d.p ? d.scale : 0.f;
    }
  }
}

// y[r, c] = x[r, c] * factor(r * width + c) for c < width (width % 8 == 0);
// one thread per 8 consecutive elements of a row, 16-byte accesses for
// bf16/f16 (two for f32).  x and y may alias.
template <typename T>
__global__ void dropout_kernel(const T* x, int ldx, int rows, int width, DropoutParams d, T* y, int ldy) {
  const long long per_row = width / 8;
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= per_row * rows) return;
  const long long r = i / per_row;
  const int c = static_cast<int>(i - r * per_row) * 8;
  float f[8], v[8];
  dropout_factors8(d, static_cast<unsigned long long>(r) * width + c, f);
  const T* xr = x + r * ldx + c;
  T* yr = y + r * ldy + c;
  if constexpr (sizeof(T) == 4) {
    load_vec(xr, v);
    load_vec(xr + 4, v + 4);
  } else {
    load_vec(xr, v);
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) v[k] *= f[k];
  if constexpr (sizeof(T) == 4) {
    store_vec(yr, v);
    store_vec(yr + 4, v + 4);
  } else {
    store_vec(yr, v);
  }
}

}  // namespace sg
