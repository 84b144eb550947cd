// Attention-pooling head (one learned probe per image; transformers
// Siglip2MultiheadAttentionPoolingHead semantics) and the small gather
// kernels around the tower.
//
// With a single query q_h per head, the head's attention needs neither K nor V
// for every token:
//   score_jh = q_h . (W_k,h x_j + b_k,h) / sqrt(hd)
//            = x_j . u_h + const_h,          u_h = W_k,h^T q_h / sqrt(hd)
// (const_h cancels in the softmax over j), and because the weights sum to 1
//   sum_j p_jh (W_v,h x_j + b_v,h) = W_v,h (sum_j p_jh x_j) + b_v,h.
// So the per-token work is two passes over the image's rows of x: scores
// against H vectors u_h, then H softmax-weighted row sums.  u_h (times
// log2 e) is precomputed once per weight load.
#pragma once

#include "rowops.cuh"

namespace sg {

// One CTA per image.  Threads = (D/8) x (H/4): thread (v, g) owns columns
// [8v, 8v+8) for heads [4g, 4g+4) in the pooling pass.
//   x:       rows of the image are base + i, i < L (base = cu[b], or b * P
//            when the hidden state is stored padded)
//   u:       [H, D] float32, already scaled by log2(e) / sqrt(hd)
//   scores:  [N_rows_total, H] float32 scratch (indexed by packed token)
//   pooled:  [B, H, D] element type T
template <typename T>
__global__ void head_pool_kernel(const T* __restrict__ x, int D, int H, const int* __restrict__ cu, int pad_P,
                                 const float* __restrict__ u, float* __restrict__ scores, T* __restrict__ pooled) {
  extern __shared__ float sh[];  // u: [H][D], then m[H], inv[H]
  float* su = sh;
  float* sm = su + H * D;
  float* sinv = sm + H;
  const int b = blockIdx.x;
  const int t0 = cu[b];
  const int L = cu[b + 1] - t0;
  const size_t base = pad_P > 0 ? static_cast<size_t>(b) * pad_P : static_cast<size_t>(t0);
  const int nthr = blockDim.x;
  for (int i = threadIdx.x; i < H * D; i += nthr) su[i] = u[i];
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = nthr >> 5;
  const int nvec = D / 8;
  // pass 1: scores[j][h] = x_j . u_h  (one warp per row)
  for (int j = warp; j < L; j += nwarps) {
    float acc[16];
#pragma unroll
    for (int h = 0; h < 16; ++h) acc[h] = 0.f;
    const T* xr = x + (base + j) * D;
    for (int v = lane; v < nvec; v += 32) {
      float f[8];
      if constexpr (sizeof(T) == 4) {
        load_vec(xr + v * 8, f);
        load_vec(xr + v * 8 + 4, f + 4);
      } else {
        load_vec(xr + v * 8, f);
      }
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        if (h < H) {
          const float* uh = su + h * D + v * 8;
#pragma unroll
          for (int k = 0; k < 8; ++k) acc[h] = fmaf(f[k], uh[k], acc[h]);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < 16; ++h) {
      if (h < H) {
        const float s = warp_sum(acc[h]);
        if (lane == h) scores[static_cast<size_t>(t0 + j) * H + h] = s;
      }
    }
  }
  __syncthreads();
  // pass 2: per-head max and normaliser (one warp per head)
  for (int h = warp; h < H; h += nwarps) {
    float m = -INFINITY;
    for (int j = lane; j < L; j += 32) m = fmaxf(m, scores[static_cast<size_t>(t0 + j) * H + h]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
    for (int j = lane; j < L; j += 32) s += exp2f(scores[static_cast<size_t>(t0 + j) * H + h] - m);
    s = warp_sum(s);
    if (lane == 0) {
      sm[h] = m;
      sinv[h] = 1.f / s;
    }
  }
  __syncthreads();
  // pass 3: pooled[b][h][:] = sum_j p_jh x_j
  const int v = threadIdx.x % nvec;
  const int g = threadIdx.x / nvec;
  if (g * 4 < H) {
    float acc[4][8];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[a][k] = 0.f;
    for (int j = 0; j < L; ++j) {
      float f[8];
      const T* xr = x + (base + j) * D + v * 8;
      if constexpr (sizeof(T) == 4) {
        load_vec(xr, f);
        load_vec(xr + 4, f + 4);
      } else {
        load_vec(xr, f);
      }
      const float* sr = scores + static_cast<size_t>(t0 + j) * H + g * 4;
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const float pw = exp2f(sr[a] - sm[g * 4 + a]) * sinv[g * 4 + a];
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[a][k] = fmaf(pw, f[k], acc[a][k]);
      }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      T* o = pooled + (static_cast<size_t>(b) * H + g * 4 + a) * D + v * 8;
      if constexpr (sizeof(T) == 4) {
        store_vec(o, acc[a]);
        store_vec(o + 4, acc[a] + 4);
      } else {
        store_vec(o, acc[a]);
      }
    }
  }
}

// attn[b][n] = Y[b*H + n / hd][n] (Y = pooled . W_v^T + b_v computed for every
// head row; row (b, h) only keeps head h's columns)
template <typename T>
__global__ void head_select_kernel(const T* __restrict__ Y, int H, int hd, int D, int B, T* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // over B * D / 8
  const int nvec = D / 8;
  if (i >= B * nvec) return;
  const int b = i / nvec, v = i - (i / nvec) * nvec;
  const int col = v * 8;
  const int h = col / hd;  // hd is a multiple of 8: a vector never straddles heads
  const uint4* src = reinterpret_cast<const uint4*>(Y + (static_cast<size_t>(b) * H + h) * D + col);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(b) * D + col);
  if constexpr (sizeof(T) == 4) {
    dst[0] = src[0];
    dst[1] = src[1];
  } else {
    dst[0] = src[0];
  }
}

// packed[t] = padded[b * P + (t - cu[b])]  (row gather of the valid rows)
template <typename T>
__global__ void gather_rows_kernel(const T* __restrict__ padded, int C, int P, const int* __restrict__ cu,
                                   const int* __restrict__ tok_img, int N, T* __restrict__ packed) {
  const int vec = 16 / sizeof(T);
  const int nvec = C / vec;
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<size_t>(N) * nvec) return;
  const int t = static_cast<int>(i / nvec);
  const int v = static_cast<int>(i - static_cast<size_t>(t) * nvec);
  const int b = tok_img[t];
  const size_t src_row = static_cast<size_t>(b) * P + (t - cu[b]);
  reinterpret_cast<uint4*>(packed + static_cast<size_t>(t) * C)[v] =
      reinterpret_cast<const uint4*>(padded + src_row * C)[v];
}

}  // namespace sg
