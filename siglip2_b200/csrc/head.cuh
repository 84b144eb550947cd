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
//   scores:  [score_rows, H] float32 scratch (indexed by packed token)
//   pooled:  [B, H, D] element type T
// An image whose score rows [cu[b], cu[b+1]) do not lie inside
// [0, score_rows) writes nothing: its CTA records kSiteHeadPoolScores in the
// device error flag and returns (the scratch may be a fixed array whose
// size the caller does not control).
template <typename T>
__global__ void head_pool_kernel(const T* __restrict__ x, int D, int H, const int* __restrict__ cu, int pad_P,
                                 const float* __restrict__ u, float* __restrict__ scores, int score_rows,
                                 T* __restrict__ pooled) {
  extern __shared__ float sh[];  // u: [H][D], then m[H], inv[H]
  float* su = sh;
  float* sm = su + H * D;
  float* sinv = sm + H;
  const int b = blockIdx.x;
  const int t0 = cu[b];
  const int L = cu[b + 1] - t0;
  if (t0 < 0 || L < 0 || static_cast<long long>(t0) + L > score_rows) {  // uniform over the CTA
    if (threadIdx.x == 0) record_error(kSiteHeadPoolScores);
    return;
  }
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

// ---------------------------------------------------------------------------
// Parallel form of the pooling (used by siglip2_head_pool / the forward):
//   head_scores_kernel: scores[t][h] = x_t . u_h for every packed token t,
//     one warp per token, u staged in shared memory; grid over all tokens.
//   head_pool_rows_kernel: one CTA per (image, 64-column chunk): per-head max
//     and normaliser of the image's scores, then rows of x and their softmax
//     weights staged through shared memory 32 rows at a time; thread
//     (head, 4 columns) accumulates sum_j p_jh x_j.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void head_scores_kernel(const T* __restrict__ x, int D, int H, const int* __restrict__ cu, int B,
                                   int pad_P, const int* __restrict__ tok_img, int N, const float* __restrict__ u,
                                   float* __restrict__ scores) {
  extern __shared__ float su[];  // [H][D]
  for (int i = threadIdx.x; i < H * D; i += blockDim.x) su[i] = u[i];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int nvec = D / 8;
  for (int t = blockIdx.x * nwarps + warp; t < N; t += gridDim.x * nwarps) {
    size_t row = static_cast<size_t>(t);
    if (pad_P > 0) {
      const int b = tok_img[t];
      row = static_cast<size_t>(b) * pad_P + (t - cu[b]);
    }
    const T* xr = x + row * D;
    float acc[16];
#pragma unroll
    for (int h = 0; h < 16; ++h) acc[h] = 0.f;
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
          const float4* uh = reinterpret_cast<const float4*>(su + h * D + v * 8);
          const float4 a = uh[0], b = uh[1];
          acc[h] = fmaf(f[0], a.x, fmaf(f[1], a.y, fmaf(f[2], a.z, fmaf(f[3], a.w, acc[h]))));
          acc[h] = fmaf(f[4], b.x, fmaf(f[5], b.y, fmaf(f[6], b.z, fmaf(f[7], b.w, acc[h]))));
        }
      }
    }
#pragma unroll
    for (int h = 0; h < 16; ++h) {
      if (h < H) {
        const float sv = warp_sum(acc[h]);
        if (lane == h) scores[static_cast<size_t>(t) * H + h] = sv;
      }
    }
  }
}

// block = 256 threads: thread (h = tid / 16, q = tid % 16) owns columns
// [c0 + 4q, c0 + 4q + 4) of head h (H <= 16, 64 columns per CTA)
template <typename T>
__global__ void __launch_bounds__(256) head_pool_rows_kernel(const T* __restrict__ x, int D, int H,
                                                             const int* __restrict__ cu, int pad_P,
                                                             const float* __restrict__ scores,
                                                             T* __restrict__ pooled) {
  constexpr int RB = 32;                  // rows per staging block
  __shared__ float sx[RB][64];            // x rows, this CTA's 64 columns
  __shared__ float sp[RB][16];            // softmax weights of those rows
  __shared__ float smx[16], sinv[16];
  const int b = blockIdx.x;
  const int c0 = blockIdx.y * 64;
  const int t0 = cu[b];
  const int L = cu[b + 1] - t0;
  const size_t base = pad_P > 0 ? static_cast<size_t>(b) * pad_P : static_cast<size_t>(t0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // per-head max and normaliser over the image (warp h handles heads h, h+8)
  for (int h = warp; h < H; h += 8) {
    float m = -INFINITY;
    for (int j = lane; j < L; j += 32) m = fmaxf(m, scores[static_cast<size_t>(t0 + j) * H + h]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.f;
    for (int j = lane; j < L; j += 32) sum += exp2f(scores[static_cast<size_t>(t0 + j) * H + h] - m);
    sum = warp_sum(sum);
    if (lane == 0) {
      smx[h] = m;
      sinv[h] = 1.f / sum;
    }
  }
  __syncthreads();
  const int h = threadIdx.x >> 4, q = threadIdx.x & 15;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j0 = 0; j0 < L; j0 += RB) {
    const int nr = min(RB, L - j0);
    // stage rows (64 columns = 8 vectors of 8 per row) and weights
    for (int i = threadIdx.x; i < RB * 8; i += 256) {
      const int r = i >> 3, v = i & 7;
      float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      const int col = c0 + v * 8;
      if (r < nr && col < D) {
        const T* src = x + (base + j0 + r) * D + col;
        if constexpr (sizeof(T) == 4) {
          load_vec(src, f);
          load_vec(src + 4, f + 4);
        } else {
          load_vec(src, f);
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) sx[r][v * 8 + k] = f[k];
    }
    for (int i = threadIdx.x; i < RB * 16; i += 256) {
      const int r = i >> 4, hh = i & 15;
      sp[r][hh] = (r < nr && hh < H) ? exp2f(scores[static_cast<size_t>(t0 + j0 + r) * H + hh] - smx[hh]) * sinv[hh]
                                     : 0.f;
    }
    __syncthreads();
    if (h < H) {
#pragma unroll 8
      for (int r = 0; r < RB; ++r) {
        const float pw = sp[r][h];
        const float4 xv = *reinterpret_cast<const float4*>(&sx[r][4 * q]);
        acc[0] = fmaf(pw, xv.x, acc[0]);
        acc[1] = fmaf(pw, xv.y, acc[1]);
        acc[2] = fmaf(pw, xv.z, acc[2]);
        acc[3] = fmaf(pw, xv.w, acc[3]);
      }
    }
    __syncthreads();
  }
  const int col = c0 + 4 * q;
  if (h < H && col < D) {
    T* o = pooled + (static_cast<size_t>(b) * H + h) * D + col;
    if constexpr (sizeof(T) == 4) {
      *reinterpret_cast<float4*>(o) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    } else {
      uint2 w;
      w.x = Pack2<T>::pack(acc[0], acc[1]);
      w.y = Pack2<T>::pack(acc[2], acc[3]);
      *reinterpret_cast<uint2*>(o) = w;
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
