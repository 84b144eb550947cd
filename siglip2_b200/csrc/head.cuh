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
// Parallel form of the pooling (used by the forward):
//   head_scores_kernel: scores[t][h] = x_t . u_h for every packed token t.
//     Each warp takes 4 tokens at a time and lane l owns the 4-column groups
//     l, l + 32, ... of D (loads two groups ahead of the FMAs), so every
//     float4 of u read from shared memory feeds 16 FMAs (4 tokens x 4
//     columns).  The 64 partial sums of a lane (4 tokens x 16 heads) are then
//     reduce-scattered across the warp (62 shuffles): lane l ends with the
//     totals of entries 2l and 2l + 1, i.e. token l / 8, heads 2 (l % 8) and
//     2 (l % 8) + 1.
//   head_pool_rows_kernel: one CTA per (image, 128-column chunk): per-head
//     max and normaliser of the image's scores (one online pass over
//     coalesced score rows, 16 loads in flight per thread), then the softmax
//     weights of 64 rows at a time in shared memory (double-buffered: the
//     next block's scores load while this block runs).  Warp w takes rows
//     w, w + 4, ... of each block (16 row loads in flight per lane) for all
//     16 heads and lane c columns 4c..4c+3 of the chunk, 64 FMAs per 8-byte
//     load; the four warps' partial sums are added in a fixed order at the
//     end, so the result is deterministic.
// ---------------------------------------------------------------------------
// 4 consecutive elements: one 8-byte load (16-bit types) or one 16-byte load
// (fp32), kept raw until used
template <typename T>
struct Raw4 {
  using type = uint2;
};
template <>
struct Raw4<float> {
  using type = float4;
};
template <typename T>
__device__ __forceinline__ T from_float(float v) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return __float2bfloat16_rn(v);
  } else if constexpr (std::is_same<T, __half>::value) {
    return __float2half_rn(v);
  } else {
    return v;
  }
}
template <typename T>
__device__ __forceinline__ typename Raw4<T>::type load_raw4(const T* p) {
  return *reinterpret_cast<const typename Raw4<T>::type*>(p);
}
template <typename T>
__device__ __forceinline__ void unpack_raw4(const typename Raw4<T>::type& r, float* f) {
  if constexpr (sizeof(T) == 4) {
    f[0] = r.x;
    f[1] = r.y;
    f[2] = r.z;
    f[3] = r.w;
  } else {
    const float2 a = Pack2<T>::unpack(r.x), b = Pack2<T>::unpack(r.y);
    f[0] = a.x;
    f[1] = a.y;
    f[2] = b.x;
    f[3] = b.y;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) head_scores_kernel(const T* __restrict__ x, int D, int H,
                                                          const int* __restrict__ cu, int pad_P,
                                                          const int* __restrict__ tok_img, int N,
                                                          const float* __restrict__ u, float* __restrict__ scores) {
  extern __shared__ float su[];  // [16][D]; heads past H are zero
  for (int i = threadIdx.x; i < 16 * D; i += blockDim.x) su[i] = i < H * D ? u[i] : 0.f;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int ngroups = D >> 2;
  using R = typename Raw4<T>::type;
  for (int t0 = (blockIdx.x * nwarps + warp) * 4; t0 < N; t0 += gridDim.x * nwarps * 4) {
    const T* xr[4];
    bool ok[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int t = t0 + k;
      ok[k] = t < N;
      size_t row = ok[k] ? static_cast<size_t>(t) : 0;
      if (pad_P > 0 && ok[k]) {
        const int b = tok_img[t];
        row = static_cast<size_t>(b) * pad_P + (t - cu[b]);
      }
      xr[k] = x + row * D;
    }
    float acc[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) acc[i] = 0.f;
    // raw loads two column groups ahead of the FMAs (8 loads in flight per lane)
    R r0[4], r1[4], r2[4];
    auto load_group = [&](int g, R (&dst)[4]) {
#pragma unroll
      for (int k = 0; k < 4; ++k) dst[k] = (ok[k] && g < ngroups) ? load_raw4(xr[k] + 4 * g) : R{};
    };
    load_group(lane, r0);
    load_group(lane + 32, r1);
    for (int g = lane; g < ngroups; g += 32) {
      load_group(g + 64, r2);
      float f[4][4];
#pragma unroll
      for (int k = 0; k < 4; ++k) unpack_raw4<T>(r0[k], f[k]);
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        const float4 w = *reinterpret_cast<const float4*>(su + h * D + 4 * g);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          acc[k * 16 + h] = fmaf(f[k][0], w.x, fmaf(f[k][1], w.y, fmaf(f[k][2], w.z, fmaf(f[k][3], w.w, acc[k * 16 + h]))));
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        r0[k] = r1[k];
        r1[k] = r2[k];
      }
    }
    // reduce-scatter over the warp: after step s a lane keeps 32 >> s entries
    // (the upper or lower half of what it held, by bit 4 - s of its index)
#pragma unroll
    for (int s = 0; s < 5; ++s) {
      const int half = 32 >> s;
      const bool up = (lane >> (4 - s)) & 1;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = up ? acc[i] : acc[i + half];
        const float keep = up ? acc[i + half] : acc[i];
        acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16 >> s);
      }
    }
    const int k = lane >> 3, h0 = 2 * (lane & 7);
    bool okk = false;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) okk = kk == k ? ok[kk] : okk;
    if (okk) {
      float* dst = scores + static_cast<size_t>(t0 + k) * H;
      if (h0 < H) dst[h0] = acc[0];
      if (h0 + 1 < H) dst[h0 + 1] = acc[1];
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(128) head_pool_rows_kernel(const T* __restrict__ x, int D, int H,
                                                             const int* __restrict__ cu, int pad_P,
                                                             const float* __restrict__ scores,
                                                             T* __restrict__ pooled) {
  constexpr int RB = 64;  // rows per block of softmax weights (16 per warp)
  __shared__ __align__(16) float sp[2][RB][16];
  __shared__ __align__(16) float red[4][16][128];  // per-warp partial sums, merged in warp order
  __shared__ float red_m[8][16], red_s[8][16];
  __shared__ float smx[16], sinv[16];
  const int b = blockIdx.x;
  const int c0 = blockIdx.y * 128;
  const int t0 = cu[b];
  const int L = cu[b + 1] - t0;
  const size_t base = pad_P > 0 ? static_cast<size_t>(b) * pad_P : static_cast<size_t>(t0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rg = tid >> 4, hh = tid & 15;  // score loads: row group, head (16 heads = one 64-byte row)
  // per-head max and normaliser over the image: thread (rg, hh) keeps an
  // online (max, sum) over rows rg, rg + 8, ..., and the 8 partials of each
  // head are merged in shared memory
  {
    float m = -INFINITY, sum = 0.f;
    if (hh < H) {
      for (int j0 = rg; j0 < L; j0 += 8 * 16) {
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int j = j0 + 8 * i;
          v[i] = j < L ? scores[static_cast<size_t>(t0 + j) * H + hh] : -INFINITY;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (v[i] > m) {
            sum = sum * exp2f(m - v[i]) + 1.f;
            m = v[i];
          } else if (v[i] > -INFINITY) {
            sum += exp2f(v[i] - m);
          }
        }
      }
    }
    red_m[rg][hh] = m;
    red_s[rg][hh] = sum;
    __syncthreads();
    if (tid < 16) {
      float M = -INFINITY;
#pragma unroll
      for (int r = 0; r < 8; ++r) M = fmaxf(M, red_m[r][tid]);
      float S = 0.f;
#pragma unroll
      for (int r = 0; r < 8; ++r)
        if (red_m[r][tid] > -INFINITY) S += red_s[r][tid] * exp2f(red_m[r][tid] - M);
      smx[tid] = M;
      sinv[tid] = 1.f / S;
    }
    __syncthreads();
  }
  // softmax weights of a 64-row block: thread (rg, hh) owns rows rg + 8i
  float pv[8];
  auto load_p = [&](int j0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int j = j0 + rg + 8 * i;
      pv[i] = (j < L && hh < H) ? scores[static_cast<size_t>(t0 + j) * H + hh] : 0.f;
    }
  };
  auto store_p = [&](int j0, int buf) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = rg + 8 * i;
      sp[buf][r][hh] = (j0 + r < L && hh < H) ? exp2f(pv[i] - smx[hh]) * sinv[hh] : 0.f;
    }
  };
  // thread (warp w, lane c): rows w, w + 4, ... of each block, all 16 heads,
  // columns c0 + 4c .. + 3
  const int col = c0 + 4 * lane;
  const bool col_ok = col < D;  // D % 8 == 0
  using R = typename Raw4<T>::type;
  float acc[16][4];
#pragma unroll
  for (int a = 0; a < 16; ++a)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[a][e] = 0.f;
  load_p(0);
  store_p(0, 0);
  __syncthreads();
  int buf = 0;
  for (int j0 = 0; j0 < L; j0 += RB, buf ^= 1) {
    const bool more = j0 + RB < L;
    if (more) load_p(j0 + RB);  // the next block's scores are in flight during this block
    if (col_ok) {
      const T* xr = x + (base + j0) * D + col;
      R raw[16];  // this warp's 16 rows of the block, all loads in flight at once
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int rr = warp + 4 * i;
        raw[i] = j0 + rr < L ? load_raw4(xr + static_cast<size_t>(rr) * D) : R{};
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int rr = warp + 4 * i;
        float f[4];
        unpack_raw4<T>(raw[i], f);
        const float4* pr = reinterpret_cast<const float4*>(&sp[buf][rr][0]);
#pragma unroll
        for (int hq = 0; hq < 4; ++hq) {
          const float4 pw = pr[hq];
          const float w4[4] = {pw.x, pw.y, pw.z, pw.w};
#pragma unroll
          for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[4 * hq + a][e] = fmaf(w4[a], f[e], acc[4 * hq + a][e]);
        }
      }
    }
    if (more) store_p(j0 + RB, buf ^ 1);
    __syncthreads();
  }
  // merge the four warps' partial sums in a fixed order (deterministic)
#pragma unroll
  for (int a = 0; a < 16; ++a)
    *reinterpret_cast<float4*>(&red[warp][a][4 * lane]) = make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
  __syncthreads();
  const int oc = c0 + tid;  // one output column per thread
  if (oc < D) {
    for (int h = 0; h < H; ++h) {
      const float v = ((red[0][h][tid] + red[1][h][tid]) + red[2][h][tid]) + red[3][h][tid];
      pooled[(static_cast<size_t>(b) * H + h) * D + oc] = from_float<T>(v);
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
