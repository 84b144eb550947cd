// Bandwidth-bound row kernels: the stand-alone LayerNorm (post_layernorm,
// whose output is last_hidden_state), the per-image antialiased resize of
// the learned position grid, LayerNorm row sums for rows no GEMM produced,
// and the L2 normalisation of embeddings before the image-text logits.  They
// move 16 bytes per thread per access (8 x bf16/f16, 4 x f32) and reduce
// with warp shuffles.
#pragma once

#include "ptx.cuh"

namespace sg {

template <typename T>
struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
};

template <typename T>
__device__ __forceinline__ void load_vec(const T* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  } else {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = Pack2<T>::unpack(w[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ void store_vec(T* p, const float* f) {
  uint4 u;
  if constexpr (sizeof(T) == 4) {
    u.x = __float_as_uint(f[0]);
    u.y = __float_as_uint(f[1]);
    u.z = __float_as_uint(f[2]);
    u.w = __float_as_uint(f[3]);
  } else {
    u.x = Pack2<T>::pack(f[0], f[1]);
    u.y = Pack2<T>::pack(f[2], f[3]);
    u.z = Pack2<T>::pack(f[4], f[5]);
    u.w = Pack2<T>::pack(f[6], f[7]);
  }
  *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// LayerNorm statistics in column-block slots.  Slot j of a row holds
// (mean, centred sum of squares) of the row's columns [j*blk, min((j+1)*blk, K)):
// producers that see a block once (the GEMM epilogues) accumulate sums of
// x - s with s the block's first value, so the variance does not cancel when
// the row's mean is large against its spread; the reader merges the slots
// with the pairwise update of Chan, Golub and LeVeque (1979):
//   mean = sum_j n_j mean_j / K,   M2 = sum_j (M2_j + n_j (mean_j - mean)^2).
// ---------------------------------------------------------------------------
constexpr int kRowSumBlock = 128;  // columns per slot

__device__ __forceinline__ float2 slot_stats_from_shifted(float s1, float s2, float shift, int n) {
  const float inv_n = 1.f / static_cast<float>(n);
  const float d = s1 * inv_n;  // mean - shift
  return make_float2(shift + d, fmaxf(s2 - s1 * d, 0.f));
}

// (mu, rstd) of a K-column row from its `slots` slot statistics (blocks of kRowSumBlock)
__device__ __forceinline__ void slot_stats_merge(const float2* __restrict__ r, int slots, int K, float eps, float& mu,
                                                 float& rstd) {
  constexpr int kMaxSlots = 16;  // K <= 2048: every slot loaded once, all loads in flight together
  if (slots <= kMaxSlots) {
    float2 v[kMaxSlots];
#pragma unroll
    for (int j = 0; j < kMaxSlots; ++j) v[j] = j < slots ? r[j] : make_float2(0.f, 0.f);
    float sm = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxSlots; ++j)
      if (j < slots) sm = fmaf(static_cast<float>(min(kRowSumBlock, K - j * kRowSumBlock)), v[j].x, sm);
    const float m = sm / static_cast<float>(K);
    float m2 = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxSlots; ++j) {
      if (j < slots) {
        const float dm = v[j].x - m;
        m2 += fmaf(static_cast<float>(min(kRowSumBlock, K - j * kRowSumBlock)) * dm, dm, v[j].y);
      }
    }
    mu = m;
    rstd = rsqrtf(m2 / static_cast<float>(K) + eps);
    return;
  }
  float sm = 0.f;
  for (int j = 0; j < slots; ++j) sm = fmaf(static_cast<float>(min(kRowSumBlock, K - j * kRowSumBlock)), r[j].x, sm);
  const float m = sm / static_cast<float>(K);
  float m2 = 0.f;
  for (int j = 0; j < slots; ++j) {
    const float2 v = r[j];
    const float dm = v.x - m;
    m2 += fmaf(static_cast<float>(min(kRowSumBlock, K - j * kRowSumBlock)) * dm, dm, v.y);
  }
  mu = m;
  rstd = rsqrtf(m2 / static_cast<float>(K) + eps);
}

// ---------------------------------------------------------------------------
// LayerNorm, one warp per row, two-pass (mean, then centred variance) from
// registers; D <= 32 * 8 * MAXV elements.
//
// Packed mode (cu == nullptr): rows = N, y[r] = LN(x[r]).
// Padded mode: rows = B * P destination rows; destination (b, i) takes source
// row cu[b] + i when i < cu[b+1] - cu[b] and is zero otherwise.
// ---------------------------------------------------------------------------
template <typename T, int MAXV>
__global__ void __launch_bounds__(256) layernorm_kernel(const T* __restrict__ x, T* __restrict__ y,
                                                        const float* __restrict__ gamma,
                                                        const float* __restrict__ beta, int rows, int D, float eps,
                                                        const int* __restrict__ cu, int P) {
  constexpr int V = Vec16<T>::N;
  const int warps_per_block = blockDim.x >> 5;
  const int row = blockIdx.x * warps_per_block + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nvec = D / V;
  int src = row;
  if (cu != nullptr) {
    const int b = row / P, i = row - (row / P) * P;
    const int L = cu[b + 1] - cu[b];
    if (i >= L) {
      float z[V];
#pragma unroll
      for (int k = 0; k < V; ++k) z[k] = 0.f;
      for (int v = lane; v < nvec; v += 32) store_vec(y + static_cast<size_t>(row) * D + v * V, z);
      return;
    }
    src = cu[b] + i;
  }
  const T* xr = x + static_cast<size_t>(src) * D;
  float f[MAXV][V];
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < MAXV; ++c) {
    const int v = lane + c * 32;
    if (v < nvec) {
      load_vec(xr + v * V, f[c]);
#pragma unroll
      for (int k = 0; k < V; ++k) s += f[c][k];
    }
  }
  const float mean = warp_sum(s) / static_cast<float>(D);
  float q = 0.f;
#pragma unroll
  for (int c = 0; c < MAXV; ++c) {
    const int v = lane + c * 32;
    if (v < nvec) {
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const float d = f[c][k] - mean;
        q = fmaf(d, d, q);
      }
    }
  }
  const float rstd = rsqrtf(warp_sum(q) / static_cast<float>(D) + eps);
  T* yr = y + static_cast<size_t>(row) * D;
#pragma unroll
  for (int c = 0; c < MAXV; ++c) {
    const int v = lane + c * 32;
    if (v < nvec) {
      float o[V], gv[V], bv[V];
#pragma unroll
      for (int k4 = 0; k4 < V / 4; ++k4) {  // gamma / beta as float4 (16-byte aligned: D % V == 0)
        const float4 g4 = __ldg(reinterpret_cast<const float4*>(gamma + v * V) + k4);
        const float4 b4 = __ldg(reinterpret_cast<const float4*>(beta + v * V) + k4);
        gv[4 * k4] = g4.x; gv[4 * k4 + 1] = g4.y; gv[4 * k4 + 2] = g4.z; gv[4 * k4 + 3] = g4.w;
        bv[4 * k4] = b4.x; bv[4 * k4 + 1] = b4.y; bv[4 * k4 + 2] = b4.z; bv[4 * k4 + 3] = b4.w;
      }
#pragma unroll
      for (int k = 0; k < V; ++k) o[k] = fmaf((f[c][k] - mean) * rstd, gv[k], bv[k]);
      store_vec(yr + v * V, o);
    }
  }
}

// ---------------------------------------------------------------------------
// Antialiased bilinear resize of the G x G position grid to each image's
// (h, w), written row-major (h outer, w inner) into the packed token order.
//
// One axis of F.interpolate(bilinear, align_corners=False, antialias=True):
//   scale = G / n; support = max(scale, 1); centre c = scale (i + 0.5);
//   taps j in [max(int(c - support + 0.5), 0), min(int(c + support + 0.5), G))
//   weight tri((j - c + 0.5) / max(scale, 1)), tri(t) = max(0, 1 - |t|),
//   normalised to sum 1.
// ---------------------------------------------------------------------------
struct AxisTaps {
  int lo, hi;
  float center, inv, norm;
};

__device__ __forceinline__ AxisTaps axis_taps(int i, int n, int G) {
  AxisTaps a;
  const float scale = static_cast<float>(G) / static_cast<float>(n);
  const float support = scale >= 1.f ? scale : 1.f;
  a.inv = scale >= 1.f ? 1.f / scale : 1.f;
  a.center = scale * (static_cast<float>(i) + 0.5f);
  a.lo = max(static_cast<int>(a.center - support + 0.5f), 0);
  a.hi = min(static_cast<int>(a.center + support + 0.5f), G);
  float tot = 0.f;
  for (int j = a.lo; j < a.hi; ++j) tot += fmaxf(0.f, 1.f - fabsf((static_cast<float>(j) - a.center + 0.5f) * a.inv));
  a.norm = tot > 0.f ? 1.f / tot : 0.f;
  return a;
}

__device__ __forceinline__ float axis_w(const AxisTaps& a, int j) {
  return fmaxf(0.f, 1.f - fabsf((static_cast<float>(j) - a.center + 0.5f) * a.inv)) * a.norm;
}

// grid: (ceil(N / tokens_per_block)), block: (D / 8 threads per token) x tokens
// tok_img[t] = image of token t; hw[2b], hw[2b+1] = (h, w); cu = row starts.
template <typename T>
__global__ void posemb_kernel(const float* __restrict__ table, int G, int D, const int* __restrict__ tok_img,
                              const int* __restrict__ hw, const int* __restrict__ cu, int N, T* __restrict__ out) {
  const int vec_per_tok = D / 8;
  const int t = blockIdx.x * blockDim.y + threadIdx.y;
  const int v = threadIdx.x;
  if (t >= N || v >= vec_per_tok) return;
  const int b = tok_img[t];
  const int h = hw[2 * b], w = hw[2 * b + 1];
  const int i = t - cu[b];
  const int yy = i / w, xx = i - (i / w) * w;
  const AxisTaps ay = axis_taps(yy, h, G);
  const AxisTaps ax = axis_taps(xx, w, G);
  float acc[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) acc[k] = 0.f;
  for (int a = ay.lo; a < ay.hi; ++a) {
    const float wa = axis_w(ay, a);
    for (int c = ax.lo; c < ax.hi; ++c) {
      const float wgt = wa * axis_w(ax, c);
      const float4* src = reinterpret_cast<const float4*>(table + (static_cast<size_t>(a) * G + c) * D + v * 8);
      const float4 p0 = __ldg(src), p1 = __ldg(src + 1);
      acc[0] = fmaf(wgt, p0.x, acc[0]);
      acc[1] = fmaf(wgt, p0.y, acc[1]);
      acc[2] = fmaf(wgt, p0.z, acc[2]);
      acc[3] = fmaf(wgt, p0.w, acc[3]);
      acc[4] = fmaf(wgt, p1.x, acc[4]);
      acc[5] = fmaf(wgt, p1.y, acc[5]);
      acc[6] = fmaf(wgt, p1.z, acc[6]);
      acc[7] = fmaf(wgt, p1.w, acc[7]);
    }
  }
  T* o = out + static_cast<size_t>(t) * D + v * 8;
  if constexpr (sizeof(T) == 4) {
    store_vec(o, acc);
    store_vec(o + 4, acc + 4);
  } else {
    store_vec(o, acc);
  }
}

// token -> image index from row starts (one thread per token, binary search)
__global__ void token_image_kernel(const int* __restrict__ cu, int B, int N, int* __restrict__ tok_img) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= N) return;
  int lo = 0, hi = B;  // find b with cu[b] <= t < cu[b+1]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (cu[mid] <= t) lo = mid; else hi = mid;
  }
  tok_img[t] = lo;
}

// y[r] = scale * x[r] / ||x[r]||_2 (fp32 sum of squares, one rounding to T;
// an all-zero row gives zeros).  One warp per row, 16-byte accesses; D, ldx
// and ldy multiples of the vector width, x and y 16-byte aligned.  The
// normalisation of the embeddings before the image-text logits.
template <typename T>
__global__ void __launch_bounds__(256) l2norm_kernel(const T* __restrict__ x, int ldx, int rows, int D, float scale,
                                                     T* __restrict__ y, int ldy) {
  constexpr int V = Vec16<T>::N;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + static_cast<size_t>(row) * ldx;
  float ss = 0.f;
  for (int c = lane * V; c < D; c += 32 * V) {
    float f[V];
    load_vec(xr + c, f);
#pragma unroll
    for (int i = 0; i < V; ++i) ss = fmaf(f[i], f[i], ss);
  }
  ss = warp_sum(ss);
  const float k = ss > 0.f ? scale / sqrtf(ss) : 0.f;
  T* yr = y + static_cast<size_t>(row) * ldy;
  for (int c = lane * V; c < D; c += 32 * V) {
    float f[V];
    load_vec(xr + c, f);
#pragma unroll
    for (int i = 0; i < V; ++i) f[i] *= k;
    store_vec(yr + c, f);
  }
}

// Slot statistics in the layout the LayerNorm-folded GEMMs read: for row r
// and column block j (columns [j*blk, min((j+1)*blk, K))), rs[r*slots + j] =
// (mean, centred sum of squares), two passes over the block (the second
// reads it from L1).  For rows that no row-sum GEMM produced (the input of a
// stand-alone encoder layer).  One warp per row, 16-byte loads; K, ldx and
// blk are multiples of the vector width and x is 16-byte aligned (the host
// checks).
template <typename T>
__global__ void __launch_bounds__(256) rowsums_kernel(const T* __restrict__ x, int ldx, int M, int K, int blk,
                                                      float2* __restrict__ rs, int slots) {
  constexpr int V = Vec16<T>::N;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const T* xr = x + static_cast<size_t>(row) * ldx;
  for (int j = 0; j < slots; ++j) {
    const int c_end = min(K, (j + 1) * blk);
    float s1 = 0.f;
    for (int c = j * blk + lane * V; c < c_end; c += 32 * V) {
      float f[V];
      load_vec(xr + c, f);
#pragma unroll
      for (int i = 0; i < V; ++i) s1 += f[i];
    }
    const float mean = warp_sum(s1) / static_cast<float>(c_end - j * blk);
    float s2 = 0.f;
    for (int c = j * blk + lane * V; c < c_end; c += 32 * V) {
      float f[V];
      load_vec(xr + c, f);
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const float d = f[i] - mean;
        s2 = fmaf(d, d, s2);
      }
    }
    s2 = warp_sum(s2);
    if (lane == 0) rs[static_cast<size_t>(row) * slots + j] = make_float2(mean, s2);
  }
}

}  // namespace sg

namespace sg {

// ---------------------------------------------------------------------------
// LayerNorm backward (the gradient of layernorm_kernel / nn.LayerNorm,
// model.py:199,201,256), two deterministic passes:
//   rows:    one warp per row loads its x and dy vectors together (both in
//            flight at once), recomputes mean and rstd from x (two-pass, as
//            the forward), then with g = dy * gamma and xh = (x - mean) rstd
//              dx = rstd (g - mean(g) - xh mean(g xh))
//            and writes dx and the row's (mean, rstd);
//   columns: per chunk of rows, dgamma[c] = sum dy xh and dbeta[c] = sum dy,
//            one partial row per chunk (summed over chunks in a fixed order
//            by the caller); each lane owns 8 columns (one 16-byte vector),
//            a warp 256 columns of a row, the 8 warps of a CTA step through
//            the chunk's rows four at a time (four rows' loads in flight)
//            and are reduced in shared memory in warp order.
// ---------------------------------------------------------------------------
template <typename T, int MAXV>
__global__ void __launch_bounds__(256) layernorm_bwd_rows_kernel(const T* __restrict__ x, const T* __restrict__ dy,
                                                                 const float* __restrict__ gamma, int rows, int D,
                                                                 float eps, T* __restrict__ dx,
                                                                 float2* __restrict__ stats) {
  constexpr int V = Vec16<T>::N;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nvec = D / V;
  const T* xr = x + static_cast<size_t>(row) * D;
  const T* dr = dy + static_cast<size_t>(row) * D;
  float f[MAXV][V], gv[MAXV][V];
#pragma unroll
  for (int c = 0; c < MAXV; ++c) {
    const int v = lane + c * 32;
    if (v < nvec) {
      load_vec(xr + v * V, f[c]);
      load_vec(dr + v * V, gv[c]);
    }
  }
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < MAXV; ++c)
    if (lane + c * 32 < nvec) {
#pragma unroll
      for (int k = 0; k < V; ++k) s += f[c][k];
    }
  const float mean = warp_sum(s) / static_cast<float>(D);
  float q = 0.f;
#pragma unroll
  for (int c = 0; c < MAXV; ++c) {
    if (lane + c * 32 < nvec) {
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const float d = f[c][k] - mean;
        q = fmaf(d, d, q);
      }
    }
  }
  const float rstd = rsqrtf(warp_sum(q) / static_cast<float>(D) + eps);
  // g = dy * gamma in gv, xh in f
  float sg = 0.f, sgx = 0.f;
#pragma unroll
  for (int c = 0; c < MAXV; ++c) {
    const int v = lane + c * 32;
    if (v < nvec) {
#pragma unroll
      for (int k4 = 0; k4 < V / 4; ++k4) {
        const float4 g4 = __ldg(reinterpret_cast<const float4*>(gamma + v * V) + k4);
        gv[c][4 * k4] *= g4.x;
        gv[c][4 * k4 + 1] *= g4.y;
        gv[c][4 * k4 + 2] *= g4.z;
        gv[c][4 * k4 + 3] *= g4.w;
      }
#pragma unroll
      for (int k = 0; k < V; ++k) {
        f[c][k] = (f[c][k] - mean) * rstd;
        sg += gv[c][k];
        sgx = fmaf(gv[c][k], f[c][k], sgx);
      }
    }
  }
  const float inv_d = 1.f / static_cast<float>(D);
  const float mg = warp_sum(sg) * inv_d, mgx = warp_sum(sgx) * inv_d;
  T* o = dx + static_cast<size_t>(row) * D;
#pragma unroll
  for (int c = 0; c < MAXV; ++c) {
    const int v = lane + c * 32;
    if (v < nvec) {
      float r[V];
#pragma unroll
      for (int k = 0; k < V; ++k) r[k] = rstd * (gv[c][k] - mg - f[c][k] * mgx);
      store_vec(o + v * V, r);
    }
  }
  if (lane == 0) stats[row] = make_float2(mean, rstd);
}

// 8 consecutive values of a row as floats (one or two 16-byte loads)
template <typename T>
__device__ __forceinline__ void load8(const T* p, float* f) {
  if constexpr (sizeof(T) == 4) {
    load_vec(p, f);
    load_vec(p + 4, f + 4);
  } else {
    load_vec(p, f);
  }
}

// grid (ceil(D / 256), chunks), 256 threads; chunk j covers rows [j * chunk_rows, ...)
template <typename T>
__global__ void __launch_bounds__(256) layernorm_bwd_cols_kernel(const T* __restrict__ x, const T* __restrict__ dy,
                                                                 const float2* __restrict__ stats, int rows, int D,
                                                                 int chunk_rows, float* __restrict__ dgamma_part,
                                                                 float* __restrict__ dbeta_part) {
  __shared__ float red[2][8][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x * 256 + 8 * lane;  // this lane's 8 columns
  const int r0 = blockIdx.y * chunk_rows;
  const int r1 = min(rows, r0 + chunk_rows);
  float g[8], b[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) g[k] = b[k] = 0.f;
  if (c < D) {
    int r = r0 + warp;
    for (; r + 24 < r1; r += 32) {  // four rows (8 apart) per step, loads first
      float xv[4][8], dv[4][8];
      float2 st[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const size_t off = static_cast<size_t>(r + 8 * u) * D + c;
        load8(x + off, xv[u]);
        load8(dy + off, dv[u]);
        st[u] = stats[r + 8 * u];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          g[k] = fmaf(dv[u][k], (xv[u][k] - st[u].x) * st[u].y, g[k]);
          b[k] += dv[u][k];
        }
    }
    for (; r < r1; r += 8) {
      float xv[8], dv[8];
      const size_t off = static_cast<size_t>(r) * D + c;
      load8(x + off, xv);
      load8(dy + off, dv);
      const float2 st = stats[r];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        g[k] = fmaf(dv[k], (xv[k] - st.x) * st.y, g[k]);
        b[k] += dv[k];
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    red[0][warp][8 * lane + k] = g[k];
    red[1][warp][8 * lane + k] = b[k];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 512; i += 256) {
    const int which = i >> 8, col = i & 255;
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[which][w][col];  // fixed order
    const int cc = blockIdx.x * 256 + col;
    if (cc < D) (which ? dbeta_part : dgamma_part)[static_cast<size_t>(blockIdx.y) * D + cc] = t;
  }
}

// Column sums of x [rows, cols] in fp32 (the bias gradient of a Linear
// layer: db = sum over tokens of dy), deterministic: grid (ceil(cols / 256),
// chunks), chunk j writes part[j][c] = sum of its chunk_rows rows; each lane
// owns 8 columns, the 8 warps of a CTA step through the chunk four rows at a
// time and are reduced in shared memory in warp order; the caller sums the
// chunks in order.
template <typename T>
__global__ void __launch_bounds__(256) colsum_part_kernel(const T* __restrict__ x, int ld, int rows, int cols,
                                                          int chunk_rows, float* __restrict__ part) {
  __shared__ float red[8][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x * 256 + 8 * lane;
  const int r0 = blockIdx.y * chunk_rows;
  const int r1 = min(rows, r0 + chunk_rows);
  float b[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) b[k] = 0.f;
  if (c < cols) {
    int r = r0 + warp;
    for (; r + 24 < r1; r += 32) {
      float v[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u) load8(x + static_cast<size_t>(r + 8 * u) * ld + c, v[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int k = 0; k < 8; ++k) b[k] += v[u][k];
    }
    for (; r < r1; r += 8) {
      float v[8];
      load8(x + static_cast<size_t>(r) * ld + c, v);
#pragma unroll
      for (int k = 0; k < 8; ++k) b[k] += v[k];
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) red[warp][8 * lane + k] = b[k];
  __syncthreads();
  {
    const int col = threadIdx.x;
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w][col];  // fixed order
    const int cc = blockIdx.x * 256 + col;
    if (cc < cols) part[static_cast<size_t>(blockIdx.y) * cols + cc] = t;
  }
}

}  // namespace sg
