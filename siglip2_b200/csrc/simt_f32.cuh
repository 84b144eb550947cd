// fp32 path (the reference's CPU-runnable configuration runs in fp32 and its
// parity bar is 1e-4 max-abs): CUDA-core FFMA kernels with the same fused
// epilogues as the tensor-core GEMM, and a per-image attention kernel.
// Exact fp32 accumulation; GELU uses tanhf.
#pragma once

#include "gemm.cuh"
#include "rowops.cuh"

namespace sg {

// C[M,N] = epi(A[M,K] . B[N,K]^T); 128x128 CTA tile, 8x8 per thread, K step 16.
constexpr int kSgBM = 128, kSgBN = 128, kSgBK = 16;

template <int EPI>
__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* __restrict__ A, int lda,
                                                       const float* __restrict__ Bm, int ldb, float* out, int ldo,
                                                       const float* res, int ldr, GemmParams p) {
  __shared__ float As[kSgBK][kSgBM + 4];
  __shared__ float Bs[kSgBK][kSgBN + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * kSgBM, n0 = blockIdx.x * kSgBN;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  for (int k0 = 0; k0 < p.K; k0 += kSgBK) {
    // 128 rows x 16 k of A and of B: 2048 floats each, 8 per thread
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = threadIdx.x + i * 256;
      const int r = idx >> 4, kk = idx & 15;
      const int gk = k0 + kk;
      As[kk][r] = (m0 + r < p.M && gk < p.K) ? A[static_cast<size_t>(m0 + r) * lda + gk] : 0.f;
      Bs[kk][r] = (n0 + r < p.N && gk < p.K) ? Bm[static_cast<size_t>(n0 + r) * ldb + gk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kSgBK; ++kk) {
      float a[8], b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = As[kk][ty * 8 + i];
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = Bs[kk][tx * 8 + j];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  constexpr bool kLnRs = (EPI == kEpiLnRs || EPI == kEpiLnRsGelu);
  constexpr bool kGelu = epi_is_gelu(EPI);
  constexpr bool kRsOut = (EPI == kEpiBiasResRs || EPI == kEpiBiasPosRs);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    // uniform across the 16 threads (tx) of this row: the row-sum shuffles below need all of them
    const int row = m0 + ty * 8 + i;
    const bool row_ok = row < p.M;
    AxisTaps ay{0, 0, 0.f, 1.f, 0.f}, ax{0, 0, 0.f, 1.f, 0.f};
    if constexpr (EPI == kEpiBiasPosRs) {
      if (row_ok) {
        const int b = p.tok_img[row];
        const int w = p.pos_hw[2 * b + 1];
        const int t = row - p.cu[b];
        ay = axis_taps(t / w, p.pos_hw[2 * b], p.pos_grid);
        ax = axis_taps(t - (t / w) * w, w, p.pos_grid);
      }
    }
    float mu = 0.f, rstd = 1.f;
    if constexpr (kLnRs) {
      if (row_ok) slot_stats_merge(p.rs_in + static_cast<size_t>(row) * p.rs_ld, p.rs_ld, p.K, p.eps, mu, rstd);
    }
    float vout[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int col = n0 + tx * 8 + j;
      vout[j] = 0.f;
      if (!row_ok || col >= p.N) continue;
      float v = acc[i][j];
      if constexpr (kLnRs) {
        v = rstd * (v - mu * p.c1[col]) + p.c2[col];
      } else {
        v += p.bias[col];
      }
      if constexpr (EPI == kEpiBiasPosRs) {
        for (int ya = ay.lo; ya < ay.hi; ++ya)
          for (int xa = ax.lo; xa < ax.hi; ++xa)
            v = fmaf(axis_w(ay, ya) * axis_w(ax, xa), p.pos_table[static_cast<size_t>(ya * p.pos_grid + xa) * p.N + col], v);
      }
      if constexpr (kGelu) v = 0.5f * v * (1.f + tanhf(0.7978845608028654f * (v + 0.044715f * v * v * v)));
      if constexpr (epi_has_res(EPI)) v += res[static_cast<size_t>(row) * ldr + col];
      out[static_cast<size_t>(row) * ldo + col] = v;
      vout[j] = v;
    }
    if constexpr (kRsOut) {
      // this CTA's 128 columns are one slot: (mean, centred sum of squares),
      // two passes over the row's values, reduced over the 16 threads of the
      // row in a fixed order
      const int n_valid = min(kSgBN, p.N - n0);
      float s1 = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) s1 += vout[j];
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      const float mean = s1 / static_cast<float>(n_valid);
      float s2 = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = n0 + tx * 8 + j < p.N ? vout[j] - mean : 0.f;
        s2 = fmaf(d, d, s2);
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
      if (tx == 0 && row_ok) p.rs_acc[static_cast<size_t>(row) * p.rs_ld + blockIdx.x] = make_float2(mean, s2);
    }
  }
}

// Slot statistics (mean, centred sum of squares) of a [M, K] fp32 matrix in
// 128-column slots ([M][ld] pairs): what the row-sum LayerNorm epilogues
// read, for rows whose producer is not a GEMM.  One warp per row, two passes.
__global__ void rowsums_f32_kernel(const float* __restrict__ x, int M, int K, float2* __restrict__ rs, int ld) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  for (int j = 0; j < ld; ++j) {
    const int k_end = min(K, (j + 1) * kRowSumBlock);
    float s1 = 0.f;
    for (int k = j * kRowSumBlock + lane; k < k_end; k += 32) s1 += x[static_cast<size_t>(row) * K + k];
    const float mean = warp_sum(s1) / static_cast<float>(k_end - j * kRowSumBlock);
    float s2 = 0.f;
    for (int k = j * kRowSumBlock + lane; k < k_end; k += 32) {
      const float d = x[static_cast<size_t>(row) * K + k] - mean;
      s2 = fmaf(d, d, s2);
    }
    s2 = warp_sum(s2);
    if (lane == 0) rs[static_cast<size_t>(row) * ld + j] = make_float2(mean, s2);
  }
}

// Per-image attention in fp32: one thread per query row, one CTA per
// (128-query tile of an image, head); keys and values of the image stream
// through shared memory 32 at a time with an online softmax.
// qkv: [N, 3*H*hd] (q | k | v, head-major inside each), out: [N, ldo].
template <int HD>
__global__ void __launch_bounds__(128) fmha_f32_kernel(const float* __restrict__ qkv, const int* __restrict__ cu,
                                                       const int2* __restrict__ tiles, int H, float scale,
                                                       float* __restrict__ out, int ldo) {
  __shared__ float Ks[32][HD + 1];
  __shared__ float Vs[32][HD];
  const int2 tile = tiles[blockIdx.x];
  const int head = blockIdx.y;
  const int row0 = cu[tile.x];
  const int L = cu[tile.x + 1] - row0;
  const int qi = tile.y * 128 + threadIdx.x;
  const bool active = qi < L;
  const int ldq = 3 * H * HD;
  float q[HD], o[HD];
  if (active) {
    const float* qp = qkv + static_cast<size_t>(row0 + qi) * ldq + head * HD;
#pragma unroll
    for (int d = 0; d < HD; ++d) q[d] = qp[d] * scale;
  }
#pragma unroll
  for (int d = 0; d < HD; ++d) o[d] = 0.f;
  float m = -INFINITY, l = 0.f;
  for (int j0 = 0; j0 < L; j0 += 32) {
    const int nk = min(32, L - j0);
    for (int i = threadIdx.x; i < 32 * HD; i += 128) {
      const int r = i / HD, d = i - (i / HD) * HD;
      const size_t base = static_cast<size_t>(row0 + j0 + r) * ldq;
      Ks[r][d] = r < nk ? qkv[base + (H + head) * HD + d] : 0.f;
      Vs[r][d] = r < nk ? qkv[base + (2 * H + head) * HD + d] : 0.f;
    }
    __syncthreads();
    if (active) {
      float sc[32];
      float mt = -INFINITY;
#pragma unroll
      for (int r = 0; r < 32; ++r) {
        float s = 0.f;
#pragma unroll
        for (int d = 0; d < HD; ++d) s = fmaf(q[d], Ks[r][d], s);
        sc[r] = r < nk ? s : -INFINITY;
        mt = fmaxf(mt, sc[r]);
      }
      const float mn = fmaxf(m, mt);
      const float alpha = expf(m - mn);
      l *= alpha;
#pragma unroll
      for (int d = 0; d < HD; ++d) o[d] *= alpha;
#pragma unroll
      for (int r = 0; r < 32; ++r) {
        const float pw = expf(sc[r] - mn);
        l += pw;
#pragma unroll
        for (int d = 0; d < HD; ++d) o[d] = fmaf(pw, Vs[r][d], o[d]);
      }
      m = mn;
    }
    __syncthreads();
  }
  if (active) {
    float* op = out + static_cast<size_t>(row0 + qi) * ldo + head * HD;
    const float inv = 1.f / l;
#pragma unroll
    for (int d = 0; d < HD; ++d) op[d] = o[d] * inv;
  }
}

}  // namespace sg
