// Image -> patch rows: the preprocessing in front of the tower (transformers
// Siglip2ImageProcessor, torchvision backend, image_processing_siglip2.py
// _preprocess): resize each uint8 image to its patch grid times the patch
// size with antialiased bilinear filtering, round to uint8, normalise with
// the rescale factor folded into mean / std, flatten every patch as
// (py, px, channel) and pad to max_patches rows with a 0/1 mask.
//
// 3 channels with 16 x 16 patches (SigLIP-2) take two kernels:
// patchify16x3_kernel, one warp per output row (image b, patch t) of
// pixel_values [B, P, 768], writes the padded rows and the images already at
// their grid size straight from 8-byte loads (HBM-bound); patchify_kernel
// then resizes the others.  Other shapes use patchify_kernel for every row.
// patchify_kernel: one CTA per output row; without a resize every thread
// converts 8 consecutive output elements; with one, the CTA stages the filter taps of its patch's p output rows and
// p output columns, then the horizontal pass over the source rows the patch
// needs (tmp[row][px][c], fp32) in shared memory, then the vertical pass.
// The sums run in the order of torch's antialiased interpolation (for each
// source row the sum over x, then the sum over y), so the rounded uint8
// values agree with torchvision's resize of a uint8 CUDA tensor (cast to
// fp32, interpolate(antialias=True), round half to even).
#pragma once

#include "rowops.cuh"

namespace sg {

constexpr int kPatchifyThreads = 256;
constexpr int kPatchifyMaxTaps = 40;     // filter taps per axis: downscale factor <= 19
constexpr int kPatchifyMaxPatch = 32;    // patch side

struct PatchifyArgs {
  const uint8_t* images;       // all images back to back
  const long long* offsets;    // [B] byte offset of image b
  const int* src_hw;           // [2B] source (H, W)
  const int* grid_hw;          // [2B] patch grid (h, w); the resized image is (h*p, w*p)
  int batch, channels, patch, channels_last, max_patches;
  int max_rows;                // shared-memory rows of tmp (host bound over the batch)
  int resize_only;             // rows of images that need no resize (and padded rows) are written elsewhere
  float mean[4], stdv[4];      // per channel, already in uint8 units (mean / rescale_factor)
};

// Antialiased bilinear taps of output index i for an axis resized in -> out
// (align_corners = False): the triangle filter widened by the downscale
// factor, weights normalised by their sum (the filter definition behind
// torch's antialiased bilinear interpolation).
__device__ __forceinline__ int patchify_taps(int i, int out, int in, float* w, int* lo) {
  const float scale = static_cast<float>(in) / static_cast<float>(out);
  const float support = scale >= 1.f ? scale : 1.f;
  const float inv = scale >= 1.f ? 1.f / scale : 1.f;
  const float center = scale * (static_cast<float>(i) + 0.5f);
  const int a = max(static_cast<int>(center - support + 0.5f), 0);
  const int b = min(static_cast<int>(center + support + 0.5f), in);
  const int n = min(b - a, kPatchifyMaxTaps);
  float tot = 0.f;
  for (int j = 0; j < n; ++j) {
    const float x = fabsf((static_cast<float>(j + a) - center + 0.5f) * inv);
    const float v = x < 1.f ? 1.f - x : 0.f;
    w[j] = v;
    tot += v;
  }
  if (tot != 0.f)
    for (int j = 0; j < n; ++j) w[j] /= tot;
  *lo = a;
  return n;
}

template <typename T>
__device__ __forceinline__ void store8(T* o, const float* f) {
  if constexpr (sizeof(T) == 4) {
    reinterpret_cast<float4*>(o)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(o)[1] = make_float4(f[4], f[5], f[6], f[7]);
  } else {
    store_vec(o, f);
  }
}

template <typename T, int kC, int kP>
__global__ void __launch_bounds__(kPatchifyThreads) patchify_kernel(const PatchifyArgs a, T* __restrict__ out,
                                                                    int* __restrict__ mask) {
  extern __shared__ float psm[];
  const int row = blockIdx.x;  // b * max_patches + t
  const int b = row / a.max_patches;
  const int t = row - b * a.max_patches;
  const int C = kC ? kC : a.channels, p = kP ? kP : a.patch;  // compile-time for the common 3 x 16 x 16
  const int E = p * p * C;     // elements per row, a multiple of 8
  const int h = a.grid_hw[2 * b], w = a.grid_hw[2 * b + 1];
  const bool valid = t < h * w;
  if (a.resize_only && (!valid || (a.src_hw[2 * b] == h * p && a.src_hw[2 * b + 1] == w * p))) return;
  if (threadIdx.x == 0) mask[row] = valid ? 1 : 0;
  T* orow = out + static_cast<size_t>(row) * E;
  if (!valid) {
    const float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int e = threadIdx.x * 8; e < E; e += blockDim.x * 8) store8(orow + e, z);
    return;
  }
  // (v - mean) / std for the 256 uint8 levels: the same fp32 division,
  // looked up (the resized values are rounded to a level first)
  __shared__ float lut[4][256];
  for (int i = threadIdx.x; i < C * 256; i += blockDim.x)
    lut[i >> 8][i & 255] = (static_cast<float>(i & 255) - a.mean[i >> 8]) / a.stdv[i >> 8];
  __syncthreads();
  const int y = t / w, x = t - (t / w) * w;
  const int H = a.src_hw[2 * b], W = a.src_hw[2 * b + 1];
  const int OH = h * p, OW = w * p;
  const uint8_t* img = a.images + a.offsets[b];
  // element (py, px, c) of the patch <- pixel (y*p + py, x*p + px), channel c
  auto src = [&](int c, int sy, int sx) -> int {
    const size_t i = a.channels_last ? (static_cast<size_t>(sy) * W + sx) * C + c
                                     : (static_cast<size_t>(c) * H + sy) * W + sx;
    return img[i];
  };
  if (H == OH && W == OW) {
    for (int e0 = threadIdx.x * 8; e0 < E; e0 += blockDim.x * 8) {
      float f[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int e = e0 + k;
        const int c = e % C, pix = e / C;
        f[k] = lut[c][src(c, y * p + pix / p, x * p + pix % p)];
      }
      store8(orow + e0, f);
    }
    return;
  }
  // ---- resize: taps of the p output rows and columns of this patch
  float* wy = psm;                                   // [p][kPatchifyMaxTaps]
  float* wx = wy + p * kPatchifyMaxTaps;             // [p][kPatchifyMaxTaps]
  int* ly = reinterpret_cast<int*>(wx + p * kPatchifyMaxTaps);  // [p] first tap, then [p] tap count
  int* ny = ly + p;
  int* lx = ny + p;
  int* nx = lx + p;
  float* tmp = reinterpret_cast<float*>(nx + p);     // [max_rows][p][C]
  const int tid = threadIdx.x;
  if (tid < p) {
    ny[tid] = patchify_taps(y * p + tid, OH, H, wy + tid * kPatchifyMaxTaps, &ly[tid]);
  } else if (tid >= 32 && tid < 32 + p) {
    const int j = tid - 32;
    nx[j] = patchify_taps(x * p + j, OW, W, wx + j * kPatchifyMaxTaps, &lx[j]);
  }
  __syncthreads();
  const int r0 = ly[0];
  const int rows = min(ly[p - 1] + ny[p - 1] - r0, a.max_rows);
  // horizontal pass: tmp[r][px][c] = sum_x wx[px][x] * src(c, r0 + r, lx[px] + x)
  for (int i = tid; i < rows * p * C; i += blockDim.x) {
    const int c = i % C, px = (i / C) % p, r = i / (C * p);
    const float* wr = wx + px * kPatchifyMaxTaps;
    float acc = 0.f;
    for (int k = 0; k < nx[px]; ++k) acc = fmaf(wr[k], static_cast<float>(src(c, r0 + r, lx[px] + k)), acc);
    tmp[i] = acc;
  }
  __syncthreads();
  // vertical pass, rounding, normalisation
  for (int e0 = tid * 8; e0 < E; e0 += blockDim.x * 8) {
    float f[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int e = e0 + k;
      const int c = e % C, pix = e / C, py = pix / p, px = pix % p;
      const float* wr = wy + py * kPatchifyMaxTaps;
      const int rb = ly[py] - r0;
      float acc = 0.f;
      for (int j = 0; j < ny[py]; ++j) {
        const int r = rb + j;
        if (r < rows) acc = fmaf(wr[j], tmp[(r * p + px) * C + c], acc);
      }
      // a convex combination of levels: in [0, 255] up to rounding; the clamp
      // only keeps the table index in range
      f[k] = lut[c][min(max(static_cast<int>(rintf(acc)), 0), 255)];
    }
    store8(orow + e0, f);
  }
}

// 3 channels, 16 x 16 patches: one warp per row of pixel_values; lane
// (py, half) converts pixels x*16 + 8*half ... +8 of patch line py, i.e. 24
// consecutive output elements, from 8-byte loads (byte loads where the
// source is not 8-byte aligned).  Writes the padded rows and every row of
// an image already at its grid size; rows of images that need a resize are
// left to patchify_kernel (resize_only).
// One lane's 24 source bytes of row `row` (3 x 16 x 16 patches): returns 0
// for a row left to the resize kernel (or past the end), 1 for a padded row,
// 2 with the bytes in px[] as (pixel, channel).
__device__ __forceinline__ int patch16x3_load(const PatchifyArgs& a, int row, int n_rows, int lane, uint8_t* px) {
  if (row >= n_rows) return 0;
  const int b = row / a.max_patches;
  const int t = row - b * a.max_patches;
  const int h = a.grid_hw[2 * b], w = a.grid_hw[2 * b + 1];
  if (t >= h * w) return 1;
  const int H = a.src_hw[2 * b], W = a.src_hw[2 * b + 1];
  if (H != h * 16 || W != w * 16) return 0;
  const int y = t / w, x = t - (t / w) * w;
  const int oy = y * 16 + (lane >> 1), ox = x * 16 + (lane & 1) * 8;
  const uint8_t* img = a.images + a.offsets[b];
  if (a.channels_last) {
    const uint8_t* sp = img + (static_cast<size_t>(oy) * W + ox) * 3;
    if ((reinterpret_cast<uintptr_t>(sp) & 7) == 0) {
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const uint2 u = reinterpret_cast<const uint2*>(sp)[q];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          px[q * 8 + k] = static_cast<uint8_t>(u.x >> (8 * k));
          px[q * 8 + 4 + k] = static_cast<uint8_t>(u.y >> (8 * k));
        }
      }
    } else {
#pragma unroll
      for (int k = 0; k < 24; ++k) px[k] = sp[k];
    }
  } else {
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const uint8_t* sp = img + (static_cast<size_t>(c) * H + oy) * W + ox;
      if ((reinterpret_cast<uintptr_t>(sp) & 7) == 0) {
        const uint2 u = *reinterpret_cast<const uint2*>(sp);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          px[k * 3 + c] = static_cast<uint8_t>(u.x >> (8 * k));
          px[(4 + k) * 3 + c] = static_cast<uint8_t>(u.y >> (8 * k));
        }
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) px[k * 3 + c] = sp[k];
      }
    }
  }
  return 2;
}

template <typename T>
__device__ __forceinline__ void patch16x3_store(const float (&lut)[3][256], T* out, int* mask, int row, int lane,
                                                int kind, const uint8_t* px) {
  if (kind == 0) return;
  if (lane == 0) mask[row] = kind == 2 ? 1 : 0;
  float f[24];
#pragma unroll
  for (int k = 0; k < 24; ++k) f[k] = kind == 2 ? lut[k % 3][px[k]] : 0.f;
  T* o = out + static_cast<size_t>(row) * 768 + lane * 24;
  store8(o, f);
  store8(o + 8, f + 8);
  store8(o + 16, f + 16);
}

template <typename T>
__global__ void __launch_bounds__(256) patchify16x3_kernel(const PatchifyArgs a, T* __restrict__ out,
                                                           int* __restrict__ mask) {
  __shared__ float lut[3][256];  // (v - mean) / std per channel and uint8 level
  for (int i = threadIdx.x; i < 3 * 256; i += blockDim.x)
    lut[i >> 8][i & 255] = (static_cast<float>(i & 255) - a.mean[i >> 8]) / a.stdv[i >> 8];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int n_rows = a.batch * a.max_patches;
  // persistent: each warp walks rows blockIdx.x * 8 + warp + k * gridDim.x * 8
  for (int row = blockIdx.x * 8 + (threadIdx.x >> 5); row < n_rows; row += gridDim.x * 8) {
    uint8_t px[24];
    const int kind = patch16x3_load(a, row, n_rows, lane, px);
    patch16x3_store(lut, out, mask, row, lane, kind, px);
  }
}

}  // namespace sg
