// Variable-length (per-image) attention on tcgen05 for the packed NaFlex
// sequence: every query row attends only to the keys of its own image, i.e.
// the block-diagonal document mask of the reference, with no padded rows.
//
// Input: the QKV projection output [N, 3*H*HDP] in the head-padded layout the
// QKV GEMM writes: column (which*H + h)*HDP + d holds q/k/v[which] of head h,
// dim d; columns d >= head_dim are exact zeros (zero weight rows), so padding
// the head dimension to HDP changes no dot product.  HDP = 64 | 80 | 96
// (head_dim 64 | 72 | 96), split into a 64-wide slab (128B swizzle) plus an
// R = HDP-64 wide slab (32B / 64B swizzle).
//
// One CTA per (128-query tile of one image, head); two CTAs share an SM
// (256 TMEM columns and <= 96 KB of shared memory each), so one CTA's MMAs run
// while the other's softmax warps work.
//   warp 0     TMA: Q once, K tiles of 128 keys into a 2-deep ring, V tiles
//   warp 1     TMEM owner + MMA issuer:
//                S_j = Q K_j^T          128x128 fp32 in TMEM columns [0,128)
//                O  += P_j V_j          P_j (bf16/f16) read from TMEM columns
//                                       [0,64) where the softmax wrote it over
//                                       S_j; O (128 x HDP fp32) in [128, 128+HDP)
//   warps 2-5  softmax: each thread owns one query row (its TMEM lane):
//              keys past the image end masked, online max with lazy rescale
//              (O is rescaled in TMEM only when the running max grows by more
//              than 2^8), P = exp2(S*scale*log2e - m) packed in pairs into
//              TMEM, final O / l stored to out[N, H*hd].
#pragma once

#include "ptx.cuh"

namespace sg {

struct FmhaParams {
  const int* cu;      // [B+1] first row of each image in the packed sequence
  const int2* tiles;  // [n_tiles] (image, query-tile index)
  int heads;
  int head_dim;
  void* out;          // [N, heads*head_dim]
  int ld_out;
  float scale_log2;   // head_dim^-0.5 * log2(e)
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int HDP>
struct FmhaCfg {
  static constexpr int R = HDP - 64;                 // remainder slab width (0, 16, 32)
  static constexpr int kSlabA = 128 * 64 * 2;        // 16 KB
  static constexpr int kSlabR = 128 * R * 2;
  static constexpr int kSlabRAl = (kSlabR + 1023) / 1024 * 1024;
  static constexpr int kTile = kSlabA + kSlabRAl;    // one 128 x HDP operand
  static constexpr int kKStages = 2;
  static constexpr int kQ = 0;
  static constexpr int kK = kTile;
  static constexpr int kV = kK + kKStages * kTile;
  static constexpr int kBar = kV + kTile;
  static constexpr int kSmem = kBar + 256 + 1024;
  static constexpr int kTileBytes = kSlabA + kSlabR;  // TMA bytes per operand tile
  static constexpr uint32_t kTmemCols = 256;
  static constexpr uint32_t kColO = 128;
};

template <typename T, int HDP>
__global__ void __launch_bounds__(192, 2)
    fmha_varlen_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmR,
                       const FmhaParams p) {
  using C = FmhaCfg<HDP>;
  constexpr int R = C::R;
  constexpr int KS = C::kKStages;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescS = make_idesc(128, 128, kBF16, false, false);
  constexpr uint32_t kIdescO64 = make_idesc(128, 64, kBF16, false, true);
  constexpr uint32_t kIdescOR = make_idesc(128, R > 0 ? R : 16, kBF16, false, true);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBar);
  uint64_t* q_full = bars;            // 1
  uint64_t* k_full = bars + 1;        // KS
  uint64_t* k_empty = k_full + KS;    // KS
  uint64_t* v_full = k_empty + KS;    // 1
  uint64_t* v_empty = v_full + 1;     // 1
  uint64_t* s_full = v_empty + 1;     // 1
  uint64_t* p_full = s_full + 1;      // 1
  uint64_t* pv_done = p_full + 1;     // 1
  uint64_t* mdone = pv_done + 1;      // 1
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mdone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int2 tile = p.tiles[blockIdx.x];
  const int head = blockIdx.y;
  const int img_row0 = __ldg(p.cu + tile.x);
  const int L = __ldg(p.cu + tile.x + 1) - img_row0;
  const int q_row0 = img_row0 + tile.y * 128;
  const int n_kv = (L + 127) / 128;
  const int colQ = head * HDP;
  const int colK = (p.heads + head) * HDP;
  const int colV = (2 * p.heads + head) * HDP;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    mbar_init(mdone, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // --------------------------------------------------------------- TMA
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      if (R > 0) tma_prefetch_desc(&tmR);
      mbar_arrive_expect_tx(q_full, C::kTileBytes);
      tma_load_2d(smem + C::kQ, &tmA, q_full, colQ, q_row0);
      if (R > 0) tma_load_2d(smem + C::kQ + C::kSlabA, &tmR, q_full, colQ + 64, q_row0);
      int k_issued = 0, v_issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int ks = j % KS;
        const int kv_row = img_row0 + j * 128;
        if (*abort_flag || !mbar_wait(&k_empty[ks], ((j / KS) & 1) ^ 1, 201)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* kb = smem + C::kK + ks * C::kTile;
        mbar_arrive_expect_tx(&k_full[ks], C::kTileBytes);
        tma_load_2d(kb, &tmA, &k_full[ks], colK, kv_row);
        if (R > 0) tma_load_2d(kb + C::kSlabA, &tmR, &k_full[ks], colK + 64, kv_row);
        ++k_issued;
        if (*abort_flag || !mbar_wait(v_empty, (j & 1) ^ 1, 202)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* vb = smem + C::kV;
        mbar_arrive_expect_tx(v_full, C::kTileBytes);
        tma_load_2d(vb, &tmA, v_full, colV, kv_row);
        if (R > 0) tma_load_2d(vb + C::kSlabA, &tmR, v_full, colV + 64, kv_row);
        ++v_issued;
      }
      // no TMA write may still be in flight when the CTA exits
      mbar_wait(q_full, 0, 203);
      for (int j = (k_issued > KS ? k_issued - KS : 0); j < k_issued; ++j)
        mbar_wait(&k_full[j % KS], (j / KS) & 1, 204);
      if (v_issued > 0) mbar_wait(v_full, (v_issued - 1) & 1, 205);
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------- MMA
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, 211);
      const uint32_t qa = smem_u32(smem + C::kQ);
      const uint32_t qr = qa + C::kSlabA;
      const uint32_t va = smem_u32(smem + C::kV);
      const uint32_t vr = va + C::kSlabA;
      for (int j = 0; j < n_kv && ok; ++j) {
        const int ks = j % KS;
        // S/P columns are reused: PV_{j-1} must have consumed P_{j-1}
        if (*abort_flag || !mbar_wait(&k_full[ks], (j / KS) & 1, 212) ||
            (j > 0 && !mbar_wait(pv_done, (j - 1) & 1, 213))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ka = smem_u32(smem + C::kK + ks * C::kTile);
        const uint32_t kr = ka + C::kSlabA;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_ss(tmem, kmajor_desc(qa + k * 32, 128), kmajor_desc(ka + k * 32, 128), kIdescS, k > 0);
#pragma unroll
        for (int k = 0; k < R / 16; ++k)
          umma_ss(tmem, kmajor_desc(qr + k * 32, R * 2), kmajor_desc(kr + k * 32, R * 2), kIdescS, 1);
        umma_commit(s_full);
        umma_commit(&k_empty[ks]);
        if (!mbar_wait(p_full, j & 1, 214) || !mbar_wait(v_full, j & 1, 215)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int s = 0; s < 8; ++s) {  // 16 keys per MMA; P columns [8s, 8s+8)
          const uint32_t acc = (j > 0 || s > 0) ? 1u : 0u;
          umma_ts(tmem + C::kColO, tmem + s * 8, mnmajor_desc(va + s * 16 * 128, 128, 0), kIdescO64, acc);
          if constexpr (R > 0)
            umma_ts(tmem + C::kColO + 64, tmem + s * 8, mnmajor_desc(vr + s * 16 * R * 2, R * 2, 0), kIdescOR, acc);
        }
        umma_commit(pv_done);
        umma_commit(v_empty);
      }
      if (!ok) *abort_flag = 1;
      umma_commit(mdone);
      mbar_wait(mdone, 0, 216);
    }
  } else {
    // --------------------------------------------------------------- softmax + epilogue
    const int q = warp & 3;       // TMEM lane quarter of this warp
    const int r = q * 32 + lane;  // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const float sc = p.scale_log2;
    float m_use = 0.f, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (*abort_flag || !mbar_wait(s_full, j & 1, 221)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int valid = L - j * 128;  // keys of this image in the tile (>= 1)
      // pass 1: row max of S_j (32 columns at a time)
      // 8 independent partial maxima (no long dependency chain); keys past
      // the image end are masked only in the image's last, partial tile
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx[i] = -INFINITY;
      const bool full_tile = valid >= 128;
#pragma unroll 1
      for (int c = 0; c < 4; c += 2) {
        uint32_t u[32], u2[32];
        SG_TMEM_LD_32(tmem + c * 32 + lane_off, u);
        SG_TMEM_LD_32(tmem + (c + 1) * 32 + lane_off, u2);
        tmem_ld_wait();
        if (full_tile) {
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            mx[k & 7] = fmaxf(mx[k & 7], __uint_as_float(u[k]));
            mx[k & 7] = fmaxf(mx[k & 7], __uint_as_float(u2[k]));
          }
        } else {
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            if (c * 32 + k < valid) mx[k & 7] = fmaxf(mx[k & 7], __uint_as_float(u[k]));
            if ((c + 1) * 32 + k < valid) mx[k & 7] = fmaxf(mx[k & 7], __uint_as_float(u2[k]));
          }
        }
      }
      float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      mt *= sc;
      float alpha = 1.f;
      if (j == 0) {
        m_use = mt;
      } else if (mt > m_use + 8.f) {
        alpha = ex2_approx(m_use - mt);
        m_use = mt;
      }
      // O is stable here: S_j was issued only after PV_{j-1} completed
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        uint32_t u[16];
#pragma unroll
        for (int c = 0; c < HDP / 16; ++c) {
          SG_TMEM_LD_16(tmem + C::kColO + c * 16 + lane_off, u);
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 16; ++k) u[k] = __float_as_uint(__uint_as_float(u[k]) * alpha);
          SG_TMEM_ST_16(tmem + C::kColO + c * 16 + lane_off, u);
        }
      }
      // pass 2: P = exp2(S*scale - m) written over S_j: P column 16c+k holds
      // keys 32c+2k (low half) and 32c+2k+1; chunk c only overwrites columns
      // of chunks already read
      float ps[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) ps[i] = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t u[32];
        SG_TMEM_LD_32(tmem + c * 32 + lane_off, u);
        tmem_ld_wait();
        uint32_t w[16];
        if (full_tile) {
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float p0 = ex2_approx(fmaf(__uint_as_float(u[2 * k]), sc, -m_use));
            const float p1 = ex2_approx(fmaf(__uint_as_float(u[2 * k + 1]), sc, -m_use));
            ps[k & 7] += p0 + p1;
            w[k] = Pack2<T>::pack(p0, p1);
          }
        } else {
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const int k0 = c * 32 + 2 * k;
            const float x0 = k0 < valid ? __uint_as_float(u[2 * k]) : -INFINITY;
            const float x1 = k0 + 1 < valid ? __uint_as_float(u[2 * k + 1]) : -INFINITY;
            const float p0 = ex2_approx(fmaf(x0, sc, -m_use));
            const float p1 = ex2_approx(fmaf(x1, sc, -m_use));
            ps[k & 7] += p0 + p1;
            w[k] = Pack2<T>::pack(p0, p1);
          }
        }
        SG_TMEM_ST_16(tmem + c * 16 + lane_off, w);
      }
      const float rs = ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
      l = l * alpha + rs;
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && n_kv > 0 && mbar_wait(pv_done, (n_kv - 1) & 1, 223)) {
      tc_fence_after();
      const int row = q_row0 + r;
      const bool row_ok = (tile.y * 128 + r) < L;
      const float inv_l = 1.f / l;
      T* orow = reinterpret_cast<T*>(p.out) + static_cast<size_t>(row) * p.ld_out + head * p.head_dim;
#pragma unroll
      for (int c = 0; c < HDP / 16; ++c) {
        uint32_t u[16];
        SG_TMEM_LD_16(tmem + C::kColO + c * 16 + lane_off, u);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            const int d0 = c * 16 + g * 8;
            if (d0 < p.head_dim) {  // head_dim is a multiple of 8
              uint4 o;
              o.x = Pack2<T>::pack(__uint_as_float(u[g * 8 + 0]) * inv_l, __uint_as_float(u[g * 8 + 1]) * inv_l);
              o.y = Pack2<T>::pack(__uint_as_float(u[g * 8 + 2]) * inv_l, __uint_as_float(u[g * 8 + 3]) * inv_l);
              o.z = Pack2<T>::pack(__uint_as_float(u[g * 8 + 4]) * inv_l, __uint_as_float(u[g * 8 + 5]) * inv_l);
              o.w = Pack2<T>::pack(__uint_as_float(u[g * 8 + 6]) * inv_l, __uint_as_float(u[g * 8 + 7]) * inv_l);
              *reinterpret_cast<uint4*>(orow + d0) = o;
            }
          }
        }
      }
    } else if (!ok) {
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

}  // namespace sg
