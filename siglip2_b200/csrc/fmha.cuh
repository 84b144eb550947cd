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
// One CTA per (128-query tile of one image, head):
//   warp 0     TMA: Q once, then K/V tiles of 128 keys into a 3-stage ring
//   warp 1     TMEM owner + MMA issuer:  S_j = Q K_j^T  (128x128, fp32 in TMEM,
//              double-buffered), then O += P_{j-1} V_{j-1}  (128xHDP in TMEM)
//   warps 2-5  softmax: each thread owns one query row (its TMEM lane):
//              masks keys past the image end, online max with lazy rescale
//              (O is rescaled in TMEM only when the running max grows by more
//              than 2^8), P = exp2(S*scale*log2e - m) in bf16/f16 written to a
//              128B-swizzled shared tile, final O / l stored to out[N, H*hd].
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
  static constexpr int kSlabR = 128 * (R > 0 ? R : 16) * 2;
  static constexpr int kSlabRAl = (kSlabR + 1023) / 1024 * 1024;
  static constexpr int kTile = kSlabA + kSlabRAl;    // one 128 x HDP operand
  static constexpr int kStages = 3;
  static constexpr int kQ = 0;
  static constexpr int kK = kTile;
  static constexpr int kV = kK + kStages * kTile;
  static constexpr int kP = kV + kStages * kTile;
  static constexpr int kBar = kP + 2 * kSlabA;       // P: 128 x 128 as two 64-wide slabs
  static constexpr int kSmem = kBar + 256 + 1024;
  static constexpr int kTileBytes = kSlabA + (R > 0 ? 128 * R * 2 : 0);  // TMA bytes per operand
};

template <typename T, int HDP>
__global__ void __launch_bounds__(192, 1)
    fmha_varlen_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmR,
                       const FmhaParams p) {
  using C = FmhaCfg<HDP>;
  constexpr int R = C::R;
  constexpr int ST = C::kStages;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescS = make_idesc(128, 128, kBF16, false, false);
  constexpr uint32_t kIdescO64 = make_idesc(128, 64, kBF16, false, true);
  constexpr uint32_t kIdescOR = make_idesc(128, R > 0 ? R : 16, kBF16, false, true);
  constexpr uint32_t kTmemCols = 512;
  constexpr uint32_t kColO = 256;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBar);
  uint64_t* q_full = bars;            // 1
  uint64_t* kv_full = bars + 1;       // ST
  uint64_t* kv_empty = kv_full + ST;  // ST
  uint64_t* s_full = kv_empty + ST;   // 2
  uint64_t* s_free = s_full + 2;      // 2
  uint64_t* p_full = s_free + 2;      // 1
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
    for (int s = 0; s < ST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    mbar_init(mdone, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
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
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % ST;
        const uint32_t ph = (j / ST) & 1;
        if (*abort_flag || !mbar_wait(&kv_empty[st], ph ^ 1, 201)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* kb = smem + C::kK + st * C::kTile;
        uint8_t* vb = smem + C::kV + st * C::kTile;
        const int kv_row = img_row0 + j * 128;
        mbar_arrive_expect_tx(&kv_full[st], 2 * C::kTileBytes);
        tma_load_2d(kb, &tmA, &kv_full[st], colK, kv_row);
        tma_load_2d(vb, &tmA, &kv_full[st], colV, kv_row);
        if (R > 0) {
          tma_load_2d(kb + C::kSlabA, &tmR, &kv_full[st], colK + 64, kv_row);
          tma_load_2d(vb + C::kSlabA, &tmR, &kv_full[st], colV + 64, kv_row);
        }
        ++issued;
      }
      // no TMA write may still be in flight when the CTA exits
      mbar_wait(q_full, 0, 202);
      for (int j = (issued > ST ? issued - ST : 0); j < issued; ++j)
        mbar_wait(&kv_full[j % ST], (j / ST) & 1, 203);
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------- MMA
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, 211);
      const uint32_t qa = smem_u32(smem + C::kQ);
      const uint32_t qr = qa + C::kSlabA;
      auto issue_pv = [&](int jj) {
        const int st = jj % ST;
        const uint32_t va = smem_u32(smem + C::kV + st * C::kTile);
        const uint32_t vr = va + C::kSlabA;
        const uint32_t pa = smem_u32(smem + C::kP);
#pragma unroll
        for (int s = 0; s < 8; ++s) {  // 16 keys per MMA
          const uint64_t adesc = kmajor_desc(pa + (s >> 2) * C::kSlabA + (s & 3) * 32, 128);
          const uint32_t acc = (jj > 0 || s > 0) ? 1u : 0u;
          umma_ss(tmem + kColO, adesc, mnmajor_desc(va + s * 16 * 128, 128, 0), kIdescO64, acc);
          if constexpr (R > 0) umma_ss(tmem + kColO + 64, adesc, mnmajor_desc(vr + s * 16 * R * 2, R * 2, 0),
                                       kIdescOR, acc);
        }
        umma_commit(pv_done);
        umma_commit(&kv_empty[st]);
      };
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j % ST;
        const int sb = j & 1;
        if (*abort_flag || !mbar_wait(&kv_full[st], (j / ST) & 1, 212) ||
            !mbar_wait(&s_free[sb], ((j >> 1) & 1) ^ 1, 213)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ka = smem_u32(smem + C::kK + st * C::kTile);
        const uint32_t kr = ka + C::kSlabA;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_ss(tmem + sb * 128, kmajor_desc(qa + k * 32, 128), kmajor_desc(ka + k * 32, 128), kIdescS, k > 0);
#pragma unroll
        for (int k = 0; k < R / 16; ++k)
          umma_ss(tmem + sb * 128, kmajor_desc(qr + k * 32, R * 2), kmajor_desc(kr + k * 32, R * 2), kIdescS, 1);
        umma_commit(&s_full[sb]);
        if (j > 0) {
          if (!mbar_wait(p_full, (j - 1) & 1, 214)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(j - 1);
        }
      }
      if (ok && n_kv > 0) {
        if (mbar_wait(p_full, (n_kv - 1) & 1, 215)) {
          tc_fence_after();
          issue_pv(n_kv - 1);
        } else {
          ok = false;
        }
      }
      if (!ok) *abort_flag = 1;
      umma_commit(mdone);
      mbar_wait(mdone, 0, 216);
    }
  } else {
    // --------------------------------------------------------------- softmax + epilogue
    const int q = warp & 3;  // TMEM lane quarter of this warp
    const int r = q * 32 + lane;  // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    uint8_t* P = smem + C::kP;
    float m_use = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int sb = j & 1;
      if (*abort_flag || !mbar_wait(&s_full[sb], (j >> 1) & 1, 221)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[128];
      {
        uint32_t u[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          SG_TMEM_LD_32(tmem + sb * 128 + c * 32 + lane_off, u);
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 32; ++k) s[c * 32 + k] = __uint_as_float(u[k]);
        }
      }
      tc_fence_before();
      mbar_arrive(&s_free[sb]);
      const int valid = L - j * 128;  // keys of this image in the tile (>= 1)
      float mt = -INFINITY;
#pragma unroll
      for (int k = 0; k < 128; ++k) {
        s[k] = k < valid ? s[k] * p.scale_log2 : -INFINITY;
        mt = fmaxf(mt, s[k]);
      }
      float alpha = 1.f;
      if (j == 0) {
        m_use = mt;
      } else if (mt > m_use + 8.f) {
        alpha = ex2_approx(m_use - mt);
        m_use = mt;
      }
      float rs = 0.f;
#pragma unroll
      for (int k = 0; k < 128; ++k) {
        s[k] = ex2_approx(s[k] - m_use);
        rs += s[k];
      }
      l = l * alpha + rs;
      if (j > 0) {
        // PV_{j-1} must be done: O is about to be rescaled and P overwritten
        if (!mbar_wait(pv_done, (j - 1) & 1, 222)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
          uint32_t u[16];
#pragma unroll
          for (int c = 0; c < HDP / 16; ++c) {
            SG_TMEM_LD_16(tmem + kColO + c * 16 + lane_off, u);
            tmem_ld_wait();
#pragma unroll
            for (int k = 0; k < 16; ++k) u[k] = __float_as_uint(__uint_as_float(u[k]) * alpha);
            SG_TMEM_ST_16(tmem + kColO + c * 16 + lane_off, u);
          }
          tmem_st_wait();
        }
      }
      // P row r -> two 64-key slabs, 128B swizzle (16B chunk c ^ (r & 7))
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        uint4 v;
        v.x = Pack2<T>::pack(s[c * 8 + 0], s[c * 8 + 1]);
        v.y = Pack2<T>::pack(s[c * 8 + 2], s[c * 8 + 3]);
        v.z = Pack2<T>::pack(s[c * 8 + 4], s[c * 8 + 5]);
        v.w = Pack2<T>::pack(s[c * 8 + 6], s[c * 8 + 7]);
        const int slab = c >> 3, cc = c & 7;
        *reinterpret_cast<uint4*>(P + slab * C::kSlabA + r * 128 + ((cc ^ (r & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
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
        SG_TMEM_LD_16(tmem + kColO + c * 16 + lane_off, u);
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
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace sg
