// Persistent warp-specialised tcgen05 GEMM for the tower's dense projections:
//
//     out[M, N] = epilogue( A[M, K] . B[N, K]^T )        (A, B row-major, K-major)
//
// One CTA per SM walks a static list of 128 x BN output tiles.  Warp roles:
//   warp 0      TMA producer: A/B tiles (128B swizzle, 64-wide K slabs) into a
//               STAGES-deep shared-memory ring, one mbarrier per stage.
//   warp 1      TMEM owner + UMMA issuer (one elected lane): 4 x
//               tcgen05.mma 128xBNx16 per stage into one of two TMEM
//               accumulators (2 x 256 columns), tcgen05.commit frees the
//               stage / publishes the accumulator.
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time (each warp owns the
//               32 TMEM lanes = rows its warp index allows), fused epilogue,
//               16-byte global stores.  Runs one tile behind the MMA.
//   warps 6-9   (LayerNorm-folded variants only) row statistics: each thread
//               owns one row of the A tile and accumulates shifted sum / sum
//               of squares straight from the swizzled stage while the MMA
//               consumes it, so LayerNorm costs no extra pass over HBM.
//
// LayerNorm folding.  For y = LN(x) = (x - mu) * rstd * gamma + beta feeding a
// Linear(W, b):   y W^T + b = rstd * (x (W*gamma)^T - mu * c1) + c2
// with c1[n] = sum_k (W*gamma)[n,k] and c2[n] = b[n] + sum_k beta[k] W[n,k].
// The GEMM runs on the raw residual stream x against the pre-scaled weight
// W*gamma; mu and rstd come from the statistics warps; the epilogue applies
// the row/column terms in fp32.
#pragma once

#include "ptx.cuh"

namespace sg {

enum GemmEpilogue : int {
  kEpiBias = 0,        // out = acc + bias
  kEpiBiasRes = 1,     // out = acc + bias + res
  kEpiLn = 2,          // out = rstd (acc - mu c1) + c2
  kEpiLnGelu = 3,      // out = gelu_tanh(rstd (acc - mu c1) + c2)
  kEpiBiasGelu = 4,    // out = gelu_tanh(acc + bias)
};

struct GemmParams {
  int M, N, K;
  void* out;             // [M, ldo] (element type T)
  int ldo;               // elements
  const float* bias;     // [N] (kEpiBias*, kEpiBiasRes)
  const void* res;       // [M, ldr] element type T (kEpiBiasRes); may alias out
  int ldr;
  const float* c1;       // [N] (kEpiLn*)
  const float* c2;       // [N] (kEpiLn*)
  float eps;             // LayerNorm epsilon (kEpiLn*)
};

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;  // 64 x 2B = one 128-byte swizzle row

template <int BN>
struct GemmCfg {
  static constexpr int kStageA = kGemmBM * kGemmBK * 2;
  static constexpr int kStageB = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kStageA + kStageB;
  static constexpr int kStages = (200 * 1024) / kStageBytes;  // 4 for BN=256, 5 for BN=192
  static constexpr int kTmemCols = 512;                        // 2 accumulators, 256-column slots
  static constexpr int kAccStride = 256;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 1024 /*barriers+stats*/ +
                                    2 * 2 * kGemmBM * 4;
};

template <bool LN>
struct GemmThreads {
  static constexpr int kWarps = LN ? 10 : 6;
  static constexpr int kThreads = kWarps * 32;
};

template <typename T, int BN, int EPI>
__global__ void __launch_bounds__(GemmThreads<(EPI == kEpiLn || EPI == kEpiLnGelu)>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmParams p) {
  constexpr bool kLN = (EPI == kEpiLn || EPI == kEpiLnGelu);
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::kStages;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdesc = make_idesc(kGemmBM, BN, kBF16, false, false);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + STAGES * Cfg::kStageA;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::kStageBytes);
  uint64_t* full = bars;                 // [STAGES]
  uint64_t* empty = bars + STAGES;       // [STAGES]
  uint64_t* tfull = bars + 2 * STAGES;   // [2]
  uint64_t* tempty = tfull + 2;          // [2]
  uint64_t* sfull = tempty + 2;          // [2]
  uint64_t* sempty = sfull + 2;          // [2]
  uint64_t* mdone = sempty + 2;          // [1] all issued MMAs complete (teardown)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mdone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* st_mean = reinterpret_cast<float*>(smem + STAGES * Cfg::kStageBytes + 1024);  // [2][128]
  float* st_rstd = st_mean + 2 * kGemmBM;                                               // [2][128]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = (p.M + kGemmBM - 1) / kGemmBM;
  const int n_tiles = (p.N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int nk = (p.K + kGemmBK - 1) / kGemmBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kLN ? 5 : 1);  // MMA commit (+ one arrive per statistics warp)
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
      mbar_init(&sfull[b], kGemmBM);
      mbar_init(&sempty[b], 4);
    }
    mbar_init(mdone, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile / n_tiles) * kGemmBM;
        const int n0 = (tile % n_tiles) * BN;
        for (int kb = 0; kb < nk; ++kb) {
          if (*abort_flag || !mbar_wait(&empty[stage], phase ^ 1, 101)) {
            ok = false;
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
          tma_load_2d(smA + stage * Cfg::kStageA, &tmA, &full[stage], kb * kGemmBK, m0);
          tma_load_2d(smB + stage * Cfg::kStageB, &tmB, &full[stage], kb * kGemmBK, n0);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Tail: make sure no TMA write is still in flight into this CTA's shared
      // memory when it exits (wait until the consumers released every stage,
      // which implies the loads landed).
      for (int i = 0; i < STAGES && i < issued; ++i) {
        if (!mbar_wait(&empty[stage], phase ^ 1, 102)) {
          // consumers gave up: wait for this slot's last load itself instead
          mbar_wait(&full[stage], phase ^ 1, 103);
        }
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int t = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++t) {
        const int buf = t & 1;
        const uint32_t tph = (t >> 1) & 1;
        if (*abort_flag || !mbar_wait(&tempty[buf], tph ^ 1, 111)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * Cfg::kAccStride;
        for (int kb = 0; kb < nk; ++kb) {
          if (*abort_flag || !mbar_wait(&full[stage], phase, 112)) {
            ok = false;
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smA + stage * Cfg::kStageA);
          const uint32_t b_base = smem_u32(smB + stage * Cfg::kStageB);
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) {
            umma_ss(d_tmem, kmajor_desc(a_base + k * 32, 128), kmajor_desc(b_base + k * 32, 128), kIdesc,
                    (kb | k) != 0);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[buf]);
      }
      // TMEM is released at teardown: first let every issued MMA finish (on the
      // normal path this is already implied by the epilogue's last wait).
      umma_commit(mdone);
      mbar_wait(mdone, 0, 113);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    int t = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++t) {
      const int buf = t & 1;
      const uint32_t tph = (t >> 1) & 1;
      const int m0 = (tile / n_tiles) * kGemmBM;
      const int n0 = (tile % n_tiles) * BN;
      if (*abort_flag || !mbar_wait(&tfull[buf], tph, 121)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      float mu = 0.f, rstd = 1.f;
      if constexpr (kLN) {
        if (!mbar_wait(&sfull[buf], tph, 122)) {
          *abort_flag = 1;
          break;
        }
        mu = st_mean[buf * kGemmBM + row_in_tile];
        rstd = st_rstd[buf * kGemmBM + row_in_tile];
        __syncwarp();
        if (lane == 0) mbar_arrive(&sempty[buf]);
      }
      const int row = m0 + row_in_tile;
      const bool row_ok = row < p.M;
      T* out_row = reinterpret_cast<T*>(p.out) + static_cast<size_t>(row) * p.ldo;
      const T* res_row = nullptr;
      if constexpr (EPI == kEpiBiasRes) res_row = reinterpret_cast<const T*>(p.res) + static_cast<size_t>(row) * p.ldr;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        const uint32_t taddr = tmem_base + buf * Cfg::kAccStride + c * 32 + (static_cast<uint32_t>(q * 32) << 16);
        SG_TMEM_LD_32(taddr, r);
        tmem_ld_wait();
        const int col0 = n0 + c * 32;
        if (col0 >= p.N) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if constexpr (EPI == kEpiLn || EPI == kEpiLnGelu) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int col = min(col0 + j, p.N - 1);
            v[j] = rstd * (v[j] - mu * __ldg(p.c1 + col)) + __ldg(p.c2 + col);
            if constexpr (EPI == kEpiLnGelu) v[j] = gelu_tanh(v[j]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int col = min(col0 + j, p.N - 1);
            v[j] += __ldg(p.bias + col);
            if constexpr (EPI == kEpiBiasGelu) v[j] = gelu_tanh(v[j]);
          }
        }
        if (row_ok) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int col = col0 + g * 8;
            if (col < p.N) {  // N is a multiple of 8: a 16-byte group is all in or all out
              if constexpr (EPI == kEpiBiasRes) {
                const uint4 rv = *reinterpret_cast<const uint4*>(res_row + col);
                const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                  const float2 f = Pack2<T>::unpack(rw[h]);
                  v[g * 8 + 2 * h] += f.x;
                  v[g * 8 + 2 * h + 1] += f.y;
                }
              }
              uint4 o;
              o.x = Pack2<T>::pack(v[g * 8 + 0], v[g * 8 + 1]);
              o.y = Pack2<T>::pack(v[g * 8 + 2], v[g * 8 + 3]);
              o.z = Pack2<T>::pack(v[g * 8 + 4], v[g * 8 + 5]);
              o.w = Pack2<T>::pack(v[g * 8 + 6], v[g * 8 + 7]);
              *reinterpret_cast<uint4*>(out_row + col) = o;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
  } else {
    // ------------------------------------------------------------ LayerNorm row statistics
    if constexpr (kLN) {
      const int r = threadIdx.x - 6 * 32;  // 0..127: row within the tile
      int stage = 0;
      uint32_t phase = 0;
      int t = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++t) {
        const int buf = t & 1;
        const uint32_t tph = (t >> 1) & 1;
        if (*abort_flag || !mbar_wait(&sempty[buf], tph ^ 1, 131)) {
          *abort_flag = 1;
          break;
        }
        float shift = 0.f, s1 = 0.f, s2 = 0.f;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (*abort_flag || !mbar_wait(&full[stage], phase, 132)) {
            ok = false;
            *abort_flag = 1;
            break;
          }
          const uint8_t* rowp = smA + stage * Cfg::kStageA + r * 128;
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            // the 128B swizzle only permutes 16B chunks within the row, and the
            // sum does not care about their order
            const uint4 u = *reinterpret_cast<const uint4*>(rowp + ch * 16);
            const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const float2 f = Pack2<T>::unpack(w4[h]);
              if (kb == 0 && ch == 0 && h == 0) shift = f.x;
              const float a = f.x - shift, b = f.y - shift;
              s1 += a + b;
              s2 = fmaf(a, a, s2);
              s2 = fmaf(b, b, s2);
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        const float inv_k = 1.0f / static_cast<float>(p.K);
        const float m1 = s1 * inv_k;
        const float var = fmaxf(s2 * inv_k - m1 * m1, 0.f);
        st_mean[buf * kGemmBM + r] = shift + m1;
        st_rstd[buf * kGemmBM + r] = rsqrtf(var + p.eps);
        mbar_arrive(&sfull[buf]);
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

}  // namespace sg
