// Persistent warp-specialised tcgen05 GEMM for the tower's dense projections:
//
//     out[M, N] = epilogue( A[M, K] . B[N, K]^T )        (A, B row-major, K-major)
//
// One CTA per SM (gemm_tc_kernel, 128 x BN tiles) or one CTA pair per two SMs
// (gemm_tc2_kernel, 256 x BN tiles, tcgen05 cta_group::2) walks a static
// list of output tiles.  Warp roles:
//   warp 0      TMA producer: A/B tiles (128B swizzle, 64-wide K slabs, SUB
//               slabs per stage) into a STAGES-deep shared-memory ring.
//   warp 1      TMEM owner + UMMA issuer (one elected lane): 4 * SUB
//               tcgen05.mma per stage into one of two TMEM accumulators
//               (2 x 256 columns); tcgen05.commit frees the stage and
//               publishes the accumulator.
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time (each warp owns the
//               32 TMEM lanes its warp index allows), fused math in fp32,
//               64B-swizzled staging, TMA stores.  Runs one tile behind the
//               MMA; the next tile's parameters, row sums and residual are
//               prefetched while the current one drains.
//   warps 6-9   (kEpiLn / kEpiLnGelu only) row statistics of the A tiles,
//               read from the swizzled stages while the MMA consumes them.
//
// LayerNorm folding.  For y = LN(x) = (x - mu) * rstd * gamma + beta feeding a
// Linear(W, b):   y W^T + b = rstd * (x (W*gamma)^T - mu * c1) + c2
// with c1[n] = sum_k (W*gamma)[n,k] and c2[n] = b[n] + sum_k beta[k] W[n,k].
// The GEMM runs on the raw residual stream x against the pre-scaled weight
// W*gamma; mu and rstd come either from the statistics warps or (kEpiLnRs*)
// from per-column-block slot statistics (mean, centred sum of squares; see
// rowops.cuh) that the GEMM which produced x wrote in its own epilogue
// (kEpiBiasResRs / kEpiBiasPosRs).
#pragma once

#include "rowops.cuh"

namespace sg {

enum GemmEpilogue : int {
  kEpiBias = 0,          // out = acc + bias
  kEpiBiasRes = 1,       // out = acc + bias + res
  kEpiLn = 2,            // out = rstd (acc - mu c1) + c2, mu/rstd from statistics warps
  kEpiLnGelu = 3,        // out = gelu_tanh(rstd (acc - mu c1) + c2), likewise
  kEpiBiasGelu = 4,      // out = gelu_tanh(acc + bias)
  kEpiLnRs = 5,          // as kEpiLn, mu/rstd from row sums accumulated by the producer of A
  kEpiLnRsGelu = 6,      // as kEpiLnGelu, likewise
  kEpiBiasResRs = 7,     // as kEpiBiasRes, and accumulates the row sums of the rounded output
  kEpiBiasPosRs = 8,     // out = acc + bias + resized position embedding of the row's token, + row sums
  kEpiBiasGeluGrad = 9,  // out = res * gelu_tanh'(acc + bias): the GELU backward fused into the GEMM that
                         // recomputes the pre-activation (res = the incoming gradient)
};

__host__ __device__ constexpr bool epi_has_stat_warps(int e) { return e == kEpiLn || e == kEpiLnGelu; }
__host__ __device__ constexpr bool epi_is_ln(int e) { return e == kEpiLn || e == kEpiLnGelu || e == kEpiLnRs || e == kEpiLnRsGelu; }
__host__ __device__ constexpr bool epi_is_gelu(int e) { return e == kEpiLnGelu || e == kEpiLnRsGelu || e == kEpiBiasGelu; }
__host__ __device__ constexpr bool epi_has_res(int e) {
  return e == kEpiBiasRes || e == kEpiBiasResRs || e == kEpiBiasGeluGrad;
}

struct GemmParams {
  int M, N, K;
  const float* bias;          // [N] (bias epilogues)
  const float* c1;            // [N] (LayerNorm-folded epilogues)
  const float* c2;            // [N]
  float eps;                  // LayerNorm epsilon
  // Row statistics in slots: [M][rs_ld] (mean, centred sum of squares) pairs,
  // slot j covering the j-th column block of the GEMM that produced the rows
  // (see rowsum_block); each slot is written exactly once and merged in slot
  // order, so the LayerNorm statistics (and the forward) are deterministic.
  const float2* rs_in;        // A's row sums over K (kEpiLnRs*), rs_ld slots per row
  float2* rs_acc;             // output row sums to write (kEpiBiasResRs, kEpiBiasPosRs), rs_ld slots per row
  int rs_ld;
  // kEpiBiasPosRs: row t is a token of image tok_img[t] at (y, x) of its
  // (h, w) = pos_hw[2b], pos_hw[2b+1] grid (t - cu[b] = y * w + x); the
  // position embedding is the antialiased bilinear resize of the
  // pos_grid x pos_grid fp32 table [pos_grid^2, N] evaluated there
  const float* pos_table;
  int pos_grid;
  const int* tok_img;
  const int* pos_hw;
  const int* cu;
  // 8-bit operands (gemm_tc2_kernel<..., kF8>): the accumulator of row m,
  // column n is a_scale[m] * b_scale[n] times the product of the stored
  // e4m3 values (per-row scales of A, per-output-channel scales of B)
  const float* a_scale;
  const float* b_scale;
  // split K (gemm_tc_kernel<..., kSplitK>): k_splits slices of k_per_split
  // (a multiple of 128) K-elements each, slice s writes its fp32 partial
  // product to part + s * M * ld_part; splitk_reduce_kernel sums them
  int k_splits;
  int k_per_split;
  float* part;
  int ld_part;
};

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;     // 64 x 2B = one 128-byte swizzle row
constexpr int kEpiCols = 32;    // epilogue chunk: 32 columns = one 64B-swizzled staging row
constexpr int kEpiBufs = 2;     // staging buffers per epilogue warp
constexpr int kEpiBufBytes = 32 * kEpiCols * 2;
constexpr int kSmemLimit = 227 * 1024;
constexpr int kGemmThreads = 320;  // 10 warps: producer, MMA, 8 epilogue (or 4 epilogue + 4 statistics)

// Epilogue warps: two per TMEM lane quarter (each drains half of the tile's
// columns) so that two warps per SM sub-partition hide each other's
// latencies; the statistics-warp variants keep one per quarter.
__host__ __device__ constexpr int epi_warps(int e) { return epi_has_stat_warps(e) ? 4 : 8; }

// Tile width of the tensor-core GEMM: 256 columns (the widest MMA; it moves
// the fewest operand bytes per FLOP).  The CTA-pair kernel runs a narrower
// last column tile at its own width, so N need not be a multiple of 256.
__host__ __device__ constexpr int gemm_bn_for(int) { return 256; }
// Column block of one row-sum slot: the columns one epilogue warp drains of
// a row-sum-producing tile (half the tile), or the SIMT fp32 tile width.
__host__ __device__ constexpr int rowsum_block(bool f32, int N) { return f32 ? kRowSumBlock : gemm_bn_for(N) / 2; }
static_assert(gemm_bn_for(1) / 2 == kRowSumBlock, "slot width of the tensor-core epilogue");
__host__ __device__ constexpr int rowsum_slots(bool f32, int N) {
  return (N + rowsum_block(f32, N) - 1) / rowsum_block(f32, N);
}
__host__ __device__ constexpr int gemm_stats_smem(int e) { return epi_has_stat_warps(e) ? 2 * 2 * kGemmBM * 4 : 0; }
// epilogue staging + barriers + statistics + alignment slack: what the stages may not use
__host__ __device__ constexpr int gemm_fixed_smem(int e) {
  return epi_warps(e) * kEpiBufs * kEpiBufBytes + 1024 + gemm_stats_smem(e) + 1024;
}

// SUB = 64-wide K slabs per pipeline stage (1 or 2).  More K per stage means
// fewer MMA-complete -> refill round trips per FLOP; measured on B200 the
// round trip, not the stage count, limits the mainloop.
template <int BN, int SUB, int EPI>
struct GemmCfg {
  static constexpr int kSub = SUB;
  static constexpr int kSlabA = kGemmBM * kGemmBK * 2;
  static constexpr int kSlabB = BN * kGemmBK * 2;
  static constexpr int kStageA = kSlabA * SUB;
  static constexpr int kStageB = kSlabB * SUB;
  static constexpr int kStageBytes = kStageA + kStageB;
  static constexpr int kStages = (kSmemLimit - gemm_fixed_smem(EPI)) / kStageBytes;  // BN=256: 4 (SUB 1) / 2 (SUB 2)
  static constexpr int kTmemCols = 512;                        // 2 accumulators, 256-column slots
  static constexpr int kAccStride = 256;
  static constexpr int kStaging = epi_warps(EPI) * kEpiBufs * kEpiBufBytes;
  static constexpr int kOffStaging = kStages * kStageBytes;
  static constexpr int kOffBars = kOffStaging + kStaging;
  static constexpr int kOffStats = kOffBars + 1024;
  static constexpr int kSmemBytes = kOffStats + gemm_stats_smem(EPI) + 1024 /*alignment slack*/;
  static_assert(kStages >= 2 && kSmemBytes <= kSmemLimit, "GEMM shared-memory budget");
};

// keeps the compiler from using tcgen05.ld destination registers before the
// tcgen05.wait::ld that makes them valid
#define SG_REG_FENCE_32(r)                                                                               \
  asm volatile(""                                                                                        \
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),       \
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),   \
                 "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),             \
                 "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),             \
                 "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]))

__device__ __forceinline__ void load_param32(const float* __restrict__ p, int col0, int N, float* v) {
  if (col0 + 32 <= N) {  // the whole chunk inside N: no per-vector checks
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(p + col0) + q);
      v[4 * q] = f.x;
      v[4 * q + 1] = f.y;
      v[4 * q + 2] = f.z;
      v[4 * q + 3] = f.w;
    }
    return;
  }
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
    if (col0 + 4 * q < N) f = __ldg(reinterpret_cast<const float4*>(p + col0) + q);  // N % 8 == 0
    v[4 * q] = f.x;
    v[4 * q + 1] = f.y;
    v[4 * q + 2] = f.z;
    v[4 * q + 3] = f.w;
  }
}


// Epilogue of one CTA: EW = epi_warps(EPI) warps; warp w drains TMEM lane
// quarter w & 3 (32 rows) and, with 8 warps, half of the tile's columns.
// Per 32-column chunk: TMEM -> registers -> fused math in fp32 ->
// 64B-swizzled staging -> TMA store; the residual (if any) arrives in the
// staging buffer by TMA.  At the start of each tile the next tile's bias /
// LayerNorm vectors and row sums are prefetched into L1 and its residual box
// into L2.  `row_offset` is the first output row of this CTA's 128-row half
// of the tile; `tempty_addr*` are the shared::cluster addresses of the
// barriers that hand each accumulator back to the MMA issuer.
template <typename T, int BN, int EPI, bool kCluster, bool kScale = false>
__device__ __forceinline__ void gemm_epilogue(const GemmParams& p, const CUtensorMap* tmO, const CUtensorMap* tmR,
                                              uint32_t tmem_base, uint32_t acc_stride, uint8_t* staging,
                                              uint64_t* resbar, uint64_t* tfull, uint32_t tempty_addr0,
                                              uint32_t tempty_addr1, uint64_t* sfull, uint64_t* sempty,
                                              const float* st_mean, const float* st_rstd, volatile int* abort_flag,
                                              int warp, int lane, int first_tile, int tile_step, int num_tiles,
                                              int n_tiles, int rows_per_tile, int row_offset) {
  constexpr bool kStat = epi_has_stat_warps(EPI);  // mu/rstd from this kernel's statistics warps
  constexpr bool kRsIn = (EPI == kEpiLnRs || EPI == kEpiLnRsGelu);  // mu/rstd from row sums
  constexpr bool kLnMath = epi_is_ln(EPI);
  constexpr bool kGelu = epi_is_gelu(EPI);
  constexpr bool kRes = epi_has_res(EPI);
  constexpr bool kRsOut = (EPI == kEpiBiasResRs || EPI == kEpiBiasPosRs);
  constexpr bool kPos = (EPI == kEpiBiasPosRs);
  constexpr int EW = epi_warps(EPI);
  constexpr int kParts = EW / 4;              // column parts per tile
  constexpr int kPartCols = BN / kParts;
  constexpr int NCH = kPartCols / kEpiCols;   // chunks per warp per tile
  static_assert(kPartCols % kEpiCols == 0, "epilogue column split");
  static_assert(!kRsOut || kPartCols == BN / 2, "a row-sum slot is half a tile (rowsum_block)");
  const int ew = warp - 2;
  const int q = warp & 3;                     // TMEM lane quarter
  const int part = ew / 4;
  const int row_in_tile = q * 32 + lane;
  uint8_t* stg = staging + ew * (kEpiBufs * kEpiBufBytes);
  uint64_t* rbar = resbar + kEpiBufs * ew;
  uint32_t rph = 0;  // bit b: parity of the next completion of rbar[b]
  int sb = 0;        // staging buffer of the current chunk

  // tile coordinates (row block, column tile), advanced by tile_step without
  // a division per tile
  const int step_rb = tile_step / n_tiles, step_col = tile_step - step_rb * n_tiles;
  int cur_rb = first_tile / n_tiles, cur_col = first_tile - cur_rb * n_tiles;
  auto advance = [&](int& rb, int& col) {
    col += step_col;
    rb += step_rb;
    if (col >= n_tiles) {
      col -= n_tiles;
      ++rb;
    }
  };
  // L1/L2 prefetch of what the epilogue of `tile` (row block rb, column tile col) reads besides TMEM
  auto prefetch_tile = [&](int tile, int rb, int col) {
    if (tile >= num_tiles) return;
    const int pm0 = rb * rows_per_tile + row_offset, pc0 = col * BN + part * kPartCols;  // this warp's first column
    if (q == 0 && lane < NCH && pc0 + lane * 32 < p.N) {  // 32 floats = one 128-byte line per lane
      if constexpr (kLnMath) {
        prefetch_l1(p.c1 + pc0 + lane * 32);
        prefetch_l1(p.c2 + pc0 + lane * 32);
      } else if (p.bias) {
        prefetch_l1(p.bias + pc0 + lane * 32);
      }
    }
    if constexpr (kRsIn) {
      if (part == 0 && pm0 + q * 32 + lane < p.M) {
        const float2* r = p.rs_in + static_cast<size_t>(pm0 + q * 32 + lane) * p.rs_ld;
        prefetch_l1(r);
        prefetch_l1(r + p.rs_ld - 1);
      }
    }
    if constexpr (kRes) {
      if (lane < NCH && pm0 + q * 32 < p.M && pc0 + lane * kEpiCols < p.N)
        tma_prefetch_l2_2d(tmR, pc0 + lane * kEpiCols, pm0 + q * 32);
    }
  };

  prefetch_tile(first_tile, cur_rb, cur_col);
  int t = 0;
  for (int tile = first_tile; tile < num_tiles; tile += tile_step, ++t) {
    const int buf = t & 1;
    const uint32_t tph = (t >> 1) & 1;
    const int m0 = cur_rb * rows_per_tile + row_offset;
    const int c0 = cur_col * BN + part * kPartCols;  // this warp's first column
    const int row0 = m0 + q * 32;
    const int my_row = row0 + lane;
    advance(cur_rb, cur_col);  // from here on: the next tile's coordinates
    prefetch_tile(tile + tile_step, cur_rb, cur_col);
    float mu = 0.f, rstd = 1.f;
    float a_s = 1.f;  // kScale: this row's scale of A
    if constexpr (kScale) {
      if (my_row < p.M) a_s = __ldg(p.a_scale + my_row);
    }
    if constexpr (kRsIn) {
      // LayerNorm statistics of the raw A row (the previous GEMM's rounded
      // output) merged from its column-block slots in a fixed order
      if (my_row < p.M) slot_stats_merge(p.rs_in + static_cast<size_t>(my_row) * p.rs_ld, p.rs_ld, p.K, p.eps, mu, rstd);
    }
    if (*abort_flag || !mbar_wait<kCluster>(&tfull[buf], tph, 121)) {
      *abort_flag = 1;
      break;
    }
    tc_fence_after();
    if constexpr (kStat) {
      if (!mbar_wait(&sfull[buf], tph, 122)) {
        *abort_flag = 1;
        break;
      }
      mu = st_mean[buf * kGemmBM + row_in_tile];
      rstd = st_rstd[buf * kGemmBM + row_in_tile];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty[buf]);
    }
    // sums over this warp's columns of the rounded outputs minus the first of
    // them (kRsOut): shifted sums keep the slot variance exact when the row's
    // mean is large against its spread
    float rs_shift = 0.f;
    float2 rs1v = make_float2(0.f, 0.f), rs2v = make_float2(0.f, 0.f);
    AxisTaps ay{0, 0, 0.f, 1.f, 0.f}, ax{0, 0, 0.f, 1.f, 0.f};  // position-embedding taps of this row (kPos)
    if constexpr (kPos) {
      if (my_row < p.M) {
        const int b = p.tok_img[my_row];
        const int w = p.pos_hw[2 * b + 1];
        const int i = my_row - p.cu[b];
        ay = axis_taps(i / w, p.pos_hw[2 * b], p.pos_grid);
        ax = axis_taps(i - (i / w) * w, w, p.pos_grid);
      }
    }
    const uint32_t tbase =
        tmem_base + buf * acc_stride + part * kPartCols + (static_cast<uint32_t>(q * 32) << 16);
    uint32_t ra[32], rb[32];
    SG_TMEM_LD_32(tbase, ra);
    tmem_ld_wait();
    SG_REG_FENCE_32(ra);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      uint32_t* cur = (c & 1) ? rb : ra;
      uint32_t* nxt = (c & 1) ? ra : rb;
      if (c + 1 < NCH) SG_TMEM_LD_32(tbase + (c + 1) * kEpiCols, nxt);
      const int col0 = c0 + c * kEpiCols;
      uint8_t* sbuf = stg + sb * kEpiBufBytes;
      // the store issued from this buffer two chunks ago must have read it
      if (lane == 0) tma_store_wait_read<1>();
      if constexpr (kRes) {
        if (lane == 0) {
          mbar_arrive_expect_tx(&rbar[sb], kEpiBufBytes);
          tma_load_2d(sbuf, tmR, &rbar[sb], col0, row0);
        }
      }
      __syncwarp();
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(cur[j]);
      if (col0 < p.N) {
        if constexpr (kLnMath) {
          float a[32], b[32];
          load_param32(p.c1, col0, p.N, a);
          load_param32(p.c2, col0, p.N, b);
          // column pairs in packed f32x2 issues (lane-wise the same roundings)
          const float2 nmu2 = make_float2(-mu, -mu), rstd2 = make_float2(rstd, rstd);
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float2 t = ffma2(rstd2, ffma2(nmu2, make_float2(a[j], a[j + 1]), make_float2(v[j], v[j + 1])),
                             make_float2(b[j], b[j + 1]));
            if constexpr (kGelu) t = gelu_tanh2(t);
            v[j] = t.x;
            v[j + 1] = t.y;
          }
        } else {
          float a[32];
          if constexpr (kScale) {
            load_param32(p.b_scale, col0, p.N, a);
            const float2 as2 = make_float2(a_s, a_s);
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const float2 t = fmul2(make_float2(v[j], v[j + 1]), fmul2(as2, make_float2(a[j], a[j + 1])));
              v[j] = t.x;
              v[j + 1] = t.y;
            }
          }
          if (p.bias) {
            load_param32(p.bias, col0, p.N, a);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) a[j] = 0.f;
          }
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float2 t = fadd2(make_float2(v[j], v[j + 1]), make_float2(a[j], a[j + 1]));
            if constexpr (kGelu) t = gelu_tanh2(t);
            v[j] = t.x;
            v[j + 1] = t.y;
          }
        }
        if constexpr (kPos) {
          // separable triangle-filter taps over the fp32 table (L2-resident):
          // 2 x 2 taps when upsampling, more when the image side is < grid
          for (int ya = ay.lo; ya < ay.hi; ++ya) {
            const float wy = axis_w(ay, ya);
            for (int xa = ax.lo; xa < ax.hi; ++xa) {
              const float wgt = wy * axis_w(ax, xa);
              const float4* src =
                  reinterpret_cast<const float4*>(p.pos_table + static_cast<size_t>(ya * p.pos_grid + xa) * p.N + col0);
#pragma unroll
              for (int q4 = 0; q4 < 8; ++q4) {
                if (col0 + 4 * q4 < p.N) {
                  const float4 f = __ldg(src + q4);
                  v[4 * q4] = fmaf(wgt, f.x, v[4 * q4]);
                  v[4 * q4 + 1] = fmaf(wgt, f.y, v[4 * q4 + 1]);
                  v[4 * q4 + 2] = fmaf(wgt, f.z, v[4 * q4 + 2]);
                  v[4 * q4 + 3] = fmaf(wgt, f.w, v[4 * q4 + 3]);
                }
              }
            }
          }
        }
      }
      // 64B-swizzled staging: 16B chunk g of row r lives at chunk g ^ ((r >> 1) & 3)
      const int sw = (lane >> 1) & 3;
      uint8_t* srow = sbuf + lane * (kEpiCols * 2);
      if constexpr (kRes) {
        if (!mbar_wait(&rbar[sb], (rph >> sb) & 1, 123)) *abort_flag = 1;
        rph ^= 1u << sb;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const uint4 rv = *reinterpret_cast<const uint4*>(srow + ((g ^ sw) << 4));
          const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const float2 f = Pack2<T>::unpack(rw[h]);
            if constexpr (EPI == kEpiBiasGeluGrad) {
              v[g * 8 + 2 * h] = f.x * gelu_tanh_grad(v[g * 8 + 2 * h]);
              v[g * 8 + 2 * h + 1] = f.y * gelu_tanh_grad(v[g * 8 + 2 * h + 1]);
            } else {
              const float2 t = fadd2(make_float2(v[g * 8 + 2 * h], v[g * 8 + 2 * h + 1]), f);
              v[g * 8 + 2 * h] = t.x;
              v[g * 8 + 2 * h + 1] = t.y;
            }
          }
        }
      }
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint4 o;
        o.x = Pack2<T>::pack(v[g * 8 + 0], v[g * 8 + 1]);
        o.y = Pack2<T>::pack(v[g * 8 + 2], v[g * 8 + 3]);
        o.z = Pack2<T>::pack(v[g * 8 + 4], v[g * 8 + 5]);
        o.w = Pack2<T>::pack(v[g * 8 + 6], v[g * 8 + 7]);
        *reinterpret_cast<uint4*>(srow + ((g ^ sw) << 4)) = o;
        if constexpr (kRsOut) {
          // statistics of exactly what the next GEMM will read (the rounded values)
          if (col0 + g * 8 < p.N) {
            const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
            for (int h2 = 0; h2 < 4; ++h2) {
              const float2 f = Pack2<T>::unpack(ow[h2]);
              if (c == 0 && g == 0 && h2 == 0) rs_shift = f.x;
              // even and odd columns in the two lanes of packed issues
              const float2 d = fadd2(f, make_float2(-rs_shift, -rs_shift));
              rs1v = fadd2(rs1v, d);
              rs2v = ffma2(d, d, rs2v);
            }
          }
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && col0 < p.N && row0 < p.M) {
        tma_store_2d(tmO, sbuf, col0, row0);
      }
      if (lane == 0) tma_store_commit();
      sb ^= 1;
      if (c + 1 < NCH) {
        tmem_ld_wait();
        SG_REG_FENCE_32(nxt);
      } else {
        // this warp's part of the accumulator is read: hand it back to the MMA issuer
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(buf ? tempty_addr1 : tempty_addr0);
      }
    }
    if constexpr (kRsOut) {
      // this warp's column block is one slot (block width kPartCols = BN / 2)
      if (my_row < p.M && c0 < p.N)
        p.rs_acc[static_cast<size_t>(my_row) * p.rs_ld + c0 / kPartCols] =
            slot_stats_from_shifted(rs1v.x + rs1v.y, rs2v.x + rs2v.y, rs_shift, min(kPartCols, p.N - c0));
    }
  }
  if (lane == 0) tma_store_wait_all<0>();
  __syncwarp();
}

// LayerNorm row statistics of the A tiles (warps 6-9; thread r = row r of
// this CTA's 128-row A half).  `ready[s]` signals that stage s has landed.
// Split-K epilogue: the fp32 accumulator of one K slice straight to its
// partial buffer (each thread one row, 128 contiguous bytes per 32-column
// chunk), then the accumulator goes back to the MMA issuer.
template <int BN>
__device__ __forceinline__ void gemm_epilogue_part(const GemmParams& p, uint32_t tmem_base, uint32_t acc_stride,
                                                   uint64_t* tfull, uint32_t tempty_addr0, uint32_t tempty_addr1,
                                                   volatile int* abort_flag, int warp, int lane, int first_tile,
                                                   int tile_step, int num_tiles, int mn_tiles, int n_tiles) {
  constexpr int kPartCols = BN / 2;  // 8 warps: two per TMEM lane quarter, half the columns each
  const int ew = warp - 2;
  const int q = warp & 3;
  const int part = ew / 4;
  int t = 0;
  for (int tile = first_tile; tile < num_tiles; tile += tile_step, ++t) {
    const int buf = t & 1;
    const uint32_t tph = (t >> 1) & 1;
    const int split = tile / mn_tiles;
    const int rem = tile - split * mn_tiles;
    const int row = (rem / n_tiles) * kGemmBM + q * 32 + lane;
    const int c0 = (rem % n_tiles) * BN + part * kPartCols;
    if (*abort_flag || !mbar_wait(&tfull[buf], tph, 124)) {
      *abort_flag = 1;
      break;
    }
    tc_fence_after();
    const uint32_t tbase = tmem_base + buf * acc_stride + part * kPartCols + (static_cast<uint32_t>(q * 32) << 16);
    float* dst = p.part + (static_cast<size_t>(split) * p.M + row) * p.ld_part;
#pragma unroll
    for (int c = 0; c < kPartCols / 32; ++c) {
      uint32_t r[32];
      SG_TMEM_LD_32(tbase + c * 32, r);
      tmem_ld_wait();
      SG_REG_FENCE_32(r);
      if (row < p.M) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int col = c0 + c * 32 + 4 * j;
          if (col < p.N)  // N % 8 == 0
            *reinterpret_cast<float4*>(dst + col) = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                                                __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(buf ? tempty_addr1 : tempty_addr0);
  }
}

// out[m, n] = sum_s part[s][m][n] (+ bias[n]), the slices added in order;
// 8 columns per thread
template <typename T>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ part, int splits, int M, int N,
                                                            int ld_part, const float* __restrict__ bias,
                                                            T* __restrict__ out, int ldo) {
  const int nv = N / 8;
  const size_t total = static_cast<size_t>(M) * nv;
  const size_t slice = static_cast<size_t>(M) * ld_part;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int m = static_cast<int>(i / nv);
    const int c = static_cast<int>(i - static_cast<size_t>(m) * nv) * 8;
    const float* src = part + static_cast<size_t>(m) * ld_part + c;
    float v[8];
    if (bias) {
      const float4 b0 = __ldg(reinterpret_cast<const float4*>(bias + c));
      const float4 b1 = __ldg(reinterpret_cast<const float4*>(bias + c) + 1);
      v[0] = b0.x; v[1] = b0.y; v[2] = b0.z; v[3] = b0.w; v[4] = b1.x; v[5] = b1.y; v[6] = b1.z; v[7] = b1.w;
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = 0.f;
    }
    for (int sp = 0; sp < splits; ++sp) {
      const float4 a0 = __ldg(reinterpret_cast<const float4*>(src + sp * slice));
      const float4 a1 = __ldg(reinterpret_cast<const float4*>(src + sp * slice) + 1);
      v[0] += a0.x; v[1] += a0.y; v[2] += a0.z; v[3] += a0.w;
      v[4] += a1.x; v[5] += a1.y; v[6] += a1.z; v[7] += a1.w;
    }
    store_vec(out + static_cast<size_t>(m) * ldo + c, v);
  }
}

template <typename T, int STAGES, int SUB, bool kCluster>
__device__ __forceinline__ void gemm_row_stats(const GemmParams& p, const uint8_t* smA, int stage_a_bytes,
                                               uint64_t* ready, uint64_t* empty, uint64_t* sfull, uint64_t* sempty,
                                               float* st_mean, float* st_rstd, volatile int* abort_flag, int r,
                                               int lane, int first_tile, int tile_step, int num_tiles, int nk) {
  int stage = 0;
  uint32_t phase = 0;
  int t = 0;
  for (int tile = first_tile; tile < num_tiles; tile += tile_step, ++t) {
    const int buf = t & 1;
    const uint32_t tph = (t >> 1) & 1;
    if (*abort_flag || !mbar_wait(&sempty[buf], tph ^ 1, 131)) {
      *abort_flag = 1;
      break;
    }
    // 4 independent (sum, sum of squares) pairs: no long FMA dependency chain
    float shift = 0.f, s1v[4] = {0.f, 0.f, 0.f, 0.f}, s2v[4] = {0.f, 0.f, 0.f, 0.f};
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      if (*abort_flag || !mbar_wait<kCluster>(&ready[stage], phase, 132)) {
        ok = false;
        *abort_flag = 1;
        break;
      }
#pragma unroll
      for (int sub = 0; sub < SUB; ++sub) {
      const uint8_t* rowp = smA + stage * stage_a_bytes + sub * (kGemmBM * 128) + r * 128;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        // the 128B swizzle permutes the 16B chunks of a row; the sum does
        // not care about order, and reading chunk ch ^ (r & 7) puts the 8
        // rows of each 8-lane phase on 8 different bank groups
        const uint4 u = *reinterpret_cast<const uint4*>(rowp + ((ch ^ (r & 7)) << 4));
        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float2 f = Pack2<T>::unpack(w4[h]);
          if (kb == 0 && sub == 0 && ch == 0 && h == 0) shift = f.x;
          const float a = f.x - shift, b = f.y - shift;
          s1v[h] += a + b;
          s2v[h] = fmaf(a, a, s2v[h]);
          s2v[h] = fmaf(b, b, s2v[h]);
        }
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
    const float m1 = ((s1v[0] + s1v[1]) + (s1v[2] + s1v[3])) * inv_k;
    const float var = fmaxf(((s2v[0] + s2v[1]) + (s2v[2] + s2v[3])) * inv_k - m1 * m1, 0.f);
    st_mean[buf * kGemmBM + r] = shift + m1;
    st_rstd[buf * kGemmBM + r] = rsqrtf(var + p.eps);
    mbar_arrive(&sfull[buf]);
  }
}

// kAT / kBT: the operand is stored transposed ("MN-major"): A as [K][M]
// (M contiguous) and/or B as [K][N], as the backward's dgrad (B = the
// forward weight [N_out][K_in] read as [K][N]) and wgrad (A = the output
// gradient [tokens][N_out], B = the forward input [tokens][K_in]) need them.
// Such a tile arrives as 64-column TMA boxes of 64 K-rows (128B swizzle),
// one 8 KB chunk per 64 M (N) columns, and the UMMA reads it through an
// MN-major descriptor (chunk stride 8 KB, 8-row groups 1 KB apart).
// kSplitK: the tiles are (K slice, row tile, column tile); each writes its
// fp32 partial product (gemm_epilogue_part) for splitk_reduce_kernel.
template <typename T, int BN, int EPI, int SUB, bool kAT = false, bool kBT = false, bool kSplitK = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmR,
                   const GemmParams p) {
  constexpr bool kLN = epi_has_stat_warps(EPI);  // statistics warps in this kernel
  constexpr bool kRes = epi_has_res(EPI);
  static_assert(!(kAT && kLN), "the statistics warps read K-major A tiles");
  static_assert(!kSplitK || (EPI == kEpiBias && epi_warps(EPI) == 8), "split K: plain products only");
  using Cfg = GemmCfg<BN, SUB, EPI>;
  constexpr int EW = epi_warps(EPI);
  constexpr int STAGES = Cfg::kStages;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdesc = make_idesc(kGemmBM, BN, kBF16, kAT, kBT);
  constexpr int kChunk = 64 * kGemmBK * 2;  // one MN-major chunk: 64 columns x 64 K-rows

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + STAGES * Cfg::kStageA;
  uint8_t* staging = smem + Cfg::kOffStaging;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBars);
  uint64_t* full = bars;                 // [STAGES]
  uint64_t* empty = bars + STAGES;       // [STAGES]
  uint64_t* tfull = bars + 2 * STAGES;   // [2]
  uint64_t* tempty = tfull + 2;          // [2]
  uint64_t* sfull = tempty + 2;          // [2]
  uint64_t* sempty = sfull + 2;          // [2]
  uint64_t* mdone = sempty + 2;          // [1] all issued MMAs complete (teardown)
  uint64_t* resbar = mdone + 1;          // [EW][kEpiBufs] residual chunk landed in staging
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(resbar + kEpiBufs * EW);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* st_mean = reinterpret_cast<float*>(smem + Cfg::kOffStats);  // [2][128]
  float* st_rstd = st_mean + 2 * kGemmBM;                              // [2][128]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = (p.M + kGemmBM - 1) / kGemmBM;
  const int n_tiles = (p.N + BN - 1) / BN;
  const int mn_tiles = m_tiles * n_tiles;
  const int num_tiles = mn_tiles * (kSplitK ? p.k_splits : 1);
  // first K element and pipeline stages of a tile (its K slice when split)
  const auto tile_k0 = [&](int tile) { return kSplitK ? (tile / mn_tiles) * p.k_per_split : 0; };
  const auto tile_nk = [&](int tile) {
    const int k0 = tile_k0(tile);
    const int klen = kSplitK ? min(p.K - k0, p.k_per_split) : p.K;
    return (klen + kGemmBK * SUB - 1) / (kGemmBK * SUB);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kLN ? 5 : 1);  // MMA commit (+ one arrive per statistics warp)
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EW);
      mbar_init(&sfull[b], kGemmBM);
      mbar_init(&sempty[b], EW);
    }
    mbar_init(mdone, 1);
    for (int i = 0; i < kEpiBufs * EW; ++i) mbar_init(&resbar[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmO);
    if (kRes) tma_prefetch_desc(&tmR);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, Cfg::kTmemCols);
    tmem_relinquish();
  }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // the previous kernel's outputs are complete and visible from here on
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int rem = tile % mn_tiles;
        const int m0 = (rem / n_tiles) * kGemmBM;
        const int n0 = (rem % n_tiles) * BN;
        const int k0 = tile_k0(tile), nk = tile_nk(tile);
        for (int kb = 0; kb < nk; ++kb) {
          if (*abort_flag || !mbar_wait(&empty[stage], phase ^ 1, 101)) {
            ok = false;
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
#pragma unroll
          for (int sub = 0; sub < SUB; ++sub) {
            const int kx = k0 + (kb * SUB + sub) * kGemmBK;
            uint8_t* sa = smA + stage * Cfg::kStageA + sub * Cfg::kSlabA;
            uint8_t* sb = smB + stage * Cfg::kStageB + sub * Cfg::kSlabB;
            if constexpr (kAT) {
#pragma unroll
              for (int c = 0; c < kGemmBM / 64; ++c) tma_load_2d(sa + c * kChunk, &tmA, &full[stage], m0 + 64 * c, kx);
            } else {
              tma_load_2d(sa, &tmA, &full[stage], kx, m0);
            }
            if constexpr (kBT) {
#pragma unroll
              for (int c = 0; c < BN / 64; ++c) tma_load_2d(sb + c * kChunk, &tmB, &full[stage], n0 + 64 * c, kx);
            } else {
              tma_load_2d(sb, &tmB, &full[stage], kx, n0);
            }
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Tail: no TMA write may still be in flight into this CTA's shared
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
        const int nk = tile_nk(tile);
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
          for (int sub = 0; sub < SUB; ++sub) {
#pragma unroll
            for (int k = 0; k < kGemmBK / 16; ++k) {
              // K-major: 16 K-elements = 32 bytes along the row; MN-major: 16 K-rows = 2 KB
              const uint64_t ad = kAT ? smem_desc(a_base + sub * Cfg::kSlabA + k * 2048, kChunk, 1024, kSw128)
                                      : kmajor_desc(a_base + sub * Cfg::kSlabA + k * 32, 128);
              const uint64_t bd = kBT ? smem_desc(b_base + sub * Cfg::kSlabB + k * 2048, kChunk, 1024, kSw128)
                                      : kmajor_desc(b_base + sub * Cfg::kSlabB + k * 32, 128);
              umma_ss(d_tmem, ad, bd, kIdesc, (kb | sub | k) != 0);
            }
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
  } else if (warp < 2 + EW) {
    // ------------------------------------------------------------ epilogue
    // Warp (warp & 3) may only touch TMEM lanes 32*(warp&3) .. +31: it owns
    // those 32 rows of the tile, 32 columns per chunk.  Each chunk goes
    // TMEM -> registers -> fused math -> 64B-swizzled staging -> TMA store
    // (the residual, if any, arrives in the same staging buffer by TMA).
    const uint32_t te0 = mapa_shared(smem_u32(&tempty[0]), 0), te1 = mapa_shared(smem_u32(&tempty[1]), 0);
    if constexpr (kSplitK)
      gemm_epilogue_part<BN>(p, tmem_base, Cfg::kAccStride, tfull, te0, te1, abort_flag, warp, lane, blockIdx.x,
                             gridDim.x, num_tiles, mn_tiles, n_tiles);
    else
      gemm_epilogue<T, BN, EPI, false>(p, &tmO, &tmR, tmem_base, Cfg::kAccStride, staging, resbar, tfull, te0, te1,
                                       sfull, sempty, st_mean, st_rstd, abort_flag, warp, lane, blockIdx.x, gridDim.x,
                                       num_tiles, n_tiles, kGemmBM, 0);
  } else {
    // ------------------------------------------------------------ LayerNorm row statistics
    if constexpr (kLN) {
      gemm_row_stats<T, STAGES, SUB, false>(p, smA, Cfg::kStageA, full, empty, sfull, sempty, st_mean, st_rstd,
                                       abort_flag, threadIdx.x - (2 + EW) * 32, lane, blockIdx.x, gridDim.x,
                                       num_tiles, tile_nk(0));
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}


// ============================================================================
// 2-SM variant: a CTA pair (cluster of 2) computes a 256 x BN tile with
// tcgen05.mma.cta_group::2.  Each CTA's smem holds its 128 rows of A and its
// BN/2 rows of B for every stage (same offsets in both CTAs); both CTAs load
// their own halves with plain TMA copies whose completion bytes go to the
// leader's (rank 0) full barrier.  The leader alone issues the MMAs and
// multicast-commits the stage-free and accumulator-ready barriers to both
// CTAs; each CTA drains its own 128 rows of the accumulator from its own TMEM
// and reports back to the leader's accumulator-free barrier.  Per SM this
// halves the B operand's shared-memory footprint and traffic.
// ============================================================================
template <int BN, int SUB, int EPI>
struct Gemm2Cfg {
  static constexpr int kSub = SUB;
  static constexpr int kSlabA = kGemmBM * kGemmBK * 2;          // this CTA's 128 rows of A
  static constexpr int kSlabB = (BN / 2) * kGemmBK * 2;         // this CTA's half of B
  static constexpr int kStageA = kSlabA * SUB;
  static constexpr int kStageB = kSlabB * SUB;
  static constexpr int kStageBytes = kStageA + kStageB;
  static constexpr int kStages = (kSmemLimit - gemm_fixed_smem(EPI)) / kStageBytes;  // BN=256: 6 (SUB 1) / 3 (SUB 2)
  static constexpr int kTmemCols = 512;
  static constexpr int kAccStride = 256;
  static constexpr int kStaging = epi_warps(EPI) * kEpiBufs * kEpiBufBytes;
  static constexpr int kOffStaging = kStages * kStageBytes;
  static constexpr int kOffBars = kOffStaging + kStaging;
  static constexpr int kOffStats = kOffBars + 1024;
  static constexpr int kSmemBytes = kOffStats + gemm_stats_smem(EPI) + 1024;
  static_assert(kStages >= 2 && kSmemBytes <= kSmemLimit, "GEMM shared-memory budget");
};

// kF8: A and B hold e4m3 values, read as pairs through the same 16-bit tensor
// maps and 128-byte rows (a 64-wide slab of pairs is 128 K-elements); the
// MMAs run kind::f8f6f4 (32 K-elements each) and the epilogue applies
// a_scale / b_scale; T is the output type.  p.K counts pairs.
// kBT: B stored transposed, [K][N] (N contiguous), as the backward's dgrad
// reads the forward weight: each CTA's half of B arrives as 64-column x
// 64-K-row boxes (8 KB chunks) and the MMA reads it as an MN-major operand.
template <typename T, int BN, int EPI, int SUB, bool kF8 = false, bool kBT = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmR,
                    const GemmParams p) {
  constexpr bool kLN = epi_has_stat_warps(EPI);  // statistics warps in this kernel
  constexpr bool kRes = epi_has_res(EPI);
  static_assert(!(kF8 && (kLN || epi_is_ln(EPI))), "8-bit operands: bias epilogues only");
  static_assert(!(kBT && (kF8 || kLN)), "MN-major B: 16-bit operands, no statistics warps");
  using Cfg = Gemm2Cfg<BN, SUB, EPI>;
  constexpr int kChunk = 64 * kGemmBK * 2;  // one MN-major chunk of B: 64 columns x 64 K-rows
  constexpr int EW = epi_warps(EPI);
  constexpr int STAGES = Cfg::kStages;
  // instruction-descriptor format bits: bf16 (1) or f16 (0) for kind::f16, e4m3 (0) for kind::f8f6f4
  constexpr bool kBF16 = !kF8 && std::is_same<T, __nv_bfloat16>::value;
  // the last column tile may be narrower (N - (n_tiles - 1) * BN, rounded up
  // to 16): its MMAs run at that width and the pair splits B at half of it
  const auto tile_width = [&](int n_tile) { return min(BN, (p.N - n_tile * BN + 15) & ~15); };
  constexpr int kTileRows = 2 * kGemmBM;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + STAGES * Cfg::kStageA;
  uint8_t* staging = smem + Cfg::kOffStaging;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBars);
  uint64_t* full = bars;                 // [STAGES] leader: both CTAs' halves landed
  uint64_t* empty = bars + STAGES;       // [STAGES] both: stage free (MMA commit + stats warps)
  uint64_t* aready = empty + STAGES;     // [STAGES] both: stage landed (forwarded for the stats warps)
  uint64_t* tfull = aready + STAGES;     // [2] both: accumulator ready
  uint64_t* tempty = tfull + 2;          // [2] leader: accumulator drained by both CTAs
  uint64_t* sfull = tempty + 2;          // [2]
  uint64_t* sempty = sfull + 2;          // [2]
  uint64_t* mdone = sempty + 2;          // [1]
  uint64_t* resbar = mdone + 1;          // [EW][kEpiBufs]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(resbar + kEpiBufs * EW);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* st_mean = reinterpret_cast<float*>(smem + Cfg::kOffStats);
  float* st_rstd = st_mean + 2 * kGemmBM;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  const int m_tiles = (p.M + kTileRows - 1) / kTileRows;
  const int n_tiles = (p.N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int nk = (p.K + kGemmBK * SUB - 1) / (kGemmBK * SUB);  // pipeline stages per tile

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kLN ? 5 : 1);
      mbar_init(&aready[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * EW);
      mbar_init(&sfull[b], kGemmBM);
      mbar_init(&sempty[b], EW);
    }
    mbar_init(mdone, 1);
    for (int i = 0; i < kEpiBufs * EW; ++i) mbar_init(&resbar[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmO);
    if (kRes) tma_prefetch_desc(&tmR);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  pdl_launch_dependents();
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised before any remote signal
  tc_fence_after();
  pdl_wait();  // the previous kernel's outputs are complete and visible from here on
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs) {
        const int m0 = (tile / n_tiles) * kTileRows + static_cast<int>(rank) * kGemmBM;
        const int n0 = (tile % n_tiles) * BN + static_cast<int>(rank) * (tile_width(tile % n_tiles) / 2);
        for (int kb = 0; kb < nk; ++kb) {
          if (*abort_flag || !mbar_wait<true>(&empty[stage], phase ^ 1, 141)) {
            ok = false;
            *abort_flag = 1;
            break;
          }
          const uint32_t fbar = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::kStageBytes);
#pragma unroll
          for (int sub = 0; sub < SUB; ++sub) {
            const int kx = (kb * SUB + sub) * kGemmBK;
            tma_load_2d_pair(smA + stage * Cfg::kStageA + sub * Cfg::kSlabA, &tmA, fbar, kx, m0);
            if constexpr (kBT) {
#pragma unroll
              for (int c = 0; c < BN / 2 / 64; ++c)
                tma_load_2d_pair(smB + stage * Cfg::kStageB + sub * Cfg::kSlabB + c * kChunk, &tmB, fbar, n0 + 64 * c,
                                 kx);
            } else {
              tma_load_2d_pair(smB + stage * Cfg::kStageB + sub * Cfg::kSlabB, &tmB, fbar, kx, n0);
            }
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Tail: every stage released again means every load landed and was consumed.
      for (int i = 0; i < STAGES && i < issued; ++i) {
        mbar_wait<true>(&empty[stage], phase ^ 1, 142);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int t = 0;
      bool ok = true;
      const uint32_t peer_aready0 = mapa_shared(smem_u32(&aready[0]), 1);
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs, ++t) {
        const int buf = t & 1;
        const uint32_t tph = (t >> 1) & 1;
        if (*abort_flag || !mbar_wait<true>(&tempty[buf], tph ^ 1, 151)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * Cfg::kAccStride;
        const uint32_t idesc = make_idesc(2 * kGemmBM, tile_width(tile % n_tiles), kBF16, false, kBT);
        for (int kb = 0; kb < nk; ++kb) {
          if (*abort_flag || !mbar_wait<true>(&full[stage], phase, 152)) {
            ok = false;
            *abort_flag = 1;
            break;
          }
          if constexpr (kLN) {
            // tell both CTAs' statistics warps that their A half landed
            mbar_arrive(&aready[stage]);
            mbar_arrive_cluster(peer_aready0 + stage * 8);
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smA + stage * Cfg::kStageA);
          const uint32_t b_base = smem_u32(smB + stage * Cfg::kStageB);
#pragma unroll
          for (int sub = 0; sub < SUB; ++sub) {
#pragma unroll
            for (int k = 0; k < kGemmBK / 16; ++k) {
              // K-major: 16 K-elements = 32 bytes along the row; MN-major: 16 K-rows = 2 KB
              const uint64_t bd = kBT ? smem_desc(b_base + sub * Cfg::kSlabB + k * 2048, kChunk, 1024, kSw128)
                                      : kmajor_desc(b_base + sub * Cfg::kSlabB + k * 32, 128);
              if constexpr (kF8)
                umma_ss_pair_f8(d_tmem, kmajor_desc(a_base + sub * Cfg::kSlabA + k * 32, 128), bd, idesc,
                                (kb | sub | k) != 0);
              else
                umma_ss_pair(d_tmem, kmajor_desc(a_base + sub * Cfg::kSlabA + k * 32, 128), bd, idesc,
                             (kb | sub | k) != 0);
            }
          }
          umma_commit_pair_mc(&empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair_mc(&tfull[buf], 0x3);
      }
      umma_commit_pair(mdone);
      mbar_wait<true>(mdone, 0, 153);
    }
  } else if (warp < 2 + EW) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const uint32_t te0 = mapa_shared(smem_u32(&tempty[0]), 0), te1 = mapa_shared(smem_u32(&tempty[1]), 0);
    gemm_epilogue<T, BN, EPI, true, kF8>(p, &tmO, &tmR, tmem_base, Cfg::kAccStride, staging, resbar, tfull, te0,
                                         te1, sfull, sempty, st_mean, st_rstd, abort_flag, warp, lane, pair,
                                         num_pairs, num_tiles, n_tiles, kTileRows, static_cast<int>(rank) * kGemmBM);
  } else {
    // ------------------------------------------------------------ LayerNorm row statistics (both CTAs)
    if constexpr (kLN) {
      gemm_row_stats<T, STAGES, SUB, true>(p, smA, Cfg::kStageA, aready, empty, sfull, sempty, st_mean, st_rstd,
                                      abort_flag, threadIdx.x - (2 + EW) * 32, lane, pair, num_pairs,
                                      num_tiles, nk);
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  cluster_sync();  // no remote arrive or TMA completion may target an exited CTA
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
}

}  // namespace sg
