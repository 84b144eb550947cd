// C-ABI entry points of libsiglip2_b200.so (see include/siglip2_b200.h).
// One translation unit: every kernel header is included here and compiled
// for sm_100a only.
#include <algorithm>
#include <climits>
#include <cmath>
#include <type_traits>
#include <vector>

#include "host_common.cuh"
#include "gemm.cuh"
#include "rowops.cuh"
#include "fmha.cuh"
#include "fmha_pair.cuh"
#include "fp8.cuh"
#include "fmha_bwd.cuh"
#include "forward.cuh"
#include "simt_f32.cuh"
#include "patchify.cuh"

using namespace sg;

namespace {

struct GemmIO {
  const void* a;
  int lda;
  const void* b;
  int ldb;
  void* out;
  int ldo;
  const void* res;
  int ldr;
};

// Programmatic dependent launch for the persistent GEMM / attention kernels:
// each may be scheduled while the previous kernel of the stream drains; the
// kernel itself waits (griddepcontrol.wait) before touching global memory.
inline void set_pdl_attr(cudaLaunchAttribute* a) {
  a->id = cudaLaunchAttributeProgrammaticStreamSerialization;
  a->val.programmaticStreamSerializationAllowed = 1;
}

template <typename T, int BN, int EPI, int SUB, bool kAT = false, bool kBT = false, bool kSplitK = false>
int launch_gemm_tc(const GemmIO& io, const GemmParams& p, cudaStream_t stream) {
  CUtensorMap ta, tb, to, tr;
  // transposed operands are [K][M] / [K][N] in memory: 64 x 64 boxes
  if (kAT) SG_TRY(make_tmap_2d(&ta, io.a, 2, p.K, p.M, io.lda, kGemmBK, 64));
  else SG_TRY(make_tmap_2d(&ta, io.a, 2, p.M, p.K, io.lda, kGemmBM, kGemmBK));
  if (kBT) SG_TRY(make_tmap_2d(&tb, io.b, 2, p.K, p.N, io.ldb, kGemmBK, 64));
  else SG_TRY(make_tmap_2d(&tb, io.b, 2, p.N, p.K, io.ldb, BN, kGemmBK));
  SG_TRY(make_tmap_2d(&to, io.out, 2, p.M, p.N, io.ldo, 32, kEpiCols));
  if (epi_has_res(EPI)) SG_TRY(make_tmap_2d(&tr, io.res, 2, p.M, p.N, io.ldr, 32, kEpiCols));
  else tr = to;
  constexpr int threads = kGemmThreads;
  constexpr int smem = GemmCfg<BN, SUB, EPI>::kSmemBytes;
  auto kern = gemm_tc_kernel<T, BN, EPI, SUB, kAT, kBT, kSplitK>;
  SG_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem));
  const int tiles = ((p.M + kGemmBM - 1) / kGemmBM) * ((p.N + BN - 1) / BN) * (kSplitK ? p.k_splits : 1);
  const int grid = tiles < sm_count() ? tiles : sm_count();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  set_pdl_attr(&attr[0]);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SG_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, to, tr, p));
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

// 2-SM variant: clusters of 2 CTAs, one pair per 2 SMs, 256 x BN tiles.
template <typename T, int BN, int EPI, int SUB, bool kF8 = false, bool kBT = false>
int launch_gemm_tc2(const GemmIO& io, const GemmParams& p, cudaStream_t stream) {
  CUtensorMap ta, tb, to, tr;
  SG_TRY(make_tmap_2d(&ta, io.a, 2, p.M, p.K, io.lda, kGemmBM, kGemmBK));
  // transposed B is [K][N] in memory: 64 x 64 boxes
  if (kBT) SG_TRY(make_tmap_2d(&tb, io.b, 2, p.K, p.N, io.ldb, kGemmBK, 64));
  else SG_TRY(make_tmap_2d(&tb, io.b, 2, p.N, p.K, io.ldb, BN / 2, kGemmBK));
  SG_TRY(make_tmap_2d(&to, io.out, 2, p.M, p.N, io.ldo, 32, kEpiCols));
  if (epi_has_res(EPI)) SG_TRY(make_tmap_2d(&tr, io.res, 2, p.M, p.N, io.ldr, 32, kEpiCols));
  else tr = to;
  constexpr int threads = kGemmThreads;
  constexpr int smem = Gemm2Cfg<BN, SUB, EPI>::kSmemBytes;
  auto kern = gemm_tc2_kernel<T, BN, EPI, SUB, kF8, kBT>;
  SG_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem));
  const int tiles = ((p.M + 2 * kGemmBM - 1) / (2 * kGemmBM)) * ((p.N + BN - 1) / BN);
  const int pairs = std::min(tiles, sm_count() / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  set_pdl_attr(&attr[1]);
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  SG_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, to, tr, p));
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

// GEMM kernel selection: 0 = automatic, 1 = one SM per tile, 2 = SM pairs.
std::atomic<int> g_gemm_variant{0};
// Attention kernel selection: 0 = automatic (one query tile per CTA), 1 = one
// query tile per CTA, 2 = paired query tiles.
std::atomic<int> g_fmha_variant{0};

// Automatic choice (measured on B200 at the tower's shapes, K = 128 per stage
// in both): LayerNorm-folded GEMMs on one SM per tile (their statistics warps
// read the A stage locally), the others on SM pairs.
template <typename T, int BN, int EPI>
int launch_gemm_any(const GemmIO& io, const GemmParams& p, cudaStream_t s) {
  constexpr bool kLN = epi_has_stat_warps(EPI);
  int v = g_gemm_variant.load();
  if (v == 0) v = kLN ? 1 : 2;
  if (v == 2) return launch_gemm_tc2<T, BN, EPI, 2>(io, p, s);
  if (BN == 256) return launch_gemm_tc<T, BN, EPI, 2>(io, p, s);
  return launch_gemm_tc<T, BN, EPI, 1>(io, p, s);  // BN=192 keeps 5 stages of K=64
}

template <typename T, int BN>
int dispatch_epi(int epi, const GemmIO& io, const GemmParams& p, cudaStream_t s) {
  switch (epi) {
    case kEpiBias: return launch_gemm_any<T, BN, kEpiBias>(io, p, s);
    case kEpiBiasRes: return launch_gemm_any<T, BN, kEpiBiasRes>(io, p, s);
    case kEpiLn: return launch_gemm_any<T, BN, kEpiLn>(io, p, s);
    case kEpiLnGelu: return launch_gemm_any<T, BN, kEpiLnGelu>(io, p, s);
    case kEpiBiasGelu: return launch_gemm_any<T, BN, kEpiBiasGelu>(io, p, s);
    case kEpiLnRs: return launch_gemm_any<T, BN, kEpiLnRs>(io, p, s);
    case kEpiLnRsGelu: return launch_gemm_any<T, BN, kEpiLnRsGelu>(io, p, s);
    case kEpiBiasResRs: return launch_gemm_any<T, BN, kEpiBiasResRs>(io, p, s);
    case kEpiBiasPosRs: return launch_gemm_any<T, BN, kEpiBiasPosRs>(io, p, s);
    case kEpiBiasGeluGrad: return launch_gemm_any<T, BN, kEpiBiasGeluGrad>(io, p, s);
    default: return set_error(SIGLIP2_ERR_ARG, "unknown epilogue %d", epi);
  }
}

// Transposed-operand GEMMs of the backward (one SM per 128 x 256 tile).
template <typename T, bool kAT, bool kBT>
int dispatch_epi_t(int epi, const GemmIO& io, const GemmParams& p, cudaStream_t s) {
  if (p.k_splits > 1) {
    // K sliced over more tiles than SMs would otherwise get; the partial
    // products are summed (+ bias) in slice order by splitk_reduce_kernel
    SG_TRY((launch_gemm_tc<T, 256, kEpiBias, 2, kAT, kBT, true>(io, p, s)));
    const size_t total = static_cast<size_t>(p.M) * (p.N / 8);
    const int grid = static_cast<int>(std::min<size_t>((total + 255) / 256, 8 * static_cast<size_t>(sm_count())));
    splitk_reduce_kernel<T><<<grid, 256, 0, s>>>(p.part, p.k_splits, p.M, p.N, p.ld_part, p.bias,
                                                 static_cast<T*>(io.out), io.ldo);
    SG_LAUNCH_CHECK();
    return SIGLIP2_OK;
  }
  // dgrad (K-major A, MN-major B): on CTA pairs like the forward's GEMMs
  if (!kAT && kBT && epi == kEpiBias && g_gemm_variant.load() != 1)
    return launch_gemm_tc2<T, 256, kEpiBias, 2, false, true>(io, p, s);
  switch (epi) {
    case kEpiBias: return launch_gemm_tc<T, 256, kEpiBias, 2, kAT, kBT>(io, p, s);
    case kEpiBiasGeluGrad: return launch_gemm_tc<T, 256, kEpiBiasGeluGrad, 2, kAT, kBT>(io, p, s);
    default: return set_error(SIGLIP2_ERR_UNSUPPORTED, "transposed-operand GEMM: epilogue %d not supported", epi);
  }
}

// Tile width: gemm_bn_for (256; the pair kernel narrows the last column tile).
template <typename T>
int dispatch_bn(int epi, const GemmIO& io, const GemmParams& p, cudaStream_t s) {
  static_assert(gemm_bn_for(1) == 256, "one tile width");
  return dispatch_epi<T, 256>(epi, io, p, s);
}

}  // namespace

// Position-embedding inputs of the fused patch-embedding epilogue (kEpiBiasPosRs).
struct PosArgs {
  const float* table;  // [grid^2, N] fp32
  int grid;
  const int* tok_img;  // [M] token -> image
  const int* hw;       // [2B] (h, w)
  const int* cu;       // [B+1] first token of each image
};

int sg_gemm_impl(int dtype, int epi, const void* a, int lda, const void* b, int ldb, void* out, int ldo, int M, int N,
                 int K, const float* bias, const void* res, int ldr, const float* c1, const float* c2, float eps,
                 cudaStream_t stream, const float2* rs_in = nullptr, float2* rs_acc = nullptr,
                 const PosArgs* pos = nullptr) {
  SG_CHECK_ARG(M >= 0 && N > 0 && K > 0, "bad GEMM shape M=%d N=%d K=%d", M, N, K);
  if (M == 0) return SIGLIP2_OK;
  SG_CHECK_ARG(a && b && out, "null operand");
  SG_CHECK_ARG(epi >= 0 && epi <= 9, "unknown epilogue %d", epi);
  SG_CHECK_ARG(epi != kEpiBiasPosRs ||
                   (pos && pos->table && pos->grid > 0 && pos->tok_img && pos->hw && pos->cu),
               "position-embedding epilogue needs table, grid, token->image map, grids and row starts");
  if (epi == kEpiBiasPosRs && !aligned16(pos->table))
    return set_error(SIGLIP2_ERR_ALIGN, "position table must be 16-byte aligned");
  const bool ln = epi_is_ln(epi);
  SG_CHECK_ARG(!ln || (c1 && c2), "LN epilogue needs c1 and c2");
  SG_CHECK_ARG(ln || bias, "bias epilogue needs bias");
  SG_CHECK_ARG(!epi_has_res(epi) || res, "residual epilogue needs res");
  SG_CHECK_ARG(!epi_has_stat_warps(epi) || K % kGemmBK == 0, "LN-folded GEMM needs K %% 64 == 0 (K=%d)", K);
  SG_CHECK_ARG(!(epi == kEpiLnRs || epi == kEpiLnRsGelu) || rs_in, "row-sum LN epilogue needs rs_in");
  SG_CHECK_ARG((epi != kEpiBiasResRs && epi != kEpiBiasPosRs) || rs_acc,
               "row-sum accumulating epilogue needs rs_acc");
  const auto misaligned8 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 7u) != 0; };
  if (misaligned8(rs_in) || misaligned8(rs_acc))
    return set_error(SIGLIP2_ERR_ALIGN, "row-sum buffers must be 8-byte aligned");
  if (dtype == SIGLIP2_F32) {
    if (epi == kEpiBiasGeluGrad)
      return set_error(SIGLIP2_ERR_UNSUPPORTED, "fp32 GEMM: the GELU-gradient epilogue is tensor-core only");
    if (epi_has_stat_warps(epi))
      return set_error(SIGLIP2_ERR_UNSUPPORTED, "fp32 GEMM: use the row-sum LayerNorm epilogues (5, 6)");
    if (epi_has_res(epi) && !res) return set_error(SIGLIP2_ERR_ARG, "residual epilogue needs res");
    GemmParams p{};
    p.M = M; p.N = N; p.K = K; p.bias = bias; p.c1 = c1; p.c2 = c2; p.eps = eps;
    p.rs_in = rs_in; p.rs_acc = rs_acc;
    p.rs_ld = rs_in ? rowsum_slots(true, K) : rowsum_slots(true, N);
    if (pos) {
      p.pos_table = pos->table; p.pos_grid = pos->grid; p.tok_img = pos->tok_img; p.pos_hw = pos->hw; p.cu = pos->cu;
    }
    dim3 grid((N + kSgBN - 1) / kSgBN, (M + kSgBM - 1) / kSgBM);
    const float* A = static_cast<const float*>(a);
    const float* Bw = static_cast<const float*>(b);
    float* O = static_cast<float*>(out);
    const float* R = static_cast<const float*>(res);
    switch (epi) {
      case kEpiBias: gemm_f32_kernel<kEpiBias><<<grid, 256, 0, stream>>>(A, lda, Bw, ldb, O, ldo, R, ldr, p); break;
      case kEpiBiasRes: gemm_f32_kernel<kEpiBiasRes><<<grid, 256, 0, stream>>>(A, lda, Bw, ldb, O, ldo, R, ldr, p); break;
      case kEpiBiasGelu: gemm_f32_kernel<kEpiBiasGelu><<<grid, 256, 0, stream>>>(A, lda, Bw, ldb, O, ldo, R, ldr, p); break;
      case kEpiLnRs: gemm_f32_kernel<kEpiLnRs><<<grid, 256, 0, stream>>>(A, lda, Bw, ldb, O, ldo, R, ldr, p); break;
      case kEpiLnRsGelu: gemm_f32_kernel<kEpiLnRsGelu><<<grid, 256, 0, stream>>>(A, lda, Bw, ldb, O, ldo, R, ldr, p); break;
      case kEpiBiasResRs: gemm_f32_kernel<kEpiBiasResRs><<<grid, 256, 0, stream>>>(A, lda, Bw, ldb, O, ldo, R, ldr, p); break;
      case kEpiBiasPosRs: gemm_f32_kernel<kEpiBiasPosRs><<<grid, 256, 0, stream>>>(A, lda, Bw, ldb, O, ldo, R, ldr, p); break;
      default: return set_error(SIGLIP2_ERR_ARG, "unknown epilogue %d", epi);
    }
    SG_LAUNCH_CHECK();
    return SIGLIP2_OK;
  }
  if (dtype != SIGLIP2_BF16 && dtype != SIGLIP2_F16)
    return set_error(SIGLIP2_ERR_UNSUPPORTED, "GEMM supports f32/bf16/f16 (dtype=%d)", dtype);
  if (N % 8 || K % 8 || lda % 8 || ldb % 8 || ldo % 8 || (epi_has_res(epi) && ldr % 8))
    return set_error(SIGLIP2_ERR_ALIGN, "N, K and leading dimensions must be multiples of 8");
  if (lda < K || ldb < K || ldo < N || (epi_has_res(epi) && ldr < N))
    return set_error(SIGLIP2_ERR_SHAPE, "leading dimension smaller than the row");
  if (!aligned16(out) || (res && !aligned16(res)))
    return set_error(SIGLIP2_ERR_ALIGN, "output/residual must be 16-byte aligned");
  if ((c1 && !aligned16(c1)) || (c2 && !aligned16(c2)) || (bias && !aligned16(bias)))
    return set_error(SIGLIP2_ERR_ALIGN, "bias / c1 / c2 vectors must be 16-byte aligned");
  GemmParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.bias = bias;
  p.c1 = c1;
  p.c2 = c2;
  p.eps = eps;
  p.rs_in = rs_in;
  p.rs_acc = rs_acc;
  p.rs_ld = rs_in ? rowsum_slots(false, K) : rowsum_slots(false, N);
  p.pos_table = nullptr;
  p.pos_grid = 0;
  p.tok_img = p.pos_hw = p.cu = nullptr;
  if (pos) {
    p.pos_table = pos->table;
    p.pos_grid = pos->grid;
    p.tok_img = pos->tok_img;
    p.pos_hw = pos->hw;
    p.cu = pos->cu;
  }
  GemmIO io{a, lda, b, ldb, out, ldo, res, ldr};
  if (dtype == SIGLIP2_BF16) return dispatch_bn<__nv_bfloat16>(epi, io, p, stream);
  return dispatch_bn<__half>(epi, io, p, stream);
}


// out[M, N] = epi(op(A) . op(B)^T) with op(A) = A [M][K] or, trans_a, A
// stored [K][M]; op(B) = B [N][K] or, trans_b, B stored [K][N].
// K slices for a transposed-operand GEMM whose 128 x 256 tiles would leave
// SMs idle (the weight gradients: few output tiles, long K = tokens).  In
// units of the GEMM's time at full occupancy, S slices cost 1 / (tile waves
// filled) for the products plus, for S > 1, the fp32 partials written and
// read back: 8 S M N bytes against 2 M N K FLOPs, i.e. about 880 S / K at
// the measured ~1.1 PFLOP/s per-tile rate and ~5 TB/s.  The cheapest S
// (slices of at least 1024 K-elements, S <= 8) is taken.
struct KSplit {
  int splits;
  int k_per_split;
};
KSplit choose_k_splits(int M, int N, int K) {
  const int tiles = ((M + kGemmBM - 1) / kGemmBM) * ((N + 255) / 256);
  const int sms = sm_count();
  KSplit best{1, K};
  double best_cost = 1e30;
  for (int s = 1; s <= 8; ++s) {
    const int kps = ((K + s - 1) / s + 127) / 128 * 128;
    const int splits = (K + kps - 1) / kps;
    if (splits != s || (s > 1 && kps < 1024)) continue;
    const long long work = static_cast<long long>(tiles) * s;
    const long long waves = (work + sms - 1) / sms;
    const double cost = static_cast<double>(waves * sms) / static_cast<double>(work) + (s > 1 ? 880.0 * s / K : 0.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = {s, kps};
    }
  }
  return best;
}

int sg_gemm_t_impl(int dtype, int epi, int trans_a, int trans_b, const void* a, int lda, const void* b, int ldb,
                   void* out, int ldo, int M, int N, int K, const float* bias, const void* res, int ldr,
                   cudaStream_t stream, void* workspace = nullptr, size_t workspace_bytes = 0) {
  SG_CHECK_ARG(M >= 0 && N > 0 && K > 0, "bad GEMM shape M=%d N=%d K=%d", M, N, K);
  if (M == 0) return SIGLIP2_OK;
  SG_CHECK_ARG(a && b && out, "null operand");
  SG_CHECK_ARG(epi == kEpiBias || epi == kEpiBiasGeluGrad, "transposed-operand GEMM: epilogue %d not supported", epi);
  SG_CHECK_ARG(epi != kEpiBiasGeluGrad || (bias && res), "GELU-gradient epilogue needs bias and res");
  if (dtype != SIGLIP2_BF16 && dtype != SIGLIP2_F16)
    return set_error(SIGLIP2_ERR_UNSUPPORTED, "transposed-operand GEMM supports bf16/f16 (dtype=%d)", dtype);
  // TMA wants 16-byte row pitches and the output / residual rows are stored
  // by TMA too; the extents themselves are free (out-of-range boxes read
  // zeros, stores are clipped), so token counts need no rounding
  if (N % 8 || lda % 8 || ldb % 8 || ldo % 8 || (res && ldr % 8))
    return set_error(SIGLIP2_ERR_ALIGN, "N and leading dimensions must be multiples of 8");
  if (lda < (trans_a ? M : K) || ldb < (trans_b ? N : K) || ldo < N || (res && ldr < N))
    return set_error(SIGLIP2_ERR_SHAPE, "leading dimension smaller than the row");
  if (!aligned16(out) || (res && !aligned16(res)) || (bias && !aligned16(bias)))
    return set_error(SIGLIP2_ERR_ALIGN, "output / residual / bias must be 16-byte aligned");
  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.bias = bias;
  p.k_splits = 1;
  if (workspace != nullptr && epi == kEpiBias && trans_b) {
    const KSplit ks = choose_k_splits(M, N, K);
    if (ks.splits > 1) {
      const size_t need = static_cast<size_t>(ks.splits) * M * N * sizeof(float);
      if (workspace_bytes < need)
        return set_error(SIGLIP2_ERR_ARG, "split-K GEMM needs %zu workspace bytes, got %zu", need, workspace_bytes);
      if (!aligned16(workspace)) return set_error(SIGLIP2_ERR_ALIGN, "workspace must be 16-byte aligned");
      p.k_splits = ks.splits;
      p.k_per_split = ks.k_per_split;
      p.part = static_cast<float*>(workspace);
      p.ld_part = N;
    }
  }
  GemmIO io{a, lda, b, ldb, out, ldo, res, ldr};
  const bool bf = dtype == SIGLIP2_BF16;
  if (!trans_a && !trans_b)
    return sg_gemm_impl(dtype, epi, a, lda, b, ldb, out, ldo, M, N, K, bias, res, ldr, nullptr, nullptr, 0.f, stream);
  if (!trans_a && trans_b)
    return bf ? dispatch_epi_t<__nv_bfloat16, false, true>(epi, io, p, stream)
              : dispatch_epi_t<__half, false, true>(epi, io, p, stream);
  if (trans_a && trans_b)
    return bf ? dispatch_epi_t<__nv_bfloat16, true, true>(epi, io, p, stream)
              : dispatch_epi_t<__half, true, true>(epi, io, p, stream);
  return set_error(SIGLIP2_ERR_UNSUPPORTED, "transposed A with K-major B is not built");
}

// ---------------------------------------------------------------------------
// LayerNorm
// ---------------------------------------------------------------------------
template <typename T>
int launch_layernorm(const void* x, void* y, const float* g, const float* b, int rows, int D, float eps, const int* cu,
                     int P, cudaStream_t s) {
  constexpr int V = Vec16<T>::N;
  SG_CHECK_ARG(D % V == 0, "LayerNorm width %d must be a multiple of %d", D, V);
  const int nvec = D / V;
  const int threads = 256, rows_per_block = threads / 32;
  const int grid = (rows + rows_per_block - 1) / rows_per_block;
  if (rows == 0) return SIGLIP2_OK;
  if (nvec <= 32 * 2)
    layernorm_kernel<T, 2><<<grid, threads, 0, s>>>(static_cast<const T*>(x), static_cast<T*>(y), g, b, rows, D, eps, cu, P);
  else if (nvec <= 32 * 4)
    layernorm_kernel<T, 4><<<grid, threads, 0, s>>>(static_cast<const T*>(x), static_cast<T*>(y), g, b, rows, D, eps, cu, P);
  else if (nvec <= 32 * 8)
    layernorm_kernel<T, 8><<<grid, threads, 0, s>>>(static_cast<const T*>(x), static_cast<T*>(y), g, b, rows, D, eps, cu, P);
  else if (nvec <= 32 * 12)
    layernorm_kernel<T, 12><<<grid, threads, 0, s>>>(static_cast<const T*>(x), static_cast<T*>(y), g, b, rows, D, eps, cu, P);
  else
    return set_error(SIGLIP2_ERR_UNSUPPORTED, "LayerNorm width %d too large", D);
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

int sg_layernorm_impl(int dtype, const void* x, void* y, const float* g, const float* b, int rows, int D, float eps,
                      const int* cu, int P, cudaStream_t s) {
  SG_CHECK_ARG(x && y && g && b && rows >= 0 && D > 0, "bad LayerNorm arguments");
  SG_CHECK_ARG(cu == nullptr || P > 0, "padded LayerNorm needs P > 0");
  if (!aligned16(x) || !aligned16(y) || !aligned16(g) || !aligned16(b))
    return set_error(SIGLIP2_ERR_ALIGN, "LayerNorm tensors and gamma / beta must be 16-byte aligned");
  SG_CHECK_ARG(D % 8 == 0, "LayerNorm width %d must be a multiple of 8", D);
  switch (dtype) {
    case SIGLIP2_BF16: return launch_layernorm<__nv_bfloat16>(x, y, g, b, rows, D, eps, cu, P, s);
    case SIGLIP2_F16: return launch_layernorm<__half>(x, y, g, b, rows, D, eps, cu, P, s);
    case SIGLIP2_F32: return launch_layernorm<float>(x, y, g, b, rows, D, eps, cu, P, s);
    default: return set_error(SIGLIP2_ERR_ARG, "unknown dtype %d", dtype);
  }
}

template <typename T>
int launch_layernorm_bwd(const void* x, const void* dy, const float* g, int rows, int D, float eps, void* dx,
                         float2* stats, float* dg, float* db, int chunk_rows, cudaStream_t s) {
  constexpr int V = Vec16<T>::N;
  const int nvec = D / V;
  const int grid = (rows + 7) / 8;
  const T* xt = static_cast<const T*>(x);
  const T* dyt = static_cast<const T*>(dy);
  T* dxt = static_cast<T*>(dx);
  // vectors per lane: exactly as many as the width needs (registers hold x and dy)
  if (nvec <= 32 * 2) layernorm_bwd_rows_kernel<T, 2><<<grid, 256, 0, s>>>(xt, dyt, g, rows, D, eps, dxt, stats);
  else if (nvec <= 32 * 3) layernorm_bwd_rows_kernel<T, 3><<<grid, 256, 0, s>>>(xt, dyt, g, rows, D, eps, dxt, stats);
  else if (nvec <= 32 * 4) layernorm_bwd_rows_kernel<T, 4><<<grid, 256, 0, s>>>(xt, dyt, g, rows, D, eps, dxt, stats);
  else if (nvec <= 32 * 5) layernorm_bwd_rows_kernel<T, 5><<<grid, 256, 0, s>>>(xt, dyt, g, rows, D, eps, dxt, stats);
  else if (nvec <= 32 * 6) layernorm_bwd_rows_kernel<T, 6><<<grid, 256, 0, s>>>(xt, dyt, g, rows, D, eps, dxt, stats);
  else if (nvec <= 32 * 8) layernorm_bwd_rows_kernel<T, 8><<<grid, 256, 0, s>>>(xt, dyt, g, rows, D, eps, dxt, stats);
  else if (nvec <= 32 * 12) layernorm_bwd_rows_kernel<T, 12><<<grid, 256, 0, s>>>(xt, dyt, g, rows, D, eps, dxt, stats);
  else return set_error(SIGLIP2_ERR_UNSUPPORTED, "LayerNorm width %d too large", D);
  SG_LAUNCH_CHECK();
  const dim3 cgrid((D + 255) / 256, (rows + chunk_rows - 1) / chunk_rows);
  layernorm_bwd_cols_kernel<T><<<cgrid, 256, 0, s>>>(xt, dyt, stats, rows, D, chunk_rows, dg, db);
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

int sg_layernorm_bwd_impl(int dtype, const void* x, const void* dy, const float* gamma, int rows, int D, float eps,
                          void* dx, float* stats, float* dgamma_part, float* dbeta_part, int chunk_rows,
                          cudaStream_t s) {
  SG_CHECK_ARG(x && dy && gamma && dx && stats && dgamma_part && dbeta_part && rows >= 0 && D > 0 && chunk_rows > 0,
               "bad LayerNorm backward arguments");
  SG_CHECK_ARG(D % 8 == 0, "LayerNorm width %d must be a multiple of 8", D);
  if (!aligned16(x) || !aligned16(dy) || !aligned16(dx) || !aligned16(gamma) ||
      (reinterpret_cast<uintptr_t>(stats) & 7u))
    return set_error(SIGLIP2_ERR_ALIGN, "LayerNorm backward: 16-byte aligned rows and gamma, 8-byte aligned stats");
  if (rows == 0) return SIGLIP2_OK;
  float2* st = reinterpret_cast<float2*>(stats);
  switch (dtype) {
    case SIGLIP2_BF16: return launch_layernorm_bwd<__nv_bfloat16>(x, dy, gamma, rows, D, eps, dx, st, dgamma_part, dbeta_part, chunk_rows, s);
    case SIGLIP2_F16: return launch_layernorm_bwd<__half>(x, dy, gamma, rows, D, eps, dx, st, dgamma_part, dbeta_part, chunk_rows, s);
    case SIGLIP2_F32: return launch_layernorm_bwd<float>(x, dy, gamma, rows, D, eps, dx, st, dgamma_part, dbeta_part, chunk_rows, s);
    default: return set_error(SIGLIP2_ERR_ARG, "unknown dtype %d", dtype);
  }
}

// ---------------------------------------------------------------------------
// position-embedding resize into packed token order
// ---------------------------------------------------------------------------
int sg_posemb_impl(int dtype, const float* table, int G, int D, const int* tok_img, const int* hw, const int* cu, int N,
                   void* out, cudaStream_t s) {
  SG_CHECK_ARG(table && tok_img && hw && cu && out && G > 0 && D > 0 && N >= 0, "bad posemb arguments");
  SG_CHECK_ARG(D % 8 == 0 && D / 8 <= 1024, "posemb width %d must be a multiple of 8 and <= 8192", D);
  if (N == 0) return SIGLIP2_OK;
  const int vpt = D / 8;
  const int tpb = vpt >= 256 ? 1 : 256 / vpt;
  dim3 block(vpt, tpb), grid((N + tpb - 1) / tpb);
  switch (dtype) {
    case SIGLIP2_BF16: posemb_kernel<__nv_bfloat16><<<grid, block, 0, s>>>(table, G, D, tok_img, hw, cu, N, static_cast<__nv_bfloat16*>(out)); break;
    case SIGLIP2_F16: posemb_kernel<__half><<<grid, block, 0, s>>>(table, G, D, tok_img, hw, cu, N, static_cast<__half*>(out)); break;
    case SIGLIP2_F32: posemb_kernel<float><<<grid, block, 0, s>>>(table, G, D, tok_img, hw, cu, N, static_cast<float*>(out)); break;
    default: return set_error(SIGLIP2_ERR_ARG, "unknown dtype %d", dtype);
  }
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

int sg_rowsums_impl(int dtype, const void* x, int ldx, int M, int K, float2* rs, cudaStream_t s) {
  SG_CHECK_ARG(x && rs && M >= 0 && K > 0 && ldx >= K, "bad rowsums arguments");
  const bool f32 = dtype == SIGLIP2_F32;
  const int v = f32 ? 4 : 8;
  if (!aligned16(x) || K % v || ldx % v || (reinterpret_cast<uintptr_t>(rs) & 7u))
    return set_error(SIGLIP2_ERR_ALIGN, "rowsums: x 16-byte aligned, K and ldx multiples of %d, rs 8-byte aligned", v);
  if (M == 0) return SIGLIP2_OK;
  const int blk = rowsum_block(f32, K), slots = rowsum_slots(f32, K);
  const dim3 grid((M + 7) / 8);
  switch (dtype) {
    case SIGLIP2_BF16: rowsums_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), ldx, M, K, blk, rs, slots); break;
    case SIGLIP2_F16: rowsums_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(x), ldx, M, K, blk, rs, slots); break;
    case SIGLIP2_F32: rowsums_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(x), ldx, M, K, blk, rs, slots); break;
    default: return set_error(SIGLIP2_ERR_ARG, "unknown dtype %d", dtype);
  }
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

// ---------------------------------------------------------------------------
// 8-bit (e4m3) operands
// ---------------------------------------------------------------------------
int sg_quantize_e4m3_impl(int dtype, const void* x, int ldx, int rows, int cols, void* q, int ldq, float* scale,
                          cudaStream_t s) {
  SG_CHECK_ARG(x && q && scale && rows >= 0 && cols > 0 && ldx >= cols && ldq >= cols, "bad quantize arguments");
  if (!aligned16(x) || !aligned16(q) || cols % 8 || ldx % 8 || ldq % 8)
    return set_error(SIGLIP2_ERR_ALIGN, "quantize: 16-byte aligned x and q, cols, ldx and ldq multiples of 8");
  if (rows == 0) return SIGLIP2_OK;
  const int grid = std::min((rows + 7) / 8, 8 * sm_count());
  uint8_t* qb = static_cast<uint8_t*>(q);
  switch (dtype) {
    case SIGLIP2_BF16: quantize_e4m3_rows_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), ldx, rows, cols, qb, ldq, scale); break;
    case SIGLIP2_F16: quantize_e4m3_rows_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(x), ldx, rows, cols, qb, ldq, scale); break;
    case SIGLIP2_F32: quantize_e4m3_rows_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(x), ldx, rows, cols, qb, ldq, scale); break;
    default: return set_error(SIGLIP2_ERR_ARG, "unknown dtype %d", dtype);
  }
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

template <typename T>
int dispatch_gemm_e4m3(int epi, const GemmIO& io, const GemmParams& p, cudaStream_t s) {
  switch (epi) {
    case kEpiBias: return launch_gemm_tc2<T, 256, kEpiBias, 2, true>(io, p, s);
    case kEpiBiasRes: return launch_gemm_tc2<T, 256, kEpiBiasRes, 2, true>(io, p, s);
    case kEpiBiasGelu: return launch_gemm_tc2<T, 256, kEpiBiasGelu, 2, true>(io, p, s);
    default: return set_error(SIGLIP2_ERR_UNSUPPORTED, "e4m3 GEMM: epilogue %d not supported (0, 1, 4)", epi);
  }
}

// out[M, N] = epilogue(a_scale[m] * b_scale[n] * (A[M, K] . B[N, K]^T)) with
// A, B e4m3 codes (row strides lda / ldb in bytes), on the CTA-pair kernel.
int sg_gemm_e4m3_impl(int out_dtype, int epi, const void* a, int lda, const float* a_scale, const void* b, int ldb,
                      const float* b_scale, void* out, int ldo, int M, int N, int K, const float* bias,
                      const void* res, int ldr, cudaStream_t stream) {
  SG_CHECK_ARG(M >= 0 && N > 0 && K > 0, "bad GEMM shape M=%d N=%d K=%d", M, N, K);
  if (M == 0) return SIGLIP2_OK;
  SG_CHECK_ARG(a && b && out && a_scale && b_scale && bias, "null operand, scale or bias");
  SG_CHECK_ARG(!epi_has_res(epi) || res, "residual epilogue needs res");
  if (out_dtype != SIGLIP2_BF16 && out_dtype != SIGLIP2_F16)
    return set_error(SIGLIP2_ERR_UNSUPPORTED, "e4m3 GEMM writes bf16 or f16 (dtype=%d)", out_dtype);
  if (K % 16 || lda % 16 || ldb % 16 || N % 8 || ldo % 8 || (epi_has_res(epi) && ldr % 8))
    return set_error(SIGLIP2_ERR_ALIGN, "e4m3 GEMM: K, lda, ldb multiples of 16; N, ldo, ldr multiples of 8");
  if (lda < K || ldb < K || ldo < N || (epi_has_res(epi) && ldr < N))
    return set_error(SIGLIP2_ERR_SHAPE, "leading dimension smaller than the row");
  GemmParams p{};
  p.M = M; p.N = N; p.K = K / 2;  // the kernel counts K in 16-bit pairs
  p.bias = bias; p.a_scale = a_scale; p.b_scale = b_scale;
  const GemmIO io{a, lda / 2, b, ldb / 2, out, ldo, res, ldr};
  return out_dtype == SIGLIP2_BF16 ? dispatch_gemm_e4m3<__nv_bfloat16>(epi, io, p, stream)
                                   : dispatch_gemm_e4m3<__half>(epi, io, p, stream);
}

// ---------------------------------------------------------------------------
// image -> patch rows (preprocessing in front of the tower)
// ---------------------------------------------------------------------------
// Patch grid of an H x W image under a patch budget: the binary search over a
// scale factor of transformers' get_image_size_for_max_num_patches
// (models/siglip2/image_processing_siglip2.py), in the same double-precision
// steps so that the grids agree exactly.
static int sg_scaled_side(double scale, int size, int patch) {
  double s = static_cast<double>(size) * scale;
  s = std::ceil(s / patch) * patch;
  if (s < patch) s = patch;
  return static_cast<int>(s);
}

int sg_image_grid(int H, int W, int patch, int max_patches, int* h, int* w) {
  SG_CHECK_ARG(H > 0 && W > 0 && patch > 0 && max_patches > 0 && h && w, "bad image_grid arguments");
  const double eps = 1e-5;
  double lo = eps / 10, hi = 100.0;
  while (hi - lo >= eps) {
    const double mid = (lo + hi) / 2;
    const int th = sg_scaled_side(mid, H, patch), tw = sg_scaled_side(mid, W, patch);
    const double n = (static_cast<double>(th) / patch) * (static_cast<double>(tw) / patch);
    if (n <= max_patches) lo = mid;
    else hi = mid;
  }
  *h = sg_scaled_side(lo, H, patch) / patch;
  *w = sg_scaled_side(lo, W, patch) / patch;
  return SIGLIP2_OK;
}

template <typename T>
int launch_patchify(const PatchifyArgs& a, bool fast, bool any_resize, size_t smem, long long n_rows, void* out,
                    int* mask, cudaStream_t s) {
  T* o = static_cast<T*>(out);
  if (fast) {
    int dev = 0, sms = 148, per_sm = 1;
    SG_CUDA(cudaGetDevice(&dev));
    SG_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    // persistent: exactly the CTAs that are resident at once (one wave)
    SG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, patchify16x3_kernel<T>, 256, 0));
    const long long blocks = std::min<long long>((n_rows + 7) / 8, static_cast<long long>(std::max(per_sm, 1)) * sms);
    patchify16x3_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, s>>>(a, o, mask);
    SG_LAUNCH_CHECK();
    if (!any_resize) return SIGLIP2_OK;
    SG_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(patchify_kernel<T, 3, 16>), static_cast<int>(smem)));
    patchify_kernel<T, 3, 16><<<static_cast<unsigned>(n_rows), kPatchifyThreads, smem, s>>>(a, o, mask);
  } else {
    SG_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(patchify_kernel<T, 0, 0>), static_cast<int>(smem)));
    patchify_kernel<T, 0, 0><<<static_cast<unsigned>(n_rows), kPatchifyThreads, smem, s>>>(a, o, mask);
  }
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

int sg_patchify_impl(int dtype, const uint8_t* images, const long long* offsets_dev, const int* src_hw_host,
                     const int* src_hw_dev, const int* grid_hw_host, const int* grid_hw_dev, int B, int C, int patch,
                     int channels_last, const float* mean, const float* stdv, int max_patches, void* out, int* mask,
                     cudaStream_t s) {
  SG_CHECK_ARG(images && offsets_dev && src_hw_host && src_hw_dev && grid_hw_host && grid_hw_dev && mean && stdv &&
                   out && mask && B > 0 && max_patches > 0,
               "bad patchify arguments");
  SG_CHECK_ARG(C >= 1 && C <= 4, "patchify: 1 to 4 channels (got %d)", C);
  SG_CHECK_ARG(patch >= 1 && patch <= kPatchifyMaxPatch, "patchify: patch side 1..%d (got %d)", kPatchifyMaxPatch,
               patch);
  SG_CHECK_ARG((patch * patch * C) % 8 == 0, "patchify: patch * patch * channels must be a multiple of 8");
  if (!aligned16(out)) return set_error(SIGLIP2_ERR_ALIGN, "pixel_values must be 16-byte aligned");
  PatchifyArgs a{};
  a.images = images;
  a.offsets = offsets_dev;
  a.src_hw = src_hw_dev;
  a.grid_hw = grid_hw_dev;
  a.batch = B;
  a.channels = C;
  a.patch = patch;
  a.channels_last = channels_last ? 1 : 0;
  a.max_patches = max_patches;
  int rows = 1;
  for (int b = 0; b < B; ++b) {
    const int H = src_hw_host[2 * b], W = src_hw_host[2 * b + 1];
    const int h = grid_hw_host[2 * b], w = grid_hw_host[2 * b + 1];
    SG_CHECK_ARG(H > 0 && W > 0 && h > 0 && w > 0, "patchify: image %d has an empty size or grid", b);
    if (static_cast<long long>(h) * w > max_patches)
      return set_error(SIGLIP2_ERR_SHAPE, "patchify: image %d grid %dx%d exceeds %d patches", b, h, w, max_patches);
    const double sy = static_cast<double>(H) / (h * patch), sx = static_cast<double>(W) / (w * patch);
    // taps per axis <= 2 * max(scale, 1) + 2
    if (2 * std::max(sy, 1.0) + 2 > kPatchifyMaxTaps || 2 * std::max(sx, 1.0) + 2 > kPatchifyMaxTaps)
      return set_error(SIGLIP2_ERR_UNSUPPORTED, "patchify: image %d is downscaled more than %dx", b,
                       (kPatchifyMaxTaps - 2) / 2);
    if (H != h * patch || W != w * patch)  // source rows under one patch row: p output rows plus the filter reach
      rows = std::max(rows, static_cast<int>(std::ceil(sy * (patch - 1) + 2 * std::max(sy, 1.0))) + 3);
  }
  rows = std::min(rows, 1 << 20);
  a.max_rows = rows;
  for (int c = 0; c < 4; ++c) {
    a.mean[c] = c < C ? mean[c] : 0.f;
    a.stdv[c] = c < C ? stdv[c] : 1.f;
  }
  const size_t smem = (2 * patch * kPatchifyMaxTaps) * sizeof(float) + 4 * patch * sizeof(int) +
                      static_cast<size_t>(rows) * patch * C * sizeof(float);
  if (smem > static_cast<size_t>(kSmemLimit))
    return set_error(SIGLIP2_ERR_UNSUPPORTED, "patchify: %zu bytes of shared memory needed", smem);
  // 3 x 16 x 16: a warp-per-row kernel for the padded rows and the images
  // already at their grid size, then the resize kernel for the others (if
  // any); other shapes: the general kernel for every row
  const bool fast = C == 3 && patch == 16;
  bool any_resize = false;
  for (int b = 0; b < B; ++b)
    any_resize = any_resize || src_hw_host[2 * b] != grid_hw_host[2 * b] * patch ||
                 src_hw_host[2 * b + 1] != grid_hw_host[2 * b + 1] * patch;
  const long long n_rows = static_cast<long long>(B) * max_patches;
  if (n_rows > (1ll << 31) - 8) return set_error(SIGLIP2_ERR_SHAPE, "patchify: too many rows");
  a.resize_only = fast ? 1 : 0;
  switch (dtype) {
    case SIGLIP2_BF16: return launch_patchify<__nv_bfloat16>(a, fast, any_resize, smem, n_rows, out, mask, s);
    case SIGLIP2_F16: return launch_patchify<__half>(a, fast, any_resize, smem, n_rows, out, mask, s);
    case SIGLIP2_F32: return launch_patchify<float>(a, fast, any_resize, smem, n_rows, out, mask, s);
    default: return set_error(SIGLIP2_ERR_ARG, "unknown dtype %d", dtype);
  }
}

int sg_l2_normalize_impl(int dtype, const void* x, int ldx, int rows, int D, float scale, void* y, int ldy,
                         cudaStream_t s) {
  SG_CHECK_ARG(x && y && rows >= 0 && D > 0 && ldx >= D && ldy >= D, "bad l2_normalize arguments");
  const int v = dtype == SIGLIP2_F32 ? 4 : 8;
  if (!aligned16(x) || !aligned16(y) || D % v || ldx % v || ldy % v)
    return set_error(SIGLIP2_ERR_ALIGN, "l2_normalize: 16-byte aligned rows, D and strides multiples of %d", v);
  if (rows == 0) return SIGLIP2_OK;
  const dim3 grid((rows + 7) / 8);
  switch (dtype) {
    case SIGLIP2_BF16: l2norm_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), ldx, rows, D, scale, static_cast<__nv_bfloat16*>(y), ldy); break;
    case SIGLIP2_F16: l2norm_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(x), ldx, rows, D, scale, static_cast<__half*>(y), ldy); break;
    case SIGLIP2_F32: l2norm_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(x), ldx, rows, D, scale, static_cast<float*>(y), ldy); break;
    default: return set_error(SIGLIP2_ERR_ARG, "unknown dtype %d", dtype);
  }
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

int sg_token_image_impl(const int* cu, int B, int N, int* tok_img, cudaStream_t s) {
  if (N == 0) return SIGLIP2_OK;
  token_image_kernel<<<(N + 255) / 256, 256, 0, s>>>(cu, B, N, tok_img);
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

// ---------------------------------------------------------------------------
// varlen attention
// ---------------------------------------------------------------------------
template <typename T, int HDP>
int launch_fmha(const void* qkv, int N, const int* cu, const int2* tiles, int n_tiles, int H, int hd, void* out, int ldo,
                const DropoutParams& drop, float* lse, cudaStream_t s) {
  using C = FmhaCfg<HDP>;
  CUtensorMap tq, tqr, tk, tkr;
  // 3-D view [N][3H][hd] of the packed q | k | v columns: the remainder box
  // (columns 64 .. HDP of a head) reads zeros past hd, so head_dim 72 is
  // padded to the 80-wide tile in shared memory, not in HBM
  const int64_t row_bytes = 3ll * H * hd * 2;
  SG_TRY(make_tmap_3d(&tq, qkv, 2, hd, 3 * H, N, hd * 2, row_bytes, 64, 1, 128));
  SG_TRY(make_tmap_3d(&tk, qkv, 2, hd, 3 * H, N, hd * 2, row_bytes, 64, 1, C::KT));
  if (HDP > 64) {
    SG_TRY(make_tmap_3d(&tqr, qkv, 2, hd, 3 * H, N, hd * 2, row_bytes, HDP - 64, 1, 128));
    SG_TRY(make_tmap_3d(&tkr, qkv, 2, hd, 3 * H, N, hd * 2, row_bytes, HDP - 64, 1, C::KT));
  } else {
    tqr = tq;
    tkr = tk;
  }
  FmhaParams p;
  p.cu = cu;
  p.tiles = tiles;
  p.n_items = n_tiles * H;
  p.heads = H;
  p.head_dim = hd;
  p.out = out;
  p.ld_out = ldo;
  p.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(hd));
  p.drop = drop;
  p.lse = lse;
  const bool pair = g_fmha_variant.load() == 2;
  auto kern = pair ? fmha_pair_kernel<T, HDP> : fmha_varlen_kernel<T, HDP>;
  const int smem = pair ? FmhaPairCfg<HDP>::kSmem : FmhaCfg<HDP>::kSmem;
  SG_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem));
  // persistent: one CTA per SM walks the (query tile pair, head) items, or
  // (single-tile kernel) two CTAs per SM walk the (query tile, head) items
  const int grid = std::min(p.n_items, (pair ? 1 : 2) * sm_count());
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(pair ? FmhaPairCfg<HDP>::kThreads : 192, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  set_pdl_attr(&attr[0]);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SG_CUDA(cudaLaunchKernelEx(&cfg, kern, tq, tqr, tk, tkr, p));
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

template <typename T>
int dispatch_fmha(const void* qkv, int N, const int* cu, const int2* tiles, int n_tiles, int H, int hd, void* out,
                  int ldo, const DropoutParams& d, float* lse, cudaStream_t s) {
  switch (hd) {
    case 64: return launch_fmha<T, 64>(qkv, N, cu, tiles, n_tiles, H, hd, out, ldo, d, lse, s);
    case 72: return launch_fmha<T, 80>(qkv, N, cu, tiles, n_tiles, H, hd, out, ldo, d, lse, s);
    case 80: return launch_fmha<T, 80>(qkv, N, cu, tiles, n_tiles, H, hd, out, ldo, d, lse, s);
    case 96: return launch_fmha<T, 96>(qkv, N, cu, tiles, n_tiles, H, hd, out, ldo, d, lse, s);
    default: return set_error(SIGLIP2_ERR_UNSUPPORTED, "head_dim %d not supported (64, 72, 80, 96)", hd);
  }
}

// attention backward: the dK/dV pass (key tiles) and the dQ pass (query tiles)
template <typename T, int HDP>
int launch_fmha_bwd(const void* qkv, const void* dout, int ld_dout, int N, const int* cu, const int2* tiles,
                    int n_tiles, int H, int hd, const float* lse, const float* dsum, void* dqkv, cudaStream_t s) {
  CUtensorMap tq, tqr, td, tdr;
  const int64_t row_bytes = 3ll * H * hd * 2;
  SG_TRY(make_tmap_3d(&tq, qkv, 2, hd, 3 * H, N, hd * 2, row_bytes, 64, 1, 128));
  SG_TRY(make_tmap_3d(&td, dout, 2, hd, H, N, hd * 2, static_cast<int64_t>(ld_dout) * 2, 64, 1, 128));
  if (HDP > 64) {
    SG_TRY(make_tmap_3d(&tqr, qkv, 2, hd, 3 * H, N, hd * 2, row_bytes, HDP - 64, 1, 128));
    SG_TRY(make_tmap_3d(&tdr, dout, 2, hd, H, N, hd * 2, static_cast<int64_t>(ld_dout) * 2, HDP - 64, 1, 128));
  } else {
    tqr = tq;
    tdr = td;
  }
  FmhaBwdParams p{};
  p.cu = cu;
  p.tiles = tiles;
  p.n_items = n_tiles * H;
  p.heads = H;
  p.head_dim = hd;
  p.scale = 1.f / sqrtf(static_cast<float>(hd));
  p.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(hd));
  p.lse = lse;
  p.dsum = dsum;
  p.dqkv = dqkv;
  p.ld_dqkv = 3 * H * hd;
  constexpr int smem = FmhaBwdCfg<HDP>::kSmem;
  const int grid = std::min(p.n_items, sm_count());
  auto kkv = fmha_bwd_kernel<T, HDP, false>;
  auto kq = fmha_bwd_kernel<T, HDP, true>;
  SG_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(kkv), smem));
  SG_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(kq), smem));
  kkv<<<grid, 192, smem, s>>>(tq, tqr, td, tdr, p);
  SG_LAUNCH_CHECK();
  kq<<<grid, 192, smem, s>>>(tq, tqr, td, tdr, p);
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

// Dropout parameters from the entry-point arguments (p in [0, 1)).
int make_dropout(float p, unsigned long long seed, unsigned long long offset, DropoutParams* d) {
  SG_CHECK_ARG(p >= 0.f && p < 1.f, "dropout probability %g outside [0, 1)", static_cast<double>(p));
  d->p = p;
  d->scale = 1.f / (1.f - p);
  d->seed_lo = static_cast<uint32_t>(seed);
  d->seed_hi = static_cast<uint32_t>(seed >> 32);
  d->off_lo = static_cast<uint32_t>(offset);
  d->off_hi = static_cast<uint32_t>(offset >> 32);
  return SIGLIP2_OK;
}

int sg_dropout_impl(int dtype, const void* x, int ldx, int rows, int width, const DropoutParams& d, void* y, int ldy,
                    cudaStream_t s) {
  SG_CHECK_ARG(x && y && rows >= 0 && width > 0 && ldx >= width && ldy >= width, "bad dropout arguments");
  SG_CHECK_ARG(width % 8 == 0, "dropout width %d must be a multiple of 8", width);
  const int v = dtype == SIGLIP2_F32 ? 4 : 8;
  if (!aligned16(x) || !aligned16(y) || ldx % v || ldy % v)
    return set_error(SIGLIP2_ERR_ALIGN, "dropout: 16-byte aligned rows with strides multiples of %d", v);
  const long long n = static_cast<long long>(rows) * (width / 8);
  if (n == 0) return SIGLIP2_OK;
  if (n > (1ll << 40)) return set_error(SIGLIP2_ERR_SHAPE, "dropout: too many elements");
  const unsigned blocks = static_cast<unsigned>((n + 255) / 256);
  switch (dtype) {
    case SIGLIP2_BF16: dropout_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), ldx, rows, width, d, static_cast<__nv_bfloat16*>(y), ldy); break;
    case SIGLIP2_F16: dropout_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(x), ldx, rows, width, d, static_cast<__half*>(y), ldy); break;
    case SIGLIP2_F32: dropout_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(x), ldx, rows, width, d, static_cast<float*>(y), ldy); break;
    default: return set_error(SIGLIP2_ERR_ARG, "unknown dtype %d", dtype);
  }
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

int sg_fmha_impl(int dtype, const void* qkv, int N, const int* cu, const int* tiles, int n_tiles, int H, int hd,
                 void* out, int ldo, cudaStream_t s, const DropoutParams* drop = nullptr, float* lse = nullptr) {
  DropoutParams d{};
  if (drop) d = *drop;
  if (lse && dtype == SIGLIP2_F32)
    return set_error(SIGLIP2_ERR_UNSUPPORTED, "attention: the log-sum-exp output is tensor-core (bf16/f16) only");
  SG_CHECK_ARG(qkv && cu && tiles && out && N >= 0 && n_tiles >= 0 && H > 0 && hd > 0, "bad attention arguments");
  SG_CHECK_ARG(hd % 8 == 0 && ldo % 8 == 0 && ldo >= H * hd, "head_dim and ldo must be multiples of 8");
  if (N == 0 || n_tiles == 0) return SIGLIP2_OK;
  if (H > 65535 || static_cast<long long>(n_tiles) * H > (1ll << 30))
    return set_error(SIGLIP2_ERR_UNSUPPORTED, "too many heads or attention tiles");
  if (!aligned16(out)) return set_error(SIGLIP2_ERR_ALIGN, "attention output must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(tiles) & 7u)
    return set_error(SIGLIP2_ERR_ALIGN, "attention tile list must be 8-byte aligned (read as int32 pairs)");
  const int2* t2 = reinterpret_cast<const int2*>(tiles);
  if (dtype == SIGLIP2_BF16) return dispatch_fmha<__nv_bfloat16>(qkv, N, cu, t2, n_tiles, H, hd, out, ldo, d, lse, s);
  if (dtype == SIGLIP2_F16) return dispatch_fmha<__half>(qkv, N, cu, t2, n_tiles, H, hd, out, ldo, d, lse, s);
  if (dtype == SIGLIP2_F32) {
    // fp32: q | k | v with head_dim columns per head (no padding)
    dim3 grid(n_tiles, H);
    const float sc = 1.f / sqrtf(static_cast<float>(hd));
    const float* q = static_cast<const float*>(qkv);
    float* o = static_cast<float*>(out);
    switch (hd) {
      case 64: fmha_f32_kernel<64><<<grid, 128, 0, s>>>(q, cu, t2, H, sc, o, ldo); break;
      case 72: fmha_f32_kernel<72><<<grid, 128, 0, s>>>(q, cu, t2, H, sc, o, ldo); break;
      case 96: fmha_f32_kernel<96><<<grid, 128, 0, s>>>(q, cu, t2, H, sc, o, ldo); break;
      default: return set_error(SIGLIP2_ERR_UNSUPPORTED, "fp32 attention: head_dim %d not supported (64, 72, 96)", hd);
    }
    SG_LAUNCH_CHECK();
    // fp32: the same dropout mask as a second (in-place) launch
    if (d.p > 0.f) return sg_dropout_impl(dtype, out, ldo, N, H * hd, d, out, ldo, s);
    return SIGLIP2_OK;
  }
  return set_error(SIGLIP2_ERR_UNSUPPORTED, "attention supports f32/bf16/f16");
}

// ---------------------------------------------------------------------------
// head + forward
// ---------------------------------------------------------------------------
template <typename T>
int launch_head_pool_parallel(const void* x, int D, int H, const int* cu, int B, int pad_P, const int* tok_img, int N,
                              const float* u, float* scores, void* pooled, cudaStream_t s) {
  const int smem = 16 * D * 4;  // u for 16 heads (zero past H)
  auto ks = head_scores_kernel<T>;
  SG_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(ks), smem));
  // 8 warps of 4 tokens per CTA and sweep; two CTAs per SM
  int blocks = (N + 31) / 32;
  blocks = std::min(blocks, 2 * sm_count());
  if (N > 0) {
    ks<<<blocks, 256, smem, s>>>(static_cast<const T*>(x), D, H, cu, pad_P, tok_img, N, u, scores);
    SG_LAUNCH_CHECK();
  }
  dim3 grid(B, (D + 127) / 128);
  head_pool_rows_kernel<T><<<grid, 128, 0, s>>>(static_cast<const T*>(x), D, H, cu, pad_P, scores,
                                                static_cast<T*>(pooled));
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

// Parallel pooling (scores over all tokens, then per (image, 64 columns)).
// tok_img (token -> image) is needed only when the hidden state is padded.
int sg_head_pool_parallel(int dtype, const void* x, int D, int H, const int* cu, int B, int pad_P, const int* tok_img,
                          int N, const float* u, float* scores, void* pooled, cudaStream_t s) {
  SG_CHECK_ARG(H <= 16 && D % 8 == 0, "head pooling needs H <= 16 and D %% 8 == 0");
  SG_CHECK_ARG(pad_P == 0 || tok_img != nullptr, "padded head pooling needs the token -> image map");
  switch (dtype) {
    case SIGLIP2_BF16: return launch_head_pool_parallel<__nv_bfloat16>(x, D, H, cu, B, pad_P, tok_img, N, u, scores, pooled, s);
    case SIGLIP2_F16: return launch_head_pool_parallel<__half>(x, D, H, cu, B, pad_P, tok_img, N, u, scores, pooled, s);
    case SIGLIP2_F32: return launch_head_pool_parallel<float>(x, D, H, cu, B, pad_P, tok_img, N, u, scores, pooled, s);
    default: return set_error(SIGLIP2_ERR_ARG, "unknown dtype %d", dtype);
  }
}

int sg_head_pool_impl(int dtype, const void* x, int D, int H, const int* cu, int B, int pad_P, const float* u,
                      float* scores, int score_rows, void* pooled, cudaStream_t s) {
  SG_CHECK_ARG(H % 4 == 0 && H <= 16 && D % 8 == 0, "head pooling needs H %% 4 == 0, H <= 16, D %% 8 == 0");
  const int threads = (D / 8) * (H / 4);
  SG_CHECK_ARG(threads <= 1024, "head pooling: D=%d H=%d needs too many threads", D, H);
  const int smem = (H * D + 2 * H) * 4;
  int nt = threads < 128 ? 128 : (threads + 31) / 32 * 32;
  switch (dtype) {
    case SIGLIP2_BF16: {
      auto k = head_pool_kernel<__nv_bfloat16>;
      SG_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(k), smem));
      k<<<B, nt, smem, s>>>(static_cast<const __nv_bfloat16*>(x), D, H, cu, pad_P, u, scores, score_rows,
                             static_cast<__nv_bfloat16*>(pooled));
      break;
    }
    case SIGLIP2_F16: {
      auto k = head_pool_kernel<__half>;
      SG_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(k), smem));
      k<<<B, nt, smem, s>>>(static_cast<const __half*>(x), D, H, cu, pad_P, u, scores, score_rows,
                             static_cast<__half*>(pooled));
      break;
    }
    case SIGLIP2_F32: {
      auto k = head_pool_kernel<float>;
      SG_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(k), smem));
      k<<<B, nt, smem, s>>>(static_cast<const float*>(x), D, H, cu, pad_P, u, scores, score_rows,
                             static_cast<float*>(pooled));
      break;
    }
    default: return set_error(SIGLIP2_ERR_ARG, "unknown dtype %d", dtype);
  }
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

template <typename T>
int launch_select(const void* Y, int H, int hd, int D, int B, void* out, cudaStream_t s) {
  const int n = B * (D / 8);
  head_select_kernel<T><<<(n + 255) / 256, 256, 0, s>>>(static_cast<const T*>(Y), H, hd, D, B, static_cast<T*>(out));
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

template <typename T>
int launch_gather(const void* padded, int C, int P, const int* cu, const int* tok, int N, void* packed, cudaStream_t s) {
  const size_t n = static_cast<size_t>(N) * (C / (16 / sizeof(T)));
  if (n == 0) return SIGLIP2_OK;
  gather_rows_kernel<T><<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(static_cast<const T*>(padded), C, P, cu, tok, N,
                                                                       static_cast<T*>(packed));
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

int validate_config(const siglip2_config* c) {
  SG_CHECK_ARG(c != nullptr, "null config");
  SG_CHECK_ARG(c->hidden > 0 && c->intermediate > 0 && c->layers >= 0 && c->heads > 0 && c->patch_dim > 0 &&
                   c->pos_grid > 0,
               "non-positive config field");
  SG_CHECK_ARG(c->head_dim * c->heads == c->hidden, "head_dim * heads != hidden");
  if (c->dtype != SIGLIP2_BF16 && c->dtype != SIGLIP2_F16 && c->dtype != SIGLIP2_F32)
    return set_error(SIGLIP2_ERR_UNSUPPORTED, "forward supports f32, bf16 and f16 (dtype %d)", c->dtype);
  if (c->hidden % 64 || c->intermediate % 8 || c->patch_dim % 8)
    return set_error(SIGLIP2_ERR_UNSUPPORTED, "hidden must be a multiple of 64, intermediate/patch_dim of 8");
  if (c->head_dim != 64 && c->head_dim != 72 && c->head_dim != 80 && c->head_dim != 96)
    return set_error(SIGLIP2_ERR_UNSUPPORTED, "head_dim %d not supported (64, 72, 80, 96)", c->head_dim);
  return SIGLIP2_OK;
}

int sg_forward_impl(const siglip2_config* c, const siglip2_weights* w, const void* patches, int B, int P,
                    const int32_t* hw_host, const int32_t* meta, void* last_hidden, void* pooled, void* ws,
                    size_t ws_bytes, cudaStream_t s) {
  SG_TRY(validate_config(c));
  SG_CHECK_ARG(w && patches && hw_host && meta && last_hidden && ws && B > 0 && P >= 0, "null forward argument");
  SG_CHECK_ARG(!pooled || c->has_head, "pooled output requested but the model has no head");
  int N = 0, T = 0;
  SG_TRY(meta_counts(hw_host, B, &N, &T));
  for (int b = 0; b < B && P > 0; ++b)
    if (hw_host[2 * b] * hw_host[2 * b + 1] > P)
      return set_error(SIGLIP2_ERR_SHAPE, "image %d: h*w = %d exceeds max_patches %d", b,
                       hw_host[2 * b] * hw_host[2 * b + 1], P);
  const size_t need = forward_workspace(c, B, N, nullptr, nullptr);
  if (ws_bytes < need) return set_error(SIGLIP2_ERR_ARG, "workspace too small: %zu < %zu bytes", ws_bytes, need);
  if (!aligned16(patches) || !aligned16(last_hidden) || (pooled && !aligned16(pooled)) || !aligned16(ws) ||
      (reinterpret_cast<uintptr_t>(meta) & 7u))
    return set_error(SIGLIP2_ERR_ALIGN, "forward buffers must be 16-byte aligned");
  FwdBuffers f;
  forward_workspace(c, B, N, &f, static_cast<uint8_t*>(ws));
  const int* cu = meta;
  const int* hw = meta + B + 1;
  const int* tiles = meta + meta_tiles_offset(B);
  const int dt = c->dtype;
  const int D = c->hidden, I = c->intermediate, H = c->heads, hd = c->head_dim;
  const int nqkv = 3 * H * hd;  // q | k | v, heads of head_dim columns (unpadded)

  // Row sums of the residual stream for the LayerNorm-folded GEMMs, in
  // slots written by the GEMM that writes x: two buffers alternate (x after
  // the embeddings / fc2 -> rs_b, after out-proj -> rs_a); every slot is
  // written before it is read, so nothing is cleared.
  const size_t rs_n = static_cast<size_t>(N) * rowsum_slots(dt == SIGLIP2_F32, D);
  float2* rs_a = f.rowsums;
  float2* rs_b = f.rowsums + rs_n;
  // embeddings: x = patches Wp^T + bp + resized position grid, one GEMM whose
  // epilogue evaluates the antialiased resize per token (and the row sums)
  SG_TRY(sg_token_image_impl(cu, B, N, f.tok_img, s));
  const void* prow = patches;
  if (P > 0) {
    if (dt == SIGLIP2_BF16) SG_TRY(launch_gather<__nv_bfloat16>(patches, c->patch_dim, P, cu, f.tok_img, N, f.hmid, s));
    else if (dt == SIGLIP2_F16) SG_TRY(launch_gather<__half>(patches, c->patch_dim, P, cu, f.tok_img, N, f.hmid, s));
    else SG_TRY(launch_gather<float>(patches, c->patch_dim, P, cu, f.tok_img, N, f.hmid, s));
    prow = f.hmid;
  }
  const PosArgs pos{w->pos_table, c->pos_grid, f.tok_img, hw, cu};
  SG_TRY(sg_gemm_impl(dt, kEpiBiasPosRs, prow, c->patch_dim, w->patch_w, c->patch_dim, f.x, D, N, D, c->patch_dim,
                      w->patch_b, nullptr, 0, nullptr, nullptr, 0.f, s, nullptr, rs_b, &pos));
  for (int l = 0; l < c->layers; ++l) {
    const siglip2_layer_weights& lw = w->layers[l];
    SG_TRY(sg_gemm_impl(dt, kEpiLnRs, f.x, D, lw.qkv_w, D, f.qkv, nqkv, N, nqkv, D, nullptr, nullptr, 0, lw.qkv_c1,
                        lw.qkv_c2, c->eps, s, rs_b, nullptr));
    SG_TRY(sg_fmha_impl(dt, f.qkv, N, cu, tiles, T, H, hd, f.attn, D, s));
    SG_TRY(sg_gemm_impl(dt, kEpiBiasResRs, f.attn, D, lw.out_w, D, f.x, D, N, D, D, lw.out_b, f.x, D, nullptr,
                        nullptr, 0.f, s, nullptr, rs_a));
    SG_TRY(sg_gemm_impl(dt, kEpiLnRsGelu, f.x, D, lw.fc1_w, D, f.hmid, I, N, I, D, nullptr, nullptr, 0, lw.fc1_c1,
                        lw.fc1_c2, c->eps, s, rs_a, nullptr));
    SG_TRY(sg_gemm_impl(dt, kEpiBiasResRs, f.hmid, I, lw.fc2_w, I, f.x, D, N, D, I, lw.fc2_b, f.x, D, nullptr,
                        nullptr, 0.f, s, nullptr, rs_b));
  }
  // post-LayerNorm -> last_hidden_state (packed or padded with zero rows)
  SG_TRY(sg_layernorm_impl(dt, f.x, last_hidden, w->post_ln_w, w->post_ln_b, P > 0 ? B * P : N, D, c->eps,
                           P > 0 ? cu : nullptr, P, s));
  if (pooled) {
    SG_TRY(sg_head_pool_parallel(dt, last_hidden, D, H, cu, B, P, f.tok_img, N, w->head_u, f.scores, f.hpool, s));
    SG_TRY(sg_gemm_impl(dt, kEpiBias, f.hpool, D, w->head_v_w, D, f.hY, D, B * H, D, D, w->head_v_b, nullptr, 0,
                        nullptr, nullptr, 0.f, s));
    if (dt == SIGLIP2_BF16) SG_TRY(launch_select<__nv_bfloat16>(f.hY, H, hd, D, B, f.hattn, s));
    else if (dt == SIGLIP2_F16) SG_TRY(launch_select<__half>(f.hY, H, hd, D, B, f.hattn, s));
    else SG_TRY(launch_select<float>(f.hY, H, hd, D, B, f.hattn, s));
    SG_TRY(sg_gemm_impl(dt, kEpiBias, f.hattn, D, w->head_o_w, D, f.ha, D, B, D, D, w->head_o_b, nullptr, 0, nullptr,
                        nullptr, 0.f, s));
    if (dt == SIGLIP2_F32) {
      rowsums_f32_kernel<<<(B + 7) / 8, 256, 0, s>>>(static_cast<const float*>(f.ha), B, D, rs_a,
                                                      rowsum_slots(true, D));
      SG_LAUNCH_CHECK();
      SG_TRY(sg_gemm_impl(dt, kEpiLnRsGelu, f.ha, D, w->head_fc1_w, D, f.hmid2, I, B, I, D, nullptr, nullptr, 0,
                          w->head_fc1_c1, w->head_fc1_c2, c->eps, s, rs_a, nullptr));
    } else {
      SG_TRY(sg_gemm_impl(dt, kEpiLnGelu, f.ha, D, w->head_fc1_w, D, f.hmid2, I, B, I, D, nullptr, nullptr, 0,
                          w->head_fc1_c1, w->head_fc1_c2, c->eps, s));
    }
    SG_TRY(sg_gemm_impl(dt, kEpiBiasRes, f.hmid2, I, w->head_fc2_w, I, pooled, D, B, D, I, w->head_fc2_b, f.ha, D,
                        nullptr, nullptr, 0.f, s));
  }
  return SIGLIP2_OK;
}

// ---------------------------------------------------------------------------
// Head pooling with no allocation at all.
//
// Some callers cannot allocate device memory when they call in: inference
// servers that carve one fixed arena at start-up and forbid any allocation
// afterwards, and plain C / FFI hosts that have no caching allocator, where a
// cudaMalloc per call would synchronise the device and stall other streams.
// For them the per-token score scratch of the pooling kernel lives in this
// fixed device array instead of caller memory.  It is reserved on every GPU
// that loads the library and held until the process exits.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocScoreCapacity = size_t(1) << 20;  // floats: 4 MiB, e.g. 65,536 tokens x 16 heads
static __device__ __align__(256) float g_noalloc_scores[kNoAllocScoreCapacity];

namespace {
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of g_noalloc_scores on the current device.  In host code the
// array's name is only a host-side stand-in, so the address is looked up once
// per device (with that device current) and cached.
int noalloc_scores_ptr(float** out) {
  int dev = 0;
  SG_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return set_error(SIGLIP2_ERR_UNSUPPORTED, "device ordinal %d beyond %d", dev, kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    SG_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scores));
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return SIGLIP2_OK;
}
}  // namespace

extern "C" {

int siglip2_version(void) { return 100; }

const char* siglip2_last_error(void) { return t_last_error; }

unsigned long long siglip2_launch_count(void) { return launch_counter().load(); }

int siglip2_selftest_wait_timeout(long long limit_ns, void* stream) {
  SG_CHECK_ARG(limit_ns > 0 && limit_ns <= 2000000000ll, "limit must be in (0, 2 s]");
  selftest_wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<unsigned long long>(limit_ns), 901);
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

int siglip2_set_gemm_variant(int variant) {
  SG_CHECK_ARG(variant >= 0 && variant <= 2, "GEMM variant must be 0 (auto), 1 (1-SM) or 2 (SM pairs)");
  g_gemm_variant.store(variant);
  return SIGLIP2_OK;
}

int siglip2_get_gemm_variant(void) { return g_gemm_variant.load(); }

int siglip2_set_fmha_variant(int variant) {
  SG_CHECK_ARG(variant >= 0 && variant <= 2, "attention variant must be 0 (auto), 1 (single tile) or 2 (tile pairs)");
  g_fmha_variant.store(variant);
  return SIGLIP2_OK;
}

int siglip2_get_fmha_variant(void) { return g_fmha_variant.load(); }

int siglip2_check_device(int reset) {
  SG_CUDA(cudaDeviceSynchronize());
  int flag = 0;
  SG_CUDA(cudaMemcpyFromSymbol(&flag, g_device_error, sizeof(int)));
  if (reset && flag) {
    const int zero = 0;
    SG_CUDA(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)));
  }
  if (flag >= kSiteBoundsFirst)
    return set_error(SIGLIP2_ERR_SHAPE, "a kernel skipped an index outside the buffer it was given (site %d)", flag);
  if (flag) return set_error(SIGLIP2_ERR_TIMEOUT, "a kernel gave up on a bounded wait (site %d)", flag);
  return SIGLIP2_OK;
}

int siglip2_gemm(int dtype, int epilogue, const void* a_dev, int lda, const void* b_dev, int ldb, void* out_dev,
                 int ldo, int M, int N, int K, const float* bias_dev, const void* res_dev, int ldr,
                 const float* c1_dev, const float* c2_dev, float eps, void* stream) {
  return sg_gemm_impl(dtype, epilogue, a_dev, lda, b_dev, ldb, out_dev, ldo, M, N, K, bias_dev, res_dev, ldr, c1_dev,
                      c2_dev, eps, static_cast<cudaStream_t>(stream));
}

int siglip2_gemm_t(int dtype, int epilogue, int trans_a, int trans_b, const void* a_dev, int lda, const void* b_dev,
                   int ldb, void* out_dev, int ldo, int M, int N, int K, const float* bias_dev, const void* res_dev,
                   int ldr, void* stream) {
  return sg_gemm_t_impl(dtype, epilogue, trans_a, trans_b, a_dev, lda, b_dev, ldb, out_dev, ldo, M, N, K, bias_dev,
                        res_dev, ldr, static_cast<cudaStream_t>(stream));
}

int siglip2_colsum_partial(int dtype, const void* x_dev, int ld, int rows, int cols, int chunk_rows, float* part_dev,
                           void* stream) {
  SG_CHECK_ARG(x_dev && part_dev && rows >= 0 && cols > 0 && ld >= cols && chunk_rows > 0, "bad colsum arguments");
  if (!aligned16(x_dev) || cols % 8 || ld % 8)
    return set_error(SIGLIP2_ERR_ALIGN, "colsum: x 16-byte aligned, cols and ld multiples of 8");
  if (rows == 0) return SIGLIP2_OK;
  const dim3 grid((cols + 255) / 256, (rows + chunk_rows - 1) / chunk_rows);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SIGLIP2_BF16: colsum_part_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x_dev), ld, rows, cols, chunk_rows, part_dev); break;
    case SIGLIP2_F16: colsum_part_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(x_dev), ld, rows, cols, chunk_rows, part_dev); break;
    case SIGLIP2_F32: colsum_part_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(x_dev), ld, rows, cols, chunk_rows, part_dev); break;
    default: return set_error(SIGLIP2_ERR_ARG, "unknown dtype %d", dtype);
  }
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

size_t siglip2_gemm_t_workspace_size(int epilogue, int trans_a, int trans_b, int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0 || epilogue != kEpiBias || !trans_b) return 0;
  (void)trans_a;
  const KSplit ks = choose_k_splits(M, N, K);
  return ks.splits > 1 ? static_cast<size_t>(ks.splits) * M * N * sizeof(float) : 0;
}

int siglip2_gemm_t_ws(int dtype, int epilogue, int trans_a, int trans_b, const void* a_dev, int lda, const void* b_dev,
                      int ldb, void* out_dev, int ldo, int M, int N, int K, const float* bias_dev, void* workspace_dev,
                      size_t workspace_bytes, void* stream) {
  return sg_gemm_t_impl(dtype, epilogue, trans_a, trans_b, a_dev, lda, b_dev, ldb, out_dev, ldo, M, N, K, bias_dev,
                        nullptr, 0, static_cast<cudaStream_t>(stream), workspace_dev, workspace_bytes);
}

int siglip2_quantize_e4m3(int dtype, const void* x_dev, int ldx, int rows, int cols, void* q_dev, int ldq,
                          float* scale_dev, void* stream) {
  return sg_quantize_e4m3_impl(dtype, x_dev, ldx, rows, cols, q_dev, ldq, scale_dev, static_cast<cudaStream_t>(stream));
}

int siglip2_gemm_e4m3(int out_dtype, int epilogue, const void* a_dev, int lda, const float* a_scale_dev,
                      const void* b_dev, int ldb, const float* b_scale_dev, void* out_dev, int ldo, int M, int N, int K,
                      const float* bias_dev, const void* res_dev, int ldr, void* stream) {
  return sg_gemm_e4m3_impl(out_dtype, epilogue, a_dev, lda, a_scale_dev, b_dev, ldb, b_scale_dev, out_dev, ldo, M, N,
                           K, bias_dev, res_dev, ldr, static_cast<cudaStream_t>(stream));
}

int siglip2_rowsum_slots(int dtype, int n) {
  SG_CHECK_ARG(n > 0, "bad row width %d", n);
  return rowsum_slots(dtype == SIGLIP2_F32, n);
}

int siglip2_rowsum_block(int dtype, int n) {
  SG_CHECK_ARG(n > 0, "bad row width %d", n);
  return rowsum_block(dtype == SIGLIP2_F32, n);
}

int siglip2_rowsums(int dtype, const void* x_dev, int ldx, int M, int K, float* rs_dev, void* stream) {
  return sg_rowsums_impl(dtype, x_dev, ldx, M, K, reinterpret_cast<float2*>(rs_dev),
                         static_cast<cudaStream_t>(stream));
}

int siglip2_gemm_rowsums(int dtype, int epilogue, const void* a_dev, int lda, const void* b_dev, int ldb,
                         void* out_dev, int ldo, int M, int N, int K, const float* bias_dev, const void* res_dev,
                         int ldr, const float* c1_dev, const float* c2_dev, float eps, const float* rs_in_dev,
                         float* rs_acc_dev, void* stream) {
  return sg_gemm_impl(dtype, epilogue, a_dev, lda, b_dev, ldb, out_dev, ldo, M, N, K, bias_dev, res_dev, ldr, c1_dev,
                      c2_dev, eps, static_cast<cudaStream_t>(stream), reinterpret_cast<const float2*>(rs_in_dev),
                      reinterpret_cast<float2*>(rs_acc_dev));
}

int siglip2_patch_embed(int dtype, const void* patches_dev, int patch_dim, const void* w_dev, const float* bias_dev,
                        const float* table_dev, int grid, const int* tok_img_dev, const int* hw_dev,
                        const int* cu_seqlens_dev, int N, int D, void* out_dev, float* rs_acc_dev, void* stream) {
  SG_CHECK_ARG(patches_dev && w_dev && bias_dev && out_dev && rs_acc_dev && N >= 0 && D > 0 && patch_dim > 0,
               "bad patch_embed arguments");
  const PosArgs pos{table_dev, grid, tok_img_dev, hw_dev, cu_seqlens_dev};
  return sg_gemm_impl(dtype, kEpiBiasPosRs, patches_dev, patch_dim, w_dev, patch_dim, out_dev, D, N, D, patch_dim,
                      bias_dev, nullptr, 0, nullptr, nullptr, 0.f, static_cast<cudaStream_t>(stream), nullptr,
                      reinterpret_cast<float2*>(rs_acc_dev), &pos);
}

int siglip2_layernorm(int dtype, const void* x_dev, void* y_dev, const float* gamma_dev, const float* beta_dev,
                      int rows, int D, float eps, const int* cu_seqlens_dev, int max_patches, void* stream) {
  return sg_layernorm_impl(dtype, x_dev, y_dev, gamma_dev, beta_dev, rows, D, eps, cu_seqlens_dev, max_patches,
                           static_cast<cudaStream_t>(stream));
}

int siglip2_layernorm_backward(int dtype, const void* x_dev, const void* dy_dev, const float* gamma_dev, int rows,
                               int D, float eps, void* dx_dev, float* stats_dev, float* dgamma_part_dev,
                               float* dbeta_part_dev, int chunk_rows, void* stream) {
  return sg_layernorm_bwd_impl(dtype, x_dev, dy_dev, gamma_dev, rows, D, eps, dx_dev, stats_dev, dgamma_part_dev,
                               dbeta_part_dev, chunk_rows, static_cast<cudaStream_t>(stream));
}

int siglip2_image_grid(int height, int width, int patch, int max_patches, int* grid_h, int* grid_w) {
  return sg_image_grid(height, width, patch, max_patches, grid_h, grid_w);
}

int siglip2_patchify(int dtype, const uint8_t* images_dev, const long long* offsets_dev, const int* src_hw_host,
                     const int* src_hw_dev, const int* grid_hw_host, const int* grid_hw_dev, int batch, int channels,
                     int patch, int channels_last, const float* mean, const float* std_dev_values, int max_patches,
                     void* pixel_values_dev, int* mask_dev, void* stream) {
  return sg_patchify_impl(dtype, images_dev, offsets_dev, src_hw_host, src_hw_dev, grid_hw_host, grid_hw_dev, batch,
                          channels, patch, channels_last, mean, std_dev_values, max_patches, pixel_values_dev,
                          mask_dev, static_cast<cudaStream_t>(stream));
}

int siglip2_l2_normalize(int dtype, const void* x_dev, int ldx, int rows, int D, float scale, void* y_dev, int ldy,
                         void* stream) {
  return sg_l2_normalize_impl(dtype, x_dev, ldx, rows, D, scale, y_dev, ldy, static_cast<cudaStream_t>(stream));
}

int siglip2_token_image(const int* cu_seqlens_dev, int B, int N, int* tok_img_dev, void* stream) {
  SG_CHECK_ARG(cu_seqlens_dev && tok_img_dev && B > 0 && N >= 0, "bad token_image arguments");
  return sg_token_image_impl(cu_seqlens_dev, B, N, tok_img_dev, static_cast<cudaStream_t>(stream));
}

int siglip2_posemb(int dtype, const float* table_dev, int grid, int D, const int* tok_img_dev, const int* hw_dev,
                   const int* cu_seqlens_dev, int N, void* out_dev, void* stream) {
  return sg_posemb_impl(dtype, table_dev, grid, D, tok_img_dev, hw_dev, cu_seqlens_dev, N, out_dev,
                        static_cast<cudaStream_t>(stream));
}

int siglip2_fmha_varlen(int dtype, const void* qkv_dev, int N, const int* cu_seqlens_dev, const int* tiles_dev,
                        int n_tiles, int heads, int head_dim, void* out_dev, int ldo, void* stream) {
  return sg_fmha_impl(dtype, qkv_dev, N, cu_seqlens_dev, tiles_dev, n_tiles, heads, head_dim, out_dev, ldo,
                      static_cast<cudaStream_t>(stream));
}

int siglip2_fmha_varlen_dropout(int dtype, const void* qkv_dev, int N, const int* cu_seqlens_dev, const int* tiles_dev,
                                int n_tiles, int heads, int head_dim, void* out_dev, int ldo, float p,
                                unsigned long long seed, unsigned long long offset, void* stream) {
  DropoutParams d{};
  SG_TRY(make_dropout(p, seed, offset, &d));
  return sg_fmha_impl(dtype, qkv_dev, N, cu_seqlens_dev, tiles_dev, n_tiles, heads, head_dim, out_dev, ldo,
                      static_cast<cudaStream_t>(stream), &d);
}

int siglip2_fmha_varlen_train(int dtype, const void* qkv_dev, int N, const int* cu_seqlens_dev, const int* tiles_dev,
                              int n_tiles, int heads, int head_dim, void* out_dev, int ldo, float* lse_dev, float p,
                              unsigned long long seed, unsigned long long offset, void* stream) {
  SG_CHECK_ARG(lse_dev != nullptr, "the training forward needs the log-sum-exp output");
  if (reinterpret_cast<uintptr_t>(lse_dev) & 3u) return set_error(SIGLIP2_ERR_ALIGN, "lse must be 4-byte aligned");
  DropoutParams d{};
  SG_TRY(make_dropout(p, seed, offset, &d));
  return sg_fmha_impl(dtype, qkv_dev, N, cu_seqlens_dev, tiles_dev, n_tiles, heads, head_dim, out_dev, ldo,
                      static_cast<cudaStream_t>(stream), &d, lse_dev);
}

int siglip2_fmha_bwd_dsum(int dtype, const void* g_dev, const void* o_dev, int ld, int N, int heads, int head_dim,
                          float* dsum_dev, void* stream) {
  SG_CHECK_ARG(g_dev && o_dev && dsum_dev && N >= 0 && heads > 0 && head_dim > 0 && ld >= heads * head_dim,
               "bad attention-backward row-dot arguments");
  const int v = dtype == SIGLIP2_F32 ? 4 : 8;
  if (head_dim % 8 || ld % v || !aligned16(g_dev) || !aligned16(o_dev))
    return set_error(SIGLIP2_ERR_ALIGN, "row-dot: head_dim a multiple of 8, 16-byte aligned rows");
  const long long n = static_cast<long long>(N) * heads;
  if (n == 0) return SIGLIP2_OK;
  const unsigned blocks = static_cast<unsigned>((n + 255) / 256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SIGLIP2_BF16: fmha_bwd_dsum_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(g_dev), static_cast<const __nv_bfloat16*>(o_dev), ld, N, heads, head_dim, dsum_dev); break;
    case SIGLIP2_F16: fmha_bwd_dsum_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(g_dev), static_cast<const __half*>(o_dev), ld, N, heads, head_dim, dsum_dev); break;
    case SIGLIP2_F32: fmha_bwd_dsum_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(g_dev), static_cast<const float*>(o_dev), ld, N, heads, head_dim, dsum_dev); break;
    default: return set_error(SIGLIP2_ERR_ARG, "unknown dtype %d", dtype);
  }
  SG_LAUNCH_CHECK();
  return SIGLIP2_OK;
}

int siglip2_fmha_varlen_backward(int dtype, const void* qkv_dev, const void* dout_dev, int ld_dout, int N,
                                 const int* cu_seqlens_dev, const int* tiles_dev, int n_tiles, int heads,
                                 int head_dim, const float* lse_dev, const float* dsum_dev, void* dqkv_dev,
                                 void* stream) {
  SG_CHECK_ARG(qkv_dev && dout_dev && cu_seqlens_dev && tiles_dev && lse_dev && dsum_dev && dqkv_dev && N >= 0 &&
                   n_tiles >= 0 && heads > 0,
               "bad attention backward arguments");
  if (dtype != SIGLIP2_BF16 && dtype != SIGLIP2_F16)
    return set_error(SIGLIP2_ERR_UNSUPPORTED, "attention backward: bf16 / f16 only");
  if (ld_dout % 8 || ld_dout < heads * head_dim || !aligned16(dout_dev) || !aligned16(dqkv_dev) ||
      (reinterpret_cast<uintptr_t>(tiles_dev) & 7u))
    return set_error(SIGLIP2_ERR_ALIGN, "attention backward: 16-byte aligned rows and pitches, 8-byte aligned tiles");
  if (N == 0 || n_tiles == 0) return SIGLIP2_OK;
  if (heads > 65535 || static_cast<long long>(n_tiles) * heads > (1ll << 30))
    return set_error(SIGLIP2_ERR_UNSUPPORTED, "too many heads or attention tiles");
  const int2* t2 = reinterpret_cast<const int2*>(tiles_dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf = dtype == SIGLIP2_BF16;
  switch (head_dim) {
    case 64: return bf ? launch_fmha_bwd<__nv_bfloat16, 64>(qkv_dev, dout_dev, ld_dout, N, cu_seqlens_dev, t2, n_tiles, heads, head_dim, lse_dev, dsum_dev, dqkv_dev, s)
                       : launch_fmha_bwd<__half, 64>(qkv_dev, dout_dev, ld_dout, N, cu_seqlens_dev, t2, n_tiles, heads, head_dim, lse_dev, dsum_dev, dqkv_dev, s);
    case 72: return bf ? launch_fmha_bwd<__nv_bfloat16, 80>(qkv_dev, dout_dev, ld_dout, N, cu_seqlens_dev, t2, n_tiles, heads, head_dim, lse_dev, dsum_dev, dqkv_dev, s)
                       : launch_fmha_bwd<__half, 80>(qkv_dev, dout_dev, ld_dout, N, cu_seqlens_dev, t2, n_tiles, heads, head_dim, lse_dev, dsum_dev, dqkv_dev, s);
    case 96: return bf ? launch_fmha_bwd<__nv_bfloat16, 96>(qkv_dev, dout_dev, ld_dout, N, cu_seqlens_dev, t2, n_tiles, heads, head_dim, lse_dev, dsum_dev, dqkv_dev, s)
                       : launch_fmha_bwd<__half, 96>(qkv_dev, dout_dev, ld_dout, N, cu_seqlens_dev, t2, n_tiles, heads, head_dim, lse_dev, dsum_dev, dqkv_dev, s);
    default: return set_error(SIGLIP2_ERR_UNSUPPORTED, "attention backward: head_dim %d not supported (64, 72, 96)", head_dim);
  }
}

int siglip2_dropout(int dtype, const void* x_dev, int ldx, int rows, int width, float p, unsigned long long seed,
                    unsigned long long offset, void* y_dev, int ldy, void* stream) {
  DropoutParams d{};
  SG_TRY(make_dropout(p, seed, offset, &d));
  return sg_dropout_impl(dtype, x_dev, ldx, rows, width, d, y_dev, ldy, static_cast<cudaStream_t>(stream));
}

int siglip2_padded_head_dim(int head_dim) { return padded_head_dim(head_dim); }

int siglip2_head_pool_noalloc(int dtype, const void* x_dev, int D, int heads, const int* cu_seqlens_dev, int B,
                              int max_patches, int n_tokens, const float* u_dev, void* pooled_dev, void* stream) {
  SG_CHECK_ARG(x_dev && cu_seqlens_dev && u_dev && pooled_dev && B > 0 && max_patches >= 0 && n_tokens >= 0 &&
                   heads > 0,
               "bad head_pool_noalloc arguments");
  if (static_cast<size_t>(n_tokens) * static_cast<size_t>(heads) > kNoAllocScoreCapacity)
    return set_error(SIGLIP2_ERR_SHAPE,
                     "head_pool_noalloc: %d tokens x %d heads needs %zu score floats, the fixed scratch holds %zu",
                     n_tokens, heads, static_cast<size_t>(n_tokens) * heads, kNoAllocScoreCapacity);
  if (!aligned16(x_dev) || !aligned16(pooled_dev))
    return set_error(SIGLIP2_ERR_ALIGN, "head_pool tensors must be 16-byte aligned");
  float* scores = nullptr;
  SG_TRY(noalloc_scores_ptr(&scores));
  // the kernel writes score rows cu[b] .. cu[b+1]-1 only when they lie below
  // n_tokens (checked above to fit the fixed array); an image past it is
  // skipped and reported by siglip2_check_device as SIGLIP2_ERR_SHAPE
  return sg_head_pool_impl(dtype, x_dev, D, heads, cu_seqlens_dev, B, max_patches, u_dev, scores, n_tokens,
                           pooled_dev, static_cast<cudaStream_t>(stream));
}

int siglip2_head_pool(int dtype, const void* x_dev, int D, int heads, const int* cu_seqlens_dev, int B,
                      int max_patches, const float* u_dev, float* scores_dev, void* pooled_dev, void* stream) {
  SG_CHECK_ARG(x_dev && cu_seqlens_dev && u_dev && scores_dev && pooled_dev && B > 0 && max_patches >= 0,
               "bad head_pool arguments");
  if (!aligned16(x_dev) || !aligned16(pooled_dev))
    return set_error(SIGLIP2_ERR_ALIGN, "head_pool tensors must be 16-byte aligned");
  return sg_head_pool_impl(dtype, x_dev, D, heads, cu_seqlens_dev, B, max_patches, u_dev, scores_dev, INT_MAX,
                           pooled_dev, static_cast<cudaStream_t>(stream));
}

int siglip2_metadata_size(const int32_t* hw_host, int batch, int* n_tokens, int* n_tiles) {
  SG_CHECK_ARG(hw_host && batch > 0, "bad metadata arguments");
  int N = 0, T = 0;
  SG_TRY(meta_counts(hw_host, batch, &N, &T));
  if (n_tokens) *n_tokens = N;
  if (n_tiles) *n_tiles = T;
  return static_cast<int>(meta_entries(batch, T));
}

int siglip2_metadata(const int32_t* hw_host, int batch, int32_t* meta_host, size_t capacity) {
  SG_CHECK_ARG(hw_host && meta_host && batch > 0, "bad metadata arguments");
  int N = 0, T = 0;
  SG_TRY(meta_counts(hw_host, batch, &N, &T));
  const size_t need = meta_entries(batch, T);
  SG_CHECK_ARG(capacity >= need, "metadata capacity %zu < %zu", capacity, need);
  for (size_t i = 0; i < need; ++i) meta_host[i] = 0;
  int32_t* cu = meta_host;
  int32_t* hw = meta_host + batch + 1;
  int32_t* tiles = meta_host + meta_tiles_offset(batch);
  cu[0] = 0;
  for (int b = 0; b < batch; ++b) {
    cu[b + 1] = cu[b] + hw_host[2 * b] * hw_host[2 * b + 1];
    hw[2 * b] = hw_host[2 * b];
    hw[2 * b + 1] = hw_host[2 * b + 1];
  }
  // attention tiles, longest images first (their CTAs start first: shorter tail)
  std::vector<int> order(batch);
  for (int b = 0; b < batch; ++b) order[b] = b;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return cu[a + 1] - cu[a] > cu[b + 1] - cu[b]; });
  int k = 0;
  for (int b : order) {
    const int nq = (cu[b + 1] - cu[b] + 127) / 128;
    for (int q = 0; q < nq; ++q) {
      tiles[2 * k] = b;
      tiles[2 * k + 1] = q;
      ++k;
    }
  }
  return SIGLIP2_OK;
}

size_t siglip2_workspace_size(const siglip2_config* cfg, int batch, int n_tokens) {
  if (!cfg || batch <= 0 || n_tokens < 0) return 0;
  return forward_workspace(cfg, batch, n_tokens, nullptr, nullptr);
}

int siglip2_forward(const siglip2_config* cfg, const siglip2_weights* w, const void* patches_dev, int batch,
                    int max_patches, const int32_t* hw_host, const int32_t* meta_dev, void* last_hidden_dev,
                    void* pooled_dev, void* workspace_dev, size_t workspace_bytes, void* stream) {
  return sg_forward_impl(cfg, w, patches_dev, batch, max_patches, hw_host, meta_dev, last_hidden_dev, pooled_dev,
                         workspace_dev, workspace_bytes, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
