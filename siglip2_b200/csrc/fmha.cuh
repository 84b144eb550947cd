// Variable-length (per-image) attention on tcgen05 for the packed NaFlex
// sequence: every query row attends only to the keys of its own image, i.e.
// the block-diagonal document mask of the reference, with no padded rows.
//
// Input: the QKV projection output [N, 3*H*hd], q | k | v with the heads of
// each in order (the reference's fused qkv_proj layout).  Each head is read
// through a 3-D tensor map [N][3H][hd] as a 64-wide slab (128B swizzle) plus
// an R = HDP-64 wide slab (32B / 64B swizzle), HDP = 64 | 80 | 96 for
// head_dim 64 | 72 | 96; the columns of the R slab past head_dim are
// out-of-bounds reads and arrive as zeros, so padding the head dimension
// changes no dot product and costs no HBM bytes.
//
// Persistent: two CTAs per SM (256 TMEM columns and <= 104 KB of shared
// memory each) walk the work items (128-query tile of one image, head) of
// the tile list, longest images first, item = blockIdx.x + k * gridDim.x.
// The TMA warp loads the next item's Q (second buffer where it fits) and K/V
// tiles while the current item runs, and the next item's first QK^T is
// issued while the softmax warps still drain this item's O, so the per-item
// prologue and epilogue overlap the other work.  Keys come in tiles of
// KT = 96.  TMEM columns: S [0, 96) fp32, P [96, 144) (bf16/f16 pairs),
// O [144, 144 + HDP) fp32.  Because P has its own columns, S_{j+1} = Q K_{j+1}^T
// runs on the tensor cores while the softmax warps turn S_j into P_j.
//   warp 0     TMA: Q per item, K and V tiles into 2-deep rings
//   warp 1     TMEM owner + MMA issuer: S_j as soon as the softmax has read
//              S_{j-1}; then O += P_{j-1} V_{j-1} (P read from TMEM); an
//              item's first PV overwrites O once the previous item's O is read
//   warps 2-5  softmax: each thread owns one query row (its TMEM lane):
//              loads S_j into registers and frees it, masks keys past the
//              image end, online max with lazy rescale (O is rescaled in TMEM
//              only when the running max grows by more than 2^8), writes
//              P = exp2(S*scale*log2e - m) packed in pairs, final O / l.
//
// Train mode: with drop.p > 0 the output store applies the reference's
// attention-output dropout (model.py:166-169) with the counter-based mask of
// dropout.cuh over the logical [N, heads*head_dim] output.
#pragma once

#include "dropout.cuh"
#include "ptx.cuh"

namespace sg {

struct FmhaParams {
  const int* cu;      // [B+1] first row of each image in the packed sequence
  const int2* tiles;  // [n_tiles] (image, query-tile index)
  int n_items;        // n_tiles * heads work items: item w = (tile w / heads, head w % heads)
  int heads;
  int head_dim;
  void* out;          // [N, heads*head_dim]
  int ld_out;
  float scale_log2;   // head_dim^-0.5 * log2(e)
  DropoutParams drop; // attention-output dropout (p = 0: off)
  float* lse;         // optional [N, heads]: base-2 log-sum-exp of each row's scaled logits (for the backward)
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max of three floats in one instruction (sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float y;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(a), "f"(b), "f"(c));
  return y;
}

// keeps the compiler from using tcgen05.ld destination registers before the
// tcgen05.wait::ld that makes them valid
#define SG_REG_FENCE_16(r)                                                                               \
  asm volatile(""                                                                                        \
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),       \
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),   \
                 "+r"(r[14]), "+r"(r[15]))

template <int HDP>
struct FmhaCfg {
  static constexpr int R = HDP - 64;                  // remainder slab width (0, 16, 32)
  static constexpr int KT = 96;                       // keys per tile
  static constexpr int kQSlabA = 128 * 64 * 2;        // Q: 128 rows
  static constexpr int kQSlabR = 128 * R * 2;
  static constexpr int kQTile = kQSlabA + (kQSlabR + 1023) / 1024 * 1024;
  static constexpr int kKSlabA = KT * 64 * 2;         // K / V: 96 rows (12 KB, a multiple of 1 KB)
  static constexpr int kKSlabR = KT * R * 2;
  static constexpr int kKTile = kKSlabA + (kKSlabR + 1023) / 1024 * 1024;
  // Two CTAs share an SM's 228 KB (1 KB reserved per CTA).  Deeper K/V rings
  // come first (K_{j+1} then loads two tiles ahead of its QK^T), then a
  // second Q buffer (the next item's Q lands while this one runs):
  // head_dim 64: 3 stages, 2 Q buffers; 72 (80-wide): 3, 1; 96: 2, 1.
  static constexpr int kPerCta = 233472 / 2 - 1024;
  static constexpr int bytes_for(int qb, int st) { return qb * kQTile + 2 * st * kKTile + 256 + 1024; }
  static constexpr int kStages = bytes_for(1, 3) <= kPerCta ? 3 : 2;
  static constexpr int kQBufs = bytes_for(2, kStages) <= kPerCta ? 2 : 1;
  static constexpr int kQ = 0;
  static constexpr int kK = kQBufs * kQTile;
  static constexpr int kV = kK + kStages * kKTile;
  static constexpr int kBar = kV + kStages * kKTile;
  static constexpr int kSmem = kBar + 256 + 1024;
  static_assert(kSmem <= kPerCta, "two attention CTAs per SM");
  static constexpr int kQBytes = kQSlabA + kQSlabR;   // TMA bytes
  static constexpr int kKBytes = kKSlabA + kKSlabR;
  static constexpr uint32_t kTmemCols = 256;
  static constexpr uint32_t kColP = KT;               // 48 columns of packed pairs
  static constexpr uint32_t kColO = KT + KT / 2;      // 144
};

template <typename T, int HDP>
__global__ void __launch_bounds__(192, 2)
    fmha_varlen_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmQR,
                       const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmKR,
                       const FmhaParams p) {
  using C = FmhaCfg<HDP>;
  constexpr int R = C::R;
  constexpr int KT = C::KT;
  constexpr int ST = C::kStages;
  constexpr int QB = C::kQBufs;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescS = make_idesc(128, KT, kBF16, false, false);
  constexpr uint32_t kIdescO64 = make_idesc(128, 64, kBF16, false, true);
  constexpr uint32_t kIdescOR = make_idesc(128, R > 0 ? R : 16, kBF16, false, true);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBar);
  uint64_t* q_full = bars;           // QB: an item's Q landed
  uint64_t* q_empty = q_full + QB;   // QB: an item's QK^T MMAs are done with its Q
  uint64_t* k_full = q_empty + QB;   // ST
  uint64_t* k_empty = k_full + ST;   // ST
  uint64_t* v_full = k_empty + ST;   // ST
  uint64_t* v_empty = v_full + ST;   // ST
  uint64_t* s_full = v_empty + ST;   // 1: S computed
  uint64_t* s_free = s_full + 1;     // 1: S read by the softmax (128 arrivals)
  uint64_t* p_full = s_free + 1;     // 1: P written, O rescaled (128 arrivals)
  uint64_t* pv_done = p_full + 1;    // 1: O += P V complete
  uint64_t* o_free = pv_done + 1;    // 1: an item's O read by the softmax warps (128 arrivals)
  uint64_t* mdone = o_free + 1;      // 1
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mdone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int H = p.heads;

  if (threadIdx.x == 0) {
    for (int b = 0; b < QB; ++b) {
      mbar_init(&q_full[b], 1);
      mbar_init(&q_empty[b], 1);
    }
    for (int s = 0; s < ST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 128);
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    mbar_init(o_free, 128);
    mbar_init(mdone, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::kTmemCols);
    tmem_relinquish();
  }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // the QKV projection is complete and visible from here on
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // --------------------------------------------------------------- TMA
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      if (R > 0) {
        tma_prefetch_desc(&tmQR);
        tma_prefetch_desc(&tmKR);
      }
      int nq = 0, nk = 0, nv = 0;  // Q, K and V loads issued by this CTA
      bool ok = true;
      for (int w = blockIdx.x; w < p.n_items && ok; w += gridDim.x) {
        const int2 tile = p.tiles[w / H];
        const int head = w - (w / H) * H;
        const int img_row0 = __ldg(p.cu + tile.x);
        const int L = __ldg(p.cu + tile.x + 1) - img_row0;
        const int n_kv = (L + KT - 1) / KT;
        const int qb = nq % QB;
        if (*abort_flag || !mbar_wait(&q_empty[qb], ((nq / QB) & 1) ^ 1, 200)) {
          ok = false;
          break;
        }
        uint8_t* qdst = smem + C::kQ + qb * C::kQTile;
        mbar_arrive_expect_tx(&q_full[qb], C::kQBytes);
        tma_load_3d(qdst, &tmQ, &q_full[qb], 0, head, img_row0 + tile.y * 128);
        if (R > 0) tma_load_3d(qdst + C::kQSlabA, &tmQR, &q_full[qb], 64, head, img_row0 + tile.y * 128);
        ++nq;
        for (int j = 0; j < n_kv; ++j) {
          const int st = nk % ST;  // nk == nv here
          const uint32_t eph = ((nk / ST) & 1) ^ 1;
          const int kv_row = img_row0 + j * KT;
          if (*abort_flag || !mbar_wait(&k_empty[st], eph, 201)) {
            ok = false;
            break;
          }
          uint8_t* kb = smem + C::kK + st * C::kKTile;
          mbar_arrive_expect_tx(&k_full[st], C::kKBytes);
          tma_load_3d(kb, &tmK, &k_full[st], 0, H + head, kv_row);
          if (R > 0) tma_load_3d(kb + C::kKSlabA, &tmKR, &k_full[st], 64, H + head, kv_row);
          ++nk;
          if (*abort_flag || !mbar_wait(&v_empty[st], eph, 202)) {
            ok = false;
            break;
          }
          uint8_t* vb = smem + C::kV + st * C::kKTile;
          mbar_arrive_expect_tx(&v_full[st], C::kKBytes);
          tma_load_3d(vb, &tmK, &v_full[st], 0, 2 * H + head, kv_row);
          if (R > 0) tma_load_3d(vb + C::kKSlabA, &tmKR, &v_full[st], 64, 2 * H + head, kv_row);
          ++nv;
        }
      }
      if (!ok) *abort_flag = 1;
      // No TMA write may still be in flight when the CTA exits: a buffer is
      // only reloaded after its previous load was consumed, so only the last
      // load of each buffer can be outstanding.
      for (int i = (nq > QB ? nq - QB : 0); i < nq; ++i) mbar_wait(&q_full[i % QB], (i / QB) & 1, 203);
      for (int i = (nk > ST ? nk - ST : 0); i < nk; ++i) mbar_wait(&k_full[i % ST], (i / ST) & 1, 204);
      for (int i = (nv > ST ? nv - ST : 0); i < nv; ++i) mbar_wait(&v_full[i % ST], (i / ST) & 1, 205);
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------- MMA
    // The whole warp runs the loop (warp-uniform control flow keeps the
    // descriptor arithmetic in uniform registers); one elected lane issues
    // each tcgen05.mma / commit.  Descriptors are built once per buffer and
    // stepped by adding the K offset (in 16-byte address units): the MMA
    // issue latency, not the tensor pipe, sets this warp's pace.
    int kv = 0, g = 0, it = 0;  // K/V tiles, S tiles and items consumed
    bool ok = true;
    auto wait_all = [&](uint64_t* bar, uint32_t parity, int site) -> bool {
      const bool w = !*abort_flag && mbar_wait(bar, parity, site);
      return __all_sync(0xffffffffu, w);
    };
    // O += P V for the K/V tile kvi, the S tile gi of item `item`; the
    // item's first PV overwrites O once the previous item's O was read
    auto issue_pv = [&](int kvi, int gi, bool first, int item) -> bool {
      const int st = kvi % ST;
      if (!wait_all(p_full, gi & 1, 214) || !wait_all(&v_full[st], (kvi / ST) & 1, 215)) return false;
      if (first && item > 0 && !wait_all(o_free, (item - 1) & 1, 217)) return false;
      tc_fence_after();
      const uint32_t va = smem_u32(smem + C::kV + st * C::kKTile);
      const uint64_t vd = mnmajor_desc(va, 128, 0);
      const uint64_t vrd = mnmajor_desc(va + C::kKSlabA, R > 0 ? R * 2 : 32, 0);
      if (elect_one()) {
#pragma unroll
        for (int s = 0; s < KT / 16; ++s) {  // 16 keys per MMA; P columns [kColP + 8s, +8)
          const uint32_t acc = (!first || s > 0) ? 1u : 0u;
          umma_ts(tmem + C::kColO, tmem + C::kColP + s * 8, vd + static_cast<uint64_t>(s * 16 * 128 / 16), kIdescO64,
                  acc);
          if constexpr (R > 0)
            umma_ts(tmem + C::kColO + 64, tmem + C::kColP + s * 8, vrd + static_cast<uint64_t>(s * 16 * R * 2 / 16),
                    kIdescOR, acc);
        }
        umma_commit(pv_done);
        umma_commit(&v_empty[st]);
      }
      __syncwarp();
      return true;
    };
    for (int w = blockIdx.x; w < p.n_items && ok; w += gridDim.x, ++it) {
      const int2 tile = p.tiles[w / H];
      const int L = __ldg(p.cu + tile.x + 1) - __ldg(p.cu + tile.x);
      const int n_kv = (L + KT - 1) / KT;
      const int qb = it % QB;
      if (!wait_all(&q_full[qb], (it / QB) & 1, 211)) {
        ok = false;
        break;
      }
      const uint32_t qa = smem_u32(smem + C::kQ + qb * C::kQTile);
      const uint64_t qd = kmajor_desc(qa, 128), qrd = kmajor_desc(qa + C::kQSlabA, R > 0 ? R * 2 : 32);
      for (int j = 0; j < n_kv; ++j, ++kv, ++g) {
        const int st = kv % ST;
        // S_g overwrites S_{g-1}: the softmax must have read it
        if (!wait_all(&k_full[st], (kv / ST) & 1, 212) || (g > 0 && !wait_all(s_free, (g - 1) & 1, 213))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ka = smem_u32(smem + C::kK + st * C::kKTile);
        const uint64_t kd = kmajor_desc(ka, 128), krd = kmajor_desc(ka + C::kKSlabA, R > 0 ? R * 2 : 32);
        if (elect_one()) {
#pragma unroll
          for (int k = 0; k < 4; ++k)  // 16 K-elements = 32 bytes = 2 address units per step
            umma_ss(tmem, qd + 2 * k, kd + 2 * k, kIdescS, k > 0);
#pragma unroll
          for (int k = 0; k < R / 16; ++k) umma_ss(tmem, qrd + 2 * k, krd + 2 * k, kIdescS, 1);
          umma_commit(s_full);
          umma_commit(&k_empty[st]);
        }
        __syncwarp();
        if (j > 0 && !issue_pv(kv - 1, g - 1, j == 1, it)) {
          ok = false;
          break;
        }
      }
      if (!ok) break;
      if (elect_one()) umma_commit(&q_empty[qb]);  // every QK^T of this item issued: Q is free once they finish
      __syncwarp();
      if (!issue_pv(kv - 1, g - 1, n_kv == 1, it)) ok = false;
    }
    if (!ok && lane == 0) *abort_flag = 1;
    if (elect_one()) {
      umma_commit(mdone);
      mbar_wait(mdone, 0, 216);
    }
    __syncwarp();
  } else {
    // --------------------------------------------------------------- softmax + epilogue
    const int q = warp & 3;       // TMEM lane quarter of this warp
    const int r = q * 32 + lane;  // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const float sc = p.scale_log2;
    bool ok = true;
    int g = 0;  // S tiles consumed
    for (int w = blockIdx.x; w < p.n_items && ok; w += gridDim.x) {
      const int2 tile = p.tiles[w / H];
      const int head = w - (w / H) * H;
      const int img_row0 = __ldg(p.cu + tile.x);
      const int L = __ldg(p.cu + tile.x + 1) - img_row0;
      const int n_kv = (L + KT - 1) / KT;
      float m_use = 0.f, l = 0.f;
      for (int j = 0; j < n_kv; ++j, ++g) {
        if (*abort_flag || !mbar_wait(s_full, g & 1, 221)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // the whole S tile in one round trip
        float s[KT];
        {
          uint32_t su[KT];
#pragma unroll
          for (int c = 0; c < KT / 32; ++c) SG_TMEM_LD_32(tmem + c * 32 + lane_off, (su + c * 32));
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < KT; ++k) s[k] = __uint_as_float(su[k]);
        }
        // S is in registers: let the MMA warp compute the next S
        tc_fence_before();
        mbar_arrive(s_free);
        const int valid = L - j * KT;  // keys of this image in the tile (>= 1)
        if (valid < KT) {
#pragma unroll
          for (int k = 0; k < KT; ++k)
            if (k >= valid) s[k] = -INFINITY;
        }
        // tile maximum (3-input max), lazy rescale, then P = exp2(s * scale - m)
        // with the scale-and-subtract and the row sums in packed f32x2 issues
        float mx[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) mx[i] = fmaxf(s[2 * i], s[2 * i + 1]);
#pragma unroll
        for (int k = 4; k < KT / 2; ++k) mx[k & 3] = fmax3(mx[k & 3], s[2 * k], s[2 * k + 1]);
        const float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * sc;
        float alpha = 1.f;
        if (j == 0) {
          m_use = mt;
        } else if (mt > m_use + 8.f) {
          alpha = ex2_approx(m_use - mt);
          m_use = mt;
        }
        float2 ps2[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) ps2[i] = make_float2(0.f, 0.f);
        uint32_t wv[KT / 2];
#pragma unroll
        for (int k = 0; k < KT / 2; ++k) {
          const float2 x = ffma2(make_float2(s[2 * k], s[2 * k + 1]), make_float2(sc, sc), make_float2(-m_use, -m_use));
          const float2 pr = make_float2(ex2_approx(x.x), ex2_approx(x.y));
          ps2[k & 3] = fadd2(ps2[k & 3], pr);
          wv[k] = Pack2<T>::pack(pr.x, pr.y);
        }
        const float2 pt = fadd2(fadd2(ps2[0], ps2[1]), fadd2(ps2[2], ps2[3]));
        l = l * alpha + (pt.x + pt.y);
        if (j > 0) {
          // the previous PV must be done: P's columns are rewritten and O may be rescaled
          // (at j == 0 the previous item's last PV was waited for before its O was read)
          if (!mbar_wait(pv_done, (g - 1) & 1, 222)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (__any_sync(0xffffffffu, alpha != 1.f)) {
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
        }
#pragma unroll
        for (int c = 0; c < KT / 16; ++c) SG_TMEM_ST_8(tmem + C::kColP + c * 8 + lane_off, (wv + c * 8));
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(p_full);
      }
      if (!ok || !mbar_wait(pv_done, (g - 1) & 1, 223)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int row = img_row0 + tile.y * 128 + r;
      const bool row_ok = (tile.y * 128 + r) < L;
      const float inv_l = 1.f / l;
      // softmax_k = exp2(s_k * scale_log2 - lse2) with lse2 = m + log2(l)
      if (p.lse != nullptr && row_ok) p.lse[static_cast<size_t>(row) * H + head] = m_use + log2f(l);
      T* orow = reinterpret_cast<T*>(p.out) + static_cast<size_t>(row) * p.ld_out + head * p.head_dim;
      // the whole O row in one TMEM round trip, then O is free for the next
      // item's first PV while this row is scaled and stored
      uint32_t ou[HDP];
#pragma unroll
      for (int c = 0; c < HDP / 16; ++c) SG_TMEM_LD_16(tmem + C::kColO + c * 16 + lane_off, (ou + c * 16));
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < HDP / 16; ++c) SG_REG_FENCE_16((ou + c * 16));
      tc_fence_before();
      mbar_arrive(o_free);
#pragma unroll
      for (int c = 0; c < HDP / 16; ++c) {
        const uint32_t* u = ou + c * 16;
        if (row_ok) {
#pragma unroll
          for (int gg = 0; gg < 2; ++gg) {
            const int d0 = c * 16 + gg * 8;
            if (d0 < p.head_dim) {  // head_dim is a multiple of 8
              float f[8];
#pragma unroll
              for (int k = 0; k < 8; ++k) f[k] = inv_l;
              if (p.drop.p > 0.f) {
                float keep[8];
                dropout_factors8(p.drop,
                                 static_cast<unsigned long long>(row) * (H * p.head_dim) + head * p.head_dim + d0,
                                 keep);
#pragma unroll
                for (int k = 0; k < 8; ++k) f[k] *= keep[k];
              }
              uint4 o;
              o.x = Pack2<T>::pack(__uint_as_float(u[gg * 8 + 0]) * f[0], __uint_as_float(u[gg * 8 + 1]) * f[1]);
              o.y = Pack2<T>::pack(__uint_as_float(u[gg * 8 + 2]) * f[2], __uint_as_float(u[gg * 8 + 3]) * f[3]);
              o.z = Pack2<T>::pack(__uint_as_float(u[gg * 8 + 4]) * f[4], __uint_as_float(u[gg * 8 + 5]) * f[5]);
              o.w = Pack2<T>::pack(__uint_as_float(u[gg * 8 + 6]) * f[6], __uint_as_float(u[gg * 8 + 7]) * f[7]);
              *reinterpret_cast<uint4*>(orow + d0) = o;
            }
          }
        }
      }
    }
    if (!ok) *abort_flag = 1;
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

}  // namespace sg
