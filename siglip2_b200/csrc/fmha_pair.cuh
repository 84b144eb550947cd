// Variable-length attention, paired query tiles: one CTA per SM computes two
// 128-row query tiles (A = tile 2t, B = tile 2t+1) of the same image and head
// against each K/V tile it loads, so every K/V tile crosses L2 -> shared
// memory once per 256 query rows instead of once per 128, and the two tiles'
// softmax warpgroups take turns on the MUFU while the tensor pipe runs the
// other tile's QK^T / PV.
//
// Semantics, inputs and outputs are those of fmha_varlen_kernel (fmha.cuh):
// per-image softmax(q k^T / sqrt(hd)) v over the packed QKV projection, the
// reference's document mask (model.py:156-163), optional train-mode output
// dropout (model.py:166-169).  Work items come from the same tile list,
// (image, 128-row query tile) x head: an item whose query tile is even owns
// the pair (its odd successor, when the image has one, is tile B); items with
// odd tiles are skipped.  The pairing depends only on the parity of the
// query tile (the list covers every tile of every image, in any order), so
// it needs no extra metadata.
//
// Warps (384 threads, one CTA per SM):
//   warp 0       TMA: Q_A and Q_B per item (double-buffered), K/V ring
//   warp 1       TMEM owner (512 columns) + MMA issuer: per K/V tile j
//                S_A(j), S_B(j), then O_A += P_A(j-1) V(j-1), O_B += ...
//   warps 2-3    idle (keep the softmax warpgroups warpgroup-aligned)
//   warps 4-7    softmax of tile A: TMEM lanes = query rows, columns [0, 256)
//   warps 8-11   softmax of tile B: columns [256, 512); on items with both
//                tiles the two warpgroups take turns on the exponentials
//                (mbarrier hand-off), half a tile apart
// Per tile the TMEM columns are laid out as in fmha.cuh: S [0, 96) fp32,
// P [96, 144) packed pairs, O [144, 144 + HDP) fp32.
#pragma once

#include "fmha.cuh"

namespace sg {

template <int HDP>
struct FmhaPairCfg {
  using C1 = FmhaCfg<HDP>;
  static constexpr int R = C1::R;
  static constexpr int KT = C1::KT;
  static constexpr int kQTile = C1::kQTile;
  static constexpr int kKTile = C1::kKTile;
  static constexpr int kQSlabA = C1::kQSlabA;
  static constexpr int kKSlabA = C1::kKSlabA;
  static constexpr int kQBytes = C1::kQBytes;
  static constexpr int kKBytes = C1::kKBytes;
  static constexpr int kLimit = 227 * 1024;
  static constexpr int kFixed = 512 + 1024;  // barriers + alignment slack
  static constexpr int kQBufs = 2;           // pairs of Q tiles in flight (this item's and the next one's)
  static constexpr int kQ = 0;
  static constexpr int kK = kQBufs * 2 * kQTile;
  static constexpr int kStages = (kLimit - kFixed - kK) / (2 * kKTile) >= 4 ? 4 : 3;
  static constexpr int kV = kK + kStages * kKTile;
  static constexpr int kBar = kV + kStages * kKTile;
  static constexpr int kSmem = kBar + kFixed;
  static_assert(kSmem <= kLimit, "paired attention shared-memory budget");
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kTileCols = 256;  // TMEM columns per query tile
  static constexpr uint32_t kColP = C1::kColP;
  static constexpr uint32_t kColO = C1::kColO;
  static constexpr int kThreads = 384;
};


template <typename T, int HDP>
__global__ void __launch_bounds__(384, 1)
    fmha_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmQR,
                     const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmKR,
                     const FmhaParams p) {
  using C = FmhaPairCfg<HDP>;
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
  uint64_t* q_full = bars;            // QB: an item's Q tiles landed
  uint64_t* q_empty = q_full + QB;    // QB: an item's QK^T MMAs are done with its Q tiles
  uint64_t* k_full = q_empty + QB;    // ST
  uint64_t* k_empty = k_full + ST;    // ST
  uint64_t* v_full = k_empty + ST;    // ST
  uint64_t* v_empty = v_full + ST;    // ST
  // per query tile X in {0 = A, 1 = B}: index [X]
  uint64_t* s_full = v_empty + ST;    // 2: S_X computed
  uint64_t* s_free = s_full + 2;      // 2: S_X read by the softmax (128 arrivals)
  uint64_t* p_full = s_free + 2;      // 2: P_X written, O_X rescaled (128 arrivals)
  uint64_t* pv_done = p_full + 2;     // 2: O_X += P_X V complete
  uint64_t* o_free = pv_done + 2;     // 2: an item's O_X read by the softmax warps (128 arrivals)
  uint64_t* turn = o_free + 2;        // 2: warpgroup X may run its exponentials (128 arrivals of the other)
  uint64_t* mdone = turn + 2;         // 1
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
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&s_free[x], 128);
      mbar_init(&p_full[x], 128);
      mbar_init(&pv_done[x], 1);
      mbar_init(&o_free[x], 128);
      mbar_init(&turn[x], 128);
    }
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

  // Item w of the tile list: (image, query tile) = tiles[w / H], head w % H.
  // Returns false for items this kernel skips (odd query tiles: tile B of
  // the preceding item).  hasB: the image has the odd tile after tile A.
  auto item = [&](int w, int& img_row0, int& L, int& qa, int& head, bool& hasB) -> bool {
    const int2 tile = p.tiles[w / H];
    if (tile.y & 1) return false;
    head = w - (w / H) * H;
    img_row0 = __ldg(p.cu + tile.x);
    L = __ldg(p.cu + tile.x + 1) - img_row0;
    qa = tile.y;
    hasB = (qa + 1) * 128 < L;
    return true;
  };

  if (warp == 0) {
    // --------------------------------------------------------------- TMA
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      if (R > 0) {
        tma_prefetch_desc(&tmQR);
        tma_prefetch_desc(&tmKR);
      }
      int nq = 0, nk = 0, nv = 0;  // Q pairs, K and V loads issued by this CTA
      bool ok = true;
      for (int w = blockIdx.x; w < p.n_items && ok; w += gridDim.x) {
        int img_row0, L, qa, head;
        bool hasB;
        if (!item(w, img_row0, L, qa, head, hasB)) continue;
        const int n_kv = (L + KT - 1) / KT;
        const int qb = nq % QB;
        if (*abort_flag || !mbar_wait(&q_empty[qb], ((nq / QB) & 1) ^ 1, 300)) {
          ok = false;
          break;
        }
        uint8_t* qdst = smem + C::kQ + qb * 2 * C::kQTile;
        mbar_arrive_expect_tx(&q_full[qb], (hasB ? 2 : 1) * C::kQBytes);
        for (int x = 0; x < (hasB ? 2 : 1); ++x) {
          const int row = img_row0 + (qa + x) * 128;
          tma_load_3d(qdst + x * C::kQTile, &tmQ, &q_full[qb], 0, head, row);
          if (R > 0) tma_load_3d(qdst + x * C::kQTile + C::kQSlabA, &tmQR, &q_full[qb], 64, head, row);
        }
        ++nq;
        for (int j = 0; j < n_kv; ++j) {
          const int st = nk % ST;  // nk == nv here
          const uint32_t eph = ((nk / ST) & 1) ^ 1;
          const int kv_row = img_row0 + j * KT;
          if (*abort_flag || !mbar_wait(&k_empty[st], eph, 301)) {
            ok = false;
            break;
          }
          uint8_t* kb = smem + C::kK + st * C::kKTile;
          mbar_arrive_expect_tx(&k_full[st], C::kKBytes);
          tma_load_3d(kb, &tmK, &k_full[st], 0, H + head, kv_row);
          if (R > 0) tma_load_3d(kb + C::kKSlabA, &tmKR, &k_full[st], 64, H + head, kv_row);
          ++nk;
          if (*abort_flag || !mbar_wait(&v_empty[st], eph, 302)) {
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
      // no TMA write may still be in flight when the CTA exits: only the last
      // load of each buffer can be outstanding
      for (int i = (nq > QB ? nq - QB : 0); i < nq; ++i) mbar_wait(&q_full[i % QB], (i / QB) & 1, 303);
      for (int i = (nk > ST ? nk - ST : 0); i < nk; ++i) mbar_wait(&k_full[i % ST], (i / ST) & 1, 304);
      for (int i = (nv > ST ? nv - ST : 0); i < nv; ++i) mbar_wait(&v_full[i % ST], (i / ST) & 1, 305);
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------- MMA
    // The whole warp runs the loop (warp-uniform control flow, so the
    // descriptor arithmetic stays in uniform registers); one elected lane
    // issues each tcgen05.mma / commit.  Descriptors are built once per
    // buffer and stepped by adding the K offset (16 bytes per address unit):
    // the issuer is latency-bound, not the tensor pipe.
    int kv = 0, it = 0;    // K/V tiles and items consumed
    int g[2] = {0, 0};     // S tiles issued per query tile
    int its[2] = {0, 0};   // items per query tile
    bool ok = true;
    auto wait_all = [&](uint64_t* bar, uint32_t parity, int site) -> bool {
      const bool w = !*abort_flag && mbar_wait(bar, parity, site);
      return __all_sync(0xffffffffu, w);
    };
    // O_x += P_x V for K/V tile kvi; S tile gi of query tile x; the item's
    // first PV overwrites O_x once the previous item's O_x was read
    auto issue_pv = [&](int x, int kvi, int gi, bool first, int itx) -> bool {
      const int st = kvi % ST;
      if (!wait_all(&p_full[x], gi & 1, 314) || !wait_all(&v_full[st], (kvi / ST) & 1, 315)) return false;
      if (first && itx > 0 && !wait_all(&o_free[x], (itx - 1) & 1, 317)) return false;
      tc_fence_after();
      const uint32_t va = smem_u32(smem + C::kV + st * C::kKTile);
      const uint64_t vd = mnmajor_desc(va, 128, 0);
      const uint64_t vrd = mnmajor_desc(va + C::kKSlabA, R > 0 ? R * 2 : 32, 0);
      const uint32_t tb = tmem + x * C::kTileCols;
      if (elect_one()) {
#pragma unroll
        for (int s = 0; s < KT / 16; ++s) {  // 16 keys per MMA; P columns [kColP + 8s, +8)
          const uint32_t acc = (!first || s > 0) ? 1u : 0u;
          umma_ts(tb + C::kColO, tb + C::kColP + s * 8, vd + static_cast<uint64_t>(s * 16 * 128 / 16), kIdescO64,
                  acc);
          if constexpr (R > 0)
            umma_ts(tb + C::kColO + 64, tb + C::kColP + s * 8, vrd + static_cast<uint64_t>(s * 16 * R * 2 / 16),
                    kIdescOR, acc);
        }
        umma_commit(&pv_done[x]);
      }
      __syncwarp();
      return true;
    };
    auto issue_s = [&](int x, uint64_t qd, uint64_t qrd, uint64_t kd, uint64_t krd, int gx) -> bool {
      if (gx > 0 && !wait_all(&s_free[x], (gx - 1) & 1, 313)) return false;  // S_x overwrites S_x(prev)
      tc_fence_after();
      const uint32_t tb = tmem + x * C::kTileCols;
      if (elect_one()) {
#pragma unroll
        for (int k = 0; k < 4; ++k)  // 16 K-elements = 32 bytes = 2 address units per step
          umma_ss(tb, qd + 2 * k, kd + 2 * k, kIdescS, k > 0);
#pragma unroll
        for (int k = 0; k < R / 16; ++k) umma_ss(tb, qrd + 2 * k, krd + 2 * k, kIdescS, 1);
        umma_commit(&s_full[x]);
      }
      __syncwarp();
      return true;
    };
    for (int w = blockIdx.x; w < p.n_items && ok; w += gridDim.x) {
      int img_row0, L, qa, head;
      bool hasB;
      if (!item(w, img_row0, L, qa, head, hasB)) continue;
      const int n_kv = (L + KT - 1) / KT;
      const int qb = it % QB;
      if (!wait_all(&q_full[qb], (it / QB) & 1, 311)) {
        ok = false;
        break;
      }
      const uint32_t qbase = smem_u32(smem + C::kQ + qb * 2 * C::kQTile);
      const uint64_t qdA = kmajor_desc(qbase, 128), qdB = kmajor_desc(qbase + C::kQTile, 128);
      const uint64_t qrdA = kmajor_desc(qbase + C::kQSlabA, R > 0 ? R * 2 : 32);
      const uint64_t qrdB = kmajor_desc(qbase + C::kQTile + C::kQSlabA, R > 0 ? R * 2 : 32);
      for (int j = 0; j < n_kv && ok; ++j, ++kv) {
        const int st = kv % ST;
        if (!wait_all(&k_full[st], (kv / ST) & 1, 312)) {
          ok = false;
          break;
        }
        const uint32_t ka = smem_u32(smem + C::kK + st * C::kKTile);
        const uint64_t kd = kmajor_desc(ka, 128), krd = kmajor_desc(ka + C::kKSlabA, R > 0 ? R * 2 : 32);
        ok = issue_s(0, qdA, qrdA, kd, krd, g[0]++);
        if (ok && hasB) ok = issue_s(1, qdB, qrdB, kd, krd, g[1]++);
        if (!ok) break;
        if (elect_one()) umma_commit(&k_empty[st]);
        __syncwarp();
        if (j > 0) {
          ok = issue_pv(0, kv - 1, g[0] - 2, j == 1, its[0]);
          if (ok && hasB) ok = issue_pv(1, kv - 1, g[1] - 2, j == 1, its[1]);
          if (ok) {
            if (elect_one()) umma_commit(&v_empty[(kv - 1) % ST]);
            __syncwarp();
          }
        }
      }
      if (!ok) break;
      if (elect_one()) umma_commit(&q_empty[qb]);  // every QK^T of this item issued: Q is free once they finish
      __syncwarp();
      ok = issue_pv(0, kv - 1, g[0] - 1, n_kv == 1, its[0]);
      if (ok && hasB) ok = issue_pv(1, kv - 1, g[1] - 1, n_kv == 1, its[1]);
      if (ok) {
        if (elect_one()) umma_commit(&v_empty[(kv - 1) % ST]);
        __syncwarp();
      }
      ++it;
      ++its[0];
      if (hasB) ++its[1];
    }
    if (!ok && lane == 0) *abort_flag = 1;
    if (elect_one()) {
      umma_commit(mdone);
      mbar_wait(mdone, 0, 316);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // --------------------------------------------------------------- softmax + epilogue of tile X
    const int x = (warp - 4) >> 2;  // 0: tile A (warps 4-7), 1: tile B (warps 8-11)
    const int q = warp & 3;         // TMEM lane quarter of this warp
    const int r = q * 32 + lane;    // query row within the tile
    const uint32_t tb = tmem + x * C::kTileCols + (static_cast<uint32_t>(q * 32) << 16);
    const float sc = p.scale_log2;
    const float2 sc2 = make_float2(sc, sc);
    bool ok = true;
    int g = 0;      // S tiles consumed by this warpgroup
    int turns = 0;  // exponential turns this warpgroup has taken
    // Ping-pong: on items with both tiles the two warpgroups take turns
    // running their exponential loops (A first), so one warpgroup's row max,
    // TMEM loads and P stores run while the other one keeps the MUFU busy,
    // instead of both contending for it and then idling together.
    if (x == 1) mbar_arrive(&turn[0]);
    for (int w = blockIdx.x; w < p.n_items && ok; w += gridDim.x) {
      int img_row0, L, qa, head;
      bool hasB;
      if (!item(w, img_row0, L, qa, head, hasB)) continue;
      if (x == 1 && !hasB) continue;
      const int n_kv = (L + KT - 1) / KT;
      float m_use = 0.f, l = 0.f;
      for (int j = 0; j < n_kv; ++j, ++g) {
        if (*abort_flag || !mbar_wait(&s_full[x], g & 1, 321)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float s[KT];
#pragma unroll
        for (int c = 0; c < KT / 16; c += 2) {
          uint32_t u[16], u2[16];
          SG_TMEM_LD_16(tb + c * 16, u);
          SG_TMEM_LD_16(tb + (c + 1) * 16, u2);
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            s[c * 16 + k] = __uint_as_float(u[k]);
            s[(c + 1) * 16 + k] = __uint_as_float(u2[k]);
          }
        }
        // S is in registers: let the MMA warp compute the next S of this tile
        tc_fence_before();
        mbar_arrive(&s_free[x]);
        const int valid = L - j * KT;  // keys of this image in the tile (>= 1)
        if (valid < KT) {
#pragma unroll
          for (int k = 0; k < KT; ++k)
            if (k >= valid) s[k] = -INFINITY;
        }
        float mx[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx[i] = s[i];
        constexpr int kMax3 = 8 + (KT - 8) / 16 * 16;  // columns covered by 3-input steps
#pragma unroll
        for (int k = 8; k < kMax3; k += 16)
#pragma unroll
          for (int i = 0; i < 8; ++i) mx[i] = fmax3(mx[i], s[k + i], s[k + 8 + i]);
#pragma unroll
        for (int k = kMax3; k < KT; k += 8)
#pragma unroll
          for (int i = 0; i < 8; ++i) mx[i] = fmaxf(mx[i], s[k + i]);
        float mt = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
        mt *= sc;
        float alpha = 1.f;
        if (j == 0) {
          m_use = mt;
        } else if (mt > m_use + 8.f) {
          alpha = ex2_approx(m_use - mt);
          m_use = mt;
        }
        if (hasB && !mbar_wait(&turn[x], turns & 1, 324)) {
          ok = false;
          break;
        }
        const float2 nm2 = make_float2(-m_use, -m_use);
        float2 ps[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) ps[i] = make_float2(0.f, 0.f);
        uint32_t wv[KT / 2];
#pragma unroll
        for (int k = 0; k < KT / 2; ++k) {
          const float2 e = ffma2(make_float2(s[2 * k], s[2 * k + 1]), sc2, nm2);
          const float2 pr = make_float2(ex2_approx(e.x), ex2_approx(e.y));
          ps[k & 3] = fadd2(ps[k & 3], pr);
          wv[k] = Pack2<T>::pack(pr.x, pr.y);
        }
        if (hasB) {
          mbar_arrive(&turn[x ^ 1]);
          ++turns;
        }
        const float2 pt = fadd2(fadd2(ps[0], ps[1]), fadd2(ps[2], ps[3]));
        l = l * alpha + (pt.x + pt.y);
        if (j > 0) {
          // the previous PV must be done: P's columns are rewritten and O may be rescaled
          if (!mbar_wait(&pv_done[x], (g - 1) & 1, 322)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (__any_sync(0xffffffffu, alpha != 1.f)) {
            uint32_t u[16];
#pragma unroll
            for (int c = 0; c < HDP / 16; ++c) {
              SG_TMEM_LD_16(tb + C::kColO + c * 16, u);
              tmem_ld_wait();
#pragma unroll
              for (int k = 0; k < 16; ++k) u[k] = __float_as_uint(__uint_as_float(u[k]) * alpha);
              SG_TMEM_ST_16(tb + C::kColO + c * 16, u);
            }
          }
        }
#pragma unroll
        for (int c = 0; c < KT / 16; ++c) SG_TMEM_ST_8(tb + C::kColP + c * 8, (wv + c * 8));
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&p_full[x]);
      }
      if (!ok || !mbar_wait(&pv_done[x], (g - 1) & 1, 323)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int trow = (qa + x) * 128 + r;  // query row within the image
      const int row = img_row0 + trow;
      const bool row_ok = trow < L;
      const float inv_l = 1.f / l;
      if (p.lse != nullptr && row_ok) p.lse[static_cast<size_t>(row) * H + head] = m_use + log2f(l);
      T* orow = reinterpret_cast<T*>(p.out) + static_cast<size_t>(row) * p.ld_out + head * p.head_dim;
#pragma unroll
      for (int c = 0; c < HDP / 16; ++c) {
        uint32_t u[16];
        SG_TMEM_LD_16(tb + C::kColO + c * 16, u);
        tmem_ld_wait();
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
      // O is in registers: the next item's first PV may overwrite it
      tc_fence_before();
      mbar_arrive(&o_free[x]);
    }
    if (!ok) *abort_flag = 1;
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

}  // namespace sg
