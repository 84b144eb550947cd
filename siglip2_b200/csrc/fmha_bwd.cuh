// Backward of the per-image attention (fmha.cuh) on tcgen05, deterministic.
//
// With logits z = scale * q k^T per image and head, P = softmax(z) recomputed
// from the forward's base-2 log-sum-exp (P = exp2(q k^T * scale * log2(e) -
// lse2)), dO the gradient of the attention output and D = rowsum(dO . O):
//   dP = dO V^T,  dS = P . (dP - D),
//   dV = P^T dO,  dK = scale * dS^T Q,  dQ = scale * dS K.
// (With the train-mode output dropout the caller passes dO through the
// forward's mask first and D = rowsum(g . out) of the incoming gradient g
// and the stored, dropped-out output: the dropped terms vanish on both sides.)
//
// One kernel template, two passes over the same (image, 128-row tile) x head
// work list:
//   kDQ = false  item = (key tile j, head): for every query tile i of the
//                image, S = Q_i K_j^T and dP = dO_i V_j^T into TMEM, P and dS
//                into shared memory, then dV_j += P^T dO_i and dK_j += dS^T Q_i
//                accumulate in TMEM; written once at the end of the item.
//   kDQ = true   item = (query tile i, head): for every key tile j,
//                the same S, dP, P, dS, then dQ_i += dS K_j.
// No atomics: each output row is written by exactly one item.
//
// Shared memory: the item's fixed operand pair ("F": K_j, V_j or Q_i, dO_i)
// and a 2-stage ring of the streamed pair ("T": Q_i, dO_i or K_j, V_j), each
// operand [128 rows][HDP] as a 64-column 128B-swizzled slab plus an R-column
// slab (HDP = 64 + R), read through 3-D tensor maps [N][heads][head_dim] whose
// columns past head_dim arrive as zeros; P and dS as [2][128 rows][64 cols]
// 128B-swizzled bf16/f16 tiles written by the compute warps.  The
// accumulating MMAs read P / dS transposed (MN-major A, M = keys) and the
// streamed dO_i / Q_i / K_j as MN-major B operands (N = head_dim), so nothing
// is transposed in memory.
// TMEM (512 columns, one CTA per SM): S [0, 128), dP [128, 256), the first
// accumulator (dV or dQ) [256, 256 + HDP), the second (dK) [384, 384 + HDP).
//
// Warps: 0 TMA, 1 TMEM owner + MMA issuer (warp-uniform, one elected lane),
// 2-5 compute (TMEM lane quarter = warp & 3; thread = row of S / of the
// accumulators) and epilogue.
#pragma once

#include "fmha.cuh"

namespace sg {

struct FmhaBwdParams {
  const int* cu;        // [B+1]
  const int2* tiles;    // [n_tiles] (image, 128-row tile)
  int n_items;          // n_tiles * heads
  int heads;
  int head_dim;
  float scale;          // head_dim^-0.5
  float scale_log2;     // scale * log2(e)
  const float* lse;     // [N, heads] base-2 log-sum-exp of the forward
  const float* dsum;    // [N, heads] D = rowsum(dO . O)
  void* dqkv;           // [N, 3 * heads * head_dim]: dq | dk | dv
  int ld_dqkv;
};

template <int HDP>
struct FmhaBwdCfg {
  static constexpr int R = HDP - 64;
  static constexpr int kSlabA = 128 * 64 * 2;                       // 16 KB
  static constexpr int kSlabR = (128 * (R > 0 ? R : 16) * 2 + 1023) / 1024 * 1024;
  static constexpr int kOp = kSlabA + (R > 0 ? kSlabR : 0);          // one [128][HDP] operand
  static constexpr int kOpBytes = 128 * HDP * 2;                     // TMA bytes of one operand
  static constexpr int ST = 2;                                       // streamed-pair ring
  static constexpr int kF = 0;                                       // fixed pair: 2 operands
  static constexpr int kT = 2 * kOp;                                 // streamed ring: ST x 2 operands
  static constexpr int kP = kT + ST * 2 * kOp;                       // P: 2 x [128][64] (32 KB)
  static constexpr int kDS = kP + 2 * 128 * 128;                     // dS: 32 KB
  static constexpr int kBar = kDS + 2 * 128 * 128;
  static constexpr int kSmem = kBar + 256 + 1024;
  static_assert(kSmem <= 227 * 1024, "attention backward shared-memory budget");
  static constexpr uint32_t kColS = 0, kColDP = 128, kColAcc1 = 256, kColAcc2 = 384;
};

// one compute thread's chunk of 32 P or dS values into the [2][128][64] swizzled tile
template <typename T>
__device__ __forceinline__ void store_row_chunk(uint8_t* tile, int row, int c, const float* v) {
  uint8_t* rowp = tile + (c >> 1) * (128 * 128) + row * 128;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int g = (c & 1) * 4 + u;  // 16-byte piece within the 128-byte row
    uint4 o;
    o.x = Pack2<T>::pack(v[8 * u + 0], v[8 * u + 1]);
    o.y = Pack2<T>::pack(v[8 * u + 2], v[8 * u + 3]);
    o.z = Pack2<T>::pack(v[8 * u + 4], v[8 * u + 5]);
    o.w = Pack2<T>::pack(v[8 * u + 6], v[8 * u + 7]);
    *reinterpret_cast<uint4*>(rowp + ((g ^ (row & 7)) << 4)) = o;
  }
}

template <typename T, int HDP, bool kDQ>
__global__ void __launch_bounds__(192, 1)
    fmha_bwd_kernel(const __grid_constant__ CUtensorMap tmQKV, const __grid_constant__ CUtensorMap tmQKVR,
                    const __grid_constant__ CUtensorMap tmDO, const __grid_constant__ CUtensorMap tmDOR,
                    const FmhaBwdParams p) {
  using C = FmhaBwdCfg<HDP>;
  constexpr int R = C::R;
  constexpr int ST = C::ST;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescS = make_idesc(128, 128, kBF16, false, false);    // S, dP: K-major A and B
  constexpr uint32_t kIdescAcc64 = make_idesc(128, 64, kBF16, !kDQ, true);   // dV/dK: MN-major A; dQ: K-major A
  constexpr uint32_t kIdescAccR = make_idesc(128, R > 0 ? R : 16, kBF16, !kDQ, true);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBar);
  uint64_t* f_full = bars;            // 1
  uint64_t* f_empty = f_full + 1;     // 1
  uint64_t* t_full = f_empty + 1;     // ST
  uint64_t* t_empty = t_full + ST;    // ST
  uint64_t* sp_full = t_empty + ST;   // 1: S and dP computed
  uint64_t* sp_free = sp_full + 1;    // 1: S and dP read by the compute warps (128 arrivals)
  uint64_t* ps_full = sp_free + 1;    // 1: P and dS written to shared memory (128 arrivals)
  uint64_t* ps_free = ps_full + 1;    // 1: the accumulating MMAs are done with P and dS
  uint64_t* acc_full = ps_free + 1;   // 1: an item's accumulators complete
  uint64_t* acc_free = acc_full + 1;  // 1: an item's accumulators read (128 arrivals)
  uint64_t* mdone = acc_free + 1;     // 1
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mdone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int H = p.heads;

  if (threadIdx.x == 0) {
    mbar_init(f_full, 1);
    mbar_init(f_empty, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&t_full[s], 1);
      mbar_init(&t_empty[s], 1);
    }
    mbar_init(sp_full, 1);
    mbar_init(sp_free, 128);
    mbar_init(ps_full, 128);
    mbar_init(ps_free, 1);
    mbar_init(acc_full, 1);
    mbar_init(acc_free, 128);
    mbar_init(mdone, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  // item w: (image, tile) = tiles[w / H], head w % H; the streamed tiles are
  // the image's 128-row tiles on the other side (query tiles for kDQ = false)
  auto item = [&](int w, int& row0, int& L, int& tile, int& head) {
    const int2 t2 = p.tiles[w / H];
    head = w - (w / H) * H;
    row0 = __ldg(p.cu + t2.x);
    L = __ldg(p.cu + t2.x + 1) - row0;
    tile = t2.y;
  };
  // operand o of a pair at smem `base`: Q (0), K (1), V (2) columns of qkv, or dO (3)
  auto load_op = [&](uint8_t* dst, uint64_t* bar, int which, int head, int row) {
    if (which < 3) {
      tma_load_3d(dst, &tmQKV, bar, 0, which * H + head, row);
      if (R > 0) tma_load_3d(dst + C::kSlabA, &tmQKVR, bar, 64, which * H + head, row);
    } else {
      tma_load_3d(dst, &tmDO, bar, 0, head, row);
      if (R > 0) tma_load_3d(dst + C::kSlabA, &tmDOR, bar, 64, head, row);
    }
  };

  if (warp == 0) {
    // --------------------------------------------------------------- TMA
    if (lane == 0) {
      tma_prefetch_desc(&tmQKV);
      tma_prefetch_desc(&tmDO);
      if (R > 0) {
        tma_prefetch_desc(&tmQKVR);
        tma_prefetch_desc(&tmDOR);
      }
      int it = 0, ts = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < p.n_items && ok; w += gridDim.x, ++it) {
        int row0, L, tile, head;
        item(w, row0, L, tile, head);
        const int n_t = (L + 127) / 128;
        if (*abort_flag || !mbar_wait(f_empty, (it & 1) ^ 1, 400)) {
          ok = false;
          break;
        }
        // fixed pair: K_j, V_j (dK/dV pass) or Q_i, dO_i (dQ pass)
        mbar_arrive_expect_tx(f_full, 2 * C::kOpBytes);
        load_op(smem + C::kF, f_full, kDQ ? 0 : 1, head, row0 + tile * 128);
        load_op(smem + C::kF + C::kOp, f_full, kDQ ? 3 : 2, head, row0 + tile * 128);
        for (int t = 0; t < n_t; ++t, ++ts) {
          const int st = ts % ST;
          if (*abort_flag || !mbar_wait(&t_empty[st], ((ts / ST) & 1) ^ 1, 401)) {
            ok = false;
            break;
          }
          uint8_t* dst = smem + C::kT + st * 2 * C::kOp;
          mbar_arrive_expect_tx(&t_full[st], 2 * C::kOpBytes);
          load_op(dst, &t_full[st], kDQ ? 1 : 0, head, row0 + t * 128);
          load_op(dst + C::kOp, &t_full[st], kDQ ? 2 : 3, head, row0 + t * 128);
        }
      }
      if (!ok) *abort_flag = 1;
      // no TMA write may be in flight at exit: only the last load of each buffer can be outstanding
      if (it > 0) mbar_wait(f_full, (it - 1) & 1, 402);
      for (int i = (ts > ST ? ts - ST : 0); i < ts; ++i) mbar_wait(&t_full[i % ST], (i / ST) & 1, 403);
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------- MMA (warp-uniform, elected lane)
    auto wait_all = [&](uint64_t* bar, uint32_t parity, int site) -> bool {
      const bool w = !*abort_flag && mbar_wait(bar, parity, site);
      return __all_sync(0xffffffffu, w);
    };
    const uint32_t sF = smem_u32(smem + C::kF);
    const uint32_t sP = smem_u32(smem + C::kP), sDS = smem_u32(smem + C::kDS);
    // K-major operand descriptors of a [128][HDP] operand at saddr: 64-wide slab + R slab
    auto kdesc = [&](uint32_t saddr) { return kmajor_desc(saddr, 128); };
    auto kdescR = [&](uint32_t saddr) { return kmajor_desc(saddr + C::kSlabA, R > 0 ? R * 2 : 32); };
    auto mndesc = [&](uint32_t saddr) { return mnmajor_desc(saddr, 128, 0); };
    auto mndescR = [&](uint32_t saddr) { return mnmajor_desc(saddr + C::kSlabA, R > 0 ? R * 2 : 32, 0); };
    // S = A . B^T over head_dim (A: query-side operand, B: key-side operand)
    auto issue_qk = [&](uint32_t d_tmem, uint32_t a, uint32_t b) {
      const uint64_t ad = kdesc(a), bd = kdesc(b), ard = kdescR(a), brd = kdescR(b);
#pragma unroll
      for (int k = 0; k < 4; ++k) umma_ss(d_tmem, ad + 2 * k, bd + 2 * k, kIdescS, k > 0);
#pragma unroll
      for (int k = 0; k < R / 16; ++k) umma_ss(d_tmem, ard + 2 * k, brd + 2 * k, kIdescS, 1);
    };
    // acc (+)= X . Y over 128 rows of the streamed side: X = P^T or dS^T (MN-major, dK/dV pass) or dS
    // (K-major, dQ pass); Y = the streamed operand read MN-major (N = head_dim)
    auto issue_acc = [&](uint32_t d_tmem, uint32_t x_tile, uint32_t y, bool first) {
      const uint64_t yd = mndesc(y), yrd = mndescR(y);
#pragma unroll
      for (int s = 0; s < 8; ++s) {  // 16 rows of the contraction per MMA
        uint64_t xd;
        if constexpr (kDQ) {
          // dS [q][k] as K-major A: k in [64c, 64c + 64) lives in chunk c = s / 4, 32 bytes per 16 k
          xd = kmajor_desc(x_tile + (s >> 2) * (128 * 128) + (s & 3) * 32, 128);
        } else {
          // P / dS [q][k] read as the MN-major A of P^T / dS^T: 16 q-rows = 2 KB; key chunks 16 KB apart
          xd = smem_desc(x_tile + s * 2048, 128 * 128, 1024, kSw128);
        }
        const uint32_t acc = (!first || s > 0) ? 1u : 0u;
        umma_ss(d_tmem, xd, yd + static_cast<uint64_t>(s * 2048 / 16), kIdescAcc64, acc);
        if constexpr (R > 0)
          umma_ss(d_tmem + 64, xd, yrd + static_cast<uint64_t>(s * 16 * R * 2 / 16), kIdescAccR, acc);
      }
    };
    int it = 0, ts = 0, gs = 0;
    bool ok = true;
    // the accumulating MMAs of step g (streamed stage st)
    auto do_acc = [&](int g, int st, bool first, int item_idx) -> bool {
      if (!wait_all(ps_full, g & 1, 412)) return false;
      if (first && item_idx > 0 && !wait_all(acc_free, (item_idx - 1) & 1, 413)) return false;
      tc_fence_after();
      const uint32_t sT = smem_u32(smem + C::kT + st * 2 * C::kOp);
      if (elect_one()) {
        if constexpr (kDQ) {
          issue_acc(tmem + C::kColAcc1, sDS, sT, first);                 // dQ += dS K_j
        } else {
          issue_acc(tmem + C::kColAcc1, sP, sT + C::kOp, first);         // dV += P^T dO_i
          issue_acc(tmem + C::kColAcc2, sDS, sT, first);                 // dK += dS^T Q_i
        }
        umma_commit(ps_free);
        umma_commit(&t_empty[st]);
      }
      __syncwarp();
      return true;
    };
    for (int w = blockIdx.x; w < p.n_items && ok; w += gridDim.x, ++it) {
      int row0, L, tile, head;
      item(w, row0, L, tile, head);
      const int n_t = (L + 127) / 128;
      if (!wait_all(f_full, it & 1, 410)) {
        ok = false;
        break;
      }
      for (int t = 0; t < n_t; ++t, ++ts, ++gs) {
        const int st = ts % ST;
        if (!wait_all(&t_full[st], (ts / ST) & 1, 411) || (gs > 0 && !wait_all(sp_free, (gs - 1) & 1, 414))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sT = smem_u32(smem + C::kT + st * 2 * C::kOp);
        if (elect_one()) {
          // query side first: dK/dV pass: Q_i, dO_i streamed; dQ pass: Q_i, dO_i fixed
          const uint32_t q = kDQ ? sF : sT, dO = kDQ ? sF + C::kOp : sT + C::kOp;
          const uint32_t k = kDQ ? sT : sF, v = kDQ ? sT + C::kOp : sF + C::kOp;
          issue_qk(tmem + C::kColS, q, k);     // S = Q K^T
          issue_qk(tmem + C::kColDP, dO, v);   // dP = dO V^T
          umma_commit(sp_full);
          if (t == n_t - 1) umma_commit(f_empty);  // the fixed pair is read by S / dP only
        }
        __syncwarp();
        if (t > 0 && !do_acc(gs - 1, (ts - 1) % ST, t == 1, it)) {
          ok = false;
          break;
        }
      }
      if (!ok) break;
      if (!do_acc(gs - 1, (ts - 1) % ST, n_t == 1, it)) {
        ok = false;
        break;
      }
      if (elect_one()) umma_commit(acc_full);
      __syncwarp();
    }
    if (!ok && lane == 0) *abort_flag = 1;
    if (elect_one()) {
      umma_commit(mdone);
      mbar_wait(mdone, 0, 416);
    }
    __syncwarp();
  } else {
    // --------------------------------------------------------------- compute + epilogue
    const int q4 = warp & 3;         // TMEM lane quarter
    const int r = q4 * 32 + lane;    // row of S (query) / of the accumulators
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    uint8_t* tP = smem + C::kP;
    uint8_t* tDS = smem + C::kDS;
    bool ok = true;
    int it = 0, gs = 0;
    for (int w = blockIdx.x; w < p.n_items && ok; w += gridDim.x, ++it) {
      int row0, L, tile, head;
      item(w, row0, L, tile, head);
      const int n_t = (L + 127) / 128;
      for (int t = 0; t < n_t; ++t, ++gs) {
        // this step's query tile and key tile (within the image)
        const int qt = kDQ ? tile : t, kt = kDQ ? t : tile;
        const int qrow = qt * 128 + r;
        const bool q_ok = qrow < L;
        const int k_valid = L - kt * 128;  // keys of this image in the key tile (>= 1)
        float lse = 0.f, dsum = 0.f;
        if (q_ok) {
          lse = __ldg(p.lse + static_cast<size_t>(row0 + qrow) * H + head);
          dsum = __ldg(p.dsum + static_cast<size_t>(row0 + qrow) * H + head);
        }
        if (*abort_flag || !mbar_wait(sp_full, gs & 1, 421) ||
            (gs > 0 && !mbar_wait(ps_free, (gs - 1) & 1, 422))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t us[32], ud[32];
          SG_TMEM_LD_32(tmem + C::kColS + c * 32 + lane_off, us);
          SG_TMEM_LD_32(tmem + C::kColDP + c * 32 + lane_off, ud);
          tmem_ld_wait();
          if (c == 3) {
            // S and dP are in registers: the next step's MMAs may overwrite them
            tc_fence_before();
            mbar_arrive(sp_free);
          }
          float pv[32], dv[32];
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            const bool valid = q_ok && (c * 32 + k) < k_valid;
            const float pk = valid ? ex2_approx(fmaf(__uint_as_float(us[k]), p.scale_log2, -lse)) : 0.f;
            pv[k] = pk;
            dv[k] = pk * (__uint_as_float(ud[k]) - dsum);
          }
          store_row_chunk<T>(tP, r, c, pv);
          store_row_chunk<T>(tDS, r, c, dv);
        }
        fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
        mbar_arrive(ps_full);
      }
      if (!ok) break;
      // ------------------------------------------------------------- epilogue: accumulators -> dqkv
      if (*abort_flag || !mbar_wait(acc_full, it & 1, 423)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int orow = tile * 128 + r;  // row of the accumulators within the image
      const bool row_ok = orow < L;
      T* base = reinterpret_cast<T*>(p.dqkv) + static_cast<size_t>(row0 + orow) * p.ld_dqkv;
#pragma unroll
      for (int a = 0; a < (kDQ ? 1 : 2); ++a) {
        // dQ pass: dQ * scale -> q columns; dK/dV pass: acc1 = dV -> v columns, acc2 = dK * scale -> k columns
        const uint32_t col = a == 0 ? C::kColAcc1 : C::kColAcc2;
        const float f = kDQ ? p.scale : (a == 0 ? 1.f : p.scale);
        const int which = kDQ ? 0 : (a == 0 ? 2 : 1);
        T* orow_p = base + (which * H + head) * p.head_dim;
#pragma unroll
        for (int c = 0; c < HDP / 16; ++c) {
          uint32_t u[16];
          SG_TMEM_LD_16(tmem + col + c * 16 + lane_off, u);
          tmem_ld_wait();
          if (row_ok) {
#pragma unroll
            for (int gg = 0; gg < 2; ++gg) {
              const int d0 = c * 16 + gg * 8;
              if (d0 < p.head_dim) {
                uint4 o;
                o.x = Pack2<T>::pack(__uint_as_float(u[gg * 8 + 0]) * f, __uint_as_float(u[gg * 8 + 1]) * f);
                o.y = Pack2<T>::pack(__uint_as_float(u[gg * 8 + 2]) * f, __uint_as_float(u[gg * 8 + 3]) * f);
                o.z = Pack2<T>::pack(__uint_as_float(u[gg * 8 + 4]) * f, __uint_as_float(u[gg * 8 + 5]) * f);
                o.w = Pack2<T>::pack(__uint_as_float(u[gg * 8 + 6]) * f, __uint_as_float(u[gg * 8 + 7]) * f);
                *reinterpret_cast<uint4*>(orow_p + d0) = o;
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(acc_free);
    }
    if (!ok) *abort_flag = 1;
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// D[r, h] = sum_d g[r, h*hd + d] * o[r, h*hd + d] (fp32), one thread per (row, head)
template <typename T>
__global__ void fmha_bwd_dsum_kernel(const T* __restrict__ g, const T* __restrict__ o, int ld, int N, int H, int hd,
                                     float* __restrict__ dsum) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(N) * H) return;
  const long long r = i / H;
  const int h = static_cast<int>(i - r * H);
  const T* gr = g + r * ld + h * hd;
  const T* orr = o + r * ld + h * hd;
  float s = 0.f;
  for (int d = 0; d < hd; d += 8) {
    float a[8], b[8];
    if constexpr (sizeof(T) == 4) {
      load_vec(gr + d, a);
      load_vec(gr + d + 4, a + 4);
      load_vec(orr + d, b);
      load_vec(orr + d + 4, b + 4);
    } else {
      load_vec(gr + d, a);
      load_vec(orr + d, b);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) s = fmaf(a[k], b[k], s);
  }
  dsum[i] = s;
}

}  // namespace sg
