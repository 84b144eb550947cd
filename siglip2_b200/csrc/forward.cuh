// Whole-tower forward on one stream: embeddings (patch GEMM + resized
// position grid), L pre-LN encoder layers, post-LayerNorm, optional
// attention-pooling head.  Every launch is one of this library's kernels;
// intermediate tensors live in the caller's workspace.
//
// Per layer (LayerNorms folded into the following GEMM, see gemm.cuh):
//   qkv  = LN1(x) Wqkv^T + b          tcgen05 GEMM, LN epilogue, head-padded layout
//   attn = varlen attention(qkv)       tcgen05 FMHA
//   x    = x + attn Wo^T + bo          tcgen05 GEMM, bias+residual epilogue (in place)
//   h    = gelu(LN2(x) W1^T + b1)      tcgen05 GEMM, LN+GELU epilogue
//   x    = x + h W2^T + b2             tcgen05 GEMM, bias+residual epilogue (in place)
#pragma once

#include <vector>

#include "head.cuh"

namespace sg {

struct Ws {  // workspace carve-up
  uint8_t* base;
  size_t off = 0;
  size_t cap;
  template <typename P>
  P* take(size_t bytes) {
    off = (off + 255) & ~size_t(255);
    P* p = reinterpret_cast<P*>(base + off);
    off += bytes;
    return p;
  }
};

inline int padded_head_dim(int hd) { return hd <= 64 ? 64 : (hd <= 80 ? 80 : 96); }

inline size_t elem_bytes(int dtype) { return dtype == SIGLIP2_F32 ? 4 : 2; }

// Layout of the metadata array (int32): cu[B+1] | hw[2B] | (pad) | tiles[2*n_tiles]
// The tile list starts at an even int32 offset: kernels read it as int2.
inline size_t meta_tiles_offset(int B) { return (3 * static_cast<size_t>(B) + 1 + 1) & ~size_t(1); }
inline size_t meta_entries(int B, int T) { return meta_tiles_offset(B) + 2 * static_cast<size_t>(T); }

inline int meta_counts(const int* hw_host, int B, int* n_tokens, int* n_tiles) {
  long long N = 0, T = 0;
  for (int b = 0; b < B; ++b) {
    const int h = hw_host[2 * b], w = hw_host[2 * b + 1];
    if (h <= 0 || w <= 0) return set_error(SIGLIP2_ERR_SHAPE, "image %d has non-positive grid %dx%d", b, h, w);
    N += static_cast<long long>(h) * w;
    T += (static_cast<long long>(h) * w + 127) / 128;
  }
  if (N > (1ll << 30)) return set_error(SIGLIP2_ERR_SHAPE, "too many tokens (%lld)", N);
  *n_tokens = static_cast<int>(N);
  *n_tiles = static_cast<int>(T);
  return SIGLIP2_OK;
}

struct FwdBuffers {
  int* tok_img;
  void* x;       // [N, D] residual stream
  void* qkv;     // [N, 3 H hd]  q | k | v
  void* attn;    // [N, D]
  void* hmid;    // [N, I]   (also the packed patch rows when the input is padded)
  float* scores; // [N, H]
  float2* rowsums; // 2 x [N][slots] (sum, sum of squares) of the residual stream rows, per column block
  void* hpool;   // [B H, D]
  void* hY;      // [B H, D]
  void* hattn;   // [B, D]
  void* ha;      // [B, D]
  void* hmid2;   // [B, I]
};

inline size_t forward_workspace(const siglip2_config* c, int B, int N, FwdBuffers* out, uint8_t* base) {
  const size_t e = elem_bytes(c->dtype);
  const int D = c->hidden, I = c->intermediate, H = c->heads;
  Ws w{base, 0, 0};
  FwdBuffers f;
  f.tok_img = w.take<int>(sizeof(int) * (N + 1));
  f.x = w.take<uint8_t>(e * N * D);
  f.qkv = w.take<uint8_t>(e * N * 3 * H * c->head_dim);
  f.attn = w.take<uint8_t>(e * N * D);
  const size_t mid = std::max<size_t>(static_cast<size_t>(I), static_cast<size_t>(c->patch_dim));
  f.hmid = w.take<uint8_t>(e * N * mid);
  f.scores = w.take<float>(sizeof(float) * N * H);
  f.rowsums = w.take<float2>(sizeof(float2) * 2 * static_cast<size_t>(N) *
                              rowsum_slots(c->dtype == SIGLIP2_F32, D));
  f.hpool = w.take<uint8_t>(e * B * H * D);
  f.hY = w.take<uint8_t>(e * B * H * D);
  f.hattn = w.take<uint8_t>(e * B * D);
  f.ha = w.take<uint8_t>(e * B * D);
  f.hmid2 = w.take<uint8_t>(e * B * I);
  if (out) *out = f;
  return w.off + 256;
}

}  // namespace sg
