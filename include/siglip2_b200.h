/* C ABI of libsiglip2_b200.so: the SigLIP-2 NaFlex vision-tower forward on
 * B200 (sm_100a).
 *
 * Conventions
 *  - Every pointer argument named *_dev is device memory owned by the caller
 *    (the library never allocates on the forward path).  Host arrays are
 *    named *_host.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *    stream).  All work is enqueued on it; nothing synchronises unless the
 *    function says so.
 *  - Every function returns a siglip2_status; on failure
 *    siglip2_last_error() (thread-local) describes the cause.  Arguments are
 *    validated on the host before any launch; kernels never trap.
 *  - Row-major 2-D tensors, leading dimensions in elements.  Element type of
 *    the activation/weight tensors is `dtype` (SIGLIP2_BF16 or SIGLIP2_F16 on
 *    the tensor-core path, SIGLIP2_F32 on the fp32 path); biases and the
 *    LayerNorm-folding vectors are always float32.
 *
 * Reference interfaces replaced (tohskai/SigLIP-2):
 *  siglip2_forward / siglip2_forward_padded
 *       -> Siglip2SequenceVisionTransformer.forward       model.py:260-292
 *          Siglip2SequenceVisionTransformerOptimized.forward
 *                                                          optimized_siglip2/model_optimized.py:356-388
 *          (+ transformers Siglip2VisionTransformer.forward head/padded entry)
 *  siglip2_gemm      -> nn.Linear projections               model.py:59-62,138-141,184-185
 *                       fused Linear+GELU                   optimized_siglip2/ops/MLP.py:233-304
 *                       LayerNorm feeding a Linear           model.py:211,219 / ops/layer_norm.py:364-547
 *  siglip2_layernorm -> nn.LayerNorm (post_layernorm)       model.py:256-258,286
 *  siglip2_patch_embed -> Siglip2SequenceEmbeddings.forward (patch Linear + resized
 *                       position grid)                       model.py:68-120
 *  siglip2_posemb    -> Siglip2SequenceEmbeddings pos-emb resize loop  model.py:90-119
 *  siglip2_fmha_varlen -> flex_attention + document block mask         model.py:156-163
 *  siglip2_map_head  -> transformers Siglip2MultiheadAttentionPoolingHead.forward
 *                       (modeling_siglip2.py:670-719; not in the reference)
 */
#ifndef SIGLIP2_B200_H
#define SIGLIP2_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  SIGLIP2_OK = 0,
  SIGLIP2_ERR_ARG = -1,
  SIGLIP2_ERR_ALIGN = -2,
  SIGLIP2_ERR_SHAPE = -3,
  SIGLIP2_ERR_CUDA = -4,
  SIGLIP2_ERR_TIMEOUT = -5,
  SIGLIP2_ERR_UNSUPPORTED = -6
} siglip2_status;

typedef enum { SIGLIP2_F32 = 0, SIGLIP2_BF16 = 1, SIGLIP2_F16 = 2 } siglip2_dtype;

typedef enum {
  SIGLIP2_EPI_BIAS = 0,       /* out = A.B^T + bias                                   */
  SIGLIP2_EPI_BIAS_RES = 1,   /* out = A.B^T + bias + res            (res may == out) */
  SIGLIP2_EPI_LN = 2,         /* out = rstd(A)*(A.B^T - mu(A)*c1) + c2   (LayerNorm of A folded) */
  SIGLIP2_EPI_LN_GELU = 3,    /* out = gelu_tanh(rstd(A)*(A.B^T - mu(A)*c1) + c2)      */
  SIGLIP2_EPI_BIAS_GELU = 4,  /* out = gelu_tanh(A.B^T + bias)                        */
  /* siglip2_gemm_rowsums only: LayerNorm statistics come from, or go to,
   * per-row (mean, centred sum of squares) float pairs of the residual
   * stream, in column-block slots (siglip2_rowsum_slots) */
  SIGLIP2_EPI_LN_ROWSUMS = 5,      /* as SIGLIP2_EPI_LN, mu/rstd from rs_in over K columns    */
  SIGLIP2_EPI_LN_ROWSUMS_GELU = 6, /* as SIGLIP2_EPI_LN_GELU, likewise                        */
  SIGLIP2_EPI_BIAS_RES_ROWSUMS = 7, /* as SIGLIP2_EPI_BIAS_RES, and rs_acc receives the slot
                                      statistics of the row's rounded outputs                 */
  /* 8 is the patch embedding's position epilogue (siglip2_patch_embed) */
  SIGLIP2_EPI_BIAS_GELU_GRAD = 9   /* out = res * gelu_tanh'(A.B^T + bias): the GELU backward
                                      fused into the GEMM that recomputes the pre-activation
                                      (res = the gradient w.r.t. the GELU output)            */
} siglip2_epilogue;

/* Library version (major*10000 + minor*100 + patch). */
int siglip2_version(void);

/* Thread-local description of the last failure. */
const char* siglip2_last_error(void);

/* Number of kernel launches this library has enqueued since it was loaded. */
unsigned long long siglip2_launch_count(void);

/* Failure-path self-test: enqueues one CTA that waits on an mbarrier nothing
 * arrives at; after limit_ns (<= 2 s) it gives up exactly as a stalled
 * pipeline stage would (device error flag, site 901) and returns.  A
 * following siglip2_check_device() reports SIGLIP2_ERR_TIMEOUT and the
 * context stays usable. */
int siglip2_selftest_wait_timeout(long long limit_ns, void* stream);

/* GEMM kernel selection for every later siglip2_gemm / siglip2_forward call of
 * the process: 0 = automatic (default), 1 = one SM per 128 x BN tile,
 * 2 = CTA pairs on two SMs per 256 x BN tile (tcgen05 cta_group::2). */
int siglip2_set_gemm_variant(int variant);
int siglip2_get_gemm_variant(void);

/* Attention kernel selection for every later attention launch of the
 * process: 0 = automatic (one query tile per CTA), 1 = one 128-row
 * query tile per CTA (two CTAs per SM), 2 = two query tiles of the same
 * image and head per CTA sharing each K/V tile (one CTA per SM). */
int siglip2_set_fmha_variant(int variant);
int siglip2_get_fmha_variant(void);

/* Synchronises the current device and returns SIGLIP2_ERR_TIMEOUT if a kernel
 * gave up on a bounded wait since the last reset, or SIGLIP2_ERR_SHAPE if a
 * kernel found an index outside a buffer it was given and skipped the access
 * (the failing site id is in siglip2_last_error()).  reset != 0 clears the
 * flag. */
int siglip2_check_device(int reset);

/* out[M,N] = epilogue(A[M,K] . B[N,K]^T).
 * Tensor-core path (dtype BF16/F16): K, lda, ldb, ldo, ldr multiples of 8;
 * N multiple of 8; base pointers 16-byte aligned.  For the LN epilogues
 * mu/rstd are the LayerNorm statistics of each row of A over its K columns
 * (eps applied), c1/c2 the folded column vectors [N]. */
int siglip2_gemm(int dtype, int epilogue, const void* a_dev, int lda, const void* b_dev, int ldb, void* out_dev,
                 int ldo, int M, int N, int K, const float* bias_dev, const void* res_dev, int ldr,
                 const float* c1_dev, const float* c2_dev, float eps, void* stream);

/* Backward GEMMs on the tensor cores without transposed copies:
 *   out[M, N] = epilogue(op(A) . op(B)^T)
 * op(A) = A stored [M][K] (trans_a = 0) or A stored [K][M] (trans_a = 1);
 * op(B) = B stored [N][K] (trans_b = 0) or B stored [K][N] (trans_b = 1).
 * dgrad of y = x W^T:  dx = dy . W    -> trans_a = 0, trans_b = 1 (B = W [N_out][K_in]);
 * wgrad:               dW = dy^T . x  -> trans_a = 1 (A = dy [tokens][N_out]),
 *                                         trans_b = 1 (B = x [tokens][K_in]).
 * Epilogues: SIGLIP2_EPI_BIAS (bias may be NULL) and SIGLIP2_EPI_BIAS_GELU_GRAD.
 * bf16/f16; M, N, K and leading dimensions multiples of 8.  The transposed
 * operand arrives by 64 x 64 TMA boxes and the tcgen05 MMA reads it as an
 * MN-major operand.  Replaces the matmuls of the autograd backward of the
 * reference's Linear layers (model.py:138-141, 183-184; the fused
 * linear+GELU backward of optimized_siglip2/ops/MLP.py:409-553). */
int siglip2_gemm_t(int dtype, int epilogue, int trans_a, int trans_b, const void* a_dev, int lda, const void* b_dev,
                   int ldb, void* out_dev, int ldo, int M, int N, int K, const float* bias_dev, const void* res_dev,
                   int ldr, void* stream);

/* siglip2_gemm_t (SIGLIP2_EPI_BIAS, trans_b = 1) with a caller-provided
 * fp32 workspace for splitting K: when the M x N output has too few
 * 128 x 256 tiles to fill the SMs (weight gradients: dW [N_out, K_in] over
 * K = tokens), K is cut into slices of at least 1024 elements, each slice's
 * partial product goes to the workspace and a second kernel sums the slices
 * in order (+ bias), so the result is deterministic.
 * siglip2_gemm_t_workspace_size returns the bytes the split needs (0: no
 * split for this shape; then siglip2_gemm_t_ws runs as siglip2_gemm_t and
 * the workspace may be NULL).  Replaces the weight-gradient matmuls of the
 * autograd backward of the reference's Linear layers (model.py:138-141,
 * 183-184). */
size_t siglip2_gemm_t_workspace_size(int epilogue, int trans_a, int trans_b, int M, int N, int K);

/* Column sums of x [rows, cols] (row stride ld) in fp32, as per-chunk
 * partials part [ceil(rows / chunk_rows), cols] that the caller sums over
 * chunks in order (deterministic): the bias gradient of a Linear layer
 * (db = sum over tokens of dy; the autograd backward of model.py:138-141,
 * 183-184).  cols and ld multiples of 8, x 16-byte aligned. */
int siglip2_colsum_partial(int dtype, const void* x_dev, int ld, int rows, int cols, int chunk_rows, float* part_dev,
                           void* stream);
int siglip2_gemm_t_ws(int dtype, int epilogue, int trans_a, int trans_b, const void* a_dev, int lda, const void* b_dev,
                      int ldb, void* out_dev, int ldo, int M, int N, int K, const float* bias_dev, void* workspace_dev,
                      size_t workspace_bytes, void* stream);

/* 8-bit (e4m3) GEMM operands, the fp8 variant of the projections (the
 * reference's nn.Linear layers, model.py:138-141, 183-184, run at bf16 there;
 * the reference has no 8-bit path).
 *
 * siglip2_quantize_e4m3: per-row quantisation of x [rows, cols] (dtype
 * F32/BF16/F16, row stride ldx elements) into e4m3 codes q [rows, cols]
 * (row stride ldq bytes) and scale [rows]:
 *   scale[r] = max_c |x[r,c]| / 448,  q[r,c] = e4m3_rne_satfinite(x[r,c] * (448 / max_c |x[r,c]|))
 * (an all-zero row: scale 0, zero codes).  Per-token scales for activations,
 * per-output-channel scales for a weight [N_out, K].  cols, ldx and ldq
 * multiples of 8 (ldq of 16 for a GEMM operand), x and q 16-byte aligned.
 *
 * siglip2_gemm_e4m3: out[M,N] = epilogue(a_scale[m] * b_scale[n] *
 * (A[M,K] . B[N,K]^T)) with A and B e4m3 codes (row strides lda / ldb in
 * bytes), fp32 accumulation (tcgen05.mma kind::f8f6f4 on SM pairs), out in
 * out_dtype (BF16 or F16).  Epilogues SIGLIP2_EPI_BIAS, SIGLIP2_EPI_BIAS_RES,
 * SIGLIP2_EPI_BIAS_GELU; bias [N] required.  K, lda, ldb multiples of 16; N,
 * ldo, ldr multiples of 8; pointers 16-byte aligned. */
int siglip2_quantize_e4m3(int dtype, const void* x_dev, int ldx, int rows, int cols, void* q_dev, int ldq,
                          float* scale_dev, void* stream);
int siglip2_gemm_e4m3(int out_dtype, int epilogue, const void* a_dev, int lda, const float* a_scale_dev,
                      const void* b_dev, int ldb, const float* b_scale_dev, void* out_dev, int ldo, int M, int N, int K,
                      const float* bias_dev, const void* res_dev, int ldr, void* stream);

/* LayerNorm statistics for the LayerNorm-folded GEMMs are kept per column
 * block ("slots"): a [rows][S] array of float pairs (mean, centred sum of
 * squares) of the block's values, S = siglip2_rowsum_slots(dtype, width) for
 * rows of `width` columns, slot j covering columns [j * blk, min((j + 1) *
 * blk, width)) with blk = siglip2_rowsum_block(dtype, width) (half a GEMM
 * tile).  Each slot is written once by the GEMM that produces the rows (from
 * sums shifted by the block's first value, so a large row mean does not
 * cancel the variance) and merged in slot order by the GEMM that reads them
 * (mean = sum n_j mean_j / width, M2 = sum M2_j + n_j (mean_j - mean)^2), so
 * results do not depend on scheduling. */
int siglip2_rowsum_slots(int dtype, int width);
int siglip2_rowsum_block(int dtype, int width);

/* Slot statistics of x [M, K] (row pitch ldx elements) in the layout above:
 * rs_dev[r * siglip2_rowsum_slots(dtype, K) + j] = (mean, centred sum of
 * squares) of row r over column block j.  For rows no row-sum GEMM produced, e.g. the
 * input of a stand-alone encoder layer (Siglip2EncoderLayer.forward,
 * model.py:204-223).  x 16-byte aligned; K and ldx multiples of 8 (bf16,
 * f16) or 4 (f32); rs_dev 8-byte aligned. */
int siglip2_rowsums(int dtype, const void* x_dev, int ldx, int M, int K, float* rs_dev, void* stream);

/* siglip2_gemm with row-sum LayerNorm plumbing: the GEMM that writes the
 * residual stream (SIGLIP2_EPI_BIAS_RES_ROWSUMS) writes each row's slot
 * statistics into rs_acc ([M][siglip2_rowsum_slots(dtype, N)] pairs), and the
 * LayerNorm-folded GEMM that reads it (SIGLIP2_EPI_LN_ROWSUMS[_GELU]) merges
 * rs_in ([M][siglip2_rowsum_slots(dtype, K)] pairs) into mu and rstd =
 * 1/sqrt(M2/K + eps), so no pass over the rows is needed for LayerNorm
 * statistics.  Pointers not used by the epilogue may be
 * NULL; row-sum buffers must be 8-byte aligned. */
int siglip2_gemm_rowsums(int dtype, int epilogue, const void* a_dev, int lda, const void* b_dev, int ldb,
                         void* out_dev, int ldo, int M, int N, int K, const float* bias_dev, const void* res_dev,
                         int ldr, const float* c1_dev, const float* c2_dev, float eps, const float* rs_in_dev,
                         float* rs_acc_dev, void* stream);

/* Patch embedding with the position embedding fused into the GEMM epilogue:
 *   out[t] = patches[t] . W^T + bias + resize(table)(t)      (out [N, D])
 * where token t is pixel (y, x) = divmod(t - cu[b], w) of image
 * b = tok_img[t] with grid (h, w) = hw[2b], hw[2b+1], and resize is the
 * antialiased bilinear interpolation of the grid x grid fp32 table
 * [grid^2, D].  rs_acc ([N][siglip2_rowsum_slots(dtype, D)] float pairs)
 * receives the slot statistics of the rounded out rows: the LayerNorm
 * statistics of the first layer.  Replaces Siglip2SequenceEmbeddings.forward,
 * model.py:68-120. */
int siglip2_patch_embed(int dtype, const void* patches_dev, int patch_dim, const void* w_dev, const float* bias_dev,
                        const float* table_dev, int grid, const int* tok_img_dev, const int* hw_dev,
                        const int* cu_seqlens_dev, int N, int D, void* out_dev, float* rs_acc_dev, void* stream);

/* LayerNorm over the last dimension (fp32 statistics, biased variance).
 * Packed mode (cu_seqlens_dev == NULL): y[r] = LN(x[r]) for r < rows.
 * Padded mode: rows = B * max_patches destination rows; destination (b, i)
 * is LN(x[cu[b] + i]) when i < cu[b+1] - cu[b], else zeros.
 * Replaces nn.LayerNorm (post_layernorm, model.py:256-258,286). */
int siglip2_layernorm(int dtype, const void* x_dev, void* y_dev, const float* gamma_dev, const float* beta_dev,
                      int rows, int D, float eps, const int* cu_seqlens_dev, int max_patches, void* stream);

/* Gradient of siglip2_layernorm (packed rows): dx [rows, D] (dtype), the
 * row statistics stats_dev [rows] (mean, rstd) float pairs (scratch), and
 * per-chunk partial sums dgamma_part / dbeta_part [ceil(rows / chunk_rows), D]
 * fp32 (the caller sums them over chunks, in order):
 *   dx = rstd (g - mean(g) - xh mean(g xh)), g = dy gamma, xh = (x - mean) rstd;
 *   dgamma = sum_rows dy xh,  dbeta = sum_rows dy.
 * Replaces the autograd backward of nn.LayerNorm (model.py:199,201,256) and
 * of the reference's Triton LayerNorm (optimized_siglip2/ops/layer_norm.py:571-940). */
int siglip2_layernorm_backward(int dtype, const void* x_dev, const void* dy_dev, const float* gamma_dev, int rows,
                               int D, float eps, void* dx_dev, float* stats_dev, float* dgamma_part_dev,
                               float* dbeta_part_dev, int chunk_rows, void* stream);

/* Patch grid (grid_h, grid_w) of a height x width image under a budget of
 * max_patches patches of patch x patch pixels: the largest scale whose
 * patch-rounded size fits, found by the binary search of transformers'
 * get_image_size_for_max_num_patches (models/siglip2/image_processing_siglip2.py),
 * restated step for step so that the grids agree exactly. Host only. */
int siglip2_image_grid(int height, int width, int patch, int max_patches, int* grid_h, int* grid_w);

/* The preprocessing in front of the tower (transformers Siglip2ImageProcessor,
 * torchvision backend, image_processing_siglip2.py _preprocess): for image b,
 * uint8 pixels at images_dev + offsets_dev[b], channels first (C x H x W) or
 * channels last (H x W x C), source size src_hw[2b], src_hw[2b+1]:
 *   - resize to (grid_h * patch, grid_w * patch) with antialiased bilinear
 *     filtering and round half to even (torchvision's resize of a uint8 CUDA
 *     tensor), skipped when the size already matches; downscaling by more
 *     than 19x per axis is rejected;
 *   - normalise channel c to (x - mean[c]) / std_dev_values[c] in fp32, where
 *     mean and std are in uint8 units (image_mean / rescale_factor, e.g. 127.5);
 *   - write patch (y, x) as row y * grid_w + x of pixel_values [batch,
 *     max_patches, patch * patch * channels] (element (py, px, c) at
 *     (py * patch + px) * channels + c, in dtype), rows past grid_h * grid_w
 *     zero, and mask [batch, max_patches] int32 = 1 for the valid rows.
 * Sizes and grids are passed twice: on the host (checks, shared-memory size)
 * and on the device (read by the kernel). channels 1..4, patch <= 32,
 * patch * patch * channels a multiple of 8, pixel_values 16-byte aligned.
 * One launch; HBM-bound without a resize. */
int siglip2_patchify(int dtype, const uint8_t* images_dev, const long long* offsets_dev, const int* src_hw_host,
                     const int* src_hw_dev, const int* grid_hw_host, const int* grid_hw_dev, int batch, int channels,
                     int patch, int channels_last, const float* mean, const float* std_dev_values, int max_patches,
                     void* pixel_values_dev, int* mask_dev, void* stream);

/* y[r] = scale * x[r] / ||x[r]||_2 for rows r < rows of width D (fp32 sum of
 * squares; an all-zero row gives zeros).  The embedding normalisation before
 * the image-text logits of transformers' Siglip2Model.forward
 * (models/siglip2/modeling_siglip2.py:964-972), with exp(logit_scale) passed
 * as scale for one side; the logits are then one siglip2_gemm with the bias
 * epilogue (bias = logit_bias).  x, y 16-byte aligned; D, ldx, ldy multiples
 * of 8 (bf16, f16) or 4 (f32). */
int siglip2_l2_normalize(int dtype, const void* x_dev, int ldx, int rows, int D, float scale, void* y_dev, int ldy,
                         void* stream);

/* tok_img[t] = image index of packed token t (cu_seqlens_dev has B+1 entries). */
int siglip2_token_image(const int* cu_seqlens_dev, int B, int N, int* tok_img_dev, void* stream);

/* Position embeddings for the packed sequence: out[t] = antialiased bilinear
 * resize of the grid x grid table (float32 [grid*grid, D], row-major h, w)
 * to image (h, w) = hw_dev[2b], hw_dev[2b+1], evaluated at token t's (y, x).
 * Replaces the per-image F.interpolate loop, model.py:90-116. */
int siglip2_posemb(int dtype, const float* table_dev, int grid, int D, const int* tok_img_dev, const int* hw_dev,
                   const int* cu_seqlens_dev, int N, void* out_dev, void* stream);

/* Per-image attention over the packed sequence.  qkv_dev: [N, 3*heads*head_dim],
 * column (w*heads + h)*head_dim + d holds q (w=0), k (w=1), v (w=2) of head
 * h, dim d (the fused qkv_proj output of model_optimized.py); row pitch
 * 3*heads*head_dim, base 16-byte aligned.  tiles_dev: n_tiles (image, query_tile) int32
 * pairs covering ceil(L_b / 128) query tiles of every image.  out_dev:
 * [N, ldo] receives softmax(q k^T / sqrt(head_dim)) v per head at columns
 * h*head_dim ...  Replaces flex_attention with the document mask,
 * model.py:156-163. */
int siglip2_fmha_varlen(int dtype, const void* qkv_dev, int N, const int* cu_seqlens_dev, const int* tiles_dev,
                        int n_tiles, int heads, int head_dim, void* out_dev, int ldo, void* stream);

/* siglip2_fmha_varlen in train mode: the reference's attention-output
 * dropout (model.py:166-169, nn.functional.dropout of the per-head output
 * before out_proj) applied in the same launch, as the output is stored:
 * element e = row * heads*head_dim + col of the logical output is kept and
 * scaled by 1 / (1 - p) when u(e) >= p, else zeroed, with u(e) in [0, 1)
 * from the counter-based generator Philox4x32-10 (counter = (e / 4, offset),
 * key = seed, word e % 4, u = (word >> 8) * 2^-24).  The mask is a pure
 * function of (seed, offset, e): siglip2_dropout with the same arguments
 * regenerates it (the backward applies it to the incoming gradient).
 * 0 <= p < 1. */
int siglip2_fmha_varlen_dropout(int dtype, const void* qkv_dev, int N, const int* cu_seqlens_dev, const int* tiles_dev,
                                int n_tiles, int heads, int head_dim, void* out_dev, int ldo, float p,
                                unsigned long long seed, unsigned long long offset, void* stream);

/* The training forward: siglip2_fmha_varlen_dropout (p = 0: no dropout) that
 * also writes lse_dev [N, heads] float32, the base-2 log-sum-exp of each
 * query row's scaled logits (softmax_k = exp2(q.k * scale * log2(e) - lse)),
 * which the backward needs.  bf16 / f16. */
int siglip2_fmha_varlen_train(int dtype, const void* qkv_dev, int N, const int* cu_seqlens_dev, const int* tiles_dev,
                              int n_tiles, int heads, int head_dim, void* out_dev, int ldo, float* lse_dev, float p,
                              unsigned long long seed, unsigned long long offset, void* stream);

/* dsum_dev[r * heads + h] = sum_d g[r, h*head_dim + d] * o[r, h*head_dim + d]
 * (fp32): the row term D of the attention backward, from the incoming
 * gradient g and the stored (possibly dropped-out) output o, both [N, ld]. */
int siglip2_fmha_bwd_dsum(int dtype, const void* g_dev, const void* o_dev, int ld, int N, int heads, int head_dim,
                          float* dsum_dev, void* stream);

/* Attention backward on the tensor cores: dqkv_dev [N, 3*heads*head_dim]
 * (dq | dk | dv, the layout of qkv_dev) from qkv_dev, dout_dev [N, ld_dout]
 * (the gradient of the attention output, after the dropout mask), the
 * forward's lse_dev and siglip2_fmha_bwd_dsum's dsum_dev [N, heads]:
 *   dV = P^T dO, dK = scale dS^T Q, dQ = scale dS K, dS = P (dO V^T - D).
 * Two passes of one kernel over the same (image, 128-row tile) list as the
 * forward (tiles_dev): key tiles accumulate dK and dV, query tiles dQ, in
 * TMEM; no atomics, deterministic.  bf16 / f16, head_dim 64, 72 or 96.
 * Replaces the autograd backward of flex_attention (model.py:156-163). */
int siglip2_fmha_varlen_backward(int dtype, const void* qkv_dev, const void* dout_dev, int ld_dout, int N,
                                 const int* cu_seqlens_dev, const int* tiles_dev, int n_tiles, int heads,
                                 int head_dim, const float* lse_dev, const float* dsum_dev, void* dqkv_dev,
                                 void* stream);

/* y[r, c] = x[r, c] * keep(r * width + c) / (1 - p) for r < rows, c < width,
 * with the mask of siglip2_fmha_varlen_dropout (x and y may be the same
 * buffer).  width a multiple of 8; rows 16-byte aligned with pitches
 * multiples of 8 (bf16, f16) or 4 (f32) elements.  Replaces
 * nn.functional.dropout at model.py:166-169 (and its gradient). */
int siglip2_dropout(int dtype, const void* x_dev, int ldx, int rows, int width, float p, unsigned long long seed,
                    unsigned long long offset, void* y_dev, int ldy, void* stream);

/* Head dimension of the attention kernel's tiles (64 -> 64, 72 -> 80,
 * 96 -> 96); the padding exists only in shared memory and TMEM. */
int siglip2_padded_head_dim(int head_dim);

/* Attention pooling of the MAP head, first half: for every image b and head h
 *   p_jh = softmax_j(x_j . u_h)   over the image's rows j,
 *   pooled[b, h, :] = sum_j p_jh x_j            ([B, heads, D], dtype)
 * x_dev rows of image b are cu[b] + j (max_patches == 0) or b*max_patches + j.
 * u_dev [heads, D] float32 = W_k,h^T q_h * log2(e) / sqrt(head_dim) (scores
 * are base-2).  scores_dev: caller scratch of N_tokens * heads floats.
 * Replaces the probe attention of transformers
 * Siglip2MultiheadAttentionPoolingHead (modeling_siglip2.py:670-719); the
 * value/out projections and MLP follow as siglip2_gemm calls. */
int siglip2_head_pool(int dtype, const void* x_dev, int D, int heads, const int* cu_seqlens_dev, int B,
                      int max_patches, const float* u_dev, float* scores_dev, void* pooled_dev, void* stream);

/* siglip2_head_pool for callers that cannot allocate device memory when they
 * call in (a serving process that plans one fixed memory arena at start-up
 * and forbids allocation afterwards; a C/FFI host without a caching
 * allocator, where a cudaMalloc per call would synchronise the device).  No
 * counterpart in the reference.  Same inputs and result as
 * siglip2_head_pool, but the score scratch is a fixed 4 MiB device array
 * inside the library (1,048,576 floats, reserved on each GPU once the
 * library's kernels are first used there, until exit): n_tokens * heads
 * above that is rejected with SIGLIP2_ERR_SHAPE.  n_tokens must equal
 * cu_seqlens[B]; cu_seqlens lives on the device, so the kernel itself checks
 * each image's score rows against n_tokens: an image reaching past it writes
 * nothing (its pooled rows are left as they were) and the next
 * siglip2_check_device() returns SIGLIP2_ERR_SHAPE.  Nothing is allocated (no
 * cudaMalloc/cudaFree).  The first call on each device looks up
 * the array's device address once (cudaGetSymbolAddress) with that device
 * current; make that first call before any stream capture.  All calls share
 * the one array, so calls that overlap on the GPU (other streams, other host
 * threads) race: serialise them.  The scratch is fully rewritten by every
 * call before it is read, so leftover contents never leak into a result. */
int siglip2_head_pool_noalloc(int dtype, const void* x_dev, int D, int heads, const int* cu_seqlens_dev, int B,
                              int max_patches, int n_tokens, const float* u_dev, void* pooled_dev, void* stream);

/* ------------------------------------------------------------------------
 * Whole-tower forward
 * ------------------------------------------------------------------------ */

/* Model hyper-parameters (Siglip2VisionConfig, model.py:39-49). */
typedef struct {
  int hidden;         /* D */
  int intermediate;   /* I */
  int layers;
  int heads;          /* H; head_dim = D / H */
  int head_dim;
  int patch_dim;      /* num_channels * patch_size^2 */
  int pos_grid;       /* sqrt(num_patches) */
  float eps;          /* layer_norm_eps */
  int dtype;          /* siglip2_dtype of weights and activations */
  int has_head;       /* attention-pooling head present */
} siglip2_config;

/* Device pointers of one encoder layer, pre-packed by the host layer:
 *  qkv_w  [3*D, D]: rows w*D + n = (W_w * ln1.gamma)[n] for w = q, k, v
 *         (the fused qkv_proj layout);
 *  qkv_c1 = row sums of qkv_w, qkv_c2 = b + W . ln1.beta;
 *  fc1_w = W1 * ln2.gamma, fc1_c1 / fc1_c2 likewise;
 *  out_w / fc2_w as in the reference, biases float32. */
typedef struct {
  const void* qkv_w;
  const float* qkv_c1;
  const float* qkv_c2;
  const void* out_w;
  const float* out_b;
  const void* fc1_w;
  const float* fc1_c1;
  const float* fc1_c2;
  const void* fc2_w;
  const float* fc2_b;
} siglip2_layer_weights;

typedef struct {
  const void* patch_w;                  /* [D, patch_dim] */
  const float* patch_b;                 /* [D] */
  const float* pos_table;               /* [pos_grid^2, D] float32 */
  const siglip2_layer_weights* layers;  /* HOST array of `layers` entries */
  const float* post_ln_w;
  const float* post_ln_b;
  /* attention-pooling head (has_head) */
  const float* head_u;        /* [H, D] float32: W_k,h^T q_h * log2(e)/sqrt(hd), q = W_q probe + b_q */
  const void* head_v_w;       /* [D, D] = in_proj_weight[2D:3D] */
  const float* head_v_b;      /* [D] */
  const void* head_o_w;       /* [D, D] out_proj */
  const float* head_o_b;
  const void* head_fc1_w;     /* [I, D] * head.layernorm.gamma */
  const float* head_fc1_c1;
  const float* head_fc1_c2;
  const void* head_fc2_w;     /* [D, I] */
  const float* head_fc2_b;
} siglip2_weights;

/* Number of int32 entries of the metadata array for `batch` images with
 * grids hw_host[2b], hw_host[2b+1]; also returns the packed token count and
 * the number of 128-row attention tiles.  Returns <0 on invalid grids. */
int siglip2_metadata_size(const int32_t* hw_host, int batch, int* n_tokens, int* n_tiles);

/* Fill the metadata array (host memory, siglip2_metadata_size() entries):
 * cu_seqlens[B+1] | hw[2B] | zero pad to an even offset | tiles[2*n_tiles]
 * (longest images first; the tile list is read as 8-byte pairs).  The
 * caller copies it to device memory (meta_dev) for siglip2_forward. */
int siglip2_metadata(const int32_t* hw_host, int batch, int32_t* meta_host, size_t capacity);

/* Workspace bytes siglip2_forward needs for this configuration. */
size_t siglip2_workspace_size(const siglip2_config* cfg, int batch, int n_tokens);

/* The forward pass.
 *  patches_dev: packed [N, patch_dim] (max_patches == 0, the reference's
 *     forward((seq_patches, token_grids))) or padded [B, max_patches,
 *     patch_dim] whose first h*w rows per image are valid (HF-style entry);
 *  hw_host: [2B] grids; meta_dev: device copy of siglip2_metadata();
 *  last_hidden_dev: packed [N, D] or padded [B, max_patches, D] (padded rows
 *     written as zeros); pooled_dev: [B, D] or NULL (needs has_head).
 * Enqueues only this library's kernels on `stream`; no allocation, no sync. */
int siglip2_forward(const siglip2_config* cfg, const siglip2_weights* w, const void* patches_dev, int batch,
                    int max_patches, const int32_t* hw_host, const int32_t* meta_dev, void* last_hidden_dev,
                    void* pooled_dev, void* workspace_dev, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SIGLIP2_B200_H */
