"""The kernels as ``torch.library`` custom ops, namespace ``siglip2_b200``.

Each op runs one C-ABI entry point of ``libsiglip2_b200.so`` on the current
CUDA stream.  Only a CUDA kernel is registered: called with CPU tensors the
ops raise, there is no CPU implementation.  Every op has a shape-only fake
implementation, so ``torch.compile`` / ``torch.export`` trace through the
module forwards instead of breaking the graph there.  This is the mechanism
the reference uses for its Triton LayerNorm
(``optimized_siglip2/ops/layer_norm.py:19-75,425-429``).

Ops (``torch.ops.siglip2_b200.<name>``):
  gemm, gemm_rowsums, rowsums  -- tensor-core GEMMs with fused epilogues
  fmha_varlen                  -- per-image attention over packed rows (with
                                  the train-mode output dropout)
  layernorm                    -- LayerNorm over the last dimension
  token_image, patch_embed     -- patch Linear + resized position grid
  vision_tower                 -- the whole tower (``siglip2_forward``)

Backward: ``gemm`` (bias, bias + GELU-tanh and bias + residual epilogues;
tensor-core dgrad / wgrad through ``gemm_t``), ``layernorm``, ``fmha_varlen``
and ``patch_embed`` have an autograd formula (below); back-propagating through
any other op raises.
"""
from __future__ import annotations

import math
from typing import Optional

import numpy as np
import torch
from torch import Tensor

from . import _lib as L
from . import ops

_TORCH_DT = {L.DTYPE_F32: torch.float32, L.DTYPE_BF16: torch.bfloat16, L.DTYPE_F16: torch.float16}


def _slots(dtype: torch.dtype, width: int) -> int:
    return ops.rowsum_slots(dtype, width)


# --------------------------------------------------------------------------- gemm
@torch.library.custom_op("siglip2_b200::gemm", mutates_args=(), device_types="cuda")
def gemm(a: Tensor, w: Tensor, epilogue: int, bias: Optional[Tensor], res: Optional[Tensor], c1: Optional[Tensor],
         c2: Optional[Tensor], eps: float) -> Tensor:
    """``epilogue(a @ w.T)`` (``siglip2_gemm``); a [M, K], w [N, K]."""
    return ops.gemm(a, w, epilogue, bias, res, c1, c2, eps)


@gemm.register_fake
def _(a, w, epilogue, bias, res, c1, c2, eps):
    return a.new_empty((a.shape[0], w.shape[0]))


@torch.library.custom_op("siglip2_b200::gemm_t", mutates_args=(), device_types="cuda")
def gemm_t(a: Tensor, b: Tensor, trans_a: bool, trans_b: bool, epilogue: int, bias: Optional[Tensor],
           res: Optional[Tensor]) -> Tensor:
    """``siglip2_gemm_t``: ``epilogue(op(a) @ op(b).T)``, op = transpose when
    the flag is set (the operand is read as MN-major tiles, not copied).
    Plain products with a transposed ``b`` (dgrad, wgrad) go through
    ``siglip2_gemm_t_ws``, which splits K when the output has few tiles."""
    if trans_b and epilogue == L.EPI_BIAS and res is None:
        return ops.gemm_t_splitk(a, b, trans_a, bias)
    return ops.gemm_t(a, b, trans_a, trans_b, epilogue, bias, res)


@gemm_t.register_fake
def _(a, b, trans_a, trans_b, epilogue, bias, res):
    M = a.shape[1] if trans_a else a.shape[0]
    N = b.shape[1] if trans_b else b.shape[0]
    return a.new_empty((M, N))


# Backward of the plain epilogues (bias, bias + GELU-tanh, bias + residual).
# bf16/f16: dgrad dA = dY W and wgrad dW = dY^T A run on the tensor cores with
# the transposed operands read in place (siglip2_gemm_t); for bias + GELU the
# pre-activation is recomputed by a GEMM whose epilogue multiplies the incoming
# gradient by GELU-tanh' (SIGLIP2_EPI_BIAS_GELU_GRAD), so the GELU backward is
# fused into that GEMM.  fp32 (and shapes the tensor-core path rejects): the
# same products on the library GEMM over transposed copies, the contracted
# dimension zero-padded to a multiple of 8.  Bias sums are fp32 torch.
_GELU_K0 = math.sqrt(2.0 / math.pi)
_GELU_K1 = 0.044715


def _gelu_tanh_grad(z: Tensor) -> Tensor:
    """d/dz of 0.5 z (1 + tanh(k0 (z + k1 z^3))), fp32."""
    t = torch.tanh(_GELU_K0 * (z + _GELU_K1 * z * z * z))
    return 0.5 * (1 + t) + 0.5 * z * (1 - t * t) * _GELU_K0 * (1 + 3 * _GELU_K1 * z * z)


def _matmul_nt(a: Tensor, b: Tensor) -> Tensor:
    """``a [M, K] @ b [N, K].T`` on ``siglip2_gemm`` (K and N zero-padded to
    multiples of 8 for the tensor-core path)."""
    mult = 1 if a.dtype == torch.float32 else 8
    M, K = a.shape
    N = b.shape[0]
    Kp, Np = -(-K // mult) * mult, -(-N // mult) * mult
    if Kp != K or not a.is_contiguous():
        a = torch.nn.functional.pad(a, (0, Kp - K)).contiguous()
    if Kp != K or Np != N or not b.is_contiguous():
        b = torch.nn.functional.pad(b, (0, Kp - K, 0, Np - N)).contiguous()
    zero = torch.zeros(Np, dtype=torch.float32, device=a.device)
    # through the registered op, so that the backward traces under torch.compile
    return gemm(a, b, L.EPI_BIAS, zero, None, None, None, 0.0)[:, :N]


@torch.library.custom_op("siglip2_b200::colsum", mutates_args=(), device_types="cuda")
def colsum(x: Tensor) -> Tensor:
    """``siglip2_colsum_partial``: fp32 column sums of ``x`` [rows, cols] (a
    bias gradient), deterministic."""
    return ops.colsum(x.contiguous())


@colsum.register_fake
def _(x):
    return x.new_empty((x.shape[1],), dtype=torch.float32)


def _bias_grad(g: Tensor) -> Tensor:
    if g.dim() == 2 and g.shape[1] % 8 == 0 and g.dtype in (torch.bfloat16, torch.float16, torch.float32):
        return colsum(g)
    return g.sum(0, dtype=torch.float32)


def _gemm_setup(ctx, inputs, output):
    a, w, epilogue, bias, res, c1, c2, eps = inputs
    ctx.epilogue = epilogue
    ctx.save_for_backward(a, w, bias)


def _tensor_core_backward(a: Tensor, w: Tensor, grad: Tensor) -> bool:
    """The transposed-operand GEMMs apply: half precision, row pitches and
    the output widths multiples of 8 elements."""
    return (a.dtype in (torch.bfloat16, torch.float16) and a.dtype == w.dtype == grad.dtype
            and a.shape[1] % 8 == 0 and w.shape[0] % 8 == 0)


def _dgrad(g: Tensor, w: Tensor) -> Tensor:
    """dA = dY W: [M, N] x [N, K] with W read as the MN-major B operand."""
    return gemm_t(g.contiguous(), w.contiguous(), False, True, L.EPI_BIAS, None, None)


def _wgrad(g: Tensor, a: Tensor) -> Tensor:
    """dW = dY^T A: [N, M] x [M, K] with both read as MN-major operands."""
    return gemm_t(g.contiguous(), a.contiguous(), True, True, L.EPI_BIAS, None, None)


def _gemm_backward(ctx, grad):
    a, w, bias = ctx.saved_tensors
    if ctx.epilogue not in (L.EPI_BIAS, L.EPI_BIAS_GELU, L.EPI_BIAS_RES):
        raise NotImplementedError("siglip2_b200::gemm: backward exists for the bias, bias+GELU and bias+residual "
                                  "epilogues only")
    g = grad
    tc = _tensor_core_backward(a, w, grad)
    if ctx.epilogue == L.EPI_BIAS_GELU:
        if tc:  # pre-activation recomputed, times GELU-tanh', in one GEMM epilogue
            g = gemm(a.contiguous(), w.contiguous(), L.EPI_BIAS_GELU_GRAD, bias, grad.contiguous(), None, None, 0.0)
        else:
            z = gemm(a.contiguous(), w.contiguous(), L.EPI_BIAS, bias, None, None, None, 0.0)
            g = (grad.float() * _gelu_tanh_grad(z.float())).to(grad.dtype)
    if tc:
        da = _dgrad(g, w) if ctx.needs_input_grad[0] else None
        dw = _wgrad(g, a) if ctx.needs_input_grad[1] else None
    else:
        da = _matmul_nt(g, w.t()) if ctx.needs_input_grad[0] else None
        dw = _matmul_nt(g.t(), a.t()) if ctx.needs_input_grad[1] else None
    db = _bias_grad(g) if ctx.needs_input_grad[3] else None
    dres = grad if ctx.needs_input_grad[4] else None
    return da, dw, None, db, dres, None, None, None


gemm.register_autograd(_gemm_backward, setup_context=_gemm_setup)


@torch.library.custom_op("siglip2_b200::gemm_rowsums", mutates_args=(), device_types="cuda")
def gemm_rowsums(a: Tensor, w: Tensor, epilogue: int, bias: Optional[Tensor], res: Optional[Tensor],
                 c1: Optional[Tensor], c2: Optional[Tensor], eps: float, rs_in: Optional[Tensor],
                 produce_rowsums: bool) -> tuple[Tensor, Tensor]:
    """``siglip2_gemm_rowsums``: returns ``(out [M, N], rs)`` where ``rs`` is
    the ``[M, slots(N), 2]`` row sums of ``out`` when ``produce_rowsums``
    (the epilogue must be a row-sum one), else an empty tensor."""
    M, N = a.shape[0], w.shape[0]
    rs = (torch.empty((M, _slots(a.dtype, N), 2), dtype=torch.float32, device=a.device) if produce_rowsums
          else torch.empty(0, dtype=torch.float32, device=a.device))
    out = ops.gemm_rowsums(a, w, epilogue, bias, res, c1, c2, eps, rs_in, rs if produce_rowsums else None)
    return out, rs


@gemm_rowsums.register_fake
def _(a, w, epilogue, bias, res, c1, c2, eps, rs_in, produce_rowsums):
    M, N = a.shape[0], w.shape[0]
    rs_shape = (M, _slots(a.dtype, N), 2) if produce_rowsums else (0,)
    return a.new_empty((M, N)), a.new_empty(rs_shape, dtype=torch.float32)


@torch.library.custom_op("siglip2_b200::rowsums", mutates_args=(), device_types="cuda")
def rowsums(x: Tensor) -> Tensor:
    """``siglip2_rowsums``: ``[M, slots(K), 2]`` row sums of ``x [M, K]``."""
    return ops.rowsums(x)


@rowsums.register_fake
def _(x):
    return x.new_empty((x.shape[0], _slots(x.dtype, x.shape[1]), 2), dtype=torch.float32)


# --------------------------------------------------------------------------- attention
@torch.library.custom_op("siglip2_b200::fmha_varlen", mutates_args=(), device_types="cuda")
def fmha_varlen(qkv: Tensor, cu_seqlens: Tensor, tiles: Tensor, heads: int, head_dim: int,
                lengths: list[int], dropout_p: float = 0.0, seed: int = 0) -> Tensor:
    """``siglip2_fmha_varlen``: qkv [N, 3*heads*head_dim] -> [N, heads*head_dim].
    ``lengths``: the sequence lengths on the host (``cu_seqlens`` is their
    device prefix sum), read only by the backward.  ``dropout_p > 0``: the
    train-mode attention-output dropout (``model.py:166-169``) with the
    counter-based mask of ``seed``, applied as the output is stored."""
    return ops.fmha_varlen(qkv, cu_seqlens, tiles, heads, head_dim, dropout_p=dropout_p, seed=seed)


@fmha_varlen.register_fake
def _(qkv, cu_seqlens, tiles, heads, head_dim, lengths, dropout_p=0.0, seed=0):
    return qkv.new_empty((qkv.shape[0], heads * head_dim))


def _fmha_setup(ctx, inputs, output):
    qkv, cu_seqlens, tiles, heads, head_dim, lengths, dropout_p, seed = inputs
    ctx.heads, ctx.head_dim, ctx.lengths = heads, head_dim, list(lengths)
    ctx.dropout_p, ctx.seed = dropout_p, seed
    ctx.save_for_backward(qkv)


def _fmha_backward(ctx, grad):
    """Stop-gap attention backward: the incoming gradient goes through the
    forward's dropout mask (regenerated from the seed by ``siglip2_dropout``),
    then the sequences are recomputed with torch's
    scaled_dot_product_attention and differentiated there (softmax(q k^T /
    sqrt(hd)) v, the forward's definition), one batched call per distinct
    sequence length."""
    (qkv,) = ctx.saved_tensors
    H, hd = ctx.heads, ctx.head_dim
    N = qkv.shape[0]
    x = qkv.detach().view(N, 3, H, hd)
    if ctx.dropout_p > 0:
        grad = dropout(grad, ctx.dropout_p, ctx.seed)
    g = grad.reshape(N, H, hd)
    # sequences of equal length go through one batched call (a batch of full
    # 16x16 grids is one call per layer)
    starts = np.concatenate([[0], np.cumsum(ctx.lengths)[:-1]]).astype(np.int64)
    by_len: dict = {}
    for i, n in enumerate(ctx.lengths):
        by_len.setdefault(int(n), []).append(i)
    dqkv = torch.empty((N, 3, H, hd), dtype=qkv.dtype, device=qkv.device)
    for n, seqs in by_len.items():
        rows = (torch.from_numpy(starts[seqs])[:, None] + torch.arange(n)[None, :]).reshape(-1).to(qkv.device)
        xs = x.index_select(0, rows).view(len(seqs), n, 3, H, hd)
        with torch.enable_grad():
            q, k, v = (xs[:, :, i].transpose(1, 2).requires_grad_(True) for i in range(3))  # [G, H, n, hd]
            o = torch.nn.functional.scaled_dot_product_attention(q, k, v, scale=hd ** -0.5)
            gs = g.index_select(0, rows).view(len(seqs), n, H, hd).transpose(1, 2)
            dq, dk, dv = torch.autograd.grad(o, (q, k, v), gs)
        dqkv.index_copy_(0, rows, torch.stack([t.transpose(1, 2) for t in (dq, dk, dv)], 2).reshape(-1, 3, H, hd))
    return dqkv.reshape(N, 3 * H * hd), None, None, None, None, None, None, None


fmha_varlen.register_autograd(_fmha_backward, setup_context=_fmha_setup)


@torch.library.custom_op("siglip2_b200::fmha_varlen_train", mutates_args=(), device_types="cuda")
def fmha_varlen_train(qkv: Tensor, cu_seqlens: Tensor, tiles: Tensor, heads: int, head_dim: int,
                      dropout_p: float = 0.0, seed: int = 0) -> tuple[Tensor, Tensor]:
    """``siglip2_fmha_varlen_train``: ``(out, lse)``, the attention output
    (train-mode output dropout when ``dropout_p > 0``) and the base-2
    log-sum-exp of every row, kept for the tensor-core backward."""
    return ops.fmha_varlen_train(qkv, cu_seqlens, tiles, heads, head_dim, dropout_p, seed)


@fmha_varlen_train.register_fake
def _(qkv, cu_seqlens, tiles, heads, head_dim, dropout_p=0.0, seed=0):
    N = qkv.shape[0]
    return qkv.new_empty((N, heads * head_dim)), qkv.new_empty((N, heads), dtype=torch.float32)


def _fmha_train_setup(ctx, inputs, output):
    qkv, cu_seqlens, tiles, heads, head_dim, dropout_p, seed = inputs
    out, lse = output
    ctx.heads, ctx.head_dim, ctx.dropout_p, ctx.seed = heads, head_dim, dropout_p, seed
    ctx.save_for_backward(qkv, cu_seqlens, tiles, out, lse)


@torch.library.custom_op("siglip2_b200::fmha_varlen_backward", mutates_args=(), device_types="cuda")
def fmha_varlen_backward(qkv: Tensor, out: Tensor, grad: Tensor, lse: Tensor, cu_seqlens: Tensor, tiles: Tensor,
                         heads: int, head_dim: int, dropout_p: float, seed: int) -> Tensor:
    """``siglip2_fmha_bwd_dsum`` + ``siglip2_fmha_varlen_backward``: dqkv of the
    training attention (the gradient through the forward's dropout mask)."""
    return ops.fmha_varlen_backward(qkv, out, grad, lse, cu_seqlens, tiles, heads, head_dim, dropout_p, seed)


@fmha_varlen_backward.register_fake
def _(qkv, out, grad, lse, cu_seqlens, tiles, heads, head_dim, dropout_p, seed):
    return torch.empty_like(qkv)


@torch.library.custom_op("siglip2_b200::dropout", mutates_args=(), device_types="cuda")
def dropout(x: Tensor, p: float, seed: int) -> Tensor:
    """``siglip2_dropout``: the train-mode mask of ``seed`` applied to ``x``."""
    return ops.dropout(x.contiguous(), p, seed)


@dropout.register_fake
def _(x, p, seed):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


def _fmha_train_backward(ctx, grad_out, grad_lse):
    """The attention backward on the tensor cores (the log-sum-exp output
    carries no gradient)."""
    qkv, cu_seqlens, tiles, out, lse = ctx.saved_tensors
    dqkv = fmha_varlen_backward(qkv, out, grad_out, lse, cu_seqlens, tiles, ctx.heads, ctx.head_dim,
                                ctx.dropout_p, ctx.seed)
    return dqkv, None, None, None, None, None, None


fmha_varlen_train.register_autograd(_fmha_train_backward, setup_context=_fmha_train_setup)


def attention_for_training(qkv: Tensor, cu_seqlens: Tensor, tiles: Tensor, heads: int, head_dim: int,
                           lengths: list[int], dropout_p: float = 0.0, seed: int = 0) -> Tensor:
    """Attention with a backward: the tensor-core forward + backward pair
    (bf16 / f16, head_dim 64, 72 or 96), else ``fmha_varlen`` with the
    recompute-in-torch backward."""
    if qkv.dtype in (torch.bfloat16, torch.float16) and head_dim in (64, 72, 96):
        return fmha_varlen_train(qkv, cu_seqlens, tiles, heads, head_dim, dropout_p, seed)[0]
    return fmha_varlen(qkv, cu_seqlens, tiles, heads, head_dim, lengths, dropout_p, seed)


# --------------------------------------------------------------------------- row ops
@torch.library.custom_op("siglip2_b200::layernorm", mutates_args=(), device_types="cuda")
def layernorm(x: Tensor, weight: Tensor, bias: Tensor, eps: float) -> Tensor:
    """``siglip2_layernorm`` over the last dimension; weight/bias float32."""
    return ops.layernorm(x.contiguous(), weight, bias, eps)


@layernorm.register_fake
def _(x, weight, bias, eps):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


def _layernorm_setup(ctx, inputs, output):
    x, weight, bias, eps = inputs
    ctx.eps = eps
    ctx.save_for_backward(x, weight)


@torch.library.custom_op("siglip2_b200::layernorm_backward", mutates_args=(), device_types="cuda")
def layernorm_backward(x: Tensor, dy: Tensor, weight: Tensor, eps: float) -> tuple[Tensor, Tensor, Tensor]:
    """``siglip2_layernorm_backward``: ``(dx, dweight, dbias)``."""
    return ops.layernorm_backward(x, dy, weight, eps)


@layernorm_backward.register_fake
def _(x, dy, weight, eps):
    D = x.shape[-1]
    return (torch.empty_like(x, memory_format=torch.contiguous_format), weight.new_empty((D,), dtype=torch.float32),
            weight.new_empty((D,), dtype=torch.float32))


def _layernorm_backward(ctx, grad):
    """LayerNorm backward on the library's kernels (statistics recomputed
    from x): dx = rstd (g - mean(g) - xh mean(g xh)), g = dy * w; dw = sum
    dy xh, db = sum dy."""
    x, weight = ctx.saved_tensors
    if x.shape[-1] % 8 == 0:
        dx, dw, db = layernorm_backward(x, grad, weight, ctx.eps)
        return (dx if ctx.needs_input_grad[0] else None, dw.to(weight.dtype) if ctx.needs_input_grad[1] else None,
                db.to(weight.dtype) if ctx.needs_input_grad[2] else None, None)
    xf = x.float()
    mu = xf.mean(-1, keepdim=True)
    rstd = torch.rsqrt(((xf - mu) ** 2).mean(-1, keepdim=True) + ctx.eps)
    xh = (xf - mu) * rstd
    dy = grad.float()
    gy = dy * weight.float()
    dx = rstd * (gy - gy.mean(-1, keepdim=True) - xh * (gy * xh).mean(-1, keepdim=True))
    rows = dy.reshape(-1, dy.shape[-1])
    dw = (rows * xh.reshape(rows.shape)).sum(0) if ctx.needs_input_grad[1] else None
    db = rows.sum(0) if ctx.needs_input_grad[2] else None
    return dx.to(x.dtype) if ctx.needs_input_grad[0] else None, dw, db, None


layernorm.register_autograd(_layernorm_backward, setup_context=_layernorm_setup)


@torch.library.custom_op("siglip2_b200::token_image", mutates_args=(), device_types="cuda")
def token_image(cu_seqlens: Tensor, n_tokens: int) -> Tensor:
    """``siglip2_token_image``: int32 image index of each packed token."""
    return ops.token_image(cu_seqlens, n_tokens)


@token_image.register_fake
def _(cu_seqlens, n_tokens):
    return cu_seqlens.new_empty((n_tokens,), dtype=torch.int32)


@torch.library.custom_op("siglip2_b200::patch_embed", mutates_args=(), device_types="cuda")
def patch_embed(patches: Tensor, w: Tensor, bias: Tensor, table: Tensor, hw: Tensor, cu_seqlens: Tensor,
                tok_img: Tensor, grids: list[int]) -> Tensor:
    """``siglip2_patch_embed``: ``patches @ w.T + bias + resize(table)`` [N, D].
    ``grids``: the (h, w) pairs on the host (``hw`` on the device), read only
    by the backward."""
    return ops.patch_embed(patches, w, bias, table, hw, cu_seqlens, tok_img)


@patch_embed.register_fake
def _(patches, w, bias, table, hw, cu_seqlens, tok_img, grids):
    return patches.new_empty((patches.shape[0], w.shape[0]))


def _patch_embed_setup(ctx, inputs, output):
    patches, w, bias, table, hw, cu_seqlens, tok_img, grids = inputs
    ctx.grids = list(grids)
    ctx.save_for_backward(patches, w, table)


def _patch_embed_backward(ctx, grad):
    """Stop-gap backward: patch and weight gradients on the library GEMM; the
    position table's gradient is the adjoint of the per-image antialiased
    bilinear resize, taken through torch's interpolate (one image at a time)."""
    patches, w, table = ctx.saved_tensors
    if _tensor_core_backward(patches, w, grad):
        d_patches = _dgrad(grad, w) if ctx.needs_input_grad[0] else None
        dw = _wgrad(grad, patches) if ctx.needs_input_grad[1] else None
    else:
        d_patches = _matmul_nt(grad, w.t()) if ctx.needs_input_grad[0] else None
        dw = _matmul_nt(grad.t(), patches.t()) if ctx.needs_input_grad[1] else None
    db = _bias_grad(grad) if ctx.needs_input_grad[2] else None
    dtable = None
    if ctx.needs_input_grad[3]:
        G2, D = table.shape
        G = int(round(G2 ** 0.5))
        grids = ctx.grids
        with torch.enable_grad():
            t = table.detach().float().reshape(G, G, D).permute(2, 0, 1)[None].requires_grad_(True)
            outs, s = [], 0
            for i in range(0, len(grids), 2):
                h, wd = grids[i], grids[i + 1]
                outs.append(torch.nn.functional.interpolate(t, size=(h, wd), mode="bilinear", align_corners=False,
                                                            antialias=True).reshape(D, h * wd))
            r = torch.cat(outs, 1)  # [D, N]
            (dt,) = torch.autograd.grad(r, (t,), grad.float().t())
        dtable = dt[0].permute(1, 2, 0).reshape(G2, D).to(table.dtype)
    return d_patches, dw, db, dtable, None, None, None, None


patch_embed.register_autograd(_patch_embed_backward, setup_context=_patch_embed_setup)


# --------------------------------------------------------------------------- whole tower
_STRUCTS: dict = {}


def _structs_for(dims, eps, weights):
    """ctypes structs over ``weights``, cached by their addresses (a few
    entries): rebuilding them costs more than the launch sequence."""
    from .model import weight_structs
    key = (tuple(dims), float(eps), tuple(t.data_ptr() for t in weights))
    hit = _STRUCTS.get(key)
    if hit is None:
        if len(_STRUCTS) >= 4:
            _STRUCTS.pop(next(iter(_STRUCTS)))
        hit = _STRUCTS[key] = weight_structs(dims, eps, weights)
    return hit


@torch.library.custom_op("siglip2_b200::vision_tower", mutates_args=(), device_types="cuda")
def vision_tower(patches: Tensor, hw: Tensor, max_patches: int, want_pooled: bool, weights: list[Tensor],
                 dims: list[int], eps: float) -> tuple[Tensor, Tensor]:
    """``siglip2_forward``.  ``patches`` packed [N, C] (max_patches = 0) or
    padded [B, max_patches, C]; ``hw`` the [B, 2] grids (read on the host);
    ``weights`` the packed tensors in the flat order of
    ``model.LAYER_FIELDS`` / ``TOWER_FIELDS`` / ``HEAD_FIELDS``; ``dims`` the
    integer fields of ``siglip2_config`` (``model.DIM_FIELDS``).  Returns
    ``(last_hidden_state, pooler_output)``; the second is empty when
    ``want_pooled`` is false."""
    from .model import run_tower
    cfg, w, _ = _structs_for(dims, eps, weights)
    hw_np = np.ascontiguousarray(hw.detach().to("cpu", torch.int32).numpy()).reshape(-1, 2)
    last, pooled = run_tower(cfg, w, patches.device, _TORCH_DT[int(dims[7])], patches, hw_np, max_patches,
                             want_pooled)
    if pooled is None:
        pooled = last.new_empty((0, int(dims[0])))
    return last, pooled


@vision_tower.register_fake
def _(patches, hw, max_patches, want_pooled, weights, dims, eps):
    D, dt = int(dims[0]), _TORCH_DT[int(dims[7])]
    B = hw.shape[0]
    shape = (patches.shape[0], D) if max_patches == 0 else (B, max_patches, D)
    last = patches.new_empty(shape, dtype=dt)
    pooled = patches.new_empty((B, D) if want_pooled else (0, D), dtype=dt)
    return last, pooled
