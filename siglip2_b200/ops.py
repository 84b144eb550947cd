"""Torch-facing wrappers over the C ABI (device pointers + current stream).

Each wrapper validates dtype/device/contiguity, allocates outputs with the
caching allocator and calls the library; nothing here computes on the CPU.
"""
from __future__ import annotations

import torch

from . import _lib as L

_DT = {torch.float32: L.DTYPE_F32, torch.bfloat16: L.DTYPE_BF16, torch.float16: L.DTYPE_F16}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}") from None


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("siglip2_b200 kernels take CUDA tensors only")


def gemm(a: torch.Tensor, w: torch.Tensor, epilogue: int, bias=None, res=None, c1=None, c2=None,
         eps: float = 1e-6, out: torch.Tensor | None = None) -> torch.Tensor:
    """``out = epilogue(a @ w.T)`` on the tensor cores (``siglip2_gemm``)."""
    _need_cuda(a, w, bias, res, c1, c2, out)
    assert a.dim() == 2 and w.dim() == 2 and a.shape[1] == w.shape[1]
    assert a.stride(1) == 1 and w.stride(1) == 1
    M, K = a.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=a.dtype, device=a.device)
    L.call("siglip2_gemm", dtype_code(a.dtype), epilogue, a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0),
           out.data_ptr(), out.stride(0), M, N, K, _ptr(bias), _ptr(res), res.stride(0) if res is not None else 0,
           _ptr(c1), _ptr(c2), float(eps), _stream(a.device))
    return out


def gemm_t(a: torch.Tensor, b: torch.Tensor, trans_a: bool, trans_b: bool, epilogue: int = L.EPI_BIAS,
           bias=None, res=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """``siglip2_gemm_t``: ``epilogue(op(a) @ op(b).T)`` with ``op(a) = a`` ([M, K])
    or ``a.T`` (``trans_a``: ``a`` is [K, M]) and ``op(b) = b`` ([N, K]) or
    ``b.T`` (``trans_b``: ``b`` is [K, N]).  Row-major operands with unit
    column stride; the transposed ones are read as MN-major tiles, no copy."""
    _need_cuda(a, b, bias, res, out)
    assert a.dim() == 2 and b.dim() == 2 and a.stride(1) == 1 and b.stride(1) == 1
    M, K = (a.shape[1], a.shape[0]) if trans_a else a.shape
    N, Kb = (b.shape[1], b.shape[0]) if trans_b else b.shape
    assert K == Kb, (a.shape, b.shape, trans_a, trans_b)
    if out is None:
        out = torch.empty((M, N), dtype=a.dtype, device=a.device)
    L.call("siglip2_gemm_t", dtype_code(a.dtype), epilogue, int(trans_a), int(trans_b), a.data_ptr(), a.stride(0),
           b.data_ptr(), b.stride(0), out.data_ptr(), out.stride(0), M, N, K, _ptr(bias), _ptr(res),
           res.stride(0) if res is not None else 0, _stream(a.device))
    return out


def gemm_t_splitk(a: torch.Tensor, b: torch.Tensor, trans_a: bool, bias=None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """``siglip2_gemm_t_ws``: ``op(a) @ b`` (+ bias) as ``gemm_t`` with
    ``trans_b`` (``b`` is [K, N]), K split over a workspace from the caching
    allocator when the output has too few tiles to fill the SMs (the weight
    gradients)."""
    _need_cuda(a, b, bias, out)
    assert a.dim() == 2 and b.dim() == 2 and a.stride(1) == 1 and b.stride(1) == 1
    M, K = (a.shape[1], a.shape[0]) if trans_a else a.shape
    Kb, N = b.shape
    assert K == Kb, (a.shape, b.shape, trans_a)
    if out is None:
        out = torch.empty((M, N), dtype=a.dtype, device=a.device)
    nbytes = L.load().siglip2_gemm_t_workspace_size(L.EPI_BIAS, int(trans_a), 1, M, N, K)
    ws = torch.empty(max(nbytes, 16) // 4, dtype=torch.float32, device=a.device) if nbytes else None
    L.call("siglip2_gemm_t_ws", dtype_code(a.dtype), L.EPI_BIAS, int(trans_a), 1, a.data_ptr(), a.stride(0),
           b.data_ptr(), b.stride(0), out.data_ptr(), out.stride(0), M, N, K, _ptr(bias), _ptr(ws), nbytes,
           _stream(a.device))
    return out


def colsum(x: torch.Tensor, chunk_rows: int = 256) -> torch.Tensor:
    """``siglip2_colsum_partial`` + an in-order sum of the chunk partials:
    the fp32 column sums of ``x`` [rows, cols] (a bias gradient)."""
    _need_cuda(x)
    assert x.dim() == 2 and x.stride(1) == 1
    rows, cols = x.shape
    chunks = max(1, -(-rows // chunk_rows))
    part = torch.empty((chunks, cols), dtype=torch.float32, device=x.device)
    if rows == 0:
        return torch.zeros(cols, dtype=torch.float32, device=x.device)
    L.call("siglip2_colsum_partial", dtype_code(x.dtype), x.data_ptr(), x.stride(0), rows, cols, chunk_rows,
           part.data_ptr(), _stream(x.device))
    return part.sum(0)


def quantize_e4m3(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``siglip2_quantize_e4m3``: per-row e4m3 codes of ``x`` [rows, cols]
    (fp32 / bf16 / f16) as a ``torch.float8_e4m3fn`` tensor and the fp32
    per-row scales (``x ~ codes * scale[:, None]``)."""
    _need_cuda(x)
    assert x.dim() == 2 and x.stride(1) == 1
    rows, cols = x.shape
    q = torch.empty((rows, cols), dtype=torch.float8_e4m3fn, device=x.device)
    scale = torch.empty(rows, dtype=torch.float32, device=x.device)
    L.call("siglip2_quantize_e4m3", dtype_code(x.dtype), x.data_ptr(), x.stride(0), rows, cols, q.data_ptr(),
           q.stride(0), scale.data_ptr(), _stream(x.device))
    return q, scale


def gemm_e4m3(a: torch.Tensor, a_scale: torch.Tensor, w: torch.Tensor, w_scale: torch.Tensor, epilogue: int,
              bias: torch.Tensor, res=None, out_dtype=torch.bfloat16, out: torch.Tensor | None = None) -> torch.Tensor:
    """``siglip2_gemm_e4m3``: ``epilogue(a_scale[:, None] * w_scale[None, :] *
    (a @ w.T))`` with ``a`` [M, K] and ``w`` [N, K] e4m3 codes (from
    ``quantize_e4m3``), fp32 accumulation, ``out_dtype`` output."""
    _need_cuda(a, a_scale, w, w_scale, bias, res, out)
    assert a.dtype == torch.float8_e4m3fn and w.dtype == torch.float8_e4m3fn
    assert a.dim() == 2 and w.dim() == 2 and a.shape[1] == w.shape[1] and a.stride(1) == 1 and w.stride(1) == 1
    M, K = a.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    L.call("siglip2_gemm_e4m3", dtype_code(out.dtype), epilogue, a.data_ptr(), a.stride(0), a_scale.data_ptr(),
           w.data_ptr(), w.stride(0), w_scale.data_ptr(), out.data_ptr(), out.stride(0), M, N, K, bias.data_ptr(),
           _ptr(res), res.stride(0) if res is not None else 0, _stream(a.device))
    return out


def fold_layernorm(w: torch.Tensor, b: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, dtype):
    """LayerNorm(gamma, beta) followed by Linear(w, b) as a GEMM on the raw
    input: returns ``(w*gamma in dtype, c1, c2)`` with ``c1 = rowsum(w*gamma)``
    (of the rounded matrix) and ``c2 = b + w @ beta`` (fp32)."""
    wf = w.float()
    wg = (wf * gamma.float()[None, :]).to(dtype)
    c1 = wg.float().sum(1)
    c2 = (b.float() if b is not None else torch.zeros(w.shape[0], device=w.device)) + wf @ beta.float()
    return wg.contiguous(), c1.contiguous(), c2.contiguous()


def layernorm(x: torch.Tensor, gamma, beta, eps: float, cu_seqlens=None, batch: int = 0, max_patches: int = 0):
    """Packed ``LN(x)`` or, with ``cu_seqlens``, the padded ``[B*P, D]`` scatter."""
    _need_cuda(x, gamma, beta)
    D = x.shape[-1]
    if cu_seqlens is None:
        rows = x.numel() // D
        y = torch.empty_like(x)
    else:
        rows = batch * max_patches
        y = torch.empty((batch, max_patches, D), dtype=x.dtype, device=x.device)
    L.call("siglip2_layernorm", dtype_code(x.dtype), x.data_ptr(), y.data_ptr(), gamma.data_ptr(), beta.data_ptr(),
           rows, D, float(eps), _ptr(cu_seqlens), max_patches, _stream(x.device))
    return y


def layernorm_backward(x: torch.Tensor, dy: torch.Tensor, gamma: torch.Tensor, eps: float, chunk_rows: int = 128):
    """``siglip2_layernorm_backward``: ``(dx, dgamma, dbeta)`` of LayerNorm over
    the last dimension (dgamma / dbeta fp32, summed over row chunks in order)."""
    _need_cuda(x, dy, gamma)
    D = x.shape[-1]
    x2, dy2 = x.reshape(-1, D).contiguous(), dy.reshape(-1, D).contiguous().to(x.dtype)
    rows = x2.shape[0]
    chunks = max(1, -(-rows // chunk_rows))
    dx = torch.empty_like(x2)
    stats = torch.empty((rows, 2), dtype=torch.float32, device=x.device)
    dg = torch.empty((chunks, D), dtype=torch.float32, device=x.device)
    db = torch.empty((chunks, D), dtype=torch.float32, device=x.device)
    L.call("siglip2_layernorm_backward", dtype_code(x.dtype), x2.data_ptr(), dy2.data_ptr(),
           gamma.float().contiguous().data_ptr(), rows, D, float(eps), dx.data_ptr(), stats.data_ptr(),
           dg.data_ptr(), db.data_ptr(), chunk_rows, _stream(x.device))
    return dx.view(x.shape), dg.sum(0), db.sum(0)


def token_image(cu_seqlens: torch.Tensor, n_tokens: int) -> torch.Tensor:
    out = torch.empty(n_tokens, dtype=torch.int32, device=cu_seqlens.device)
    L.call("siglip2_token_image", cu_seqlens.data_ptr(), cu_seqlens.numel() - 1, n_tokens, out.data_ptr(),
           _stream(cu_seqlens.device))
    return out


def posemb(table_f32: torch.Tensor, hw: torch.Tensor, cu_seqlens: torch.Tensor, tok_img: torch.Tensor, n_tokens: int,
           dtype) -> torch.Tensor:
    G = int(round(table_f32.shape[0] ** 0.5))
    D = table_f32.shape[1]
    out = torch.empty((n_tokens, D), dtype=dtype, device=table_f32.device)
    L.call("siglip2_posemb", dtype_code(dtype), table_f32.data_ptr(), G, D, tok_img.data_ptr(), hw.data_ptr(),
           cu_seqlens.data_ptr(), n_tokens, out.data_ptr(), _stream(table_f32.device))
    return out


def padded_head_dim(head_dim: int) -> int:
    return int(L.load().siglip2_padded_head_dim(head_dim))


def attention_tiles(lens) -> torch.Tensor:
    """(image, query-tile) int32 pairs for every 128-row query tile, longest
    images first (better tail behaviour)."""
    order = sorted(range(len(lens)), key=lambda b: -int(lens[b]))
    t = [(b, q) for b in order for q in range((int(lens[b]) + 127) // 128)]
    return torch.tensor(t, dtype=torch.int32).reshape(-1, 2)


def fmha_varlen(qkv: torch.Tensor, cu_seqlens: torch.Tensor, tiles: torch.Tensor, heads: int, head_dim: int,
                out: torch.Tensor | None = None, dropout_p: float = 0.0, seed: int = 0,
                offset: int = 0) -> torch.Tensor:
    """Per-sequence attention (``siglip2_fmha_varlen``); with ``dropout_p > 0``
    the attention-output dropout of train mode is applied as the output is
    stored (``siglip2_fmha_varlen_dropout``, mask from ``seed``/``offset``)."""
    _need_cuda(qkv, cu_seqlens, tiles)
    N = qkv.shape[0]
    if out is None:
        out = torch.empty((N, heads * head_dim), dtype=qkv.dtype, device=qkv.device)
    if dropout_p > 0:
        L.call("siglip2_fmha_varlen_dropout", dtype_code(qkv.dtype), qkv.data_ptr(), N, cu_seqlens.data_ptr(),
               tiles.data_ptr(), tiles.shape[0], heads, head_dim, out.data_ptr(), out.stride(0), float(dropout_p),
               int(seed) & (2 ** 64 - 1), int(offset) & (2 ** 64 - 1), _stream(qkv.device))
    else:
        L.call("siglip2_fmha_varlen", dtype_code(qkv.dtype), qkv.data_ptr(), N, cu_seqlens.data_ptr(),
               tiles.data_ptr(), tiles.shape[0], heads, head_dim, out.data_ptr(), out.stride(0), _stream(qkv.device))
    return out


def fmha_varlen_train(qkv: torch.Tensor, cu_seqlens: torch.Tensor, tiles: torch.Tensor, heads: int, head_dim: int,
                      dropout_p: float = 0.0, seed: int = 0, offset: int = 0):
    """``siglip2_fmha_varlen_train``: ``(out [N, heads*head_dim], lse [N, heads])``,
    the attention output (train-mode dropout when ``dropout_p > 0``) and the
    base-2 log-sum-exp of each row the backward recomputes P from."""
    _need_cuda(qkv, cu_seqlens, tiles)
    N = qkv.shape[0]
    out = torch.empty((N, heads * head_dim), dtype=qkv.dtype, device=qkv.device)
    lse = torch.empty((N, heads), dtype=torch.float32, device=qkv.device)
    L.call("siglip2_fmha_varlen_train", dtype_code(qkv.dtype), qkv.data_ptr(), N, cu_seqlens.data_ptr(),
           tiles.data_ptr(), tiles.shape[0], heads, head_dim, out.data_ptr(), out.stride(0), lse.data_ptr(),
           float(dropout_p), int(seed) & (2 ** 64 - 1), int(offset) & (2 ** 64 - 1), _stream(qkv.device))
    return out, lse


def fmha_varlen_backward(qkv: torch.Tensor, out: torch.Tensor, grad: torch.Tensor, lse: torch.Tensor,
                         cu_seqlens: torch.Tensor, tiles: torch.Tensor, heads: int, head_dim: int,
                         dropout_p: float = 0.0, seed: int = 0, offset: int = 0) -> torch.Tensor:
    """Gradient of ``fmha_varlen_train`` w.r.t. ``qkv``: the row term
    D = rowsum(grad . out) (``siglip2_fmha_bwd_dsum``), the incoming gradient
    through the forward's dropout mask, then ``siglip2_fmha_varlen_backward``."""
    _need_cuda(qkv, out, grad, lse)
    N = qkv.shape[0]
    grad = grad.contiguous()
    dsum = torch.empty((N, heads), dtype=torch.float32, device=qkv.device)
    L.call("siglip2_fmha_bwd_dsum", dtype_code(grad.dtype), grad.data_ptr(), out.data_ptr(), grad.stride(0), N,
           heads, head_dim, dsum.data_ptr(), _stream(qkv.device))
    g = dropout(grad, dropout_p, seed, offset) if dropout_p > 0 else grad
    dqkv = torch.empty_like(qkv)
    L.call("siglip2_fmha_varlen_backward", dtype_code(qkv.dtype), qkv.data_ptr(), g.data_ptr(), g.stride(0), N,
           cu_seqlens.data_ptr(), tiles.data_ptr(), tiles.shape[0], heads, head_dim, lse.data_ptr(),
           dsum.data_ptr(), dqkv.data_ptr(), _stream(qkv.device))
    return dqkv


def dropout(x: torch.Tensor, p: float, seed: int, offset: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """``siglip2_dropout``: ``x * keep / (1 - p)`` with the counter-based mask of
    the attention kernel's train mode (same ``seed``/``offset``, element index
    ``row * width + col`` of the ``[rows, width]`` matrix)."""
    _need_cuda(x)
    assert x.dim() == 2 and x.stride(1) == 1
    if out is None:
        out = torch.empty_like(x)
    L.call("siglip2_dropout", dtype_code(x.dtype), x.data_ptr(), x.stride(0), x.shape[0], x.shape[1], float(p),
           int(seed) & (2 ** 64 - 1), int(offset) & (2 ** 64 - 1), out.data_ptr(), out.stride(0), _stream(x.device))
    return out


def head_pool(x: torch.Tensor, u: torch.Tensor, cu_seqlens: torch.Tensor, n_tokens: int, max_patches: int = 0,
              scores: torch.Tensor | None = None) -> torch.Tensor:
    """``pooled[b, h] = sum_j softmax_j(x_j . u_h) x_j`` (``siglip2_head_pool``)."""
    _need_cuda(x, u, cu_seqlens)
    H, D = u.shape
    B = cu_seqlens.numel() - 1
    if scores is None:
        scores = torch.empty(n_tokens * H, dtype=torch.float32, device=x.device)
    pooled = torch.empty((B, H, D), dtype=x.dtype, device=x.device)
    L.call("siglip2_head_pool", dtype_code(x.dtype), x.data_ptr(), D, H, cu_seqlens.data_ptr(), B, max_patches,
           u.data_ptr(), scores.data_ptr(), pooled.data_ptr(), _stream(x.device))
    return pooled


def rowsum_slots(dtype: torch.dtype, width: int) -> int:
    """``siglip2_rowsum_slots``: column-block slots per row of the row-sum
    buffers for rows of ``width`` columns."""
    return L.check_value(L.load().siglip2_rowsum_slots(dtype_code(dtype), width))


def rowsums_reference(x: torch.Tensor) -> torch.Tensor:
    """Slot statistics of ``x`` in the layout the LayerNorm-folded GEMMs read
    (``[M, S, 2]`` float32: per column block the mean and the centred sum of
    squares), computed with torch: for tests and callers whose rows were not
    produced by a row-sum GEMM."""
    M, K = x.shape
    S = rowsum_slots(x.dtype, K)
    blk = L.check_value(L.load().siglip2_rowsum_block(dtype_code(x.dtype), K))
    xf = x.float()
    out = torch.zeros(M, S, 2, dtype=torch.float32, device=x.device)
    for j in range(S):
        part = xf[:, j * blk:(j + 1) * blk]
        mean = part.mean(1)
        out[:, j, 0] = mean
        out[:, j, 1] = ((part - mean[:, None]) ** 2).sum(1)
    return out


def slot_stats_merge(rs: torch.Tensor, width: int, blk: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """Row mean and biased variance from ``[M, S, 2]`` slot statistics (the
    merge the LayerNorm-folded GEMMs do), for tests."""
    n = torch.tensor([min(blk, width - j * blk) for j in range(rs.shape[1])], dtype=torch.float32,
                     device=rs.device)
    mean = (rs[..., 0] * n).sum(1) / width
    m2 = (rs[..., 1] + n * (rs[..., 0] - mean[:, None]) ** 2).sum(1)
    return mean, m2 / width


def rowsums(x: torch.Tensor) -> torch.Tensor:
    """``siglip2_rowsums``: slot statistics of ``x [M, K]`` in the layout the
    LayerNorm-folded GEMMs read (``[M, rowsum_slots(dtype, K), 2]`` float32)."""
    _need_cuda(x)
    assert x.dim() == 2 and x.stride(1) == 1
    M, K = x.shape
    out = torch.empty((M, rowsum_slots(x.dtype, K), 2), dtype=torch.float32, device=x.device)
    L.call("siglip2_rowsums", dtype_code(x.dtype), x.data_ptr(), x.stride(0), M, K, out.data_ptr(),
           _stream(x.device))
    return out


def gemm_rowsums(a: torch.Tensor, w: torch.Tensor, epilogue: int, bias=None, res=None, c1=None, c2=None,
                 eps: float = 1e-6, rs_in=None, rs_acc=None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """``siglip2_gemm_rowsums``: row-sum LayerNorm epilogues.  ``rs_in`` is
    ``[M, rowsum_slots(dtype, K), 2]`` and ``rs_acc`` ``[M, rowsum_slots(dtype, N), 2]``
    float32 (mean, centred sum of squares) per column block."""
    _need_cuda(a, w, bias, res, c1, c2, rs_in, rs_acc, out)
    M, K = a.shape
    N = w.shape[0]
    for t, width in ((rs_in, K), (rs_acc, N)):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous()
                              or t.numel() != M * rowsum_slots(a.dtype, width) * 2):
            raise ValueError("row-sum buffer must be contiguous float32 [M, rowsum_slots(dtype, width), 2]")
    if out is None:
        out = torch.empty((M, N), dtype=a.dtype, device=a.device)
    L.call("siglip2_gemm_rowsums", dtype_code(a.dtype), epilogue, a.data_ptr(), a.stride(0), w.data_ptr(),
           w.stride(0), out.data_ptr(), out.stride(0), M, N, K, _ptr(bias), _ptr(res),
           res.stride(0) if res is not None else 0, _ptr(c1), _ptr(c2), float(eps), _ptr(rs_in), _ptr(rs_acc),
           _stream(a.device))
    return out


def patch_embed(patches: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, table_f32: torch.Tensor,
                hw: torch.Tensor, cu_seqlens: torch.Tensor, tok_img: torch.Tensor, rs_acc: torch.Tensor | None = None):
    """``siglip2_patch_embed``: patch Linear with the resized position grid
    added in the GEMM epilogue; also writes the slot statistics of its rows
    into ``rs_acc``."""
    _need_cuda(patches, w, bias, table_f32, hw, cu_seqlens, tok_img)
    N, C = patches.shape
    D = w.shape[0]
    G = int(round(table_f32.shape[0] ** 0.5))
    out = torch.empty((N, D), dtype=patches.dtype, device=patches.device)
    if rs_acc is None:
        rs_acc = torch.empty((N, rowsum_slots(patches.dtype, D), 2), dtype=torch.float32, device=patches.device)
    L.call("siglip2_patch_embed", dtype_code(patches.dtype), patches.data_ptr(), C, w.data_ptr(), bias.data_ptr(),
           table_f32.data_ptr(), G, tok_img.data_ptr(), hw.data_ptr(), cu_seqlens.data_ptr(), N, D, out.data_ptr(),
           rs_acc.data_ptr(), _stream(patches.device))
    return out
