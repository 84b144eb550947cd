"""Image-text logits after the tower (the step after ``pooler_output``).

transformers' ``Siglip2Model.forward`` (``models/siglip2/modeling_siglip2.py:964-974``)
normalises the image and text embeddings to unit L2 norm and takes
``logits_per_text = text @ image.T * exp(logit_scale) + logit_bias``,
``logits_per_image = logits_per_text.T``.  Here: two ``siglip2_l2_normalize``
launches (``exp(logit_scale)`` folded into the text rows) and one
``siglip2_gemm`` with the bias epilogue on the tensor cores.  The reference
has no text tower; the text embeddings come from the caller.
"""
from __future__ import annotations

import math

import torch

from . import _lib as L
from . import ops
from .ops import dtype_code


def l2_normalize(x: torch.Tensor, scale: float = 1.0, rows_out: int | None = None) -> torch.Tensor:
    """``scale * x / ||x||`` per row (``siglip2_l2_normalize``); with
    ``rows_out`` > rows the extra output rows are zero."""
    ops._need_cuda(x)
    assert x.dim() == 2 and x.stride(1) == 1
    R, D = x.shape
    n = rows_out or R
    y = torch.zeros((n, D), dtype=x.dtype, device=x.device) if n > R else torch.empty_like(x)
    L.call("siglip2_l2_normalize", dtype_code(x.dtype), x.data_ptr(), x.stride(0), R, D, float(scale), y.data_ptr(),
           y.stride(0), ops._stream(x.device))
    return y


def image_text_logits(image_embeds: torch.Tensor, text_embeds: torch.Tensor, logit_scale, logit_bias):
    """``(logits_per_image [B, T], logits_per_text [T, B])`` in the embeddings'
    dtype; ``logit_scale`` is the parameter before ``exp`` (as in
    transformers), ``logit_bias`` is added after scaling.  Zero-norm
    embeddings give logits equal to ``logit_bias`` (transformers gives NaN)."""
    if image_embeds.dtype != text_embeds.dtype or image_embeds.shape[1] != text_embeds.shape[1]:
        raise ValueError("image and text embeddings need the same dtype and width")
    scale = math.exp(float(logit_scale))
    bias = float(logit_bias)
    img = image_embeds.contiguous()
    txt = text_embeds.contiguous()
    B = img.shape[0]
    Bp = (B + 7) // 8 * 8  # the tensor-core GEMM wants N % 8 == 0: zero rows, cut off below
    img_n = l2_normalize(img, 1.0, rows_out=Bp)
    txt_n = l2_normalize(txt, scale)
    b = torch.full((Bp,), bias, dtype=torch.float32, device=img.device)
    per_text = ops.gemm(txt_n, img_n, L.EPI_BIAS, bias=b)[:, :B]
    return per_text.t(), per_text
