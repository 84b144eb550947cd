"""CPU restatement of the SigLIP-2 NaFlex vision-tower forward (numpy).

TEST INFRASTRUCTURE ONLY.  This module is the parity oracle: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
it, and only as the checker / the timed CPU baseline.  The product path
(``siglip2_b200``) never imports it and has no CPU fallback.

What it restates (reference = tohskai/SigLIP-2):

* ``model.py:52-120``  ``Siglip2SequenceEmbeddings``: patch Linear, then the
  16x16 position table resized per image with
  ``F.interpolate(mode="bilinear", align_corners=False, antialias=True)``
  (``model.py:100-108``), flattened row-major (h outer, w inner), added.
* ``model.py:123-176`` ``Siglip2Attention``: q/k/v Linear, per-head scaled
  dot-product attention restricted to each image's own tokens (the
  ``document_ids[q] == document_ids[kv]`` block mask of ``model.py:156-161``),
  out Linear.  Dropout is inactive (eval / ``attention_dropout=0``).
* ``model.py:179-191`` ``Siglip2MLP``: fc1, GELU-tanh (``nn.GELU("tanh")``), fc2.
* ``model.py:194-223`` pre-LN encoder layer with two residual adds.
* ``model.py:250-292`` the packed forward ``(seq_patches, token_grids)`` ->
  ``[N, D]`` after ``post_layernorm``.
* The attention-pooling head is not in the reference; it follows the
  third-party ``transformers==5.5.0``
  ``models/siglip2/modeling_siglip2.py:670-719``
  (``Siglip2MultiheadAttentionPoolingHead``: one learned probe, an
  ``nn.MultiheadAttention`` over the image's valid tokens, then
  ``h + MLP(LayerNorm(h))``) and the padded entry ``:521-555``.

Parameters are a dict keyed by the reference's ``state_dict`` names
(``embeddings.patch_embedding.weight`` ...).  Parity of this restatement with
the reference itself is pinned by ``tests/golden/*.npz`` (written by
``tests/golden/make_golden.py`` from the reference's own ``model.py`` and
from ``transformers``), checked in ``tests/test_oracle.py``.
"""
from __future__ import annotations

import math

import numpy as np

# ---------------------------------------------------------------------------
# antialiased bilinear resize (ATen upsample_bilinear2d_aa semantics)
# ---------------------------------------------------------------------------


def aa_bilinear_weights(n_in: int, n_out: int) -> np.ndarray:
    """Separable weights ``W[n_out, n_in]`` of one axis of
    ``F.interpolate(mode="bilinear", align_corners=False, antialias=True)``
    (called at ``model.py:102-108``).

    For output index ``i``: ``scale = n_in / n_out``; the triangle filter's
    support is ``scale`` when downsampling and 1 otherwise; the centre is
    ``scale * (i + 0.5)``; taps ``j`` run over
    ``[max(int(c - support + 0.5), 0), min(int(c + support + 0.5), n_in))``
    with weight ``tri((j - c + 0.5) / max(scale, 1))``, normalised to sum 1.
    Upsampling therefore reduces to plain bilinear with edge clamping.
    """
    scale = n_in / n_out
    support = scale if scale >= 1.0 else 1.0
    invscale = 1.0 / scale if scale >= 1.0 else 1.0
    w = np.zeros((n_out, n_in), dtype=np.float64)
    for i in range(n_out):
        center = scale * (i + 0.5)
        xmin = max(int(center - support + 0.5), 0)
        xmax = min(int(center + support + 0.5), n_in)
        taps = []
        for j in range(xmin, xmax):
            x = (j - center + 0.5) * invscale
            taps.append(max(0.0, 1.0 - abs(x)))
        total = sum(taps)
        if total > 0.0:
            for t, j in enumerate(range(xmin, xmax)):
                w[i, j] = taps[t] / total
    return w


def resize_position_table(table: np.ndarray, h: int, w: int) -> np.ndarray:
    """``[G*G, D]`` learned grid -> ``[h*w, D]`` for one image
    (``model.py:90-113``: reshape to ``[1, D, G, G]``, AA resize, back to
    ``[h*w, D]`` with h outer and w inner)."""
    g = int(round(math.sqrt(table.shape[0])))
    grid = table.reshape(g, g, -1).astype(np.float64)  # [gy, gx, D]
    wy = aa_bilinear_weights(g, h)  # [h, g]
    wx = aa_bilinear_weights(g, w)  # [w, g]
    out = np.einsum("ya,xb,abd->yxd", wy, wx, grid)
    return out.reshape(h * w, -1)


# ---------------------------------------------------------------------------
# elementwise pieces
# ---------------------------------------------------------------------------


def layer_norm(x: np.ndarray, gamma: np.ndarray, beta: np.ndarray, eps: float) -> np.ndarray:
    """``nn.LayerNorm`` (biased variance), ``model.py:199,201,256``."""
    mu = x.mean(axis=-1, keepdims=True)
    var = ((x - mu) ** 2).mean(axis=-1, keepdims=True)
    return (x - mu) / np.sqrt(var + eps) * gamma + beta


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """``nn.GELU(approximate="tanh")`` (``model.py:183``)."""
    return 0.5 * x * (1.0 + np.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x ** 3)))


def linear(x: np.ndarray, w: np.ndarray, b: np.ndarray | None) -> np.ndarray:
    y = x @ w.T
    if b is not None:
        y = y + b
    return y


def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    m = x.max(axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=axis, keepdims=True)


# ---------------------------------------------------------------------------
# the tower
# ---------------------------------------------------------------------------


class OracleConfig:
    """Mirror of ``Siglip2VisionConfig`` (``model.py:39-49``)."""

    def __init__(self, hidden_size=1152, intermediate_size=4304, num_hidden_layers=27,
                 num_attention_heads=16, num_channels=3, patch_size=16,
                 layer_norm_eps=1e-6, num_patches=256, **_):
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.num_hidden_layers = num_hidden_layers
        self.num_attention_heads = num_attention_heads
        self.num_channels = num_channels
        self.patch_size = patch_size
        self.layer_norm_eps = layer_norm_eps
        self.num_patches = num_patches


def _p(params, key, dt):
    return np.asarray(params[key], dtype=dt)


def qkv_weights(params, prefix, dt):
    """q/k/v weights from either key layout: ``model.py:138-141``
    (``q_proj``/``k_proj``/``v_proj``) or the fused
    ``qkv_proj = cat([q, k, v], 0)`` of ``model_optimized.py:215,223``."""
    if prefix + "qkv_proj.weight" in params:
        w = _p(params, prefix + "qkv_proj.weight", dt)
        b = _p(params, prefix + "qkv_proj.bias", dt)
        d = w.shape[1]
        return (w[:d], b[:d]), (w[d:2 * d], b[d:2 * d]), (w[2 * d:], b[2 * d:])
    return tuple((_p(params, prefix + f"{n}_proj.weight", dt), _p(params, prefix + f"{n}_proj.bias", dt))
                 for n in ("q", "k", "v"))


def embeddings(params, cfg, seq_patches, grids, dt=np.float32):
    """``model.py:68-120``: packed ``[N, C*p*p]`` -> ``[N, D]``."""
    x = linear(np.asarray(seq_patches, dtype=dt), _p(params, "embeddings.patch_embedding.weight", dt),
               _p(params, "embeddings.patch_embedding.bias", dt))
    table = _p(params, "embeddings.position_embedding.weight", np.float64)
    pos = np.concatenate([resize_position_table(table, int(h), int(w)) for h, w in grids], axis=0)
    return (x + pos.astype(dt)).astype(dt)


def attention_block(params, cfg, prefix, x, seqlens, dt):
    """``model.py:144-176`` with the document mask realised as per-image
    attention (rows of different images never attend to each other)."""
    d = cfg.hidden_size
    nh = cfg.num_attention_heads
    hd = d // nh
    (wq, bq), (wk, bk), (wv, bv) = qkv_weights(params, prefix + "self_attn.", dt)
    q = linear(x, wq, bq)
    k = linear(x, wk, bk)
    v = linear(x, wv, bv)
    out = np.empty_like(q)
    scale = hd ** -0.5
    start = 0
    for L in seqlens:
        sl = slice(start, start + L)
        qh = q[sl].reshape(L, nh, hd).transpose(1, 0, 2)
        kh = k[sl].reshape(L, nh, hd).transpose(1, 0, 2)
        vh = v[sl].reshape(L, nh, hd).transpose(1, 0, 2)
        p = softmax((qh @ kh.transpose(0, 2, 1)) * scale, axis=-1)
        out[sl] = (p @ vh).transpose(1, 0, 2).reshape(L, d)
        start += L
    return linear(out, _p(params, prefix + "self_attn.out_proj.weight", dt),
                  _p(params, prefix + "self_attn.out_proj.bias", dt))


def encoder_layer(params, cfg, i, x, seqlens, dt):
    """``model.py:204-223``."""
    pre = f"encoder.layers.{i}."
    eps = cfg.layer_norm_eps
    h = layer_norm(x, _p(params, pre + "layer_norm1.weight", dt), _p(params, pre + "layer_norm1.bias", dt), eps)
    x = x + attention_block(params, cfg, pre, h, seqlens, dt)
    h = layer_norm(x, _p(params, pre + "layer_norm2.weight", dt), _p(params, pre + "layer_norm2.bias", dt), eps)
    h = gelu_tanh(linear(h, _p(params, pre + "mlp.fc1.weight", dt), _p(params, pre + "mlp.fc1.bias", dt)))
    h = linear(h, _p(params, pre + "mlp.fc2.weight", dt), _p(params, pre + "mlp.fc2.bias", dt))
    return (x + h).astype(dt)


def forward_packed(params, cfg, seq_patches, token_grids, dt=np.float32):
    """``Siglip2SequenceVisionTransformer.forward`` (``model.py:260-292``):
    ``(seq_patches [N, C*p*p], token_grids [B, 2])`` -> ``[N, D]``."""
    grids = [(int(h), int(w)) for h, w in np.asarray(token_grids)]
    seqlens = [h * w for h, w in grids]
    assert sum(seqlens) == seq_patches.shape[0], "token_grids do not cover seq_patches"
    x = embeddings(params, cfg, seq_patches, grids, dt)
    for i in range(cfg.num_hidden_layers):
        x = encoder_layer(params, cfg, i, x, seqlens, dt)
    return layer_norm(x, _p(params, "post_layernorm.weight", dt), _p(params, "post_layernorm.bias", dt),
                      cfg.layer_norm_eps).astype(dt)


def map_head(params, cfg, hidden_list, dt=np.float32):
    """Attention-pooling head, ``transformers==5.5.0``
    ``modeling_siglip2.py:670-719``: for each image, the probe attends over
    that image's valid rows only (key padding mask), then
    ``h + fc2(gelu(fc1(LN(h))))``.  ``hidden_list``: one ``[L_i, D]`` array
    per image.  Returns ``[B, D]``."""
    d = cfg.hidden_size
    nh = cfg.num_attention_heads
    hd = d // nh
    w_in = _p(params, "head.attention.in_proj_weight", dt)
    b_in = _p(params, "head.attention.in_proj_bias", dt)
    probe = _p(params, "head.probe", dt).reshape(1, d)
    q = linear(probe, w_in[:d], b_in[:d]).reshape(nh, 1, hd)
    outs = []
    for xh in hidden_list:
        L = xh.shape[0]
        k = linear(xh, w_in[d:2 * d], b_in[d:2 * d]).reshape(L, nh, hd).transpose(1, 0, 2)
        v = linear(xh, w_in[2 * d:], b_in[2 * d:]).reshape(L, nh, hd).transpose(1, 0, 2)
        p = softmax((q @ k.transpose(0, 2, 1)) / math.sqrt(hd), axis=-1)
        outs.append((p @ v).transpose(1, 0, 2).reshape(1, d))
    a = np.concatenate(outs, axis=0)
    a = linear(a, _p(params, "head.attention.out_proj.weight", dt), _p(params, "head.attention.out_proj.bias", dt))
    h = layer_norm(a, _p(params, "head.layernorm.weight", dt), _p(params, "head.layernorm.bias", dt),
                   cfg.layer_norm_eps)
    h = gelu_tanh(linear(h, _p(params, "head.mlp.fc1.weight", dt), _p(params, "head.mlp.fc1.bias", dt)))
    h = linear(h, _p(params, "head.mlp.fc2.weight", dt), _p(params, "head.mlp.fc2.bias", dt))
    return (a + h).astype(dt)


def forward_padded(params, cfg, pixel_values, attention_mask, spatial_shapes, dt=np.float32):
    """HF-style entry (``modeling_siglip2.py:521-555``):
    ``pixel_values [B, P, C*p*p]``, ``attention_mask [B, P]`` (1 for the first
    ``h*w`` rows), ``spatial_shapes [B, 2]`` ->
    ``(last_hidden_state [B, P, D], pooler_output [B, D])``.

    Valid rows equal the packed forward's rows; padded rows are returned as
    zeros (the reference computes and then ignores them)."""
    pixel_values = np.asarray(pixel_values)
    mask = np.asarray(attention_mask)
    grids = [(int(h), int(w)) for h, w in np.asarray(spatial_shapes)]
    B, P, _ = pixel_values.shape
    lens = [h * w for h, w in grids]
    for b, L in enumerate(lens):
        assert int(mask[b].sum()) == L and mask[b, :L].all(), "mask must mark the first h*w rows"
    packed = np.concatenate([pixel_values[b, :L] for b, L in enumerate(lens)], axis=0)
    last = forward_packed(params, cfg, packed, np.array(grids), dt)
    out = np.zeros((B, P, cfg.hidden_size), dtype=dt)
    start = 0
    chunks = []
    for b, L in enumerate(lens):
        out[b, :L] = last[start:start + L]
        chunks.append(last[start:start + L])
        start += L
    pooled = map_head(params, cfg, chunks, dt) if "head.probe" in params else None
    return out, pooled


# ---------------------------------------------------------------------------
# FLOP model used for the roofline numerator (valid tokens only)
# ---------------------------------------------------------------------------


def flops_per_image(cfg, L: int, with_head: bool = True) -> float:
    """Dense-contraction FLOPs for one image of ``L`` valid tokens:
    ``2*768*D*L + layers*(L*(8D^2 + 4DI) + 4L^2 D) + head``, with
    ``head = 4D^2 + 4L D^2 + 4L D + 4 D I``."""
    D, I = cfg.hidden_size, cfg.intermediate_size
    cin = cfg.num_channels * cfg.patch_size ** 2
    f = 2 * cin * D * L + cfg.num_hidden_layers * (L * (8 * D * D + 4 * D * I) + 4 * L * L * D)
    if with_head:
        f += 4 * D * D + 4 * L * D * D + 4 * L * D + 4 * D * I
    return float(f)


# ---------------------------------------------------------------------------
# Train-mode attention-output dropout mask (model.py:166-169 applies
# nn.functional.dropout to the attention output; the kernels draw its mask
# from a counter-based generator so that the backward can regenerate it).
# Philox4x32-10 as published by Salmon, Moraes, Dror and Shaw ("Parallel
# random numbers: as easy as 1, 2, 3", SC 2011): ten rounds of two 32x32->64
# multiplications with the round multipliers below, the key bumped by the
# Weyl increments between rounds.
# ---------------------------------------------------------------------------
_PHILOX_M = (np.uint64(0xD2511F53), np.uint64(0xCD9E8D57))
_PHILOX_W = (np.uint32(0x9E3779B9), np.uint32(0xBB67AE85))


def philox4x32_10(ctr: np.ndarray, key: tuple[int, int]) -> np.ndarray:
    """``ctr``: uint32 ``[n, 4]`` counters; returns the uint32 ``[n, 4]`` outputs."""
    c = [ctr[:, i].astype(np.uint64) for i in range(4)]
    k0, k1 = np.uint32(key[0] & 0xFFFFFFFF), np.uint32(key[1] & 0xFFFFFFFF)
    mask = np.uint64(0xFFFFFFFF)
    for _ in range(10):
        p0 = _PHILOX_M[0] * c[0]
        p1 = _PHILOX_M[1] * c[2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & mask
        hi1, lo1 = p1 >> np.uint64(32), p1 & mask
        c = [hi1 ^ c[1] ^ np.uint64(k0), lo1, hi0 ^ c[3] ^ np.uint64(k1), lo0]
        k0 = np.uint32((int(k0) + int(_PHILOX_W[0])) & 0xFFFFFFFF)
        k1 = np.uint32((int(k1) + int(_PHILOX_W[1])) & 0xFFFFFFFF)
    return np.stack(c, 1).astype(np.uint32)


def dropout_keep(seed: int, offset: int, first: int, count: int, p: float) -> np.ndarray:
    """Keep flags of elements ``first .. first+count-1`` of the logical
    ``[rows, width]`` attention output (element e = row * width + col): u(e)
    = (word e % 4 of Philox4x32-10(counter = (e / 4, offset), key = seed)
    >> 8) * 2^-24, kept when u >= p (in fp32, as the kernels compare)."""
    e = np.arange(first, first + count, dtype=np.uint64)
    q = e >> np.uint64(2)
    ctr = np.stack([q & np.uint64(0xFFFFFFFF), q >> np.uint64(32),
                    np.full_like(q, offset & 0xFFFFFFFF), np.full_like(q, (offset >> 32) & 0xFFFFFFFF)], 1)
    out = philox4x32_10(ctr.astype(np.uint32), (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))
    word = out[np.arange(count), (e & np.uint64(3)).astype(np.int64)]
    u = (word >> np.uint32(8)).astype(np.float32) * np.float32(1.0 / 16777216.0)
    return u >= np.float32(p)
