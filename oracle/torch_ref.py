"""Torch restatement of the reference forward for same-dtype comparisons.

TEST INFRASTRUCTURE ONLY (see ``oracle/siglip2_oracle.py``).  The reference's
``model.py`` cannot be shipped to the GPU host, so this module replays its op
sequence with the same torch ops and in the same dtype (bf16/fp16 on the GPU),
which is what "the reference run at the same dtype" means in the parity
tests.  The functions are differentiable (autograd records when the weights
or inputs require grad), so the same replay is the gradient reference of the
training tests.  Ops, in order (tohskai/SigLIP-2):

* ``model.py:86-87``   patch Linear in the weight dtype;
* ``model.py:90-119``  position grid ``F.interpolate(bilinear, antialias)`` per
  image in the weight dtype, then added;
* ``model.py:204-223`` LN1 -> q/k/v Linear -> per-image softmax attention
  (the document mask; ``scale = hd^-0.5``) -> out Linear -> residual; LN2 ->
  fc1 -> GELU-tanh -> fc2 -> residual;
* ``model.py:286``     post LayerNorm;
* head: ``transformers`` ``modeling_siglip2.py:670-719`` (probe attention over
  the image's rows, LN, MLP, residual).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _w(sd, k, dt, dev):
    return sd[k].to(device=dev, dtype=dt)


def _qkv(sd, pre, dt, dev):
    if pre + "qkv_proj.weight" in sd:
        w = _w(sd, pre + "qkv_proj.weight", dt, dev)
        b = _w(sd, pre + "qkv_proj.bias", dt, dev)
        return list(zip(w.chunk(3, 0), b.chunk(3, 0)))
    return [(_w(sd, pre + f"{n}_proj.weight", dt, dev), _w(sd, pre + f"{n}_proj.bias", dt, dev)) for n in "qkv"]


def embeddings(sd, cfg, seq_patches, grids, dtype, device="cuda", pre="embeddings."):
    """``model.py:68-120``: patch Linear + per-image resized position grid."""
    D = cfg.hidden_size
    x = F.linear(seq_patches.to(device=device, dtype=dtype), _w(sd, pre + "patch_embedding.weight", dtype, device),
                 _w(sd, pre + "patch_embedding.bias", dtype, device))
    g = int(round(cfg.num_patches ** 0.5))
    table = _w(sd, pre + "position_embedding.weight", dtype, device).reshape(g, g, D).permute(2, 0, 1)[None]
    pos = torch.cat([F.interpolate(table, size=(int(h), int(w)), mode="bilinear", align_corners=False, antialias=True)
                     .reshape(D, int(h) * int(w)).transpose(0, 1) for h, w in grids], 0)
    return x + pos


def attention(sd, cfg, pre, h, lens, dtype, device="cuda"):
    """``model.py:144-176`` on packed rows ``h [N, D]``: q/k/v Linear,
    softmax attention within each run of ``lens`` rows, out Linear."""
    D, H = cfg.hidden_size, cfg.num_attention_heads
    hd = D // H
    (wq, bq), (wk, bk), (wv, bv) = _qkv(sd, pre, dtype, device)
    q, k, v = F.linear(h, wq, bq), F.linear(h, wk, bk), F.linear(h, wv, bv)
    outs = []
    s = 0
    for Ln in lens:
        sl = slice(s, s + Ln)
        qh, kh, vh = (t[sl].view(Ln, H, hd).transpose(0, 1) for t in (q, k, v))
        outs.append(F.scaled_dot_product_attention(qh[None], kh[None], vh[None], scale=hd ** -0.5)[0]
                    .transpose(0, 1).reshape(Ln, D))
        s += Ln
    a = torch.cat(outs, 0)
    return F.linear(a, _w(sd, pre + "out_proj.weight", dtype, device), _w(sd, pre + "out_proj.bias", dtype, device))


def mlp(sd, pre, h, dtype, device="cuda"):
    """``model.py:187-191``: fc2(gelu_tanh(fc1 h))."""
    h = F.gelu(F.linear(h, _w(sd, pre + "fc1.weight", dtype, device), _w(sd, pre + "fc1.bias", dtype, device)),
               approximate="tanh")
    return F.linear(h, _w(sd, pre + "fc2.weight", dtype, device), _w(sd, pre + "fc2.bias", dtype, device))


def encoder_layer(sd, cfg, pre, x, lens, dtype, device="cuda"):
    """``model.py:204-223`` on packed rows ``x [N, D]``."""
    D, eps = cfg.hidden_size, cfg.layer_norm_eps
    h = F.layer_norm(x, (D,), _w(sd, pre + "layer_norm1.weight", dtype, device),
                     _w(sd, pre + "layer_norm1.bias", dtype, device), eps)
    x = x + attention(sd, cfg, pre + "self_attn.", h, lens, dtype, device)
    h = F.layer_norm(x, (D,), _w(sd, pre + "layer_norm2.weight", dtype, device),
                     _w(sd, pre + "layer_norm2.bias", dtype, device), eps)
    return x + mlp(sd, pre + "mlp.", h, dtype, device)


def forward_packed(sd, cfg, seq_patches, grids, dtype, device="cuda"):
    D, eps = cfg.hidden_size, cfg.layer_norm_eps
    grids = [(int(h), int(w)) for h, w in grids]
    lens = [h * w for h, w in grids]
    x = embeddings(sd, cfg, seq_patches, grids, dtype, device)
    for i in range(cfg.num_hidden_layers):
        x = encoder_layer(sd, cfg, f"encoder.layers.{i}.", x, lens, dtype, device)
    return F.layer_norm(x, (D,), _w(sd, "post_layernorm.weight", dtype, device), _w(sd, "post_layernorm.bias", dtype, device),
                        eps)


def map_head(sd, cfg, last_packed, grids, dtype, device="cuda"):
    D, H = cfg.hidden_size, cfg.num_attention_heads
    hd = D // H
    win = _w(sd, "head.attention.in_proj_weight", dtype, device)
    bin_ = _w(sd, "head.attention.in_proj_bias", dtype, device)
    probe = _w(sd, "head.probe", dtype, device).reshape(1, D)
    q = F.linear(probe, win[:D], bin_[:D]).view(1, H, hd).transpose(0, 1)
    outs = []
    s = 0
    for h_, w_ in grids:
        Ln = int(h_) * int(w_)
        xh = last_packed[s:s + Ln]
        k = F.linear(xh, win[D:2 * D], bin_[D:2 * D]).view(Ln, H, hd).transpose(0, 1)
        v = F.linear(xh, win[2 * D:], bin_[2 * D:]).view(Ln, H, hd).transpose(0, 1)
        p = torch.softmax((q @ k.transpose(1, 2)) / math.sqrt(hd), -1)
        outs.append((p @ v).transpose(0, 1).reshape(1, D))
        s += Ln
    a = F.linear(torch.cat(outs, 0), _w(sd, "head.attention.out_proj.weight", dtype, device),
                 _w(sd, "head.attention.out_proj.bias", dtype, device))
    h = F.layer_norm(a, (D,), _w(sd, "head.layernorm.weight", dtype, device), _w(sd, "head.layernorm.bias", dtype, device),
                     cfg.layer_norm_eps)
    h = F.gelu(F.linear(h, _w(sd, "head.mlp.fc1.weight", dtype, device), _w(sd, "head.mlp.fc1.bias", dtype, device)),
               approximate="tanh")
    return a + F.linear(h, _w(sd, "head.mlp.fc2.weight", dtype, device), _w(sd, "head.mlp.fc2.bias", dtype, device))
