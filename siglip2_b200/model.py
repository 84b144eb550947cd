"""Drop-in SigLIP-2 NaFlex vision tower whose forward runs on this package's
sm_100a kernels through the C ABI (``siglip2_forward``).

Mirrors the reference's module tree and parameter names
(tohskai/SigLIP-2 ``model.py:39-292``; ``optimized_siglip2/model_optimized.py:341-388``)
so that ``state_dict``s move between them unchanged, plus the optional
attention-pooling head of ``transformers`` (``head.*``).

Forward forms
* ``model((seq_patches [N, C*p*p], token_grids [B, 2]))`` -> ``[N, D]``
  (the reference's packed API, ``model.py:260-292``);
* ``model(pixel_values [B, P, C*p*p], attention_mask [B, P], spatial_shapes [B, 2])``
  -> ``Siglip2Output(last_hidden_state [B, P, D], pooler_output [B, D])``
  (the HF-style padded API; padded rows of ``last_hidden_state`` are zero).

Accepted ``state_dict`` layouts: ``model.py`` (``self_attn.{q,k,v}_proj``),
the fused ``self_attn.qkv_proj`` of ``model_optimized.py:215`` (chunk order
Q, K, V), and ``head.*`` from ``transformers``.

Only inference is implemented: the forward runs without autograd, and
``train()`` mode with ``attention_dropout > 0`` is refused (the reference
applies dropout there, ``model.py:166-169``).
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import NamedTuple

import numpy as np
import torch
import torch.nn as nn

from . import _lib as L
from .ops import dtype_code, fold_layernorm


@dataclass
class Siglip2VisionConfig:
    """``model.py:39-49`` plus ``vision_use_head`` (the MAP head)."""

    hidden_size: int = 1152
    intermediate_size: int = 4304
    num_hidden_layers: int = 27
    num_attention_heads: int = 16
    num_channels: int = 3
    patch_size: int = 16
    layer_norm_eps: float = 1e-6
    attention_dropout: float = 0.1
    num_patches: int = 256
    vision_use_head: bool = True


class Siglip2Output(NamedTuple):
    last_hidden_state: torch.Tensor
    pooler_output: torch.Tensor | None


# ---------------------------------------------------------------------------
# parameter containers with the reference's names (no forward of their own)
# ---------------------------------------------------------------------------


class Siglip2SequenceEmbeddings(nn.Module):
    """Parameters of ``model.py:52-66``."""

    def __init__(self, config: Siglip2VisionConfig):
        super().__init__()
        self.config = config
        self.embed_dim = config.hidden_size
        self.patch_size = config.patch_size
        self.patch_embedding = nn.Linear(config.num_channels * config.patch_size ** 2, config.hidden_size)
        self.num_patches = config.num_patches
        self.position_embedding_size = int(config.num_patches ** 0.5)
        self.position_embedding = nn.Embedding(config.num_patches, config.hidden_size)


class Siglip2Attention(nn.Module):
    """Parameters of ``model.py:123-142``; also loads the fused ``qkv_proj``
    of ``model_optimized.py:215`` (rows = cat([q, k, v]))."""

    def __init__(self, config):
        super().__init__()
        self.embed_dim = config.hidden_size
        self.num_heads = config.num_attention_heads
        self.head_dim = self.embed_dim // self.num_heads
        if self.head_dim * self.num_heads != self.embed_dim:
            raise ValueError("embed_dim must be divisible by num_heads")
        self.scale = self.head_dim ** -0.5
        self.dropout = config.attention_dropout
        self.k_proj = nn.Linear(self.embed_dim, self.embed_dim)
        self.v_proj = nn.Linear(self.embed_dim, self.embed_dim)
        self.q_proj = nn.Linear(self.embed_dim, self.embed_dim)
        self.out_proj = nn.Linear(self.embed_dim, self.embed_dim)

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs):
        for kind in ("weight", "bias"):
            key = f"{prefix}qkv_proj.{kind}"
            if key in state_dict:
                q, k, v = state_dict.pop(key).chunk(3, dim=0)
                state_dict[f"{prefix}q_proj.{kind}"] = q
                state_dict[f"{prefix}k_proj.{kind}"] = k
                state_dict[f"{prefix}v_proj.{kind}"] = v
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                                      error_msgs)


class Siglip2MLP(nn.Module):
    """Parameters of ``model.py:179-185`` (GELU-tanh between fc1 and fc2)."""

    def __init__(self, config):
        super().__init__()
        self.fc1 = nn.Linear(config.hidden_size, config.intermediate_size)
        self.fc2 = nn.Linear(config.intermediate_size, config.hidden_size)


class Siglip2EncoderLayer(nn.Module):
    """Parameters of ``model.py:194-201``."""

    def __init__(self, config: Siglip2VisionConfig):
        super().__init__()
        self.embed_dim = config.hidden_size
        self.self_attn = Siglip2Attention(config)
        self.layer_norm1 = nn.LayerNorm(self.embed_dim, eps=config.layer_norm_eps)
        self.mlp = Siglip2MLP(config)
        self.layer_norm2 = nn.LayerNorm(self.embed_dim, eps=config.layer_norm_eps)


class Siglip2Encoder(nn.Module):
    def __init__(self, config: Siglip2VisionConfig):
        super().__init__()
        self.layers = nn.ModuleList([Siglip2EncoderLayer(config) for _ in range(config.num_hidden_layers)])


class Siglip2MultiheadAttentionPoolingHead(nn.Module):
    """Parameters of ``transformers`` ``modeling_siglip2.py:670-681``."""

    def __init__(self, config: Siglip2VisionConfig):
        super().__init__()
        self.probe = nn.Parameter(torch.randn(1, 1, config.hidden_size))
        self.attention = nn.MultiheadAttention(config.hidden_size, config.num_attention_heads, batch_first=True)
        self.layernorm = nn.LayerNorm(config.hidden_size, eps=config.layer_norm_eps)
        self.mlp = Siglip2MLP(config)
        self.num_heads = config.num_attention_heads


# ---------------------------------------------------------------------------
# weight packing for the C ABI
# ---------------------------------------------------------------------------


class _Packed:
    """Device tensors in the layout ``siglip2_weights`` documents, plus the
    ctypes structs pointing at them (kept alive together)."""

    def __init__(self, model: "Siglip2SequenceVisionTransformer"):
        cfg = model.config
        p0 = model.embeddings.patch_embedding.weight
        dev, dt = p0.device, p0.dtype
        if dev.type != "cuda":
            raise RuntimeError("siglip2_b200 runs on CUDA only: move the model with .to('cuda') first")
        D, I, H = cfg.hidden_size, cfg.intermediate_size, cfg.num_attention_heads
        hd = D // H
        f32 = torch.float32
        keep = []

        def k(t):
            t = t.contiguous()
            keep.append(t)
            return t.data_ptr()

        with torch.no_grad():
            emb = model.embeddings
            self.cfg = L.Config(hidden=D, intermediate=I, layers=cfg.num_hidden_layers, heads=H, head_dim=hd,
                                patch_dim=cfg.num_channels * cfg.patch_size ** 2,
                                pos_grid=int(round(cfg.num_patches ** 0.5)), eps=float(cfg.layer_norm_eps),
                                dtype=dtype_code(dt), has_head=int(model.head is not None))
            layers = (L.LayerWeights * max(1, cfg.num_hidden_layers))()
            for i, lyr in enumerate(model.encoder.layers):
                at = lyr.self_attn
                # q | k | v rows (the fused qkv_proj layout of model_optimized.py), LN1 folded in
                wp = torch.cat([lin.weight.float() for lin in (at.q_proj, at.k_proj, at.v_proj)], 0)
                bp = torch.cat([lin.bias.float() for lin in (at.q_proj, at.k_proj, at.v_proj)], 0)
                wg, c1, c2 = fold_layernorm(wp, bp, lyr.layer_norm1.weight, lyr.layer_norm1.bias, dt)
                f1, f1c1, f1c2 = fold_layernorm(lyr.mlp.fc1.weight, lyr.mlp.fc1.bias, lyr.layer_norm2.weight,
                                                lyr.layer_norm2.bias, dt)
                layers[i] = L.LayerWeights(
                    qkv_w=k(wg), qkv_c1=k(c1), qkv_c2=k(c2),
                    out_w=k(at.out_proj.weight.to(dt)), out_b=k(at.out_proj.bias.float()),
                    fc1_w=k(f1), fc1_c1=k(f1c1), fc1_c2=k(f1c2),
                    fc2_w=k(lyr.mlp.fc2.weight.to(dt)), fc2_b=k(lyr.mlp.fc2.bias.float()))
            self.layers = layers
            w = L.Weights()
            w.patch_w = k(emb.patch_embedding.weight.to(dt))
            w.patch_b = k(emb.patch_embedding.bias.float())
            w.pos_table = k(emb.position_embedding.weight.float())
            w.layers = ctypes.cast(layers, ctypes.POINTER(L.LayerWeights))
            w.post_ln_w = k(model.post_layernorm.weight.float())
            w.post_ln_b = k(model.post_layernorm.bias.float())
            if model.head is not None:
                hm = model.head
                win = hm.attention.in_proj_weight.float()
                bin_ = hm.attention.in_proj_bias.float()
                q = win[:D] @ hm.probe.float().reshape(D) + bin_[:D]
                u = torch.einsum("hd,hdk->hk", q.view(H, hd), win[D:2 * D].view(H, hd, D))
                u = u * (math.log2(math.e) / math.sqrt(hd))
                w.head_u = k(u)
                w.head_v_w = k(win[2 * D:].to(dt))
                w.head_v_b = k(bin_[2 * D:])
                w.head_o_w = k(hm.attention.out_proj.weight.to(dt))
                w.head_o_b = k(hm.attention.out_proj.bias.float())
                hf1, hc1, hc2 = fold_layernorm(hm.mlp.fc1.weight, hm.mlp.fc1.bias, hm.layernorm.weight,
                                               hm.layernorm.bias, dt)
                w.head_fc1_w, w.head_fc1_c1, w.head_fc1_c2 = k(hf1), k(hc1), k(hc2)
                w.head_fc2_w = k(hm.mlp.fc2.weight.to(dt))
                w.head_fc2_b = k(hm.mlp.fc2.bias.float())
            self.w = w
        self.keep = keep
        self.device = dev
        self.dtype = dt


def _metadata(hw: np.ndarray, device) -> tuple[torch.Tensor, int, int]:
    """cu_seqlens | hw | attention tiles (``siglip2_metadata``) on the device."""
    lib = L.load()
    hw = np.ascontiguousarray(hw, dtype=np.int32).reshape(-1)
    B = hw.size // 2
    n_tok, n_tiles = ctypes.c_int(), ctypes.c_int()
    size = lib.siglip2_metadata_size(hw.ctypes.data, B, ctypes.byref(n_tok), ctypes.byref(n_tiles))
    if size < 0:
        L.check(size)
    host = torch.empty(size, dtype=torch.int32, pin_memory=True)
    L.call("siglip2_metadata", hw.ctypes.data, B, host.data_ptr(), size)
    return host.to(device, non_blocking=True), n_tok.value, n_tiles.value


def tower_forward(packed: _Packed, patches: torch.Tensor, hw: np.ndarray, max_patches: int, want_pooled: bool):
    """Run ``siglip2_forward``.  ``patches`` packed ``[N, C]`` (max_patches=0)
    or padded ``[B, P, C]``.  Returns ``(last_hidden_state, pooler_output)``."""
    lib = L.load()
    dev = packed.device
    if patches.device != dev or patches.dtype != packed.dtype:
        patches = patches.to(device=dev, dtype=packed.dtype)
    patches = patches.contiguous()
    B = hw.shape[0]
    meta, N, _ = _metadata(hw, dev)
    D = packed.cfg.hidden
    if max_patches > 0:
        last = torch.empty((B, max_patches, D), dtype=packed.dtype, device=dev)
    else:
        if patches.shape[0] != N:
            raise ValueError(f"seq_patches has {patches.shape[0]} rows but token_grids cover {N}")
        last = torch.empty((N, D), dtype=packed.dtype, device=dev)
    pooled = torch.empty((B, D), dtype=packed.dtype, device=dev) if want_pooled else None
    ws_bytes = lib.siglip2_workspace_size(ctypes.byref(packed.cfg), B, N)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    L.call("siglip2_forward", ctypes.byref(packed.cfg), ctypes.byref(packed.w), patches.data_ptr(), B, max_patches,
           np.ascontiguousarray(hw, dtype=np.int32).ctypes.data, meta.data_ptr(), last.data_ptr(),
           pooled.data_ptr() if pooled is not None else None, ws.data_ptr(), ws_bytes, stream)
    return last, pooled


# ---------------------------------------------------------------------------
# the tower
# ---------------------------------------------------------------------------


class Siglip2SequenceVisionTransformer(nn.Module):
    """``model.py:250-292`` with the forward on sm_100a kernels."""

    def __init__(self, config: Siglip2VisionConfig):
        super().__init__()
        self.config = config
        self.embeddings = Siglip2SequenceEmbeddings(config)
        self.encoder = Siglip2Encoder(config)
        self.post_layernorm = nn.LayerNorm(config.hidden_size, eps=config.layer_norm_eps)
        self.head = Siglip2MultiheadAttentionPoolingHead(config) if getattr(config, "vision_use_head", False) else None
        self._packed = None
        self._packed_key = None

    # -- weight cache -----------------------------------------------------
    def _weights_key(self):
        return tuple((p.data_ptr(), p._version, p.dtype, p.device) for p in self.parameters())

    def packed_weights(self) -> _Packed:
        key = self._weights_key()
        if self._packed is None or key != self._packed_key:
            self._packed = _Packed(self)
            self._packed_key = key
        return self._packed

    def load_state_dict(self, state_dict, strict: bool = True, assign: bool = False):
        sd = dict(state_dict)
        if self.head is None:
            extra = [k for k in sd if k.startswith("head.")]
            for k in extra:
                sd.pop(k)
        res = super().load_state_dict(sd, strict=strict, assign=assign)
        self._packed = None
        return res

    def _check_mode(self):
        if self.training and self.config.attention_dropout > 0:
            raise NotImplementedError(
                "siglip2_b200 implements inference only: call .eval() (or set attention_dropout=0); "
                "the reference applies attention dropout in train mode")

    # -- forward ----------------------------------------------------------
    def forward(self, *args, **kwargs):
        self._check_mode()
        if len(args) == 1 and isinstance(args[0], (tuple, list)) and not kwargs:
            seq_patches, token_grids = args[0]
            return self.forward_packed(seq_patches, token_grids)
        names = ("pixel_values", "attention_mask", "spatial_shapes")
        vals = dict(zip(names, args))
        vals.update({k: v for k, v in kwargs.items() if k in names})
        if set(vals) != set(names):
            raise TypeError("forward takes (seq_patches, token_grids) or "
                            "(pixel_values, attention_mask, spatial_shapes)")
        return self.forward_padded(vals["pixel_values"], vals["attention_mask"], vals["spatial_shapes"])

    @torch.no_grad()
    def forward_packed(self, seq_patches: torch.Tensor, token_grids: torch.Tensor) -> torch.Tensor:
        """``model.py:260-292``: packed rows in, ``[N, D]`` out."""
        pk = self.packed_weights()
        hw = np.asarray(token_grids.detach().to("cpu", torch.int64).numpy(), dtype=np.int32).reshape(-1, 2)
        last, _ = tower_forward(pk, seq_patches, hw, 0, False)
        return last

    @torch.no_grad()
    def forward_padded(self, pixel_values, attention_mask, spatial_shapes) -> Siglip2Output:
        """HF ``Siglip2VisionTransformer.forward``: padded rows in;
        ``last_hidden_state [B, P, D]`` (zeros on padded rows) and
        ``pooler_output [B, D]`` (None without a head)."""
        pk = self.packed_weights()
        hw = np.asarray(spatial_shapes.detach().to("cpu", torch.int64).numpy(), dtype=np.int32).reshape(-1, 2)
        B, P = pixel_values.shape[:2]
        lens = hw[:, 0].astype(np.int64) * hw[:, 1]
        if attention_mask is not None:
            # spatial_shapes defines the valid rows; the mask must agree.  Its
            # contents are checked when it is on the host (checking a device
            # mask would synchronise the stream on every call).
            if tuple(attention_mask.shape) != (B, P):
                raise ValueError(f"attention_mask must be [B, P] = [{B}, {P}]")
            if not attention_mask.is_cuda:
                m = attention_mask.detach()
                if not torch.equal(m.sum(1).to(torch.int64), torch.from_numpy(lens)):
                    raise ValueError("attention_mask must mark exactly the first h*w rows of every image")
        last, pooled = tower_forward(pk, pixel_values, hw, P, self.head is not None)
        return Siglip2Output(last, pooled)


class Siglip2SequenceVisionTransformerOptimized(Siglip2SequenceVisionTransformer):
    """Same module under the name of ``optimized_siglip2/model_optimized.py:341``."""


# HF / BASELINE name of the tower
Siglip2VisionTransformer = Siglip2SequenceVisionTransformer
