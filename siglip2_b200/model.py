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

Inference (``eval()`` under ``torch.no_grad()`` / ``torch.inference_mode()``)
runs the whole tower as one library call.  When autograd records (grad mode
on and the input or a parameter requires grad) or in ``train()`` mode, the
forward runs through the submodules instead, one registered op per launch,
each with a backward formula, and ``train()`` mode applies the reference's
attention-output dropout (``model.py:166-169``) inside the attention kernel.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import NamedTuple

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib as L
from . import ops
from . import torch_ops  # registers torch.ops.siglip2_b200
from .ops import dtype_code, fold_layernorm

_OPS = torch.ops.siglip2_b200


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
# packed sequences: which rows attend to which
# ---------------------------------------------------------------------------


def create_document_ids(seq_sizes, device=None) -> torch.Tensor:
    """``model.py:12-36``: the image index of every packed token, padded to a
    multiple of 128 entries with ids that name no image (the pad ids count
    up from the token count)."""
    sizes = torch.as_tensor(seq_sizes).to(device)
    ids = torch.repeat_interleave(torch.arange(sizes.numel(), device=sizes.device), sizes)
    n = ids.numel()
    pad = (-n) % 128
    if pad:
        ids = torch.cat([ids, torch.arange(n, n + pad, device=ids.device, dtype=ids.dtype)])
    return ids


def _mask_runs(mask_mod, b: int, seq_len: int, device) -> list[int]:
    """Lengths of the contiguous runs of a document mask ``mask_mod(b, h, q,
    kv)`` over ``seq_len`` rows.  A run starts at row i when row i does not
    attend to row i-1.  Every row is then checked against both ends of its
    run and the rows just outside it, and ``mask_mod`` is compared with
    "same run" on every (row, column) pair up to 4096 rows, on a seeded
    sample of 64 columns per row above that.  A document mask passes; a
    causal, sliding-window or interleaved mask does not."""
    i = torch.arange(seq_len, device=device)
    bt = torch.full((), b, dtype=torch.int64, device=device)
    ht = torch.zeros((), dtype=torch.int64, device=device)

    def attends(q, k):
        return torch.broadcast_to(torch.as_tensor(mask_mod(bt, ht, q, k), device=device), q.shape).to(torch.bool)

    start = torch.ones(seq_len, dtype=torch.bool, device=device)
    start[1:] = ~attends(i[1:], i[:-1])
    starts = i[start]
    ends = torch.cat([starts[1:], torch.tensor([seq_len], device=device)])
    run = torch.cumsum(start.to(torch.int64), 0) - 1
    lo, hi = starts[run], ends[run]
    ok = bool(attends(i, lo).all()) and bool(attends(i, hi - 1).all())
    left, right = lo > 0, hi < seq_len
    ok = ok and not bool(attends(i[left], lo[left] - 1).any()) and not bool(attends(i[right], hi[right]).any())
    if ok and seq_len <= 4096:
        step = max(1, (1 << 22) // seq_len)
        for r0 in range(0, seq_len, step):
            q = i[r0:r0 + step, None].expand(-1, seq_len).reshape(-1)
            k = i[None, :].expand(min(step, seq_len - r0), -1).reshape(-1)
            ok = ok and bool(torch.equal(attends(q, k), run[q] == run[k]))
    elif ok:
        gen = torch.Generator().manual_seed(seq_len)
        k = torch.randint(0, seq_len, (seq_len * 64,), generator=gen).to(device)
        q = i.repeat_interleave(64)
        ok = bool(torch.equal(attends(q, k), run[q] == run[k]))
    if not ok:
        raise NotImplementedError("only document masks (rows attend to exactly their own contiguous run) "
                                  "are supported")
    return (ends - starts).tolist()


class Sequences:
    """The independent attention sequences of a row set (one per image and
    batch entry): their lengths on the host, ``cu_seqlens`` [n+1] and the
    128-row query tiles (``(sequence, tile)`` int32 pairs, longest sequences
    first) on the device.  Built once per encoder call and shared by its
    layers, as ``model_optimized.py:316-338`` shares one block mask."""

    def __init__(self, lengths, device):
        self.lengths = [int(n) for n in lengths]
        if not self.lengths or min(self.lengths) <= 0:
            raise ValueError("every sequence needs at least one row")
        cu = np.zeros(len(self.lengths) + 1, dtype=np.int64)
        np.cumsum(self.lengths, out=cu[1:])
        if cu[-1] >= 2 ** 31:
            raise ValueError("more than 2^31 - 1 rows")
        self.n_tokens = int(cu[-1])
        tiles = ops.attention_tiles(self.lengths).reshape(-1)
        nc = cu.size + (cu.size & 1)  # the tile pairs are read as 8-byte words
        host = torch.zeros(nc + tiles.numel(), dtype=torch.int32)
        host[:cu.size] = torch.from_numpy(cu.astype(np.int32))
        host[nc:] = tiles
        dev = host.to(device)
        self.cu_seqlens = dev[:cu.size]
        self.tiles = dev[nc:].view(-1, 2)

    @classmethod
    def full(cls, seq_len: int, batch: int, device) -> "Sequences":
        return cls([seq_len] * batch, device)

    @classmethod
    def from_document_ids(cls, document_ids, seq_len: int, batch: int, device) -> "Sequences":
        """``document_ids[q] == document_ids[kv]`` (``model.py:156-157``) over
        the first ``seq_len`` ids, the same for every batch entry.  Each
        document must be one contiguous run of rows."""
        ids = torch.as_tensor(document_ids).reshape(-1)
        if ids.numel() < seq_len:
            raise ValueError(f"document_ids has {ids.numel()} entries for {seq_len} rows")
        vals, counts = torch.unique_consecutive(ids[:seq_len], return_counts=True)
        if torch.unique(vals).numel() != vals.numel():
            raise NotImplementedError("each document must be one contiguous run of rows")
        return cls(counts.tolist() * batch, device)

    @classmethod
    def from_block_mask(cls, block_mask, seq_len: int, batch: int, device) -> "Sequences":
        """The runs of a ``flex_attention`` ``BlockMask`` built from a document
        mask (``model_optimized.py:323-330``); other masks are refused."""
        if tuple(block_mask.seq_lengths) != (seq_len, seq_len):
            raise ValueError(f"block mask is for {tuple(block_mask.seq_lengths)} rows, input has {seq_len}")
        nb, nh = block_mask.kv_num_blocks.shape[:2]
        if nh != 1 or nb not in (1, batch):
            raise NotImplementedError("block masks must have one head entry and 1 or batch batch entries")
        mdev = block_mask.kv_num_blocks.device
        runs = [_mask_runs(block_mask.mask_mod, b, seq_len, mdev) for b in range(nb)]
        if nb == 1:
            runs = runs * batch
        return cls([n for r in runs for n in r], device)


@torch.compiler.disable
def _sequences(x: torch.Tensor, document_ids=None, block_mask=None) -> Sequences:
    if x.dim() != 3:
        raise ValueError(f"hidden_states must be [batch, rows, hidden], got {tuple(x.shape)}")
    B, S = x.shape[:2]
    if block_mask is not None:
        return Sequences.from_block_mask(block_mask, S, B, x.device)
    if document_ids is not None:
        return Sequences.from_document_ids(document_ids, S, B, x.device)
    return Sequences.full(S, B, x.device)


# ---------------------------------------------------------------------------
# modules with the reference's names; forwards on the library's kernels
# ---------------------------------------------------------------------------


@torch.compiler.disable
def _derived(module: nn.Module, build):
    """Tensors derived from a module's parameters (concatenated, folded,
    cast), rebuilt when a parameter changes address, version, dtype or
    device."""
    key = tuple((p.data_ptr(), p._version, p.dtype, p.device) for p in module.parameters())
    hit = module.__dict__.get("_sg_derived")
    if hit is None or hit[0] != key:
        if any(p.device.type != "cuda" for p in module.parameters()):
            raise RuntimeError("siglip2_b200 runs on CUDA only: move the module with .to('cuda') first")
        with torch.no_grad():
            hit = (key, tuple(t.detach().contiguous() for t in build()))
        module.__dict__["_sg_derived"] = hit
    return hit[1]


def _rows(x: torch.Tensor, dtype) -> torch.Tensor:
    """``x [..., D]`` as a contiguous ``[rows, D]`` matrix of ``dtype``."""
    x2 = x.reshape(-1, x.shape[-1])
    return (x2 if x2.dtype == dtype else x2.to(dtype)).contiguous()


def _needs_grad(module: nn.Module, *xs) -> bool:
    """Autograd is recording something: the forward then passes the live
    parameters (the ops' backward reaches them) instead of the cached copies."""
    return torch.is_grad_enabled() and (any(x is not None and x.requires_grad for x in xs)
                                        or any(p.requires_grad for p in module.parameters()))


@torch.compiler.disable
def _dropout_args(module: nn.Module, p: float) -> tuple[float, int]:
    """``(p, seed)`` of the attention-output dropout of one call: active in
    ``train()`` mode as in ``model.py:166-169``; the 63-bit seed of the
    counter-based mask comes from torch's default CPU generator (so
    ``torch.manual_seed`` makes it reproducible) and travels to the backward,
    which regenerates the same mask."""
    if not (module.training and p > 0):
        return 0.0, 0
    return float(p), int(torch.randint(0, 2 ** 63 - 1, (1,), dtype=torch.int64).item())


class LayerNorm(nn.LayerNorm):
    """``nn.LayerNorm`` (``model.py:199,201,256``) whose forward is
    ``siglip2_layernorm``: fp32 statistics, biased variance."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if _needs_grad(self, x):
            w, b = self.weight.float(), self.bias.float()
        else:
            w, b = _derived(self, lambda: (self.weight.float(), self.bias.float()))
        return _OPS.layernorm(_rows(x, x.dtype), w, b, float(self.eps)).view(x.shape)


class LayerNormImproved(nn.Module):
    """``optimized_siglip2/model_optimized.py:23-80``: LayerNorm with the
    residual interface of its ``layer_norm_fn``.  ``residual`` is added first
    (in fp32) and the sum is what is normalised; with ``prenorm`` the sum is
    returned too, in fp32 when ``residual_in_fp32``, else in the residual's
    dtype.  As in the reference, ``is_rms_norm`` is not read.  Dropout,
    ``rowscale``, the second input (``x1``/``weight1``/``bias1``) and
    zero-centred weights are not implemented and raise."""

    def __init__(self, hidden_size, eps, bias=True, init_fn="ones"):
        super().__init__()
        if init_fn not in ("ones", "zeros"):
            raise ValueError(f"init_fn must be either 'ones' or 'zeros', got {init_fn}")
        self.hidden_size = hidden_size
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size) if init_fn == "ones" else torch.zeros(hidden_size))
        self.bias = nn.Parameter(torch.randn(hidden_size) if bias else torch.zeros(hidden_size))
        self.variance_epsilon = eps

    def forward(self, hidden_states, residual=None, x1=None, weight1=None, bias1=None, dropout_p=0.0, rowscale=None,
                prenorm=False, residual_in_fp32=False, zero_centered_weight=False, is_rms_norm=False,
                return_dropout_mask=False, out_dtype=None, out=None, residual_out=None):
        if (x1 is not None or weight1 is not None or bias1 is not None or rowscale is not None or dropout_p
                or zero_centered_weight or return_dropout_mask):
            raise NotImplementedError("siglip2_b200 LayerNormImproved: dropout, rowscale, x1/weight1/bias1 and "
                                      "zero_centered_weight are not implemented")
        x = hidden_states
        if _needs_grad(self, x, residual):
            w, b = self.weight.float(), self.bias.float()
        else:
            w, b = _derived(self, lambda: (self.weight.float(), self.bias.float()))
        if residual is None and not residual_in_fp32:
            y = _OPS.layernorm(_rows(x, x.dtype), w, b, float(self.variance_epsilon)).view(x.shape)
            res = x
        else:
            s = x.float() if residual is None else x.float() + residual.float()
            y = _OPS.layernorm(_rows(s, torch.float32), w, b, float(self.variance_epsilon)).view(x.shape)
            res = s.to(torch.float32 if residual_in_fp32 else residual.dtype)
        y = y.to(out_dtype or x.dtype)
        if out is not None:
            y = out.copy_(y)
        if residual_out is not None:
            res = residual_out.copy_(res)
        return (y, res) if prenorm else y

    def extra_repr(self):
        return f"{self.hidden_size}, eps={self.eps}"


class Siglip2SequenceEmbeddings(nn.Module):
    """``model.py:52-120``: patch Linear plus the learned position grid
    resized (antialiased bilinear) to each image, as one ``siglip2_patch_embed``
    launch."""

    def __init__(self, config: Siglip2VisionConfig):
        super().__init__()
        self.config = config
        self.embed_dim = config.hidden_size
        self.patch_size = config.patch_size
        self.patch_embedding = nn.Linear(config.num_channels * config.patch_size ** 2, config.hidden_size)
        self.num_patches = config.num_patches
        self.position_embedding_size = int(config.num_patches ** 0.5)
        self.position_embedding = nn.Embedding(config.num_patches, config.hidden_size)

    def forward(self, packed_seq_patches):
        """``(seq_patches [N, C*p*p], seq_sizes [B], spatial_shapes [B, 2])``
        -> ``[N, D]``; image b's rows are its ``h*w`` patches, row-major."""
        seq_patches, seq_sizes, spatial_shapes = packed_seq_patches
        params = lambda: (self.patch_embedding.weight, self.patch_embedding.bias.float(),  # noqa: E731
                          self.position_embedding.weight.float())
        w, b, table = params() if _needs_grad(self, seq_patches) else _derived(self, params)
        hw = _grids(spatial_shapes)
        if seq_sizes is not None:
            sizes = torch.as_tensor(seq_sizes).detach().to("cpu", torch.int64).reshape(-1).numpy()
            if not np.array_equal(sizes, hw[:, 0].astype(np.int64) * hw[:, 1]):
                raise ValueError("seq_sizes must equal h*w of spatial_shapes")
        meta, N, _ = _metadata(hw, w.device)
        B = hw.shape[0]
        cu, hw_dev = meta[:B + 1], meta[B + 1:3 * B + 1]
        tok = _OPS.token_image(cu, N)
        return _OPS.patch_embed(_rows(seq_patches, w.dtype), w, b, table, hw_dev, cu, tok,
                                [int(v) for v in hw.reshape(-1)])


def _attention(m: nn.Module, x: torch.Tensor, seqs: Sequences) -> torch.Tensor:
    """QKV projection -> per-sequence attention -> out projection
    (``model.py:144-176``), three launches."""
    params = lambda: (*m.qkv_params(), m.out_proj.weight, m.out_proj.bias)  # noqa: E731
    qkv_w, qkv_b, out_w, out_b = params() if _needs_grad(m, x) else _derived(m, params)
    x2 = _rows(x, qkv_w.dtype)
    if x2.shape[0] != seqs.n_tokens:
        raise ValueError(f"{x2.shape[0]} rows but the sequences cover {seqs.n_tokens}")
    qkv = _OPS.gemm(x2, qkv_w, L.EPI_BIAS, qkv_b.float(), None, None, None, 0.0)
    attn = torch_ops.attention_for_training if _needs_grad(m, x) else _OPS.fmha_varlen
    a = attn(qkv, seqs.cu_seqlens, seqs.tiles, m.num_heads, m.head_dim, seqs.lengths, *_dropout_args(m, m.dropout))
    return _OPS.gemm(a, out_w, L.EPI_BIAS, out_b.float(), None, None, None, 0.0).view(*x.shape[:-1], -1)


class Siglip2Attention(nn.Module):
    """``model.py:123-176``; also loads the fused ``qkv_proj`` of
    ``model_optimized.py:215`` (rows = cat([q, k, v]))."""

    def __init__(self, config):
        super().__init__()
        self.config = config
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

    def qkv_params(self):
        """The fused projection ``[3D, D]`` / ``[3D]`` (q | k | v rows)."""
        lins = (self.q_proj, self.k_proj, self.v_proj)
        return torch.cat([m.weight for m in lins], 0), torch.cat([m.bias for m in lins], 0)

    def forward(self, hidden_states, document_ids=None, output_attentions=False):
        """``[B, S, D]`` -> ``(out [B, S, D], None)``; rows q and kv attend
        when ``document_ids[q] == document_ids[kv]`` (all rows when None).
        In ``train()`` mode the attention output is dropped out with
        probability ``attention_dropout`` before ``out_proj``."""
        return _attention(self, hidden_states, _sequences(hidden_states, document_ids=document_ids)), None


class Siglip2AttentionImproved(Siglip2Attention):
    """``optimized_siglip2/model_optimized.py:200-243``: fused ``qkv_proj``;
    the mask is a ``flex_attention`` ``BlockMask`` built from a document
    mask (or ``document_ids`` directly)."""

    def __init__(self, config):
        nn.Module.__init__(self)
        self.config = config
        self.embed_dim = config.hidden_size
        self.num_heads = config.num_attention_heads
        self.head_dim = self.embed_dim // self.num_heads
        if self.head_dim * self.num_heads != self.embed_dim:
            raise ValueError("embed_dim must be divisible by num_heads")
        self.scale = self.head_dim ** -0.5
        self.dropout = config.attention_dropout
        self.qkv_proj = nn.Linear(self.embed_dim, 3 * self.embed_dim)
        self.out_proj = nn.Linear(self.embed_dim, self.embed_dim)

    def _load_from_state_dict(self, *args, **kwargs):
        nn.Module._load_from_state_dict(self, *args, **kwargs)

    def qkv_params(self):
        return self.qkv_proj.weight, self.qkv_proj.bias

    def forward(self, hidden_states, block_mask=None, output_attentions=False, document_ids=None):
        seqs = _sequences(hidden_states, document_ids=document_ids, block_mask=block_mask)
        return _attention(self, hidden_states, seqs), None


class Siglip2MLP(nn.Module):
    """``model.py:179-191``: ``fc2(gelu_tanh(fc1 x))`` as two GEMMs, GELU in
    the first one's epilogue."""

    def __init__(self, config):
        super().__init__()
        self.config = config
        self.fc1 = nn.Linear(config.hidden_size, config.intermediate_size)
        self.fc2 = nn.Linear(config.intermediate_size, config.hidden_size)

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        if _needs_grad(self, hidden_states):
            w1, b1, w2, b2 = self.fc1.weight, self.fc1.bias.float(), self.fc2.weight, self.fc2.bias.float()
        else:
            w1, b1, w2, b2 = _derived(self, lambda: (self.fc1.weight, self.fc1.bias.float(), self.fc2.weight,
                                                     self.fc2.bias.float()))
        h = _OPS.gemm(_rows(hidden_states, w1.dtype), w1, L.EPI_BIAS_GELU, b1, None, None, None, 0.0)
        return _OPS.gemm(h, w2, L.EPI_BIAS, b2, None, None, None, 0.0).view(*hidden_states.shape[:-1], -1)


class MLPImproved(Siglip2MLP):
    """``optimized_siglip2/model_optimized.py:246-260`` (same parameters and
    result as ``Siglip2MLP``)."""


class Siglip2SequenceEmbeddingsImproved(Siglip2SequenceEmbeddings):
    """``optimized_siglip2/model_optimized.py:123-197`` (same parameters and
    result as ``Siglip2SequenceEmbeddings``)."""


def _layer_tensors(layer: nn.Module):
    """The ten per-layer tensors of ``siglip2_layer_weights`` (LAYER_FIELDS
    order): QKV with LayerNorm 1 folded, out projection, fc1 with LayerNorm 2
    folded, fc2."""
    at, mlp = layer.self_attn, layer.mlp
    wp, bp = at.qkv_params()
    dt = wp.dtype
    return (*fold_layernorm(wp, bp, layer.layer_norm1.weight, layer.layer_norm1.bias, dt),
            at.out_proj.weight.to(dt), at.out_proj.bias.float(),
            *fold_layernorm(mlp.fc1.weight, mlp.fc1.bias, layer.layer_norm2.weight, layer.layer_norm2.bias, dt),
            mlp.fc2.weight.to(dt), mlp.fc2.bias.float())


def _encoder_layer(layer: nn.Module, x: torch.Tensor, seqs: Sequences, rs: torch.Tensor | None = None):
    """One pre-LN layer (``model.py:204-223``) as the launch sequence the
    tower runs: LN1 folded into the QKV GEMM, attention, out projection with
    the residual, LN2 folded into fc1 (+GELU), fc2 with the residual.  The
    LayerNorm statistics travel as row sums (``rs`` in, the output's out).
    Returns ``(y, rs_y)``."""
    if _needs_grad(layer, x):
        return _encoder_layer_unfused(layer, x, seqs), None
    qw, qc1, qc2, ow, ob, f1w, f1c1, f1c2, f2w, f2b = _derived(layer, lambda: _layer_tensors(layer))
    eps1, eps2 = float(layer.layer_norm1.eps), float(layer.layer_norm2.eps)
    at = layer.self_attn
    x2 = _rows(x, qw.dtype)
    if x2.shape[0] != seqs.n_tokens:
        raise ValueError(f"{x2.shape[0]} rows but the sequences cover {seqs.n_tokens}")
    if rs is None:
        rs = _OPS.rowsums(x2)
    qkv, _ = _OPS.gemm_rowsums(x2, qw, L.EPI_LN_ROWSUMS, None, None, qc1, qc2, eps1, rs, False)
    a = _OPS.fmha_varlen(qkv, seqs.cu_seqlens, seqs.tiles, at.num_heads, at.head_dim, seqs.lengths,
                         *_dropout_args(at, at.dropout))
    h, rs_h = _OPS.gemm_rowsums(a, ow, L.EPI_BIAS_RES_ROWSUMS, ob, x2, None, None, 0.0, None, True)
    m, _ = _OPS.gemm_rowsums(h, f1w, L.EPI_LN_ROWSUMS_GELU, None, None, f1c1, f1c2, eps2, rs_h, False)
    y, rs_y = _OPS.gemm_rowsums(m, f2w, L.EPI_BIAS_RES_ROWSUMS, f2b, h, None, None, 0.0, None, True)
    return y.view(x.shape), rs_y


def _encoder_layer_unfused(layer: nn.Module, x: torch.Tensor, seqs: Sequences) -> torch.Tensor:
    """The layer for autograd: the same arithmetic as ``model.py:204-223``
    with the LayerNorms as their own launches (folding them into the GEMM
    weights has no backward here), every op one with a backward formula."""
    at, mlp = layer.self_attn, layer.mlp
    x2 = _rows(x, at.out_proj.weight.dtype)
    if x2.shape[0] != seqs.n_tokens:
        raise ValueError(f"{x2.shape[0]} rows but the sequences cover {seqs.n_tokens}")
    ln1, ln2 = layer.layer_norm1, layer.layer_norm2
    h = _OPS.layernorm(x2, ln1.weight.float(), ln1.bias.float(), float(ln1.eps))
    wq, bq = at.qkv_params()
    qkv = _OPS.gemm(h, wq, L.EPI_BIAS, bq.float(), None, None, None, 0.0)
    a = torch_ops.attention_for_training(qkv, seqs.cu_seqlens, seqs.tiles, at.num_heads, at.head_dim, seqs.lengths,
                                         *_dropout_args(at, at.dropout))
    r = _OPS.gemm(a, at.out_proj.weight, L.EPI_BIAS_RES, at.out_proj.bias.float(), x2, None, None, 0.0)
    h = _OPS.layernorm(r, ln2.weight.float(), ln2.bias.float(), float(ln2.eps))
    m = _OPS.gemm(h, mlp.fc1.weight, L.EPI_BIAS_GELU, mlp.fc1.bias.float(), None, None, None, 0.0)
    y = _OPS.gemm(m, mlp.fc2.weight, L.EPI_BIAS_RES, mlp.fc2.bias.float(), r, None, None, 0.0)
    return y.view(x.shape)


class Siglip2EncoderLayer(nn.Module):
    """``model.py:194-223``."""

    def __init__(self, config: Siglip2VisionConfig):
        super().__init__()
        self.embed_dim = config.hidden_size
        self.self_attn = Siglip2Attention(config)
        self.layer_norm1 = LayerNorm(self.embed_dim, eps=config.layer_norm_eps)
        self.mlp = Siglip2MLP(config)
        self.layer_norm2 = LayerNorm(self.embed_dim, eps=config.layer_norm_eps)

    def forward(self, hidden_states: torch.Tensor, document_ids: torch.Tensor | None = None) -> torch.Tensor:
        return _encoder_layer(self, hidden_states, _sequences(hidden_states, document_ids=document_ids))[0]


class Siglip2EncoderLayerImproved(nn.Module):
    """``optimized_siglip2/model_optimized.py:263-301`` (fused ``qkv_proj``,
    ``LayerNormImproved``); the mask is a document-mask ``BlockMask``."""

    def __init__(self, config: Siglip2VisionConfig):
        super().__init__()
        self.embed_dim = config.hidden_size
        self.self_attn = Siglip2AttentionImproved(config)
        self.layer_norm1 = LayerNormImproved(self.embed_dim, eps=config.layer_norm_eps)
        self.mlp = MLPImproved(config)
        self.layer_norm2 = LayerNormImproved(self.embed_dim, eps=config.layer_norm_eps)

    def forward(self, hidden_states: torch.Tensor, block_mask=None, document_ids=None) -> torch.Tensor:
        seqs = _sequences(hidden_states, document_ids=document_ids, block_mask=block_mask)
        return _encoder_layer(self, hidden_states, seqs)[0]


def _encoder(enc: nn.Module, inputs_embeds: torch.Tensor, document_ids) -> torch.Tensor:
    seqs = _sequences(inputs_embeds, document_ids=document_ids)
    x, rs = inputs_embeds, None
    for layer in enc.layers:
        x, rs = _encoder_layer(layer, x, seqs, rs)
    return x


class Siglip2Encoder(nn.Module):
    """``model.py:226-247``: the layers over one shared set of sequences."""

    def __init__(self, config: Siglip2VisionConfig):
        super().__init__()
        self.config = config
        self.layers = nn.ModuleList([Siglip2EncoderLayer(config) for _ in range(config.num_hidden_layers)])

    def forward(self, inputs_embeds: torch.Tensor, document_ids: torch.Tensor | None = None) -> torch.Tensor:
        return _encoder(self, inputs_embeds, document_ids)


class Siglip2EncoderImproved(nn.Module):
    """``optimized_siglip2/model_optimized.py:304-338``."""

    def __init__(self, config: Siglip2VisionConfig):
        super().__init__()
        self.config = config
        self.layers = nn.ModuleList([Siglip2EncoderLayerImproved(config) for _ in range(config.num_hidden_layers)])

    def forward(self, inputs_embeds: torch.Tensor, document_ids: torch.Tensor | None = None) -> torch.Tensor:
        return _encoder(self, inputs_embeds, document_ids)


class Siglip2MultiheadAttentionPoolingHead(nn.Module):
    """``transformers`` ``modeling_siglip2.py:670-713``: the attention-pooling
    (MAP) head.  Runs inside the tower's forward (``pooler_output``); its own
    forward does the same on padded rows."""

    def __init__(self, config: Siglip2VisionConfig):
        super().__init__()
        self.probe = nn.Parameter(torch.randn(1, 1, config.hidden_size))
        self.attention = nn.MultiheadAttention(config.hidden_size, config.num_attention_heads, batch_first=True)
        self.layernorm = LayerNorm(config.hidden_size, eps=config.layer_norm_eps)
        self.mlp = Siglip2MLP(config)
        self.num_heads = config.num_attention_heads

    def _tensors(self):
        """Per-head key vectors of the probe (base-2 scores: the query
        projection of the probe through each head's key rows, times
        log2(e) / sqrt(head_dim); the key bias shifts all scores of a head
        equally and drops out), then the value / out projections, LayerNorm
        and MLP parameters."""
        D = self.probe.shape[-1]
        H = self.num_heads
        hd = D // H
        win = self.attention.in_proj_weight.float()
        bin_ = self.attention.in_proj_bias.float()
        q = win[:D] @ self.probe.float().reshape(D) + bin_[:D]
        u = torch.einsum("hd,hdk->hk", q.view(H, hd), win[D:2 * D].view(H, hd, D)) * (math.log2(math.e) /
                                                                                      math.sqrt(hd))
        dt = self.attention.in_proj_weight.dtype
        return (u, self.attention.in_proj_weight[2 * D:], bin_[2 * D:], self.attention.out_proj.weight,
                self.attention.out_proj.bias.float(), self.layernorm.weight.float(), self.layernorm.bias.float(),
                self.mlp.fc1.weight.to(dt), self.mlp.fc1.bias.float(), self.mlp.fc2.weight.to(dt),
                self.mlp.fc2.bias.float())

    def forward(self, hidden_state: torch.Tensor, attention_mask: torch.Tensor | None = None) -> torch.Tensor:
        """``hidden_state [B, P, D]`` -> ``[B, D]``: the probe attends over each
        image's valid rows (``siglip2_head_pool``), then the value and out
        projections, LayerNorm, MLP and residual (library GEMMs).  The valid
        rows of an image must be its first ones, as ``attention_mask`` marks
        them in the padded forward (other masks raise); without a mask every
        row is valid.  With autograd recording (grad mode on and the input
        or a parameter requiring grad) the head runs as differentiable steps
        instead (``_forward_autograd``)."""
        B, P, D = hidden_state.shape
        H = self.num_heads
        if attention_mask is None:
            lens = torch.full((B,), P, dtype=torch.int64)
        else:
            m = attention_mask.detach().to("cpu", torch.int64).reshape(B, P)
            lens = m.sum(1)
            if not torch.equal(m, (torch.arange(P)[None] < lens[:, None]).to(m.dtype)) or bool((lens == 0).any()):
                raise NotImplementedError("attention_mask must mark a non-empty prefix of every image's rows")
        if _needs_grad(self, hidden_state):
            return self._forward_autograd(hidden_state, lens)
        (u, wv, bv, wo, bo, lw, lb, w1, b1, w2, b2) = _derived(self, self._tensors)
        x = hidden_state.to(wv.dtype).contiguous()
        cu = torch.zeros(B + 1, dtype=torch.int32)
        cu[1:] = torch.cumsum(lens, 0).to(torch.int32)
        cu = cu.to(x.device)
        with torch.no_grad():
            pooled = ops.head_pool(x, u, cu, B * P, max_patches=P)                 # [B, H, D]
            v = ops.gemm(pooled.view(B * H, D), wv, L.EPI_BIAS, bias=bv).view(B, H, H, D // H)
            idx = torch.arange(H, device=x.device)
            a = ops.gemm(v[:, idx, idx, :].reshape(B, D).contiguous(), wo, L.EPI_BIAS, bias=bo)
            h = ops.layernorm(a, lw, lb, float(self.layernorm.eps))
            h = ops.gemm(h, w1, L.EPI_BIAS_GELU, bias=b1)
            return ops.gemm(h, w2, L.EPI_BIAS_RES, bias=b2, res=a)

    def _forward_autograd(self, hidden_state: torch.Tensor, lens: torch.Tensor) -> torch.Tensor:
        """The head (``modeling_siglip2.py:684-713``) as differentiable steps
        for training: the key/value projection of every row, the out
        projection and the MLP on the library GEMM ops (each with a backward),
        the probe's attention over each image's valid keys through torch's
        scaled_dot_product_attention with a key-padding mask, LayerNorm on
        the LayerNorm op."""
        B, P, D = hidden_state.shape
        H = self.num_heads
        hd = D // H
        att = self.attention
        dt = att.in_proj_weight.dtype
        win, bin_ = att.in_proj_weight, att.in_proj_bias
        q = F.linear(self.probe.reshape(1, D).to(dt), win[:D], bin_[:D].to(dt))                      # [1, D]
        kv = _OPS.gemm(_rows(hidden_state, dt), win[D:], L.EPI_BIAS, bin_[D:].float(), None, None, None, 0.0)
        k, v = kv.view(B, P, 2, H, hd).unbind(2)                                                     # [B, P, H, hd]
        keep = (torch.arange(P)[None] < lens[:, None]).to(hidden_state.device)[:, None, None, :]     # [B, 1, 1, P]
        o = F.scaled_dot_product_attention(q.view(1, H, 1, hd).expand(B, H, 1, hd), k.transpose(1, 2),
                                           v.transpose(1, 2), attn_mask=keep)                        # [B, H, 1, hd]
        a = _OPS.gemm(o.reshape(B, D).contiguous(), att.out_proj.weight, L.EPI_BIAS, att.out_proj.bias.float(),
                      None, None, None, 0.0)
        h = self.layernorm(a)
        h = _OPS.gemm(h, self.mlp.fc1.weight, L.EPI_BIAS_GELU, self.mlp.fc1.bias.float(), None, None, None, 0.0)
        return _OPS.gemm(h, self.mlp.fc2.weight, L.EPI_BIAS_RES, self.mlp.fc2.bias.float(), a, None, None, 0.0)

# ---------------------------------------------------------------------------
# weight packing for the C ABI
# ---------------------------------------------------------------------------


# Flat order of the packed weight tensors: LAYER_FIELDS for every layer,
# then TOWER_FIELDS, then HEAD_FIELDS when the head is present.
LAYER_FIELDS = ("qkv_w", "qkv_c1", "qkv_c2", "out_w", "out_b", "fc1_w", "fc1_c1", "fc1_c2", "fc2_w", "fc2_b")
TOWER_FIELDS = ("patch_w", "patch_b", "pos_table", "post_ln_w", "post_ln_b")
HEAD_FIELDS = ("head_u", "head_v_w", "head_v_b", "head_o_w", "head_o_b", "head_fc1_w", "head_fc1_c1", "head_fc1_c2",
               "head_fc2_w", "head_fc2_b")
# siglip2_config's integer fields, in the order of the dims list
DIM_FIELDS = ("hidden", "intermediate", "layers", "heads", "head_dim", "patch_dim", "pos_grid", "dtype", "has_head")


def weight_structs(dims, eps: float, tensors):
    """ctypes ``siglip2_config`` / ``siglip2_weights`` (and the layer array
    they point into) over ``tensors`` in the flat order above.  The structs
    hold raw pointers: the tensors must outlive every call that uses them."""
    cfg = L.Config(eps=float(eps), **dict(zip(DIM_FIELDS, (int(d) for d in dims))))
    n_layers = cfg.layers
    want = n_layers * len(LAYER_FIELDS) + len(TOWER_FIELDS) + (len(HEAD_FIELDS) if cfg.has_head else 0)
    if len(tensors) != want:
        raise ValueError(f"expected {want} packed weight tensors, got {len(tensors)}")
    ptrs = [t.data_ptr() for t in tensors]
    layers = (L.LayerWeights * max(1, n_layers))()
    for i in range(n_layers):
        layers[i] = L.LayerWeights(*ptrs[i * len(LAYER_FIELDS):(i + 1) * len(LAYER_FIELDS)])
    rest = ptrs[n_layers * len(LAYER_FIELDS):]
    w = L.Weights(**dict(zip(TOWER_FIELDS, rest)))
    w.layers = ctypes.cast(layers, ctypes.POINTER(L.LayerWeights))
    if cfg.has_head:
        for name, p in zip(HEAD_FIELDS, rest[len(TOWER_FIELDS):]):
            setattr(w, name, p)
    return cfg, w, layers


class _Packed:
    """Device tensors in the layout ``siglip2_weights`` documents (``tensors``,
    flat in the order of LAYER_FIELDS / TOWER_FIELDS / HEAD_FIELDS), plus the
    ctypes structs pointing at them (kept alive together)."""

    def __init__(self, model: "Siglip2SequenceVisionTransformer"):
        cfg = model.config
        p0 = model.embeddings.patch_embedding.weight
        dev, dt = p0.device, p0.dtype
        if dev.type != "cuda":
            raise RuntimeError("siglip2_b200 runs on CUDA only: move the model with .to('cuda') first")
        D, I, H = cfg.hidden_size, cfg.intermediate_size, cfg.num_attention_heads
        hd = D // H
        ts = []

        def k(*xs):
            ts.extend(x.detach().contiguous() for x in xs)

        with torch.no_grad():
            emb = model.embeddings
            for lyr in model.encoder.layers:
                k(*_layer_tensors(lyr))
            k(emb.patch_embedding.weight.to(dt), emb.patch_embedding.bias.float(),
              emb.position_embedding.weight.float(), model.post_layernorm.weight.float(),
              model.post_layernorm.bias.float())
            if model.head is not None:
                hm = model.head
                win = hm.attention.in_proj_weight.float()
                bin_ = hm.attention.in_proj_bias.float()
                q = win[:D] @ hm.probe.float().reshape(D) + bin_[:D]
                u = torch.einsum("hd,hdk->hk", q.view(H, hd), win[D:2 * D].view(H, hd, D))
                k(u * (math.log2(math.e) / math.sqrt(hd)))
                k(win[2 * D:].to(dt), bin_[2 * D:])
                k(hm.attention.out_proj.weight.to(dt), hm.attention.out_proj.bias.float())
                k(*fold_layernorm(hm.mlp.fc1.weight, hm.mlp.fc1.bias, hm.layernorm.weight, hm.layernorm.bias, dt))
                k(hm.mlp.fc2.weight.to(dt), hm.mlp.fc2.bias.float())
        self.dims = [D, I, cfg.num_hidden_layers, H, hd, cfg.num_channels * cfg.patch_size ** 2,
                     int(round(cfg.num_patches ** 0.5)), dtype_code(dt), int(model.head is not None)]
        self.eps = float(cfg.layer_norm_eps)
        self.tensors = ts
        self.cfg, self.w, self.layers = weight_structs(self.dims, self.eps, ts)
        self.device = dev
        self.dtype = dt


def _grids(spatial_shapes) -> np.ndarray:
    """``[B, 2]`` int32 (h, w) grids on the host (one device read when the
    shapes live on the GPU)."""
    t = torch.as_tensor(spatial_shapes).detach().to("cpu", torch.int64)
    return np.ascontiguousarray(t.numpy(), dtype=np.int32).reshape(-1, 2)


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


def run_tower(cfg: L.Config, w: L.Weights, dev, dtype, patches: torch.Tensor, hw: np.ndarray, max_patches: int,
              want_pooled: bool):
    """Run ``siglip2_forward`` with the given structs.  ``patches`` packed
    ``[N, C]`` (max_patches=0) or padded ``[B, P, C]``.  Returns
    ``(last_hidden_state, pooler_output)`` (the second None unless
    ``want_pooled``)."""
    lib = L.load()
    if want_pooled and not cfg.has_head:
        raise ValueError("pooler_output needs the attention-pooling head")
    if patches.device != dev or patches.dtype != dtype:
        patches = patches.to(device=dev, dtype=dtype)
    patches = patches.contiguous()
    B = hw.shape[0]
    meta, N, _ = _metadata(hw, dev)
    D = cfg.hidden
    if max_patches > 0:
        if tuple(patches.shape[:2]) != (B, max_patches):
            raise ValueError(f"pixel_values must be [B, max_patches, C] = [{B}, {max_patches}, C]")
        last = torch.empty((B, max_patches, D), dtype=dtype, device=dev)
    else:
        if patches.shape[0] != N:
            raise ValueError(f"seq_patches has {patches.shape[0]} rows but token_grids cover {N}")
        last = torch.empty((N, D), dtype=dtype, device=dev)
    pooled = torch.empty((B, D), dtype=dtype, device=dev) if want_pooled else None
    ws_bytes = lib.siglip2_workspace_size(ctypes.byref(cfg), B, N)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    L.call("siglip2_forward", ctypes.byref(cfg), ctypes.byref(w), patches.data_ptr(), B, max_patches,
           np.ascontiguousarray(hw, dtype=np.int32).ctypes.data, meta.data_ptr(), last.data_ptr(),
           pooled.data_ptr() if pooled is not None else None, ws.data_ptr(), ws_bytes, stream)
    return last, pooled


def tower_forward(packed: _Packed, patches: torch.Tensor, hw: np.ndarray, max_patches: int, want_pooled: bool):
    """``run_tower`` with a module's packed weights."""
    return run_tower(packed.cfg, packed.w, packed.device, packed.dtype, patches, hw, max_patches, want_pooled)


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
        self.post_layernorm = LayerNorm(config.hidden_size, eps=config.layer_norm_eps)
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

    def _submodule_path(self, x: torch.Tensor) -> bool:
        """Autograd records (the submodule ops carry the backward) or
        ``train()`` mode applies dropout: run the submodules instead of the
        one-call inference forward."""
        return _needs_grad(self, x) or (self.training and self.config.attention_dropout > 0)

    def _forward_rows(self, rows: torch.Tensor, hw: np.ndarray) -> torch.Tensor:
        """Packed rows through the submodules (``model.py:260-292`` step by
        step): embeddings, every encoder layer over one shared set of
        sequences, post-LayerNorm.  Each step is a registered op with a
        backward; in ``train()`` mode the attention output is dropped out."""
        x = self.embeddings((rows, None, torch.from_numpy(np.ascontiguousarray(hw))))
        lens = (hw[:, 0].astype(np.int64) * hw[:, 1]).tolist()
        seqs = Sequences(lens, x.device)
        rs = None
        for layer in self.encoder.layers:
            x, rs = _encoder_layer(layer, x, seqs, rs)
        return self.post_layernorm(x)

    # -- forward ----------------------------------------------------------
    # Opaque to torch.compile: the grids are read on the host and the whole
    # tower is one library call (torch.ops.siglip2_b200.vision_tower is the
    # same call as a traceable op).
    @torch.compiler.disable
    def forward(self, *args, **kwargs):
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

    def forward_packed(self, seq_patches: torch.Tensor, token_grids: torch.Tensor) -> torch.Tensor:
        """``model.py:260-292``: packed rows in, ``[N, D]`` out."""
        hw = _grids(token_grids)
        if self._submodule_path(seq_patches):
            dt = self.embeddings.patch_embedding.weight.dtype
            return self._forward_rows(seq_patches.to(dt), hw)
        with torch.no_grad():
            last, _ = tower_forward(self.packed_weights(), seq_patches, hw, 0, False)
        return last

    def forward_padded(self, pixel_values, attention_mask, spatial_shapes) -> Siglip2Output:
        """HF ``Siglip2VisionTransformer.forward``: padded rows in;
        ``last_hidden_state [B, P, D]`` (zeros on padded rows) and
        ``pooler_output [B, D]`` (None without a head)."""
        hw = _grids(spatial_shapes)
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
        if self._submodule_path(pixel_values):
            dt = self.embeddings.patch_embedding.weight.dtype
            rows = torch.cat([pixel_values[b, :int(n)] for b, n in enumerate(lens)], 0).to(dt)
            x = self._forward_rows(rows, hw)
            idx = torch.cat([torch.arange(int(n)) + b * P for b, n in enumerate(lens)]).to(x.device)
            last = x.new_zeros((B * P, x.shape[-1])).index_copy(0, idx, x).view(B, P, -1)
            pooled = None
            if self.head is not None:
                mask = (torch.arange(P)[None] < torch.from_numpy(lens)[:, None]).to(torch.int64)
                pooled = self.head(last, mask)
            return Siglip2Output(last, pooled)
        with torch.no_grad():
            last, pooled = tower_forward(self.packed_weights(), pixel_values, hw, P, self.head is not None)
        return Siglip2Output(last, pooled)


class Siglip2SequenceVisionTransformerOptimized(Siglip2SequenceVisionTransformer):
    """Same module under the name of ``optimized_siglip2/model_optimized.py:341``."""


# the transformers name of the tower
Siglip2VisionTransformer = Siglip2SequenceVisionTransformer
