"""Seeded synthetic workloads: model presets, NaFlex grid samplers, pixels and
random-init weights for the five benchmark configurations of the SigLIP-2
NaFlex vision tower.

No datasets or checkpoints are used anywhere: pixels are uniform in [-1, 1]
(valid rows) and zero (padded rows); weights are truncated-normal with
std 0.02 (bounds +-2 std), biases 0, LayerNorm gamma 1 / beta 0, seed 1337.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

# name -> (hidden, intermediate, layers, heads)
PRESETS = {
    "b16": (768, 3072, 12, 12),
    "so400m": (1152, 4304, 27, 16),
    "l16": (1024, 4096, 24, 16),
    "g16": (1536, 6144, 40, 16),
}


@dataclass
class Workload:
    """One benchmark configuration: model preset, dtype, images, max patches."""

    name: str
    preset: str
    dtype: torch.dtype
    batch: int
    max_patches: int
    sampler: str
    overrides: dict = field(default_factory=dict)


WORKLOADS = {
    # B/16 fp32, 8 images, P=256, h,w in [4,32] with h*w <= 256
    "cfg0": Workload("cfg0-b16-fp32-8x256", "b16", torch.float32, 8, 256, "uniform_hw"),
    # B/16 bf16, 64-image mini-batches of full 16x16 grids
    "cfg1": Workload("cfg1-b16-bf16-64x256-full", "b16", torch.bfloat16, 64, 256, "full"),
    # So400m bf16, 64 images, P=1024, area U[256,1024], aspect log-U[1/4,4]
    "cfg2": Workload("cfg2-so400m-bf16-64x1024-naflex", "so400m", torch.bfloat16, 64, 1024, "area_aspect"),
    # L/16 fp16, 256 images, P=576, area U[64,576], both orientations
    "cfg3": Workload("cfg3-l16-fp16-256x576-naflex", "l16", torch.float16, 256, 576, "area_aspect"),
    # g/16 bf16, 512 images per GPU, P=1024, distribution as cfg2
    "cfg4": Workload("cfg4-g16-bf16-512x1024-naflex", "g16", torch.bfloat16, 512, 1024, "area_aspect"),
}


def preset_config(preset: str, config_cls=None, **overrides):
    """Build a ``Siglip2VisionConfig`` (``model.py:39-49`` fields) for a preset."""
    if config_cls is None:
        from .model import Siglip2VisionConfig as config_cls
    d, i, l, h = PRESETS[preset]
    kw = dict(hidden_size=d, intermediate_size=i, num_hidden_layers=l, num_attention_heads=h,
              attention_dropout=0.0)
    kw.update(overrides)
    return config_cls(**kw)


def sample_spatial_shapes(sampler: str, batch: int, max_patches: int, seed: int = 1337) -> torch.Tensor:
    """``[B, 2]`` int64 (h, w) grids with ``h*w <= max_patches``.

    * ``uniform_hw``: h, w ~ U{4..32}, redrawn until ``h*w <= P``.
    * ``full``: every image is the full ``sqrt(P) x sqrt(P)`` grid.
    * ``area_aspect``: area A ~ U[P/4, P] (U[64, 576] for P=576 is the same
      rule with A >= 64), aspect r = exp(U[-ln 4, ln 4]);
      ``h = clamp(round(sqrt(A r)), 1, P)``,
      ``w = clamp(round(A / h), 1, floor(P / h))``.  Both orientations occur.
    """
    g = torch.Generator().manual_seed(seed)
    out = []
    if sampler == "full":
        s = int(math.isqrt(max_patches))
        return torch.full((batch, 2), s, dtype=torch.int64)
    for _ in range(batch):
        if sampler == "uniform_hw":
            while True:
                h = int(torch.randint(4, 33, (1,), generator=g))
                w = int(torch.randint(4, 33, (1,), generator=g))
                if h * w <= max_patches:
                    break
        elif sampler == "area_aspect":
            lo = 64 if max_patches == 576 else max_patches // 4
            a = lo + (max_patches - lo) * float(torch.rand((), generator=g))
            r = math.exp(math.log(4.0) * (2.0 * float(torch.rand((), generator=g)) - 1.0))
            h = min(max(int(round(math.sqrt(a * r))), 1), max_patches)
            w = min(max(int(round(a / h)), 1), max_patches // h)
        else:
            raise ValueError(f"unknown sampler {sampler!r}")
        out.append((h, w))
    return torch.tensor(out, dtype=torch.int64)


def make_pixels(spatial_shapes: torch.Tensor, max_patches: int, patch_dim: int, seed: int = 1337,
                dtype=torch.float32):
    """Padded NaFlex inputs: ``pixel_values [B, P, patch_dim]`` uniform in
    [-1, 1] on valid rows and 0 on padded rows; ``attention_mask [B, P]`` int32
    with 1 on the first ``h*w`` rows."""
    g = torch.Generator().manual_seed(seed + 1)
    B = spatial_shapes.shape[0]
    pv = torch.rand((B, max_patches, patch_dim), generator=g) * 2.0 - 1.0
    lens = (spatial_shapes[:, 0] * spatial_shapes[:, 1])
    ar = torch.arange(max_patches)[None, :]
    mask = (ar < lens[:, None]).to(torch.int32)
    pv = pv * mask[..., None]
    return pv.to(dtype), mask


def make_pixels_indexed(spatial_shapes: torch.Tensor, image_ids, max_patches: int, patch_dim: int,
                        seed: int = 1337, dtype=torch.float32):
    """As ``make_pixels``, but image ``i`` of a global batch draws its rows
    from a generator of its own (seeded by ``seed`` and its global index
    ``image_ids[k]``), so any subset of the batch, e.g. one rank's shard,
    gets exactly the pixels it has in the whole batch."""
    B = spatial_shapes.shape[0]
    assert len(image_ids) == B
    pv = torch.zeros((B, max_patches, patch_dim), dtype=dtype)
    mask = torch.zeros((B, max_patches), dtype=torch.int32)
    for k, i in enumerate(image_ids):
        L = int(spatial_shapes[k, 0] * spatial_shapes[k, 1])
        g = torch.Generator().manual_seed((seed + 1) * 1_000_003 + int(i))
        pv[k, :L] = (torch.rand((L, patch_dim), generator=g) * 2.0 - 1.0).to(dtype)
        mask[k, :L] = 1
    return pv, mask


def pack_rows(pixel_values: torch.Tensor, spatial_shapes: torch.Tensor) -> torch.Tensor:
    """Padded ``[B, P, C]`` -> packed ``[sum h*w, C]`` (valid rows only)."""
    lens = (spatial_shapes[:, 0] * spatial_shapes[:, 1]).tolist()
    return torch.cat([pixel_values[b, :L] for b, L in enumerate(lens)], dim=0)


def init_state_dict(cfg, seed: int = 1337, with_head: bool = True, random_affine: bool = False,
                    dtype=torch.float32) -> dict:
    """Reference-named weights (``model.py`` state_dict keys, plus HF
    ``head.*``): truncated normal std 0.02 (+-2 std) for every matrix, the
    position table and the probe; biases 0; LayerNorm gamma 1 / beta 0.

    ``random_affine=True`` instead draws biases and LayerNorm beta ~ N(0, 0.02)
    and gamma ~ 1 + N(0, 0.1) so that tests exercise every affine term."""
    g = torch.Generator().manual_seed(seed)
    D, I = cfg.hidden_size, cfg.intermediate_size
    cin = cfg.num_channels * cfg.patch_size * cfg.patch_size
    sd = {}

    def mat(*shape):
        t = torch.empty(shape)
        torch.nn.init.trunc_normal_(t, std=0.02, a=-0.04, b=0.04, generator=g)
        return t

    def bias(n):
        return torch.randn(n, generator=g) * 0.02 if random_affine else torch.zeros(n)

    def gamma(n):
        return 1.0 + torch.randn(n, generator=g) * 0.1 if random_affine else torch.ones(n)

    sd["embeddings.patch_embedding.weight"] = mat(D, cin)
    sd["embeddings.patch_embedding.bias"] = bias(D)
    sd["embeddings.position_embedding.weight"] = mat(cfg.num_patches, D)
    for i in range(cfg.num_hidden_layers):
        p = f"encoder.layers.{i}."
        for n in ("k_proj", "v_proj", "q_proj", "out_proj"):
            sd[p + f"self_attn.{n}.weight"] = mat(D, D)
            sd[p + f"self_attn.{n}.bias"] = bias(D)
        sd[p + "layer_norm1.weight"] = gamma(D)
        sd[p + "layer_norm1.bias"] = bias(D)
        sd[p + "mlp.fc1.weight"] = mat(I, D)
        sd[p + "mlp.fc1.bias"] = bias(I)
        sd[p + "mlp.fc2.weight"] = mat(D, I)
        sd[p + "mlp.fc2.bias"] = bias(D)
        sd[p + "layer_norm2.weight"] = gamma(D)
        sd[p + "layer_norm2.bias"] = bias(D)
    sd["post_layernorm.weight"] = gamma(D)
    sd["post_layernorm.bias"] = bias(D)
    if with_head:
        sd["head.probe"] = mat(1, 1, D)
        sd["head.attention.in_proj_weight"] = mat(3 * D, D)
        sd["head.attention.in_proj_bias"] = bias(3 * D)
        sd["head.attention.out_proj.weight"] = mat(D, D)
        sd["head.attention.out_proj.bias"] = bias(D)
        sd["head.layernorm.weight"] = gamma(D)
        sd["head.layernorm.bias"] = bias(D)
        sd["head.mlp.fc1.weight"] = mat(I, D)
        sd["head.mlp.fc1.bias"] = bias(I)
        sd["head.mlp.fc2.weight"] = mat(D, I)
        sd["head.mlp.fc2.bias"] = bias(D)
    return {k: v.to(dtype) for k, v in sd.items()}
