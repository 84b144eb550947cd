"""Write the golden fixtures that pin the numpy oracle to the reference.

Run once, in a container that has the reference checkout and transformers:

    python tests/golden/make_golden.py <path to the tohskai/SigLIP-2 checkout>

It imports the reference's own ``model.py`` (tohskai/SigLIP-2) on the CPU in
fp32 and runs its packed forward (``model.py:260-292``).  Two adjustments are
needed for a CPU-only host and are applied from outside, without editing the
reference: ``create_block_mask`` is rebound with ``device="cpu"`` (the
reference hard-wires the default CUDA device at ``model.py:159-161``) and
TorchDynamo is disabled so that ``torch.compile(create_block_mask)`` runs
eagerly.  The attention-pooling head and the padded entry come from the
third-party ``transformers`` ``Siglip2VisionTransformer`` (the reference has
no head), loaded with the same weights plus ``head.*``.

Fixtures written next to this script:

* ``tiny_mixed.npz``  -- a small tower (patch 4, hidden 64, 2 heads,
  2 layers) with random affine terms, grids that both down- and up-sample the
  16x16 position table; all weights, inputs and full outputs are stored.
* ``b16_cfg0.npz``    -- the B/16 fp32 workload (8 images, P=256,
  h,w in [4,32], seed 1337) at full size.  Weights are regenerated from the
  seed by ``siglip2_b200.workloads.init_state_dict``; the fixture keeps the
  grids, every 4th output row, per-image row sums and the pooled output.
"""
from __future__ import annotations

import functools
import os
import sys

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from siglip2_b200 import workloads as W  # noqa: E402


def load_reference(ref_root: str):
    sys.path.insert(0, ref_root)
    import model as ref_model  # the reference's own model.py
    from torch.nn.attention.flex_attention import create_block_mask

    ref_model.create_block_mask = functools.partial(create_block_mask, device="cpu")
    return ref_model


def hf_tower(cfg, sd):
    from transformers.models.siglip2.configuration_siglip2 import Siglip2VisionConfig as HFCfg
    from transformers.models.siglip2.modeling_siglip2 import Siglip2VisionTransformer as HFTower

    hcfg = HFCfg(hidden_size=cfg.hidden_size, intermediate_size=cfg.intermediate_size,
                 num_hidden_layers=cfg.num_hidden_layers, num_attention_heads=cfg.num_attention_heads,
                 num_channels=cfg.num_channels, patch_size=cfg.patch_size,
                 layer_norm_eps=cfg.layer_norm_eps, num_patches=cfg.num_patches, attention_dropout=0.0)
    hcfg._attn_implementation = "eager"
    m = HFTower(hcfg).eval()
    missing, unexpected = m.load_state_dict(sd, strict=True), None
    return m


def run_case(ref_model, cfg_kwargs, grids, seed, random_affine, max_patches=None):
    cfg = ref_model.Siglip2VisionConfig(**cfg_kwargs)
    sd = W.init_state_dict(cfg, seed=seed, with_head=True, random_affine=random_affine)
    tower = ref_model.Siglip2SequenceVisionTransformer(cfg).eval()
    tower.load_state_dict({k: v for k, v in sd.items() if not k.startswith("head.")}, strict=True)
    grids_t = torch.tensor(grids, dtype=torch.int64)
    lens = (grids_t[:, 0] * grids_t[:, 1]).tolist()
    P = max_patches or max(lens)
    cin = cfg.num_channels * cfg.patch_size ** 2
    pv, mask = W.make_pixels(grids_t, P, cin, seed=seed)
    packed = W.pack_rows(pv, grids_t)
    with torch.no_grad():
        last = tower((packed, grids_t)).float()
        hf = hf_tower(cfg, sd)
        out = hf(pixel_values=pv, attention_mask=mask, spatial_shapes=grids_t)
    hf_last = out.last_hidden_state
    hf_valid = torch.cat([hf_last[b, :L] for b, L in enumerate(lens)], 0)
    print(f"  model.py vs transformers on valid rows: max-abs {(hf_valid - last).abs().max().item():.3e}")
    return cfg, sd, grids_t, pv, mask, packed, last, out.pooler_output.float()


def main(ref_root: str):
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ref_model = load_reference(ref_root)

    print("tiny_mixed")
    kw = dict(hidden_size=64, intermediate_size=96, num_hidden_layers=2, num_attention_heads=2,
              num_channels=3, patch_size=4, layer_norm_eps=1e-6, attention_dropout=0.0, num_patches=256)
    grids = [(3, 5), (16, 16), (20, 7), (1, 1), (8, 12), (5, 33), (24, 24)]
    cfg, sd, g, pv, mask, packed, last, pooled = run_case(ref_model, kw, grids, 7, True)
    np.savez_compressed(
        os.path.join(HERE, "tiny_mixed.npz"),
        cfg=np.array([kw["hidden_size"], kw["intermediate_size"], kw["num_hidden_layers"],
                      kw["num_attention_heads"], kw["num_channels"], kw["patch_size"], kw["num_patches"]]),
        grids=g.numpy(), packed=packed.numpy(),
        last_hidden_state=last.numpy(), pooler_output=pooled.numpy(),
        **{"w/" + k: v.numpy() for k, v in sd.items()})

    print("b16_cfg0")
    wl = W.WORKLOADS["cfg0"]
    cfg0 = W.preset_config("b16", config_cls=ref_model.Siglip2VisionConfig)
    grids0 = W.sample_spatial_shapes(wl.sampler, wl.batch, wl.max_patches, seed=1337)
    kw0 = {k: getattr(cfg0, k) for k in ("hidden_size", "intermediate_size", "num_hidden_layers",
                                         "num_attention_heads", "num_channels", "patch_size",
                                         "layer_norm_eps", "attention_dropout", "num_patches")}
    cfg, sd, g, pv, mask, packed, last, pooled = run_case(ref_model, kw0, grids0.tolist(), 1337, False,
                                                                  max_patches=wl.max_patches)
    lens = (g[:, 0] * g[:, 1]).tolist()
    starts = np.cumsum([0] + lens[:-1])
    rowsums = np.stack([last[s:s + L].sum(0).numpy() for s, L in zip(starts, lens)])
    np.savez_compressed(
        os.path.join(HERE, "b16_cfg0.npz"), grids=g.numpy(), rows_every4=last[::4].numpy(),
        image_rowsums=rowsums, pooler_output=pooled.numpy(),
        pixel_checksum=np.array([float(pv.double().sum())]))
    print("done")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to a tohskai/SigLIP-2 checkout>")
    main(sys.argv[1])
