"""The numpy oracle against the reference's own outputs (golden fixtures
written by ``tests/golden/make_golden.py`` from ``model.py`` and
``transformers``), and its antialiased resize against ATen directly."""
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import siglip2_oracle as O
from siglip2_b200 import workloads as W


def _tiny(golden_dir):
    z = np.load(os.path.join(golden_dir, "tiny_mixed.npz"))
    d, i, l, h, c, p, npch = [int(v) for v in z["cfg"]]
    cfg = O.OracleConfig(hidden_size=d, intermediate_size=i, num_hidden_layers=l, num_attention_heads=h,
                         num_channels=c, patch_size=p, num_patches=npch)
    params = {k[2:]: z[k] for k in z.files if k.startswith("w/")}
    return z, cfg, params


def test_aa_weights_match_aten():
    """Every (h, w) the workloads can produce except the w == 1 column path
    (no workload draws a side of 1 except the 1x1 grid)."""
    g = torch.randn(1, 5, 16, 16, dtype=torch.float64)
    for h in list(range(1, 40)) + [64, 100]:
        for w in (2, 3, 5, 8, 13, 16, 17, 31, 32, 33, 64):
            ref = F.interpolate(g, size=(h, w), mode="bilinear", align_corners=False, antialias=True)
            wy, wx = O.aa_bilinear_weights(16, h), O.aa_bilinear_weights(16, w)
            ours = np.einsum("ya,xb,cab->cyx", wy, wx, g[0].numpy())
            assert np.abs(ours - ref[0].numpy()).max() < 1e-12, (h, w)
    ref = F.interpolate(g, size=(1, 1), mode="bilinear", align_corners=False, antialias=True)
    ours = np.einsum("ya,xb,cab->cyx", O.aa_bilinear_weights(16, 1), O.aa_bilinear_weights(16, 1), g[0].numpy())
    assert np.abs(ours - ref[0].numpy()).max() < 1e-12


def test_oracle_tiny_matches_reference(golden_dir):
    z, cfg, params = _tiny(golden_dir)
    out = O.forward_packed(params, cfg, z["packed"], z["grids"], dt=np.float64)
    err = np.abs(out - z["last_hidden_state"]).max()
    assert err < 2e-5, err


def test_oracle_tiny_head_matches_transformers(golden_dir):
    z, cfg, params = _tiny(golden_dir)
    grids = z["grids"]
    lens = (grids[:, 0] * grids[:, 1]).tolist()
    P = max(lens)
    pv = np.zeros((len(lens), P, z["packed"].shape[1]), np.float64)
    mask = np.zeros((len(lens), P), np.int32)
    s = 0
    for b, L in enumerate(lens):
        pv[b, :L] = z["packed"][s:s + L]
        mask[b, :L] = 1
        s += L
    last, pooled = O.forward_padded(params, cfg, pv, mask, grids, dt=np.float64)
    assert np.abs(pooled - z["pooler_output"]).max() < 2e-5
    valid = np.concatenate([last[b, :L] for b, L in enumerate(lens)], 0)
    assert np.abs(valid - z["last_hidden_state"]).max() < 2e-5
    for b, L in enumerate(lens):
        assert not last[b, L:].any()


@pytest.mark.slow
def test_oracle_b16_cfg0_matches_reference(golden_dir):
    z = np.load(os.path.join(golden_dir, "b16_cfg0.npz"))
    wl = W.WORKLOADS["cfg0"]
    cfg = W.preset_config("b16", config_cls=O.OracleConfig)
    grids = W.sample_spatial_shapes(wl.sampler, wl.batch, wl.max_patches, seed=1337)
    assert (grids.numpy() == z["grids"]).all()
    sd = {k: v.numpy() for k, v in W.init_state_dict(cfg, seed=1337, with_head=True).items()}
    pv, mask = W.make_pixels(grids, wl.max_patches, 768, seed=1337)
    assert abs(float(pv.double().sum()) - z["pixel_checksum"][0]) < 1e-6
    last, pooled = O.forward_padded(sd, cfg, pv.numpy(), mask.numpy(), grids.numpy(), dt=np.float32)
    lens = (grids[:, 0] * grids[:, 1]).tolist()
    valid = np.concatenate([last[b, :L] for b, L in enumerate(lens)], 0)
    assert np.abs(valid[::4] - z["rows_every4"]).max() < 1e-4
    sums = np.stack([last[b, :L].sum(0) for b, L in enumerate(lens)])
    assert np.abs(sums - z["image_rowsums"]).max() < 1e-3
    assert np.abs(pooled - z["pooler_output"]).max() < 1e-4


def test_flop_model():
    cfg = W.preset_config("so400m", config_cls=O.OracleConfig)
    assert abs(O.flops_per_image(cfg, 256) / 1e9 - 220.5) < 0.5
    assert abs(O.flops_per_image(cfg, 1024) / 1e9 - 979.6) < 0.5
    cfg = W.preset_config("b16", config_cls=O.OracleConfig)
    assert abs(O.flops_per_image(cfg, 256) / 1e9 - 46.8) < 0.2


def test_philox_known_answers():
    """The oracle's Philox4x32-10 against the generator's published
    known-answer vectors (counter, key -> output)."""
    kat = [((0, 0, 0, 0), (0, 0), (0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8)),
           ((0xffffffff,) * 4, (0xffffffff, 0xffffffff), (0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd)),
           ((0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344), (0xa4093822, 0x299f31d0),
            (0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1))]
    for ctr, key, want in kat:
        got = O.philox4x32_10(np.array([ctr], dtype=np.uint32), key)[0]
        assert tuple(int(v) for v in got) == want


def test_dropout_keep_rate_and_streams():
    keep = O.dropout_keep(seed=0x1234_5678_9abc, offset=0, first=0, count=1 << 20, p=0.1)
    rate = keep.mean()
    assert abs(rate - 0.9) < 5 * (0.9 * 0.1 / keep.size) ** 0.5, rate
    other = O.dropout_keep(seed=0x1234_5678_9abc, offset=1, first=0, count=1 << 20, p=0.1)
    assert (keep != other).mean() > 0.1  # another offset is another stream
    tail = O.dropout_keep(seed=0x1234_5678_9abc, offset=0, first=1000, count=500, p=0.1)
    assert np.array_equal(tail, keep[1000:1500])  # a pure function of the element index
    assert O.dropout_keep(seed=7, offset=0, first=0, count=4096, p=0.0).all()
