"""fp32 path (the reference's CPU-runnable configuration): the tower on the
GPU in fp32 against the reference's own outputs (golden fixture written from
model.py + transformers) and against the numpy oracle, at 1e-4 max-abs."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from oracle import siglip2_oracle as O  # noqa: E402
from siglip2_b200 import Siglip2SequenceVisionTransformer, Siglip2VisionConfig  # noqa: E402
from siglip2_b200 import workloads as W  # noqa: E402


def test_cfg0_fp32_matches_reference_outputs(golden_dir):
    z = np.load(os.path.join(golden_dir, "b16_cfg0.npz"))
    wl = W.WORKLOADS["cfg0"]
    cfg = W.preset_config("b16", config_cls=Siglip2VisionConfig)
    grids = W.sample_spatial_shapes(wl.sampler, wl.batch, wl.max_patches, seed=1337)
    sd = W.init_state_dict(cfg, seed=1337, with_head=True)
    m = Siglip2SequenceVisionTransformer(cfg)
    m.load_state_dict(sd)
    m = m.cuda().float().eval()
    pv, mask = W.make_pixels(grids, wl.max_patches, 768, seed=1337)
    with torch.inference_mode():
        out = m(pv.cuda(), mask, grids)
    torch.cuda.synchronize()
    lens = (grids[:, 0] * grids[:, 1]).tolist()
    valid = torch.cat([out.last_hidden_state[b, :L] for b, L in enumerate(lens)], 0).cpu().numpy()
    err = np.abs(valid[::4] - z["rows_every4"]).max()
    perr = np.abs(out.pooler_output.cpu().numpy() - z["pooler_output"]).max()
    print(f"\n[parity] cfg0 fp32 vs reference: last_hidden max-abs {err:.2e}, pooler max-abs {perr:.2e}")
    assert err < 1e-4, err
    assert perr < 1e-4, perr
    for b, L in enumerate(lens):
        assert not out.last_hidden_state[b, L:].any()


@pytest.mark.parametrize("preset,layers", [("b16", 2), ("so400m", 1), ("g16", 1)])
def test_fp32_tower_vs_oracle_random_affine(preset, layers):
    cfg = W.preset_config(preset, config_cls=Siglip2VisionConfig, num_hidden_layers=layers)
    sd = W.init_state_dict(cfg, seed=5, with_head=True, random_affine=True)
    m = Siglip2SequenceVisionTransformer(cfg)
    m.load_state_dict(sd)
    m = m.cuda().float().eval()
    grids = torch.tensor([(21, 8), (3, 5), (16, 16), (1, 1), (30, 9)])
    P = 300
    pv, mask = W.make_pixels(grids, P, 768, seed=5)
    with torch.inference_mode():
        out = m(pv.cuda(), mask, grids)
    torch.cuda.synchronize()
    last, pooled = O.forward_padded({k: v.numpy() for k, v in sd.items()}, O.OracleConfig(**cfg.__dict__),
                                    pv.numpy(), mask.numpy(), grids.numpy(), dt=np.float64)
    assert np.abs(out.last_hidden_state.cpu().numpy() - last).max() < 1e-4
    assert np.abs(out.pooler_output.cpu().numpy() - pooled).max() < 1e-4
