"""Host side of the GPU image preprocessing: the patch grid of an image
under a patch budget (``siglip2_image_grid``) equals transformers'
``get_image_size_for_max_num_patches`` (``models/siglip2/image_processing_siglip2.py``,
transformers 5.5), and the processor's argument checks."""
import random

import pytest
import torch

from siglip2_b200 import _lib as L
from siglip2_b200.image_processor import Siglip2ImageProcessor, image_grid

hf = pytest.importorskip("transformers.models.siglip2.image_processing_siglip2")


@pytest.mark.parametrize("patch,budget", [(16, 256), (16, 1024), (14, 729), (16, 64), (16, 4096)])
def test_image_grid_matches_transformers(patch, budget):
    rnd = random.Random(patch * 10007 + budget)
    sizes = [(1, 1), (16, 16), (15, 17), (4000, 16), (16, 4000), (256, 256), (512, 512), (1024, 768), (3, 5000)]
    sizes += [(rnd.randint(1, 4096), rnd.randint(1, 4096)) for _ in range(400)]
    for H, W in sizes:
        th, tw = hf.get_image_size_for_max_num_patches(H, W, patch, budget)
        assert image_grid(H, W, patch, budget) == (th // patch, tw // patch), (H, W)


def test_image_grid_rejects_bad_sizes():
    with pytest.raises(L.Siglip2Error):
        image_grid(0, 10, 16, 256)
    with pytest.raises(L.Siglip2Error):
        image_grid(10, 10, 16, 0)


def test_processor_argument_checks():
    proc = Siglip2ImageProcessor()
    with pytest.raises(TypeError):
        proc([torch.zeros(3, 32, 32)], device="cuda")            # not uint8
    with pytest.raises(RuntimeError, match="CUDA"):
        proc([torch.zeros(3, 32, 32, dtype=torch.uint8)], device="cpu")
    with pytest.raises(ValueError):
        proc([torch.zeros(3, 32, 32, dtype=torch.uint8)], data_format="nhwc")
    with pytest.raises(ValueError):
        proc([torch.zeros(3, 32, 32, dtype=torch.uint8), torch.zeros(1, 32, 32, dtype=torch.uint8)])
    with pytest.raises(ValueError):
        Siglip2ImageProcessor(do_resize=False)([torch.zeros(3, 30, 32, dtype=torch.uint8)])
