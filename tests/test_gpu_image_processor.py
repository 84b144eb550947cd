"""GPU image preprocessing against transformers' ``Siglip2ImageProcessor``
(torchvision backend, transformers 5.5): without a resize the fp32
``pixel_values`` are bit-identical (and their bf16 rounding too); with a
resize they agree with the processor run on CUDA (uint8 resized in fp32,
rounded half to even) except for rare one-level rounding ties; masks and
spatial shapes are identical.  The processed batch then drives the tower."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from siglip2_b200 import _lib as L  # noqa: E402
from siglip2_b200.image_processor import Siglip2ImageProcessor  # noqa: E402

hf = pytest.importorskip("transformers.models.siglip2.image_processing_siglip2")
ONE_LEVEL = 1 / 127.5


def _images(sizes, seed=0, channels=3):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, 256, (channels, H, W), dtype=torch.uint8, generator=g) for H, W in sizes]


def test_no_resize_is_bit_exact():
    sizes = [(64, 48), (16, 16), (256, 256), (32, 512), (160, 96)]
    imgs = _images(sizes, seed=1)
    ref = hf.Siglip2ImageProcessor()(images=imgs, return_tensors="pt", do_resize=False, max_num_patches=256)
    ours = Siglip2ImageProcessor(do_resize=False)(imgs, max_num_patches=256)
    assert torch.equal(ours["pixel_values"].cpu(), ref["pixel_values"])
    assert torch.equal(ours["pixel_attention_mask"].cpu(), ref["pixel_attention_mask"])
    assert torch.equal(ours["spatial_shapes"], ref["spatial_shapes"])
    bf = Siglip2ImageProcessor(do_resize=False, dtype=torch.bfloat16)(imgs, max_num_patches=256)
    assert torch.equal(bf["pixel_values"].cpu(), ref["pixel_values"].to(torch.bfloat16))
    # channels-last input, device-resident input: same result
    hwc = [im.permute(1, 2, 0).contiguous().cuda() for im in imgs]
    last = Siglip2ImageProcessor(do_resize=False)(hwc, max_num_patches=256, data_format="channels_last")
    assert torch.equal(last["pixel_values"], ours["pixel_values"])


@pytest.mark.parametrize("budget", [256, 1024])
def test_resize_matches_the_cuda_processor(budget):
    sizes = [(333, 517), (1024, 768), (50, 40), (7, 5), (1, 1), (2000, 300), (480, 640), (1500, 1500)]
    imgs = _images(sizes, seed=2)
    ref = hf.Siglip2ImageProcessor()(images=[im.cuda() for im in imgs], return_tensors="pt", device="cuda",
                                     max_num_patches=budget)
    ours = Siglip2ImageProcessor()(imgs, max_num_patches=budget)
    assert torch.equal(ours["spatial_shapes"], ref["spatial_shapes"].cpu())
    assert torch.equal(ours["pixel_attention_mask"], ref["pixel_attention_mask"].to(ours["pixel_attention_mask"]))
    d = (ours["pixel_values"] - ref["pixel_values"].to(ours["pixel_values"])).abs()
    frac = (d > 1e-6).float().mean().item()
    print(f"\n[parity] resize budget {budget}: max diff {d.max().item():.6f}, fraction differing {frac:.2e}")
    assert d.max().item() <= ONE_LEVEL + 1e-6 and frac < 1e-3


def test_channels_last_and_device_inputs_agree_with_resize():
    imgs = _images([(300, 200), (90, 700)], seed=3)
    a = Siglip2ImageProcessor()(imgs)
    b = Siglip2ImageProcessor()([im.permute(1, 2, 0).contiguous().cuda() for im in imgs], data_format="channels_last")
    assert torch.equal(a["pixel_values"], b["pixel_values"])


def test_downscale_limit_is_an_error():
    with pytest.raises(L.Siglip2Error, match="downscaled"):
        Siglip2ImageProcessor()(_images([(4000, 4000)]), max_num_patches=16)


def test_processed_batch_drives_the_tower():
    from siglip2_b200 import Siglip2SequenceVisionTransformer, Siglip2VisionConfig
    from siglip2_b200 import workloads as W
    cfg = W.preset_config("b16", config_cls=Siglip2VisionConfig, num_hidden_layers=2)
    m = Siglip2SequenceVisionTransformer(cfg)
    m.load_state_dict(W.init_state_dict(cfg, seed=4, with_head=True))
    m = m.to("cuda", torch.bfloat16).eval()
    imgs = _images([(333, 517), (64, 64), (1000, 200)], seed=4)
    ours = Siglip2ImageProcessor(dtype=torch.bfloat16)(imgs, max_num_patches=256)
    ref = hf.Siglip2ImageProcessor()(images=[im.cuda() for im in imgs], return_tensors="pt", device="cuda")
    with torch.inference_mode():
        a = m(ours["pixel_values"], ours["pixel_attention_mask"], ours["spatial_shapes"])
        b = m(ref["pixel_values"].to(torch.bfloat16), ref["pixel_attention_mask"], ref["spatial_shapes"])
    cos = torch.nn.functional.cosine_similarity(a.pooler_output.float(), b.pooler_output.float(), dim=1)
    assert cos.min().item() > 0.9999


@pytest.mark.parametrize("do_resize", [False, True])
def test_general_kernel_patch8(do_resize):
    """Shapes other than 3 channels x 16 x 16 run the general kernel."""
    sizes = [(64, 48), (40, 120)] if not do_resize else [(333, 517), (50, 40), (900, 128)]
    imgs = _images(sizes, seed=5)
    ref = hf.Siglip2ImageProcessor(patch_size=8)(images=[im.cuda() for im in imgs], return_tensors="pt",
                                                 device="cuda", do_resize=do_resize, max_num_patches=300)
    ours = Siglip2ImageProcessor(patch_size=8, do_resize=do_resize)(imgs, max_num_patches=300)
    assert torch.equal(ours["spatial_shapes"], ref["spatial_shapes"].cpu())
    d = (ours["pixel_values"] - ref["pixel_values"].to(ours["pixel_values"])).abs()
    if not do_resize:
        assert d.max().item() == 0
    assert d.max().item() <= ONE_LEVEL + 1e-6 and (d > 1e-6).float().mean().item() < 1e-3
