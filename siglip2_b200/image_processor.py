"""Image preprocessing in front of the tower, on the GPU.

``Siglip2ImageProcessor`` has the interface and the results of transformers'
``Siglip2ImageProcessor`` (torchvision backend,
``models/siglip2/image_processing_siglip2.py``): each uint8 image is resized
to the largest patch grid within ``max_num_patches`` (antialiased bilinear,
rounded back to uint8), normalised with the rescale factor folded into
mean / std, cut into patches flattened as (py, px, channel), and padded to
``max_num_patches`` rows with a mask.  Grid sizes come from
``siglip2_image_grid`` (the same binary search, on the host); the pixels go
to the device in one copy and through one ``siglip2_patchify`` launch.  The
resize follows torchvision's resize of a uint8 CUDA tensor (interpolate in
fp32, round half to even); transformers' CPU path uses a fixed-point uint8
kernel instead, which can differ by one level.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib as L
from .ops import dtype_code


def image_grid(height: int, width: int, patch_size: int, max_num_patches: int) -> tuple[int, int]:
    """``siglip2_image_grid``: the (h, w) patch grid of a height x width image."""
    h, w = ctypes.c_int(), ctypes.c_int()
    L.call("siglip2_image_grid", int(height), int(width), int(patch_size), int(max_num_patches), ctypes.byref(h),
           ctypes.byref(w))
    return h.value, w.value


class Siglip2ImageProcessor:
    """Batch preprocessing to ``pixel_values [B, max_num_patches, p*p*C]``,
    ``pixel_attention_mask [B, max_num_patches]`` (int32) and
    ``spatial_shapes [B, 2]`` (int64), the inputs of the tower's padded
    forward.  Images are uint8 tensors (host or device), ``[C, H, W]``
    (``data_format="channels_first"``, as transformers' torch path) or
    ``[H, W, C]`` (``"channels_last"``, as decoded images usually are)."""

    model_input_names = ["pixel_values", "pixel_attention_mask", "spatial_shapes"]

    def __init__(self, patch_size: int = 16, max_num_patches: int = 256, image_mean=(0.5, 0.5, 0.5),
                 image_std=(0.5, 0.5, 0.5), rescale_factor: float = 1 / 255, do_resize: bool = True,
                 device="cuda", dtype: torch.dtype = torch.float32):
        self.patch_size = patch_size
        self.max_num_patches = max_num_patches
        self.image_mean = list(image_mean)
        self.image_std = list(image_std)
        self.rescale_factor = rescale_factor
        self.do_resize = do_resize
        self.device = torch.device(device)
        self.dtype = dtype

    def _mean_std(self, channels: int):
        # transformers folds the rescale into the normalisation in float32:
        # tensor(mean) * (1 / rescale_factor), likewise std
        k = np.float32(1.0 / self.rescale_factor)
        mean = np.broadcast_to(np.asarray(self.image_mean, dtype=np.float32), (channels,)) * k
        std = np.broadcast_to(np.asarray(self.image_std, dtype=np.float32), (channels,)) * k
        return np.ascontiguousarray(mean, dtype=np.float32), np.ascontiguousarray(std, dtype=np.float32)

    def __call__(self, images, max_num_patches: int | None = None, data_format: str = "channels_first",
                 dtype: torch.dtype | None = None, device=None) -> dict:
        return self.preprocess(images, max_num_patches, data_format, dtype, device)

    def preprocess(self, images, max_num_patches: int | None = None, data_format: str = "channels_first",
                   dtype: torch.dtype | None = None, device=None) -> dict:
        if isinstance(images, torch.Tensor) and images.dim() == 3:
            images = [images]
        images = list(images)
        if not images:
            raise ValueError("no images")
        P = int(max_num_patches or self.max_num_patches)
        p = self.patch_size
        dt = dtype or self.dtype
        dev = torch.device(device) if device is not None else self.device
        if dev.type != "cuda":
            raise RuntimeError("siglip2_b200 preprocessing runs on CUDA only")
        if data_format not in ("channels_first", "channels_last"):
            raise ValueError("data_format must be 'channels_first' or 'channels_last'")
        last = data_format == "channels_last"
        B = len(images)
        src_hw = np.zeros((B, 2), dtype=np.int32)
        grid_hw = np.zeros((B, 2), dtype=np.int32)
        C = None
        for b, im in enumerate(images):
            if not isinstance(im, torch.Tensor) or im.dtype != torch.uint8 or im.dim() != 3:
                raise TypeError("images must be 3-D uint8 tensors")
            c, H, W = (im.shape[2], im.shape[0], im.shape[1]) if last else tuple(im.shape)
            if C is None:
                C = int(c)
            elif c != C:
                raise ValueError("all images need the same number of channels")
            src_hw[b] = (H, W)
            if self.do_resize:
                grid_hw[b] = image_grid(H, W, p, P)
            else:
                if H % p or W % p or (H // p) * (W // p) > P:
                    raise ValueError(f"image {b} ({H}x{W}) is not a patch multiple within {P} patches")
                grid_hw[b] = (H // p, W // p)
        sizes = [im.numel() for im in images]
        offsets = np.zeros(B, dtype=np.int64)
        np.cumsum(sizes[:-1], out=offsets[1:])
        flat = [im.contiguous().reshape(-1) for im in images]
        if all(im.is_cuda for im in images):
            pixels = torch.cat([f.to(dev) for f in flat])
        else:
            host = torch.empty(sum(sizes), dtype=torch.uint8, pin_memory=True)
            torch.cat([f.cpu() for f in flat], out=host)
            pixels = host.to(dev, non_blocking=True)
        meta_host = torch.from_numpy(np.concatenate([offsets.view(np.int32), src_hw.reshape(-1),
                                                     grid_hw.reshape(-1)]).astype(np.int32))
        meta = meta_host.to(dev)
        offs_dev = meta[:2 * B]                 # int64 offsets as int32 pairs (8-byte aligned)
        src_dev = meta[2 * B:4 * B]
        grid_dev = meta[4 * B:6 * B]
        out = torch.empty((B, P, p * p * C), dtype=dt, device=dev)
        mask = torch.empty((B, P), dtype=torch.int32, device=dev)
        mean, std = self._mean_std(C)
        stream = torch.cuda.current_stream(dev).cuda_stream
        with torch.cuda.device(dev):
            L.call("siglip2_patchify", dtype_code(dt), pixels.data_ptr(), offs_dev.data_ptr(), src_hw.ctypes.data,
                   src_dev.data_ptr(), grid_hw.ctypes.data, grid_dev.data_ptr(), B, C, p, int(last),
                   mean.ctypes.data, std.ctypes.data, P, out.data_ptr(), mask.data_ptr(), stream)
        # the host buffers must outlive the copy and the launch
        self._keep = (pixels, meta_host, meta)
        return {"pixel_values": out, "pixel_attention_mask": mask,
                "spatial_shapes": torch.from_numpy(grid_hw.astype(np.int64))}
