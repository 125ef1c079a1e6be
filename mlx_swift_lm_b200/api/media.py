"""Image / video inputs for vision-language models.

Parity: MLXVLM/MediaProcessing.swift:11 and the Qwen VL processor helpers
(MLXVLM/Models/QwenVL.swift - ``targetSize`` :162 smart resize to multiples
of patch * merge within [min_pixels, max_pixels], ``patchify`` :251 with
temporal padding, and the ``<|vision_start|><|image_pad|>...<|vision_end|>``
placeholder expansion of the Qwen2-VL processor). Pixels are normalised with
the CLIP mean / std the Qwen VL processors use.

Inputs are numpy / torch arrays [H, W, 3] (uint8 or float in [0, 1]), PIL
images, or file paths (decoded with PIL). Videos are lists of frames.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

CLIP_MEAN = (0.48145466, 0.4578275, 0.40821073)
CLIP_STD = (0.26862954, 0.26130258, 0.27577711)


@dataclass
class MediaConfig:
    patch_size: int = 14
    temporal_patch_size: int = 2
    merge_size: int = 2
    min_pixels: int = 56 * 56
    max_pixels: int = 28 * 28 * 1280
    mean: tuple = CLIP_MEAN
    std: tuple = CLIP_STD


def target_size(height: int, width: int, factor: int, min_pixels: int, max_pixels: int) -> tuple[int, int]:
    """Round both sides to multiples of `factor`, then rescale (keeping the
    aspect ratio) into [min_pixels, max_pixels]."""
    if height < factor or width < factor:
        raise ValueError(f"image {width}x{height} is smaller than the {factor}-pixel patch grid")
    if max(height, width) / min(height, width) > 200:
        raise ValueError("absolute aspect ratio must be below 200")
    h = max(factor, round(height / factor) * factor)
    w = max(factor, round(width / factor) * factor)
    if h * w > max_pixels:
        beta = math.sqrt(height * width / max_pixels)
        h = math.floor(height / beta / factor) * factor
        w = math.floor(width / beta / factor) * factor
    elif h * w < min_pixels:
        beta = math.sqrt(min_pixels / (height * width))
        h = math.ceil(height * beta / factor) * factor
        w = math.ceil(width * beta / factor) * factor
    return h, w


def load_image(img) -> torch.Tensor:
    """[3, H, W] float in [0, 1]."""
    if isinstance(img, str):
        from PIL import Image

        img = Image.open(img).convert("RGB")
    if hasattr(img, "convert") and not isinstance(img, (np.ndarray, torch.Tensor)):
        img = np.asarray(img.convert("RGB"))
    t = torch.as_tensor(np.asarray(img))
    if t.dtype == torch.uint8:
        t = t.float() / 255.0
    if t.ndim == 3 and t.shape[-1] in (3, 4):
        t = t[..., :3].permute(2, 0, 1)
    return t.float().contiguous()


def resize(img: torch.Tensor, h: int, w: int) -> torch.Tensor:
    if img.shape[-2:] == (h, w):
        return img
    return torch.nn.functional.interpolate(img[None], size=(h, w), mode="bicubic", align_corners=False,
                                           antialias=True)[0].clamp(0.0, 1.0)


def patchify(frames: torch.Tensor, cfg: MediaConfig) -> tuple[torch.Tensor, tuple[int, int, int]]:
    """frames [F, C, H, W] (normalised) -> patches [t*h*w, C*tp*p*p] in the
    order that groups each merge_size x merge_size block of patches, and the
    grid (t, h, w) in patches."""
    p, tp, m = cfg.patch_size, cfg.temporal_patch_size, cfg.merge_size
    if frames.shape[0] % tp:
        pad = tp - frames.shape[0] % tp
        frames = torch.cat([frames, frames[-1:].expand(pad, -1, -1, -1)], 0)
    F, C, H, W = frames.shape
    t, h, w = F // tp, H // p, W // p
    x = frames.reshape(t, tp, C, h // m, m, p, w // m, m, p)
    x = x.permute(0, 3, 6, 4, 7, 2, 1, 5, 8)
    return x.reshape(t * h * w, C * tp * p * p).contiguous(), (t, h, w)


def process_image(img, cfg: MediaConfig | None = None, size: tuple[int, int] | None = None):
    """(patches, grid) of one image (repeated to the temporal patch size)."""
    cfg = cfg or MediaConfig()
    x = load_image(img)
    factor = cfg.patch_size * cfg.merge_size
    h, w = size or target_size(x.shape[1], x.shape[2], factor, cfg.min_pixels, cfg.max_pixels)
    x = resize(x, h, w)
    mean = torch.tensor(cfg.mean)[:, None, None]
    std = torch.tensor(cfg.std)[:, None, None]
    x = (x - mean) / std
    return patchify(x[None], cfg)


def process_video(frames: list, cfg: MediaConfig | None = None, size: tuple[int, int] | None = None):
    cfg = cfg or MediaConfig()
    xs = [load_image(f) for f in frames]
    factor = cfg.patch_size * cfg.merge_size
    h, w = size or target_size(xs[0].shape[1], xs[0].shape[2], factor, cfg.min_pixels, cfg.max_pixels)
    mean = torch.tensor(cfg.mean)[:, None, None]
    std = torch.tensor(cfg.std)[:, None, None]
    x = torch.stack([(resize(f, h, w) - mean) / std for f in xs])
    return patchify(x, cfg)


@dataclass
class MediaInput:
    """The media of one request: images and videos, in prompt order."""
    images: list = field(default_factory=list)
    videos: list = field(default_factory=list)
