"""Data transforms (include/dlvk/data/transforms.h:17-430,
src/data/transforms.cpp, src/data/transform_factory.cpp).

Every transform takes one sample [C, H, W] or a batch [N, C, H, W] (fp32).
On a CUDA tensor the whole batch is transformed by one device kernel
(augment.cu via `_C.image`); on a CPU tensor the same math runs in plain
torch (the oracle the GPU tests compare against).  Random transforms draw
their per-sample parameters on the host from their own seeded
`torch.Generator`, so a run is reproducible and the CPU and GPU paths see
identical parameters.

Formulas follow transforms.cpp: Normalize (x - mean[c]) / std[c] for the
channels listed (:26-60); Standardize per sample with population std
(:69-95); MinMaxScale (:106-125); flips; RandomRotation about (W/2, H/2)
with nearest-round sampling and zero fill (:256-300); RandomCrop with zero
padding (:315-380); CenterCrop (:381-428); RandomNoise N(0, sigma)
(:430-450); RandomBrightness clamp(x + U(-b, b), 0, 1) (:452-475);
RandomContrast clamp(mean + U(1-r, 1+r)(x - mean), 0, 1) (:476-505);
ColorJitter = brightness then contrast (saturation is accepted and, as in
the reference, unused) (:506-520); Resize nearest/bilinear (:592-660).

Deviation: RandomScale keeps the sample's H x W (zoom in/out anchored at
the top-left, src = dst / s, zero fill) because all samples of a batch must
share one shape; the reference returned a per-sample size (:541-590).
"""
from __future__ import annotations

import enum
import math
from typing import Dict, List, Optional, Sequence

import torch

from .. import _ext


def _img():
    return _ext.C().image


def _round_half_away(v: torch.Tensor) -> torch.Tensor:
    return torch.sign(v) * torch.floor(v.abs() + 0.5)


def affine_sample_reference(x: torch.Tensor, theta: torch.Tensor, oh: int, ow: int, mode: int,
                            fill: float = 0.0) -> torch.Tensor:
    """CPU restatement of image_affine_sample (oracle)."""
    N, C, H, W = x.shape
    oy, ox = torch.meshgrid(torch.arange(oh, dtype=torch.float32), torch.arange(ow, dtype=torch.float32),
                            indexing="ij")
    out = torch.full((N, C, oh, ow), float(fill), dtype=torch.float32)
    for n in range(N):
        t = theta[n].float()
        sx = t[0] * ox + t[1] * oy + t[2]
        sy = t[3] * ox + t[4] * oy + t[5]
        src = x[n].float()
        if mode == 2:
            fx, fy = torch.floor(sx), torch.floor(sy)
            x1, y1 = fx.long(), fy.long()
            ok = (x1 >= 0) & (x1 < W) & (y1 >= 0) & (y1 < H)
            x1c, y1c = x1.clamp(0, W - 1), y1.clamp(0, H - 1)
            x2c, y2c = (x1c + 1).clamp(max=W - 1), (y1c + 1).clamp(max=H - 1)
            dx, dy = sx - fx, sy - fy
            v = (src[:, y1c, x1c] * (1 - dy) * (1 - dx) + src[:, y1c, x2c] * (1 - dy) * dx
                 + src[:, y2c, x1c] * dy * (1 - dx) + src[:, y2c, x2c] * dy * dx)
        else:
            ix = (_round_half_away(sx) if mode == 1 else torch.floor(sx)).long()
            iy = (_round_half_away(sy) if mode == 1 else torch.floor(sy)).long()
            ok = (ix >= 0) & (ix < W) & (iy >= 0) & (iy < H)
            v = src[:, iy.clamp(0, H - 1), ix.clamp(0, W - 1)]
        out[n] = torch.where(ok, v, torch.full_like(v, float(fill)))
    return out


def _affine(x: torch.Tensor, theta: torch.Tensor, oh: int, ow: int, mode: int) -> torch.Tensor:
    if x.is_cuda:
        return _img().affine_sample(x.contiguous(), theta.to(x.device).contiguous(), oh, ow, mode, 0.0)
    return affine_sample_reference(x, theta, oh, ow, mode)


def per_sample_stats_reference(x: torch.Tensor, kind: int, params: Optional[torch.Tensor], clamp01: bool):
    N = x.shape[0]
    flat = x.reshape(N, -1).float()
    mean = flat.mean(1, keepdim=True)
    if kind == 0:
        f = params[:, 0:1]
        y = mean + f * (flat - mean)
    elif kind == 1:
        std = torch.sqrt(((flat - mean) ** 2).mean(1, keepdim=True))
        y = torch.where(std > 1e-8, (flat - mean) / std.clamp(min=1e-30), flat)
    else:
        mn, mx = flat.min(1, keepdim=True).values, flat.max(1, keepdim=True).values
        rng = mx - mn
        lo, hi = params[:, 0:1], params[:, 1:2]
        y = torch.where(rng > 1e-8, lo + (flat - mn) * (hi - lo) / rng.clamp(min=1e-30), flat)
    if clamp01:
        y = y.clamp(0.0, 1.0)
    return y.reshape(x.shape)


def _stats(x, kind, params=None, clamp01=False):
    if x.is_cuda:
        p = params.to(x.device).contiguous() if params is not None else None
        return _img().per_sample_stats(x.contiguous(), kind, p, clamp01)
    return per_sample_stats_reference(x, kind, params, clamp01)


class Transform:
    """Base: `__call__` accepts [C,H,W] or [N,C,H,W]; subclasses implement
    `apply_batch` on 4-D input."""

    def __init__(self, seed: Optional[int] = None):
        self.gen = torch.Generator()
        self.gen.manual_seed(seed if seed is not None else torch.seed() & 0x7FFFFFFF)

    def __call__(self, x):
        batched = x.dim() == 4
        xb = x if batched else x.unsqueeze(0)
        if xb.dtype != torch.float32:
            xb = xb.float()
        y = self.apply_batch(xb)
        return y if batched else y[0]

    def apply(self, x):
        return self(x)

    def apply_batch(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def clone(self) -> "Transform":
        import copy

        return copy.deepcopy(self)

    def _uniform(self, n: int, lo: float, hi: float) -> torch.Tensor:
        return lo + (hi - lo) * torch.rand(n, generator=self.gen)


TensorTransform = Transform


def _require_image(x):
    if x.dim() != 4:
        raise ValueError("image transforms need [C,H,W] or [N,C,H,W] input")


class Normalize(Transform):
    def __init__(self, mean: Sequence[float], std: Sequence[float]):
        super().__init__(0)
        self.mean, self.std = [float(m) for m in mean], [float(s) for s in std]

    def apply_batch(self, x):
        N, C = x.shape[0], x.shape[1]
        m = torch.zeros(C)
        inv = torch.ones(C)
        for c in range(min(C, len(self.mean))):
            m[c] = self.mean[c]
            inv[c] = 1.0 / self.std[c]
        if x.is_cuda:
            return _img().channel_affine(x.contiguous(), m.to(x.device), inv.to(x.device), None, False)
        shape = [1, C] + [1] * (x.dim() - 2)
        return (x - m.reshape(shape)) * inv.reshape(shape)

    def __call__(self, x):
        if x.dim() < 3:  # reference: scalar normalisation with mean[0], std[0]
            return (x.float() - self.mean[0]) / self.std[0]
        return super().__call__(x)


class Standardize(Transform):
    def __init__(self):
        super().__init__(0)

    def apply_batch(self, x):
        return _stats(x, 1)


class MinMaxScale(Transform):
    def __init__(self, min_val: float = 0.0, max_val: float = 1.0):
        super().__init__(0)
        self.min_val, self.max_val = float(min_val), float(max_val)

    def apply_batch(self, x):
        p = torch.tensor([[self.min_val, self.max_val]] * x.shape[0], dtype=torch.float32)
        return _stats(x, 2, p)


class ToOneHot(Transform):
    def __init__(self, num_classes: int):
        super().__init__(0)
        self.num_classes = int(num_classes)

    def __call__(self, labels):
        lab = torch.as_tensor(labels).reshape(-1).long()
        out = torch.zeros((lab.numel(), self.num_classes), dtype=torch.float32, device=lab.device)
        out.scatter_(1, lab.unsqueeze(1), 1.0)
        return out if torch.as_tensor(labels).dim() > 0 else out[0]


class _Flip(Transform):
    axis = "h"

    def __init__(self, probability: float = 0.5, seed: Optional[int] = None):
        super().__init__(seed)
        self.p = float(probability)

    def apply_batch(self, x):
        _require_image(x)
        N, C, H, W = x.shape
        flip = torch.rand(N, generator=self.gen) < self.p
        th = torch.tensor([1.0, 0.0, 0.0, 0.0, 1.0, 0.0]).repeat(N, 1)
        if self.axis == "h":
            th[flip, 0] = -1.0
            th[flip, 2] = W - 1.0
        else:
            th[flip, 4] = -1.0
            th[flip, 5] = H - 1.0
        return _affine(x, th, H, W, 0)


class RandomHorizontalFlip(_Flip):
    axis = "h"


class RandomVerticalFlip(_Flip):
    axis = "v"


class RandomRotation(Transform):
    def __init__(self, max_angle: float = 30.0, seed: Optional[int] = None):
        super().__init__(seed)
        self.max_angle = float(max_angle)

    @staticmethod
    def theta_for(angles_deg: torch.Tensor, H: int, W: int) -> torch.Tensor:
        a = angles_deg.double() * math.pi / 180.0
        c, s = torch.cos(a), torch.sin(a)
        cx, cy = W / 2.0, H / 2.0
        return torch.stack([c, -s, cx - c * cx + s * cy, s, c, cy - s * cx - c * cy], 1).float()

    def apply_batch(self, x):
        _require_image(x)
        N, C, H, W = x.shape
        ang = self._uniform(N, -self.max_angle, self.max_angle)
        return _affine(x, self.theta_for(ang, H, W), H, W, 1)


class RandomCrop(Transform):
    def __init__(self, crop_height: int, crop_width: int, padding: int = 0, seed: Optional[int] = None):
        super().__init__(seed)
        self.ch, self.cw, self.pad = int(crop_height), int(crop_width), int(padding)

    def apply_batch(self, x):
        _require_image(x)
        N, C, H, W = x.shape
        ph, pw = H + 2 * self.pad, W + 2 * self.pad
        if self.ch > ph or self.cw > pw:
            raise ValueError("Crop size is larger than padded input size")
        sh = torch.randint(0, ph - self.ch + 1, (N,), generator=self.gen).float()
        sw = torch.randint(0, pw - self.cw + 1, (N,), generator=self.gen).float()
        th = torch.zeros(N, 6)
        th[:, 0], th[:, 2] = 1.0, sw - self.pad
        th[:, 4], th[:, 5] = 1.0, sh - self.pad
        return _affine(x, th, self.ch, self.cw, 0)


class CenterCrop(Transform):
    def __init__(self, crop_height: int, crop_width: int):
        super().__init__(0)
        self.ch, self.cw = int(crop_height), int(crop_width)

    def apply_batch(self, x):
        _require_image(x)
        N, C, H, W = x.shape
        if self.ch > H or self.cw > W:
            raise ValueError("Crop size is larger than input size")
        th = torch.tensor([1.0, 0.0, float((W - self.cw) // 2), 0.0, 1.0, float((H - self.ch) // 2)]).repeat(N, 1)
        return _affine(x, th, self.ch, self.cw, 0)


class RandomNoise(Transform):
    def __init__(self, noise_factor: float = 0.1, seed: Optional[int] = None):
        super().__init__(seed)
        self.sigma = float(noise_factor)
        self._calls = 0

    def apply_batch(self, x):
        self._calls += 1
        if x.is_cuda:
            seed = int(torch.randint(0, 2 ** 62, (1,), generator=self.gen))
            return _img().gaussian_noise(x.contiguous(), self.sigma, seed, self._calls & 0xFFFFFFFF)
        return x + self.sigma * torch.randn(x.shape, generator=self.gen)


class RandomBrightness(Transform):
    def __init__(self, brightness_factor: float = 0.2, seed: Optional[int] = None):
        super().__init__(seed)
        self.b = float(brightness_factor)

    def apply_batch(self, x):
        N = x.shape[0]
        delta = self._uniform(N, -self.b, self.b)
        if x.is_cuda:
            return _img().channel_affine(x.contiguous(), None, None, delta.to(x.device), True)
        return (x + delta.reshape([N] + [1] * (x.dim() - 1))).clamp(0.0, 1.0)


class RandomContrast(Transform):
    def __init__(self, contrast_range: float = 0.3, seed: Optional[int] = None):
        super().__init__(seed)
        self.r = float(contrast_range)

    def apply_batch(self, x):
        N = x.shape[0]
        f = self._uniform(N, 1.0 - self.r, 1.0 + self.r)
        return _stats(x, 0, torch.stack([f, torch.zeros(N)], 1), True)


class ColorJitter(Transform):
    def __init__(self, brightness: float = 0.2, contrast: float = 0.2, saturation: float = 0.2,
                 seed: Optional[int] = None):
        super().__init__(seed)
        self.brightness, self.contrast, self.saturation = float(brightness), float(contrast), float(saturation)
        s = int(torch.randint(0, 2 ** 31 - 1, (1,), generator=self.gen))
        self._b = RandomBrightness(self.brightness, seed=s) if self.brightness > 0 else None
        self._c = RandomContrast(self.contrast, seed=s + 1) if self.contrast > 0 else None

    def apply_batch(self, x):
        if self._b is not None:
            x = self._b.apply_batch(x)
        if self._c is not None:
            x = self._c.apply_batch(x)
        return x


class RandomScale(Transform):
    def __init__(self, min_scale: float = 0.8, max_scale: float = 1.2, seed: Optional[int] = None):
        super().__init__(seed)
        self.min_scale, self.max_scale = float(min_scale), float(max_scale)

    def apply_batch(self, x):
        _require_image(x)
        N, C, H, W = x.shape
        s = self._uniform(N, self.min_scale, self.max_scale)
        th = torch.zeros(N, 6)
        th[:, 0] = 1.0 / s
        th[:, 4] = 1.0 / s
        return _affine(x, th, H, W, 0)


class InterpolationMode(enum.Enum):
    NEAREST = 0
    BILINEAR = 2


class Resize(Transform):
    InterpolationMode = InterpolationMode

    def __init__(self, height: int, width: int, mode: InterpolationMode = InterpolationMode.BILINEAR):
        super().__init__(0)
        self.h, self.w, self.mode = int(height), int(width), mode

    def apply_batch(self, x):
        _require_image(x)
        N, C, H, W = x.shape
        if (H, W) == (self.h, self.w):
            return x.clone()
        th = torch.tensor([W / self.w, 0.0, 0.0, 0.0, H / self.h, 0.0]).repeat(N, 1)
        return _affine(x, th, self.h, self.w, self.mode.value)


class Compose(Transform):
    def __init__(self, transforms: Sequence[Transform] = ()):
        super().__init__(0)
        self.transforms: List = list(transforms)

    def add_transform(self, t) -> None:
        self.transforms.append(t)

    def size(self) -> int:
        return len(self.transforms)

    def __len__(self):
        return len(self.transforms)

    def apply_batch(self, x):
        for t in self.transforms:
            x = t.apply_batch(x) if isinstance(t, Transform) else t(x)
        return x


class RandomChoice(Transform):
    """Each sample goes through one transform picked uniformly."""

    def __init__(self, transforms: Sequence[Transform], seed: Optional[int] = None):
        super().__init__(seed)
        self.transforms = list(transforms)

    def apply_batch(self, x):
        N = x.shape[0]
        pick = torch.randint(0, len(self.transforms), (N,), generator=self.gen)
        out = None
        for k, t in enumerate(self.transforms):
            sel = (pick == k).nonzero().reshape(-1)
            if sel.numel() == 0:
                continue
            selx = sel.to(x.device)
            y = t.apply_batch(x.index_select(0, selx).contiguous())
            if out is None:
                out = torch.empty((N, *y.shape[1:]), dtype=y.dtype, device=y.device)
            out.index_copy_(0, selx, y)
        return out if out is not None else x.clone()


class RandomApply(Transform):
    """Apply `transform` to each sample with probability p (shape-preserving
    transforms)."""

    def __init__(self, transform: Transform, probability: float = 0.5, seed: Optional[int] = None):
        super().__init__(seed)
        self.transform, self.p = transform, float(probability)

    def apply_batch(self, x):
        N = x.shape[0]
        sel = (torch.rand(N, generator=self.gen) < self.p).nonzero().reshape(-1)
        out = x.clone()
        if sel.numel():
            selx = sel.to(x.device)
            y = self.transform.apply_batch(x.index_select(0, selx).contiguous())
            if y.shape[1:] != x.shape[1:]:
                raise ValueError("RandomApply needs a shape-preserving transform")
            out.index_copy_(0, selx, y)
        return out


# ------------------------------------------------------------ strategies (transforms.cpp:755-785)
class AugmentationStrategy:
    def create_transform(self) -> Compose:
        raise NotImplementedError

    def name(self) -> str:
        raise NotImplementedError


class LightAugmentation(AugmentationStrategy):
    def create_transform(self):
        return Compose([RandomHorizontalFlip(0.5), RandomBrightness(0.1)])

    def name(self):
        return "light"


class MediumAugmentation(AugmentationStrategy):
    def create_transform(self):
        return Compose([RandomHorizontalFlip(0.5), RandomVerticalFlip(0.2), RandomRotation(15.0),
                        ColorJitter(0.2, 0.2, 0.2), RandomNoise(0.05)])

    def name(self):
        return "medium"


class HeavyAugmentation(AugmentationStrategy):
    def __init__(self, crop: int = 224):
        self.crop = crop

    def create_transform(self):
        return Compose([RandomHorizontalFlip(0.5), RandomVerticalFlip(0.3), RandomRotation(30.0),
                        RandomScale(0.7, 1.3), ColorJitter(0.4, 0.4, 0.4), RandomNoise(0.1),
                        RandomCrop(self.crop, self.crop, 4)])

    def name(self):
        return "heavy"


class PreprocessingPipeline:
    """Named, ordered transform list (transforms.cpp:788-846)."""

    def __init__(self):
        self.transforms = Compose([])
        self.named: Dict[str, Transform] = {}

    def add_transform(self, name: str, transform) -> "PreprocessingPipeline":
        self.named[name] = transform
        self.transforms.add_transform(transform)
        return self

    def add_normalization(self, mean, std):
        return self.add_transform("normalize", Normalize(mean, std))

    def add_standardization(self):
        return self.add_transform("standardize", Standardize())

    def add_min_max_scaling(self, min_val: float = 0.0, max_val: float = 1.0):
        return self.add_transform("min_max_scale", MinMaxScale(min_val, max_val))

    def add_resize(self, height: int, width: int):
        return self.add_transform("resize", Resize(height, width))

    def add_augmentation_strategy(self, strategy: AugmentationStrategy):
        return self.add_transform("augmentation_" + strategy.name(), strategy.create_transform())

    def process(self, x):
        return self.transforms(x)

    __call__ = process

    def has_transform(self, name: str) -> bool:
        return name in self.named

    def remove_transform(self, name: str) -> None:
        t = self.named.pop(name, None)
        if t is not None:
            self.transforms.transforms = [u for u in self.transforms.transforms if u is not t]

    def clear(self) -> None:
        self.named.clear()
        self.transforms.transforms.clear()


# ------------------------------------------------------------ factory (transform_factory.cpp:9-247)
_IMAGENET_MEAN, _IMAGENET_STD = [0.485, 0.456, 0.406], [0.229, 0.224, 0.225]


def create_imagenet_pipeline(training: bool = True) -> PreprocessingPipeline:
    p = PreprocessingPipeline()
    if training:
        p.add_resize(256, 256)
        p.add_transform("random_crop", RandomCrop(224, 224, 4))
        p.add_transform("random_flip", RandomHorizontalFlip(0.5))
        p.add_transform("color_jitter", ColorJitter(0.4, 0.4, 0.4))
    else:
        p.add_resize(224, 224)
        p.add_transform("center_crop", CenterCrop(224, 224))
    return p.add_normalization(_IMAGENET_MEAN, _IMAGENET_STD)


def create_cifar10_pipeline(training: bool = True) -> PreprocessingPipeline:
    p = PreprocessingPipeline()
    if training:
        p.add_transform("random_crop", RandomCrop(32, 32, 4))
        p.add_transform("random_flip", RandomHorizontalFlip(0.5))
    return p.add_normalization([0.4914, 0.4822, 0.4465], [0.2023, 0.1994, 0.2010])


def create_mnist_pipeline(training: bool = True) -> PreprocessingPipeline:
    p = PreprocessingPipeline()
    if training:
        p.add_transform("random_rotation", RandomRotation(10.0))
        p.add_transform("random_crop", RandomCrop(28, 28, 2))
    return p.add_normalization([0.1307], [0.3081])


def create_coco_pipeline(training: bool = True) -> PreprocessingPipeline:
    p = PreprocessingPipeline()
    if training:
        p.add_transform("random_scale", RandomScale(0.8, 1.2))
        p.add_transform("random_flip", RandomHorizontalFlip(0.5))
        p.add_transform("color_jitter", ColorJitter(0.1, 0.1, 0.1))
    p.add_resize(416, 416)
    return p.add_normalization(_IMAGENET_MEAN, _IMAGENET_STD)


def create_classification_pipeline(input_size: int, training: bool = True) -> PreprocessingPipeline:
    p = PreprocessingPipeline()
    if training:
        big = int(input_size * 1.15)
        p.add_resize(big, big)
        p.add_transform("random_crop", RandomCrop(input_size, input_size))
        p.add_transform("random_flip", RandomHorizontalFlip(0.5))
        p.add_transform("color_jitter", ColorJitter(0.3, 0.3, 0.3))
        p.add_transform("random_rotation", RandomRotation(15.0))
    else:
        p.add_resize(input_size, input_size)
    return p.add_standardization()


def create_segmentation_pipeline(input_size: int, training: bool = True) -> PreprocessingPipeline:
    p = PreprocessingPipeline()
    if training:
        p.add_transform("random_scale", RandomScale(0.5, 2.0))
        p.add_transform("random_crop", RandomCrop(input_size, input_size))
        p.add_transform("random_flip", RandomHorizontalFlip(0.5))
        p.add_transform("color_jitter", ColorJitter(0.2, 0.2, 0.2))
    else:
        p.add_resize(input_size, input_size)
    return p.add_normalization(_IMAGENET_MEAN, _IMAGENET_STD)


def create_detection_pipeline(input_size: int, training: bool = True) -> PreprocessingPipeline:
    p = PreprocessingPipeline()
    if training:
        p.add_transform("random_scale", RandomScale(0.8, 1.2))
        p.add_transform("random_flip", RandomHorizontalFlip(0.5))
        p.add_transform("color_jitter", ColorJitter(0.1, 0.1, 0.1))
        p.add_transform("random_brightness", RandomBrightness(0.1))
    p.add_resize(input_size, input_size)
    return p.add_normalization(_IMAGENET_MEAN, _IMAGENET_STD)


class PreprocessingPipelineBuilder:
    def __init__(self):
        self.p = PreprocessingPipeline()
        self._n = 0

    def _add(self, name, t):
        self._n += 1
        self.p.add_transform(f"{name}_{self._n}", t)
        return self

    def resize(self, h, w):
        return self._add("resize", Resize(h, w))

    def random_crop(self, h, w, padding=0):
        return self._add("random_crop", RandomCrop(h, w, padding))

    def center_crop(self, h, w):
        return self._add("center_crop", CenterCrop(h, w))

    def random_horizontal_flip(self, p=0.5):
        return self._add("random_hflip", RandomHorizontalFlip(p))

    def random_vertical_flip(self, p=0.5):
        return self._add("random_vflip", RandomVerticalFlip(p))

    def random_rotation(self, max_angle=15.0):
        return self._add("random_rotation", RandomRotation(max_angle))

    def random_scale(self, lo=0.8, hi=1.2):
        return self._add("random_scale", RandomScale(lo, hi))

    def color_jitter(self, b=0.2, c=0.2, s=0.2):
        return self._add("color_jitter", ColorJitter(b, c, s))

    def random_noise(self, f=0.05):
        return self._add("random_noise", RandomNoise(f))

    def normalize(self, mean, std):
        return self._add("normalize", Normalize(mean, std))

    def standardize(self):
        return self._add("standardize", Standardize())

    def min_max_scale(self, lo=0.0, hi=1.0):
        return self._add("min_max_scale", MinMaxScale(lo, hi))

    def to_one_hot(self, num_classes):
        return self._add("to_one_hot", ToOneHot(num_classes))

    def augmentation_strategy(self, strategy: AugmentationStrategy):
        return self._add("augmentation_" + strategy.name(), strategy.create_transform())

    def light_augmentation(self):
        return self.augmentation_strategy(LightAugmentation())

    def medium_augmentation(self):
        return self.augmentation_strategy(MediumAugmentation())

    def heavy_augmentation(self):
        return self.augmentation_strategy(HeavyAugmentation())

    def custom_transform(self, name, t):
        return self._add(name, t)

    def build(self) -> PreprocessingPipeline:
        return self.p


# The reference's factory::SimpleBuilder (include/dlvk/data/transforms_clean.h:172-184):
# resize / random_horizontal_flip / random_crop / normalize / build.
SimpleBuilder = PreprocessingPipelineBuilder
