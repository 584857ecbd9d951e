"""SigLIP vision tower on the device (internal/siglip/vision.go, encoder.go).

The Python side of the C ABI's ig_vision_*: a Vision built from float32
weights in transformers layouts, whose Embed and Forward run a whole batch of
images through the int8 layers and the float32 patch embedding, attention
and pooling head of the reference, with its roundings. No CPU fallback: the
library must be built and a B200 present.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _capi


class SiglipError(ValueError):
    """An error the reference reports as a Go error ("siglip: ...")."""


@dataclass
class VisionConfig:
    """Config (siglip.go:26-33) after ReadConfig's defaults (:83-97)."""
    hidden: int = 768
    layers: int = 12
    heads: int = 12
    mlp: int = 3072
    image_size: int = 224
    patch_size: int = 16
    eps: float = 1e-6
    simd_lanes: int = 8

    @classmethod
    def from_dict(cls, d: dict) -> "VisionConfig":
        return cls(hidden=d.get("hidden", 768), layers=d.get("layers", 12), heads=d.get("heads", 12),
                   mlp=d.get("mlp", 3072), image_size=d.get("image_size", 224), patch_size=d.get("patch_size", 16),
                   eps=d.get("eps", 1e-6) or 1e-6, simd_lanes=d.get("V", 8))

    def Patches(self) -> int:
        g = self.image_size // self.patch_size
        return g * g

    def validate(self):
        if self.hidden % self.heads != 0 or self.image_size % self.patch_size != 0:
            raise SiglipError("siglip: inconsistent dimensions")

    def to_c(self) -> _capi.IgVisionConfig:
        return _capi.IgVisionConfig(hidden=self.hidden, layers=self.layers, heads=self.heads, mlp=self.mlp,
                                    image_size=self.image_size, patch_size=self.patch_size, eps=self.eps,
                                    simd_lanes=self.simd_lanes)


class Vision:
    """The image tower on one GPU (Vision, vision.go:11-27)."""

    def __init__(self, cfg: VisionConfig, handle, device: int):
        self.cfg, self._h, self.device = cfg, handle, device

    @classmethod
    def from_arrays(cls, cfg: VisionConfig, w: dict, device: int = 0) -> "Vision":
        """Weights as synthetic.siglip_weights lays them out ([out][in] matrices)."""
        cfg.validate()
        L = cfg.layers
        keep = {k: (np.ascontiguousarray(v, np.float32) if not isinstance(v, list)
                    else [np.ascontiguousarray(a, np.float32) for a in v]) for k, v in w.items()}
        fields, arrs = {}, []
        for n in _capi.VISION_FLAT + _capi.VISION_TAIL:
            fields[n] = keep[n].ctypes.data
        for n in _capi.VISION_LAYER:
            if len(keep[n]) != L:
                raise SiglipError(f"siglip: {n}: {len(keep[n])} layers, expected {L}")
            a = (C.c_void_p * L)(*[x.ctypes.data for x in keep[n]])
            arrs.append(a)
            fields[n] = C.cast(a, C.POINTER(C.c_void_p))
        cw = _capi.IgVisionWeights(**fields)
        h = C.c_void_p()
        rc = _capi.load().ig_vision_create(C.byref(cfg.to_c()), C.byref(cw), device, C.byref(h))
        if rc == _capi.IG_ERR_BAD_ARG:
            raise SiglipError(_capi.last_error())
        _capi.check(rc)
        return cls(cfg, h.value, device)

    def close(self):
        if getattr(self, "_h", None):
            _capi.load().ig_vision_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _pixels(self, pixels) -> np.ndarray:
        S = self.cfg.image_size
        px = np.ascontiguousarray(pixels, np.float32)
        if px.ndim == 3:
            px = px[None]
        if px.ndim != 4 or px.shape[1:] != (3, S, S):
            raise SiglipError(f"siglip: {px.size // max(px.shape[0], 1) if px.ndim else px.size} pixel values, "
                              f"expected 3×{S}×{S}")
        return px

    def Forward(self, pixels, layer: int = 0, pool: bool = False):
        """Vision.Forward (vision.go:94-99) on a batch [n][3][S][S]: patch
        features [n][T][H] (after `layer` layers, or final for 0) and, with
        pool, the embeddings [n][H]."""
        px = self._pixels(pixels)
        n, H = px.shape[0], self.cfg.hidden
        pa = np.empty((n, self.cfg.Patches(), H), np.float32)  # every entry is written
        po = np.empty((n, H), np.float32) if pool else None
        rc = _capi.load().ig_vision_forward(self._h, px.ctypes.data, n, int(layer), pa.ctypes.data, pa.size,
                                            po.ctypes.data if po is not None else None, po.size if po is not None else 0)
        if rc == _capi.IG_ERR_BAD_ARG:
            raise SiglipError(_capi.last_error())
        _capi.check(rc)
        return pa, po

    def Embed(self, pixels) -> np.ndarray:
        """Vision.Embed (vision.go:85-88): the pooled embedding [n][H] of each image."""
        px = self._pixels(pixels)
        n, H = px.shape[0], self.cfg.hidden
        po = np.empty((n, H), np.float32)
        rc = _capi.load().ig_vision_forward(self._h, px.ctypes.data, n, 0, None, 0, po.ctypes.data, po.size)
        if rc == _capi.IG_ERR_BAD_ARG:
            raise SiglipError(_capi.last_error())
        _capi.check(rc)
        return po

    def dump(self, pixels, layer: int):
        """Intermediates of one layer (and the embeddings) for parity checks."""
        px = self._pixels(pixels)
        n, H, M, T = px.shape[0], self.cfg.hidden, self.cfg.mlp, self.cfg.Patches()
        N = n * T
        arrays = dict(x_embed=np.zeros((N, H), np.float32), h1q=np.zeros((N, H), np.uint8),
                      h1q_s=np.zeros(N, np.float32), qkv=np.zeros((N, 3 * H), np.float32),
                      attn=np.zeros((N, H), np.float32), x_attn=np.zeros((N, H), np.float32),
                      h2q=np.zeros((N, H), np.uint8), h2q_s=np.zeros(N, np.float32), mlp=np.zeros((N, M), np.float32),
                      outliers=np.zeros((n, 32), np.int32), noutliers=np.zeros(n, np.int32),
                      mq=np.zeros((N, M), np.uint8), mq_s=np.zeros(N, np.float32), x_mlp=np.zeros((N, H), np.float32))
        d = _capi.IgVisionDump(layer=layer, **{k: v.ctypes.data for k, v in arrays.items()})
        po = np.zeros((n, H), np.float32)
        _capi.check(_capi.load().ig_vision_dump_layer(self._h, px.ctypes.data, n, C.byref(d), po.ctypes.data, po.size))
        return arrays, po
