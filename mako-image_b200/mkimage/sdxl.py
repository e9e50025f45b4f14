"""The SDXL UNet and VAE decoder handles (include/mkb_image.h part 3) as Python objects."""

import ctypes
import dataclasses
from dataclasses import dataclass, field

import numpy as np

from ._lib import lib, check
from .dit import _PROBE_FN, _fptr


@dataclass
class UnetConfig:
    channels: tuple = (320, 640, 1280)
    depth: tuple = (0, 2, 10)
    layers: int = 2
    context_dim: int = 2048
    pooled_dim: int = 1280
    max_batch: int = 2
    max_gh: int = 64
    max_gw: int = 64
    max_context: int = 77
    slots: int = 2


class _CUnet(ctypes.Structure):
    _fields_ = [("channels", ctypes.c_int * 3), ("depth", ctypes.c_int * 3), ("layers", ctypes.c_int),
                ("context_dim", ctypes.c_int), ("pooled_dim", ctypes.c_int), ("max_batch", ctypes.c_int),
                ("max_gh", ctypes.c_int), ("max_gw", ctypes.c_int), ("max_context", ctypes.c_int),
                ("slots", ctypes.c_int)]


@dataclass
class VaeConfig:
    channels: tuple = (128, 256, 512, 512)
    layers: int = 2
    latent: int = 4
    scale: float = 0.13025
    max_gh: int = 64
    max_gw: int = 64


class _CVae(ctypes.Structure):
    _fields_ = [("channels", ctypes.c_int * 4), ("layers", ctypes.c_int), ("latent", ctypes.c_int),
                ("scale", ctypes.c_float), ("max_gh", ctypes.c_int), ("max_gw", ctypes.c_int)]


class _Weights:
    _prefix = ""

    def _fn(self, n):
        return getattr(lib, f"mkb_{self._prefix}_{n}")

    def weight_names(self):
        out = []
        name, dims, nd = ctypes.c_char_p(), (ctypes.c_long * 4)(), ctypes.c_int()
        for i in range(self._fn("weight_count")(self.h)):
            check(self._fn("weight_info")(self.h, i, ctypes.byref(name), dims, ctypes.byref(nd)))
            out.append((name.value.decode(), tuple(dims[:nd.value])))
        return out

    def read_weight(self, name, shape):
        a = np.empty(shape, np.float32)
        check(self._fn("weight_read")(self.h, name.encode(), _fptr(a)))
        return a

    def write_weight(self, name, a):
        a = np.ascontiguousarray(a, np.float32)
        check(self._fn("weight_write")(self.h, name.encode(), _fptr(a)))

    def weights(self):
        return {n: self.read_weight(n, s) for n, s in self.weight_names()}

    def init_random(self, seed, std=0.02):
        check(self._fn("init_random")(self.h, seed, std))

    def load_safetensors(self, paths, strict=True):
        """Weights from checkpoint files by their own tensor names (mkb_unet / mkb_vae_load_safetensors); returns
        the number of weights written."""
        import os

        if isinstance(paths, (str, bytes, os.PathLike)):
            paths = [paths]
        arr = (ctypes.c_char_p * len(paths))(*[str(p).encode() for p in paths])
        n = ctypes.c_int()
        check(self._fn("load_safetensors")(self.h, arr, len(paths), int(strict), ctypes.byref(n)))
        return n.value

    def set_probe(self, fn):
        if fn is None:
            self._probe = None
            check(self._fn("set_probe")(self.h, None, None))
            return

        def tramp(name, layer, data, count, user):
            fn(name.decode(), layer, np.ctypeslib.as_array(data, shape=(count,)).copy())

        self._probe = _PROBE_FN(tramp)
        check(self._fn("set_probe")(self.h, ctypes.cast(self._probe, ctypes.c_void_p), None))

    def close(self):
        if getattr(self, "h", None):
            self._fn("destroy")(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Unet(_Weights):
    _prefix = "unet"

    def __init__(self, cfg: UnetConfig):
        self.cfg = cfg
        c = _CUnet((ctypes.c_int * 3)(*cfg.channels), (ctypes.c_int * 3)(*cfg.depth), cfg.layers, cfg.context_dim,
                   cfg.pooled_dim, cfg.max_batch, cfg.max_gh, cfg.max_gw, cfg.max_context, cfg.slots)
        h = ctypes.c_void_p()
        check(lib.mkb_unet_create(ctypes.byref(c), ctypes.byref(h)))
        self.h = h
        self._probe = None

    def begin(self, context, pooled, gh, gw, slot=0):
        ctx = np.ascontiguousarray(context, np.float32)
        pl = np.ascontiguousarray(pooled, np.float32)
        check(lib.mkb_unet_begin(self.h, _fptr(ctx), ctx.shape[0], _fptr(pl), gh, gw, slot))

    def step_batch(self, latents, sigmas, slot0=0):
        x = np.ascontiguousarray(latents, np.float32)
        out = np.empty_like(x)
        n = len(sigmas)
        check(lib.mkb_unet_step_batch(self.h, n, slot0, _fptr(x), (ctypes.c_float * n)(*sigmas), _fptr(out)))
        return out

    def step(self, latents, sigma, slot=0):
        x = np.ascontiguousarray(latents, np.float32)
        out = np.empty_like(x)
        check(lib.mkb_unet_step(self.h, _fptr(x), sigma, _fptr(out), slot))
        return out

    def step_cfg_dev(self, latents_dev, sigma, sigma_next, guidance, stream=None):
        check(lib.mkb_unet_step_cfg_dev(self.h, ctypes.c_void_p(latents_dev), sigma, sigma_next, guidance, stream))

    def step_flops(self, n):
        return lib.mkb_unet_step_flops(self.h, n)

    def lora_merge(self, module, A, B, scale=1.0):
        """W += scale * B A for a transformer projection of the UNet (mkb_unet_lora_merge)."""
        A = np.ascontiguousarray(A, np.float32)
        B = np.ascontiguousarray(B, np.float32)
        if A.ndim != 2 or B.ndim != 2 or B.shape[1] != A.shape[0]:
            raise ValueError(f"lora_merge: A {A.shape} and B {B.shape} are not [rank][in] and [out][rank]")
        check(lib.mkb_unet_lora_merge(self.h, module.encode(), _fptr(A), _fptr(B), A.shape[0], A.shape[1], B.shape[0],
                                      scale))

    def load_lora(self, path, scale=1.0):
        """Merges every pair of a LoRA safetensors file into the UNet; returns the number of modules."""
        n = ctypes.c_int()
        check(lib.mkb_unet_load_lora(self.h, str(path).encode(), scale, ctypes.byref(n)))
        return n.value


class Vae(_Weights):
    _prefix = "vae"

    def __init__(self, cfg: VaeConfig):
        self.cfg = cfg
        c = _CVae((ctypes.c_int * 4)(*cfg.channels), cfg.layers, cfg.latent, cfg.scale, cfg.max_gh, cfg.max_gw)
        h = ctypes.c_void_p()
        check(lib.mkb_vae_create(ctypes.byref(c), ctypes.byref(h)))
        self.h = h
        self._probe = None

    def decode(self, latents, gh, gw):
        x = np.ascontiguousarray(latents, np.float32)
        out = np.empty((16 * gh, 16 * gw, 4), np.float32)
        check(lib.mkb_vae_decode(self.h, _fptr(x), gh, gw, _fptr(out)))
        return out

    def decode_dev(self, latents_dev, gh, gw, out_dev, stream=None):
        check(lib.mkb_vae_decode_dev(self.h, ctypes.c_void_p(latents_dev), gh, gw, ctypes.c_void_p(out_dev), stream))

    def set_latent_stats(self, mean, std):
        """Per token value (4 x latent of them): latents enter the decoder as tokens * std + mean."""
        m = np.ascontiguousarray(mean, np.float32)
        s = np.ascontiguousarray(std, np.float32)
        check(lib.mkb_vae_set_latent_stats(self.h, _fptr(m), _fptr(s), m.size))

    def decode_flops(self, gh, gw):
        return lib.mkb_vae_decode_flops(self.h, gh, gw)


@dataclass
class ClipConfig:
    """which 0: CLIP ViT-L (768 wide, 12 layers); 1: OpenCLIP bigG (1280, 32 layers, pooled state)."""
    which: int = 0
    width: int = 768
    heads: int = 12
    layers: int = 12
    ffn: int = 3072
    vocab: int = 49408
    max_chunks: int = 4

    @staticmethod
    def sdxl(which, **over):
        c = ClipConfig() if which == 0 else ClipConfig(which=1, width=1280, heads=20, layers=32, ffn=5120)
        return dataclasses.replace(c, **over)


class _CClip(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("which", "width", "heads", "layers", "ffn", "vocab", "max_chunks")]


class Clip(_Weights):
    """One of SDXL's text encoders (mkb_clip_*)."""

    _prefix = "clip"

    def __init__(self, cfg: ClipConfig):
        self.cfg = cfg
        c = _CClip(*(getattr(cfg, n) for n, _ in _CClip._fields_))
        h = ctypes.c_void_p()
        check(lib.mkb_clip_create(ctypes.byref(c), ctypes.byref(h)))
        self.h = h
        self._probe = None

    def encode(self, ids):
        """ids [chunks][77] -> (hidden [chunks * 77][E], pooled [chunks][1280] for bigG else None)."""
        ids = np.ascontiguousarray(np.asarray(ids, np.int32).reshape(-1, 77))
        n = ids.shape[0]
        hidden = np.empty((n * 77, self.cfg.width), np.float32)
        pooled = np.empty((n, 1280), np.float32) if self.cfg.which == 1 else None
        check(lib.mkb_clip_encode(self.h, ids.ctypes.data_as(ctypes.c_void_p), n, _fptr(hidden),
                                  _fptr(pooled) if pooled is not None else None))
        return hidden, pooled


def prompt_embeddings(clip_l, clip_g, ids_l, ids_g, weights=None):
    """mkb_sdxl_prompt_embeddings: ([chunks * 77][E_L + E_G] context, [1280] pooled)."""
    ids_l = np.ascontiguousarray(np.asarray(ids_l, np.int32).reshape(-1, 77))
    ids_g = np.ascontiguousarray(np.asarray(ids_g, np.int32).reshape(-1, 77))
    n = ids_l.shape[0]
    w = None if weights is None else np.ascontiguousarray(np.asarray(weights, np.float32).reshape(n, 77))
    ctx = np.empty((n * 77, clip_l.cfg.width + clip_g.cfg.width), np.float32)
    pooled = np.empty(1280, np.float32)
    check(lib.mkb_sdxl_prompt_embeddings(clip_l.h, clip_g.h, ids_l.ctypes.data_as(ctypes.c_void_p),
                                         ids_g.ctypes.data_as(ctypes.c_void_p), _fptr(w) if w is not None else None,
                                         n, _fptr(ctx), _fptr(pooled)))
    return ctx, pooled


def sdxl_sigmas(steps):
    out = np.empty(steps + 1, np.float32)
    check(lib.mkb_sdxl_sigmas(steps, _fptr(out)))
    return out


def sdxl_timestep(sigma):
    return lib.mkb_sdxl_timestep(sigma)
