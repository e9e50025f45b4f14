"""The denoiser handle (include/mkb_image.h part 2) as a Python object: the reference's Engine::begin / step on host
numpy arrays, plus the batched, guided and device-buffer steps."""

import ctypes
import os
from dataclasses import dataclass, asdict

import numpy as np

from ._lib import lib, check

QWEN1, REF21 = 0, 1

_PROBE_FN = ctypes.CFUNCTYPE(None, ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float), ctypes.c_long,
                             ctypes.c_void_p)


@dataclass
class DitConfig:
    variant: int = QWEN1
    hidden: int = 3072
    heads: int = 24
    ffn: int = 12288
    blocks: int = 60
    text_dim: int = 3584
    max_batch: int = 2
    max_text_tokens: int = 256
    max_image_tokens: int = 4096
    slots: int = 2


class _CConfig(ctypes.Structure):
    _fields_ = [(k, ctypes.c_int) for k in DitConfig.__dataclass_fields__]


def _fptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


class Dit:
    def __init__(self, cfg: DitConfig):
        self.cfg = cfg
        c = _CConfig(**asdict(cfg))
        h = ctypes.c_void_p()
        check(lib.mkb_dit_create(ctypes.byref(c), ctypes.byref(h)))
        self.h = h
        self._probe = None
        self.grid = None

    def close(self):
        if self.h:
            lib.mkb_dit_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def init_random(self, seed, std=0.02):
        check(lib.mkb_dit_init_random(self.h, seed, std))

    def weight_names(self):
        out = []
        name, r, c = ctypes.c_char_p(), ctypes.c_long(), ctypes.c_long()
        for i in range(lib.mkb_dit_weight_count(self.h)):
            check(lib.mkb_dit_weight_info(self.h, i, ctypes.byref(name), ctypes.byref(r), ctypes.byref(c)))
            out.append((name.value.decode(), (r.value, c.value) if c.value else (r.value,)))
        return out

    def read_weight(self, name, shape):
        a = np.empty(shape, np.float32)
        check(lib.mkb_dit_weight_read(self.h, name.encode(), _fptr(a)))
        return a

    def write_weight(self, name, a):
        a = np.ascontiguousarray(a, np.float32)
        check(lib.mkb_dit_weight_write(self.h, name.encode(), _fptr(a)))

    def weights(self):
        return {n: self.read_weight(n, s) for n, s in self.weight_names()}

    def begin(self, prompt, h, w, slot=0):
        p = np.ascontiguousarray(prompt, np.float32)
        check(lib.mkb_dit_begin(self.h, _fptr(p), p.shape[0], h, w, slot))
        self.grid = (h, w)

    def step(self, latents, sigma, slot=0):
        x = np.ascontiguousarray(latents, np.float32)
        out = np.empty_like(x)
        check(lib.mkb_dit_step(self.h, _fptr(x), sigma, _fptr(out), slot))
        return out

    def step_batch(self, slots, latents, sigmas):
        n = len(slots)
        x = np.ascontiguousarray(latents, np.float32)
        out = np.empty_like(x)
        sl = (ctypes.c_int * n)(*slots)
        sg = (ctypes.c_float * n)(*sigmas)
        check(lib.mkb_dit_step_batch(self.h, n, sl, _fptr(x), sg, _fptr(out)))
        return out

    def step_batch_dev(self, slots, latents_dev, sigmas, out_dev, stream=None):
        n = len(slots)
        sl = (ctypes.c_int * n)(*slots)
        sg = (ctypes.c_float * n)(*sigmas)
        check(lib.mkb_dit_step_batch_dev(self.h, n, sl, ctypes.c_void_p(latents_dev), sg, ctypes.c_void_p(out_dev),
                                         stream))

    def step_cfg(self, latents, sigma, sigma_next, guidance):
        """One guided Euler step on host latents [N][64] (slots 0 / 1 = cond / uncond); returns the new latents."""
        x = np.array(latents, np.float32, copy=True, order="C")
        check(lib.mkb_dit_step_cfg(self.h, _fptr(x), sigma, sigma_next, guidance))
        return x

    def step_cfg_inplace(self, latents):
        """step_cfg on a caller-owned C-contiguous float32 array (e.g. a pinned buffer), updated in place."""

        def run(sigma, sigma_next, guidance):
            check(lib.mkb_dit_step_cfg(self.h, _fptr(latents), sigma, sigma_next, guidance))

        return run

    def step_cfg_dev(self, n_images, latents_dev, sigma, sigma_next, guidance, stream=None):
        check(lib.mkb_dit_step_cfg_dev(self.h, n_images, ctypes.c_void_p(latents_dev), sigma, sigma_next, guidance,
                                       stream))

    def guided_velocity_dev(self, n_images, latents_dev, sigma, guidance, v_out_dev, stream=None):
        """The guided velocity of the CFG batch into v_out_dev (device pointers), latents unchanged."""
        check(lib.mkb_dit_guided_velocity_dev(self.h, n_images, ctypes.c_void_p(latents_dev), sigma, guidance,
                                              ctypes.c_void_p(v_out_dev), stream))

    def set_probe(self, fn):
        """fn(name, layer, array) is called with host copies of named stages; None turns probing off."""
        if fn is None:
            self._probe = None
            check(lib.mkb_dit_set_probe(self.h, None, None))
            return

        def tramp(name, layer, data, count, user):
            fn(name.decode(), layer, np.ctypeslib.as_array(data, shape=(count,)).copy())

        self._probe = _PROBE_FN(tramp)
        check(lib.mkb_dit_set_probe(self.h, ctypes.cast(self._probe, ctypes.c_void_p), None))

    def step_flops(self, n, first_step=True):
        return lib.mkb_dit_step_flops(self.h, n, int(first_step))

    def load_safetensors(self, paths, strict=True):
        """Loads checkpoint files by their tensor names (mkb_dit_load_safetensors); returns the tensors written."""
        if isinstance(paths, (str, bytes, os.PathLike)):
            paths = [paths]
        arr = (ctypes.c_char_p * len(paths))(*[str(p).encode() for p in paths])
        n = ctypes.c_int()
        check(lib.mkb_dit_load_safetensors(self.h, arr, len(paths), int(strict), ctypes.byref(n)))
        return n.value

    def lora_merge(self, module, A, B, scale=1.0):
        """W += scale * B A for module `module` (A [rank][in], B [out][rank])."""
        A = np.ascontiguousarray(A, np.float32)
        B = np.ascontiguousarray(B, np.float32)
        if A.ndim != 2 or B.ndim != 2 or B.shape[1] != A.shape[0]:
            raise ValueError(f"lora_merge: A {A.shape} and B {B.shape} are not [rank][in] and [out][rank]")
        check(lib.mkb_dit_lora_merge(self.h, module.encode(), _fptr(A), _fptr(B), A.shape[0], A.shape[1], B.shape[0],
                                     scale))

    def load_lora(self, path, scale=1.0):
        """Merges every pair of a LoRA safetensors file; returns the number of modules."""
        n = ctypes.c_int()
        check(lib.mkb_dit_load_lora(self.h, str(path).encode(), scale, ctypes.byref(n)))
        return n.value

    def set_sequence_parallel(self, nccl_id: bytes, rank: int, world: int):
        """Joins this handle to a sequence-parallel group (collective over the `world` ranks; see
        mkb_dit_set_sequence_parallel). nccl_id comes from nccl_unique_id() on one rank."""
        buf = ctypes.create_string_buffer(bytes(nccl_id), NCCL_ID_BYTES)
        check(lib.mkb_dit_set_sequence_parallel(self.h, buf, rank, world))

    def set_peer_exchange(self, enable: bool = True):
        """Moves the per-block K/V exchange from the NCCL all-gather to copy-engine pushes into the peers' memory
        (collective; see mkb_dit_sp_peer_exchange)."""
        check(lib.mkb_dit_sp_peer_exchange(self.h, int(bool(enable))))

    def set_head_exchange(self, mode: int = 1):
        """Replaces the per-block K/V all-gather by the head-parallel exchange: each rank attends over all rows of
        heads / world heads, the rows reaching it by NCCL all-to-alls (mode 1) or by stores into the peers' memory
        from the QKV and attention epilogues (mode 2); 0 goes back (collective; see mkb_dit_sp_head_exchange)."""
        check(lib.mkb_dit_sp_head_exchange(self.h, int(mode)))


NCCL_ID_BYTES = 128


def nccl_unique_id() -> bytes:
    """A fresh NCCL communicator id (NCCL_ID_BYTES bytes) for set_sequence_parallel."""
    buf = ctypes.create_string_buffer(NCCL_ID_BYTES)
    check(lib.mkb_nccl_unique_id(buf, NCCL_ID_BYTES))
    return buf.raw


def sp_rows(S, N, world, rank):
    """(text_rows, image_rows, image_row0, shard_rows) that rank `rank` of `world` owns (mkb_dit_sp_rows)."""
    out = [ctypes.c_int() for _ in range(4)]
    check(lib.mkb_dit_sp_rows(S, N, world, rank, *[ctypes.byref(o) for o in out]))
    return tuple(o.value for o in out)


def st_read(path):
    """Every tensor of a safetensors file as {name: (dtype, float32 array)} through the library's reader."""
    h = ctypes.c_void_p()
    check(lib.mkb_st_open(str(path).encode(), ctypes.byref(h)))
    try:
        out = {}
        name, dtype = ctypes.c_char_p(), ctypes.c_char_p()
        dims, nd = (ctypes.c_int64 * 8)(), ctypes.c_int()
        for i in range(lib.mkb_st_count(h)):
            check(lib.mkb_st_info(h, i, ctypes.byref(name), ctypes.byref(dtype), dims, ctypes.byref(nd)))
            shape = tuple(dims[k] for k in range(nd.value))
            a = np.empty(shape, np.float32)
            check(lib.mkb_st_read_f32(h, name.value, _fptr(a), a.size))
            out[name.value.decode()] = (dtype.value.decode(), a)
        return out
    finally:
        lib.mkb_st_close(h)
