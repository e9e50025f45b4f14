"""ctypes loader for libmkb_image.so. Importing fails loudly when the library has not been built: there is no
fallback implementation."""

import ctypes
import os

# MKB_IMAGE_LIB overrides the in-tree build (an alternative build of the same library, e.g. for A/B timing).
LIB_PATH = os.environ.get("MKB_IMAGE_LIB") or os.path.join(
    os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "lib", "libmkb_image.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with `make -C mako-image_b200` (or __graft_entry__.build())")

lib = ctypes.CDLL(LIB_PATH)

_vp, _i, _l, _f, _u64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_long, ctypes.c_float, ctypes.c_uint64
_u32p = ctypes.POINTER(ctypes.c_uint32)

_SIGS = {
    "mkb_last_error": (ctypes.c_char_p, []),
    "mkb_kernel_launches": (_u64, []),
    "mkb_proj": (_i, [_vp, _l, _vp, _l, _vp, _vp, _l, _i, _i, _i, _i, _i, _vp]),
    "mkb_proj_gate_add": (_i, [_vp, _l, _vp, _l, _vp, _vp, _l, _vp, _l, _i, _i, _i, _i, _i, _vp]),
    "mkb_proj_qkv_heads": (_i, [_vp, _l, _vp, _l, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _i, _i, _vp]),
    "mkb_proj_swiglu": (_i, [_vp, _l, _vp, _l, _vp, _vp, _l, _i, _i, _i, _vp]),
    "mkb_swiglu_interleave": (_i, []),
    "mkb_check_kernels": (_i, [_u32p]),
    "mkb_selftest_stalled_gemm": (_i, [_vp, _l, _vp, _l, _vp, _l, _i, _i, _i, _vp]),
    "mkb_selftest_peer_wait": (_i, [_vp, _i, _i, _vp, _vp]),
    "mkb_proj_add": (_i, [_vp, _l, _vp, _l, _vp, _vp, _l, _i, _vp, _l, _vp, _l, _i, _i, _i, _i, _vp]),
    "mkb_proj_heads": (_i, [_vp, _l, _vp, _l, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "mkb_proj_geglu": (_i, [_vp, _l, _vp, _l, _vp, _vp, _l, _i, _i, _i, _vp]),
    "mkb_conv2d": (_i, [_vp, _i, _i, _i, _i, _vp, _i, _i, _i, _vp, _vp, _l, _vp, _l, _vp, _l, _i, _vp]),
    "mkb_ln_modulate": (_i, [_vp, _vp, _vp, _vp, _l, _i, _f, _l, _l, _l, _vp]),
    "mkb_group_norm_workspace_size": (ctypes.c_size_t, [_i, _i, _i, _i]),
    "mkb_group_norm": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _i, _vp, ctypes.c_size_t, _vp]),
    "mkb_group_norm_static_max_bytes": (ctypes.c_size_t, []),
    "mkb_group_norm_static": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _i, _vp]),
    "mkb_dit_create": (_i, [_vp, ctypes.POINTER(_vp)]),
    "mkb_dit_destroy": (None, [_vp]),
    "mkb_dit_init_random": (_i, [_vp, _u64, _f]),
    "mkb_dit_weight_count": (_i, [_vp]),
    "mkb_dit_weight_info": (_i, [_vp, _i, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_l), ctypes.POINTER(_l)]),
    "mkb_dit_weight_read": (_i, [_vp, ctypes.c_char_p, _vp]),
    "mkb_dit_weight_write": (_i, [_vp, ctypes.c_char_p, _vp]),
    "mkb_dit_begin": (_i, [_vp, _vp, _i, _i, _i, _i]),
    "mkb_dit_step": (_i, [_vp, _vp, _f, _vp, _i]),
    "mkb_dit_step_batch": (_i, [_vp, _i, _vp, _vp, _vp, _vp]),
    "mkb_dit_step_batch_dev": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _vp]),
    "mkb_dit_step_cfg": (_i, [_vp, _vp, _f, _f, _f]),
    "mkb_dit_step_cfg_dev": (_i, [_vp, _i, _vp, _f, _f, _f, _vp]),
    "mkb_dit_set_probe": (_i, [_vp, _vp, _vp]),
    "mkb_dit_step_flops": (ctypes.c_double, [_vp, _i, _i]),
    "mkb_schedule_default": (None, [_vp]),
    "mkb_unet_create": (_i, [_vp, ctypes.POINTER(_vp)]),
    "mkb_unet_destroy": (None, [_vp]),
    "mkb_unet_init_random": (_i, [_vp, _u64, _f]),
    "mkb_unet_weight_count": (_i, [_vp]),
    "mkb_unet_weight_info": (_i, [_vp, _i, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_l), ctypes.POINTER(_i)]),
    "mkb_unet_weight_read": (_i, [_vp, ctypes.c_char_p, _vp]),
    "mkb_unet_weight_write": (_i, [_vp, ctypes.c_char_p, _vp]),
    "mkb_unet_begin": (_i, [_vp, _vp, _i, _vp, _i, _i, _i]),
    "mkb_unet_step": (_i, [_vp, _vp, _f, _vp, _i]),
    "mkb_unet_step_batch": (_i, [_vp, _i, _i, _vp, _vp, _vp]),
    "mkb_unet_step_batch_dev": (_i, [_vp, _i, _i, _vp, _vp, _vp, _vp]),
    "mkb_unet_step_cfg_dev": (_i, [_vp, _vp, _f, _f, _f, _vp]),
    "mkb_unet_set_probe": (_i, [_vp, _vp, _vp]),
    "mkb_unet_step_flops": (ctypes.c_double, [_vp, _i]),
    "mkb_sdxl_sigmas": (_i, [ctypes.c_uint32, _vp]),
    "mkb_sdxl_timestep": (_i, [_f]),
    "mkb_vae_create": (_i, [_vp, ctypes.POINTER(_vp)]),
    "mkb_vae_destroy": (None, [_vp]),
    "mkb_vae_init_random": (_i, [_vp, _u64, _f]),
    "mkb_vae_weight_count": (_i, [_vp]),
    "mkb_vae_weight_info": (_i, [_vp, _i, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_l), ctypes.POINTER(_i)]),
    "mkb_vae_weight_read": (_i, [_vp, ctypes.c_char_p, _vp]),
    "mkb_vae_weight_write": (_i, [_vp, ctypes.c_char_p, _vp]),
    "mkb_vae_decode": (_i, [_vp, _vp, _i, _i, _vp]),
    "mkb_vae_decode_dev": (_i, [_vp, _vp, _i, _i, _vp, _vp]),
    "mkb_vae_set_probe": (_i, [_vp, _vp, _vp]),
    "mkb_vae_decode_flops": (ctypes.c_double, [_vp, _i, _i]),
    "mkb_vae_set_latent_stats": (_i, [_vp, _vp, _vp, _i]),
    "mkb_clip_create": (_i, [_vp, ctypes.POINTER(_vp)]),
    "mkb_clip_destroy": (None, [_vp]),
    "mkb_clip_init_random": (_i, [_vp, _u64, _f]),
    "mkb_clip_weight_count": (_i, [_vp]),
    "mkb_clip_weight_info": (_i, [_vp, _i, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_l), ctypes.POINTER(_i)]),
    "mkb_clip_weight_read": (_i, [_vp, ctypes.c_char_p, _vp]),
    "mkb_clip_weight_write": (_i, [_vp, ctypes.c_char_p, _vp]),
    "mkb_clip_load_safetensors": (_i, [_vp, ctypes.POINTER(ctypes.c_char_p), _i, _i, ctypes.POINTER(_i)]),
    "mkb_clip_set_probe": (_i, [_vp, _vp, _vp]),
    "mkb_clip_encode": (_i, [_vp, _vp, _i, _vp, _vp]),
    "mkb_sdxl_prompt_embeddings": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _vp, _vp]),
    "mkb_to_rgba8": (_i, [_vp, ctypes.c_size_t, _vp]),
    "mkb_png_encode": (_i, [_vp, ctypes.c_uint32, ctypes.c_uint32, _i, _vp, ctypes.c_size_t,
                            ctypes.POINTER(ctypes.c_size_t)]),
    "mkb_sigmas": (_i, [_vp, ctypes.c_uint32, ctypes.c_uint32, _vp]),
    "mkb_top_sigma": (_f, [_vp, ctypes.c_uint32]),
    "mkb_guided_euler": (None, [_vp, _vp, _vp, _f, _f, _f, _l]),
    "mkb_er_sde_create": (_i, [_vp, _i, _i, _f, ctypes.POINTER(_vp)]),
    "mkb_er_sde_destroy": (None, [_vp]),
    "mkb_er_sde_sigma": (_f, [_vp, _i]),
    "mkb_er_sde_step": (_i, [_vp, _i, _vp, _vp, _vp, _l, _f]),
    "mkb_cfg_combine_dev": (_i, [_vp, _vp, _vp, _f, _l, _vp]),
    "mkb_axpy_dev": (_i, [_vp, _vp, _f, _l, _vp]),
    "mkb_euler_ancestral_dev": (_i, [_vp, _vp, _f, _f, _u64, _u64, _l, _vp]),
    "mkb_er_sde_step_dev": (_i, [_vp, _i, _vp, _vp, _vp, _u64, _u64, _l, _f, _vp]),
    "mkb_dit_guided_velocity_dev": (_i, [_vp, _i, _vp, _f, _f, _vp, _vp]),
    "mkb_attention": (_i, [_vp, _i, _i, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp, _l, _i, _vp, _l, _i, _vp]),
    "mkb_attention_kv_shards": (_i, [_vp, _i, _i, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp, _l, _i, _vp, _l,
                                     _i, _i, _i, _vp]),
    "mkb_attention_kv_arriving": (_i, [_vp, _i, _i, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp, _l, _i, _vp,
                                       _l, _i, _i, _i, _i, _vp, _vp, _vp]),
    "mkb_dit_sp_peer_exchange": (_i, [_vp, _i]),
    "mkb_dit_sp_head_exchange": (_i, [_vp, _i]),
    "mkb_attention_wide": (_i, [_vp, _l, _i, _i, _i, _i, _i, _vp, _l, _vp]),
    "mkb_nccl_unique_id": (_i, [_vp, ctypes.c_size_t]),
    "mkb_dit_variant": (_i, [_vp]),
    "mkb_unet_load_safetensors": (_i, [_vp, ctypes.POINTER(ctypes.c_char_p), _i, _i, ctypes.POINTER(_i)]),
    "mkb_vae_load_safetensors": (_i, [_vp, ctypes.POINTER(ctypes.c_char_p), _i, _i, ctypes.POINTER(_i)]),
    "mkb_unet_lora_merge": (_i, [_vp, ctypes.c_char_p, _vp, _vp, _i, _i, _i, _f]),
    "mkb_unet_load_lora": (_i, [_vp, ctypes.c_char_p, _f, ctypes.POINTER(_i)]),
    "mkb_unet_weight_lora_rows": (_i, [_vp, ctypes.c_char_p, _l, _l, _vp, _vp, _i, _f]),
    "mkb_dit_weight_write_rows": (_i, [_vp, ctypes.c_char_p, _l, _l, _vp]),
    "mkb_dit_weight_lora_rows": (_i, [_vp, ctypes.c_char_p, _l, _l, _vp, _vp, _i, _f]),
    "mkb_dit_load_safetensors": (_i, [_vp, ctypes.POINTER(ctypes.c_char_p), _i, _i, ctypes.POINTER(_i)]),
    "mkb_dit_lora_merge": (_i, [_vp, ctypes.c_char_p, _vp, _vp, _i, _i, _i, _f]),
    "mkb_dit_load_lora": (_i, [_vp, ctypes.c_char_p, _f, ctypes.POINTER(_i)]),
    "mkb_st_open": (_i, [ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "mkb_st_close": (None, [_vp]),
    "mkb_st_count": (_i, [_vp]),
    "mkb_st_info": (_i, [_vp, _i, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_char_p),
                         ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(_i)]),
    "mkb_st_read_f32": (_i, [_vp, ctypes.c_char_p, _vp, ctypes.c_int64]),
    "mkb_dit_set_sequence_parallel": (_i, [_vp, _vp, _i, _i]),
    "mkb_dit_sp_rows": (_i, [_i, _i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i), ctypes.POINTER(_i),
                             ctypes.POINTER(_i)]),
}


def _bind(name, restype, argtypes):
    fn = getattr(lib, name, None)
    if fn is None:
        return None
    fn.restype = restype
    fn.argtypes = argtypes
    return fn


for _name, (_res, _args) in _SIGS.items():
    _bind(_name, _res, _args)


class MkbError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"mkb error {code}: {msg}")
        self.code = code


def check(code):
    """Raise MkbError for a non-zero mkb_status."""
    if code != 0:
        raise MkbError(code, lib.mkb_last_error().decode())
    return code


def stream_ptr(stream=None):
    """The raw cudaStream_t of a torch stream (None: torch's current stream)."""
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)
