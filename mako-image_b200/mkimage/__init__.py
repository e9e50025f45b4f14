"""Python binding of libmkb_image.so (the C ABI in include/mkb_image.h), for the tests and the bench.

The library is the product; this module only loads it with ctypes and turns error codes into exceptions. Device
buffers are passed as raw pointers (for example ``tensor.data_ptr()`` of a torch CUDA tensor)."""

from ._lib import lib, MkbError, check, LIB_PATH, stream_ptr  # noqa: F401
from . import ops  # noqa: F401
from .dit import Dit, DitConfig, QWEN1, REF21, nccl_unique_id, sp_rows, NCCL_ID_BYTES, st_read  # noqa: F401
from .sdxl import Unet, UnetConfig, Vae, VaeConfig, Clip, ClipConfig, prompt_embeddings, sdxl_sigmas, sdxl_timestep  # noqa: F401,E501
from .sampler import Schedule, sigmas, top_sigma, guided_euler, ErSde, cfg_combine_dev, euler_ancestral_dev  # noqa: F401,E501
