"""vokra_b200 — B200-native (sm_100a) quantized-Whisper hot path behind vokra's seams.

The product is ``libvkb200.so`` (CUDA kernels + the C ABI in include/vkb200.h);
this package is its Python host mirror. Importing it loads the library and
fails loudly if it was not built — there is no CPU fallback.
"""
from ._lib import load as _load, VkbError, LIB_PATH  # noqa: F401

_load()

__all__ = ["VkbError", "LIB_PATH"]
