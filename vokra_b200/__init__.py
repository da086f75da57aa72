"""vokra_b200 — B200-native (sm_100a) quantized-Whisper hot path behind vokra's seams.

The product is ``libvkb200.so`` (CUDA kernels + the C ABI in include/vkb200.h);
the modules of this package are its Python host mirror. ``ops``, ``whisper``
and ``beam`` load the library when they are imported (``batching`` when it
runs) and fail loudly if it was not built — there is no CPU fallback. ``synth`` (the GGUF
writer and quantizers used to make synthetic checkpoints) is plain numpy and
loads nothing, so tooling that only writes model files does not pull the
library into its process.
"""

__all__ = ["ops", "whisper", "beam", "batching", "synth"]
