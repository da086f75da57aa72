"""ctypes binding of libvkb200.so (the C ABI declared in include/vkb200.h).

The library is built in-tree by ``vokra_b200/csrc/Makefile`` (``build()`` in
``__graft_entry__.py``). Loading fails loudly when it is missing: there is no
fallback implementation of any entry point.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# VKB_LIB_PATH selects another build of the same library (the sanitizer build)
LIB_PATH = os.environ.get("VKB_LIB_PATH") or os.path.join(_HERE, "libvkb200.so")

# Status codes (vkb_status == vokra_status_t numbering, include/vokra.h:58-78).
OK = 0
ERROR_IO = 1
ERROR_MODEL_LOAD = 2
ERROR_UNSUPPORTED_OP = 3
ERROR_BACKEND_UNAVAILABLE = 4
ERROR_INVALID_ARGUMENT = 5
ERROR_GRAPH_VALIDATION = 6
ERROR_NOT_IMPLEMENTED = 7
ERROR_PANIC = 8
ERROR_OTHER = 9
ERROR_KV_CACHE_EXHAUSTED = 10

STATUS_NAMES = {
    0: "OK", 1: "Io", 2: "ModelLoad", 3: "UnsupportedOp", 4: "BackendUnavailable",
    5: "InvalidArgument", 6: "GraphValidation", 7: "NotImplemented", 8: "Panic",
    9: "Other", 10: "KvCacheExhausted",
}

# ggml dtype tags
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_BF16 = 0, 1, 2, 8, 12, 13, 14, 30
# KvQuant
KV_FP32, KV_Q4_0, KV_Q5_0, KV_Q8_0 = 0, 1, 2, 3
DT_F32, DT_F16, DT_F16X2 = 0, 1, 2
PREC_SPLIT, PREC_F16, PREC_ENCODER_F16 = 0, 1, 2
EPI_NONE, EPI_GELU, EPI_RESIDUAL, EPI_SCALE = 0, 1, 2, 3
KV_LAYOUT_REFERENCE, KV_LAYOUT_SEQUENCE = 0, 1


class VkbError(RuntimeError):
    """A non-OK vkb_status, carrying the code and vkb_last_error()."""

    def __init__(self, code: int, message: str):
        self.code = code
        self.kind = STATUS_NAMES.get(code, str(code))
        super().__init__(f"{self.kind}: {message}")


class KvPoolDesc(C.Structure):
    _fields_ = [
        ("n_layer", C.c_int32), ("n_head", C.c_int32), ("d_head", C.c_int32),
        ("n_stream", C.c_int32), ("n_codebook", C.c_int32), ("max_time", C.c_int32),
        ("page_tokens", C.c_int32), ("mode", C.c_int32), ("layout", C.c_int32),
        ("n_pages", C.c_int32),
    ]


SELF_KV_Q8_0, SELF_KV_F32, SELF_KV_Q4_0, SELF_KV_Q5_0 = 0, 1, 2, 3


class SessionOptions(C.Structure):
    _fields_ = [("max_streams", C.c_int32), ("max_step_tokens", C.c_int32), ("max_clips", C.c_int32),
                ("cross_kv_q8", C.c_int32), ("kv_page_tokens", C.c_int32), ("self_kv_mode", C.c_int32)]


class WhisperDims(C.Structure):
    _fields_ = [
        ("n_mels", C.c_int32), ("n_audio_ctx", C.c_int32), ("d_model", C.c_int32),
        ("n_audio_head", C.c_int32), ("n_audio_layer", C.c_int32), ("n_text_ctx", C.c_int32),
        ("n_text_head", C.c_int32), ("n_text_layer", C.c_int32), ("n_vocab", C.c_int32),
        ("ffn_dim", C.c_int32), ("eot", C.c_int32), ("n_start_ids", C.c_int32),
        ("start_ids", C.c_int32 * 8),
    ]


P = C.c_void_p
I32, I64, U32, U64, SZ, F32 = C.c_int32, C.c_int64, C.c_uint32, C.c_uint64, C.c_size_t, C.c_float
PP = C.POINTER(C.c_void_p)

# name -> (restype, argtypes). Every symbol declared in include/vkb200.h.
SIGNATURES = {
    "vkb_last_error": (C.c_char_p, []),
    "vkb_abi_version": (C.c_int, []),
    "vkb_context_create": (C.c_int, [C.c_int, PP]),
    "vkb_context_destroy": (C.c_int, [P]),
    "vkb_context_set_stream": (C.c_int, [P, P]),
    "vkb_context_synchronize": (C.c_int, [P]),
    "vkb_context_launch_count": (U64, [P]),
    "vkb_context_workspace_bytes": (SZ, [P]),
    "vkb_context_set_precision": (C.c_int, [P, C.c_int]),
    "vkb_weight_upload": (C.c_int, [P, U32, I64, I64, P, SZ, PP]),
    "vkb_weight_destroy": (C.c_int, [P]),
    "vkb_weight_device_bytes": (SZ, [P]),
    "vkb_linear": (C.c_int, [P, P, I64, P, C.c_int, P, P, C.c_int, C.c_int, P, F32]),
    "vkb_gemm_q_f32": (C.c_int, [P, I64, I64, I64, P, P, SZ, U32, P, P]),
    "vkb_kv_dequant_gemv": (C.c_int, [P, C.c_int, P, SZ, SZ, SZ, P, SZ, P]),
    "vkb_kv_dequant_gemv_host": (C.c_int, [P, C.c_int, P, SZ, SZ, SZ, P, SZ, P]),
    "vkb_kv_pool_create": (C.c_int, [P, C.POINTER(KvPoolDesc), PP]),
    "vkb_kv_pool_destroy": (C.c_int, [P]),
    "vkb_kv_begin_step": (C.c_int, [P, I32, P, P]),
    "vkb_kv_append": (C.c_int, [P, I32, P, P]),
    "vkb_kv_attention": (C.c_int, [P, I32, P, P, C.c_int]),
    "vkb_kv_append_attention": (C.c_int, [P, I32, P, I64, P, C.c_int]),
    "vkb_kv_decode_fused": (I32, [P]),
    "vkb_gguf_inspect": (C.c_int, [P, SZ, P, P]),
    "vkb_kv_copy_stream": (C.c_int, [P, I32, I32, I32]),
    "vkb_context_selftest_bounded_wait": (C.c_int, [P, U32]),
    "vkb_kv_release_seq": (C.c_int, [P, I32]),
    "vkb_kv_release_layer": (C.c_int, [P, I32]),
    "vkb_kv_reset": (C.c_int, [P]),
    "vkb_kv_set_page_table": (C.c_int, [P, P, SZ]),
    "vkb_kv_table_len": (SZ, [P]),
    "vkb_kv_page_table": (C.c_int, [P, P, SZ]),
    "vkb_kv_pages_in_use": (I32, [P]),
    "vkb_kv_page_bytes": (SZ, [P]),
    "vkb_kv_on_wire_bytes": (SZ, [P]),
    "vkb_kv_read_page": (C.c_int, [P, I32, I32, P, P]),
    "vkb_kv_read_step": (C.c_int, [P, I32, I32, I32, P, P]),
    "vkb_attention_dense": (C.c_int, [P, I32, I32, I32, P, P, P, P, P, P, I32, I32, P, I32]),
    "vkb_log_mel": (C.c_int, [P, P, I64, I64, P, I32, P]),
    "vkb_session_copy_stream": (C.c_int, [P, I32, I32, I32, I32]),
    "vkb_session_cross_kv": (C.c_int, [P, I32, P, P, P, P]),
    "vkb_quantize_rows_q8_0": (C.c_int, [P, P, I64, I32, P, P]),
    "vkb_attention_dense_noalloc": (C.c_int, [P, I32, I32, I32, P, P, P, P, P, P, I32, I32, P, I32]),
    "vkb_whisper_load": (C.c_int, [P, C.c_char_p, PP]),
    "vkb_whisper_get_dims": (C.c_int, [P, C.POINTER(WhisperDims)]),
    "vkb_whisper_destroy": (C.c_int, [P]),
    "vkb_session_create": (C.c_int, [P, C.POINTER(SessionOptions), PP]),
    "vkb_session_destroy": (C.c_int, [P]),
    "vkb_session_encode": (C.c_int, [P, I32, P, P]),
    "vkb_session_encoder_output": (P, [P]),
    "vkb_session_read_encoder_output": (C.c_int, [P, P, SZ]),
    "vkb_session_step": (C.c_int, [P, I32, P, P, P, P, P]),
    "vkb_session_step_feed": (C.c_int, [P, I32, P, P, P, P, P, P, P]),
    "vkb_session_logits": (P, [P]),
    "vkb_session_ids": (P, [P]),
    "vkb_session_release": (C.c_int, [P, I32]),
}

_lib = None


def load() -> C.CDLL:
    """Loads libvkb200.so once; raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build the CUDA library first "
            "(python -c 'import __graft_entry__ as g; g.build()' or make -C vokra_b200/csrc)")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int) -> None:
    if status != OK:
        msg = load().vkb_last_error()
        raise VkbError(status, msg.decode("utf-8", "replace") if msg else "")


def exported_symbols() -> list[str]:
    """The vkb_* names the loaded library actually exports."""
    lib = load()
    return [n for n in SIGNATURES if hasattr(lib, n)]
