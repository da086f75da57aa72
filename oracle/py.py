"""ctypes wrapper of liboracle (TEST INFRASTRUCTURE ONLY: the checker, never the product)."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.environ.get("VKB_ORACLE_LIB") or os.path.join(_HERE, "libvkb_oracle.so")
_l = None


def lib():
    global _l
    if _l is None:
        if not os.path.exists(LIB):
            import subprocess
            subprocess.run(["make", "-C", _HERE], check=True, capture_output=True)
        _l = C.CDLL(LIB)
        P = C.c_void_p
        sig = {
            "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
            "orc_f32_to_f16": (C.c_uint16, [C.c_float]),
            "orc_kv_block_bytes": (C.c_int, [C.c_int]),
            "orc_kv_pack": (C.c_int, [C.c_int, P, C.c_size_t, P]),
            "orc_kv_unpack": (C.c_int, [C.c_int, P, C.c_size_t, P]),
            "orc_dequant_gemv": (C.c_int, [C.c_int, P, C.c_size_t, C.c_size_t, C.c_size_t, P, C.c_size_t, P]),
            "orc_payload_size": (C.c_int64, [C.c_uint32, C.c_uint64]),
            "orc_dequantize": (C.c_int, [C.c_uint32, P, C.c_size_t, C.c_size_t, P]),
            "orc_quantize": (C.c_int, [C.c_uint32, P, C.c_size_t, P]),
            "orc_set_threads": (None, [C.c_int]),
            "orc_linear_f32": (None, [C.c_int, C.c_int, C.c_int, P, P, P, P]),
            "orc_gemm_f32": (None, [C.c_int, C.c_int, C.c_int, P, P, P, P]),
            "orc_linear_q": (C.c_int, [C.c_uint32, C.c_int, C.c_int, C.c_int, P, P, C.c_size_t, P, P]),
            "orc_kquant_gemm_i8": (C.c_int, [C.c_uint32, C.c_int, C.c_int, C.c_int, P, P, C.c_size_t, P, P]),
            "orc_int8_error_bound": (C.c_float, [C.c_uint32, P, C.c_int, P]),
            "orc_gelu1": (C.c_float, [C.c_float]),
            "orc_erf": (C.c_float, [C.c_float]),
            "orc_gelu": (None, [P, P, C.c_size_t]),
            "orc_layer_norm": (None, [P, P, C.c_int, C.c_int, P, P, C.c_float]),
            "orc_attention": (None, [P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P]),
            "orc_conv1d": (None, [P, C.c_int, C.c_int, P, C.c_int, C.c_int, P, C.c_int, C.c_int, P]),
            "orc_pkv_create": (P, [C.c_int] * 8),
            "orc_pkv_destroy": (None, [P]),
            "orc_pkv_append": (C.c_int, [P, C.c_int, C.c_int, C.c_int, C.c_int, P, P]),
            "orc_pkv_read": (C.c_int, [P, C.c_int, C.c_int, C.c_int, C.c_int, P, P]),
            "orc_pkv_reset": (None, [P]),
            "orc_pkv_release_layer": (C.c_int, [P, C.c_int]),
            "orc_pkv_table_len": (C.c_int, [P]),
            "orc_pkv_table": (None, [P, P]),
            "orc_pkv_pages_in_use": (C.c_int, [P]),
            "orc_pkv_page_bytes": (C.c_size_t, [P]),
            "orc_pkv_on_wire_bytes": (C.c_size_t, [P]),
            "orc_pkv_page": (None, [P, C.c_int, P, P]),
            "orc_mel_filterbank": (None, [C.c_int, C.c_int, C.c_double, C.c_double, C.c_double, P]),
            "orc_hann_periodic": (None, [C.c_int, P]),
            "orc_log_mel_raw": (C.c_float, [P, C.c_int64, C.c_int, P]),
            "orc_log_mel": (None, [P, C.c_int64, C.c_int, P]),
        }
        for n, (r, a) in sig.items():
            f = getattr(_l, n)
            f.restype = r
            f.argtypes = a
    return _l


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def u8(a):
    return np.ascontiguousarray(np.frombuffer(a, dtype=np.uint8) if isinstance(a, (bytes, bytearray)) else a,
                                dtype=np.uint8)


def f32_to_f16(x: float) -> int:
    return int(lib().orc_f32_to_f16(C.c_float(x)))


def f16_to_f32(h: int) -> float:
    return float(lib().orc_f16_to_f32(h))


def kv_pack(mode: int, x) -> np.ndarray:
    x = f32(x).reshape(-1)
    bb = lib().orc_kv_block_bytes(mode)
    out = np.zeros(x.size // 32 * bb, np.uint8)
    rc = lib().orc_kv_pack(mode, _p(x), x.size // 32, _p(out))
    assert rc == 0
    return out


def kv_unpack(mode: int, b) -> np.ndarray:
    b = u8(b)
    bb = lib().orc_kv_block_bytes(mode)
    out = np.zeros(b.size // bb * 32, np.float32)
    rc = lib().orc_kv_unpack(mode, _p(b), b.size, _p(out))
    assert rc == 0
    return out


def dequant_gemv(mode, blocks, n_rows, nbpr, x):
    b = u8(blocks)
    x = f32(x)
    y = np.zeros(n_rows, np.float32)
    rc = lib().orc_dequant_gemv(mode, _p(b), b.size, n_rows, nbpr, _p(x), x.size, _p(y))
    return rc, y


def dequantize(tag, data, n):
    b = u8(data)
    out = np.zeros(n, np.float32)
    rc = lib().orc_dequantize(tag, _p(b), b.size, n, _p(out))
    if rc:
        raise ValueError(f"dequantize rc={rc}")
    return out


def quantize(tag, x):
    x = f32(x).reshape(-1)
    nbytes = lib().orc_payload_size(tag, x.size)
    out = np.zeros(nbytes, np.uint8)
    rc = lib().orc_quantize(tag, _p(x), x.size, _p(out))
    assert rc == 0, rc
    return out


def linear_q(tag, a, wq, n, k, bias=None):
    a = f32(a)
    m = a.size // k
    w = u8(wq)
    out = np.zeros((m, n), np.float32)
    rc = lib().orc_linear_q(tag, m, n, k, _p(a), _p(w), w.size, _p(None if bias is None else f32(bias)), _p(out))
    assert rc == 0, rc
    return out


def linear_f32(a, w, bias=None):
    a = f32(a)
    w = f32(w)
    n, k = w.shape
    m = a.size // k
    out = np.zeros((m, n), np.float32)
    lib().orc_linear_f32(m, n, k, _p(a), _p(w), _p(None if bias is None else f32(bias)), _p(out))
    return out


def gemm_kn(a, wt, bias=None):
    """gemm_f32 with a pre-transposed [k][n] weight (the reference's load-time layout)."""
    a = f32(a)
    wt = f32(wt)
    k, n = wt.shape
    m = a.size // k
    out = np.zeros((m, n), np.float32)
    lib().orc_gemm_f32(m, n, k, _p(a), _p(wt), _p(None if bias is None else f32(bias)), _p(out))
    return out


def kquant_gemm_i8(tag, a, wq, n, k, bias=None):
    a = f32(a)
    m = a.size // k
    w = u8(wq)
    out = np.zeros((m, n), np.float32)
    rc = lib().orc_kquant_gemm_i8(tag, m, n, k, _p(a), _p(w), w.size, _p(None if bias is None else f32(bias)),
                                  _p(out))
    assert rc == 0, rc
    return out


def int8_error_bound(tag, w_row, k, x):
    w = u8(w_row)
    x = f32(x)
    return float(lib().orc_int8_error_bound(tag, _p(w), k, _p(x)))


def erf(x: float) -> float:
    return float(lib().orc_erf(C.c_float(x)))


def gelu(x):
    x = f32(x)
    y = np.zeros_like(x)
    lib().orc_gelu(_p(x), _p(y), x.size)
    return y


def layer_norm(x, g, b, eps=1e-5):
    x = f32(x)
    rows, cols = x.shape
    y = np.zeros_like(x)
    lib().orc_layer_norm(_p(x), _p(y), rows, cols, _p(f32(g)), _p(f32(b)), C.c_float(eps))
    return y


def attention(q, k, v, n_head, causal=False, q_off=0):
    q, k, v = f32(q), f32(k), f32(v)
    t_q, d = q.shape
    t_kv = k.shape[0]
    ctx = np.zeros_like(q)
    lib().orc_attention(_p(q), _p(k), _p(v), t_q, t_kv, d, n_head, int(causal), q_off, _p(ctx))
    return ctx


def conv1d(x, w, bias, stride, pad):
    x = f32(x)
    w = f32(w)
    in_ch, in_len = x.shape
    out_ch, _, kern = w.shape
    out_len = (in_len + 2 * pad - kern) // stride + 1
    out = np.zeros((out_ch, out_len), np.float32)
    lib().orc_conv1d(_p(x), in_ch, in_len, _p(w), out_ch, kern, _p(None if bias is None else f32(bias)), stride, pad,
                     _p(out))
    return out


class PagedKv:
    """Oracle QuantizedPagedKvCache (cache/paged_quant.rs)."""

    def __init__(self, n_layer, n_head, d_head, n_stream, n_codebook, max_time, bs, mode):
        self.h = lib().orc_pkv_create(n_layer, n_head, d_head, n_stream, n_codebook, max_time, bs, mode)
        if not self.h:
            raise ValueError("invalid paged cache configuration")
        self.w = n_head * d_head

    def append_step(self, layer, t, s, c, k, v):
        return lib().orc_pkv_append(self.h, layer, t, s, c, _p(f32(k)), _p(f32(v)))

    def read_step(self, layer, t, s, c=0):
        k = np.zeros(self.w, np.float32)
        v = np.zeros(self.w, np.float32)
        if lib().orc_pkv_read(self.h, layer, t, s, c, _p(k), _p(v)):
            return k, v
        return None

    def reset(self):
        lib().orc_pkv_reset(self.h)

    def release_layer(self, layer):
        return lib().orc_pkv_release_layer(self.h, layer)

    def page_table(self):
        n = lib().orc_pkv_table_len(self.h)
        out = np.zeros(n, np.int64)
        lib().orc_pkv_table(self.h, _p(out))
        return out

    def pages_in_use(self):
        return lib().orc_pkv_pages_in_use(self.h)

    def on_wire_storage_bytes(self):
        return lib().orc_pkv_on_wire_bytes(self.h)

    def page(self, pid):
        n = lib().orc_pkv_page_bytes(self.h)
        k = np.zeros(n, np.uint8)
        v = np.zeros(n, np.uint8)
        lib().orc_pkv_page(self.h, pid, _p(k), _p(v))
        return k, v

    def __del__(self):
        try:
            lib().orc_pkv_destroy(self.h)
        except Exception:
            pass


def mel_filterbank(n_mels: int, n_fft: int = 400, sr: float = 16000.0, fmin: float = 0.0, fmax: float = 8000.0):
    """MelFilterbank::new (Slaney scale and norm, Hz interpolation): [n_mels, n_fft/2+1] f32."""
    w = np.empty((n_mels, n_fft // 2 + 1), np.float32)
    lib().orc_mel_filterbank(n_fft, n_mels, sr, fmin, fmax, _p(w))
    return w


def hann_periodic(n: int):
    w = np.empty(n, np.float32)
    lib().orc_hann_periodic(n, _p(w))
    return w


def log_mel(pcm, n_mels: int):
    """whisper::mel::log_mel: [n_mels, 3000] log-mel features of one clip of 16 kHz PCM."""
    x = np.ascontiguousarray(pcm, dtype=np.float32)
    out = np.empty((n_mels, 3000), np.float32)
    lib().orc_log_mel(_p(x) if x.size else None, x.size, n_mels, _p(out))
    return out
