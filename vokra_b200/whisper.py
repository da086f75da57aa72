"""Whisper on the B200 through the C ABI: model load and a batched decode session.

Mirrors the reference's ASR flow (crates/vokra-models/src/whisper/asr.rs:113,
decoder.rs:413, greedy.rs:32): encode once per utterance, then step the decoder
one token per stream, teacher-forced or greedy.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import check
from .ops import Context

_L = _lib.load()


class WhisperModel:
    def __init__(self, ctx: Context, gguf_path: str):
        h = C.c_void_p()
        check(_L.vkb_whisper_load(ctx.h, gguf_path.encode(), C.byref(h)))
        self.h, self.ctx = h, ctx
        d = _lib.WhisperDims()
        check(_L.vkb_whisper_get_dims(self.h, C.byref(d)))
        self.dims = d
        self.start_ids = [d.start_ids[i] for i in range(d.n_start_ids)]

    def close(self):
        if self.h:
            check(_L.vkb_whisper_destroy(self.h))
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    """A batched decoding session (paged self-attention KV + cross-attention store)."""

    def __init__(self, model: WhisperModel, max_streams: int, max_step_tokens: int | None = None,
                 max_clips: int = 0, cross_kv_q8: bool = True, kv_page_tokens: int = 16,
                 self_kv: int = _lib.SELF_KV_Q8_0):
        """self_kv: SELF_KV_Q8_0 (int8 pages, default), SELF_KV_F32 (the reference
        decoder's dense f32 cache numerics), SELF_KV_Q4_0 or SELF_KV_Q5_0."""
        o = _lib.SessionOptions(max_streams, max_step_tokens or 4 * max_streams, max_clips, int(cross_kv_q8),
                                kv_page_tokens, self_kv)
        h = C.c_void_p()
        check(_L.vkb_session_create(model.h, C.byref(o), C.byref(h)))
        self.h, self.model, self.ctx = h, model, model.ctx

    def encode(self, logmel_dev, streams):
        """logmel_dev: torch f32 [n_clips, n_mels, 2*n_audio_ctx] on the device."""
        s = np.ascontiguousarray(streams, dtype=np.int32)
        check(_L.vkb_session_encode(self.h, s.size, C.c_void_p(logmel_dev.data_ptr()), s.ctypes.data_as(C.c_void_p)))

    def encoder_output(self, n_clips: int) -> np.ndarray:
        """The last encoder output [n_clips, n_audio_ctx, d_model] (after ln_post), on the host."""
        d = self.model.dims
        host = np.empty((n_clips, d.n_audio_ctx, d.d_model), np.float32)
        check(_L.vkb_session_read_encoder_output(self.h, host.ctypes.data_as(C.c_void_p), host.size))
        return host

    def step(self, streams, positions, tokens, logits_dev=None, ids_dev=None):
        s = np.ascontiguousarray(streams, dtype=np.int32)
        p = np.ascontiguousarray(positions, dtype=np.int32)
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        check(_L.vkb_session_step(self.h, s.size, s.ctypes.data_as(C.c_void_p), p.ctypes.data_as(C.c_void_p),
                                  t.ctypes.data_as(C.c_void_p),
                                  C.c_void_p(logits_dev.data_ptr() if logits_dev is not None else None),
                                  C.c_void_p(ids_dev.data_ptr() if ids_dev is not None else None)))

    def step_feed(self, streams, positions, tokens, feed_rows, feed_ids_dev, logits_dev=None, ids_dev=None):
        """step() where token i is feed_ids_dev[feed_rows[i]] wherever feed_rows[i] >= 0 (read on the device)."""
        s = np.ascontiguousarray(streams, dtype=np.int32)
        p = np.ascontiguousarray(positions, dtype=np.int32)
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        f = np.ascontiguousarray(feed_rows, dtype=np.int32)
        check(_L.vkb_session_step_feed(self.h, s.size, s.ctypes.data_as(C.c_void_p), p.ctypes.data_as(C.c_void_p),
                                       t.ctypes.data_as(C.c_void_p), f.ctypes.data_as(C.c_void_p),
                                       C.c_void_p(feed_ids_dev.data_ptr()),
                                       C.c_void_p(logits_dev.data_ptr() if logits_dev is not None else None),
                                       C.c_void_p(ids_dev.data_ptr() if ids_dev is not None else None)))

    def release(self, stream: int):
        check(_L.vkb_session_release(self.h, stream))

    def close(self):
        if self.h:
            check(_L.vkb_session_destroy(self.h))
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
