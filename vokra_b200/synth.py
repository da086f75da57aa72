"""Synthetic GGUF models and quantizers (load-time tooling, not the hot path).

* numpy block quantizers for Q8_0 (the arithmetic of BlockQ8_0::pack,
  crates/vokra-core/src/kv_quant/q8_0.rs:40), Q4_0 (the public ggml reference
  quantizer; ggml is an external dependency not vendored in the reference) and
  Q4_K (vokra-convert's uniform-sub-scale quantizer,
  crates/vokra-convert/src/quantize.rs:96-143);
* a GGUF v3 writer following ``GgufBuilder::to_bytes``
  (crates/vokra-core/src/gguf/writer.rs:176-225): little-endian header, metadata,
  tensor infos with dims in PyTorch order, 32-byte-aligned payloads;
* seeded synthetic Whisper checkpoints (random N(0, 0.02) weights, layer norms
  1/0) with the tensor names of crates/vokra-models/src/whisper/weights.rs:302-360.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

GGUF_MAGIC = b"GGUF"
GGUF_VERSION = 3
DEFAULT_ALIGNMENT = 32

F32, F16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 2, 8, 12, 13, 14, 30

# GGUF metadata value type tags (crates/vokra-core/src/gguf/value.rs:33-57)
VT_U32, VT_I32, VT_F32, VT_BOOL, VT_STRING, VT_ARRAY = 4, 5, 6, 7, 8, 9


def payload_size(tag: int, n: int) -> int:
    if tag == F32:
        return 4 * n
    if tag in (F16, BF16):
        return 2 * n
    if tag == Q4_0:
        assert n % 32 == 0
        return n // 32 * 18
    if tag == Q8_0:
        assert n % 32 == 0
        return n // 32 * 34
    if tag == Q4_K:
        assert n % 256 == 0
        return n // 256 * 144
    if tag == Q5_K:
        assert n % 256 == 0
        return n // 256 * 176
    if tag == Q6_K:
        assert n % 256 == 0
        return n // 256 * 210
    raise ValueError(f"unsupported tag {tag}")


# ---------------------------------------------------------------------------
# Rounding helpers with Rust / C semantics (exact in float32)
# ---------------------------------------------------------------------------
def round_half_away(x: np.ndarray) -> np.ndarray:
    """f32::round: half away from zero, computed exactly."""
    x = np.asarray(x, dtype=np.float32)
    t = np.trunc(x)
    frac = np.abs(x - t)
    return (t + np.where(frac >= np.float32(0.5), np.sign(x), np.float32(0))).astype(np.float32)


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    """IEEE round-to-nearest-even (numpy's cast), as half.rs:80 for finite inputs."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


# ---------------------------------------------------------------------------
# Quantizers
# ---------------------------------------------------------------------------
def quantize_q8_0(x: np.ndarray) -> bytes:
    x = np.asarray(x, dtype=np.float32).reshape(-1, 32)
    amax = np.max(np.abs(x), axis=1)
    d = np.where(amax == 0, np.float32(0), amax / np.float32(127)).astype(np.float32)
    inv = np.zeros_like(d)
    nz = d != 0
    inv[nz] = np.float32(1) / d[nz]
    s = (x * inv[:, None]).astype(np.float32)
    c = np.clip(s, -127, 127)
    q = round_half_away(c).astype(np.int8)
    out = np.empty((x.shape[0], 34), dtype=np.uint8)
    out[:, 0:2] = f32_to_f16_bits(d).reshape(-1, 1).view(np.uint8)
    out[:, 2:] = q.view(np.uint8)
    return out.tobytes()


def quantize_q4_0(x: np.ndarray) -> bytes:
    x = np.asarray(x, dtype=np.float32).reshape(-1, 32)
    idx = np.argmax(np.abs(x), axis=1)
    mx = x[np.arange(x.shape[0]), idx]
    d = (mx / np.float32(-8)).astype(np.float32)
    inv = np.zeros_like(d)
    nz = d != 0
    inv[nz] = np.float32(1) / d[nz]
    xs = (x * inv[:, None]).astype(np.float32)
    q = np.trunc((xs + np.float32(8.5)).astype(np.float32)).astype(np.int32)
    q = np.minimum(q, 15).astype(np.uint8)
    out = np.empty((x.shape[0], 18), dtype=np.uint8)
    out[:, 0:2] = f32_to_f16_bits(d).reshape(-1, 1).view(np.uint8)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out.tobytes()


def quantize_q4_k(x: np.ndarray) -> bytes:
    x = np.asarray(x, dtype=np.float32).reshape(-1, 256)
    lo = x.min(axis=1)
    hi = x.max(axis=1)
    base = np.minimum(lo, np.float32(0))
    rng = (hi - base).astype(np.float32)
    step = (rng / np.float32(15)).astype(np.float32)
    d = np.where(step > 0, step / np.float32(63), np.float32(0)).astype(np.float32)
    dmin = np.where(base < 0, -base / np.float32(63), np.float32(0)).astype(np.float32)
    safe = np.where(step > 0, step, np.float32(1)).astype(np.float32)
    qf = round_half_away(((x - base[:, None]).astype(np.float32) / safe[:, None]).astype(np.float32))
    q = np.where(step[:, None] > 0, np.clip(qf, 0, 15), 0).astype(np.uint8)
    out = np.empty((x.shape[0], 144), dtype=np.uint8)
    out[:, 0:2] = f32_to_f16_bits(d).reshape(-1, 1).view(np.uint8)
    out[:, 2:4] = f32_to_f16_bits(dmin).reshape(-1, 1).view(np.uint8)
    out[:, 4:16] = 0xFF
    qq = q.reshape(-1, 4, 64)
    out[:, 16:] = (qq[:, :, :32] | (qq[:, :, 32:] << 4)).reshape(-1, 128)
    return out.tobytes()


def _affine_quants(x: np.ndarray, max_q: int):
    """Per 256-block affine map y = step*q + base with uniform sub-scales
    (affine_quants, crates/vokra-convert/src/quantize.rs:99-121)."""
    lo = x.min(axis=1)
    hi = x.max(axis=1)
    base = np.minimum(lo, np.float32(0))
    step = ((hi - base).astype(np.float32) / np.float32(max_q)).astype(np.float32)
    d = np.where(step > 0, step / np.float32(63), np.float32(0)).astype(np.float32)
    dmin = np.where(base < 0, -base / np.float32(63), np.float32(0)).astype(np.float32)
    safe = np.where(step > 0, step, np.float32(1)).astype(np.float32)
    qf = round_half_away(((x - base[:, None]).astype(np.float32) / safe[:, None]).astype(np.float32))
    q = np.where(step[:, None] > 0, np.clip(qf, 0, max_q), 0).astype(np.uint8)
    return q, d, dmin


def quantize_q5_k(x: np.ndarray) -> bytes:
    """vokra-convert's Q5_K encoder (crates/vokra-convert/src/quantize.rs:144-170)."""
    x = np.asarray(x, dtype=np.float32).reshape(-1, 256)
    q, d, dmin = _affine_quants(x, 31)
    out = np.empty((x.shape[0], 176), dtype=np.uint8)
    out[:, 0:2] = f32_to_f16_bits(d).reshape(-1, 1).view(np.uint8)
    out[:, 2:4] = f32_to_f16_bits(dmin).reshape(-1, 1).view(np.uint8)
    out[:, 4:16] = 0xFF
    qq = q.reshape(-1, 4, 64)
    lo, hi = qq[:, :, :32], qq[:, :, 32:]
    qh = np.zeros((x.shape[0], 32), np.uint8)
    for k in range(4):
        qh |= ((lo[:, k] >> 4) & 1) << (2 * k)
        qh |= ((hi[:, k] >> 4) & 1) << (2 * k + 1)
    out[:, 16:48] = qh
    out[:, 48:] = ((lo & 0xF) | ((hi & 0xF) << 4)).reshape(-1, 128)
    return out.tobytes()


def quantize_q6_k(x: np.ndarray) -> bytes:
    """vokra-convert's Q6_K encoder (crates/vokra-convert/src/quantize.rs:176-230):
    one symmetric scale per block, uniform int8 sub-scales 31."""
    x = np.asarray(x, dtype=np.float32).reshape(-1, 256)
    amax = np.abs(x).max(axis=1)
    step = (amax / np.float32(31)).astype(np.float32)
    d = np.where(step > 0, step / np.float32(31), np.float32(0)).astype(np.float32)
    safe = np.where(step > 0, step, np.float32(1)).astype(np.float32)
    q = np.where(step[:, None] > 0, np.clip(round_half_away((x / safe[:, None]).astype(np.float32)), -32, 31), 0)
    st = (q.astype(np.int32) + 32).astype(np.uint8).reshape(-1, 2, 4, 32)  # [block][half][quarter][l]
    low4, hi2 = st & 0xF, (st >> 4) & 3
    ql = np.concatenate([low4[:, :, 0] | (low4[:, :, 2] << 4), low4[:, :, 1] | (low4[:, :, 3] << 4)], axis=2)
    qh = hi2[:, :, 0] | (hi2[:, :, 1] << 2) | (hi2[:, :, 2] << 4) | (hi2[:, :, 3] << 6)
    out = np.empty((x.shape[0], 210), dtype=np.uint8)
    out[:, 0:128] = ql.reshape(-1, 128)
    out[:, 128:192] = qh.reshape(-1, 64)
    out[:, 192:208] = 31
    out[:, 208:210] = f32_to_f16_bits(d).reshape(-1, 1).view(np.uint8)
    return out.tobytes()


def random_kquant_blocks(tag: int, n: int, rng, scale: float = 0.02) -> bytes:
    """Valid Q5_K / Q6_K blocks with every field random (sub-scales, mins, high
    bits), the f16 super-scales sized so values come out around `scale`: covers
    the decode paths the uniform-scale encoders above never reach."""
    nb = n // 256
    if tag == Q5_K:
        out = rng.integers(0, 256, (nb, 176), dtype=np.uint8)
        out[:, 0:2] = f32_to_f16_bits(rng.uniform(0.2, 1.0, nb).astype(np.float32) * np.float32(scale / 500)
                                      ).reshape(-1, 1).view(np.uint8)
        out[:, 2:4] = f32_to_f16_bits(rng.uniform(0.2, 1.0, nb).astype(np.float32) * np.float32(scale / 30)
                                      ).reshape(-1, 1).view(np.uint8)
        return out.tobytes()
    if tag == Q6_K:
        out = rng.integers(0, 256, (nb, 210), dtype=np.uint8)
        out[:, 208:210] = f32_to_f16_bits(rng.uniform(0.2, 1.0, nb).astype(np.float32) * np.float32(scale / 1000)
                                          ).reshape(-1, 1).view(np.uint8)
        return out.tobytes()
    raise ValueError(f"no random blocks for tag {tag}")


def quantize(tag: int, x: np.ndarray) -> bytes:
    if tag == Q8_0:
        return quantize_q8_0(x)
    if tag == Q4_0:
        return quantize_q4_0(x)
    if tag == Q4_K:
        return quantize_q4_k(x)
    if tag == Q5_K:
        return quantize_q5_k(x)
    if tag == Q6_K:
        return quantize_q6_k(x)
    if tag == BF16:
        b = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
        rne = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)  # round to nearest even
        return rne.tobytes()
    if tag == F32:
        return np.asarray(x, dtype=np.float32).tobytes()
    if tag == F16:
        return np.asarray(x, dtype=np.float32).astype(np.float16).tobytes()
    raise ValueError(f"no quantizer for tag {tag}")


def dequantize(tag: int, data: bytes, n: int) -> np.ndarray:
    """numpy dequantizers (same values as crates/vokra-core/src/gguf/quant)."""
    b = np.frombuffer(data, dtype=np.uint8)
    if tag == F32:
        return b.view(np.float32).copy()
    if tag == F16:
        return b.view(np.float16).astype(np.float32)
    if tag == Q8_0:
        blk = b.reshape(-1, 34)
        d = blk[:, :2].copy().view(np.float16).astype(np.float32)
        return (blk[:, 2:].view(np.int8).astype(np.float32) * d).reshape(-1)
    if tag == Q4_0:
        blk = b.reshape(-1, 18)
        d = blk[:, :2].copy().view(np.float16).astype(np.float32)
        qs = blk[:, 2:]
        q = np.concatenate([(qs & 0xF).astype(np.int32) - 8, (qs >> 4).astype(np.int32) - 8], axis=1)
        return (q.astype(np.float32) * d).reshape(-1)
    if tag == Q4_K:
        blk = b.reshape(-1, 144)
        d = blk[:, 0:2].copy().view(np.float16).astype(np.float32)[:, 0]
        dmin = blk[:, 2:4].copy().view(np.float16).astype(np.float32)[:, 0]
        s = blk[:, 4:16].astype(np.int32)
        sc = np.zeros((blk.shape[0], 8), np.int32)
        mn = np.zeros((blk.shape[0], 8), np.int32)
        for j in range(8):
            if j < 4:
                sc[:, j] = s[:, j] & 63
                mn[:, j] = s[:, j + 4] & 63
            else:
                sc[:, j] = (s[:, j + 4] & 0xF) | ((s[:, j - 4] >> 6) << 4)
                mn[:, j] = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
        qs = blk[:, 16:].reshape(-1, 4, 32)
        y = np.empty((blk.shape[0], 256), np.float32)
        for c in range(4):
            d1 = (d * sc[:, 2 * c].astype(np.float32)).astype(np.float32)
            m1 = (dmin * mn[:, 2 * c].astype(np.float32)).astype(np.float32)
            d2 = (d * sc[:, 2 * c + 1].astype(np.float32)).astype(np.float32)
            m2 = (dmin * mn[:, 2 * c + 1].astype(np.float32)).astype(np.float32)
            y[:, 64 * c:64 * c + 32] = d1[:, None] * (qs[:, c] & 0xF).astype(np.float32) - m1[:, None]
            y[:, 64 * c + 32:64 * c + 64] = d2[:, None] * (qs[:, c] >> 4).astype(np.float32) - m2[:, None]
        return y.reshape(-1)
    raise ValueError(f"no dequantizer for tag {tag}")


# ---------------------------------------------------------------------------
# GGUF writer
# ---------------------------------------------------------------------------
def _s(x: str) -> bytes:
    b = x.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _value(v) -> bytes:
    if isinstance(v, bool):
        return struct.pack("<I", VT_BOOL) + struct.pack("<B", int(v))
    if isinstance(v, int):
        return struct.pack("<I", VT_U32) + struct.pack("<I", v)
    if isinstance(v, float):
        return struct.pack("<I", VT_F32) + struct.pack("<f", v)
    if isinstance(v, str):
        return struct.pack("<I", VT_STRING) + _s(v)
    if isinstance(v, (list, tuple)):
        return struct.pack("<I", VT_ARRAY) + struct.pack("<I", VT_U32) + struct.pack("<Q", len(v)) + b"".join(
            struct.pack("<I", int(e)) for e in v)
    raise TypeError(type(v))


@dataclass
class TensorDecl:
    name: str
    tag: int
    dims: list
    nbytes: int = 0


@dataclass
class GgufStreamWriter:
    """Header first, then each tensor payload in declaration order (GgufStreamWriter, writer.rs:295)."""
    path: str
    metadata: dict
    tensors: list = field(default_factory=list)
    alignment: int = DEFAULT_ALIGNMENT

    def begin(self):
        head = bytearray()
        head += GGUF_MAGIC + struct.pack("<I", GGUF_VERSION)
        head += struct.pack("<QQ", len(self.tensors), len(self.metadata))
        for k, v in self.metadata.items():
            head += _s(k) + _value(v)
        off = 0
        self._offsets = []
        for t in self.tensors:
            n = int(np.prod(t.dims)) if t.dims else 1
            t.nbytes = payload_size(t.tag, n)
            self._offsets.append(off)
            off = (off + t.nbytes + self.alignment - 1) // self.alignment * self.alignment
        for t, o in zip(self.tensors, self._offsets):
            head += _s(t.name) + struct.pack("<I", len(t.dims)) + b"".join(struct.pack("<Q", d) for d in t.dims)
            head += struct.pack("<IQ", t.tag, o)
        pad = (-len(head)) % self.alignment
        head += b"\0" * pad
        self._f = open(self.path, "wb")
        self._f.write(head)
        self._i = 0

    def write(self, data: bytes):
        t = self.tensors[self._i]
        assert len(data) == t.nbytes, (t.name, len(data), t.nbytes)
        self._f.write(data)
        pad = (-t.nbytes) % self.alignment
        if pad:
            self._f.write(b"\0" * pad)
        self._i += 1

    def finish(self):
        assert self._i == len(self.tensors)
        self._f.close()


# ---------------------------------------------------------------------------
# Synthetic Whisper checkpoints
# ---------------------------------------------------------------------------
@dataclass
class WhisperArch:
    n_mels: int
    n_audio_ctx: int
    d_model: int
    n_audio_head: int
    n_audio_layer: int
    n_text_ctx: int
    n_text_head: int
    n_text_layer: int
    n_vocab: int
    ffn_dim: int
    eot: int
    start_ids: tuple


WHISPER_BASE = WhisperArch(80, 1500, 512, 8, 6, 448, 8, 6, 51865, 2048, 50257, (50258, 50259, 50359, 50363))
WHISPER_LARGE_V3 = WhisperArch(128, 1500, 1280, 20, 32, 448, 20, 32, 51866, 5120, 50257,
                               (50258, 50259, 50360, 50364))
# A small architecture for fast tests (same structure, tiny sizes).
WHISPER_TINY_TEST = WhisperArch(16, 64, 256, 4, 2, 32, 4, 2, 500, 512, 499, (1, 2, 3, 4))


def whisper_tensor_decls(a: WhisperArch, qtag: int):
    d, f = a.d_model, a.ffn_dim
    out = [("model.encoder.conv1.weight", F32, [d, a.n_mels, 3]), ("model.encoder.conv1.bias", F32, [d]),
           ("model.encoder.conv2.weight", F32, [d, d, 3]), ("model.encoder.conv2.bias", F32, [d]),
           ("model.encoder.embed_positions.weight", F32, [a.n_audio_ctx, d])]

    def attn(p):
        return [(f"{p}.q_proj.weight", qtag, [d, d]), (f"{p}.q_proj.bias", F32, [d]),
                (f"{p}.k_proj.weight", qtag, [d, d]),
                (f"{p}.v_proj.weight", qtag, [d, d]), (f"{p}.v_proj.bias", F32, [d]),
                (f"{p}.out_proj.weight", qtag, [d, d]), (f"{p}.out_proj.bias", F32, [d])]

    def ln(p):
        return [(f"{p}.weight", F32, [d]), (f"{p}.bias", F32, [d])]

    def mlp(p):
        return [(f"{p}.fc1.weight", qtag, [f, d]), (f"{p}.fc1.bias", F32, [f]),
                (f"{p}.fc2.weight", qtag, [d, f]), (f"{p}.fc2.bias", F32, [d])]

    for i in range(a.n_audio_layer):
        p = f"model.encoder.layers.{i}"
        out += ln(f"{p}.self_attn_layer_norm") + attn(f"{p}.self_attn") + ln(f"{p}.final_layer_norm") + mlp(p)
    out += ln("model.encoder.layer_norm")
    out += [("model.decoder.embed_tokens.weight", qtag, [a.n_vocab, d]),
            ("model.decoder.embed_positions.weight", F32, [a.n_text_ctx, d])]
    for i in range(a.n_text_layer):
        p = f"model.decoder.layers.{i}"
        out += (ln(f"{p}.self_attn_layer_norm") + attn(f"{p}.self_attn") + ln(f"{p}.encoder_attn_layer_norm") +
                attn(f"{p}.encoder_attn") + ln(f"{p}.final_layer_norm") + mlp(p))
    out += ln("model.decoder.layer_norm")
    return out


def whisper_metadata(a: WhisperArch) -> dict:
    return {
        "general.architecture": "whisper",
        "vokra.whisper.n_mels": a.n_mels,
        "vokra.whisper.n_audio_ctx": a.n_audio_ctx,
        "vokra.whisper.n_audio_state": a.d_model,
        "vokra.whisper.n_audio_head": a.n_audio_head,
        "vokra.whisper.n_audio_layer": a.n_audio_layer,
        "vokra.whisper.n_text_ctx": a.n_text_ctx,
        "vokra.whisper.n_text_state": a.d_model,
        "vokra.whisper.n_text_head": a.n_text_head,
        "vokra.whisper.n_text_layer": a.n_text_layer,
        "vokra.whisper.n_vocab": a.n_vocab,
        "vokra.whisper.ffn_dim": a.ffn_dim,
        "vokra.whisper.eot": a.eot,
        "vokra.whisper.decoder_start_ids": list(a.start_ids),
    }


def _synthetic_tensor(args):
    seed, i, name, tag, dims = args
    n = int(np.prod(dims))
    if "layer_norm" in name:
        v = np.ones(n, np.float32) if name.endswith(".weight") else np.zeros(n, np.float32)
    else:
        v = np.random.default_rng([seed, i]).standard_normal(n, dtype=np.float32) * np.float32(0.02)
    return quantize(tag, v)


def write_synthetic_whisper(path: str, a: WhisperArch, qtag: int, seed: int = 0, workers: int | None = None) -> None:
    """Seeded N(0, 0.02) weights (layer norms 1/0), Linear + embed_tokens in `qtag`.
    Tensor i draws from rng([seed, i]), so the file does not depend on how many
    worker processes quantize the tensors."""
    import os
    decls = whisper_tensor_decls(a, qtag)
    w = GgufStreamWriter(path, whisper_metadata(a), [TensorDecl(n, t, dims) for n, t, dims in decls])
    w.begin()
    jobs = [(seed, i, name, tag, dims) for i, (name, tag, dims) in enumerate(decls)]
    n_workers = workers if workers is not None else min(16, os.cpu_count() or 1)
    big = sum(int(np.prod(d)) for _, _, _, _, d in jobs) > (64 << 20)
    if n_workers > 1 and big:
        import multiprocessing as mp
        with mp.get_context("fork").Pool(n_workers) as pool:
            for data in pool.imap(_synthetic_tensor, jobs, chunksize=1):
                w.write(data)
    else:
        for j in jobs:
            w.write(_synthetic_tensor(j))
    w.finish()


def synthetic_audio(seed: int, seconds: float = 30.0, sr: int = 16000) -> np.ndarray:
    """White noise at -20 dBFS RMS plus three sinusoids (100-4000 Hz, amplitude 0.05), clipped to +-1."""
    rng = np.random.default_rng(seed)
    n = int(seconds * sr)
    x = rng.standard_normal(n).astype(np.float32) * np.float32(0.1)
    t = np.arange(n, dtype=np.float64) / sr
    for _ in range(3):
        f = rng.uniform(100, 4000)
        ph = rng.uniform(0, 2 * np.pi)
        x += (0.05 * np.sin(2 * np.pi * f * t + ph)).astype(np.float32)
    return np.clip(x, -1, 1).astype(np.float32)
