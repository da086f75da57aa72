"""Oracle Whisper forward — TEST INFRASTRUCTURE ONLY.

Restates the reference CPU forward (route R1: every Linear dequantized to f32
at load and run through gemm_f32) with the C++ primitives of vkb_oracle.cpp:
  encoder  crates/vokra-models/src/whisper/encoder.rs:41-110, :180-236
  decoder  crates/vokra-models/src/whisper/decoder.rs:183-216 (cross K/V once),
           :413-566 (step_into), :754-773 (tied logits)
  nn       whisper/nn.rs:62-300
The self-attention cache can be the reference's dense f32 KvCache
(kv_mode="f32") or its QuantizedPagedKvCache in Q8_0, Q4_0 or Q5_0
(kv_mode="q8" / "q4" / "q5": every appended K/V row goes through the block's
pack / unpack); the cross K/V can be
kept f32, rounded to f16, or stored as Q8_0 (cross_mode="f32"|"f16"|"q8").
"""
from __future__ import annotations

import struct

import numpy as np

from . import py as o


def read_gguf(path: str):
    """Minimal GGUF v3 reader (crates/vokra-core/src/gguf/reader.rs): returns (meta, tensors)."""
    data = open(path, "rb").read()
    pos = 0

    def get(fmt):
        nonlocal pos
        v = struct.unpack_from(fmt, data, pos)
        pos += struct.calcsize(fmt)
        return v[0]

    def gstr():
        n = get("<Q")
        nonlocal pos
        s = data[pos:pos + n].decode()
        pos += n
        return s

    def value(t):
        if t == 4:
            return get("<I")
        if t == 5:
            return get("<i")
        if t == 6:
            return get("<f")
        if t == 7:
            return get("<B")
        if t == 8:
            return gstr()
        if t == 9:
            et = get("<I")
            n = get("<Q")
            return [value(et) for _ in range(n)]
        if t == 10:
            return get("<Q")
        raise ValueError(t)

    assert data[:4] == b"GGUF"
    pos = 4
    assert get("<I") == 3
    nt, nkv = get("<Q"), get("<Q")
    meta = {}
    for _ in range(nkv):
        k = gstr()
        meta[k] = value(get("<I"))
    infos = []
    for _ in range(nt):
        name = gstr()
        nd = get("<I")
        dims = [get("<Q") for _ in range(nd)]
        tag = get("<I")
        off = get("<Q")
        infos.append((name, dims, tag, off))
    align = meta.get("general.alignment", 32)
    base = (pos + align - 1) // align * align
    tensors = {}
    for name, dims, tag, off in infos:
        n = int(np.prod(dims))
        nbytes = int(o.lib().orc_payload_size(tag, n))
        tensors[name] = (dims, tag, data[base + off: base + off + nbytes])
    return meta, tensors


class RefWhisper:
    def __init__(self, path: str):
        self.meta, raw = read_gguf(path)
        m = self.meta
        self.n_mels = m["vokra.whisper.n_mels"]
        self.d = m["vokra.whisper.n_audio_state"]
        self.n_audio_head = m["vokra.whisper.n_audio_head"]
        self.n_audio_layer = m["vokra.whisper.n_audio_layer"]
        self.n_text_head = m["vokra.whisper.n_text_head"]
        self.n_text_layer = m["vokra.whisper.n_text_layer"]
        self.n_vocab = m["vokra.whisper.n_vocab"]
        self.n_text_ctx = m["vokra.whisper.n_text_ctx"]
        self.t = {}
        for name, (dims, tag, b) in raw.items():
            arr = o.dequantize(tag, np.frombuffer(b, np.uint8), int(np.prod(dims))).reshape(dims)
            self.t[name] = arr
        # dense_w_t: every 2-D Linear weight bound transposed [in, out] (weights.rs:506-518)
        self.wt = {n: np.ascontiguousarray(v.T) for n, v in self.t.items()
                   if v.ndim == 2 and (n.endswith("proj.weight") or ".fc" in n)}
        self.emb_t = np.ascontiguousarray(self.t["model.decoder.embed_tokens.weight"].T)

    def lin(self, x, name, bias=True):
        b = self.t.get(name + ".bias") if bias else None
        return o.gemm_kn(x, self.wt[name + ".weight"], b)

    def ln(self, x, name):
        return o.layer_norm(x, self.t[name + ".weight"], self.t[name + ".bias"])

    def attn_block(self, x_q, k, v, p, n_head, causal=False, q_off=0):
        hd = self.d // n_head
        q = self.lin(x_q, p + ".q_proj") * np.float32(hd ** -0.5)
        ctx = o.attention(q, k, v, n_head, causal=causal, q_off=q_off)
        return self.lin(ctx, p + ".out_proj")

    def encode(self, logmel: np.ndarray) -> np.ndarray:
        t = self.t
        c1 = o.gelu(o.conv1d(logmel, t["model.encoder.conv1.weight"], t["model.encoder.conv1.bias"], 1, 1))
        c2 = o.gelu(o.conv1d(c1, t["model.encoder.conv2.weight"], t["model.encoder.conv2.bias"], 2, 1))
        h = (c2.T + t["model.encoder.embed_positions.weight"]).astype(np.float32)
        for i in range(self.n_audio_layer):
            p = f"model.encoder.layers.{i}"
            x = self.ln(h, p + ".self_attn_layer_norm")
            k = self.lin(x, p + ".self_attn.k_proj", bias=False)
            v = self.lin(x, p + ".self_attn.v_proj")
            h = h + self.attn_block(x, k, v, p + ".self_attn", self.n_audio_head)
            x = self.ln(h, p + ".final_layer_norm")
            h = h + self.lin(o.gelu(self.lin(x, p + ".fc1")), p + ".fc2")
        return self.ln(h, "model.encoder.layer_norm")

    def decoder(self, enc_out: np.ndarray, kv_mode: str = "q8", cross_mode: str = "q8"):
        return RefDecoder(self, enc_out, kv_mode, cross_mode)


def _store(x: np.ndarray, mode: str) -> np.ndarray:
    """K/V rows as a cache of `mode` returns them: "q8" / "q4" / "q5" through
    BlockQ8_0 / BlockQ4_0 / BlockQ5_0 pack + unpack, "f16" rounded, "f32" as is."""
    kv = {"q4": 1, "q5": 2, "q8": 3}
    if mode in kv:
        return o.kv_unpack(kv[mode], o.kv_pack(kv[mode], x)).reshape(x.shape)
    if mode == "f16":
        return x.astype(np.float16).astype(np.float32)
    return x


class RefDecoder:
    def __init__(self, m: RefWhisper, enc_out, kv_mode, cross_mode):
        self.m = m
        self.kv_mode = kv_mode
        self.cross = []
        for i in range(m.n_text_layer):
            p = f"model.decoder.layers.{i}.encoder_attn"
            k = m.lin(enc_out, p + ".k_proj", bias=False)
            v = m.lin(enc_out, p + ".v_proj")
            self.cross.append((_store(k, cross_mode), _store(v, cross_mode)))
        self.k = [np.zeros((0, m.d), np.float32) for _ in range(m.n_text_layer)]
        self.v = [np.zeros((0, m.d), np.float32) for _ in range(m.n_text_layer)]
        self.pos = 0

    def step(self, tokens) -> np.ndarray:
        m, t = self.m, self.m.t
        n = len(tokens)
        start = self.pos
        h = np.stack([t["model.decoder.embed_tokens.weight"][tok] + t["model.decoder.embed_positions.weight"][start + i]
                      for i, tok in enumerate(tokens)]).astype(np.float32)
        for i in range(m.n_text_layer):
            p = f"model.decoder.layers.{i}"
            x = m.ln(h, p + ".self_attn_layer_norm")
            k = m.lin(x, p + ".self_attn.k_proj", bias=False)
            v = m.lin(x, p + ".self_attn.v_proj")
            qk = self.kv_mode if self.kv_mode in ("q4", "q5", "q8") else "f32"
            self.k[i] = np.concatenate([self.k[i], _store(k, qk)])
            self.v[i] = np.concatenate([self.v[i], _store(v, qk)])
            h = h + m.attn_block(x, self.k[i], self.v[i], p + ".self_attn", m.n_text_head, causal=True, q_off=start)
            x = m.ln(h, p + ".encoder_attn_layer_norm")
            ck, cv = self.cross[i]
            h = h + m.attn_block(x, ck, cv, p + ".encoder_attn", m.n_text_head)
            x = m.ln(h, p + ".final_layer_norm")
            h = h + m.lin(o.gelu(m.lin(x, p + ".fc1")), p + ".fc2")
        x = m.ln(h, "model.decoder.layer_norm")
        self.pos += n
        return o.gemm_kn(x, m.emb_t)
