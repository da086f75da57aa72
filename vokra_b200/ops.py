"""Host-side mirror of the reference seams over the C ABI.

Names and argument meanings follow the reference so that tests read like the
reference's own:

* :func:`gemm_q_f32` — ``Compute::gemm_q_f32`` (crates/vokra-models/src/compute.rs:943)
* :class:`KvQuantDequantGemvOps` — ``KvQuantDequantGemvOps::fused_dequant_gemv``
  (crates/vokra-core/src/kv_quant/gpu_ops.rs:70)
* :class:`QuantizedPagedKvCache` — ``QuantizedPagedKvCache`` (cache/paged_quant.rs:240)
  on the device, plus the step-batched append / attention of the decode path.

Device tensors are torch tensors (plumbing only); every computation runs in
libvkb200.so. There is no CPU fallback: a missing library raises at import.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import check, VkbError  # noqa: F401

_L = _lib.load()


def _ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


class Context:
    """One vkb_context per GPU. ``use_torch_stream`` launches on torch's current stream."""

    def __init__(self, device: int = 0, use_torch_stream: bool = True):
        h = C.c_void_p()
        check(_L.vkb_context_create(device, C.byref(h)))
        self.h = h
        self.device = device
        if use_torch_stream:
            import torch
            s = torch.cuda.current_stream(device)
            # torch's default stream has handle 0, the legacy default stream; pass it
            # as cudaStreamLegacy (0x1) because NULL selects the context's own stream.
            check(_L.vkb_context_set_stream(self.h, C.c_void_p(s.cuda_stream or 1)))

    def set_stream(self, stream_handle: int | None):
        check(_L.vkb_context_set_stream(self.h, C.c_void_p(stream_handle) if stream_handle else None))

    def synchronize(self):
        check(_L.vkb_context_synchronize(self.h))

    @property
    def launch_count(self) -> int:
        return int(_L.vkb_context_launch_count(self.h))

    def close(self):
        if self.h:
            check(_L.vkb_context_destroy(self.h))
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Weight:
    """An uploaded [n][k] GGUF weight, repacked once into the device tile layout."""

    def __init__(self, ctx: Context, ggml_type: int, n: int, k: int, payload: bytes | np.ndarray):
        buf = np.ascontiguousarray(np.frombuffer(payload, dtype=np.uint8) if isinstance(payload, (bytes, bytearray))
                                   else payload.view(np.uint8).reshape(-1))
        h = C.c_void_p()
        check(_L.vkb_weight_upload(ctx.h, ggml_type, n, k, buf.ctypes.data_as(C.c_void_p), buf.nbytes, C.byref(h)))
        self.h = h
        self.ctx = ctx
        self.n, self.k, self.ggml_type = n, k, ggml_type

    @property
    def device_bytes(self) -> int:
        return int(_L.vkb_weight_device_bytes(self.h))

    def close(self):
        if self.h:
            check(_L.vkb_weight_destroy(self.h))
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def linear(ctx: Context, w: Weight, a, out, bias=None, epilogue: int = _lib.EPI_NONE, residual=None,
           scale: float = 1.0):
    """out = epilogue(a @ dequant(W)^T + bias) on the device (torch tensors)."""
    import torch
    m = a.shape[0]
    a_dt = _lib.DT_F16 if a.dtype == torch.float16 else _lib.DT_F32
    o_dt = _lib.DT_F16 if out.dtype == torch.float16 else _lib.DT_F32
    check(_L.vkb_linear(ctx.h, w.h, m, C.c_void_p(_ptr(a)), a_dt, C.c_void_p(_ptr(bias)), C.c_void_p(_ptr(out)), o_dt,
                        epilogue, C.c_void_p(_ptr(residual)), C.c_float(scale)))


def gemm_q_f32(ctx: Context, m: int, n: int, k: int, a: np.ndarray, wq: bytes | np.ndarray, dtype: int,
               bias: np.ndarray | None, out: np.ndarray) -> None:
    """``Compute::gemm_q_f32`` with host buffers: ``out[t, j] = bias[j] + sum_l a[t, l] * dequant(wq[j, l])``."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    wq = np.frombuffer(wq, dtype=np.uint8) if isinstance(wq, (bytes, bytearray)) else np.ascontiguousarray(wq).view(np.uint8)
    if out.dtype != np.float32 or not out.flags.c_contiguous:
        raise ValueError("out must be a contiguous float32 array")
    if a.size != m * k:
        raise VkbError(_lib.ERROR_INVALID_ARGUMENT, f"a.len()={a.size} != m*k={m * k}")
    if out.size != m * n:
        raise VkbError(_lib.ERROR_INVALID_ARGUMENT, f"out.len()={out.size} != m*n={m * n}")
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    if b is not None and b.size != n:
        raise VkbError(_lib.ERROR_INVALID_ARGUMENT, f"bias.len()={b.size} != n={n}")
    check(_L.vkb_gemm_q_f32(ctx.h, m, n, k, a.ctypes.data_as(C.c_void_p), wq.ctypes.data_as(C.c_void_p), wq.nbytes,
                            dtype, None if b is None else b.ctypes.data_as(C.c_void_p),
                            out.ctypes.data_as(C.c_void_p)))


class KvQuantDequantGemvOps:
    """The GPU arm of ``KvQuantDequantGemvOps`` (gpu_ops.rs:70)."""

    def __init__(self, ctx: Context):
        self.ctx = ctx

    def fused_dequant_gemv(self, mode: int, blocks_bytes: bytes | np.ndarray, n_rows: int, n_blocks_per_row: int,
                           x: np.ndarray) -> np.ndarray:
        blk = np.frombuffer(blocks_bytes, dtype=np.uint8) if isinstance(blocks_bytes, (bytes, bytearray)) \
            else np.ascontiguousarray(blocks_bytes).view(np.uint8)
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(n_rows, dtype=np.float32)
        check(_L.vkb_kv_dequant_gemv_host(self.ctx.h, mode, blk.ctypes.data_as(C.c_void_p), blk.nbytes, n_rows,
                                          n_blocks_per_row, x.ctypes.data_as(C.c_void_p), x.size,
                                          y.ctypes.data_as(C.c_void_p)))
        return y


@dataclass
class KvDims:
    """``KvDims`` (cache/paged.rs:155)."""
    n_layer: int
    n_head: int
    d_head: int
    n_stream: int = 1
    n_codebook: int = 1
    max_time: int = 448


class QuantizedPagedKvCache:
    """The device paged quantized KV cache (``QuantizedPagedKvCache``, paged_quant.rs:240).

    ``layout`` is ``KV_LAYOUT_REFERENCE`` (pages per (layer, time-block) with every
    stream inside, block size 2/4 or 16) or ``KV_LAYOUT_SEQUENCE`` (per-stream pages
    shared by all layers).
    """

    def __init__(self, ctx: Context, dims: KvDims, block_size: int, mode: int = _lib.KV_Q8_0,
                 layout: int = _lib.KV_LAYOUT_REFERENCE, n_pages: int = 0):
        d = _lib.KvPoolDesc(dims.n_layer, dims.n_head, dims.d_head, dims.n_stream, dims.n_codebook, dims.max_time,
                            block_size, mode, layout, n_pages)
        h = C.c_void_p()
        check(_L.vkb_kv_pool_create(ctx.h, C.byref(d), C.byref(h)))
        self.h, self.ctx, self.dims, self.block_size, self.mode, self.layout = h, ctx, dims, block_size, mode, layout
        self._pos = 0

    # ---- step-batched device path ------------------------------------------
    def begin_step(self, seq_ids, positions):
        s = np.ascontiguousarray(seq_ids, dtype=np.int32)
        p = np.ascontiguousarray(positions, dtype=np.int32)
        check(_L.vkb_kv_begin_step(self.h, s.size, s.ctypes.data_as(C.c_void_p), p.ctypes.data_as(C.c_void_p)))

    def append(self, layer: int, k, v):
        check(_L.vkb_kv_append(self.h, layer, C.c_void_p(_ptr(k)), C.c_void_p(_ptr(v))))

    def attention(self, layer: int, q, out):
        import torch
        dt = _lib.DT_F16 if out.dtype == torch.float16 else _lib.DT_F32
        check(_L.vkb_kv_attention(self.h, layer, C.c_void_p(_ptr(q)), C.c_void_p(_ptr(out)), dt))

    def append_attention(self, layer: int, qkv, out) -> None:
        """Append the step's K/V and attend, one call (``vkb_kv_append_attention``):
        qkv is f32 [n_tok][ld] holding scaled q | k | v."""
        import torch
        dt = _lib.DT_F16 if out.dtype == torch.float16 else _lib.DT_F32
        check(_L.vkb_kv_append_attention(self.h, layer, C.c_void_p(_ptr(qkv)), qkv.stride(0),
                                         C.c_void_p(_ptr(out)), dt))

    def decode_fused(self) -> bool:
        return bool(_L.vkb_kv_decode_fused(self.h))

    # ---- reference-shaped API ----------------------------------------------
    def append_step(self, layer: int, t: int, s: int, c: int, k_row: np.ndarray, v_row: np.ndarray):
        """``append_step`` (paged_quant.rs:396) for one (layer, t, stream) row, host arrays."""
        import torch
        if c != 0 or c >= self.dims.n_codebook:
            raise VkbError(_lib.ERROR_INVALID_ARGUMENT, f"codebook {c} >= n_codebook {self.dims.n_codebook}")
        w = self.dims.n_head * self.dims.d_head
        if len(k_row) != w or len(v_row) != w:
            raise VkbError(_lib.ERROR_INVALID_ARGUMENT,
                           f"append_step: expected k/v row len {w}, got k={len(k_row)} v={len(v_row)}")
        self.begin_step([s], [t])
        dev = f"cuda:{self.ctx.device}"
        kt = torch.as_tensor(np.ascontiguousarray(k_row, dtype=np.float32)).to(dev)
        vt = torch.as_tensor(np.ascontiguousarray(v_row, dtype=np.float32)).to(dev)
        self.append(layer, kt, vt)
        self.ctx.synchronize()

    def read_step(self, layer: int, t: int, s: int, c: int = 0):
        w = self.dims.n_head * self.dims.d_head
        k = np.zeros(w, np.float32)
        v = np.zeros(w, np.float32)
        if c != 0:
            return None
        st = _L.vkb_kv_read_step(self.h, layer, t, s, k.ctypes.data_as(C.c_void_p), v.ctypes.data_as(C.c_void_p))
        if st == _lib.ERROR_OTHER or st == _lib.ERROR_INVALID_ARGUMENT:
            return None
        check(st)
        return k, v

    def advance(self, n: int):
        self._pos += n

    def positions(self) -> int:
        return self._pos

    def reset(self):
        check(_L.vkb_kv_reset(self.h))
        self._pos = 0

    def release_layer(self, layer: int):
        check(_L.vkb_kv_release_layer(self.h, layer))

    def copy_stream(self, src: int, dst: int, n_pos: int):
        """dst := the first n_pos positions of src (filled pages shared, copy on write)."""
        check(_L.vkb_kv_copy_stream(self.h, src, dst, n_pos))

    def release_seq(self, seq: int):
        check(_L.vkb_kv_release_seq(self.h, seq))

    def set_page_table(self, table: np.ndarray):
        t = np.ascontiguousarray(table, dtype=np.int32)
        check(_L.vkb_kv_set_page_table(self.h, t.ctypes.data_as(C.c_void_p), t.size))

    def page_table(self) -> np.ndarray:
        n = int(_L.vkb_kv_table_len(self.h))
        out = np.zeros(n, np.int64)
        check(_L.vkb_kv_page_table(self.h, out.ctypes.data_as(C.c_void_p), n))
        return out

    def pages_in_use(self) -> int:
        return int(_L.vkb_kv_pages_in_use(self.h))

    def page_bytes(self) -> int:
        return int(_L.vkb_kv_page_bytes(self.h))

    def on_wire_storage_bytes(self) -> int:
        return int(_L.vkb_kv_on_wire_bytes(self.h))

    def read_page(self, page: int, layer: int = 0):
        nb = self.page_bytes()
        k = np.zeros(nb, np.uint8)
        v = np.zeros(nb, np.uint8)
        check(_L.vkb_kv_read_page(self.h, layer, page, k.ctypes.data_as(C.c_void_p), v.ctypes.data_as(C.c_void_p)))
        return k, v

    def close(self):
        if self.h:
            check(_L.vkb_kv_pool_destroy(self.h))
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def attention_dense(ctx: Context, q, seq_of_tok, k, v, n_ctx: int, n_head: int, d_head: int, out,
                    k_scale=None, v_scale=None):
    """Non-causal attention of q rows over per-stream dense K/V (f16, or int8 + f16 scales)."""
    import torch
    kv_dt = _lib.DT_F16 if k.dtype == torch.float16 else _lib.KV_Q8_0
    o_dt = _lib.DT_F16 if out.dtype == torch.float16 else _lib.DT_F32
    check(_L.vkb_attention_dense(ctx.h, q.shape[0], n_head, d_head, C.c_void_p(_ptr(q)), C.c_void_p(_ptr(seq_of_tok)),
                                 C.c_void_p(_ptr(k)), C.c_void_p(_ptr(v)), C.c_void_p(_ptr(k_scale)),
                                 C.c_void_p(_ptr(v_scale)), n_ctx, kv_dt, C.c_void_p(_ptr(out)), o_dt))


def quantize_rows_q8_0(ctx: Context, x, q_out, d_out):
    check(_L.vkb_quantize_rows_q8_0(ctx.h, C.c_void_p(_ptr(x)), x.shape[0], x.shape[1], C.c_void_p(_ptr(q_out)),
                                    C.c_void_p(_ptr(d_out))))


def log_mel(ctx: Context, pcm, n_mels: int, out=None, lengths=None):
    """whisper::mel::log_mel on the device for a batch: pcm is a torch f32
    [n_clips, n_samples] CUDA tensor (16 kHz); lengths (optional int32 CUDA
    tensor) the valid samples per clip. Returns (or fills) f32
    [n_clips, n_mels, 3000]."""
    import torch
    if pcm.dim() == 1:
        pcm = pcm.unsqueeze(0)
    assert pcm.dtype == torch.float32 and pcm.is_contiguous()
    n = pcm.shape[0]
    if out is None:
        out = torch.empty((n, n_mels, 3000), dtype=torch.float32, device=pcm.device)
    check(_L.vkb_log_mel(ctx.h, C.c_void_p(_ptr(pcm)) if pcm.numel() else None, n, pcm.shape[1],
                         C.c_void_p(_ptr(lengths)) if lengths is not None else None, n_mels, C.c_void_p(_ptr(out))))
    return out
