"""The allocation-free cross-attention entry point.

vkb_attention_dense_noalloc serves callers that cannot let a library allocate
device memory during a call (a host with its own fixed device-memory budget, a
real-time audio path, an engine recording work). It keeps its split partials in
a fixed array inside the library instead of the context workspace. This test
calls it through the C ABI and checks it against vkb_attention_dense on two
calls in a row (the second with new inputs, so stale scratch contents from the
first call must not leak into the result), against the oracle's attention at
a size that takes the reduced-CTA plan of the Q8_0 kernel, that a fresh
context's workspace stays unallocated through it, and the size limit.

Kept in its own file named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import py as o
from vokra_b200 import _lib

pytestmark = pytest.mark.gpu


def _call(fn, ctx, q, seq, k, v, ks, vs, n_ctx, n_head, d_head, kv_dt, out):
    return fn(ctx.h, q.shape[0], n_head, d_head, C.c_void_p(q.data_ptr()), C.c_void_p(seq.data_ptr()),
              C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()),
              C.c_void_p(ks.data_ptr()) if ks is not None else None,
              C.c_void_p(vs.data_ptr()) if vs is not None else None, n_ctx, kv_dt, C.c_void_p(out.data_ptr()),
              _lib.DT_F32)


@pytest.mark.parametrize("kv", ["q8", "f16"])
def test_noalloc_attention_matches_the_allocating_entry_point(ctx, kv):
    import torch
    from vokra_b200 import ops
    L = _lib.load()
    n_head, d_head, n_ctx, n_seq, n_tok = 20, 64, 1500, 4, 7
    w = n_head * d_head
    for call in range(2):
        rng = np.random.default_rng(100 + call)
        K = torch.from_numpy(rng.standard_normal((n_seq * n_ctx, w)).astype(np.float32)).cuda()
        V = torch.from_numpy(rng.standard_normal((n_seq * n_ctx, w)).astype(np.float32)).cuda()
        q = torch.from_numpy(rng.standard_normal((n_tok, w)).astype(np.float32) * np.float32(0.125)).cuda()
        seq = torch.from_numpy(rng.integers(0, n_seq, n_tok).astype(np.int32)).cuda()
        if kv == "q8":
            kq = torch.empty((n_seq * n_ctx, w), dtype=torch.int8, device="cuda")
            vq = torch.empty_like(kq)
            kd = torch.empty((n_seq * n_ctx, w // 32), dtype=torch.float16, device="cuda")
            vd = torch.empty_like(kd)
            ops.quantize_rows_q8_0(ctx, K, kq, kd)
            ops.quantize_rows_q8_0(ctx, V, vq, vd)
            args = (kq, vq, kd, vd, _lib.KV_Q8_0)
        else:
            args = (K.half(), V.half(), None, None, _lib.DT_F16)
        ref = torch.zeros((n_tok, w), dtype=torch.float32, device="cuda")
        got = torch.full((n_tok, w), float("nan"), dtype=torch.float32, device="cuda")
        _lib.check(_call(L.vkb_attention_dense, ctx, q, seq, args[0], args[1], args[2], args[3], n_ctx, n_head,
                         d_head, args[4], ref))
        _lib.check(_call(L.vkb_attention_dense_noalloc, ctx, q, seq, args[0], args[1], args[2], args[3], n_ctx,
                         n_head, d_head, args[4], got))
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert float((got - ref).abs().max()) <= 1e-4, call


def test_noalloc_attention_rejects_sizes_beyond_its_scratch(ctx):
    import torch
    L = _lib.load()
    n_head, d_head = 20, 64
    w = n_head * d_head
    cap = 4 * 1024 * 1024
    n_tok = cap // (w + 2 * n_head) + 1
    q = torch.zeros((n_tok, w), dtype=torch.float32, device="cuda")
    seq = torch.zeros(n_tok, dtype=torch.int32, device="cuda")
    kv = torch.zeros((16, w), dtype=torch.float16, device="cuda")
    out = torch.zeros_like(q)
    st = _call(L.vkb_attention_dense_noalloc, ctx, q, seq, kv, kv, None, None, 16, n_head, d_head, _lib.DT_F16, out)
    assert st == _lib.ERROR_INVALID_ARGUMENT
    assert b"fixed scratch" in L.vkb_last_error()


def test_noalloc_attention_reduced_plan_matches_oracle_without_workspace():
    """3000 query rows over 32-key contexts: one partial slot per row, so the
    148-CTA plan needs more than the fixed scratch and the kernel runs on 74
    CTAs. Results against the oracle's attention over the unpacked Q8_0 rows
    (crates/vokra-models/src/whisper/nn.rs:209-300); a fresh context's
    workspace is still unallocated afterwards, on both paths."""
    import torch
    from vokra_b200 import ops
    L = _lib.load()
    ctx = ops.Context(0)
    assert L.vkb_context_workspace_bytes(ctx.h) == 0
    n_head, d_head, n_ctx, n_seq, n_tok = 20, 64, 32, 4, 3000
    w = n_head * d_head
    rng = np.random.default_rng(77)
    K = rng.standard_normal((n_seq * n_ctx, w)).astype(np.float32)
    V = rng.standard_normal((n_seq * n_ctx, w)).astype(np.float32)
    q = rng.standard_normal((n_tok, w)).astype(np.float32) * np.float32(0.125)
    seq_of_tok = rng.integers(0, n_seq, n_tok).astype(np.int32)
    dev = lambda a: torch.from_numpy(a).cuda()
    kq = torch.empty((n_seq * n_ctx, w), dtype=torch.int8, device="cuda")
    vq = torch.empty_like(kq)
    kd = torch.empty((n_seq * n_ctx, w // 32), dtype=torch.float16, device="cuda")
    vd = torch.empty_like(kd)
    ops.quantize_rows_q8_0(ctx, dev(K), kq, kd)
    ops.quantize_rows_q8_0(ctx, dev(V), vq, vd)
    out = torch.full((n_tok, w), float("nan"), dtype=torch.float32, device="cuda")
    _lib.check(_call(L.vkb_attention_dense_noalloc, ctx, dev(q), dev(seq_of_tok), kq, vq, kd, vd, n_ctx, n_head,
                     d_head, _lib.KV_Q8_0, out))
    out16 = torch.full((n_tok, w), float("nan"), dtype=torch.float32, device="cuda")
    _lib.check(_call(L.vkb_attention_dense_noalloc, ctx, dev(q), dev(seq_of_tok), dev(K).half(), dev(V).half(),
                     None, None, n_ctx, n_head, d_head, _lib.DT_F16, out16))
    torch.cuda.synchronize()
    assert L.vkb_context_workspace_bytes(ctx.h) == 0
    Kr = o.kv_unpack(3, o.kv_pack(3, K)).reshape(K.shape)
    Vr = o.kv_unpack(3, o.kv_pack(3, V)).reshape(V.shape)
    K16 = K.astype(np.float16).astype(np.float32)
    V16 = V.astype(np.float16).astype(np.float32)
    got, got16 = out.cpu().numpy(), out16.cpu().numpy()
    for s in range(n_seq):
        rows = np.nonzero(seq_of_tok == s)[0]
        ref = o.attention(q[rows], Kr[s * n_ctx:(s + 1) * n_ctx], Vr[s * n_ctx:(s + 1) * n_ctx], n_head)
        assert np.max(np.abs(got[rows] - ref)) <= 1e-4, s
        ref16 = o.attention(q[rows], K16[s * n_ctx:(s + 1) * n_ctx], V16[s * n_ctx:(s + 1) * n_ctx], n_head)
        assert np.max(np.abs(got16[rows] - ref16)) <= 1e-4, s
