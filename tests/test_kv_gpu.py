"""Paged quantized KV cache on the B200: bit-exact Q8_0 bytes and page tables
against the oracle QuantizedPagedKvCache, and decode attention over the pages."""
import numpy as np
import pytest

from oracle import py as o
from vokra_b200 import _lib

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to("cuda:0")


def _rows(rng, n, w):
    x = rng.standard_normal((n, w)).astype(np.float32)
    # edge blocks: all-zero, huge, tiny, one NaN, exact ties
    x[0, :32] = 0.0
    x[0, 32:64] = 1e30
    if n > 1:
        x[1, :32] = 1e-30
        x[1, 40] = np.nan
        if w >= 96:
            x[1, 64:96] = np.float32(127.0) * np.arange(32, dtype=np.float32) / 64
    return x


@pytest.mark.parametrize("mode", [_lib.KV_Q8_0, _lib.KV_Q4_0, _lib.KV_Q5_0])
def test_append_bytes_and_page_table_match_reference_layout(ctx, mode):
    """BlockQ8_0 / BlockQ4_0 / BlockQ5_0 ::pack on the device: page bytes, page
    table, read_step, release_layer and reset against the oracle cache."""
    from vokra_b200 import ops
    n_layer, n_head, d_head, n_stream, max_time, bs = 2, 2, 32, 3, 12, 4
    dims = ops.KvDims(n_layer, n_head, d_head, n_stream, 1, max_time)
    dev = ops.QuantizedPagedKvCache(ctx, dims, bs, mode, _lib.KV_LAYOUT_REFERENCE)
    ref = o.PagedKv(n_layer, n_head, d_head, n_stream, 1, max_time, bs, mode)
    w = n_head * d_head
    rng = np.random.default_rng(0)
    steps = [([0, 0, 1], [0, 1, 0]), ([0, 1, 2], [2, 1, 0]), ([2], [1]), ([1, 1, 1, 1], [2, 3, 4, 5])]
    for seqs, poss in steps:
        dev.begin_step(seqs, poss)
        for layer in range(n_layer):
            k = _rows(rng, len(seqs), w)
            v = _rows(rng, len(seqs), w)
            dev.append(layer, _dev(k), _dev(v))
            for i, (s, t) in enumerate(zip(seqs, poss)):
                assert ref.append_step(layer, t, s, 0, k[i], v[i]) == 0
        ctx.synchronize()
        assert np.array_equal(dev.page_table(), ref.page_table())
    assert dev.pages_in_use() == ref.pages_in_use()
    assert dev.on_wire_storage_bytes() == ref.on_wire_storage_bytes()
    for pid in range(ref.page_table().size):
        dk, dv = dev.read_page(pid)
        rk, rv = ref.page(pid)
        assert np.array_equal(dk, rk), pid
        assert np.array_equal(dv, rv), pid
    kk, vv = dev.read_step(1, 3, 1)
    rk, rv = ref.read_step(1, 3, 1)
    assert np.array_equal(kk, rk) and np.array_equal(vv, rv)
    dev.release_layer(0)
    ref.release_layer(0)
    assert np.array_equal(dev.page_table(), ref.page_table())
    dev.reset()
    ref.reset()
    assert dev.pages_in_use() == 0 and dev.read_step(0, 0, 0) is None


def test_reference_layout_exhaustion(ctx):
    from vokra_b200 import ops
    dims = ops.KvDims(1, 1, 32, 1, 1, 4)
    c = ops.QuantizedPagedKvCache(ctx, dims, 4, _lib.KV_Q8_0, _lib.KV_LAYOUT_REFERENCE)
    with pytest.raises(ops.VkbError) as e:
        c.begin_step([0], [4])
    assert e.value.code == _lib.ERROR_INVALID_ARGUMENT
    with pytest.raises(ops.VkbError) as e:
        ops.QuantizedPagedKvCache(ctx, dims, 4, _lib.KV_FP32)
    assert e.value.code == _lib.ERROR_INVALID_ARGUMENT
    with pytest.raises(ops.VkbError) as e:
        ops.QuantizedPagedKvCache(ctx, ops.KvDims(1, 1, 33, 1, 1, 4), 4, _lib.KV_Q8_0)
    assert e.value.code == _lib.ERROR_INVALID_ARGUMENT


def test_sequence_pool_exhaustion_is_reported(ctx):
    from vokra_b200 import ops
    dims = ops.KvDims(2, 2, 32, 4, 1, 64)
    c = ops.QuantizedPagedKvCache(ctx, dims, 16, _lib.KV_Q8_0, _lib.KV_LAYOUT_SEQUENCE, n_pages=2)
    c.begin_step([0, 1], [0, 0])
    with pytest.raises(ops.VkbError) as e:
        c.begin_step([2], [0])
    assert e.value.code == _lib.ERROR_KV_CACHE_EXHAUSTED
    c.release_seq(0)
    c.begin_step([2], [0])
    assert c.pages_in_use() == 2


def _oracle_attention(kv_rows_k, kv_rows_v, q, n_head, causal_pos):
    # q: [n_q, w] with positions causal_pos[i]; keys 0..pos
    out = np.zeros_like(q)
    for i in range(q.shape[0]):
        L = causal_pos[i] + 1
        out[i] = o.attention(q[i:i + 1], kv_rows_k[:L], kv_rows_v[:L], n_head)[0]
    return out


def _store(mode, x):
    """What a pool of `mode` gives back for rows x (the block pack round trip)."""
    if mode == _lib.KV_FP32:
        return x
    return o.kv_unpack(mode, o.kv_pack(mode, x)).reshape(x.shape)


@pytest.mark.parametrize("n_head,d_head,mode", [(2, 64, _lib.KV_Q8_0), (20, 64, _lib.KV_Q8_0), (8, 64, _lib.KV_Q8_0),
                                                (20, 64, _lib.KV_Q4_0), (20, 64, _lib.KV_Q5_0),
                                                (20, 64, _lib.KV_FP32), (4, 32, _lib.KV_Q5_0)])
def test_paged_attention_sequence_layout(ctx, n_head, d_head, mode):
    import torch
    from vokra_b200 import ops
    rng = np.random.default_rng(n_head)
    n_layer, n_seq, max_time, bs = 2, 5, 200, 16
    w = n_head * d_head
    dims = ops.KvDims(n_layer, n_head, d_head, n_seq, 1, max_time)
    pool = ops.QuantizedPagedKvCache(ctx, dims, bs, mode, _lib.KV_LAYOUT_SEQUENCE)
    # scatter pages by a seeded permutation (config 3)
    pps = (max_time + bs - 1) // bs
    perm = rng.permutation(n_seq * pps).astype(np.int32)
    pool.set_page_table(perm)
    lengths = [1, 17, 64, 130, 199]
    Ks = [[rng.standard_normal((L, w)).astype(np.float32) for L in lengths] for _ in range(n_layer)]
    Vs = [[rng.standard_normal((L, w)).astype(np.float32) for L in lengths] for _ in range(n_layer)]
    # fill with a prefix step (4 tokens per stream) then one-token steps
    maxlen = max(lengths)
    t = 0
    while t < maxlen:
        seqs, poss = [], []
        for s, L in enumerate(lengths):
            take = 4 if t == 0 else 1
            for j in range(t, min(L, t + take)):
                seqs.append(s)
                poss.append(j)
        pool.begin_step(seqs, poss)
        for layer in range(n_layer):
            k = np.stack([Ks[layer][s][p] for s, p in zip(seqs, poss)])
            v = np.stack([Vs[layer][s][p] for s, p in zip(seqs, poss)])
            pool.append(layer, _dev(k), _dev(v))
        t += 4 if t == 0 else 1
    # final step: one query per stream at its last position (attends 0..L-1)
    seqs = list(range(n_seq))
    poss = [L - 1 for L in lengths]
    # re-declare the last positions (the pages exist; appends overwrite identical bytes)
    pool.begin_step(seqs, poss)
    layer = 1
    kl = np.stack([Ks[layer][s][p] for s, p in zip(seqs, poss)])
    vl = np.stack([Vs[layer][s][p] for s, p in zip(seqs, poss)])
    pool.append(layer, _dev(kl), _dev(vl))
    q = rng.standard_normal((n_seq, w)).astype(np.float32) * np.float32(d_head ** -0.5)
    out = torch.zeros((n_seq, w), dtype=torch.float32, device="cuda:0")
    pool.attention(layer, _dev(q), out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for s, L in enumerate(lengths):
        kd = _store(mode, Ks[layer][s])
        vd = _store(mode, Vs[layer][s])
        ref = o.attention(q[s:s + 1], kd, vd, n_head)[0]
        assert np.max(np.abs(got[s] - ref)) <= 1e-4, (s, np.max(np.abs(got[s] - ref)))
    if mode != _lib.KV_FP32:  # the last rows' page bytes: the reference block encoding
        table = pool.page_table().reshape(n_seq, -1)
        for s, L in enumerate(lengths):
            kp, _ = pool.read_page(int(table[s, (L - 1) // bs]), layer)
            n_rows = (L - 1) % bs + 1
            rows = Ks[layer][s][(L - 1) // bs * bs:L]
            assert np.array_equal(kp.reshape(bs, -1)[:n_rows].reshape(-1), o.kv_pack(mode, rows))


def test_paged_attention_prefix_causal(ctx):
    import torch
    from vokra_b200 import ops
    rng = np.random.default_rng(9)
    n_head, d_head = 4, 64
    w = n_head * d_head
    dims = ops.KvDims(1, n_head, d_head, 2, 1, 64)
    pool = ops.QuantizedPagedKvCache(ctx, dims, 16, _lib.KV_Q8_0, _lib.KV_LAYOUT_SEQUENCE)
    seqs = [0, 0, 0, 0, 1, 1, 1, 1, 1, 1]
    poss = [0, 1, 2, 3, 0, 1, 2, 3, 4, 5]
    k = rng.standard_normal((10, w)).astype(np.float32)
    v = rng.standard_normal((10, w)).astype(np.float32)
    q = rng.standard_normal((10, w)).astype(np.float32) * np.float32(0.125)
    pool.begin_step(seqs, poss)
    pool.append(0, _dev(k), _dev(v))
    out = torch.zeros((10, w), dtype=torch.float32, device="cuda:0")
    pool.attention(0, _dev(q), out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    kd = o.kv_unpack(3, o.kv_pack(3, k)).reshape(10, w)
    vd = o.kv_unpack(3, o.kv_pack(3, v)).reshape(10, w)
    for base, n in [(0, 4), (4, 6)]:
        ref = o.attention(q[base:base + n], kd[base:base + n], vd[base:base + n], n_head, causal=True, q_off=0)
        assert np.max(np.abs(got[base:base + n] - ref)) <= 1e-4


def test_reference_layout_attention(ctx):
    import torch
    from vokra_b200 import ops
    rng = np.random.default_rng(4)
    n_head, d_head, n_stream = 2, 64, 3
    w = n_head * d_head
    dims = ops.KvDims(1, n_head, d_head, n_stream, 1, 40)
    pool = ops.QuantizedPagedKvCache(ctx, dims, 4, _lib.KV_Q8_0, _lib.KV_LAYOUT_REFERENCE)
    L = 23
    K = rng.standard_normal((n_stream, L, w)).astype(np.float32)
    V = rng.standard_normal((n_stream, L, w)).astype(np.float32)
    for t in range(L):
        pool.begin_step(list(range(n_stream)), [t] * n_stream)
        pool.append(0, _dev(K[:, t]), _dev(V[:, t]))
    q = rng.standard_normal((n_stream, w)).astype(np.float32) * np.float32(0.125)
    pool.begin_step(list(range(n_stream)), [L - 1] * n_stream)
    pool.append(0, _dev(K[:, L - 1]), _dev(V[:, L - 1]))
    out = torch.zeros((n_stream, w), dtype=torch.float16, device="cuda:0")
    pool.attention(0, _dev(q), out)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    for s in range(n_stream):
        kd = o.kv_unpack(3, o.kv_pack(3, K[s])).reshape(L, w)
        vd = o.kv_unpack(3, o.kv_pack(3, V[s])).reshape(L, w)
        ref = o.attention(q[s:s + 1], kd, vd, n_head)[0]
        assert np.max(np.abs(got[s] - ref)) <= 2e-3


@pytest.mark.parametrize("kv", ["f16", "q8"])
def test_dense_cross_attention(ctx, kv):
    import torch
    from vokra_b200 import ops
    rng = np.random.default_rng(5)
    n_head, d_head, n_ctx, n_seq = 20, 64, 1500, 3
    w = n_head * d_head
    K = rng.standard_normal((n_seq * n_ctx, w)).astype(np.float32)
    V = rng.standard_normal((n_seq * n_ctx, w)).astype(np.float32)
    q = rng.standard_normal((5, w)).astype(np.float32) * np.float32(0.125)
    seq_of_tok = np.array([0, 2, 1, 2, 0], np.int32)
    out = torch.zeros((5, w), dtype=torch.float32, device="cuda:0")
    st = torch.from_numpy(seq_of_tok).to("cuda:0")
    if kv == "f16":
        kt, vt = _dev(K).half(), _dev(V).half()
        ops.attention_dense(ctx, _dev(q), st, kt, vt, n_ctx, n_head, d_head, out)
        Kr = K.astype(np.float16).astype(np.float32)
        Vr = V.astype(np.float16).astype(np.float32)
    else:
        kq = torch.zeros((n_seq * n_ctx, w), dtype=torch.int8, device="cuda:0")
        vq = torch.zeros_like(kq)
        kd = torch.zeros((n_seq * n_ctx, w // 32), dtype=torch.float16, device="cuda:0")
        vd = torch.zeros_like(kd)
        ops.quantize_rows_q8_0(ctx, _dev(K), kq, kd)
        ops.quantize_rows_q8_0(ctx, _dev(V), vq, vd)
        torch.cuda.synchronize()
        # bit-exact against BlockQ8_0::pack
        blocks = o.kv_pack(3, K[:64]).reshape(-1, 34)
        assert np.array_equal(kq[:64].cpu().numpy().reshape(-1, 32).view(np.uint8), blocks[:, 2:])
        assert np.array_equal(kd[:64].cpu().numpy().reshape(-1).view(np.uint16),
                              blocks[:, :2].copy().view(np.uint16).reshape(-1))
        ops.attention_dense(ctx, _dev(q), st, kq, vq, n_ctx, n_head, d_head, out, k_scale=kd, v_scale=vd)
        Kr = o.kv_unpack(3, o.kv_pack(3, K)).reshape(K.shape)
        Vr = o.kv_unpack(3, o.kv_pack(3, V)).reshape(V.shape)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for i, s in enumerate(seq_of_tok):
        ref = o.attention(q[i:i + 1], Kr[s * n_ctx:(s + 1) * n_ctx], Vr[s * n_ctx:(s + 1) * n_ctx], n_head)[0]
        assert np.max(np.abs(got[i] - ref)) <= 1e-4


@pytest.mark.parametrize("n_head,n_ctx,n_tok,n_seq", [
    (8, 1000, 40, 10),   # ragged last chunk of keys, several CTAs per query row
    (20, 7, 3, 2),       # fewer keys than one chunk
    (12, 1500, 1, 1),    # one query row spread over every SM
    (6, 100, 4, 2),      # n_head*d_head = 384: served by the row-group kernel
    (16, 333, 300, 5),   # many query rows per stream, rows crossing CTA ranges
])
def test_dense_cross_attention_q8_shapes(ctx, n_head, n_ctx, n_tok, n_seq):
    import torch
    from vokra_b200 import ops
    rng = np.random.default_rng(n_head * 1000 + n_ctx)
    d_head = 64
    w = n_head * d_head
    K = rng.standard_normal((n_seq * n_ctx, w)).astype(np.float32)
    V = rng.standard_normal((n_seq * n_ctx, w)).astype(np.float32)
    q = rng.standard_normal((n_tok, w)).astype(np.float32) * np.float32(0.125)
    seq_of_tok = rng.integers(0, n_seq, n_tok).astype(np.int32)
    kq = torch.zeros((n_seq * n_ctx, w), dtype=torch.int8, device="cuda:0")
    vq = torch.zeros_like(kq)
    kd = torch.zeros((n_seq * n_ctx, w // 32), dtype=torch.float16, device="cuda:0")
    vd = torch.zeros_like(kd)
    ops.quantize_rows_q8_0(ctx, _dev(K), kq, kd)
    ops.quantize_rows_q8_0(ctx, _dev(V), vq, vd)
    out = torch.zeros((n_tok, w), dtype=torch.float32, device="cuda:0")
    st = torch.from_numpy(seq_of_tok).to("cuda:0")
    ops.attention_dense(ctx, _dev(q), st, kq, vq, n_ctx, n_head, d_head, out, k_scale=kd, v_scale=vd)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    Kr = o.kv_unpack(3, o.kv_pack(3, K)).reshape(K.shape)
    Vr = o.kv_unpack(3, o.kv_pack(3, V)).reshape(V.shape)
    for i, s in enumerate(seq_of_tok):
        ref = o.attention(q[i:i + 1], Kr[s * n_ctx:(s + 1) * n_ctx], Vr[s * n_ctx:(s + 1) * n_ctx], n_head)[0]
        assert np.max(np.abs(got[i] - ref)) <= 1e-4, (i, s)


@pytest.mark.parametrize("mode", [_lib.KV_Q4_0, _lib.KV_Q5_0, _lib.KV_Q8_0])
def test_dequant_gemv_m3_04_shapes(ctx, kats, mode):
    from vokra_b200 import ops
    gemv = ops.KvQuantDequantGemvOps(ctx)
    for n_rows, nbpr in kats["m3_04_shapes"]:
        per = nbpr * 32
        rng = np.random.default_rng(0xD3 ^ (n_rows * 131 + nbpr))
        a = rng.uniform(-1, 1, (n_rows, per)).astype(np.float32)
        x = rng.uniform(-1, 1, per).astype(np.float32)
        blocks = o.kv_pack(mode, a)
        rc, ref = o.dequant_gemv(mode, blocks, n_rows, nbpr, x)
        assert rc == 0
        got = gemv.fused_dequant_gemv(mode, blocks, n_rows, nbpr, x)
        assert np.max(np.abs(got - ref)) <= kats["dequant_gemv_atol"]
    with pytest.raises(ops.VkbError) as e:
        gemv.fused_dequant_gemv(_lib.KV_FP32, b"", 0, 0, np.zeros(0, np.float32))
    assert e.value.code == _lib.ERROR_INVALID_ARGUMENT


def _config2_pool(ctx, rng, n_seq=256, n_head=20, d_head=64, max_time=448, bs=16):
    """n_seq sequences, lengths U[16, 448], 16-token int8
    pages with one f16 scale per 32 channels, pages scattered by a seeded
    permutation; K/V of every position but the last already stored."""
    from vokra_b200 import ops
    w = n_head * d_head
    pool = ops.QuantizedPagedKvCache(ctx, ops.KvDims(1, n_head, d_head, n_seq, 1, max_time), bs, _lib.KV_Q8_0,
                                     _lib.KV_LAYOUT_SEQUENCE)
    pps = (max_time + bs - 1) // bs
    pool.set_page_table(rng.permutation(n_seq * pps).astype(np.int32))
    lengths = rng.integers(16, max_time + 1, n_seq)
    K = [rng.standard_normal((int(L), w)).astype(np.float32) for L in lengths]
    V = [rng.standard_normal((int(L), w)).astype(np.float32) for L in lengths]
    s0 = 0
    while s0 < n_seq:  # prefill steps of whole sequences, at most 2048 tokens each
        s1, n_tok = s0, 0
        while s1 < n_seq and n_tok + int(lengths[s1]) - 1 <= 2048:
            n_tok += int(lengths[s1]) - 1
            s1 += 1
        seqs, poss = [], []
        for s in range(s0, s1):
            seqs += [s] * (int(lengths[s]) - 1)
            poss += list(range(int(lengths[s]) - 1))
        pool.begin_step(seqs, poss)
        pool.append(0, _dev(np.concatenate([K[s][:-1] for s in range(s0, s1)])),
                    _dev(np.concatenate([V[s][:-1] for s in range(s0, s1)])))
        s0 = s1
    return pool, lengths, K, V


def test_fused_decode_step_config2(ctx):
    """The decode step's fused append + attention (the kernel vkb_session_step
    runs) over BASELINE configs[2]: 256 sequences, 20 heads, d_head 64, lengths
    U[16, 448], permuted pages. Each sequence appends its last K/V row and its
    one query attends over all of its keys; the context matches the oracle's
    attention over the Q8_0-dequantized K/V (nn.rs:209-300) within 1e-4, and
    the appended rows' page bytes equal BlockQ8_0::pack."""
    import torch
    rng = np.random.default_rng(2024)
    pool, lengths, K, V = _config2_pool(ctx, rng)
    n_seq, w, n_head = len(lengths), K[0].shape[1], 20
    pool.begin_step(list(range(n_seq)), [int(L) - 1 for L in lengths])
    assert pool.decode_fused()
    q = rng.standard_normal((n_seq, w)).astype(np.float32) * np.float32(64 ** -0.5)
    qkv = np.concatenate([q, np.stack([k[-1] for k in K]), np.stack([v[-1] for v in V])], axis=1)
    out = torch.zeros((n_seq, w), dtype=torch.float32, device="cuda:0")
    pool.append_attention(0, _dev(qkv), out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    worst = 0.0
    for s, L in enumerate(lengths):
        kd = o.kv_unpack(3, o.kv_pack(3, K[s])).reshape(int(L), w)
        vd = o.kv_unpack(3, o.kv_pack(3, V[s])).reshape(int(L), w)
        ref = o.attention(q[s:s + 1], kd, vd, n_head)[0]
        worst = max(worst, float(np.max(np.abs(got[s] - ref))))
    assert worst <= 1e-4, worst
    # the page holding each sequence's last row: bytes of the whole page prefix
    table = pool.page_table().reshape(n_seq, -1)
    for s in (0, 1, 100, n_seq - 1):
        L = int(lengths[s])
        pid = int(table[s, (L - 1) // 16])
        kp, vp = pool.read_page(pid, 0)
        n_rows = (L - 1) % 16 + 1
        rows = slice((L - 1) // 16 * 16, L)
        assert np.array_equal(kp.reshape(16, -1)[:n_rows].reshape(-1), o.kv_pack(3, K[s][rows]))
        assert np.array_equal(vp.reshape(16, -1)[:n_rows].reshape(-1), o.kv_pack(3, V[s][rows]))


def test_fused_decode_matches_unfused_route(ctx):
    """The fused kernel and the separate append + attention kernels give the
    same context (within 1e-5) on one decode step of 40 sequences."""
    import torch
    outs = []
    for fused in (True, False):
        rng = np.random.default_rng(77)
        pool, lengths, K, V = _config2_pool(ctx, rng, n_seq=40)
        n_seq, w = len(lengths), K[0].shape[1]
        pool.begin_step(list(range(n_seq)), [int(L) - 1 for L in lengths])
        q = rng.standard_normal((n_seq, w)).astype(np.float32) * np.float32(0.125)
        kl, vl = np.stack([k[-1] for k in K]), np.stack([v[-1] for v in V])
        out = torch.zeros((n_seq, w), dtype=torch.float32, device="cuda:0")
        if fused:
            pool.append_attention(0, _dev(np.concatenate([q, kl, vl], axis=1)), out)
        else:
            pool.append(0, _dev(kl), _dev(vl))
            pool.attention(0, _dev(q), out)
        torch.cuda.synchronize()
        outs.append(out.cpu().numpy())
        pool.close()
    assert np.max(np.abs(outs[0] - outs[1])) <= 1e-5


def test_copy_stream_shares_pages_copy_on_write(ctx):
    """Beam branching on the pool: vkb_kv_copy_stream shares the source's
    filled pages (only a partly filled last page is copied), and a later write
    into a shared page copies it first, so no stream sees another's K/V."""
    import torch
    from vokra_b200 import ops
    rng = np.random.default_rng(31)
    n_head, d_head, bs = 4, 64, 16
    w = n_head * d_head
    pool = ops.QuantizedPagedKvCache(ctx, ops.KvDims(1, n_head, d_head, 4, 1, 128), bs, _lib.KV_Q8_0,
                                     _lib.KV_LAYOUT_SEQUENCE)
    K = rng.standard_normal((40, w)).astype(np.float32)
    V = rng.standard_normal((40, w)).astype(np.float32)
    pool.begin_step([0] * 37, list(range(37)))
    pool.append(0, _dev(K[:37]), _dev(V[:37]))
    assert pool.pages_in_use() == 3
    pool.copy_stream(0, 1, 37)  # two full pages shared, the third copied
    assert pool.pages_in_use() == 4
    pool.copy_stream(0, 2, 32)  # two full pages shared, nothing copied
    assert pool.pages_in_use() == 4
    table = pool.page_table().reshape(4, -1)
    assert table[1, 0] == table[0, 0] and table[1, 1] == table[0, 1] and table[1, 2] != table[0, 2]
    assert table[2, 0] == table[0, 0] and table[2, 2] == -1
    # stream 2 overwrites position 20 (inside a shared page): it gets its own copy
    K2 = rng.standard_normal((1, w)).astype(np.float32)
    pool.begin_step([2], [20])
    pool.append(0, _dev(K2), _dev(K2))
    assert pool.pages_in_use() == 5
    table = pool.page_table().reshape(4, -1)
    assert table[2, 1] != table[0, 1] and table[2, 0] == table[0, 0]
    # every stream still reads its own history
    got0, _ = pool.read_step(0, 20, 0)
    got2, _ = pool.read_step(0, 20, 2)
    got2b, _ = pool.read_step(0, 21, 2)
    ref = lambda x: o.kv_unpack(3, o.kv_pack(3, x)).reshape(-1, w)
    assert np.array_equal(got0, ref(K[20:21])[0])
    assert np.array_equal(got2, ref(K2)[0])
    assert np.array_equal(got2b, ref(K[21:22])[0])  # the rest of the copied page came along
    # the branches attend over their own keys
    pool.begin_step([0, 1], [37, 37])
    kn = rng.standard_normal((2, w)).astype(np.float32)
    pool.append(0, _dev(kn), _dev(kn))
    q = rng.standard_normal((2, w)).astype(np.float32) * np.float32(0.125)
    out = torch.zeros((2, w), dtype=torch.float32, device="cuda:0")
    pool.attention(0, _dev(q), out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for s in range(2):
        kd = ref(np.concatenate([K[:37], kn[s:s + 1]]))
        vd = ref(np.concatenate([V[:37], kn[s:s + 1]]))
        assert np.max(np.abs(got[s] - o.attention(q[s:s + 1], kd, vd, n_head)[0])) <= 1e-4
    # releasing the source keeps the shared pages for the branches
    pool.release_seq(0)
    assert pool.pages_in_use() == 4  # page 0 (streams 1, 2), page 1 (stream 1), stream 1's page 2, stream 2's page 1
    pool.release_seq(1)
    pool.release_seq(2)
    assert pool.pages_in_use() == 0
