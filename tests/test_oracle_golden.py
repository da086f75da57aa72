"""The CPU oracle pinned against the reference's own known-answer tests
(tests/golden/kats.json, restated from the reference test sources)."""
import math

import numpy as np
import pytest

from oracle import py as o


def test_f16_decode_known_values(kats):
    for h, want in kats["f16_to_f32"]:
        assert o.f16_to_f32(h) == want
    assert math.isinf(o.f16_to_f32(kats["f16_to_f32_inf"][0]))
    assert math.isnan(o.f16_to_f32(kats["f16_to_f32_nan"][0]))


def test_f16_encode_corners(kats):
    for x in kats["f16_roundtrip"]:
        assert o.f16_to_f32(o.f32_to_f16(x)) == x
    for x, bits in kats["f32_to_f16_bits"]:
        assert o.f32_to_f16(float(x)) == bits
    n = o.f32_to_f16(float("nan"))
    assert (n >> 10) & 0x1F == 0x1F and n & 0x3FF != 0
    x = np.frombuffer(np.uint32(kats["f32_bits_to_f16_mantissa_zero"][0]).tobytes(), np.float32)[0]
    assert o.f32_to_f16(float(x)) & 0x3FF == 0
    sub = 2.0 ** -24
    assert o.f16_to_f32(o.f32_to_f16(sub)) == sub


def test_f16_encode_matches_ieee_rne_exhaustively_on_a_sample():
    # numpy's float16 cast is IEEE RNE; the restated encoder must agree on finite values.
    rng = np.random.default_rng(7)
    xs = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-7, 1e-5, 1e-2, 1, 100, 6e4)])
    for x in xs[::7]:
        assert o.f32_to_f16(float(x)) == int(np.float32(x).astype(np.float16).view(np.uint16))


def test_q4k_closed_form(kats):
    k = kats["q4k_closed_form"]
    out = o.dequantize(12, bytes(k["block"]), 256)
    d, dmin = o.f16_to_f32(k["d"]), o.f16_to_f32(k["dmin"])
    for n in range(256):
        kk = n // 64
        sub = 2 * kk if n % 64 < 32 else 2 * kk + 1
        want = np.float32(d) * np.float32(k["sc"][sub]) * np.float32(n % 16) - np.float32(dmin) * np.float32(k["m"][sub])
        assert abs(out[n] - want) < 1e-4


def test_q4k_uniform_and_two_blocks(kats):
    u = kats["q4k_uniform"]
    assert np.all(np.abs(o.dequantize(12, bytes(u["block"]), 256) - u["value"]) < 1e-4)
    t = kats["q4k_two_blocks"]
    out = o.dequantize(12, bytes(t["blocks"]), 512)
    assert np.all(np.abs(out[:256] - t["values"][0]) < 1e-4)
    assert np.all(np.abs(out[256:] - t["values"][1]) < 1e-4)


def test_kquant_zero_blocks_and_size_rejection(kats):
    for tag, size in kats["kquant_zero_block_sizes"]:
        assert np.all(o.dequantize(tag, bytes(size), 256) == 0.0)
    for tag, nbytes, n in kats["payload_mismatch"]:
        with pytest.raises(ValueError):
            o.dequantize(tag, bytes(nbytes), n)


def test_kv_block_saturation(kats):
    x = np.zeros(32, np.float32)
    s = kats["kv_q8_0_saturation"]
    x[0], x[1] = s["input_0"], s["input_1"]
    b = o.kv_pack(3, x)
    assert np.int8(b[2]) == s["qs0"] and np.int8(b[3]) == s["qs1"]
    s = kats["kv_q4_0_saturation"]
    x[0], x[1] = s["input_0"], s["input_1"]
    b = o.kv_pack(1, x)
    assert b[2] & 0xF == s["lo"] and (b[2] >> 4) & 0xF == s["hi"]
    s = kats["kv_q4_0_negative_bias"]
    x[0], x[1] = s["input_0"], s["input_1"]
    assert o.kv_pack(1, x)[2] & 0xF == s["lo"]
    s = kats["kv_q5_0_saturation"]
    x[0], x[1] = s["input_0"], s["input_1"]
    b = o.kv_pack(2, x)
    qh, qs = b[2:6], b[6:22]
    assert (qs[0] & 0xF) | ((qh[0] & 1) << 4) == s["b0"]
    assert ((qs[0] >> 4) & 0xF) | (((qh[0] >> 1) & 1) << 4) == s["b1"]


@pytest.mark.parametrize("mode,den", [(1, 7.0), (2, 15.0), (3, 127.0)])
def test_kv_round_trip_and_zeros(mode, den, kats):
    assert o.lib().orc_kv_block_bytes(mode) == kats["kv_block_bytes"][str(mode)]
    x = (np.arange(32, dtype=np.float32) / np.float32(31) * 2 - 1).astype(np.float32)
    y = o.kv_unpack(mode, o.kv_pack(mode, x))
    tol = 0.6 * (1.0 / den)
    assert np.all(np.abs(x - y) <= tol)
    z = o.kv_pack(mode, np.zeros(32, np.float32))
    assert z[0] == 0 and z[1] == 0
    assert np.all(o.kv_unpack(mode, z) == 0)


def test_erf_known_values(kats):
    for x, want in kats["erf"]:
        assert abs(o.erf(x) - want) < 1e-5


def test_paged_cache_invariants(kats):
    w = kats["pkv_on_wire"]
    c = o.PagedKv(*w["dims"], w["bs"], w["mode"])
    assert c.on_wire_storage_bytes() == w["bytes"]
    m = kats["pkv_multi_page"]
    c = o.PagedKv(*m["dims"], m["bs"], m["mode"])
    row = np.arange(32, dtype=np.float32) / 31
    for t in range(m["steps"]):
        assert c.append_step(0, t, 0, 0, row, np.zeros(32, np.float32)) == 0
    assert c.pages_in_use() == m["pages"]
    c.reset()
    assert c.pages_in_use() == 0 and c.read_step(0, 0, 0) is None
    cc = kats["pkv_construct"]
    c = o.PagedKv(*cc["dims"], cc["bs"], 3)
    assert c.page_table().size == cc["pages"]


def test_paged_cache_release_layer_and_isolation():
    c = o.PagedKv(2, 1, 32, 1, 1, 4, 4, 3)
    row = np.full(32, 0.5, np.float32)
    for layer in range(2):
        c.append_step(layer, 0, 0, 0, row, row)
    assert c.pages_in_use() == 2
    assert c.release_layer(0) == 0 and c.pages_in_use() == 1
    assert c.read_step(0, 0, 0) is None and c.read_step(1, 0, 0) is not None
    assert c.release_layer(2) == 5
    s = o.PagedKv(1, 1, 32, 2, 1, 2, 2, 3)
    s0 = np.arange(32, dtype=np.float32) / 100
    s1 = s0 + 1
    s.append_step(0, 0, 0, 0, s0, s0)
    s.append_step(0, 0, 1, 0, s1, s1)
    k0, _ = s.read_step(0, 0, 0)
    k1, _ = s.read_step(0, 0, 1)
    assert k0[0] != k1[0]


def test_dequant_gemv_validation_and_exactness():
    rc, _ = o.dequant_gemv(0, np.zeros(0, np.uint8), 0, 0, np.zeros(0, np.float32))
    assert rc == 5
    rc, _ = o.dequant_gemv(3, np.zeros(4 * 2 * 34, np.uint8), 4, 2, np.zeros(63, np.float32))
    assert rc == 5
    rc, _ = o.dequant_gemv(3, np.zeros(100, np.uint8), 4, 2, np.zeros(64, np.float32))
    assert rc == 5
    rng = np.random.default_rng(0)
    a = rng.uniform(-1, 1, (8, 64)).astype(np.float32)
    x = rng.uniform(-1, 1, 64).astype(np.float32)
    b = o.kv_pack(3, a)
    rc, y = o.dequant_gemv(3, b, 8, 2, x)
    assert rc == 0
    deq = o.kv_unpack(3, b).reshape(8, 64)
    assert np.allclose(y, deq @ x, atol=1e-5)


def test_int8_route_equals_repeated_gemv_and_bound():
    # kquant_gemm_parity.rs:130 (GEMM == repeated GEMV, exact) and :205 (derived bound)
    rng = np.random.default_rng(3)
    n, k, m = 16, 512, 5
    w = rng.standard_normal(n * k).astype(np.float32) * 0.02
    wq = o.quantize(12, w)
    a = rng.standard_normal((m, k)).astype(np.float32)
    full = o.kquant_gemm_i8(12, a, wq, n, k)
    for i in range(m):
        row = o.kquant_gemm_i8(12, a[i:i + 1], wq, n, k)
        assert np.array_equal(full[i], row[0])
    ref = o.linear_q(12, a, wq, n, k)
    rb = wq.size // n
    for i in range(m):
        for j in range(n):
            bound = o.int8_error_bound(12, wq[j * rb:(j + 1) * rb], k, a[i])
            assert abs(full[i, j] - ref[i, j]) <= 2 * bound + 1e-6


def test_linear_r1_is_ascending_fma_chain():
    rng = np.random.default_rng(5)
    a = rng.standard_normal((3, 64)).astype(np.float32)
    w = rng.standard_normal((4, 64)).astype(np.float32)
    b = rng.standard_normal(4).astype(np.float32)
    out = o.linear_f32(a, w, b)
    # a*b is exact in float64 and one float64 add then a float32 rounding equals the
    # single-rounded fma except on measure-zero ties.
    for i in range(3):
        for j in range(4):
            acc = np.float32(b[j])
            for l in range(64):
                acc = np.float32(float(a[i, l]) * float(w[j, l]) + float(acc))
            assert out[i, j] == acc
