"""Writes tests/golden/kats.json: the reference's own known-answer tests for this
path, restated as data. Every literal below is read from the reference test
sources named beside it (paths relative to the reference repository root);
nothing is computed here except the closed forms those tests state.

Run: python tests/golden/make_golden.py
"""
import json
import os

HERE = os.path.dirname(os.path.abspath(__file__))


def pack_scales(sc, m):
    # inverse of get_scale_min_k4, as the in-test encoder of
    # crates/vokra-core/src/gguf/quant/q4_k.rs:96-110
    s = [0] * 12
    for j in range(8):
        if j < 4:
            s[j] = sc[j] & 63
            s[j + 4] = m[j] & 63
        else:
            s[j + 4] = (sc[j] & 0xF) | ((m[j] & 0xF) << 4)
            s[j - 4] |= (sc[j] >> 4) << 6
            s[j] |= (m[j] >> 4) << 6
    return s


def q4k_block(d, dmin, scales, quants):
    # build_block (q4_k.rs:112-130): low nibble = element 64k+l, high = 64k+32+l
    b = [d & 0xFF, d >> 8, dmin & 0xFF, dmin >> 8] + list(scales)
    qs = [0] * 128
    for k in range(4):
        for l in range(32):
            qs[32 * k + l] = (quants[64 * k + l] & 0xF) | ((quants[64 * k + 32 + l] & 0xF) << 4)
    return b + qs


kats = {
    # crates/vokra-core/src/gguf/quant/mod.rs:152-162 f16_to_f32_matches_known_values
    "f16_to_f32": [[0x3C00, 1.0], [0x4000, 2.0], [0xC000, -2.0], [0x0000, 0.0], [0x3800, 0.5],
                   [0x0001, 2.0 ** -24]],
    "f16_to_f32_inf": [0x7C00],
    "f16_to_f32_nan": [0x7E00],
    # crates/vokra-core/src/kv_quant/half.rs:158-215
    "f16_roundtrip": [1.0, 2.0, -2.0, 0.5, 0.25, 3.25, 65504.0, -65504.0],
    "f32_to_f16_bits": [[0.0, 0x0000], ["-0.0", 0x8000], [1.0e5, 0x7C00], [-1.0e5, 0xFC00], ["inf", 0x7C00],
                        [1.0e-10, 0x0000], [-1.0e-10, 0x8000]],
    "f32_bits_to_f16_mantissa_zero": [0x3F800800],   # round_to_nearest_even_direction
    # q4_k.rs:132-160 closed_form_matches_distinct_scales_and_quants
    "q4k_closed_form": {"d": 0x3C00, "dmin": 0x3800, "sc": [1, 2, 3, 4, 5, 6, 7, 8], "m": [8, 7, 6, 5, 4, 3, 2, 1],
                        "block": q4k_block(0x3C00, 0x3800, pack_scales([1, 2, 3, 4, 5, 6, 7, 8],
                                                                        [8, 7, 6, 5, 4, 3, 2, 1]),
                                           [i % 16 for i in range(256)])},
    # q4_k.rs:163-175 uniform_block_is_a_known_constant -> 19.0
    "q4k_uniform": {"block": q4k_block(0x4000, 0x3C00, pack_scales([3] * 8, [5] * 8), [4] * 256), "value": 19.0},
    # q4_k.rs:177-188 two_blocks_decode_independently -> 7.0 then 6.0
    "q4k_two_blocks": {"blocks": q4k_block(0x3C00, 0x0000, pack_scales([1] * 8, [0] * 8), [7] * 256) +
                       q4k_block(0x3C00, 0x0000, pack_scales([2] * 8, [0] * 8), [3] * 256), "values": [7.0, 6.0]},
    # gguf/quant/mod.rs:190-205: all-zero K-quant blocks decode to zeros; size rejections
    "kquant_zero_block_sizes": [[12, 144], [13, 176], [14, 210]],
    "payload_mismatch": [[12, 100, 256], [14, 210, 200]],
    # kv_quant/q8_0.rs:140-160 saturation_at_range_edges: qs[0] = 127, qs[1] = -127
    "kv_q8_0_saturation": {"input_0": 1000.0, "input_1": -1000.0, "qs0": 127, "qs1": -127},
    # kv_quant/q4_0.rs:141-170 saturation (low nibble 15, high nibble 1) and negative bias (low nibble 1)
    "kv_q4_0_saturation": {"input_0": 1000.0, "input_1": -1000.0, "lo": 15, "hi": 1},
    "kv_q4_0_negative_bias": {"input_0": -1000.0, "input_1": 500.0, "lo": 1},
    # kv_quant/q5_0.rs:184-196 saturation: biased 31 and 1
    "kv_q5_0_saturation": {"input_0": 1000.0, "input_1": -1000.0, "b0": 31, "b1": 1},
    # block byte sizes (q4_0/q5_0/q8_0 block_size_bytes_pin)
    "kv_block_bytes": {"1": 18, "2": 22, "3": 34},
    # kernels/scalar.rs:236-248 erf_matches_reference_values (|err| < 1e-5)
    "erf": [[0.0, 0.0], [0.5, 0.5204999], [1.0, 0.8427008], [2.0, 0.9953223], [-1.0, -0.8427008]],
    # cache/paged_quant.rs:795-805 on_wire_storage_bytes_matches_arithmetic
    "pkv_on_wire": {"dims": [1, 1, 32, 1, 1, 8], "bs": 4, "mode": 3, "bytes": 544},
    # paged_quant.rs:707-735 multi_page_reuse_and_reset: 6 steps at bs=2 -> 3 pages in use
    "pkv_multi_page": {"dims": [1, 1, 32, 1, 1, 6], "bs": 2, "mode": 1, "steps": 6, "pages": 3},
    # paged_quant.rs:602-612 all_three_modes_construct_ok: dims (1,32,4) at bs=4 -> 1 page
    "pkv_construct": {"dims": [1, 1, 32, 1, 1, 4], "bs": 4, "pages": 1},
    # crates/vokra-backend-cuda/tests/parity_kernels_cuda.rs:2169-2178 M3_04_SHAPES, bound 1e-4
    "m3_04_shapes": [[1, 1], [1, 8], [2, 2], [4, 2], [16, 2], [32, 4], [128, 2], [256, 4]],
    "dequant_gemv_atol": 1e-4,
}

if __name__ == "__main__":
    with open(os.path.join(HERE, "kats.json"), "w") as f:
        json.dump(kats, f, indent=1)
    print("wrote kats.json")
