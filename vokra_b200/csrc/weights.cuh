// weights.cuh — device layout of an uploaded (repacked) Linear weight and the
// per-stage dequantization shared by the GEMV and the tcgen05 GEMM kernels.
//
// Layout (built once at upload by repack_weight, never on the hot path):
// rows are grouped in tiles of 128 (n padded to a multiple of 128 with zero
// rows) and K in stages of 64 elements. For tile t, stage s, row r:
//   Q4_0: qs  [t][K/32][128][16 B] (ggml nibble order kept), d [t][K/32][128] f16
//   Q8_0: qs  [t][K/32][128][32 B],                          d [t][K/32][128] f16
//   Q4_K: qs  [t][K/64][128][32 B] (the 32 qs bytes of the 64-chunk),
//         hdr [t][K/256][128][16 B] (f16 d, f16 dmin, 12 scale bytes, verbatim)
//   F16 : val [t][K/64][128][128 B] (64 halves)
//   Q5_K: qs  [t][K/64][128][48 B]: the chunk's 32 nibble bytes (element l in
//         the low nibble of byte l, element 32+l in the high one), a 32-bit
//         mask of the low half's 5th bits, one of the high half's, f16 d,
//         f16 dmin, then sc, m of the low half and sc, m of the high half
//         (the 6-bit values get_scale_min_k4 decodes, stored as bytes)
//   Q6_K: qs  [t][K/64][128][64 B]: 32 nibble bytes (low 4 bits of element e
//         in byte e%32, nibble e/32), 16 bytes of high 2-bit pairs (element e
//         at bits 2*(e%4) of byte e/4), 4 int8 sub-scales (16 elements each),
//         f16 d, 10 bytes of padding
//   F16X2: val [t][K/64][128][256 B]: 64 halves hi = f16(w), then 64 halves
//         lo = f16(w - hi) (dense f32 / bf16 weights at about fp32 precision)
// so that one stage of one tile is a few contiguous, 16-byte-aligned runs
// (one bulk copy each) and a warp's 32 rows read 512+ contiguous bytes.
#pragma once
#include "common.cuh"

namespace vkb {

enum WFmt : int { W_Q4_0 = 0, W_Q8_0 = 1, W_Q4_K = 2, W_F16 = 3, W_Q5_K = 4, W_Q6_K = 5, W_F16X2 = 6 };

// Calls f(std::integral_constant<int, FMT>{}) for the runtime format.
template <class F>
inline void with_fmt(int fmt, F&& f) {
    switch (fmt) {
        case W_Q4_0: f(std::integral_constant<int, W_Q4_0>{}); break;
        case W_Q8_0: f(std::integral_constant<int, W_Q8_0>{}); break;
        case W_Q4_K: f(std::integral_constant<int, W_Q4_K>{}); break;
        case W_F16: f(std::integral_constant<int, W_F16>{}); break;
        case W_Q5_K: f(std::integral_constant<int, W_Q5_K>{}); break;
        case W_Q6_K: f(std::integral_constant<int, W_Q6_K>{}); break;
        case W_F16X2: f(std::integral_constant<int, W_F16X2>{}); break;
        default: fail(VKB_ERROR_OTHER, "weight: unknown device format " + std::to_string(fmt));
    }
}

constexpr int TILE_N = 128;   // weight rows per tile (= tcgen05 MMA M)
constexpr int STAGE_K = 64;   // K elements per pipeline stage

// Bytes per row per stage in the quant plane and in the scale/header plane.
__host__ __device__ constexpr int qs_bytes_per_row_stage(int fmt) {
    return fmt == W_Q4_0 ? 32 : fmt == W_Q8_0 ? 64 : fmt == W_Q4_K ? 32 : fmt == W_Q5_K ? 48 : fmt == W_Q6_K ? 64
           : fmt == W_F16X2 ? 256 : 128;
}


}  // namespace vkb

struct vkb_weight {
    vkb_context* ctx = nullptr;
    uint32_t tag = 0;
    int fmt = 0;
    int64_t n = 0, k = 0, n_pad = 0;
    vkb::DevBuf qs;  // quant / value plane
    vkb::DevBuf sc;  // scale (Q4_0, Q8_0) or header (Q4_K) plane; empty for F16
};

namespace vkb {

// Pointers of one (tile, stage) inside the planes.
struct StagePtrs {
    const uint8_t* qs;  // start of the stage's quant run (all 128 rows)
    const uint8_t* sc;  // start of the stage's scale/header run (all 128 rows)
};

__host__ __device__ __forceinline__ StagePtrs stage_ptrs(int fmt, const uint8_t* qs, const uint8_t* sc, int64_t K,
                                                         int64_t tile, int64_t stage) {
    StagePtrs p;
    if (fmt == W_Q4_0 || fmt == W_Q8_0) {
        int64_t KB = K / 32;
        int bpb = fmt == W_Q4_0 ? 16 : 32;
        p.qs = qs + ((tile * KB + 2 * stage) * TILE_N) * bpb;
        p.sc = sc + ((tile * KB + 2 * stage) * TILE_N) * 2;
    } else if (fmt == W_Q4_K) {
        int64_t KC = K / 64, KSB = K / 256;
        p.qs = qs + ((tile * KC + stage) * TILE_N) * 32;
        p.sc = sc + ((tile * KSB + stage / 4) * TILE_N) * 16;
    } else {
        int64_t KC = K / 64;
        p.qs = qs + ((tile * KC + stage) * TILE_N) * qs_bytes_per_row_stage(fmt);
        p.sc = nullptr;
    }
    return p;
}
// Bytes of one stage's runs for all 128 rows.
__host__ __device__ constexpr int stage_qs_bytes(int fmt) { return qs_bytes_per_row_stage(fmt) * TILE_N; }
__host__ __device__ constexpr int stage_sc_bytes(int fmt) {
    return fmt == W_Q4_0 || fmt == W_Q8_0 ? 2 * 2 * TILE_N : fmt == W_Q4_K ? 16 * TILE_N : 0;
}

// Dequantizes the 64 weights of row r of one stage into fp32 (values equal to
// the reference dequantizers: (q-8)*d, q*d, d*sc*q - dmin*m, all exact or
// rounded once exactly as in crates/vokra-core/src/gguf/quant/q4_k.rs:58-66).
// `qs`/`sc` point at the stage's runs (global or shared memory); `stage` is
// needed for Q4_K to pick the 64-chunk's sub-scales.
template <int FMT>
__device__ __forceinline__ void dequant_row_stage(const uint8_t* qs, const uint8_t* sc, int r, int stage,
                                                  float (&w)[64]) {
    if constexpr (FMT == W_Q4_0) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            uint4 q = *reinterpret_cast<const uint4*>(qs + j * (16 * TILE_N) + r * 16);
            float d = h2f(*reinterpret_cast<const uint16_t*>(sc + j * (2 * TILE_N) + r * 2));
            uint32_t qq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int b = 0; b < 16; ++b) {
                uint32_t byte = (qq[b >> 2] >> (8 * (b & 3))) & 0xffu;
                w[32 * j + b] = (float)((int)(byte & 0xfu) - 8) * d;
                w[32 * j + b + 16] = (float)((int)(byte >> 4) - 8) * d;
            }
        }
    } else if constexpr (FMT == W_Q8_0) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint4* p = reinterpret_cast<const uint4*>(qs + j * (32 * TILE_N) + r * 32);
            uint4 q0 = p[0], q1 = p[1];
            float d = h2f(*reinterpret_cast<const uint16_t*>(sc + j * (2 * TILE_N) + r * 2));
            uint32_t qq[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
            for (int b = 0; b < 32; ++b) {
                int8_t v = (int8_t)((qq[b >> 2] >> (8 * (b & 3))) & 0xffu);
                w[32 * j + b] = (float)v * d;
            }
        }
    } else if constexpr (FMT == W_Q4_K) {
        const uint4* p = reinterpret_cast<const uint4*>(qs + r * 32);
        uint4 q0 = p[0], q1 = p[1];
        uint4 h = *reinterpret_cast<const uint4*>(sc + r * 16);
        uint32_t hh[4] = {h.x, h.y, h.z, h.w};
        const uint8_t* hb = reinterpret_cast<const uint8_t*>(hh);
        float d = h2f((uint16_t)(hh[0] & 0xffffu));
        float dmin = h2f((uint16_t)(hh[0] >> 16));
        const uint8_t* s = hb + 4;
        int c = stage & 3;
        int j0 = 2 * c, j1 = 2 * c + 1;
        uint32_t sc0, m0, sc1, m1;
        // get_scale_min_k4 (crates/vokra-core/src/gguf/quant/mod.rs:140)
        if (j0 < 4) { sc0 = s[j0] & 63; m0 = s[j0 + 4] & 63; }
        else { sc0 = (s[j0 + 4] & 0xf) | ((s[j0 - 4] >> 6) << 4); m0 = (s[j0 + 4] >> 4) | ((s[j0] >> 6) << 4); }
        if (j1 < 4) { sc1 = s[j1] & 63; m1 = s[j1 + 4] & 63; }
        else { sc1 = (s[j1 + 4] & 0xf) | ((s[j1 - 4] >> 6) << 4); m1 = (s[j1 + 4] >> 4) | ((s[j1] >> 6) << 4); }
        float d1 = d * (float)sc0, mm1 = dmin * (float)m0;
        float d2 = d * (float)sc1, mm2 = dmin * (float)m1;
        uint32_t qq[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int l = 0; l < 32; ++l) {
            uint32_t byte = (qq[l >> 2] >> (8 * (l & 3))) & 0xffu;
            // two roundings, as the reference (no contraction into an FMA)
            w[l] = __fsub_rn(__fmul_rn(d1, (float)(byte & 0xfu)), mm1);
            w[32 + l] = __fsub_rn(__fmul_rn(d2, (float)(byte >> 4)), mm2);
        }
    } else if constexpr (FMT == W_Q5_K) {
        // q5_k.rs:36-80: y = (d*sc)*q - dmin*m, q = nibble + 16*(5th bit)
        const uint4* p = reinterpret_cast<const uint4*>(qs + r * 48);
        const uint4 q0 = p[0], q1 = p[1], t = p[2];
        const float d = h2f((uint16_t)(t.z & 0xffffu)), dmin = h2f((uint16_t)(t.z >> 16));
        const float d1 = __fmul_rn(d, (float)(t.w & 0xffu)), m1 = __fmul_rn(dmin, (float)((t.w >> 8) & 0xffu));
        const float d2 = __fmul_rn(d, (float)((t.w >> 16) & 0xffu)), m2 = __fmul_rn(dmin, (float)(t.w >> 24));
        const uint32_t qq[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int l = 0; l < 32; ++l) {
            const uint32_t byte = (qq[l >> 2] >> (8 * (l & 3))) & 0xffu;
            const uint32_t lo = (byte & 0xfu) | (((t.x >> l) & 1u) << 4), hi = (byte >> 4) | (((t.y >> l) & 1u) << 4);
            w[l] = __fsub_rn(__fmul_rn(d1, (float)lo), m1);
            w[32 + l] = __fsub_rn(__fmul_rn(d2, (float)hi), m2);
        }
    } else if constexpr (FMT == W_Q6_K) {
        // q6_k.rs:36-70: y = (d*sc)*(q - 32), q = low nibble | high pair << 4
        const uint4* p = reinterpret_cast<const uint4*>(qs + r * 64);
        const uint4 q0 = p[0], q1 = p[1], h = p[2], t = p[3];
        const float d = h2f((uint16_t)(t.y & 0xffffu));
        const uint32_t qq[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        const uint32_t hh[4] = {h.x, h.y, h.z, h.w};
        float ds[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) ds[j] = __fmul_rn(d, (float)(int8_t)((t.x >> (8 * j)) & 0xffu));
#pragma unroll
        for (int e = 0; e < 64; ++e) {
            const uint32_t byte = (qq[(e & 31) >> 2] >> (8 * (e & 3))) & 0xffu;
            const uint32_t low4 = e < 32 ? (byte & 0xfu) : (byte >> 4);
            const uint32_t hi2 = (hh[e >> 4] >> (2 * (e & 15))) & 3u;
            w[e] = __fmul_rn(ds[e >> 4], (float)((int)(low4 | (hi2 << 4)) - 32));
        }
    } else if constexpr (FMT == W_F16X2) {
        const uint4* p = reinterpret_cast<const uint4*>(qs + r * 256);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint4 v = p[i], u = p[8 + i];
            const uint32_t vv[4] = {v.x, v.y, v.z, v.w}, uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&vv[e]));
                const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&uu[e]));
                w[8 * i + 2 * e] = a.x + b.x;
                w[8 * i + 2 * e + 1] = a.y + b.y;
            }
        }
    } else {
        const uint4* p = reinterpret_cast<const uint4*>(qs + r * 128);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            uint4 v = p[i];
            uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                __half2 h2 = *reinterpret_cast<__half2*>(&vv[e]);
                float2 f = __half22float2(h2);
                w[8 * i + 2 * e] = f.x;
                w[8 * i + 2 * e + 1] = f.y;
            }
        }
    }
}


__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// hi = f16(q*d) and lo = f16(q*d - hi) for a pair of small integers given as
// the f16 bit patterns 0x6400|byte (= 1024 + byte, exact) minus `bias`. Both
// are exact roundings: q*d has at most 19 significant bits (|q| <= 255, d f16),
// so the residual q*d - hi fits an f16 and the fused multiply-add returns it.
template <bool SPLIT>
__device__ __forceinline__ void q_pair_to_f16(uint32_t biased_bits, __half2 bias, __half2 d2, uint32_t& hi,
                                              uint32_t& lo) {
    __half2 q = __hsub2(u2h(biased_bits), bias);
    __half2 h = __hmul2(q, d2);
    hi = h2u(h);
    if (SPLIT) lo = h2u(__hfma2(q, d2, __hneg2(h)));
}

// Dequantizes the 64 weights of row r of one stage straight to f16 pairs
// (hi[j] holds elements 2j, 2j+1; lo the residuals when SPLIT) without any
// int/float conversion instruction. Values equal f16-rounding of the exact
// reference dequantization (q-8)*d, q*d and d*sc*q - dmin*m.
template <int FMT, bool SPLIT>
__device__ __forceinline__ void dequant_row_stage_h(const uint8_t* qs, const uint8_t* sc, int r, int stage,
                                                    uint32_t (&hi)[32], uint32_t (&lo)[32]) {
    if constexpr (FMT == W_Q4_0) {
        const __half2 bias = __float2half2_rn(1032.0f);  // 1024 + 8
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            uint4 q = *reinterpret_cast<const uint4*>(qs + j * (16 * TILE_N) + r * 16);
            __half d = __ushort_as_half(*reinterpret_cast<const uint16_t*>(sc + j * (2 * TILE_N) + r * 2));
            __half2 d2 = __half2half2(d);
            uint32_t wds[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
                uint32_t lo4 = wds[wi] & 0x0F0F0F0Fu, hi4 = (wds[wi] >> 4) & 0x0F0F0F0Fu;
                // low nibbles: elements 4wi..4wi+3 ; high nibbles: 16 + 4wi ..
                q_pair_to_f16<SPLIT>(__byte_perm(lo4, 0x64u, 0x4140), bias, d2, hi[16 * j + 2 * wi], lo[16 * j + 2 * wi]);
                q_pair_to_f16<SPLIT>(__byte_perm(lo4, 0x64u, 0x4342), bias, d2, hi[16 * j + 2 * wi + 1],
                                     lo[16 * j + 2 * wi + 1]);
                q_pair_to_f16<SPLIT>(__byte_perm(hi4, 0x64u, 0x4140), bias, d2, hi[16 * j + 8 + 2 * wi],
                                     lo[16 * j + 8 + 2 * wi]);
                q_pair_to_f16<SPLIT>(__byte_perm(hi4, 0x64u, 0x4342), bias, d2, hi[16 * j + 8 + 2 * wi + 1],
                                     lo[16 * j + 8 + 2 * wi + 1]);
            }
        }
    } else if constexpr (FMT == W_Q8_0) {
        const __half2 bias = __float2half2_rn(1152.0f);  // 1024 + 128
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint4* p = reinterpret_cast<const uint4*>(qs + j * (32 * TILE_N) + r * 32);
            uint4 q0 = p[0], q1 = p[1];
            __half d = __ushort_as_half(*reinterpret_cast<const uint16_t*>(sc + j * (2 * TILE_N) + r * 2));
            __half2 d2 = __half2half2(d);
            uint32_t wds[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
            for (int wi = 0; wi < 8; ++wi) {
                uint32_t u = wds[wi] ^ 0x80808080u;  // int8 -> byte + 128
                q_pair_to_f16<SPLIT>(__byte_perm(u, 0x64u, 0x4140), bias, d2, hi[16 * j + 2 * wi], lo[16 * j + 2 * wi]);
                q_pair_to_f16<SPLIT>(__byte_perm(u, 0x64u, 0x4342), bias, d2, hi[16 * j + 2 * wi + 1],
                                     lo[16 * j + 2 * wi + 1]);
            }
        }
    } else if constexpr (FMT == W_F16X2) {
        const uint4* p = reinterpret_cast<const uint4*>(qs + r * 256);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            uint4 v = p[i];
            hi[4 * i] = v.x; hi[4 * i + 1] = v.y; hi[4 * i + 2] = v.z; hi[4 * i + 3] = v.w;
            if (SPLIT) {
                uint4 u = p[8 + i];
                lo[4 * i] = u.x; lo[4 * i + 1] = u.y; lo[4 * i + 2] = u.z; lo[4 * i + 3] = u.w;
            }
        }
    } else if constexpr (FMT == W_F16) {
        const uint4* p = reinterpret_cast<const uint4*>(qs + r * 128);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            uint4 v = p[i];
            hi[4 * i] = v.x; hi[4 * i + 1] = v.y; hi[4 * i + 2] = v.z; hi[4 * i + 3] = v.w;
            if (SPLIT) { lo[4 * i] = 0; lo[4 * i + 1] = 0; lo[4 * i + 2] = 0; lo[4 * i + 3] = 0; }
        }
    } else {
        float w[64];
        dequant_row_stage<FMT>(qs, sc, r, stage, w);
#pragma unroll
        for (int q = 0; q < 32; ++q) {
            __half2 h = __floats2half2_rn(w[2 * q], w[2 * q + 1]);
            hi[q] = h2u(h);
            if (SPLIT) {
                float2 hf = __half22float2(h);
                lo[q] = h2u(__floats2half2_rn(w[2 * q] - hf.x, w[2 * q + 1] - hf.y));
            }
        }
    }
}

}  // namespace vkb
