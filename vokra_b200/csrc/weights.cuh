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
// so that one stage of one tile is a few contiguous, 16-byte-aligned runs
// (one bulk copy each) and a warp's 32 rows read 512+ contiguous bytes.
#pragma once
#include "common.cuh"

namespace vkb {

enum WFmt : int { W_Q4_0 = 0, W_Q8_0 = 1, W_Q4_K = 2, W_F16 = 3 };

constexpr int TILE_N = 128;   // weight rows per tile (= tcgen05 MMA M)
constexpr int STAGE_K = 64;   // K elements per pipeline stage

// Bytes per row per stage in the quant plane and in the scale/header plane.
__host__ __device__ constexpr int qs_bytes_per_row_stage(int fmt) {
    return fmt == W_Q4_0 ? 32 : fmt == W_Q8_0 ? 64 : fmt == W_Q4_K ? 32 : 128;
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
        p.qs = qs + ((tile * KC + stage) * TILE_N) * 128;
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
            w[l] = d1 * (float)(byte & 0xfu) - mm1;
            w[32 + l] = d2 * (float)(byte >> 4) - mm2;
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
