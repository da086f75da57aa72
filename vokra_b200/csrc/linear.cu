// linear.cu — the quantized Linear of the Whisper hot path: weight upload and
// repack, the small-m streaming GEMV, the tcgen05/TMEM GEMM, split-K reduce,
// and the C ABI entry points vkb_weight_upload / vkb_linear / vkb_gemm_q_f32
// (the B200 arm of Compute::gemm_q_f32, crates/vokra-models/src/compute.rs:943).
#include "common.cuh"
#include "weights.cuh"
#include "tc_ptx.cuh"
#include "linear.cuh"

#include <cudaTypedefs.h>
#include <mutex>
#include <memory>
#include <algorithm>

namespace vkb {

// ---------------------------------------------------------------------------
// Host repack of GGUF block bytes [n][k] into the tile layout of weights.cuh.
// ---------------------------------------------------------------------------
static void repack_host(int fmt, const uint8_t* src, int64_t n, int64_t k, int64_t n_pad, std::vector<uint8_t>& qs,
                        std::vector<uint8_t>& sc, uint32_t tag) {
    int64_t T = n_pad / TILE_N;
    if (fmt == W_Q4_0 || fmt == W_Q8_0) {
        int bpb = fmt == W_Q4_0 ? 16 : 32, blk = fmt == W_Q4_0 ? 18 : 34;
        int64_t KB = k / 32;
        qs.assign((size_t)T * KB * TILE_N * bpb, 0);
        sc.assign((size_t)T * KB * TILE_N * 2, 0);
        for (int64_t row = 0; row < n; ++row) {
            int64_t t = row / TILE_N, r = row % TILE_N;
            const uint8_t* rb = src + (size_t)row * KB * blk;
            for (int64_t b = 0; b < KB; ++b) {
                size_t o = (size_t)((t * KB + b) * TILE_N + r);
                memcpy(&sc[o * 2], rb + b * blk, 2);
                memcpy(&qs[o * bpb], rb + b * blk + 2, bpb);
            }
        }
    } else if (fmt == W_Q4_K) {
        int64_t KC = k / 64, KSB = k / 256;
        qs.assign((size_t)T * KC * TILE_N * 32, 0);
        sc.assign((size_t)T * KSB * TILE_N * 16, 0);
        for (int64_t row = 0; row < n; ++row) {
            int64_t t = row / TILE_N, r = row % TILE_N;
            const uint8_t* rb = src + (size_t)row * KSB * 144;
            for (int64_t sb = 0; sb < KSB; ++sb) {
                const uint8_t* blkp = rb + sb * 144;
                memcpy(&sc[(size_t)((t * KSB + sb) * TILE_N + r) * 16], blkp, 16);
                for (int c = 0; c < 4; ++c)
                    memcpy(&qs[(size_t)((t * KC + sb * 4 + c) * TILE_N + r) * 32], blkp + 16 + 32 * c, 32);
            }
        }
    } else if (fmt == W_Q5_K) {
        // per 64-chunk c of a 176-byte block (q5_k.rs): qs nibbles, the qh bits
        // 2c / 2c+1 as two masks, d, dmin and the chunk's decoded sub-scales
        const int64_t KC = k / 64, KSB = k / 256;
        qs.assign((size_t)T * KC * TILE_N * 48, 0);
        for (int64_t row = 0; row < n; ++row) {
            const int64_t t = row / TILE_N, r = row % TILE_N;
            for (int64_t sb = 0; sb < KSB; ++sb) {
                const uint8_t* b = src + (size_t)(row * KSB + sb) * 176;
                for (int c = 0; c < 4; ++c) {
                    uint8_t* dst = &qs[(size_t)((t * KC + sb * 4 + c) * TILE_N + r) * 48];
                    memcpy(dst, b + 48 + 32 * c, 32);
                    uint32_t mlo = 0, mhi = 0;
                    for (int l = 0; l < 32; ++l) {
                        mlo |= (uint32_t)((b[16 + l] >> (2 * c)) & 1) << l;
                        mhi |= (uint32_t)((b[16 + l] >> (2 * c + 1)) & 1) << l;
                    }
                    memcpy(dst + 32, &mlo, 4);
                    memcpy(dst + 36, &mhi, 4);
                    memcpy(dst + 40, b, 4);  // d, dmin
                    const uint8_t* sc6 = b + 4;
                    for (int h = 0; h < 2; ++h) {
                        const int j = 2 * c + h;  // get_scale_min_k4 (gguf/quant/mod.rs:140)
                        uint8_t scv, mv;
                        if (j < 4) { scv = sc6[j] & 63; mv = sc6[j + 4] & 63; }
                        else { scv = (sc6[j + 4] & 0xf) | ((sc6[j - 4] >> 6) << 4); mv = (sc6[j + 4] >> 4) | ((sc6[j] >> 6) << 4); }
                        dst[44 + 2 * h] = scv;
                        dst[45 + 2 * h] = mv;
                    }
                }
            }
        }
    } else if (fmt == W_Q6_K) {
        // per 64-chunk c of a 210-byte block (q6_k.rs): chunk element e is
        // n = 64c + e at (half, quarter, l) = (n/128, n%128/32, n%32)
        const int64_t KC = k / 64, KSB = k / 256;
        qs.assign((size_t)T * KC * TILE_N * 64, 0);
        for (int64_t row = 0; row < n; ++row) {
            const int64_t t = row / TILE_N, r = row % TILE_N;
            for (int64_t sb = 0; sb < KSB; ++sb) {
                const uint8_t* b = src + (size_t)(row * KSB + sb) * 210;
                for (int c = 0; c < 4; ++c) {
                    uint8_t* dst = &qs[(size_t)((t * KC + sb * 4 + c) * TILE_N + r) * 64];
                    const int half = c / 2;
                    for (int e = 0; e < 64; ++e) {
                        const int o = 64 * (c % 2) + e, quarter = o / 32, l = o % 32;
                        const uint8_t low4 = (b[64 * half + (quarter & 1) * 32 + l] >> (4 * (quarter >> 1))) & 0xf;
                        const uint8_t hi2 = (b[128 + 32 * half + l] >> (2 * quarter)) & 3;
                        dst[e % 32] |= (uint8_t)(low4 << (4 * (e / 32)));
                        dst[32 + e / 4] |= (uint8_t)(hi2 << (2 * (e % 4)));
                    }
                    // sub-scales of the chunk's 16-element groups: is = l/16 + 2*quarter
                    for (int j = 0; j < 4; ++j) {
                        const int o = 64 * (c % 2) + 16 * j, quarter = o / 32, l = o % 32;
                        dst[48 + j] = b[192 + 8 * half + l / 16 + 2 * quarter];
                    }
                    memcpy(dst + 52, b + 208, 2);
                }
            }
        }
    } else {
        // dense: F16 kept as one plane; F32 / BF16 as hi = f16(w), lo = f16(w - hi)
        const bool two = fmt == W_F16X2;
        const int rb = two ? 256 : 128;
        int64_t KC = k / 64;
        qs.assign((size_t)T * KC * TILE_N * rb, 0);
        for (int64_t row = 0; row < n; ++row) {
            int64_t t = row / TILE_N, r = row % TILE_N;
            for (int64_t c = 0; c < KC; ++c) {
                uint16_t* dst = reinterpret_cast<uint16_t*>(&qs[(size_t)((t * KC + c) * TILE_N + r) * rb]);
                for (int e = 0; e < 64; ++e) {
                    int64_t idx = row * k + c * 64 + e;
                    if (tag == VKB_GGML_F16) {
                        memcpy(&dst[e], src + idx * 2, 2);
                        continue;
                    }
                    float f;
                    if (tag == VKB_GGML_BF16) {
                        uint32_t b = (uint32_t)(src[idx * 2] | (src[idx * 2 + 1] << 8)) << 16;
                        memcpy(&f, &b, 4);
                    } else {
                        memcpy(&f, src + idx * 4, 4);
                    }
                    const uint16_t h = f32_to_f16_bits(f);
                    dst[e] = h;
                    if (two) dst[64 + e] = f32_to_f16_bits(f - f16_bits_to_f32(h));
                }
            }
        }
    }
}

static int64_t payload_bytes(uint32_t tag, int64_t n, int64_t k) {
    int64_t e = n * k;
    switch (tag) {
        case VKB_GGML_F32: return e * 4;
        case VKB_GGML_F16: case VKB_GGML_BF16: return e * 2;
        case VKB_GGML_Q4_0: return e / 32 * 18;
        case VKB_GGML_Q8_0: return e / 32 * 34;
        case VKB_GGML_Q4_K: return e / 256 * 144;
        case VKB_GGML_Q5_K: return e / 256 * 176;
        case VKB_GGML_Q6_K: return e / 256 * 210;
        default: return -1;
    }
}

vkb_weight* upload_weight(vkb_context* ctx, uint32_t tag, int64_t n, int64_t k, const void* bytes, size_t len) {
    if (!ctx) fail(VKB_ERROR_INVALID_ARGUMENT, "weight_upload: null context");
    if (!bytes) fail(VKB_ERROR_INVALID_ARGUMENT, "weight_upload: null bytes");
    if (n <= 0 || k <= 0) fail(VKB_ERROR_INVALID_ARGUMENT, "weight_upload: n and k must be positive");
    int fmt;
    switch (tag) {
        case VKB_GGML_Q4_0: fmt = W_Q4_0; break;
        case VKB_GGML_Q8_0: fmt = W_Q8_0; break;
        case VKB_GGML_Q4_K: fmt = W_Q4_K; break;
        case VKB_GGML_Q5_K: fmt = W_Q5_K; break;
        case VKB_GGML_Q6_K: fmt = W_Q6_K; break;
        case VKB_GGML_F16: fmt = W_F16; break;
        case VKB_GGML_F32: case VKB_GGML_BF16: fmt = W_F16X2; break;
        default:
            fail(VKB_ERROR_UNSUPPORTED_OP, "weight_upload: ggml type " + std::to_string(tag) +
                                               " has no B200 kernel (supported: Q4_0, Q8_0, Q4_K, Q5_K, Q6_K, F16, "
                                               "BF16, F32)");
    }
    int64_t kmul = (fmt == W_Q4_K || fmt == W_Q5_K || fmt == W_Q6_K) ? 256 : 64;
    if (k % kmul)
        fail(VKB_ERROR_UNSUPPORTED_OP, "weight_upload: k=" + std::to_string(k) + " must be a multiple of " +
                                           std::to_string(kmul) + " for this dtype");
    int64_t want = payload_bytes(tag, n, k);
    if ((int64_t)len != want)
        fail(VKB_ERROR_INVALID_ARGUMENT, "weight_upload: payload is " + std::to_string(len) + " bytes, want " +
                                             std::to_string(want));
    auto* w = new vkb_weight();
    try {
        w->ctx = ctx;
        w->tag = tag;
        w->fmt = fmt;
        w->n = n;
        w->k = k;
        w->n_pad = (n + TILE_N - 1) / TILE_N * TILE_N;
        std::vector<uint8_t> qs, sc;
        repack_host(fmt, (const uint8_t*)bytes, n, k, w->n_pad, qs, sc, tag);
        VKB_CUDA(cudaSetDevice(ctx->device));
        w->qs.alloc(qs.size());
        VKB_CUDA(cudaMemcpy(w->qs.p, qs.data(), qs.size(), cudaMemcpyHostToDevice));
        if (!sc.empty()) {
            w->sc.alloc(sc.size());
            VKB_CUDA(cudaMemcpy(w->sc.p, sc.data(), sc.size(), cudaMemcpyHostToDevice));
        }
    } catch (...) {
        delete w;
        throw;
    }
    return w;
}

// ---------------------------------------------------------------------------
// Epilogue shared by every Linear kernel.
// ---------------------------------------------------------------------------
struct Epi {
    const float* bias;
    const float* residual;
    void* out;
    int out_fmt;       // VKB_DT_F32, VKB_DT_F16 or VKB_DT_F16X2 (hi plane, then lo plane)
    int kind;
    float scale;
    int64_t ldo;       // = n
    int64_t n_scaled;  // EPI_SCALE scales columns [0, n_scaled) only
    int64_t col_block; // > 0: column block c of width col_block is written as its own [rows][col_block] plane
    int64_t out_rows;  // rows of each plane (col_block layout)
    const int32_t* row_map;  // optional: row m lands in row_map[m / row_group] * row_group + m % row_group
    int row_group;
    int64_t plane;     // elements per plane of an F16X2 output
};

// Destination row of token m under the row-group map (32-bit division: token
// counts stay far below 2^31).
__device__ __forceinline__ int64_t epi_row(const Epi& e, int64_t m) {
    if (!e.row_map) return m;
    const unsigned g = (unsigned)m / (unsigned)e.row_group;
    return (int64_t)e.row_map[g] * e.row_group + ((unsigned)m - g * (unsigned)e.row_group);
}

__device__ __forceinline__ void epi_store(const Epi& e, int64_t m, int64_t n, float acc, float bias_n) {
    float v = acc + bias_n;
    int64_t mr = epi_row(e, m);
    int64_t idx = e.col_block > 0 ? (n / e.col_block) * (e.out_rows * e.col_block) + mr * e.col_block + n % e.col_block
                                  : mr * e.ldo + n;
    if (e.kind == VKB_EPI_GELU) v = gelu_as_fast(v);
    else if (e.kind == VKB_EPI_SCALE) v = n < e.n_scaled ? v * e.scale : v;
    else if (e.kind == VKB_EPI_RESIDUAL) v = e.residual[idx] + v;
    if (e.out_fmt == VKB_DT_F32) {
        reinterpret_cast<float*>(e.out)[idx] = v;
    } else {
        __half hi = __float2half_rn(v);
        reinterpret_cast<__half*>(e.out)[idx] = hi;
        if (e.out_fmt == VKB_DT_F16X2) reinterpret_cast<__half*>(e.out)[e.plane + idx] = __float2half_rn(v - __half2float(hi));
    }
}

// ---------------------------------------------------------------------------
// Small-m streaming GEMV: one thread per weight row (128 per CTA), the CTA's
// stage range of K, activations broadcast from shared memory, fp32 FMA.
// grid = (n_pad/128 tiles, k splits). With one split the epilogue is applied
// here, else fp32 partials go to ws[split][m][n].
// ---------------------------------------------------------------------------
template <int FMT, int MM>
__global__ void __launch_bounds__(128) gemv_kernel(const uint8_t* __restrict__ qs, const uint8_t* __restrict__ sc,
                                                   int64_t K, int64_t N, int64_t M, const void* __restrict__ a,
                                                   int a_fmt, int stages_per_split, int n_splits, float* ws, Epi e) {
    pdl_entry();
    extern __shared__ float xs[];  // [MM][stages_per_split*64]
    const int tile = blockIdx.x, split = blockIdx.y, r = threadIdx.x;
    const int64_t total_stages = K / STAGE_K;
    const int64_t s0 = (int64_t)split * stages_per_split;
    const int64_t s1 = min(total_stages, s0 + stages_per_split);
    const int ks = (int)((s1 - s0) * STAGE_K);
    // Stage the activations of this K range (rows >= M are zero).
    for (int i = threadIdx.x; i < MM * ks; i += blockDim.x) {
        int m = i / ks, kk = i % ks;
        float v = 0.0f;
        if (m < M) {
            int64_t g = (int64_t)m * K + s0 * STAGE_K + kk;
            if (a_fmt == VKB_DT_F32) {
                v = reinterpret_cast<const float*>(a)[g];
            } else {
                const __half* ah = reinterpret_cast<const __half*>(a);
                v = __half2float(ah[g]);
                if (a_fmt == VKB_DT_F16X2) v += __half2float(ah[M * K + g]);
            }
        }
        xs[m * ks + kk] = v;
    }
    __syncthreads();
    float acc[MM];
#pragma unroll
    for (int m = 0; m < MM; ++m) acc[m] = 0.0f;
    for (int64_t s = s0; s < s1; ++s) {
        StagePtrs p = stage_ptrs(FMT, qs, sc, K, tile, s);
        float w[64];
        dequant_row_stage<FMT>(p.qs, p.sc, r, (int)s, w);
        const float* xb = xs + (s - s0) * STAGE_K;
#pragma unroll
        for (int m = 0; m < MM; ++m) {
            const float4* x4 = reinterpret_cast<const float4*>(xb + m * ks);
            float am = acc[m];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                float4 xv = x4[i];
                am = fmaf(w[4 * i], xv.x, am);
                am = fmaf(w[4 * i + 1], xv.y, am);
                am = fmaf(w[4 * i + 2], xv.z, am);
                am = fmaf(w[4 * i + 3], xv.w, am);
            }
            acc[m] = am;
        }
    }
    const int64_t n = (int64_t)tile * TILE_N + r;
    if (n >= N) return;
    if (n_splits == 1) {
        float b = e.bias ? e.bias[n] : 0.0f;
#pragma unroll
        for (int m = 0; m < MM; ++m)
            if (m < M) epi_store(e, m, n, acc[m], b);
    } else {
#pragma unroll
        for (int m = 0; m < MM; ++m)
            if (m < M) ws[((int64_t)split * M + m) * N + n] = acc[m];
    }
}

// ---------------------------------------------------------------------------
// Small-m streaming GEMV (m <= 8) for Q4_0, Q8_0 and Q4_K: one CTA = one
// 128-row weight tile x one K range of units (32-blocks; 64-chunks for Q4_K);
// thread = row. In the tile layout the CTA's weights are a few contiguous
// runs (quants, scales or super-block headers), so thread 0 requests them
// with bulk copies into shared memory, in two halves on two mbarriers, before
// waiting on the previous kernel (weights are never written by one); the
// threads then stage the activations (f32; hi + lo summed for F16X2) and
// decode from shared memory while the second half lands. The quants enter the
// dot product as exact small-integer floats (packed f32x2 subtract and FMA):
// acc += d * sum(q * x) per block; Q4_K: d1 * sum(q x) - m1 * sum(x) per half
// chunk. Split-K partials go to ws[split][m][n]; the last CTA of a tile to
// arrive (a counter that resets itself) sums them in split order and applies
// the epilogue, so the result does not depend on arrival order and no reduce
// kernel runs. Every mbarrier wait is bounded: on timeout the CTA sets the
// error flag, waits (bounded) for its copies in flight and skips its work.
// ---------------------------------------------------------------------------
template <int FMT>
struct GvUnit {
    static constexpr int K = FMT == W_Q4_K ? 64 : 32;  // K elements per unit
};

// Bytes of one unit for the whole 128-row tile in the quant plane and in the
// scale plane (Q4_K: a 16-byte header per row per super-block of 4 units).
template <int FMT>
struct GvBytes {
    static constexpr int Q = TILE_N * (FMT == W_Q4_0 ? 16 : 32);
    static constexpr int S = FMT == W_Q4_K ? 0 : TILE_N * 2;
    static constexpr int HDR = TILE_N * 16;
};

template <int FMT>
struct GvRaw {
    uint4 q0, q1;  // Q4_0: q0; Q8_0 and Q4_K: q0, q1
    uint4 h;       // Q4_K: the super-block header (d, dmin, 12 scale bytes)
    uint32_t d;    // Q4_0 / Q8_0: f16 scale bits
};

template <int FMT>
__device__ __forceinline__ void gv_read(const uint8_t* q_s, const uint8_t* s_s, int i, int64_t unit, int64_t sb0,
                                        int r, GvRaw<FMT>& o) {
    constexpr int QB = GvBytes<FMT>::Q;
    if constexpr (FMT == W_Q4_0) {
        o.q0 = *reinterpret_cast<const uint4*>(q_s + i * QB + r * 16);
        o.d = *reinterpret_cast<const unsigned short*>(s_s + i * GvBytes<FMT>::S + r * 2);
    } else if constexpr (FMT == W_Q8_0) {
        const uint4* q = reinterpret_cast<const uint4*>(q_s + i * QB + r * 32);
        o.q0 = q[0];
        o.q1 = q[1];
        o.d = *reinterpret_cast<const unsigned short*>(s_s + i * GvBytes<FMT>::S + r * 2);
    } else {
        const uint4* q = reinterpret_cast<const uint4*>(q_s + i * QB + r * 32);
        o.q0 = q[0];
        o.q1 = q[1];
        o.h = *reinterpret_cast<const uint4*>(s_s + (unit / 4 - sb0) * GvBytes<FMT>::HDR + r * 16);
    }
}

// Byte b of w as the float 2^23 + byte (exact).
__device__ __forceinline__ float gv_magic(uint32_t w, int b) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u + b));
}

// 16 quants of four words as 8 exact float pairs q - bias (packed f32x2 subtraction).
__device__ __forceinline__ void gv_pairs(const uint32_t (&w)[4], float bias, float2 (&q)[8]) {
    const float2 c = make_float2(-(8388608.0f + bias), -(8388608.0f + bias));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        q[2 * i] = __fadd2_rn(make_float2(gv_magic(w[i], 0), gv_magic(w[i], 1)), c);
        q[2 * i + 1] = __fadd2_rn(make_float2(gv_magic(w[i], 2), gv_magic(w[i], 3)), c);
    }
}

// acc + q * x over 16 elements (x: 16 consecutive floats in shared memory), as a float2
__device__ __forceinline__ float2 gv_dot16(const float2 (&q)[8], const float* x, float2 acc) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 v = x4[i];
        acc = __ffma2_rn(q[2 * i], make_float2(v.x, v.y), acc);
        acc = __ffma2_rn(q[2 * i + 1], make_float2(v.z, v.w), acc);
    }
    return acc;
}

__device__ __forceinline__ void gv_nibbles(const uint4& v, uint32_t (&lo)[4], uint32_t (&hi)[4]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        lo[i] = w[i] & 0x0F0F0F0Fu;
        hi[i] = (w[i] >> 4) & 0x0F0F0F0Fu;
    }
}

template <int FMT, int MM>
__device__ __forceinline__ void gv_unit(const GvRaw<FMT>& u, int64_t unit, const float* __restrict__ xs, int ks,
                                        const float* __restrict__ xsum, int ns, float (&acc)[MM]) {
    if constexpr (FMT == W_Q4_0 || FMT == W_Q8_0) {
        float2 qa[8], qb[8];  // elements 0..15 and 16..31 of the block
        if constexpr (FMT == W_Q4_0) {
            // ggml order: element j in the low nibble of byte j, j + 16 in the high one
            uint32_t lo[4], hi[4];
            gv_nibbles(u.q0, lo, hi);
            gv_pairs(lo, 8.0f, qa);
            gv_pairs(hi, 8.0f, qb);
        } else {
            const uint32_t a[4] = {u.q0.x ^ 0x80808080u, u.q0.y ^ 0x80808080u, u.q0.z ^ 0x80808080u,
                                   u.q0.w ^ 0x80808080u};
            const uint32_t b[4] = {u.q1.x ^ 0x80808080u, u.q1.y ^ 0x80808080u, u.q1.z ^ 0x80808080u,
                                   u.q1.w ^ 0x80808080u};
            gv_pairs(a, 128.0f, qa);
            gv_pairs(b, 128.0f, qb);
        }
        const float d = __half2float(__ushort_as_half((unsigned short)u.d));
#pragma unroll
        for (int m = 0; m < MM; ++m) {
            float2 sacc = gv_dot16(qa, xs + m * ks, make_float2(0.0f, 0.0f));
            sacc = gv_dot16(qb, xs + m * ks + 16, sacc);
            acc[m] = fmaf(d, sacc.x + sacc.y, acc[m]);
        }
    } else {
        // Q4_K chunk c of its super-block: element l in the low nibble of byte
        // l, 32 + l in the high one; w = d1*q - m1 (low half), d2*q - m2 (high)
        const uint32_t hh[4] = {u.h.x, u.h.y, u.h.z, u.h.w};
        const float d = __half2float(__ushort_as_half((unsigned short)(hh[0] & 0xffffu)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hh[0] >> 16)));
        const int c = (int)(unit & 3), j0 = 2 * c, j1 = 2 * c + 1;
        auto byte6 = [&](int k) { return (hh[1 + (k >> 2)] >> (8 * (k & 3))) & 0xffu; };  // scale byte k
        uint32_t sc0, m0, sc1, m1;  // get_scale_min_k4 (crates/vokra-core/src/gguf/quant/mod.rs:140)
        if (j0 < 4) { sc0 = byte6(j0) & 63; m0 = byte6(j0 + 4) & 63; }
        else { sc0 = (byte6(j0 + 4) & 0xf) | ((byte6(j0 - 4) >> 6) << 4); m0 = (byte6(j0 + 4) >> 4) | ((byte6(j0) >> 6) << 4); }
        if (j1 < 4) { sc1 = byte6(j1) & 63; m1 = byte6(j1 + 4) & 63; }
        else { sc1 = (byte6(j1 + 4) & 0xf) | ((byte6(j1 - 4) >> 6) << 4); m1 = (byte6(j1 + 4) >> 4) | ((byte6(j1) >> 6) << 4); }
        const float d1 = __fmul_rn(d, (float)sc0), mm1 = __fmul_rn(dmin, (float)m0);
        const float d2 = __fmul_rn(d, (float)sc1), mm2 = __fmul_rn(dmin, (float)m1);
        float2 la[8], lb[8], ha[8], hb[8];
        {
            uint32_t l0[4], h0[4], l1[4], h1[4];
            gv_nibbles(u.q0, l0, h0);
            gv_nibbles(u.q1, l1, h1);
            gv_pairs(l0, 0.0f, la);
            gv_pairs(l1, 0.0f, lb);
            gv_pairs(h0, 0.0f, ha);
            gv_pairs(h1, 0.0f, hb);
        }
#pragma unroll
        for (int m = 0; m < MM; ++m) {
            const float* x = xs + m * ks;
            float2 s1 = gv_dot16(la, x, make_float2(0.0f, 0.0f));
            s1 = gv_dot16(lb, x + 16, s1);
            float2 s2 = gv_dot16(ha, x + 32, make_float2(0.0f, 0.0f));
            s2 = gv_dot16(hb, x + 48, s2);
            const float t1 = xsum[m * ns], t2 = xsum[m * ns + 1];
            acc[m] = fmaf(d1, s1.x + s1.y, acc[m]);
            acc[m] = fmaf(-mm1, t1, acc[m]);
            acc[m] = fmaf(d2, s2.x + s2.y, acc[m]);
            acc[m] = fmaf(-mm2, t2, acc[m]);
        }
    }
}

template <int FMT, int MM>
__global__ void __launch_bounds__(128) gemv2_kernel(const uint8_t* __restrict__ qs, const uint8_t* __restrict__ sc,
                                                    int64_t K, int64_t N, int64_t M, const void* __restrict__ a,
                                                    int a_fmt, int units_per_split, int n_splits, float* ws,
                                                    unsigned* ctr, int* err, Epi e) {
    constexpr int UK = GvUnit<FMT>::K;
    constexpr int QB = GvBytes<FMT>::Q, SB = GvBytes<FMT>::S, HB = GvBytes<FMT>::HDR;
    extern __shared__ __align__(128) uint8_t gv_smem[];
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ unsigned last;
    const int tile = blockIdx.x, split = blockIdx.y, r = threadIdx.x;
    const int64_t total = K / UK;
    const int64_t u0 = (int64_t)split * units_per_split;
    const int64_t u1 = min(total, u0 + units_per_split);
    const int nu = (int)(u1 - u0);
    const int ks = units_per_split * UK;
    const int ns = ks / 32;
    // shared memory: quants [ups][QB] | scales [ups][SB] or headers | x [MM][ks] | sums [MM][ns]
    const int64_t sb0 = u0 / 4, n_sb = FMT == W_Q4_K ? (u1 - 1) / 4 - sb0 + 1 : 0;
    uint8_t* q_s = gv_smem;
    uint8_t* s_s = q_s + (size_t)units_per_split * QB;
    const size_t s_bytes = FMT == W_Q4_K ? (size_t)((units_per_split + 6) / 4) * HB : (size_t)units_per_split * SB;
    float* xs = reinterpret_cast<float*>(s_s + s_bytes);
    float* xsum = xs + MM * ks;
    const int h0 = (nu + 1) / 2;  // units in the first half
    pdl_launch();
    if (threadIdx.x == 0) {
        ptx::mbar_init(&bars[0], 1);
        ptx::mbar_init(&bars[1], 1);
        ptx::fence_mbar_init();
        const uint8_t* qsrc = qs + ((int64_t)tile * total + u0) * QB;
        if constexpr (FMT == W_Q4_K) {
            const uint8_t* hsrc = sc + ((int64_t)tile * (K / 256) + sb0) * HB;
            ptx::mbar_expect_tx(&bars[0], (uint32_t)(h0 * QB + n_sb * HB));
            ptx::bulk_load(s_s, hsrc, (uint32_t)(n_sb * HB), &bars[0]);
            if (nu > h0) ptx::mbar_expect_tx(&bars[1], (uint32_t)((nu - h0) * QB));
        } else {
            const uint8_t* ssrc = sc + ((int64_t)tile * total + u0) * SB;
            ptx::mbar_expect_tx(&bars[0], (uint32_t)(h0 * (QB + SB)));
            ptx::bulk_load(s_s, ssrc, (uint32_t)(h0 * SB), &bars[0]);
            if (nu > h0) {
                ptx::mbar_expect_tx(&bars[1], (uint32_t)((nu - h0) * (QB + SB)));
                ptx::bulk_load(s_s + h0 * SB, ssrc + (size_t)h0 * SB, (uint32_t)((nu - h0) * SB), &bars[1]);
            }
        }
        ptx::bulk_load(q_s, qsrc, (uint32_t)(h0 * QB), &bars[0]);
        if (nu > h0)
            ptx::bulk_load(q_s + (size_t)h0 * QB, qsrc + (size_t)h0 * QB, (uint32_t)((nu - h0) * QB), &bars[1]);
    }
    pdl_wait();
    // this K range of the activations (rows >= M are zero)
    const int kspan = nu * UK;
    for (int i = threadIdx.x; i < MM * ks / 4; i += blockDim.x) {
        const int m = i / (ks / 4), kk = 4 * (i % (ks / 4));
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (m < M && kk < kspan) {
            const int64_t g = (int64_t)m * K + u0 * UK + kk;
            if (a_fmt == VKB_DT_F32) {
                v = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a) + g);
            } else {
                const __half* ah = reinterpret_cast<const __half*>(a);
                const float2 p0 = __half22float2(*reinterpret_cast<const __half2*>(ah + g));
                const float2 p1 = __half22float2(*reinterpret_cast<const __half2*>(ah + g + 2));
                v = make_float4(p0.x, p0.y, p1.x, p1.y);
                if (a_fmt == VKB_DT_F16X2) {
                    const float2 l0 = __half22float2(*reinterpret_cast<const __half2*>(ah + M * K + g));
                    const float2 l1 = __half22float2(*reinterpret_cast<const __half2*>(ah + M * K + g + 2));
                    v.x += l0.x; v.y += l0.y; v.z += l1.x; v.w += l1.y;
                }
            }
        }
        *reinterpret_cast<float4*>(xs + m * ks + kk) = v;
    }
    __syncthreads();
    if constexpr (FMT == W_Q4_K) {  // sum of each 32 activations (the min terms)
        for (int i = threadIdx.x; i < MM * ns; i += blockDim.x) {
            const float* x = xs + (i / ns) * ks + (i % ns) * 32;
            float t = 0.0f;
            for (int j = 0; j < 32; ++j) t += x[j];
            xsum[i] = t;
        }
        __syncthreads();
    }
    float acc[MM];
#pragma unroll
    for (int m = 0; m < MM; ++m) acc[m] = 0.0f;
    bool ok = ptx::mbar_wait(&bars[0], 0);
    for (int i = 0; i < nu && ok; ++i) {
        if (i == h0) ok = ptx::mbar_wait(&bars[1], 0);
        if (!ok) break;
        GvRaw<FMT> cur;
        gv_read<FMT>(q_s, s_s, i, u0 + i, sb0, r, cur);
        gv_unit<FMT, MM>(cur, u0 + i, xs + i * UK, ks, xsum + i * (UK / 32), ns, acc);
    }
    if (!ok) {
        if (threadIdx.x == 0) atomicExch(err, 1);
        // let copies still in flight land before the CTA's shared memory goes away
        ptx::mbar_wait(&bars[0], 0);
        if (nu > h0) ptx::mbar_wait(&bars[1], 0);
    }
    const int64_t n = (int64_t)tile * TILE_N + r;
    if (n_splits == 1) {
        if (n < N && ok) {
            const float b = e.bias ? e.bias[n] : 0.0f;
#pragma unroll
            for (int m = 0; m < MM; ++m)
                if (m < M) epi_store(e, m, n, acc[m], b);
        }
        return;
    }
    if (n < N) {
#pragma unroll
        for (int m = 0; m < MM; ++m)
            if (m < M) ws[((int64_t)split * M + m) * N + n] = acc[m];
    }
    // the last CTA of this tile sums the partials in split order
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(ctr + tile, 1u) == (unsigned)(n_splits - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (n < N) {
        const float b = e.bias ? e.bias[n] : 0.0f;
        for (int m = 0; m < (int)M && m < MM; ++m) {
            // loads issued 8 at a time, added in split order
            float t = 0.0f;
            for (int sp0 = 0; sp0 < n_splits; sp0 += 8) {
                float v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    v[j] = sp0 + j < n_splits ? __ldcg(ws + ((int64_t)(sp0 + j) * M + m) * N + n) : 0.0f;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if (sp0 + j < n_splits) t += v[j];
            }
            epi_store(e, m, n, t, b);
        }
    }
    if (threadIdx.x == 0) ctr[tile] = 0;
}

// Sums split-K partials ws[split][m][n] in split order and applies the epilogue.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int n_splits, int64_t M, int64_t N, Epi e) {
    pdl_launch();
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= M * N) return;
    int64_t m, n;
    if (M * N < (int64_t(1) << 31)) {  // 32-bit division where it is exact
        m = (unsigned)i / (unsigned)N;
        n = (unsigned)i - (unsigned)m * (unsigned)N;
    } else {
        m = i / N;
        n = i % N;
    }
    const float bias_n = e.bias ? __ldg(e.bias + n) : 0.0f;  // a model weight: read before the wait
    pdl_wait();
    // partials in split order, up to 8 loads in flight
    float acc = 0.0f;
    for (int s0 = 0; s0 < n_splits; s0 += 8) {
        float t[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) t[u] = s0 + u < n_splits ? __ldcg(ws + (int64_t)(s0 + u) * M * N + i) : 0.0f;
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (s0 + u < n_splits) acc += t[u];
    }
    epi_store(e, m, n, acc, bias_n);
}

// x (f32) -> f16 plane, or hi / lo f16 planes (x = hi + lo to ~2^-22) when split.
__global__ void split_f16_kernel(const float* __restrict__ x, __half* __restrict__ y, int64_t n, int split) {
    pdl_entry();
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float v = x[i];
    __half hi = __float2half_rn(v);
    y[i] = hi;
    if (split) y[n + i] = __float2half_rn(v - __half2float(hi));
}

void run_split_f16(vkb_context* ctx, const float* x, int64_t n, __half* y, bool split) {
    launch_pdl(ctx, split_f16_kernel, (unsigned)((n + 255) / 256), 256, 0, x, y, n, split ? 1 : 0);
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}

// ---------------------------------------------------------------------------
// tcgen05 GEMM: D[n][m] = W[n][:] . X[m][:] with W dequantized into shared
// memory (128 rows x 64 K per stage, f16, 128-byte swizzle) and X staged by
// TMA (BN tokens x 64 K, f16, 128-byte swizzle). The dequantized weight tile
// (the MMA's A operand, 128 rows x 64 K f16) is written straight into tensor
// memory by the dequant warps (tcgen05.st, thread = row = TMEM lane), so the
// MMAs read only B from shared memory. Accumulator in TMEM (128 lanes x BN
// fp32 columns); A tiles in TMEM columns after it (2 stages x planes x 32).
//
// SPLIT = true is the high-precision mode: the weight is dequantized to
// W_hi = f16(w) and W_lo = f16(w - W_hi) and the activation arrives as two f16
// planes X_hi, X_lo (x = X_hi + X_lo, written by the producing kernel); each
// K=16 step issues W_hi.X_hi + W_hi.X_lo + W_lo.X_hi, which reproduces the
// fp32 product to about 2^-21 relative (the W_lo.X_lo term is below that).
//
// Warp roles (64 + 128 * EG threads):
//   warp 0      : producer — TMA for X, bulk copies for the raw weight stage
//   warp 1      : TMEM allocator; lane 0 issues tcgen05.mma and commits
//   warps 2..5  : dequantize raw stage -> A tile(s); then the epilogue
//                 (thread = one weight row = one TMEM lane)
//   warps 6..   : epilogue only (up to 3 more groups of 4 warps), on the same
//                 TMEM lanes as warps 2..5 and their share of the token columns
// Rings: S stages of (X tile(s) + raw weights) in shared memory, AS stages of
// A tiles in tensor memory. A stage's raw weights and its X tiles complete on
// separate mbarriers (w_full, full): weights are never written by a kernel,
// so they are fetched and the first stages dequantized before the wait for
// the previous kernel; after it only the X loads, the MMAs and the epilogue
// remain (the latency a decode-step GEMM is made of).
// Every mbarrier wait is bounded; on timeout the kernel records an error flag
// and returns without hanging.
// ---------------------------------------------------------------------------
template <int FMT, int BN, bool SPLIT>
struct TcCfg {
    // Token tiles up to 64 (the decode step) run two CTAs per SM: half the
    // shared memory, 256 TMEM columns, 2 epilogue groups, so one CTA's setup and
    // epilogue (and the next GEMM's, launched early) overlap another's MMAs.
    static constexpr bool DUAL = BN <= 64;
    static constexpr int MINB = DUAL ? 2 : 1;
    static constexpr int NP = SPLIT ? 2 : 1;                   // operand planes
    static constexpr int B_BYTES = BN * 128;                   // BN rows x 128 B per plane
    static constexpr int RAW_Q = stage_qs_bytes(FMT);
    static constexpr int RAW_S = stage_sc_bytes(FMT);
    static constexpr int RAW_BYTES = ((RAW_Q + RAW_S) + 1023) / 1024 * 1024;
    static constexpr int STAGE_BYTES = NP * B_BYTES + RAW_BYTES;
    static constexpr int BUDGET = (DUAL ? 110 * 1024 : 225 * 1024) - 2048;
    static constexpr int S0 = BUDGET / STAGE_BYTES;
    static constexpr int SMAX = DUAL ? 4 : 6;
    static constexpr int S = S0 > SMAX ? SMAX : S0;
    static constexpr int SMEM = 1024 /*align slack*/ + S * STAGE_BYTES + 1024 /*barriers*/;
    // Stacked split mode (token tiles up to 128): the hi and lo activation
    // tiles, adjacent in shared memory, form ONE B operand of 2*BN rows, so a
    // K=16 step is two MMAs (W_hi and W_lo against [X_hi; X_lo]) instead of
    // three at N=BN; the accumulator holds W.X_hi in columns [0, BN) and W.X_lo
    // in [BN, 2BN), added in the epilogue. Small-N MMAs cost about the same
    // issue time as N=128..256 ones, so this is faster where M is small.
    static constexpr bool STACK = SPLIT && BN <= 128;
    static constexpr int ACC_COLS = STACK ? 2 * BN : (BN < 32 ? 32 : BN);
    static constexpr int A_COL0 = ACC_COLS;                     // first A column
    static constexpr int AS = DUAL ? 2 : 4;                     // A stages in tensor memory
    static constexpr int NEED_COLS = ACC_COLS + AS * NP * 32;
    static constexpr uint32_t TMEM_COLS = NEED_COLS <= 32 ? 32 : NEED_COLS <= 64 ? 64 : NEED_COLS <= 128 ? 128
                                          : NEED_COLS <= 256 ? 256 : 512;
    static_assert(NEED_COLS <= 512, "tensor memory budget");
    static_assert(!DUAL || TMEM_COLS <= 256, "two CTAs per SM share 512 TMEM columns");
    static_assert(S >= 2, "pipeline needs at least two stages");
    // epilogue groups of 4 warps (one per TMEM lane quarter), each taking
    // BN / EG token columns; group 0 is also the dequant group
    static constexpr int EG0 = BN / 16 < 4 ? BN / 16 : 4;
    static constexpr int EG = DUAL && EG0 > 2 ? 2 : EG0;
    static constexpr int THREADS = 64 + 128 * EG;
};

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

template <int FMT, int BN, bool SPLIT>
__global__ void __launch_bounds__(TcCfg<FMT, BN, SPLIT>::THREADS, TcCfg<FMT, BN, SPLIT>::MINB)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap xmap_lo,
                   const uint8_t* __restrict__ qs, const uint8_t* __restrict__ sc, int64_t K, int64_t N, int64_t M,
                   int n_tiles, int m_tiles, int stages_per_split, int n_splits, float* ws, Epi e, int* err,
                   const __grid_constant__ CUtensorMap omap,
                   const __grid_constant__ CUtensorMap omap_lo, const __grid_constant__ CUtensorMap rmap,
                   int tma_epi) {
    using C = TcCfg<FMT, BN, SPLIT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* st_ring = smem;
    uint64_t* bars = reinterpret_cast<uint64_t*>(st_ring + C::S * C::STAGE_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + C::S;
    uint64_t* a_full = bars + 2 * C::S;
    uint64_t* a_empty = a_full + C::AS;
    uint64_t* acc_full = a_empty + C::AS;
    uint64_t* res_full = acc_full + 1;
    uint64_t* w_full = res_full + 1;  // [S] the raw weights of a stage (full[] counts the activations)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(w_full + C::S);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int bid = blockIdx.x;
    const int n_tile = bid % n_tiles;
    bid /= n_tiles;
    const int m_tile = bid % m_tiles;
    const int split = bid / m_tiles;
    const int64_t total_stages = K / STAGE_K;
    const int64_t s0 = (int64_t)split * stages_per_split;
    const int64_t s1 = min(total_stages, s0 + stages_per_split);
    const int nst = (int)(s1 - s0);

    if (threadIdx.x == 0) {
        for (int i = 0; i < C::S; ++i) {
            ptx::mbar_init(&full[i], 1);
            ptx::mbar_init(&empty[i], 1);
            ptx::mbar_init(&w_full[i], 1);
        }
        for (int i = 0; i < C::AS; ++i) {
            ptx::mbar_init(&a_full[i], 128);
            ptx::mbar_init(&a_empty[i], 1);
        }
        ptx::mbar_init(acc_full, 1);
        ptx::mbar_init(res_full, 1);
        ptx::fence_mbar_init();
    }
    if (warp == 1) {
        ptx::tmem_alloc(tmem_slot, C::TMEM_COLS);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;
    // Programmatic dependent launch: the next kernel may be scheduled now; this
    // one waits for the previous kernel only where it reads activations
    // (producer) or writes results (epilogue). Weights are never written by a
    // kernel, so their first stages are fetched before that wait.
    pdl_launch();

    if (warp == 0) {
        if (lane == 0) {
            // weights of the first ring stages, then wait for the previous kernel
            ptx::prefetch_tmap(&xmap);
            if (SPLIT) ptx::prefetch_tmap(&xmap_lo);
            if (tma_epi) ptx::prefetch_tmap(&omap);
            const int pre = nst < C::S ? nst : C::S;
            for (int i = 0; i < pre; ++i) {
                uint8_t* raw_dst = st_ring + i * C::STAGE_BYTES + C::NP * C::B_BYTES;
                StagePtrs p = stage_ptrs(FMT, qs, sc, K, n_tile, s0 + i);
                ptx::mbar_expect_tx(&w_full[i], C::RAW_Q + C::RAW_S);
                ptx::bulk_load(raw_dst, p.qs, C::RAW_Q, &w_full[i]);
                if (C::RAW_S) ptx::bulk_load(raw_dst + C::RAW_Q, p.sc, C::RAW_S, &w_full[i]);
            }
            pdl_wait();
            for (int i = 0; i < nst && ok; ++i) {
                int s = i % C::S;
                uint8_t* b_dst = st_ring + s * C::STAGE_BYTES;
                int64_t stage = s0 + i;
                if (i >= pre) {
                    if (!ptx::mbar_wait(&empty[s], ((i / C::S) & 1) ^ 1)) { ok = false; break; }
                    uint8_t* raw_dst = b_dst + C::NP * C::B_BYTES;
                    StagePtrs p = stage_ptrs(FMT, qs, sc, K, n_tile, stage);
                    ptx::mbar_expect_tx(&w_full[s], C::RAW_Q + C::RAW_S);
                    ptx::bulk_load(raw_dst, p.qs, C::RAW_Q, &w_full[s]);
                    if (C::RAW_S) ptx::bulk_load(raw_dst + C::RAW_Q, p.sc, C::RAW_S, &w_full[s]);
                }
                ptx::mbar_expect_tx(&full[s], C::NP * C::B_BYTES);
                ptx::tma_load_2d(b_dst, &xmap, &full[s], (int32_t)(stage * STAGE_K), m_tile * BN);
                if (SPLIT)
                    ptx::tma_load_2d(b_dst + C::B_BYTES, &xmap_lo, &full[s], (int32_t)(stage * STAGE_K), m_tile * BN);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = ptx::idesc_f16_f32(TILE_N, C::STACK ? 2 * BN : BN);
            for (int i = 0; i < nst && ok; ++i) {
                int s = i % C::S, a = i % C::AS;
                if (!ptx::mbar_wait(&full[s], (i / C::S) & 1)) { ok = false; break; }
                if (!ptx::mbar_wait(&a_full[a], (i / C::AS) & 1)) { ok = false; break; }
                ptx::tc_fence_after();
                const uint32_t a_t = tmem + C::A_COL0 + a * C::NP * 32;
                uint32_t b_addr = ptx::smem_u32(st_ring + s * C::STAGE_BYTES);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    uint64_t bd = ptx::sdesc_sw128(b_addr + kk * 32);
                    ptx::mma_f16_ts(tmem, a_t + kk * 8, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
                    if (C::STACK) {
                        ptx::mma_f16_ts(tmem, a_t + 32 + kk * 8, bd, idesc, 1u);
                    } else if (SPLIT) {
                        uint64_t bd_lo = ptx::sdesc_sw128(b_addr + C::B_BYTES + kk * 32);
                        ptx::mma_f16_ts(tmem, a_t + kk * 8, bd_lo, idesc, 1u);
                        ptx::mma_f16_ts(tmem, a_t + 32 + kk * 8, bd, idesc, 1u);
                    }
                }
                ptx::mma_commit(&empty[s]);
                ptx::mma_commit(&a_empty[a]);
            }
            ptx::mma_commit(acc_full);
        }
    } else if (warp < 6) {
        // Dequant warps: row r of the 128-row tile = TMEM lane r.
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        for (int i = 0; i < nst && ok; ++i) {
            int s = i % C::S, a = i % C::AS;
            // only the weights: the first stages dequantize before the previous kernel ends
            if (!ptx::mbar_wait(&w_full[s], (i / C::S) & 1)) { ok = false; break; }
            if (!ptx::mbar_wait(&a_empty[a], ((i / C::AS) & 1) ^ 1)) { ok = false; break; }
            const uint8_t* raw = st_ring + s * C::STAGE_BYTES + C::NP * C::B_BYTES;
            uint32_t hi[32], lo[32];
            dequant_row_stage_h<FMT, SPLIT>(raw, raw + C::RAW_Q, r, (int)(s0 + i), hi, lo);
            ptx::tc_fence_after();
            const uint32_t a_t = tmem + ((uint32_t)(quarter * 32) << 16) + C::A_COL0 + a * C::NP * 32;
            ptx::tmem_st32(a_t, hi);
            if (SPLIT) ptx::tmem_st32(a_t + 32, lo);
            ptx::tmem_st_wait();
            ptx::tc_fence_before();
            ptx::mbar_arrive(&a_full[a]);
        }
    }
    if (warp >= 2) {
        // Epilogue, EG groups of 4 warps: warps w, w + 4, ... read the same TMEM
        // lanes (quarter w % 4, thread = weight row) and split the BN token
        // columns. It runs after the previous kernel (which may still read what
        // it overwrites).
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        constexpr int HALF = BN / C::EG;  // columns per group
        const int cb = ((warp - 2) >> 2) * HALF;
        const int64_t n = (int64_t)n_tile * TILE_N + r;
        const float bias_n = (e.bias && n < N) ? __ldg(e.bias + n) : 0.0f;  // a model weight: before the wait
        pdl_wait();
        const bool go = ok && ptx::mbar_wait(acc_full, 0);
        ptx::tc_fence_after();
        const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
        // 32 accumulator columns per tcgen05.ld (16 for narrow tiles)
        constexpr int CW = HALF >= 32 ? 32 : 16;
        auto load_cols = [&](int c0, uint32_t(&v)[CW]) {
            if constexpr (CW == 32) ptx::tmem_ld32(lane_addr + c0, v);
            else ptx::tmem_ld16(lane_addr + c0, v);
            if (C::STACK) {
                uint32_t v2[CW];
                if constexpr (CW == 32) ptx::tmem_ld32(lane_addr + BN + c0, v2);
                else ptx::tmem_ld16(lane_addr + BN + c0, v2);
                ptx::tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < CW; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(v2[j]));
            } else {
                ptx::tmem_ld_wait();
            }
        };
        if (tma_epi) {
            // Stage the [BN tokens][128 features] tile in the idle ring, then one
            // TMA tensor store per plane writes whole row segments.
            float* sf = reinterpret_cast<float*>(st_ring);
            __half* sh = reinterpret_cast<__half*>(st_ring);
            const bool partial = tma_epi == 2;  // split-K: raw fp32 partial sums, no epilogue op
            bool good = go;
            if (good && !partial && e.kind == VKB_EPI_RESIDUAL) {
                if (threadIdx.x == 64) {
                    ptx::mbar_expect_tx(res_full, BN * TILE_N * 4);
                    ptx::tma_load_2d(st_ring, &rmap, res_full, n_tile * TILE_N, m_tile * BN);
                }
                if (!ptx::mbar_wait(res_full, 0)) good = false;
            }
            if (good) {
#pragma unroll 1
                for (int c0 = cb; c0 < cb + HALF; c0 += CW) {
                    uint32_t v[CW];
                    load_cols(c0, v);
                    if (!partial && e.kind == VKB_EPI_GELU && e.out_fmt == VKB_DT_F16X2) {
                        // the MLP's hidden layer: GELU on pairs of tokens with packed f32x2 math
#pragma unroll
                        for (int j = 0; j < CW; j += 2) {
                            const float2 x = gelu_as_fast2(make_float2(__uint_as_float(v[j]) + bias_n,
                                                                       __uint_as_float(v[j + 1]) + bias_n));
                            const __half h0 = __float2half_rn(x.x), h1 = __float2half_rn(x.y);
                            const int row = c0 + j;
                            sh[row * TILE_N + r] = h0;
                            sh[(row + 1) * TILE_N + r] = h1;
                            sh[BN * TILE_N + row * TILE_N + r] = __float2half_rn(x.x - __half2float(h0));
                            sh[BN * TILE_N + (row + 1) * TILE_N + r] = __float2half_rn(x.y - __half2float(h1));
                        }
                        continue;
                    }
#pragma unroll
                    for (int j = 0; j < CW; ++j) {
                        const int row = c0 + j;
                        if (partial) {
                            sf[row * TILE_N + r] = __uint_as_float(v[j]);
                            continue;
                        }
                        float x = __uint_as_float(v[j]) + bias_n;
                        if (e.kind == VKB_EPI_GELU) x = gelu_as_fast(x);
                        else if (e.kind == VKB_EPI_SCALE) x = n < e.n_scaled ? x * e.scale : x;
                        else if (e.kind == VKB_EPI_RESIDUAL) x += sf[row * TILE_N + r];
                        if (e.out_fmt == VKB_DT_F32) {
                            sf[row * TILE_N + r] = x;
                        } else {
                            __half h = __float2half_rn(x);
                            sh[row * TILE_N + r] = h;
                            if (e.out_fmt == VKB_DT_F16X2) sh[BN * TILE_N + row * TILE_N + r] = __float2half_rn(x - __half2float(h));
                        }
                    }
                }
            }
            ptx::fence_proxy_async_smem();
            // every epilogue thread reaches this barrier; the store needs all of them good
            const bool all_good = !ptx::named_bar_or(1, 128 * C::EG, !good);
            if (!good) ok = false;
            if (threadIdx.x == 64 && all_good && partial) {
                ptx::tma_store_3d(&omap, st_ring, n_tile * TILE_N, m_tile * BN, split);
                ptx::bulk_commit();
                ptx::bulk_wait_read0();
            } else if (threadIdx.x == 64 && all_good) {
                ptx::tma_store_2d(&omap, st_ring, n_tile * TILE_N, m_tile * BN);
                if (e.out_fmt == VKB_DT_F16X2) ptx::tma_store_2d(&omap_lo, sh + BN * TILE_N, n_tile * TILE_N, m_tile * BN);
                ptx::bulk_commit();
                ptx::bulk_wait_read0();
            }
        } else if (go) {
#pragma unroll 1
            for (int c0 = cb; c0 < cb + HALF; c0 += CW) {
                uint32_t v[CW];
                load_cols(c0, v);
                if (n < N) {
#pragma unroll
                    for (int j = 0; j < CW; ++j) {
                        int64_t m = (int64_t)m_tile * BN + c0 + j;
                        if (m < M) {
                            float acc = __uint_as_float(v[j]);
                            if (n_splits == 1) epi_store(e, m, n, acc, bias_n);
                            else ws[((int64_t)split * M + m) * N + n] = acc;
                        }
                    }
                }
            }
        } else {
            ok = false;
        }
    }
    if (!ok && err) atomicExch(err, 1);
    // Reconverge each warp (only one lane of the producer and MMA warps ran its
    // role) before the block barrier: bar.sync requires converged warps.
    __syncwarp();
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// Host dispatch
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    if (!fn) fail(VKB_ERROR_BACKEND_UNAVAILABLE, "cuTensorMapEncodeTiled is unavailable from the driver");
    return fn;
}

// 2-D tensor map over a row-major f16 matrix [rows][cols], box [box_rows][64], 128-byte swizzle.
void make_tmap_f16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows) {
    if (((uintptr_t)base & 15) || (cols * 2) % 16)
        fail(VKB_ERROR_INVALID_ARGUMENT, "activation rows must be 16-byte aligned (k % 8 == 0, aligned base)");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = get_encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(VKB_ERROR_BACKEND_UNAVAILABLE, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
}

// 2-D tensor map over a row-major matrix [rows][cols] of 2- or 4-byte elements,
// box [box_rows][box_cols], no swizzle (the epilogue's staging layout).
void make_tmap_2d(CUtensorMap* map, const void* base, int esz, int64_t rows, int64_t cols, int box_cols, int box_rows) {
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(cols * esz)};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = get_encode_fn()(map, esz == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                                 const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                 CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(VKB_ERROR_BACKEND_UNAVAILABLE, "cuTensorMapEncodeTiled (epilogue) failed: " + std::to_string(r));
}

// 3-D f32 tensor map over [planes][rows][cols], box [1][box_rows][box_cols] (split-K partials).
void make_tmap_3d_f32(CUtensorMap* map, const void* base, int64_t planes, int64_t rows, int64_t cols, int box_cols,
                      int box_rows) {
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)planes};
    cuuint64_t strides[2] = {(cuuint64_t)(cols * 4), (cuuint64_t)(cols * 4 * rows)};
    cuuint32_t box[3] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = get_encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                 CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(VKB_ERROR_BACKEND_UNAVAILABLE, "cuTensorMapEncodeTiled (partials) failed: " + std::to_string(r));
}

static int* device_err_flag(vkb_context* ctx) { return ctx->err_flag.as<int>(); }

// Largest m the streaming GEMVs take (VKB_GEMV_MAX_M overrides, for measurements).
int gemv_max_m() {
    static const int v = [] { const char* e = std::getenv("VKB_GEMV_MAX_M"); return e ? std::atoi(e) : 8; }();
    return v;
}

// Most K splits of one streaming-GEMV tile (the last CTA sums them all).
static int gv2_max_splits() {
    static const int v = [] { const char* e = std::getenv("VKB_GV2_MAX_SPLITS"); return e ? std::atoi(e) : 16; }();
    return v;
}

static bool gemv2_fmt(int fmt) { return fmt == W_Q4_0 || fmt == W_Q8_0 || fmt == W_Q4_K; }

// Shared memory of one gemv2 CTA (see the kernel's layout).
static size_t gemv2_smem(int fmt, int mm, int ups) {
    const int uk = fmt == W_Q4_K ? 64 : 32;
    const size_t qb = (size_t)TILE_N * (fmt == W_Q4_0 ? 16 : 32);
    const size_t sbytes = fmt == W_Q4_K ? (size_t)((ups + 6) / 4) * TILE_N * 16 : (size_t)ups * TILE_N * 2;
    const size_t ks = (size_t)ups * uk;
    return (size_t)ups * qb + sbytes + (size_t)mm * ks * 4 + (size_t)mm * (ks / 32) * 4;
}


template <int FMT>
static void launch_gemv2(vkb_context* ctx, const vkb_weight* w, int64_t m, const void* a, int a_fmt, const Epi& e,
                         float* ws, int units_per_split, int splits) {
    const int n_tiles = (int)(w->n_pad / TILE_N);
    if (splits > 1 && n_tiles > kTileCounters) fail(VKB_ERROR_UNSUPPORTED_OP, "linear: too many weight tiles");
    dim3 grid((unsigned)n_tiles, (unsigned)splits);
    const uint8_t* qs = w->qs.as<uint8_t>();
    const uint8_t* sc = w->sc.as<uint8_t>();
    unsigned* ctr = ctx->tile_ctr.as<unsigned>();
    auto go = [&](auto MMc) {
        constexpr int MMv = decltype(MMc)::value;
        const size_t sm = gemv2_smem(FMT, MMv, units_per_split);
        smem_optin(gemv2_kernel<FMT, MMv>, 200 * 1024);
        launch_pdl(ctx, gemv2_kernel<FMT, MMv>, grid, 128, sm, qs, sc, w->k, w->n, m, a, a_fmt, units_per_split,
                   splits, ws, ctr, device_err_flag(ctx), e);
    };
    if (m <= 1) go(std::integral_constant<int, 1>{});
    else if (m <= 2) go(std::integral_constant<int, 2>{});
    else if (m <= 4) go(std::integral_constant<int, 4>{});
    else go(std::integral_constant<int, 8>{});
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}

template <int FMT>
static void launch_gemv(vkb_context* ctx, const vkb_weight* w, int64_t m, const void* a, int a_fmt, const Epi& e,
                        float* ws, int stages_per_split, int splits) {
    dim3 grid((unsigned)(w->n_pad / TILE_N), (unsigned)splits);
    const uint8_t* qs = w->qs.as<uint8_t>();
    const uint8_t* sc = w->sc.as<uint8_t>();
#define VKB_GEMV(MMv)                                                                                           \
    {                                                                                                           \
        size_t sm = (size_t)(MMv)*stages_per_split * STAGE_K * sizeof(float);                                   \
        smem_optin(gemv_kernel<FMT, MMv>, 200 * 1024);                                                          \
        launch_pdl(ctx, gemv_kernel<FMT, MMv>, grid, 128, sm, qs, sc, w->k, w->n, m, a, a_fmt, stages_per_split, \
                                                              splits, ws, e);                                   \
    }
    if (m <= 1) VKB_GEMV(1) else if (m <= 2) VKB_GEMV(2) else VKB_GEMV(4)
#undef VKB_GEMV
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}

template <int FMT, int BN, bool SPLIT>
static void launch_tc(vkb_context* ctx, const vkb_weight* w, int64_t m, const __half* a16, const Epi& e, float* ws,
                      int stages_per_split, int splits, int m_tiles) {
    using C = TcCfg<FMT, BN, SPLIT>;
    smem_optin(tc_gemm_kernel<FMT, BN, SPLIT>, C::SMEM);
    CUtensorMap map, map_lo, omap, omap_lo, rmap;
    make_tmap_f16(&map, a16, m, w->k, BN);
    if (SPLIT) make_tmap_f16(&map_lo, a16 + m * w->k, m, w->k, BN);
    else map_lo = map;
    // TMA epilogue: plain row-major output whose rows are 16-byte aligned.
    const int esz = e.out_fmt == VKB_DT_F32 ? 4 : 2;
    int tma_epi = e.col_block == 0 && e.row_map == nullptr && ((uintptr_t)e.out % 16) == 0 &&
                  (w->n * esz) % 16 == 0 && (e.kind != VKB_EPI_RESIDUAL || ((uintptr_t)e.residual % 16) == 0) &&
                  (int64_t)BN * TILE_N * 4 * (e.out_fmt == VKB_DT_F16X2 ? 1 : 1) <= (int64_t)C::S * C::STAGE_BYTES;
    const bool partial_ok = (w->n * 4) % 16 == 0 && ((uintptr_t)ws % 16) == 0 &&
                            (int64_t)BN * TILE_N * 4 <= (int64_t)C::S * C::STAGE_BYTES;
    if (splits > 1) {
        tma_epi = partial_ok ? 2 : 0;
        if (tma_epi) make_tmap_3d_f32(&omap, ws, splits, m, w->n, TILE_N, BN);
        omap_lo = rmap = map;
        if (!tma_epi) omap = map;
    } else if (tma_epi) {
        make_tmap_2d(&omap, e.out, esz, m, w->n, TILE_N, BN);
        if (e.out_fmt == VKB_DT_F16X2) make_tmap_2d(&omap_lo, reinterpret_cast<const __half*>(e.out) + e.plane, 2, m, w->n, TILE_N, BN);
        else omap_lo = omap;
        if (e.kind == VKB_EPI_RESIDUAL) make_tmap_2d(&rmap, e.residual, 4, m, w->n, TILE_N, BN);
        else rmap = omap;
    } else {
        omap = omap_lo = rmap = map;
    }
    int n_tiles = (int)(w->n_pad / TILE_N);
    dim3 grid((unsigned)(n_tiles * m_tiles * splits));
    launch_pdl(ctx, tc_gemm_kernel<FMT, BN, SPLIT>, grid, C::THREADS, C::SMEM, 
        map, map_lo, w->qs.as<uint8_t>(), w->sc.as<uint8_t>(), w->k, w->n, m, n_tiles, m_tiles, stages_per_split,
        splits, ws, e, device_err_flag(ctx), omap, omap_lo, rmap, tma_epi);
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}

template <int FMT, bool SPLIT>
static void dispatch_tc(vkb_context* ctx, const vkb_weight* w, int64_t m, const __half* a16, const Epi& e, float* ws,
                        int bn, int sps, int splits, int m_tiles) {
    switch (bn) {
        case 32: launch_tc<FMT, 32, SPLIT>(ctx, w, m, a16, e, ws, sps, splits, m_tiles); break;
        case 64: launch_tc<FMT, 64, SPLIT>(ctx, w, m, a16, e, ws, sps, splits, m_tiles); break;
        case 128: launch_tc<FMT, 128, SPLIT>(ctx, w, m, a16, e, ws, sps, splits, m_tiles); break;
        default: launch_tc<FMT, 256, SPLIT>(ctx, w, m, a16, e, ws, sps, splits, m_tiles); break;
    }
}

template <bool SPLIT>
static void dispatch_fmt(vkb_context* ctx, const vkb_weight* w, int64_t m, const __half* a16, const Epi& e, float* ws,
                         const LinearPlan& p) {
    with_fmt(w->fmt, [&](auto F) { dispatch_tc<decltype(F)::value, SPLIT>(ctx, w, m, a16, e, ws, p.bn, p.sps, p.splits, p.m_tiles); });
}

LinearPlan plan_linear(const vkb_context* ctx, const vkb_weight* w, int64_t m, bool split) {
    LinearPlan p;
    const int64_t total = w->k / STAGE_K;
    const int n_tiles = (int)(w->n_pad / TILE_N);
    const int sms = ctx->sm_count;
    static const bool gv2_off = [] { const char* v = std::getenv("VKB_GEMV2"); return v && v[0] == '0'; }();
    // the streaming GEMV wins at m = 1, and up to m = 4 for wide weights (the
    // logits head); the tensor-core GEMM's fixed cost is lower elsewhere
    // (configs[1] sweep, CUDA-graph timing)
    if (m <= gemv_max_m() && gemv2_fmt(w->fmt) && !gv2_off && (m == 1 || (m <= 4 && w->n >= 16384))) {
        // the streaming GEMV: about 8 CTAs per SM, at least 2 units each, at
        // most ~28 KB of shared memory per CTA
        p.tc = false;
        p.gv2 = true;
        const int uk = w->fmt == W_Q4_K ? 64 : 32;
        const int64_t units = w->k / uk;
        const int mm = m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : 8;
        int splits = (int)std::max<int64_t>(
            1, std::min<int64_t>({units / 2, (8LL * sms + n_tiles - 1) / n_tiles, (int64_t)gv2_max_splits()}));
        int ups = (int)((units + splits - 1) / splits);
        static const size_t cap = [] {
            const char* v = std::getenv("VKB_GV2_SMEM_KB");
            return (size_t)(v ? std::atoi(v) : 28) * 1024;
        }();
        while (ups > 2 && gemv2_smem(w->fmt, mm, ups) > cap) --ups;
        splits = (int)((units + ups - 1) / ups);
        p.splits = splits;
        p.sps = ups;
    } else if (m <= std::min(4, gemv_max_m()) && !gemv2_fmt(w->fmt)) {
        p.tc = false;
        // Enough CTAs to cover the SMs several times; at least 2 stages each.
        int splits = std::max(1, std::min<int>((int)(total / 2), (4 * sms + n_tiles - 1) / n_tiles));
        int sps = (int)((total + splits - 1) / splits);
        sps = std::min(sps, 48);  // activation staging <= 48 KB per row of m
        splits = (int)((total + sps - 1) / sps);
        p.splits = splits;
        p.sps = sps;
    } else {
        p.tc = true;
        p.split = split;
        int bn = m <= 32 ? 32 : m <= 64 ? 64 : m <= 128 ? 128 : 256;
        int m_tiles = (int)((m + bn - 1) / bn);
        if (bn == 256 && (int64_t)n_tiles * m_tiles < sms) {
            bn = 128;
            m_tiles = (int)((m + bn - 1) / bn);
        }
        int ctas = n_tiles * m_tiles;
        int splits = 1;
        // K splits to fill the SMs (VKB_TC_CTA_TARGET scales the CTA target, for measurements)
        static const int target = [] { const char* v = std::getenv("VKB_TC_CTA_TARGET"); return v ? std::atoi(v) : 100; }();
        const int want = std::max(1, sms * target / 100);
        if (ctas < want) splits = std::max(1, std::min<int>((int)(total / 2), want / ctas));
        int sps = (int)((total + splits - 1) / splits);
        splits = (int)((total + sps - 1) / sps);
        p.bn = bn;
        p.m_tiles = m_tiles;
        p.splits = splits;
        p.sps = sps;
    }
    p.ws_bytes = (p.splits > 1 ? (size_t)p.splits * m * w->n * sizeof(float) : 0);
    return p;
}

LinearPlan plan_linear(const vkb_context* ctx, const vkb_weight* w, int64_t m) {
    return plan_linear(ctx, w, m, ctx->precision != VKB_PREC_F16);
}

void run_linear(vkb_context* ctx, const vkb_weight* w, int64_t m, const void* a, int a_dtype, const float* bias,
                void* out, int out_dtype, int epilogue, const float* residual, float scale, float* ws_override,
                __half* a16_override) {
    LinearExtra x;
    run_linear_ex(ctx, w, m, a, a_dtype, bias, out, out_dtype, epilogue, residual, scale, ws_override, a16_override, x);
}

void run_linear_ex(vkb_context* ctx, const vkb_weight* w, int64_t m, const void* a, int a_dtype, const float* bias,
                   void* out, int out_dtype, int epilogue, const float* residual, float scale, float* ws_override,
                   __half* a16_override, const LinearExtra& x) {
    NvtxRange nvtx_range(m <= gemv_max_m() ? "vkb.linear.small_m" : "vkb.linear.gemm");
    if (m <= 0) fail(VKB_ERROR_INVALID_ARGUMENT, "linear: m must be positive");
    if (!a || !out) fail(VKB_ERROR_INVALID_ARGUMENT, "linear: null activation or output pointer");
    if (a_dtype != VKB_DT_F32 && a_dtype != VKB_DT_F16 && a_dtype != VKB_DT_F16X2)
        fail(VKB_ERROR_INVALID_ARGUMENT, "linear: bad a_dtype");
    if (out_dtype != VKB_DT_F32 && out_dtype != VKB_DT_F16 && out_dtype != VKB_DT_F16X2)
        fail(VKB_ERROR_INVALID_ARGUMENT, "linear: bad out_dtype");
    if (epilogue < VKB_EPI_NONE || epilogue > VKB_EPI_SCALE) fail(VKB_ERROR_INVALID_ARGUMENT, "linear: bad epilogue");
    if (epilogue == VKB_EPI_RESIDUAL && (out_dtype != VKB_DT_F32 || !residual))
        fail(VKB_ERROR_INVALID_ARGUMENT, "linear: the residual epilogue needs an f32 output and a residual pointer");
    if (x.col_block > 0 && out_dtype == VKB_DT_F16X2)
        fail(VKB_ERROR_INVALID_ARGUMENT, "linear: a column-block layout needs an f32 or f16 output");
    // A single f16 activation plane carries no low part: the GEMM then runs unsplit.
    const bool split = ctx->precision != VKB_PREC_F16 && a_dtype != VKB_DT_F16;
    LinearPlan p = plan_linear(ctx, w, m, split);
    const int64_t out_rows = x.out_rows > 0 ? x.out_rows : m;
    Epi e{bias, residual, out, out_dtype, epilogue, scale, w->n,
          x.n_scaled >= 0 ? x.n_scaled : w->n, x.col_block, out_rows, x.row_map,
          x.row_group > 0 ? x.row_group : 1, out_rows * w->n};
    if (x.col_block > 0 && (w->n % x.col_block)) fail(VKB_ERROR_INVALID_ARGUMENT, "linear: n not a multiple of col_block");
    // Workspace: [f16 (or f16 hi+lo) copy of a: tc path with f32 input] [split-K partials]
    size_t a16_bytes = (p.tc && a_dtype == VKB_DT_F32 && !a16_override)
                           ? ((size_t)m * w->k * 2 * (split ? 2 : 1) + 255) / 256 * 256
                           : 0;
    size_t ws_bytes = ws_override ? 0 : p.ws_bytes;
    if (a16_bytes + ws_bytes) ctx->ensure_workspace(a16_bytes + ws_bytes);
    uint8_t* wsb = ctx->workspace.as<uint8_t>();
    float* ws = ws_override ? ws_override : reinterpret_cast<float*>(wsb + a16_bytes);
    if (!p.tc) {
        if (p.gv2) {
            if (w->fmt == W_Q4_0) launch_gemv2<W_Q4_0>(ctx, w, m, a, a_dtype, e, ws, p.sps, p.splits);
            else if (w->fmt == W_Q8_0) launch_gemv2<W_Q8_0>(ctx, w, m, a, a_dtype, e, ws, p.sps, p.splits);
            else launch_gemv2<W_Q4_K>(ctx, w, m, a, a_dtype, e, ws, p.sps, p.splits);
        } else {
            with_fmt(w->fmt, [&](auto F) { launch_gemv<decltype(F)::value>(ctx, w, m, a, a_dtype, e, ws, p.sps, p.splits); });
        }
    } else {
        const __half* a16;
        if (a_dtype != VKB_DT_F32) {
            a16 = reinterpret_cast<const __half*>(a);
        } else {
            __half* dst = a16_override ? a16_override : reinterpret_cast<__half*>(wsb);
            run_split_f16(ctx, reinterpret_cast<const float*>(a), m * w->k, dst, split);
            a16 = dst;
        }
        // Large-M split-precision GEMMs (the encoder): the persistent kernel
        // with a double-buffered accumulator, when there are tiles for several
        // waves and K is short enough (<= 20 stages) for the per-tile setup and
        // epilogue it hides to matter; at longer K the 256-token tile of the
        // classic kernel streams faster (encoder fc2, K = 5120: 2.45 vs 2.65 ms).
        // VKB_GEMM_PERSIST: "0" never, "force" for every unsplit-K GEMM (tests).
        const char* pv = std::getenv("VKB_GEMM_PERSIST");
        const bool p_off = pv && pv[0] == '0', p_force = pv && pv[0] == 'f';
        const int64_t p_tiles = (w->n_pad / TILE_N) * ((m + persist_bn() - 1) / persist_bn());
        // (single-f16 operands: not for the residual projections, measured faster on the classic kernel)
        // The SS kernel (single f16: weights dequantized once per call into an f16 plane, both operands
        // by TMA) takes every such GEMM, residual projections and K = 5120 included.
        const bool ss = !p.split && persist_ss_enabled();
        if (!p_off && p.splits == 1 && x.col_block == 0 && !x.row_map &&
            (p.split || ss || epilogue != VKB_EPI_RESIDUAL) &&
            (p_force || (p_tiles >= 4 * (int64_t)ctx->sm_count && (ss || w->k <= 20 * STAGE_K)))) {
            PEpi pe;
            pe.bias = bias;
            pe.residual = residual;
            pe.out = out;
            pe.out_fmt = out_dtype;
            pe.kind = epilogue;
            pe.scale = scale;
            pe.ldo = w->n;
            pe.n_scaled = e.n_scaled;
            pe.plane = e.plane;
            run_tc_persistent(ctx, w, m, a16, pe, device_err_flag(ctx), p.split);
        } else if (p.split) {
            dispatch_fmt<true>(ctx, w, m, a16, e, ws, p);
        } else {
            dispatch_fmt<false>(ctx, w, m, a16, e, ws, p);
        }
    }
    if (x.splits_out) *x.splits_out = p.splits;
    if (p.gv2 && x.splits_out) *x.splits_out = 1;  // reduced in the kernel
    if (p.splits > 1 && !x.splits_out && !p.gv2) {
        int64_t tot = m * w->n;
        launch_pdl(ctx, splitk_reduce_kernel, (unsigned)((tot + 255) / 256), 256, 0, ws, p.splits, m, w->n, e);
        VKB_CUDA(cudaGetLastError());
        ctx->count();
    }
}

bool run_linear_q8_pair(vkb_context* ctx, const vkb_weight* w, int64_t m, const __half* a16, const float* bias,
                        int64_t width, int8_t* kq, __half* kd, int8_t* vq, __half* vd, const int32_t* row_map,
                        int row_group, bool split) {
    const char* pv = std::getenv("VKB_GEMM_PERSIST");
    if (pv && pv[0] == '0') return false;
    const char* fq = std::getenv("VKB_FUSED_CROSS_Q8");
    if (fq && fq[0] == '0') return false;
    // split: hi + lo activation planes (TMEM-operand kernel); single f16: the shared-operand kernels only
    if (split ? ctx->precision == VKB_PREC_F16 : !persist_ss_enabled()) return false;
    if (m <= 0 || w->n != 2 * width || width % TILE_N || w->n_pad != w->n) return false;
    if (plan_linear(ctx, w, m, split).splits != 1) return false;
    PEpi pe;
    pe.bias = bias;
    pe.residual = nullptr;
    pe.out = nullptr;
    pe.out_fmt = VKB_DT_F32;
    pe.kind = VKB_EPI_NONE;
    pe.scale = 1.0f;
    pe.ldo = w->n;
    pe.n_scaled = w->n;
    pe.plane = 0;
    pe.q8_width = width;
    pe.q8[0] = kq;
    pe.q8[1] = vq;
    pe.q8d[0] = kd;
    pe.q8d[1] = vd;
    pe.row_map = row_map;
    pe.row_group = row_group > 0 ? row_group : 1;
    run_tc_persistent(ctx, w, m, a16, pe, device_err_flag(ctx), split);
    return true;
}

// A wait that can never complete (an mbarrier nothing arrives at), bounded by
// `polls` polls, exactly as every pipeline wait of the library is bounded: on
// giving up it records the error flag and returns, and the context stays usable.
__global__ void bounded_wait_selftest_kernel(int* err, uint32_t polls) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        ptx::mbar_init(&bar, 1);
        ptx::fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0 && !ptx::mbar_wait(&bar, 0, polls)) atomicExch(err, 1);
}

int read_and_clear_err_flag(vkb_context* ctx) {
    int* f = device_err_flag(ctx);
    int h = 0;
    VKB_CUDA(cudaMemcpyAsync(&h, f, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
    VKB_CUDA(cudaStreamSynchronize(ctx->stream));
    if (h) VKB_CUDA(cudaMemsetAsync(f, 0, sizeof(int), ctx->stream));
    return h;
}

}  // namespace vkb

using namespace vkb;

extern "C" {

vkb_status vkb_weight_upload(vkb_context* ctx, uint32_t ggml_type, int64_t n, int64_t k, const void* bytes,
                             size_t len, vkb_weight** out) {
    return guard([&] {
        if (!out) fail(VKB_ERROR_INVALID_ARGUMENT, "weight_upload: null out");
        *out = upload_weight(ctx, ggml_type, n, k, bytes, len);
    });
}

vkb_status vkb_weight_destroy(vkb_weight* w) {
    return guard([&] { delete w; });
}

size_t vkb_weight_device_bytes(const vkb_weight* w) { return w ? w->qs.n + w->sc.n : 0; }

vkb_status vkb_linear(vkb_context* ctx, const vkb_weight* w, int64_t m, const void* a_dev, int a_dtype,
                      const float* bias_dev, void* out_dev, int out_dtype, int epilogue, const float* residual_dev,
                      float scale) {
    return guard([&] {
        if (!ctx || !w) fail(VKB_ERROR_INVALID_ARGUMENT, "linear: null context or weight");
        if (w->ctx != ctx) fail(VKB_ERROR_INVALID_ARGUMENT, "linear: weight belongs to another context");
        run_linear(ctx, w, m, a_dev, a_dtype, bias_dev, out_dev, out_dtype, epilogue, residual_dev, scale, nullptr,
                   nullptr);
    });
}

vkb_status vkb_gemm_q_f32(vkb_context* ctx, int64_t m, int64_t n, int64_t k, const float* a_host, const void* wq_host,
                          size_t wq_len, uint32_t ggml_type, const float* bias_host, float* out_host) {
    return guard([&] {
        if (!ctx) fail(VKB_ERROR_INVALID_ARGUMENT, "gemm_q_f32: null context");
        if (!a_host || !wq_host || !out_host) fail(VKB_ERROR_INVALID_ARGUMENT, "gemm_q_f32: null buffer");
        if (m <= 0) fail(VKB_ERROR_INVALID_ARGUMENT, "gemm_q_f32: m must be positive");
        std::unique_ptr<vkb_weight> w(upload_weight(ctx, ggml_type, n, k, wq_host, wq_len));
        DevBuf a((size_t)m * k * 4), o((size_t)m * n * 4), b(bias_host ? (size_t)n * 4 : 0);
        VKB_CUDA(cudaMemcpyAsync(a.p, a_host, a.n, cudaMemcpyHostToDevice, ctx->stream));
        if (bias_host) VKB_CUDA(cudaMemcpyAsync(b.p, bias_host, b.n, cudaMemcpyHostToDevice, ctx->stream));
        run_linear(ctx, w.get(), m, a.p, VKB_DT_F32, bias_host ? b.as<float>() : nullptr, o.p, VKB_DT_F32,
                   VKB_EPI_NONE, nullptr, 1.0f, nullptr, nullptr);
        VKB_CUDA(cudaMemcpyAsync(out_host, o.p, o.n, cudaMemcpyDeviceToHost, ctx->stream));
        VKB_CUDA(cudaStreamSynchronize(ctx->stream));
        if (read_and_clear_err_flag(ctx)) fail(VKB_ERROR_OTHER, "gemm_q_f32: a pipeline wait timed out on the device");
    });
}

vkb_status vkb_context_selftest_bounded_wait(vkb_context* ctx, uint32_t polls) {
    return guard([&] {
        if (!ctx) fail(VKB_ERROR_INVALID_ARGUMENT, "selftest_bounded_wait: null context");
        if (polls == 0 || polls > (1u << 20)) fail(VKB_ERROR_INVALID_ARGUMENT, "selftest_bounded_wait: polls in 1..2^20");
        VKB_CUDA(cudaSetDevice(ctx->device));
        if (read_and_clear_err_flag(ctx)) fail(VKB_ERROR_OTHER, "selftest_bounded_wait: the error flag was already set");
        bounded_wait_selftest_kernel<<<1, 32, 0, ctx->stream>>>(device_err_flag(ctx), polls);
        VKB_CUDA(cudaGetLastError());
        ctx->count();
        if (read_and_clear_err_flag(ctx)) fail(VKB_ERROR_OTHER, "selftest_bounded_wait: the wait gave up after " +
                                                                    std::to_string(polls) + " polls");
    });
}

}  // extern "C"
