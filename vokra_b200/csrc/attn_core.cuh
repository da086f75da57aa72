// attn_core.cuh — decode attention over K/V rows fetched through a policy
// (paged int8 pages, dense int8 or dense f16), fp32 online softmax.
//
// Work decomposition: one CTA per (query group, key split). A query group is
// up to MAXQ consecutive query tokens of one stream (the decode step's token,
// or a prefix). The CTA holds R row-groups of W/16 threads; a row-group owns
// one key at a time and each of its threads owns 16 consecutive channels, so
// the d_head/16 threads of a head reduce their partial q.k with two shuffles.
// Row-groups walk keys j = j0 + g, j0 + g + R, ...; at the end the R partial
// (max, sum, acc) triples are merged in shared memory. With one split the
// CTA writes ctx = acc / sum, else the triple goes to a workspace and
// attn_combine_kernel merges the splits.
#pragma once
#include "common.cuh"

namespace vkb {

constexpr int ATTN_MAX_THREADS = 256;

// 16 int8 values of a 32-bit-word quadruple -> floats, exactly, without I2F:
// the byte is placed in the low mantissa of 2^23 and the bias removed.
__device__ __forceinline__ void i8x16_to_f32(uint4 q, float (&f)[16]) {
    uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int b = 0; b < 4; ++b)
            f[4 * i + b] = __uint_as_float(__byte_perm(w[i], 0x4B000000u, 0x7440u + b)) - 8388736.0f;
    }
}

// Raw bytes of 16 channels of one K or V row, kept in registers until use
// (the fields a policy does not load are dropped by the compiler).
struct RawRow {
    uint4 a, b, c, e;  // int8: a; Q4_0: a.xy; Q5_0: a.xy + 16 high bits in a.z; f16: a, b; f32: a, b, c, e
    float s;           // block scale (1 for f16 / f32)
};

// 16 channels of a Q4_0 / Q5_0 KV block (kv_quant/q4_0.rs:73, q5_0.rs:84):
// channel 2i / 2i+1 in the low / high nibble of byte i, biased by 8 (Q4_0) or,
// with its 5th bit from qh, by 16 (Q5_0). Exact small integers.
template <bool Q5>
__device__ __forceinline__ void nib16_to_f32(const uint4& a, float (&f)[16]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t byte = ((i < 4 ? a.x : a.y) >> (8 * (i & 3))) & 0xffu;
        uint32_t lo = byte & 0xfu, hi = byte >> 4;
        if (Q5) {
            lo |= ((a.z >> (2 * i)) & 1u) << 4;
            hi |= ((a.z >> (2 * i + 1)) & 1u) << 4;
        }
        f[2 * i] = (float)((int)lo - (Q5 ? 16 : 8));
        f[2 * i + 1] = (float)((int)hi - (Q5 ? 16 : 8));
    }
}

// ---- fetch policies: value of 16 channels [c0, c0+16) of key j ------------
// Paged K/V of any pool mode (vkb_kv_quant): quant plane rows of qrow bytes,
// Q5_0 high-bit rows of hrow bytes, f16 scale rows of W/32.
template <int MODE>
struct FetchPaged {
    const uint8_t* kq;
    const __half* kd;
    const uint8_t* kh;
    const uint8_t* vq;
    const __half* vd;
    const uint8_t* vh;
    const int32_t* table;
    int W, qrow, hrow;
    int layout;      // 0 reference, 1 sequence
    int table_base;  // reference: layer*ppl ; sequence: seq*ppseq
    int bs;
    int n_sc;        // slots per token row (reference: n_stream; sequence: 1)
    int slot;        // reference: stream index ; sequence: 0
    int64_t arena_row0;  // sequence: layer*n_pages*rpp ; reference: 0
    __device__ __forceinline__ int64_t row(int j) const {
        int pid = table[table_base + j / bs];
        return arena_row0 + ((int64_t)pid * bs + (j % bs)) * n_sc + slot;
    }
    __device__ __forceinline__ void load_raw(int64_t rw, int c0, bool is_v, RawRow& r) const {
        const uint8_t* q = (is_v ? vq : kq) + rw * qrow;
        if constexpr (MODE == VKB_KV_Q8_0) {
            r.a = __ldg(reinterpret_cast<const uint4*>(q + c0));
        } else if constexpr (MODE == VKB_KV_FP32) {
            const uint4* p = reinterpret_cast<const uint4*>(q + 4 * c0);
            r.a = __ldg(p);
            r.b = __ldg(p + 1);
            r.c = __ldg(p + 2);
            r.e = __ldg(p + 3);
            r.s = 1.0f;
            return;
        } else {
            const uint2 t = __ldg(reinterpret_cast<const uint2*>(q + c0 / 2));
            r.a.x = t.x;
            r.a.y = t.y;
            if constexpr (MODE == VKB_KV_Q5_0)
                r.a.z = __ldg(reinterpret_cast<const uint16_t*>((is_v ? vh : kh) + rw * hrow + c0 / 8));
        }
        r.s = __half2float(__ldg((is_v ? vd : kd) + rw * (W / 32) + c0 / 32));
    }
    static __device__ __forceinline__ void convert(const RawRow& r, float (&f)[16]) {
        if constexpr (MODE == VKB_KV_Q8_0) {
            i8x16_to_f32(r.a, f);
        } else if constexpr (MODE == VKB_KV_FP32) {
            const uint4 w[4] = {r.a, r.b, r.c, r.e};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                f[4 * i] = __uint_as_float(w[i].x);
                f[4 * i + 1] = __uint_as_float(w[i].y);
                f[4 * i + 2] = __uint_as_float(w[i].z);
                f[4 * i + 3] = __uint_as_float(w[i].w);
            }
        } else {
            nib16_to_f32<MODE == VKB_KV_Q5_0>(r.a, f);
        }
    }
};
using FetchPagedQ8 = FetchPaged<VKB_KV_Q8_0>;

struct FetchDenseQ8 {
    const int8_t* kq;
    const __half* kd;
    const int8_t* vq;
    const __half* vd;
    int W;
    int64_t seq_row0;  // seq * n_ctx
    __device__ __forceinline__ int64_t row(int j) const { return seq_row0 + j; }
    __device__ __forceinline__ void load_raw(int64_t rw, int c0, bool is_v, RawRow& r) const {
        r.a = __ldg(reinterpret_cast<const uint4*>((is_v ? vq : kq) + rw * W + c0));
        r.s = __half2float(__ldg((is_v ? vd : kd) + rw * (W / 32) + c0 / 32));
    }
    static __device__ __forceinline__ void convert(const RawRow& r, float (&f)[16]) { i8x16_to_f32(r.a, f); }
};

struct FetchDenseF16 {
    const __half* k;
    const __half* v;
    int W;
    int64_t seq_row0;
    __device__ __forceinline__ int64_t row(int j) const { return seq_row0 + j; }
    __device__ __forceinline__ void load_raw(int64_t rw, int c0, bool is_v, RawRow& r) const {
        const __half* p = (is_v ? v : k) + rw * W + c0;
        r.a = __ldg(reinterpret_cast<const uint4*>(p));
        r.b = __ldg(reinterpret_cast<const uint4*>(p + 8));
        r.s = 1.0f;
    }
    static __device__ __forceinline__ void convert(const RawRow& r, float (&f)[16]) {
        uint32_t w[8] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float2 t = __half22float2(*reinterpret_cast<__half2*>(&w[i]));
            f[2 * i] = t.x;
            f[2 * i + 1] = t.y;
        }
    }
};

// Per-CTA query group descriptor.
struct AttnGroup {
    int first_tok;  // index of the first query row in q / ctx
    int n_q;        // queries in the group (<= MAXQ)
    int seq;        // stream
    int pos0;       // absolute position of the first query; query i sees keys 0..pos0+i
};

// Partial layout in the workspace, per (group, split, query):
//   acc[W] then m[H] then l[H]  (floats)
template <class F, int MAXQ>
__device__ __forceinline__ void attn_body(const F& fetch, const float* __restrict__ q, int64_t q_ld, const AttnGroup& g,
                                          int n_head,
                                          int d_head, int W, int key_begin, int key_end, int split, int n_splits,
                                          void* ctx_out, int out_fmt, int64_t out_plane, float* ws) {
    extern __shared__ float sm[];
    const int tpr = W / 16;                // threads per key row
    const int R = blockDim.x / tpr;        // row-groups
    const int tid = threadIdx.x;
    const int rg = tid / tpr, tr = tid % tpr;
    const int c0 = tr * 16;
    const int tph = d_head / 16;           // threads per head
    const bool active = rg < R;

    float qv[MAXQ][16];
    float m[MAXQ], l[MAXQ], acc[MAXQ][16];
#pragma unroll
    for (int i = 0; i < MAXQ; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int c = 0; c < 16; ++c) acc[i][c] = 0.0f;
        if (active && i < g.n_q) {
            const float4* q4 = reinterpret_cast<const float4*>(q + (int64_t)(g.first_tok + i) * q_ld + c0);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                float4 t = q4[c];
                qv[i][4 * c] = t.x; qv[i][4 * c + 1] = t.y; qv[i][4 * c + 2] = t.z; qv[i][4 * c + 3] = t.w;
            }
        } else {
#pragma unroll
            for (int c = 0; c < 16; ++c) qv[i][c] = 0.0f;
        }
    }

    // Every row-group runs the same trip count so that the head shuffles
    // always see full warps (a warp can hold threads of two row-groups).
    // KU keys per row-group per iteration: their loads are issued together and
    // the running softmax is rescaled once per iteration.
    constexpr int KU = 2;
    const int n_iter = (key_end - key_begin + R * KU - 1) / (R * KU);
    if (active) {
        for (int it = 0; it < n_iter; ++it) {
            int jj[KU];
            bool valid[KU];
            RawRow kr[KU], vr[KU];
#pragma unroll
            for (int u = 0; u < KU; ++u) {
                jj[u] = key_begin + rg + (it * KU + u) * R;
                valid[u] = jj[u] < key_end;
                if (valid[u]) {
                    int64_t rw = fetch.row(jj[u]);
                    fetch.load_raw(rw, c0, false, kr[u]);
                    fetch.load_raw(rw, c0, true, vr[u]);
                } else {
                    kr[u].a = make_uint4(0, 0, 0, 0);
                    kr[u].b = kr[u].c = kr[u].e = kr[u].a;
                    kr[u].s = 0.0f;
                    vr[u] = kr[u];
                }
            }
#pragma unroll
            for (int i = 0; i < MAXQ; ++i) {
                if (i >= g.n_q) break;
                float part[KU];
#pragma unroll
                for (int u = 0; u < KU; ++u) {
                    float kf[16];
                    F::convert(kr[u], kf);
                    float acc_d = 0.0f;
#pragma unroll
                    for (int c = 0; c < 16; ++c) acc_d = fmaf(qv[i][c], kf[c], acc_d);
                    acc_d *= kr[u].s;
                    // sum over the head's threads (consecutive, aligned to tph)
                    for (int o = 1; o < tph; o <<= 1) acc_d += __shfl_xor_sync(0xffffffffu, acc_d, o);
                    const bool use = valid[u] && jj[u] <= g.pos0 + i;  // causal: keys up to this query
                    part[u] = use ? acc_d : -INFINITY;
                }
                float mx = part[0];
#pragma unroll
                for (int u = 1; u < KU; ++u) mx = fmaxf(mx, part[u]);
                if (mx == -INFINITY) continue;
                const float mn = fmaxf(m[i], mx);
                const float corr = __expf(m[i] - mn);
                float lsum = l[i] * corr;
#pragma unroll
                for (int c = 0; c < 16; ++c) acc[i][c] *= corr;
#pragma unroll
                for (int u = 0; u < KU; ++u) {
                    const float p = __expf(part[u] - mn);  // 0 for unused keys
                    lsum += p;
                    float vf[16];
                    F::convert(vr[u], vf);
                    const float pv = p * vr[u].s;
#pragma unroll
                    for (int c = 0; c < 16; ++c) acc[i][c] = fmaf(pv, vf[c], acc[i][c]);
                }
                l[i] = lsum;
                m[i] = mn;
            }
        }
    }

    // Merge the R row-groups: row-group 0 gathers (m, l, acc) of the others.
    const int H = n_head;
    float* s_acc = sm;                       // [R][MAXQ][W]
    float* s_m = sm + (size_t)R * MAXQ * W;  // [R][MAXQ][H]
    float* s_l = s_m + (size_t)R * MAXQ * H;
    const int head = c0 / d_head;
    if (active) {
#pragma unroll
        for (int i = 0; i < MAXQ; ++i) {
#pragma unroll
            for (int c = 0; c < 16; ++c) s_acc[((size_t)rg * MAXQ + i) * W + c0 + c] = acc[i][c];
            if ((tr % tph) == 0) {
                s_m[((size_t)rg * MAXQ + i) * H + head] = m[i];
                s_l[((size_t)rg * MAXQ + i) * H + head] = l[i];
            }
        }
    }
    __syncthreads();
    if (rg == 0) {
#pragma unroll
        for (int i = 0; i < MAXQ; ++i) {
            if (i >= g.n_q) break;
            float M = -INFINITY;
            for (int r = 0; r < R; ++r) M = fmaxf(M, s_m[((size_t)r * MAXQ + i) * H + head]);
            float L = 0.0f, o[16];
#pragma unroll
            for (int c = 0; c < 16; ++c) o[c] = 0.0f;
            for (int r = 0; r < R; ++r) {
                float mr = s_m[((size_t)r * MAXQ + i) * H + head];
                float w = (mr == -INFINITY) ? 0.0f : __expf(mr - M);
                L += s_l[((size_t)r * MAXQ + i) * H + head] * w;
#pragma unroll
                for (int c = 0; c < 16; ++c) o[c] += s_acc[((size_t)r * MAXQ + i) * W + c0 + c] * w;
            }
            const int64_t tok = g.first_tok + i;
            if (n_splits == 1) {
                float inv = 1.0f / L;
                if (out_fmt != 0) {
                    __half* dst = reinterpret_cast<__half*>(ctx_out) + tok * W + c0;
#pragma unroll
                    for (int c = 0; c < 16; c += 2) {
                        float v0 = o[c] * inv, v1 = o[c + 1] * inv;
                        __half2 hi = __floats2half2_rn(v0, v1);
                        *reinterpret_cast<__half2*>(dst + c) = hi;
                        if (out_fmt == 2) {
                            float2 hf = __half22float2(hi);
                            *reinterpret_cast<__half2*>(dst + out_plane + c) = __floats2half2_rn(v0 - hf.x, v1 - hf.y);
                        }
                    }
                } else {
                    float* dst = reinterpret_cast<float*>(ctx_out) + tok * W + c0;
#pragma unroll
                    for (int c = 0; c < 16; ++c) dst[c] = o[c] * inv;
                }
            } else {
                // ws layout per (token, split): acc[W] m[H] l[H]
                float* p = ws + ((size_t)tok * n_splits + split) * (W + 2 * H);
#pragma unroll
                for (int c = 0; c < 16; ++c) p[c0 + c] = o[c];
                if ((tr % tph) == 0) {
                    p[W + head] = M;
                    p[W + H + head] = L;
                }
            }
        }
    }
}

// Merges split partials: one thread per (token, channel).
__global__ void attn_combine_kernel(const float* __restrict__ ws, int n_tok, int n_splits, int n_head, int d_head,
                                    void* ctx_out, int out_fmt);

inline size_t attn_smem_bytes(int R, int maxq, int W, int H) {
    return (size_t)R * maxq * (W + 2 * H) * sizeof(float);
}

}  // namespace vkb
