// xattn.cu — decode cross-attention over a dense Q8_0 (or f16) K/V store, built to
// stream the store at HBM bandwidth.
//
// Semantics are those of dense_attn_kernel (the softmax attention of
// crates/vokra-models/src/whisper/nn.rs:209-300 with K/V as Q8_0 rows):
// for every query row t of stream s = seq_of_tok[t],
//   score_j = sum_c q[t][c] * dK[s,j,c/32] * K[s,j,c]   (per head)
//   ctx[t]  = sum_j softmax(score)_j * dV[s,j,c/32] * V[s,j,c].
//
// Work decomposition (persistent, balanced): the key axis of every query row
// is cut into chunks of XA_T keys; the n_tok * chunks sequence is cut into G
// equal contiguous ranges, one per CTA (G <= SM count), so every SM streams
// the same number of bytes whatever n_tok is. A CTA range crosses at most a
// few query rows; at each crossing it writes the (acc, max, sum) partial of
// the finished row, and xattn_combine_kernel merges the partials of a row.
//
// Per CTA, a ring of S stages is filled by bulk copies (cp.async.bulk, one
// thread issues them): stage = XA_T rows of K quants, K scales, V quants and
// V scales, all contiguous in the store. 16*H threads:
//   Q.K   thread (head h = i/16, keys k = i%16 and k+16): the head's 64
//         channels of each key against q held as three int8 planes (q = s*(r1 + r2/254 +
//         r3/254^2), 2^-24-level accuracy) with dp4a; integer sums are exact,
//         the two block scales are applied in fp32. The 16 keys of a head are
//         16 lanes of one warp, so the stage max / sum are shuffles. Each
//         thread reads its 16-byte chunks in an order rotated by k, so the 8
//         threads of a shared-memory phase hit distinct banks.
//   P.V   thread i owns channels 4i..4i+3 (the same head h): per key one
//         32-bit load of V and one weight p*dV from shared memory.
// A warp holds two heads in both roles, so warps never wait for each other:
// each releases a stage on its own (an `empty` mbarrier counting H/2 warps)
// and one extra producer warp refills the ring.
// Every mbarrier wait is bounded; on timeout the CTA flags the error, waits
// (bounded) for its copies in flight and returns.
#include "common.cuh"
#include "tc_ptx.cuh"
#include "xattn.cuh"
#include <algorithm>

namespace vkb {

constexpr int XA_T = 32;        // keys per stage (Q8_0 store)
constexpr int XA_T16 = 16;      // keys per stage (f16 store: the same bytes per stage)
constexpr int XA_DH = 64;       // head width this kernel handles
constexpr int XA_MAX_STAGES = 6;
constexpr int XA_SMEM_BUDGET = 200 * 1024;

struct XaArgs {
    const float* q;
    const int32_t* seq_of_tok;
    const int8_t* kq;
    const __half* kd;
    const int8_t* vq;
    const __half* vd;
    int n_tok, n_ctx, H, W, chunks, G, max_seg, S;
    int total;
    float* ws;                      // partials [G][max_seg][W + 2H]
    int* err;
    // 1: no kernel still in flight writes K/V or seq_of_tok (the decode step:
    // the store is written by the encoder and the step starts with host
    // copies, a full barrier), so the ring is filled before the wait for the
    // previous kernel (the query projection) and overlaps its tail
    int kv_ready;
};

// First chunk of CTA c (the host guarantees total * G < 2^31, so 32-bit math is exact).
__host__ __device__ inline int xa_bound(int c, int total, int G) { return (int)((unsigned)(c * total) / (unsigned)G); }
__device__ __forceinline__ float xa_i8_f32(uint32_t w, int b) {
    // byte b of (w ^ 0x80808080) in the low mantissa of 2^23, bias removed: exact
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u + b)) - 8388736.0f;
}

__device__ __forceinline__ uint32_t xa_pack4(int a, int b, int c, int d) {
    return (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) | ((uint32_t)(c & 0xff) << 16) |
           ((uint32_t)(d & 0xff) << 24);
}

// Query planes of one head for one thread: chunk c of the rotated order holds
// channels 16*((c + rot) & 3) .. +16 of the head.
struct XaQ {
    uint32_t p1[16], p2[16], p3[16];
    float s[4];  // scale of the block of each rotated chunk
};

__device__ __forceinline__ void xa_load_q(const float* __restrict__ qrow, int rot, XaQ& Q) {
    // block scales (blocks 0 and 1 of the head: channels 0-31, 32-63)
    float amax[2] = {0.0f, 0.0f};
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        const float4* p = reinterpret_cast<const float4*>(qrow + 32 * b);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float4 v = p[i];
            amax[b] = fmaxf(amax[b], fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const int pc = (c + rot) & 3;  // physical chunk
        const int b = pc >> 1;
        const float am = b ? amax[1] : amax[0];
        const float inv = am > 0.0f ? 127.0f / am : 0.0f;
        Q.s[c] = am > 0.0f ? am / 127.0f : 0.0f;
        const float4* p = reinterpret_cast<const float4*>(qrow + 16 * pc);
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            float4 v = p[w];
            float x[4] = {v.x * inv, v.y * inv, v.z * inv, v.w * inv};
            int r1[4], r2[4], r3[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                float a = rintf(x[e]);
                float e1 = (x[e] - a) * 254.0f;
                float b2 = rintf(e1);
                float e2 = (e1 - b2) * 254.0f;
                r1[e] = (int)a;
                r2[e] = (int)b2;
                r3[e] = (int)rintf(e2);
            }
            Q.p1[4 * c + w] = xa_pack4(r1[0], r1[1], r1[2], r1[3]);
            Q.p2[4 * c + w] = xa_pack4(r2[0], r2[1], r2[2], r2[3]);
            Q.p3[4 * c + w] = xa_pack4(r3[0], r3[1], r3[2], r3[3]);
        }
    }
}

// F16 = true: the store holds K and V as f16 rows (no scales); XT = 16 keys
// per stage, q held as 64 fp32 registers per thread (rotated like the int8
// planes), Q.K and P.V in fp32 with packed f32x2 FMAs.
template <bool F16>
__global__ void __launch_bounds__(512, 1) xattn_q8_kernel(XaArgs a) {
    constexpr int XT = F16 ? XA_T16 : XA_T;  // keys per stage
    constexpr int KPL = XT / 16;               // keys per lane in the Q.K role
    pdl_launch();
    extern __shared__ __align__(128) uint8_t xa_smem[];
    const int W = a.W, H = a.H, S = a.S;
    const int nb = W / 32;
    const int kq_bytes = F16 ? XT * W * 2 : XT * W, kd_bytes = F16 ? 0 : XT * nb * 2;
    const int stage_bytes = 2 * (kq_bytes + kd_bytes);
    const int n_cw = H / 2;  // compute warps: two heads each
    uint8_t* ring = xa_smem;
    float* wt = reinterpret_cast<float*>(ring + (size_t)S * stage_bytes);  // [XT][nb]
    uint64_t* full = reinterpret_cast<uint64_t*>(wt + XT * nb);
    uint64_t* empty = full + S;

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x;
    const int x0 = xa_bound(c, a.total, a.G), x1 = xa_bound(c + 1, a.total, a.G);
    const int n_my = x1 - x0;

    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            ptx::mbar_init(&full[i], 1);
            ptx::mbar_init(&empty[i], n_cw);
        }
        ptx::fence_mbar_init();
    }
    __syncthreads();

    bool failed = false;
    int issued = 0;
    if (warp == n_cw) {
        // ---- producer warp: one lane streams the CTA's chunks through the ring ----
        if (lane == 0) {
            if (!a.kv_ready) pdl_wait();
            int tok = (int)(x0 / a.chunks), j = (int)(x0 % a.chunks);
            for (int i = 0; i < n_my; ++i, ++j) {
                if (j == a.chunks) {
                    j = 0;
                    ++tok;
                }
                const int s = i % S;
                if (i >= S && !ptx::mbar_wait(&empty[s], (uint32_t)(((i / S) - 1) & 1))) {
                    failed = true;
                    break;
                }
                const int nk = min(XT, a.n_ctx - j * XT);
                const int64_t row = (int64_t)a.seq_of_tok[tok] * a.n_ctx + (int64_t)j * XT;
                uint8_t* st = ring + (size_t)s * stage_bytes;
                uint64_t* bar = &full[s];
                if constexpr (F16) {
                    // K and V rows as f16: W * 2 bytes per key
                    ptx::mbar_expect_tx(bar, (uint32_t)(4 * nk * W));
                    ptx::bulk_load(st, a.kq + row * W * 2, (uint32_t)(nk * W * 2), bar);
                    ptx::bulk_load(st + kq_bytes, a.vq + row * W * 2, (uint32_t)(nk * W * 2), bar);
                } else {
                    ptx::mbar_expect_tx(bar, (uint32_t)(2 * nk * (W + nb * 2)));
                    ptx::bulk_load(st, a.kq + row * W, (uint32_t)(nk * W), bar);
                    ptx::bulk_load(st + kq_bytes, a.kd + row * nb, (uint32_t)(nk * nb * 2), bar);
                    ptx::bulk_load(st + kq_bytes + kd_bytes, a.vq + row * W, (uint32_t)(nk * W), bar);
                    ptx::bulk_load(st + 2 * kq_bytes + kd_bytes, a.vd + row * nb, (uint32_t)(nk * nb * 2), bar);
                }
                issued = i + 1;
            }
        }
    } else {
        // ---- compute warps: heads 2*warp, 2*warp+1 ----
        pdl_wait();  // q and the partial slots belong to earlier kernels
        const int h = tid >> 4;     // head of this thread (both roles)
        const int kk = tid & 15;    // key of this thread in the Q.K role
        XaQ Q;
        float qf[F16 ? XA_DH : 1];  // f16 store: q of the head, chunk cc = channels 8*((cc + kk) & 7) ..
        float m = -INFINITY, l = 0.0f;
        float2 acc01 = make_float2(0.0f, 0.0f), acc23 = make_float2(0.0f, 0.0f);
        int cur_tok = -1, seg = 0;
        auto flush = [&]() {
            float* p = a.ws + ((size_t)c * a.max_seg + seg) * (W + 2 * H);
            *reinterpret_cast<float4*>(p + 4 * tid) = make_float4(acc01.x, acc01.y, acc23.x, acc23.y);
            if (kk == 0) {
                p[W + h] = m;
                p[W + H + h] = l;
            }
        };
        int tok = (int)(x0 / a.chunks), j = (int)(x0 % a.chunks);
        for (int i = 0; i < n_my; ++i, ++j) {
            if (j == a.chunks) {
                j = 0;
                ++tok;
            }
            if (tok != cur_tok) {
                if (cur_tok >= 0) {
                    flush();
                    ++seg;
                }
                cur_tok = tok;
                m = -INFINITY;
                l = 0.0f;
                acc01 = make_float2(0.0f, 0.0f);
                acc23 = acc01;
                if constexpr (F16) {
                    const float* qrow = a.q + (int64_t)tok * W + h * XA_DH;
#pragma unroll
                    for (int cc = 0; cc < 8; ++cc) {
                        const int pc = (cc + kk) & 7;
                        const float4 v0 = *reinterpret_cast<const float4*>(qrow + 8 * pc);
                        const float4 v1 = *reinterpret_cast<const float4*>(qrow + 8 * pc + 4);
                        qf[8 * cc + 0] = v0.x; qf[8 * cc + 1] = v0.y; qf[8 * cc + 2] = v0.z; qf[8 * cc + 3] = v0.w;
                        qf[8 * cc + 4] = v1.x; qf[8 * cc + 5] = v1.y; qf[8 * cc + 6] = v1.z; qf[8 * cc + 7] = v1.w;
                    }
                } else {
                    xa_load_q(a.q + (int64_t)tok * W + h * XA_DH, kk, Q);
                }
            }
            const int nk = min(XT, a.n_ctx - j * XT);
            const int s = i % S;
            if (!ptx::mbar_wait(&full[s], (uint32_t)((i / S) & 1))) {
                failed = true;
                break;
            }
            const uint8_t* st = ring + (size_t)s * stage_bytes;
            const int8_t* Ks = reinterpret_cast<const int8_t*>(st);
            const __half* Kd = reinterpret_cast<const __half*>(st + kq_bytes);
            const int8_t* Vs = reinterpret_cast<const int8_t*>(st + kq_bytes + kd_bytes);
            const __half* Vd = reinterpret_cast<const __half*>(st + 2 * kq_bytes + kd_bytes);

            // ---- Q.K and the online softmax (16 lanes per head, KPL keys per lane) ----
            float score[KPL];
#pragma unroll
            for (int u = 0; u < KPL; ++u) {
                const int key = kk + 16 * u;
                score[u] = -INFINITY;
                if (F16 && key < nk) {
                    // 8 chunks of 8 channels in the rotated order of qf (16-byte loads on distinct banks)
                    const __half* krow = reinterpret_cast<const __half*>(st) + (size_t)key * W + h * XA_DH;
                    float2 acc2 = make_float2(0.0f, 0.0f);
#pragma unroll
                    for (int cc = 0; cc < 8; ++cc) {
                        const int pc = (cc + kk) & 7;
                        const uint4 kv = *reinterpret_cast<const uint4*>(krow + 8 * pc);
                        const uint32_t kw[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
                        for (int w = 0; w < 4; ++w) {
                            const float2 kf = __half22float2(*reinterpret_cast<const __half2*>(&kw[w]));
                            acc2 = __ffma2_rn(kf, make_float2(qf[8 * cc + 2 * w], qf[8 * cc + 2 * w + 1]), acc2);
                        }
                    }
                    score[u] = acc2.x + acc2.y;
                } else if (!F16 && key < nk) {
                    const uint8_t* krow = reinterpret_cast<const uint8_t*>(Ks + key * W + h * XA_DH);
                    const __half2 kd2 = *reinterpret_cast<const __half2*>(Kd + key * nb + 2 * h);
                    const float ks0 = __low2float(kd2), ks1 = __high2float(kd2);
                    float sc = 0.0f;
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) {
                        const int pc = (cc + kk) & 3;  // key = kk (mod 4): same rotation as the q planes
                        const uint4 kv = *reinterpret_cast<const uint4*>(krow + 16 * pc);
                        const uint32_t kw[4] = {kv.x, kv.y, kv.z, kv.w};
                        int d1 = 0, d2 = 0, d3 = 0;
#pragma unroll
                        for (int w = 0; w < 4; ++w) {
                            d1 = __dp4a((int)kw[w], (int)Q.p1[4 * cc + w], d1);
                            d2 = __dp4a((int)kw[w], (int)Q.p2[4 * cc + w], d2);
                            d3 = __dp4a((int)kw[w], (int)Q.p3[4 * cc + w], d3);
                        }
                        const float part =
                            fmaf((float)d3, 1.0f / 64516.0f, fmaf((float)d2, 1.0f / 254.0f, (float)d1));
                        const float ks = (pc >> 1) ? ks1 : ks0;
                        sc = fmaf(ks * Q.s[cc], part, sc);
                    }
                    score[u] = sc;
                }
            }
            float mx = score[0];
#pragma unroll
            for (int u = 1; u < KPL; ++u) mx = fmaxf(mx, score[u]);
#pragma unroll
            for (int o = 8; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float mn = fmaxf(m, mx);
            const float corr = (m == -INFINITY) ? 0.0f : __expf(m - mn);
            float ps = 0.0f;
#pragma unroll
            for (int u = 0; u < KPL; ++u) {
                const int key = kk + 16 * u;
                const float p = (key < nk && mn != -INFINITY) ? __expf(score[u] - mn) : 0.0f;
                ps += p;
                float w0 = 0.0f, w1 = 0.0f;
                if (F16) {
                    w0 = w1 = p;
                } else if (key < nk) {
                    const __half2 vd2 = *reinterpret_cast<const __half2*>(Vd + key * nb + 2 * h);
                    w0 = p * __low2float(vd2);
                    w1 = p * __high2float(vd2);
                }
                *reinterpret_cast<float2*>(wt + key * nb + 2 * h) = make_float2(w0, w1);
            }
#pragma unroll
            for (int o = 8; o >= 1; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            l = fmaf(l, corr, ps);
            m = mn;
            __syncwarp();

            // ---- P.V: channels 4*tid .. 4*tid+3 (heads of this warp) ----
            {
                const int b = tid >> 3;
                const float2 cr = make_float2(corr, corr);
                const float2 bias = make_float2(-8388736.0f, -8388736.0f);
                acc01 = __fmul2_rn(acc01, cr);
                acc23 = __fmul2_rn(acc23, cr);
                if constexpr (F16) {
                    const __half* Vh = reinterpret_cast<const __half*>(Vs);
#pragma unroll 4
                    for (int t = 0; t < nk; ++t) {
                        const float wv = wt[t * nb + b];
                        const uint2 v = *reinterpret_cast<const uint2*>(Vh + (size_t)t * W + 4 * tid);
                        const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
                        const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
                        const float2 w2 = make_float2(wv, wv);
                        acc01 = __ffma2_rn(w2, f01, acc01);
                        acc23 = __ffma2_rn(w2, f23, acc23);
                    }
                } else {
#pragma unroll 4
                for (int t = 0; t < nk; ++t) {
                    const float wv = wt[t * nb + b];
                    const uint32_t v = *reinterpret_cast<const uint32_t*>(Vs + t * W + 4 * tid) ^ 0x80808080u;
                    float2 f01 = make_float2(__uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440u)),
                                             __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7441u)));
                    float2 f23 = make_float2(__uint_as_float(__byte_perm(v, 0x4B000000u, 0x7442u)),
                                             __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7443u)));
                    f01 = __fadd2_rn(f01, bias);
                    f23 = __fadd2_rn(f23, bias);
                    const float2 w2 = make_float2(wv, wv);
                    acc01 = __ffma2_rn(w2, f01, acc01);
                    acc23 = __ffma2_rn(w2, f23, acc23);
                }
                }
            }
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&empty[s]);
        }
        if (!failed && cur_tok >= 0) flush();
    }
    __syncwarp();  // the producer warp ran on one lane: reconverge before the block barrier
    if (__syncthreads_or(failed)) {
        if (tid == 0) atomicExch(a.err, 1);
        if (warp == n_cw && lane == 0) {
            // let the copies still in flight land before the CTA's shared memory goes away
            for (int i = max(0, issued - S); i < issued; ++i)
                ptx::mbar_wait(&full[i % S], (uint32_t)((i / S) & 1), 1u << 20);
        }
        __syncwarp();
        __syncthreads();
    }
}

// One CTA per query row: thread 0 lists the partial slots of the CTAs whose
// range covers the row (in shared memory), then each thread merges 4 channels.
__global__ void xattn_combine_kernel(XaArgs a, void* out, int out_fmt) {
    pdl_launch();  // the slot list below is plan arithmetic: it runs before the wait
    extern __shared__ int s_slot[];  // [G]
    __shared__ int s_n;
    const int W = a.W, H = a.H;
    const int tok = blockIdx.x;
    if (threadIdx.x == 0) {
        const int xa = tok * a.chunks, xb = xa + a.chunks - 1;
        int cc = (int)((unsigned)(xa * a.G) / (unsigned)a.total);
        while (cc + 1 < a.G && xa_bound(cc + 1, a.total, a.G) <= xa) ++cc;
        while (cc > 0 && xa_bound(cc, a.total, a.G) > xa) --cc;
        int n = 0;
        for (; cc < a.G && xa_bound(cc, a.total, a.G) <= xb; ++cc) {
            const int seg = tok - xa_bound(cc, a.total, a.G) / a.chunks;
            s_slot[n++] = cc * a.max_seg + seg;
        }
        s_n = n;
    }
    __syncthreads();
    pdl_wait();
    const int n = s_n;
    const size_t stride = (size_t)(W + 2 * H);
    for (int ch = 4 * threadIdx.x; ch < W; ch += 4 * blockDim.x) {
        const int hh = ch / XA_DH;
        float M = -INFINITY;
        for (int k = 0; k < n; ++k) M = fmaxf(M, a.ws[(size_t)s_slot[k] * stride + W + hh]);
        float L = 0.0f;
        float4 O = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int k = 0; k < n; ++k) {
            const float* p = a.ws + (size_t)s_slot[k] * stride;
            const float ms = p[W + hh];
            const float w = ms == -INFINITY ? 0.0f : __expf(ms - M);
            L += p[W + H + hh] * w;
            const float4 v = *reinterpret_cast<const float4*>(p + ch);
            O.x += v.x * w; O.y += v.y * w; O.z += v.z * w; O.w += v.w * w;
        }
        const float inv = 1.0f / L;
        const float r[4] = {O.x * inv, O.y * inv, O.z * inv, O.w * inv};
        const int64_t i = (int64_t)tok * W + ch;
        if (out_fmt == 0) {
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + i) = make_float4(r[0], r[1], r[2], r[3]);
        } else {
            __half* o = reinterpret_cast<__half*>(out) + i;
#pragma unroll
            for (int e = 0; e < 4; e += 2) {
                const __half2 hi = __floats2half2_rn(r[e], r[e + 1]);
                *reinterpret_cast<__half2*>(o + e) = hi;
                if (out_fmt == 2) {
                    const float2 hf = __half22float2(hi);
                    *reinterpret_cast<__half2*>(o + (int64_t)a.n_tok * W + e) = __floats2half2_rn(r[e] - hf.x, r[e + 1] - hf.y);
                }
            }
        }
    }
}

static int xa_keys(bool f16) { return f16 ? XA_T16 : XA_T; }
static int xa_stage_bytes(int W, bool f16) { return f16 ? 2 * XA_T16 * W * 2 : 2 * XA_T * (W + W / 16); }
static int xa_stages(int W, bool f16) {
    const int extra = xa_keys(f16) * (W / 32) * 4 + 2 * XA_MAX_STAGES * 8;
    return std::min(XA_MAX_STAGES, (XA_SMEM_BUDGET - extra) / xa_stage_bytes(W, f16));
}

XaPlan xattn_q8_plan(const vkb_context* ctx, int n_tok, int n_head, int d_head, int n_ctx, const float* q,
                     const void* k, const void* v, const void* ks, const void* vs, size_t ws_cap_floats, bool f16) {
    XaPlan p;
    const int W = n_head * d_head;
    if (d_head != XA_DH || W % 256 || (W + 2 * n_head) % 4 || 16 * n_head + 32 > 512 || n_tok <= 0 || n_ctx <= 0) return p;
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)ks | (uintptr_t)vs) & 15) return p;
    if (xa_stages(W, f16) < 2) return p;
    const int chunks = (n_ctx + xa_keys(f16) - 1) / xa_keys(f16);
    const int64_t total = (int64_t)n_tok * chunks;
    if (total * ctx->sm_count >= (int64_t(1) << 31)) return p;
    int G = (int)std::min<int64_t>(ctx->sm_count, total);
    auto ws_floats = [&](int g, int* ms) {
        const int64_t per = (total + g - 1) / g;
        *ms = (int)((per + chunks - 1) / chunks + 1);
        return (size_t)g * *ms * (W + 2 * n_head);
    };
    int max_seg = 0;
    size_t need = ws_floats(G, &max_seg);
    while (ws_cap_floats && need > ws_cap_floats && G > 1) {
        G = std::max(1, G / 2);
        need = ws_floats(G, &max_seg);
    }
    if (ws_cap_floats && need > ws_cap_floats) return p;
    p.ok = true;
    p.f16 = f16;
    p.G = G;
    p.max_seg = max_seg;
    p.ws_floats = need;
    return p;
}

void run_xattn_q8(vkb_context* ctx, const XaPlan& plan, int n_tok, int n_head, int n_ctx, const float* q,
                  const int32_t* seq_of_tok, const void* k, const void* v, const void* ks, const void* vs, void* out,
                  int out_fmt, float* ws, bool kv_ready) {
    const int W = n_head * XA_DH;
    XaArgs a;
    a.kv_ready = kv_ready ? 1 : 0;
    a.q = q;
    a.seq_of_tok = seq_of_tok;
    a.kq = reinterpret_cast<const int8_t*>(k);
    a.kd = reinterpret_cast<const __half*>(ks);
    a.vq = reinterpret_cast<const int8_t*>(v);
    a.vd = reinterpret_cast<const __half*>(vs);
    a.n_tok = n_tok;
    a.n_ctx = n_ctx;
    a.H = n_head;
    a.W = W;
    const bool f16 = plan.f16;
    a.chunks = (n_ctx + xa_keys(f16) - 1) / xa_keys(f16);
    a.total = n_tok * a.chunks;
    a.G = plan.G;
    a.max_seg = plan.max_seg;
    a.S = xa_stages(W, f16);
    a.ws = ws;

    a.err = ctx->err_flag.as<int>();
    const size_t smem =
        (size_t)a.S * xa_stage_bytes(W, f16) + (size_t)xa_keys(f16) * (W / 32) * 4 + (size_t)a.S * 16;
    if (f16) {
        smem_optin(xattn_q8_kernel<true>, XA_SMEM_BUDGET);
        launch_pdl(ctx, xattn_q8_kernel<true>, plan.G, 16 * n_head + 32, smem, a);
    } else {
        smem_optin(xattn_q8_kernel<false>, XA_SMEM_BUDGET);
        launch_pdl(ctx, xattn_q8_kernel<false>, plan.G, 16 * n_head + 32, smem, a);
    }
    VKB_CUDA(cudaGetLastError());
    ctx->count();
    launch_pdl(ctx, xattn_combine_kernel, (unsigned)n_tok, std::min(256, W / 4), (size_t)plan.G * sizeof(int), a, out, out_fmt);
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}

}  // namespace vkb
