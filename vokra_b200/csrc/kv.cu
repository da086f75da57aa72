// kv.cu — the paged quantized KV cache on the device, its host page allocator,
// the bit-exact Q8_0 append kernel, decode attention over the pages, dense
// (cross-) attention, and the KvQuantDequantGemvOps arm.
//
// Host allocator semantics follow QuantizedPagedKvCache
// (crates/vokra-core/src/cache/paged_quant.rs:152-560): the arena is allocated
// up front, the free list is LIFO and initially pops 0, 1, 2, ..., pages are
// acquired on first touch in (layer, token) order, reset zeroes every page
// and rebuilds the free list, release_layer zeroes and frees one layer.
//
// Device page storage keeps the quants and the f16 scales of each token row in
// separate planes ("split planes"): row r of an arena has qrow quant bytes at
// q + r*qrow (Q8_0: W int8; Q4_0 and Q5_0: W/2 bytes of pair-packed low
// nibbles; FP32: 4W bytes of values), for Q5_0 W/8 bytes of 5th bits at
// h + r*(W/8), and W/32 f16 scales at d + r*(W/32). A row is one (token, stream) slot:
// REFERENCE layout rows are ((page*bs + offset)*n_stream + stream); SEQUENCE
// layout rows are (layer*n_pages + page)*bs + offset. vkb_kv_read_page
// reassembles the reference's 34-byte on-wire blocks from the two planes.
#include "common.cuh"
#include "attn_core.cuh"
#include "kv.cuh"
#include "xattn.cuh"
#include <cstdlib>
#include <algorithm>

using namespace vkb;

struct vkb_kv_pool {
    vkb_context* ctx = nullptr;
    vkb_kv_pool_desc d{};
    int W = 0, row_blocks = 0, ppl = 0, ppseq = 0, rpp = 0, n_arena = 1;
    int qrow = 0, hrow = 0;          // bytes per row of the quant plane and of the Q5_0 high-bit plane
    int64_t n_pages = 0, table_len = 0;
    std::vector<int32_t> table;      // host mirror (-1 = empty)
    std::vector<int32_t> free_list;  // LIFO
    std::vector<int32_t> refs;       // SEQUENCE layout: streams whose table holds each page (beams share pages)
    // device
    DevBuf kq, kd, vq, vd;           // arena planes: quants (or f32 values), f16 scales
    DevBuf kh, vh;                   // Q5_0 5th-bit planes
    DevBuf table_dev;
    DevBuf rows_dev;                 // int64 [n_layer][max_step]: row of each step token per layer
    DevBuf groups_dev;               // AttnGroup [max_groups]
    DevBuf part_dev;                 // split partials of the attention
    DevBuf pairs_dev;                // (source, destination) pages of a stream copy
    int max_step = 0;
    // pinned staging
    int32_t* h_table = nullptr;
    int64_t* h_rows = nullptr;
    AttnGroup* h_groups = nullptr;
    cudaEvent_t staged = nullptr;
    bool staged_pending = false;
    // current step
    int n_tok = 0, n_groups = 0, maxq = 1, splits = 1, max_keys = 0;
    std::vector<int32_t> step_seq, step_pos;
    int64_t rows_in_arena() const { return n_pages * rpp; }
    int srow_bytes() const { return d.mode == VKB_KV_FP32 ? 0 : row_blocks * 2; }
    // on-wire bytes of one token row (the reference's block encoding; f32 values for FP32)
    int wire_row_bytes() const {
        return d.mode == VKB_KV_FP32 ? 4 * W : row_blocks * (d.mode == VKB_KV_Q8_0 ? 34 : d.mode == VKB_KV_Q5_0 ? 22 : 18);
    }
};

namespace vkb {

// ---------------------------------------------------------------------------
// Append: one warp per 32-element block; the arithmetic of BlockQ8_0::pack
// (crates/vokra-core/src/kv_quant/q8_0.rs:40-66) in IEEE fp32 with Rust's
// NaN rules (max ignores NaN, clamp keeps NaN, NaN casts to 0).
// ---------------------------------------------------------------------------

template <int MODE>
__global__ void kv_append_kernel(const float* __restrict__ k, const float* __restrict__ v, int64_t ld,
                                 const int64_t* __restrict__ rows, int n_tok, int W, int qrow, int hrow, uint8_t* kq,
                                 __half* kd, uint8_t* kh, uint8_t* vq, __half* vd, uint8_t* vh) {
    pdl_entry();
    const int nb = W / 32;
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= (int64_t)n_tok * nb * 2) return;
    const int is_v = (int)(gw / ((int64_t)n_tok * nb));
    const int64_t rem = gw % ((int64_t)n_tok * nb);
    const int tok = (int)(rem / nb), b = (int)(rem % nb);
    const float x = ((is_v ? v : k) + (int64_t)tok * ld + b * 32)[lane];
    const int64_t row = rows[tok];
    uint8_t* q = (is_v ? vq : kq) + row * qrow;
    __half* d = (is_v ? vd : kd) + row * nb + b;
    if constexpr (MODE == VKB_KV_Q8_0) {
        q8_0_block_warp(x, lane, reinterpret_cast<int8_t*>(q) + b * 32, d);
    } else if constexpr (MODE == VKB_KV_Q4_0) {
        q4_0_block_warp(x, lane, q + b * 16, d);
    } else if constexpr (MODE == VKB_KV_Q5_0) {
        q5_0_block_warp(x, lane, q + b * 16, (is_v ? vh : kh) + row * hrow + b * 4, d);
    } else {
        reinterpret_cast<float*>(q)[b * 32 + lane] = x;
    }
}

// ---------------------------------------------------------------------------
// Fused decode self-attention (one query per stream, SEQUENCE layout, d_head
// 64): one CTA of 64 x HG threads per (stream, group of HG heads = 64 x HG channels; HG = 2 or 4).
// Before waiting for the QKV projection it looks up the key rows and requests
// their K and V bytes into L2; then it appends the step's K/V for its channels
// (the bit-exact BlockQ8_0::pack of kv_append_kernel) and attends over every
// key of the stream without key splits, so no partials and no combine launch:
//   scores  thread (head h = t/64, key slot t%64): 64 int8 K of the key
//           converted exactly, dotted with q (shared memory), x block scales
//   softmax one warp per head over the scores in shared memory
//   P.V     thread = (16 channels, key group); 16 bytes of V per key, its
//           block scale, p; the 16 key groups summed in shared memory
// ---------------------------------------------------------------------------
// With splits > 0 the q|k|v row is read from the QKV projection's split-K
// partials [splits][n_tok][ld] instead: value = (sum of partials in split
// order + bias) x (qscale for the q columns), the reduce kernel's epilogue.
template <int HG>
__global__ void __launch_bounds__(64 * HG) paged_decode_kernel(
    const float* __restrict__ qkv, int64_t ld, const float* __restrict__ part, int splits, int64_t plane,
    const float* __restrict__ bias, float qscale,
    const AttnGroup* __restrict__ groups, const int64_t* __restrict__ new_rows, const int32_t* __restrict__ table,
    int ppseq, int64_t arena_row0, int bs, int8_t* kq, __half* kd, int8_t* vq, __half* vd, int W, int max_keys,
    void* out, int out_fmt, int64_t out_plane) {
    pdl_launch();
    constexpr int NT = 64 * HG;  // threads = channels of the group
    constexpr int KP = NT / 128; // 128-byte pieces of a key's K (or V) row in the group
    extern __shared__ __align__(16) float pd_smem[];
    float* sc = pd_smem;                               // [HG][max_keys]; later the [16][NT] P.V sums
    float* qs = sc + (HG * max_keys > 16 * NT ? HG * max_keys : 16 * NT);  // [NT]
    int64_t* rows_s = reinterpret_cast<int64_t*>(qs + NT);                // [max_keys]
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    // The query groups, the rows of the new keys and the page table come from
    // host copies that precede the step, so the key rows are looked up, and
    // the K and V bytes of every key (this group's 64 * HG channels and their
    // scales) requested into L2, while the QKV projection still runs; an L2
    // prefetch is correct whatever writes those bytes.
    const AttnGroup g = groups[blockIdx.x];
    const int tok = g.first_tok, n_keys = g.pos0 + 1;
    const int c0 = blockIdx.y * NT, nb = W / 32, b0 = c0 / 32;
    for (int k = t; k < n_keys; k += NT) {
        const int pid = table[g.seq * ppseq + k / bs];
        rows_s[k] = arena_row0 + (int64_t)pid * bs + k % bs;
    }
    __syncthreads();
    constexpr int PP = 2 * KP + 2;  // L2 lines requested per key
    for (int i = t; i < PP * n_keys; i += NT) {
        const int64_t row = rows_s[i / PP];
        const int pt = i % PP;
        const void* pp = pt < KP           ? static_cast<const void*>(kq + row * W + c0 + 128 * pt)
                         : pt == KP        ? static_cast<const void*>(kd + row * nb + b0)
                         : pt < 2 * KP + 1 ? static_cast<const void*>(vq + row * W + c0 + 128 * (pt - KP - 1))
                                           : static_cast<const void*>(vd + row * nb + b0);
        asm volatile("prefetch.global.L2 [%0];" ::"l"(pp));
    }
    // the projection's bias (model weights) before the wait as well
    const int ck = W + c0 + warp * 32 + lane, cv = 2 * W + c0 + warp * 32 + lane, cq = c0 + t;
    float bk = 0.0f, bv = 0.0f, bq = 0.0f;
    if (splits > 0 && bias) {
        bk = bias[ck];
        bv = bias[cv];
        bq = bias[cq];
    }
    pdl_wait();
    // phase 0: this token's K, V (warp w: block w of the group) and q columns; from split-K
    // partials the three sums' loads are issued together, each summed in split order
    float xk, xv, xq;
    {
        const int64_t r0 = (int64_t)tok * ld;
        if (splits == 0) {
            xk = qkv[r0 + ck];
            xv = qkv[r0 + cv];
            xq = qkv[r0 + cq];
        } else {
            float ak = 0.0f, av = 0.0f, aq = 0.0f;
#pragma unroll 4
            for (int sp = 0; sp < splits; ++sp) {
                const float* pp = part + sp * plane + r0;
                const float a = __ldcg(pp + ck), b = __ldcg(pp + cv), c = __ldcg(pp + cq);
                ak += a;
                av += b;
                aq += c;
            }
            xk = ak + bk;
            xv = av + bv;
            xq = (aq + bq) * qscale;
        }
    }
    // append this token's K and V blocks of the group
    {
        const int64_t row = new_rows[tok];
        q8_0_block_warp(xk, lane, kq + row * W + c0 + warp * 32, kd + row * nb + b0 + warp);
        q8_0_block_warp(xv, lane, vq + row * W + c0 + warp * 32, vd + row * nb + b0 + warp);
        qs[t] = xq;
    }
    __syncthreads();
    // phase 1: scores, two keys per iteration (their 8 loads issued together)
    {
        const int hl = t >> 6, slot = t & 63;
        const float* qh = qs + hl * 64;
        for (int k0 = slot; k0 < n_keys; k0 += 128) {
            uint4 kv4[2][4];
            __half2 s2[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int k = k0 + 64 * u;
                if (k < n_keys) {
                    const int64_t row = rows_s[k];
                    const uint4* kp = reinterpret_cast<const uint4*>(kq + row * W + c0 + hl * 64);
#pragma unroll
                    for (int i = 0; i < 4; ++i) kv4[u][i] = __ldcg(kp + i);
                    s2[u] = __ldcg(reinterpret_cast<const __half2*>(kd + row * nb + b0 + hl * 2));
                }
            }
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int k = k0 + 64 * u;
                if (k >= n_keys) break;
                float part[2] = {0.0f, 0.0f};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t w4[4] = {kv4[u][i].x ^ 0x80808080u, kv4[u][i].y ^ 0x80808080u,
                                            kv4[u][i].z ^ 0x80808080u, kv4[u][i].w ^ 0x80808080u};
#pragma unroll
                    for (int wd = 0; wd < 4; ++wd)
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const float kf =
                                __uint_as_float(__byte_perm(w4[wd], 0x4B000000u, 0x7440u + b)) - 8388736.0f;
                            part[i >> 1] = fmaf(qh[16 * i + 4 * wd + b], kf, part[i >> 1]);
                        }
                }
                sc[hl * max_keys + k] = part[0] * __low2float(s2[u]) + part[1] * __high2float(s2[u]);
            }
        }
    }
    __syncthreads();
    // phase 2: softmax per head (warps 0 .. HG - 1), p normalised in place
    if (warp < HG) {
        float* s = sc + warp * max_keys;
        float m = -INFINITY;
        for (int k = lane; k < n_keys; k += 32) m = fmaxf(m, s[k]);
        m = warp_max(m);
        float l = 0.0f;
        for (int k = lane; k < n_keys; k += 32) {
            const float e = __expf(s[k] - m);
            s[k] = e;
            l += e;
        }
        l = warp_sum(l);
        const float inv = 1.0f / l;
        for (int k = lane; k < n_keys; k += 32) s[k] *= inv;
    }
    __syncthreads();
    // phase 3: P.V; thread = (16-channel group t % 16, key group t / 16): one
    // 16-byte load of V per key over every 16th key (16 loads in flight per
    // 16 keys), the 16 key groups summed in shared memory
    {
        const int cg = t % (4 * HG), kg = t / (4 * HG);  // 16 key groups
        const float* p = sc + (cg >> 2) * max_keys;
        const int8_t* vcol = vq + c0 + 16 * cg;
        const __half* vdc = vd + b0 + (cg >> 1);
        float a[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) a[i] = 0.0f;
#pragma unroll 4
        for (int k = kg; k < n_keys; k += 16) {
            const int64_t row = rows_s[k];
            const uint4 v4 = __ldcg(reinterpret_cast<const uint4*>(vcol + row * W));
            const float w = p[k] * __half2float(__ldcg(vdc + row * nb));
            const uint32_t vw[4] = {v4.x ^ 0x80808080u, v4.y ^ 0x80808080u, v4.z ^ 0x80808080u, v4.w ^ 0x80808080u};
#pragma unroll
            for (int wd = 0; wd < 4; ++wd)
#pragma unroll
                for (int bb = 0; bb < 4; ++bb)
                    a[4 * wd + bb] = fmaf(w, __uint_as_float(__byte_perm(vw[wd], 0x4B000000u, 0x7440u + bb)) - 8388736.0f,
                                          a[4 * wd + bb]);
        }
        __syncthreads();  // the score rows are no longer read: reuse them for the key-group sums
        float* red = sc;  // [16][NT]
#pragma unroll
        for (int i = 0; i < 4; ++i)
            *reinterpret_cast<float4*>(red + kg * NT + 16 * cg + 4 * i) =
                make_float4(a[4 * i], a[4 * i + 1], a[4 * i + 2], a[4 * i + 3]);
        __syncthreads();
        float acc = 0.0f;
#pragma unroll
        for (int g2 = 0; g2 < 16; ++g2) acc += red[g2 * NT + t];
        const int64_t o = (int64_t)tok * W + c0 + t;
        if (out_fmt == 0) {
            reinterpret_cast<float*>(out)[o] = acc;
        } else {
            const __half hi = __float2half_rn(acc);
            reinterpret_cast<__half*>(out)[o] = hi;
            if (out_fmt == 2) reinterpret_cast<__half*>(out)[out_plane + o] = __float2half_rn(acc - __half2float(hi));
        }
    }
}

// Quantizes dense rows [n_rows][W] (row stride ld) into the two planes (same
// arithmetic). With a group map, source row r lands in destination row
// map[r / group] * group + r % group.
__global__ void quantize_rows_kernel(const float* __restrict__ x, int64_t ld, int64_t n_rows, int W, int8_t* q,
                                     __half* d, const int32_t* __restrict__ map, int group) {
    pdl_entry();
    // One thread per 32-element block: 8 float4 loads, then the BlockQ8_0::pack
    // arithmetic (the same expressions as q8_0_block_warp, sequentially).
    const int nb = W / 32;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n_rows * nb) return;
    const int64_t row = t / nb;
    const int b = (int)(t % nb);
    const float4* src = reinterpret_cast<const float4*>(x + row * ld + b * 32);
    float v[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float4 f = src[i];
        v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const float dd = amax == 0.0f ? 0.0f : amax / 127.0f;
    const float inv = dd == 0.0f ? 0.0f : 1.0f / dd;
    uint32_t packed[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        uint32_t wv = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float s = v[4 * i + e] * inv;
            float c = s < -127.0f ? -127.0f : (s > 127.0f ? 127.0f : s);
            int qv = isnan(c) ? 0 : (int)roundf(c);
            wv |= ((uint32_t)(qv & 0xff)) << (8 * e);
        }
        packed[i] = wv;
    }
    const int64_t dst = map ? (int64_t)map[row / group] * group + row % group : row;
    uint4* qo = reinterpret_cast<uint4*>(q + dst * W + b * 32);
    qo[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    qo[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
    *reinterpret_cast<uint16_t*>(d + dst * nb + b) = f32_to_f16_bits(dd);
}

// ---------------------------------------------------------------------------
// Attention kernels
// ---------------------------------------------------------------------------
// Key splits are fixed per launch (n_splits); each CTA derives its key range
// from its group's key count, so the launch shape does not depend on the step.
template <class FP, int MAXQ>
__global__ void __launch_bounds__(ATTN_MAX_THREADS, MAXQ > 1 ? 1 : 2) paged_attn_kernel(FP f, const float* __restrict__ q, int64_t q_ld, const AttnGroup* __restrict__ groups,
                                  int n_head, int d_head, int n_splits, void* ctx_out,
                                  int out_fmt, float* ws, int per_seq_base, int ppseq, int64_t out_plane) {
    pdl_entry();
    const AttnGroup g = groups[blockIdx.x];
    const int split = blockIdx.y;
    const int n_keys = g.pos0 + g.n_q;  // keys 0 .. last query's position
    const int kps = (n_keys + n_splits - 1) / n_splits;
    const int kb = min(n_keys, split * kps);
    const int ke = min(n_keys, kb + kps);
    FP ff = f;
    if (per_seq_base) ff.table_base = g.seq * ppseq;
    else ff.slot = g.seq;
    attn_body<FP, MAXQ>(ff, q, q_ld, g, n_head, d_head, f.W, kb, ke, split, n_splits, ctx_out,
                                  out_fmt, out_plane, ws);
}

template <class F>
__global__ void __launch_bounds__(ATTN_MAX_THREADS, 2) dense_attn_kernel(F f, const float* __restrict__ q, const int32_t* __restrict__ seq_of_tok, int n_ctx,
                                  int n_head, int d_head, int keys_per_split, int n_splits, void* ctx_out,
                                  int out_fmt, float* ws, int64_t out_plane) {
    pdl_entry();
    AttnGroup g;
    g.first_tok = blockIdx.x;
    g.n_q = 1;
    g.seq = seq_of_tok[blockIdx.x];
    g.pos0 = n_ctx;  // non-causal: every key is visible
    const int split = blockIdx.y;
    const int kb = split * keys_per_split;
    const int ke = min(n_ctx, kb + keys_per_split);
    F ff = f;
    ff.seq_row0 = (int64_t)g.seq * n_ctx;
    attn_body<F, 1>(ff, q, (int64_t)f.W, g, n_head, d_head, f.W, kb, max(kb, ke), split, n_splits, ctx_out, out_fmt,
                    out_plane, ws);
}

__global__ void attn_combine_kernel(const float* __restrict__ ws, int n_tok, int n_splits, int n_head, int d_head,
                                    void* ctx_out, int out_fmt) {
    pdl_entry();
    const int W = n_head * d_head;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)n_tok * W) return;
    const int tok = (int)(i / W), c = (int)(i % W), h = c / d_head;
    const float* base = ws + (size_t)tok * n_splits * (W + 2 * n_head);
    float M = -INFINITY;
    for (int s = 0; s < n_splits; ++s) M = fmaxf(M, base[(size_t)s * (W + 2 * n_head) + W + h]);
    float L = 0.0f, O = 0.0f;
    for (int s = 0; s < n_splits; ++s) {
        const float* p = base + (size_t)s * (W + 2 * n_head);
        float ms = p[W + h];
        float w = ms == -INFINITY ? 0.0f : __expf(ms - M);
        L += p[W + n_head + h] * w;
        O += p[c] * w;
    }
    float v = O / L;
    if (out_fmt == 0) {
        reinterpret_cast<float*>(ctx_out)[i] = v;
    } else {
        __half hi = __float2half_rn(v);
        reinterpret_cast<__half*>(ctx_out)[i] = hi;
        if (out_fmt == 2) reinterpret_cast<__half*>(ctx_out)[(int64_t)n_tok * W + i] = __float2half_rn(v - __half2float(hi));
    }
}

// Thread shape of the attention CTA: R row-groups of W/16 threads with
// R*W/16 a multiple of 32 and at most ATTN_MAX_THREADS threads.
static int attn_rowgroups(int W, int maxq = 1) {
    const int limit = ATTN_MAX_THREADS;
    int tpr = W / 16;
    int best = 0;
    for (int R = 1; R * tpr <= limit; ++R)
        if ((R * tpr) % 32 == 0) best = R;
    if (!best) fail(VKB_ERROR_UNSUPPORTED_OP, "attention: n_head*d_head=" + std::to_string(W) + " has no thread shape");
    return best;
}

static void check_heads(int n_head, int d_head) {
    if (n_head <= 0 || d_head <= 0) fail(VKB_ERROR_INVALID_ARGUMENT, "attention: bad head shape");
    if (d_head % 16 || d_head > 512 || (d_head / 16) & (d_head / 16 - 1))
        fail(VKB_ERROR_UNSUPPORTED_OP, "attention: d_head must be 16 x a power of two (got " +
                                           std::to_string(d_head) + ")");
    if ((n_head * d_head) % 32) fail(VKB_ERROR_UNSUPPORTED_OP, "attention: n_head*d_head must be a multiple of 32");
}

// Dense attention (cross-attention): launch helper shared with the session.
void run_dense_attention(vkb_context* ctx, int n_tok, int n_head, int d_head, const float* q, const int32_t* seq_of_tok,
                         const void* k, const void* v, const void* k_scale, const void* v_scale, int n_ctx,
                         int kv_fmt, void* out, int out_dtype, float* ws_override, size_t ws_cap_floats,
                         bool kv_ready) {
    check_heads(n_head, d_head);
    const int W = n_head * d_head;
    {
        // the streaming kernel for both stores (Q8_0 rows + scales, or f16 rows);
        // VKB_XATTN_ROWGROUPS selects the row-group kernel below instead
        static const bool old_path = std::getenv("VKB_XATTN_ROWGROUPS") != nullptr;
        XaPlan xp = old_path ? XaPlan{} : xattn_q8_plan(ctx, n_tok, n_head, d_head, n_ctx, q, k, v, k_scale, v_scale,
                                                        ws_cap_floats, kv_fmt == VKB_DT_F16);
        if (xp.ok) {
            float* ws = ws_override;
            if (!ws) {
                ctx->ensure_workspace(xp.ws_floats * sizeof(float));
                ws = ctx->workspace.as<float>();
            }
            run_xattn_q8(ctx, xp, n_tok, n_head, n_ctx, q, seq_of_tok, k, v, k_scale, v_scale, out, out_dtype, ws,
                         kv_ready);
            return;
        }
    }
    const int R = attn_rowgroups(W);
    // Splits: about 8 CTAs per SM overall, at least 4*R keys per split.
    int splits = std::max(1, std::min((8 * ctx->sm_count + n_tok - 1) / n_tok, n_ctx / (4 * R)));
    if (ws_cap_floats) {  // a caller-fixed scratch bounds the number of split partials
        const size_t per_split = (size_t)n_tok * (W + 2 * n_head);
        splits = (int)std::max<size_t>(1, std::min<size_t>((size_t)splits, ws_cap_floats / per_split));
    }
    int kps = (n_ctx + splits - 1) / splits;
    splits = (n_ctx + kps - 1) / kps;
    float* ws = nullptr;
    if (splits > 1) {
        if (ws_override) ws = ws_override;
        else {
            size_t bytes = (size_t)n_tok * splits * (W + 2 * n_head) * sizeof(float);
            ctx->ensure_workspace(bytes);
            ws = ctx->workspace.as<float>();
        }
    }
    size_t sm = attn_smem_bytes(R, 1, W, n_head);
    dim3 grid((unsigned)n_tok, (unsigned)splits);
    const int threads = R * (W / 16);
    if (kv_fmt == VKB_DT_F16) {
        FetchDenseF16 f{reinterpret_cast<const __half*>(k), reinterpret_cast<const __half*>(v), W, 0};
        smem_optin(dense_attn_kernel<FetchDenseF16>, 200 * 1024);
        launch_pdl(ctx, dense_attn_kernel<FetchDenseF16>, grid, threads, sm, f, q, seq_of_tok, n_ctx, n_head, d_head, kps,
                                                                            splits, out, out_dtype, ws, (int64_t)n_tok * W);
    } else {
        FetchDenseQ8 f{reinterpret_cast<const int8_t*>(k), reinterpret_cast<const __half*>(k_scale),
                       reinterpret_cast<const int8_t*>(v), reinterpret_cast<const __half*>(v_scale), W, 0};
        smem_optin(dense_attn_kernel<FetchDenseQ8>, 200 * 1024);
        launch_pdl(ctx, dense_attn_kernel<FetchDenseQ8>, grid, threads, sm, f, q, seq_of_tok, n_ctx, n_head, d_head, kps,
                                                                           splits, out, out_dtype, ws, (int64_t)n_tok * W);
    }
    VKB_CUDA(cudaGetLastError());
    ctx->count();
    if (splits > 1) {
        int64_t tot = (int64_t)n_tok * W;
        launch_pdl(ctx, attn_combine_kernel, (unsigned)((tot + 255) / 256), 256, 0, ws, n_tok, splits, n_head, d_head,
                                                                                   out, out_dtype);
        VKB_CUDA(cudaGetLastError());
        ctx->count();
    }
}

void run_quantize_rows(vkb_context* ctx, const float* x, int64_t ld, int64_t n_rows, int W, int8_t* q, __half* d,
                       const int32_t* map, int group) {
    if (W % 32) fail(VKB_ERROR_INVALID_ARGUMENT, "quantize_rows: row width must be a multiple of 32");
    if (ld % 4 || ((uintptr_t)x & 15)) fail(VKB_ERROR_INVALID_ARGUMENT, "quantize_rows: rows must be 16-byte aligned");
    int64_t blocks = n_rows * (W / 32);
    launch_pdl(ctx, quantize_rows_kernel, (unsigned)((blocks + 255) / 256), 256, 0, x, ld, n_rows, W, q, d, map, group);
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}

// ---------------------------------------------------------------------------
// Host side of the pool
// ---------------------------------------------------------------------------
vkb_kv_pool* kv_pool_create(vkb_context* ctx, const vkb_kv_pool_desc* desc) {
    if (!ctx || !desc) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_pool_create: null argument");
    const vkb_kv_pool_desc& d = *desc;
    // The reference's QuantizedPagedKvCache takes the quantized modes only;
    // FP32 pages exist here in the SEQUENCE layout, as the dense f32 cache the
    // reference's Whisper decoder keeps (whisper/decoder.rs:183-200).
    if (d.mode == VKB_KV_FP32 && d.layout != VKB_KV_LAYOUT_SEQUENCE)
        fail(VKB_ERROR_INVALID_ARGUMENT, "kv_pool_create: mode=Fp32 — the paged quant cache needs a quantized mode");
    if (d.mode != VKB_KV_FP32 && d.mode != VKB_KV_Q4_0 && d.mode != VKB_KV_Q5_0 && d.mode != VKB_KV_Q8_0)
        fail(VKB_ERROR_INVALID_ARGUMENT, "kv_pool_create: unknown mode " + std::to_string(d.mode));
    if (d.n_layer <= 0 || d.n_head <= 0 || d.d_head <= 0 || d.n_stream <= 0 || d.n_codebook <= 0 || d.max_time <= 0)
        fail(VKB_ERROR_INVALID_ARGUMENT, "kv_pool_create: every axis must be > 0");
    if ((d.n_head * d.d_head) % 32) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_pool_create: n_head*d_head not a multiple of 32");
    if (d.n_codebook != 1) fail(VKB_ERROR_UNSUPPORTED_OP, "kv_pool_create: n_codebook must be 1 on the device");
    if (d.page_tokens != 2 && d.page_tokens != 4 && d.page_tokens != 16)
        fail(VKB_ERROR_INVALID_ARGUMENT, "kv_pool_create: page_tokens must be 2, 4 or 16");
    if (d.layout != VKB_KV_LAYOUT_REFERENCE && d.layout != VKB_KV_LAYOUT_SEQUENCE)
        fail(VKB_ERROR_INVALID_ARGUMENT, "kv_pool_create: bad layout");
    check_heads(d.n_head, d.d_head);
    auto* p = new vkb_kv_pool();
    try {
        p->ctx = ctx;
        p->d = d;
        p->W = d.n_head * d.d_head;
        p->row_blocks = p->W / 32;
        p->qrow = d.mode == VKB_KV_Q8_0 ? p->W : d.mode == VKB_KV_FP32 ? 4 * p->W : p->W / 2;
        p->hrow = d.mode == VKB_KV_Q5_0 ? p->W / 8 : 0;
        if (d.layout == VKB_KV_LAYOUT_REFERENCE) {
            p->ppl = (d.max_time + d.page_tokens - 1) / d.page_tokens;
            p->n_pages = (int64_t)p->ppl * d.n_layer;  // paged_quant.rs:300 total_pages
            if (d.n_pages > 0 && d.n_pages != p->n_pages)
                fail(VKB_ERROR_INVALID_ARGUMENT, "kv_pool_create: the reference layout sizes its own arena");
            p->rpp = d.page_tokens * d.n_stream;
            p->table_len = p->n_pages;
            p->n_arena = 1;
        } else {
            p->ppseq = (d.max_time + d.page_tokens - 1) / d.page_tokens;
            p->n_pages = d.n_pages > 0 ? d.n_pages : (int64_t)p->ppseq * d.n_stream;
            p->rpp = d.page_tokens;
            p->table_len = (int64_t)p->ppseq * d.n_stream;
            p->n_arena = d.n_layer;
        }
        p->table.assign(p->table_len, -1);
        for (int64_t i = p->n_pages - 1; i >= 0; --i) p->free_list.push_back((int32_t)i);
        p->refs.assign(p->n_pages, 0);
        const int64_t rows = (int64_t)p->n_arena * p->n_pages * p->rpp;
        VKB_CUDA(cudaSetDevice(ctx->device));
        const size_t sbytes = d.mode == VKB_KV_FP32 ? 0 : (size_t)p->row_blocks * 2;
        for (DevBuf* b : {&p->kq, &p->vq}) b->alloc((size_t)rows * p->qrow);
        for (DevBuf* b : {&p->kd, &p->vd}) b->alloc((size_t)rows * sbytes);
        for (DevBuf* b : {&p->kh, &p->vh}) b->alloc((size_t)rows * p->hrow);
        for (DevBuf* b : {&p->kq, &p->vq, &p->kd, &p->vd, &p->kh, &p->vh})
            if (b->n) VKB_CUDA(cudaMemsetAsync(b->p, 0, b->n, ctx->stream));
        p->table_dev.alloc((size_t)p->table_len * 4);
        // page copies of one call: a stream's pages (copy_stream) or one per step token (copy-on-write)
        p->pairs_dev.alloc((size_t)std::max<int64_t>(p->ppseq, std::max(2048, d.n_stream * 8)) * sizeof(int2));
        p->max_step = std::max(2048, d.n_stream * 8);  // tokens per step (prefills)
        p->rows_dev.alloc((size_t)d.n_layer * p->max_step * 8);
        p->groups_dev.alloc((size_t)p->max_step * sizeof(AttnGroup));
        // Partials: up to 4096 CTAs x 4 queries of (W + 2H) floats.
        p->part_dev.alloc((size_t)4096 * 4 * (p->W + 2 * d.n_head) * sizeof(float));
        VKB_CUDA(cudaMallocHost(&p->h_table, (size_t)p->table_len * 4));
        VKB_CUDA(cudaMallocHost(&p->h_rows, (size_t)d.n_layer * p->max_step * 8));
        VKB_CUDA(cudaMallocHost(&p->h_groups, (size_t)p->max_step * sizeof(AttnGroup)));
        VKB_CUDA(cudaEventCreateWithFlags(&p->staged, cudaEventDisableTiming));
        std::fill(p->h_table, p->h_table + p->table_len, -1);
        VKB_CUDA(cudaMemcpyAsync(p->table_dev.p, p->h_table, p->table_dev.n, cudaMemcpyHostToDevice, ctx->stream));
        VKB_CUDA(cudaStreamSynchronize(ctx->stream));
    } catch (...) {
        delete p;
        throw;
    }
    return p;
}

void kv_pool_destroy(vkb_kv_pool* p) {
    if (!p) return;
    if (p->ctx) cudaStreamSynchronize(p->ctx->stream);
    if (p->h_table) cudaFreeHost(p->h_table);
    if (p->h_rows) cudaFreeHost(p->h_rows);
    if (p->h_groups) cudaFreeHost(p->h_groups);
    if (p->staged) cudaEventDestroy(p->staged);
    delete p;
}

static int32_t acquire(vkb_kv_pool* p) {
    if (p->free_list.empty())
        fail(VKB_ERROR_KV_CACHE_EXHAUSTED, "paged KV cache exhausted: arena has " + std::to_string(p->n_pages) +
                                               " pages, " + std::to_string(p->n_pages) + " in use");
    int32_t id = p->free_list.back();
    p->free_list.pop_back();
    p->refs[id] = 1;
    return id;
}

// One table entry lets go of its page; the page returns to the free list when
// no stream holds it any more.
static void drop(vkb_kv_pool* p, int32_t id) {
    if (--p->refs[id] <= 0) {
        p->refs[id] = 0;
        p->free_list.push_back(id);
    }
}

static void copy_pages(vkb_kv_pool* p, const std::vector<int2>& pairs);

static int64_t row_of(const vkb_kv_pool* p, int layer, int t, int s) {
    const int bs = p->d.page_tokens;
    if (p->d.layout == VKB_KV_LAYOUT_REFERENCE) {
        int32_t pid = p->table[(int64_t)layer * p->ppl + t / bs];
        if (pid < 0) return -1;
        return ((int64_t)pid * bs + t % bs) * p->d.n_stream + s;
    }
    int32_t pid = p->table[(int64_t)s * p->ppseq + t / bs];
    if (pid < 0) return -1;
    return ((int64_t)layer * p->n_pages + pid) * bs + t % bs;
}

static void wait_staging(vkb_kv_pool* p) {
    if (p->staged_pending) {
        VKB_CUDA(cudaEventSynchronize(p->staged));
        p->staged_pending = false;
    }
}

static void upload_table(vkb_kv_pool* p) {
    wait_staging(p);
    memcpy(p->h_table, p->table.data(), (size_t)p->table_len * 4);
    VKB_CUDA(cudaMemcpyAsync(p->table_dev.p, p->h_table, (size_t)p->table_len * 4, cudaMemcpyHostToDevice,
                             p->ctx->stream));
    VKB_CUDA(cudaEventRecord(p->staged, p->ctx->stream));
    p->staged_pending = true;
}

void kv_begin_step(vkb_kv_pool* p, int n_tok, const int32_t* seq, const int32_t* pos) {
    const auto& d = p->d;
    if (n_tok <= 0 || n_tok > p->max_step)
        fail(VKB_ERROR_INVALID_ARGUMENT, "kv_begin_step: n_tok must be in 1.." + std::to_string(p->max_step));
    if (!seq || !pos) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_begin_step: null arrays");
    for (int i = 0; i < n_tok; ++i) {
        if (seq[i] < 0 || seq[i] >= d.n_stream)
            fail(VKB_ERROR_INVALID_ARGUMENT, "stream " + std::to_string(seq[i]) + " >= n_stream " + std::to_string(d.n_stream));
        if (pos[i] < 0 || pos[i] >= d.max_time)
            fail(VKB_ERROR_INVALID_ARGUMENT, "t " + std::to_string(pos[i]) + " >= max_time " + std::to_string(d.max_time));
        if (i > 0 && seq[i] == seq[i - 1] && pos[i] != pos[i - 1] + 1)
            fail(VKB_ERROR_INVALID_ARGUMENT, "kv_begin_step: tokens of one stream must be consecutive positions");
    }
    wait_staging(p);
    // SEQUENCE layout: one page id serves every layer, acquired here in token
    // order. REFERENCE layout: pages are acquired lazily per layer by
    // vkb_kv_append, in the order the reference's append_step would
    // (paged_quant.rs:396-420).
    if (d.layout == VKB_KV_LAYOUT_SEQUENCE) {
        std::vector<int2> cow;
        for (int i = 0; i < n_tok; ++i) {
            int64_t idx = (int64_t)seq[i] * p->ppseq + pos[i] / d.page_tokens;
            if (p->table[idx] < 0) {
                p->table[idx] = acquire(p);
            } else if (p->refs[p->table[idx]] > 1) {
                // a page shared with another stream (a beam branch) is written:
                // this stream gets its own copy first (copy on write)
                const int32_t old = p->table[idx];
                p->table[idx] = acquire(p);
                cow.push_back(make_int2(old, p->table[idx]));
                drop(p, old);
            }
        }
        if (!cow.empty()) copy_pages(p, cow);
        memcpy(p->h_table, p->table.data(), (size_t)p->table_len * 4);
        for (int layer = 0; layer < d.n_layer; ++layer)
            for (int i = 0; i < n_tok; ++i) p->h_rows[(size_t)layer * n_tok + i] = row_of(p, layer, pos[i], seq[i]);
    }
    // Query groups: runs of one stream, at most 4 queries each.
    int ng = 0, maxq = 1, max_keys = 0;
    for (int i = 0; i < n_tok;) {
        int j = i + 1;
        while (j < n_tok && seq[j] == seq[i] && j - i < 4) ++j;
        AttnGroup g{i, j - i, seq[i], pos[i]};
        p->h_groups[ng++] = g;
        maxq = std::max(maxq, j - i);
        max_keys = std::max(max_keys, pos[j - 1] + 1);
        i = j;
    }
    cudaStream_t st = p->ctx->stream;
    if (d.layout == VKB_KV_LAYOUT_SEQUENCE) {
        VKB_CUDA(cudaMemcpyAsync(p->table_dev.p, p->h_table, (size_t)p->table_len * 4, cudaMemcpyHostToDevice, st));
        VKB_CUDA(cudaMemcpyAsync(p->rows_dev.p, p->h_rows, (size_t)d.n_layer * n_tok * 8, cudaMemcpyHostToDevice, st));
    }
    VKB_CUDA(cudaMemcpyAsync(p->groups_dev.p, p->h_groups, (size_t)ng * sizeof(AttnGroup), cudaMemcpyHostToDevice, st));
    VKB_CUDA(cudaEventRecord(p->staged, st));
    p->staged_pending = true;
    p->n_tok = n_tok;
    p->n_groups = ng;
    p->maxq = maxq;
    p->max_keys = max_keys;
    p->step_seq.assign(seq, seq + n_tok);
    p->step_pos.assign(pos, pos + n_tok);
    // Key splits: about 64 keys per split of the longest possible context, at
    // most ~8 CTAs per SM, and the partials must fit the pool's buffer. The
    // count depends only on the step's shape (not on its positions), so a
    // recorded step replays unchanged; each CTA computes its own key range.
    int splits = std::max(1, std::min((8 * p->ctx->sm_count + ng - 1) / ng, (d.max_time + 63) / 64));
    while ((int64_t)ng * splits > 4096 && splits > 1) --splits;
    p->splits = splits;
}

int pool_groups(const vkb_kv_pool* p) { return p->n_groups; }
int pool_maxq(const vkb_kv_pool* p) { return p->maxq; }
int pool_splits(const vkb_kv_pool* p) { return p->splits; }

void kv_append_ex(vkb_kv_pool* p, int layer, const float* k, const float* v, int64_t ld) {
    if (p->n_tok == 0) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_append: no step was begun");
    if (layer < 0 || layer >= p->d.n_layer) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_append: layer out of range");
    if (!k || !v) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_append: null k/v");
    if (p->d.layout == VKB_KV_LAYOUT_REFERENCE) {
        // Lazy per-layer acquisition, then upload this layer's table slice and
        // row list (disjoint staging slots per layer within a step).
        const int bs = p->d.page_tokens;
        for (int i = 0; i < p->n_tok; ++i) {
            int64_t idx = (int64_t)layer * p->ppl + p->step_pos[i] / bs;
            if (p->table[idx] < 0) p->table[idx] = acquire(p);
        }
        int32_t* ht = p->h_table + (size_t)layer * p->ppl;
        memcpy(ht, p->table.data() + (size_t)layer * p->ppl, (size_t)p->ppl * 4);
        int64_t* hr = p->h_rows + (size_t)layer * p->n_tok;
        for (int i = 0; i < p->n_tok; ++i) hr[i] = row_of(p, layer, p->step_pos[i], p->step_seq[i]);
        cudaStream_t st = p->ctx->stream;
        VKB_CUDA(cudaMemcpyAsync(p->table_dev.as<int32_t>() + (size_t)layer * p->ppl, ht, (size_t)p->ppl * 4,
                                 cudaMemcpyHostToDevice, st));
        VKB_CUDA(cudaMemcpyAsync(p->rows_dev.as<int64_t>() + (size_t)layer * p->n_tok, hr, (size_t)p->n_tok * 8,
                                 cudaMemcpyHostToDevice, st));
        VKB_CUDA(cudaEventRecord(p->staged, st));
        p->staged_pending = true;
    }
    const int64_t warps = (int64_t)p->n_tok * p->row_blocks * 2;
    const int64_t* rows = p->rows_dev.as<int64_t>() + (size_t)layer * p->n_tok;
    with_kv_mode(p->d.mode, [&](auto M) {
        launch_pdl(p->ctx, kv_append_kernel<decltype(M)::value>, (unsigned)((warps * 32 + 255) / 256), 256, 0, k, v,
                   ld, rows, p->n_tok, p->W, p->qrow, p->hrow, p->kq.as<uint8_t>(), p->kd.as<__half>(),
                   p->kh.as<uint8_t>(), p->vq.as<uint8_t>(), p->vd.as<__half>(), p->vh.as<uint8_t>());
    });
    VKB_CUDA(cudaGetLastError());
    p->ctx->count();
}

// Whether the decode step's append + attention of this pool runs as the fused
// paged_decode_kernel: one query per stream in the SEQUENCE layout, d_head 64,
// heads in groups of 4.
bool kv_decode_fused(const vkb_kv_pool* p) {
    static const bool off = std::getenv("VKB_DECODE_ATTN_SPLIT") != nullptr;
    const auto& d = p->d;
    return !off && p->n_tok > 0 && d.mode == VKB_KV_Q8_0 && d.layout == VKB_KV_LAYOUT_SEQUENCE && p->maxq == 1 &&
           p->n_groups == p->n_tok && d.d_head == 64 && d.n_head % 4 == 0;
}

// Append + attention of one decode step for one layer: the fused kernel when
// kv_decode_fused(p), else kv_append_ex + kv_attention_ex. `qkv` rows hold
// q | k | v (stride ld); with splits > 0 (fused path only) they are read from
// the projection's split-K partials with its bias and q scale.
void kv_append_attention_ex(vkb_kv_pool* p, int layer, const float* qkv, int64_t ld, void* out, int out_dtype,
                            const float* part, int splits, const float* bias, float qscale) {
    NvtxRange nvtx_range("vkb.kv.append_attention");
    const auto& d = p->d;
    if (layer < 0 || layer >= d.n_layer) fail(VKB_ERROR_INVALID_ARGUMENT, "decode attention: layer out of range");
    if (out_dtype != VKB_DT_F32 && out_dtype != VKB_DT_F16 && out_dtype != VKB_DT_F16X2)
        fail(VKB_ERROR_INVALID_ARGUMENT, "decode attention: bad out dtype");
    if (!kv_decode_fused(p)) {
        if (splits > 0) fail(VKB_ERROR_OTHER, "decode attention: partials need the fused kernel");
        kv_append_ex(p, layer, qkv + p->W, qkv + 2 * p->W, ld);
        kv_attention_ex(p, layer, qkv, ld, out, out_dtype);
        return;
    }
    const int max_keys = d.max_time;
    // heads per CTA: 2 (default: twice the CTAs of 4, half the channels each; decode step 4.080 vs
    // 4.097 ms at 64 streams, configs[2] 80.5 vs 82.4 us) or 4 (VKB_DECODE_HEADS=4)
    static const int hg = [] { const char* v = std::getenv("VKB_DECODE_HEADS"); return v && v[0] == '4' ? 4 : 2; }();
    const int nt = 64 * hg;
    const size_t smem = (size_t)(std::max(hg * max_keys, 16 * nt) + nt) * sizeof(float) + (size_t)max_keys * sizeof(int64_t);
    if (smem > 200 * 1024) fail(VKB_ERROR_UNSUPPORTED_OP, "decode attention: max_time too large");
    dim3 grid((unsigned)p->n_tok, (unsigned)(d.n_head / hg));
    auto kern = hg == 2 ? paged_decode_kernel<2> : paged_decode_kernel<4>;
    smem_optin(kern, 200 * 1024);
    launch_pdl(p->ctx, kern, grid, nt, smem, qkv, ld, part, splits, (int64_t)p->n_tok * ld, bias,
               qscale, p->groups_dev.as<AttnGroup>(), p->rows_dev.as<int64_t>() + (size_t)layer * p->n_tok,
               p->table_dev.as<int32_t>(), p->ppseq, (int64_t)layer * p->n_pages * p->rpp, d.page_tokens,
               p->kq.as<int8_t>(), p->kd.as<__half>(), p->vq.as<int8_t>(), p->vd.as<__half>(), p->W, max_keys, out,
               out_dtype, (int64_t)p->n_tok * p->W);
    VKB_CUDA(cudaGetLastError());
    p->ctx->count();
}

void kv_attention_ex(vkb_kv_pool* p, int layer, const float* q, int64_t q_ld, void* out, int out_dtype) {
    if (p->n_tok == 0) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_attention: no step was begun");
    if (layer < 0 || layer >= p->d.n_layer) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_attention: layer out of range");
    if (!q || !out) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_attention: null q/out");
    if (out_dtype != VKB_DT_F32 && out_dtype != VKB_DT_F16 && out_dtype != VKB_DT_F16X2)
        fail(VKB_ERROR_INVALID_ARGUMENT, "kv_attention: bad out dtype");
    const auto& d = p->d;
    const int W = p->W;
    const int R = attn_rowgroups(W, p->maxq);
    float* ws = p->part_dev.as<float>();
    with_kv_mode(d.mode, [&](auto M) {
        using FP = FetchPaged<decltype(M)::value>;
        FP f;
        f.kq = p->kq.as<uint8_t>();
        f.kd = p->kd.as<__half>();
        f.kh = p->kh.as<uint8_t>();
        f.vq = p->vq.as<uint8_t>();
        f.vd = p->vd.as<__half>();
        f.vh = p->vh.as<uint8_t>();
        f.table = p->table_dev.as<int32_t>();
        f.W = W;
        f.qrow = p->qrow;
        f.hrow = p->hrow;
        f.layout = d.layout;
        f.bs = d.page_tokens;
        int per_seq_base;
        if (d.layout == VKB_KV_LAYOUT_REFERENCE) {
            f.table_base = layer * p->ppl;
            f.n_sc = d.n_stream;
            f.slot = 0;
            f.arena_row0 = 0;
            per_seq_base = 0;
        } else {
            f.table_base = 0;
            f.n_sc = 1;
            f.slot = 0;
            f.arena_row0 = (int64_t)layer * p->n_pages * p->rpp;
            per_seq_base = 1;
        }
        dim3 grid((unsigned)p->n_groups, (unsigned)p->splits);
        const int threads = R * (W / 16);
        const int64_t oplane = (int64_t)p->n_tok * W;
        if (p->maxq == 1) {
            smem_optin(paged_attn_kernel<FP, 1>, 200 * 1024);
            launch_pdl(p->ctx, paged_attn_kernel<FP, 1>, grid, threads, attn_smem_bytes(R, 1, W, d.n_head), f, q, q_ld,
                       p->groups_dev.as<AttnGroup>(), d.n_head, d.d_head, p->splits, out, out_dtype, ws, per_seq_base,
                       p->ppseq, oplane);
        } else {
            smem_optin(paged_attn_kernel<FP, 4>, 200 * 1024);
            launch_pdl(p->ctx, paged_attn_kernel<FP, 4>, grid, threads, attn_smem_bytes(R, 4, W, d.n_head), f, q, q_ld,
                       p->groups_dev.as<AttnGroup>(), d.n_head, d.d_head, p->splits, out, out_dtype, ws, per_seq_base,
                       p->ppseq, oplane);
        }
    });
    const int of16 = out_dtype;  // 0 f32, 1 f16, 2 f16 hi+lo planes
    VKB_CUDA(cudaGetLastError());
    p->ctx->count();
    if (p->splits > 1) {
        int64_t tot = (int64_t)p->n_tok * W;
        launch_pdl(p->ctx, attn_combine_kernel, (unsigned)((tot + 255) / 256), 256, 0, ws, p->n_tok, p->splits,
                                                                                       d.n_head, d.d_head, out, of16);
        VKB_CUDA(cudaGetLastError());
        p->ctx->count();
    }
}

// Zeroes the device rows of one page (all layers' arenas for SEQUENCE layout).
// Copies whole pages of every layer (SEQUENCE layout): pair i = (source page,
// destination page); one CTA per (pair, layer), 16-byte moves of the K and V
// quants and scales of the page's rows.
__global__ void kv_copy_pages_kernel(const int2* __restrict__ pairs, int64_t n_pages, int bs, int qrow, int hrow,
                                     int srow, uint8_t* kq, uint8_t* kd, uint8_t* kh, uint8_t* vq, uint8_t* vd,
                                     uint8_t* vh) {
    pdl_entry();
    const int2 pr = pairs[blockIdx.x];
    const int64_t layer = blockIdx.y;
    const int64_t src = (layer * n_pages + pr.x) * bs, dst = (layer * n_pages + pr.y) * bs;
    auto move = [&](uint8_t* plane, int row_bytes) {
        if (!row_bytes) return;
        const uint4* from = reinterpret_cast<const uint4*>(plane + src * row_bytes);
        uint4* to = reinterpret_cast<uint4*>(plane + dst * row_bytes);
        const int n = bs * row_bytes / 16;
        for (int i = threadIdx.x; i < n; i += blockDim.x) to[i] = from[i];
    };
    move(kq, qrow);
    move(vq, qrow);
    move(kd, srow);
    move(vd, srow);
    move(kh, hrow);
    move(vh, hrow);
}

// Copies whole pages of every layer on the device: pair i = (source page,
// destination page), one launch of kv_copy_pages_kernel.
static void copy_pages(vkb_kv_pool* p, const std::vector<int2>& pairs) {
    if (pairs.empty()) return;
    if (p->pairs_dev.n < pairs.size() * sizeof(int2)) fail(VKB_ERROR_OTHER, "kv: too many page copies in one call");
    // pageable source: the copy is staged before cudaMemcpyAsync returns
    VKB_CUDA(cudaMemcpyAsync(p->pairs_dev.p, pairs.data(), pairs.size() * sizeof(int2), cudaMemcpyHostToDevice,
                             p->ctx->stream));
    dim3 grid((unsigned)pairs.size(), (unsigned)p->d.n_layer);
    launch_pdl(p->ctx, kv_copy_pages_kernel, grid, 256, 0, p->pairs_dev.as<int2>(), p->n_pages, p->d.page_tokens,
               p->qrow, p->hrow, p->srow_bytes(), p->kq.as<uint8_t>(), p->kd.as<uint8_t>(), p->kh.as<uint8_t>(),
               p->vq.as<uint8_t>(), p->vd.as<uint8_t>(), p->vh.as<uint8_t>());
    VKB_CUDA(cudaGetLastError());
    p->ctx->count();
}

// Makes stream dst a copy of the first n_pos positions of stream src (the
// per-beam branch of the self-attention cache; the reference deep-copies the
// host cache, whisper/decoder.rs:343-368). dst's own pages are let go; the
// pages src has filled completely are shared (reference counts, nothing is
// copied), only a partly filled last page is copied, in one launch. A later
// write into a shared page (a step at a position it holds) copies it first
// (kv_begin_step).
void kv_copy_stream(vkb_kv_pool* p, int src, int dst, int n_pos) {
    const auto& d = p->d;
    if (d.layout != VKB_KV_LAYOUT_SEQUENCE) fail(VKB_ERROR_INVALID_ARGUMENT, "copy_stream: sequence layout only");
    if (src < 0 || src >= d.n_stream || dst < 0 || dst >= d.n_stream)
        fail(VKB_ERROR_INVALID_ARGUMENT, "copy_stream: bad stream");
    if (n_pos < 0 || n_pos > d.max_time) fail(VKB_ERROR_INVALID_ARGUMENT, "copy_stream: bad position count");
    if (src == dst) return;
    if (d.page_tokens * p->srow_bytes() % 16 || d.page_tokens * p->hrow % 16 || d.page_tokens * p->qrow % 16)
        fail(VKB_ERROR_UNSUPPORTED_OP, "copy_stream: page planes not 16-byte sized");
    const int full = n_pos / d.page_tokens, n_pg = (n_pos + d.page_tokens - 1) / d.page_tokens;
    const int copied = n_pg - full;  // 0 or 1
    // Validate everything before touching dst, so a failed call leaves both
    // streams and the device page table as they were.
    size_t dst_freed = 0;
    for (int i = 0; i < p->ppseq; ++i) {
        const int32_t e = p->table[(int64_t)dst * p->ppseq + i];
        dst_freed += e >= 0 && p->refs[e] == 1;
    }
    for (int i = 0; i < n_pg; ++i)
        if (p->table[(int64_t)src * p->ppseq + i] < 0)
            fail(VKB_ERROR_INVALID_ARGUMENT, "copy_stream: source stream has no page for position " +
                                                 std::to_string(i * d.page_tokens));
    if (p->free_list.size() + dst_freed < (size_t)copied)
        fail(VKB_ERROR_KV_CACHE_EXHAUSTED, "copy_stream: " + std::to_string(copied) + " page needed, " +
                                               std::to_string(p->free_list.size() + dst_freed) + " free");
    // take src's pages first: dst may already share some of them
    for (int i = 0; i < full; ++i) ++p->refs[p->table[(int64_t)src * p->ppseq + i]];
    for (int i = 0; i < p->ppseq; ++i) {
        int32_t& e = p->table[(int64_t)dst * p->ppseq + i];
        if (e >= 0) {
            drop(p, e);
            e = -1;
        }
    }
    for (int i = 0; i < full; ++i) p->table[(int64_t)dst * p->ppseq + i] = p->table[(int64_t)src * p->ppseq + i];
    std::vector<int2> pairs;
    if (copied) {
        const int32_t sp = p->table[(int64_t)src * p->ppseq + full];
        const int32_t dp = acquire(p);
        p->table[(int64_t)dst * p->ppseq + full] = dp;
        pairs.push_back(make_int2(sp, dp));
    }
    upload_table(p);
    copy_pages(p, pairs);
}

static void zero_page(vkb_kv_pool* p, int32_t pid, int layer_for_seq) {
    cudaStream_t st = p->ctx->stream;
    const int64_t row0 = p->d.layout == VKB_KV_LAYOUT_REFERENCE ? (int64_t)pid * p->rpp
                                                                 : ((int64_t)layer_for_seq * p->n_pages + pid) * p->rpp;
    const int64_t nrows = p->rpp;
    for (int side = 0; side < 2; ++side) {
        VKB_CUDA(cudaMemsetAsync((side ? p->vq : p->kq).as<uint8_t>() + row0 * p->qrow, 0, (size_t)nrows * p->qrow, st));
        if (p->srow_bytes())
            VKB_CUDA(cudaMemsetAsync((side ? p->vd : p->kd).as<uint8_t>() + row0 * p->srow_bytes(), 0,
                                     (size_t)nrows * p->srow_bytes(), st));
        if (p->hrow)
            VKB_CUDA(cudaMemsetAsync((side ? p->vh : p->kh).as<uint8_t>() + row0 * p->hrow, 0, (size_t)nrows * p->hrow, st));
    }
}

// ---------------------------------------------------------------------------
// dequant GEMV (KvQuantDequantGemvOps): one warp per row, lanes over blocks.
// ---------------------------------------------------------------------------
template <int MODE>
__global__ void kv_dequant_gemv_kernel(const uint8_t* __restrict__ blocks, int64_t n_rows, int64_t nbpr,
                                       const float* __restrict__ x, float* __restrict__ y) {
    pdl_entry();
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= n_rows) return;
    constexpr int BB = MODE == VKB_KV_Q4_0 ? 18 : MODE == VKB_KV_Q5_0 ? 22 : 34;
    float acc = 0.0f;
    for (int64_t b = lane; b < nbpr; b += 32) {
        const uint8_t* blk = blocks + (row * nbpr + b) * BB;
        const float* xb = x + b * 32;
        float d = __half2float(__ushort_as_half((uint16_t)(blk[0] | (blk[1] << 8))));
        float part = 0.0f;
        if (MODE == VKB_KV_Q8_0) {
            for (int i = 0; i < 32; ++i) part = fmaf((float)(int8_t)blk[2 + i], xb[i], part);
        } else if (MODE == VKB_KV_Q4_0) {
            // vokra KV Q4_0: elements 2i / 2i+1 in the low / high nibble of byte i (kv_quant/q4_0.rs:73)
            for (int i = 0; i < 16; ++i) {
                uint8_t q = blk[2 + i];
                part = fmaf((float)((int)(q & 0xf) - 8), xb[2 * i], part);
                part = fmaf((float)((int)(q >> 4) - 8), xb[2 * i + 1], part);
            }
        } else {
            // Q5_0 (kv_quant/q5_0.rs:84): low 4 bits pair-packed, 5th bit in qh
            const uint8_t* qh = blk + 2;
            const uint8_t* qs = blk + 6;
            for (int i = 0; i < 32; ++i) {
                uint8_t lo4 = (i & 1) ? (qs[i / 2] >> 4) : (qs[i / 2] & 0xf);
                uint8_t hi1 = (qh[i / 8] >> (i % 8)) & 1;
                part = fmaf((float)((int)((hi1 << 4) | lo4) - 16), xb[i], part);
            }
        }
        acc = fmaf(part, d, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) y[row] = acc;
}

static void validate_dequant_gemv(int mode, size_t n_bytes, size_t n_rows, size_t nbpr, size_t x_len) {
    // validate_dequant_gemv (crates/vokra-core/src/kv_quant/gpu_ops.rs:95-130)
    if (mode == VKB_KV_FP32)
        fail(VKB_ERROR_INVALID_ARGUMENT,
             "fused_dequant_gemv: mode=Fp32 has no on-wire block layout; use dense_gemv_f32 instead");
    if (mode != VKB_KV_Q4_0 && mode != VKB_KV_Q5_0 && mode != VKB_KV_Q8_0)
        fail(VKB_ERROR_INVALID_ARGUMENT, "fused_dequant_gemv: unknown mode");
    if (x_len != nbpr * 32)
        fail(VKB_ERROR_INVALID_ARGUMENT, "fused_dequant_gemv: x.len()=" + std::to_string(x_len) +
                                             " != n_blocks_per_row*32 = " + std::to_string(nbpr * 32));
    size_t bb = mode == VKB_KV_Q4_0 ? 18 : mode == VKB_KV_Q5_0 ? 22 : 34;
    if (nbpr && n_rows > SIZE_MAX / nbpr / bb) fail(VKB_ERROR_INVALID_ARGUMENT, "fused_dequant_gemv: byte-length overflow");
    if (n_bytes != n_rows * nbpr * bb)
        fail(VKB_ERROR_INVALID_ARGUMENT, "fused_dequant_gemv: blocks_bytes.len()=" + std::to_string(n_bytes) +
                                             " != " + std::to_string(n_rows * nbpr * bb));
}

static void run_dequant_gemv(vkb_context* ctx, int mode, const void* blocks, size_t n_rows, size_t nbpr,
                             const float* x, float* y) {
    if (n_rows == 0) return;
    unsigned grid = (unsigned)((n_rows * 32 + 255) / 256);
    const uint8_t* b = reinterpret_cast<const uint8_t*>(blocks);
    if (mode == VKB_KV_Q8_0) launch_pdl(ctx, kv_dequant_gemv_kernel<VKB_KV_Q8_0>, grid, 256, 0, b, n_rows, nbpr, x, y);
    else if (mode == VKB_KV_Q4_0) launch_pdl(ctx, kv_dequant_gemv_kernel<VKB_KV_Q4_0>, grid, 256, 0, b, n_rows, nbpr, x, y);
    else launch_pdl(ctx, kv_dequant_gemv_kernel<VKB_KV_Q5_0>, grid, 256, 0, b, n_rows, nbpr, x, y);
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}

}  // namespace vkb

extern "C" {

vkb_status vkb_kv_pool_create(vkb_context* ctx, const vkb_kv_pool_desc* desc, vkb_kv_pool** out) {
    return guard([&] {
        if (!out) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_pool_create: null out");
        *out = kv_pool_create(ctx, desc);
    });
}

vkb_status vkb_kv_pool_destroy(vkb_kv_pool* pool) {
    return guard([&] { kv_pool_destroy(pool); });
}

vkb_status vkb_kv_begin_step(vkb_kv_pool* pool, int32_t n_tok, const int32_t* seq_ids_host,
                             const int32_t* positions_host) {
    return guard([&] {
        if (!pool) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_begin_step: null pool");
        kv_begin_step(pool, n_tok, seq_ids_host, positions_host);
    });
}

vkb_status vkb_kv_append(vkb_kv_pool* pool, int32_t layer, const float* k_dev, const float* v_dev) {
    return guard([&] {
        if (!pool) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_append: null pool");
        kv_append_ex(pool, layer, k_dev, v_dev, pool->W);
    });
}

vkb_status vkb_kv_attention(vkb_kv_pool* pool, int32_t layer, const float* q_dev, void* ctx_out_dev, int out_dtype) {
    return guard([&] {
        if (!pool) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_attention: null pool");
        kv_attention_ex(pool, layer, q_dev, pool->W, ctx_out_dev, out_dtype);
    });
}

vkb_status vkb_kv_append_attention(vkb_kv_pool* pool, int32_t layer, const float* qkv_dev, int64_t ld,
                                   void* ctx_out_dev, int out_dtype) {
    return guard([&] {
        if (!pool) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_append_attention: null pool");
        if (!qkv_dev || !ctx_out_dev) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_append_attention: null qkv/out");
        if (pool->n_tok == 0) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_append_attention: no step was begun");
        if (ld < 3 * (int64_t)pool->W || ld % 4)
            fail(VKB_ERROR_INVALID_ARGUMENT, "kv_append_attention: ld must be >= 3*n_head*d_head and a multiple of 4");
        kv_append_attention_ex(pool, layer, qkv_dev, ld, ctx_out_dev, out_dtype, nullptr, 0, nullptr, 1.0f);
    });
}

vkb_status vkb_kv_copy_stream(vkb_kv_pool* pool, int32_t src, int32_t dst, int32_t n_pos) {
    return guard([&] {
        if (!pool) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_copy_stream: null pool");
        kv_copy_stream(pool, src, dst, n_pos);
    });
}

int32_t vkb_kv_decode_fused(const vkb_kv_pool* pool) { return pool && kv_decode_fused(pool) ? 1 : 0; }

vkb_status vkb_kv_release_seq(vkb_kv_pool* pool, int32_t seq_id) {
    return guard([&] {
        if (!pool) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_release_seq: null pool");
        if (pool->d.layout != VKB_KV_LAYOUT_SEQUENCE)
            fail(VKB_ERROR_INVALID_ARGUMENT, "kv_release_seq: only the sequence layout frees per stream");
        if (seq_id < 0 || seq_id >= pool->d.n_stream) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_release_seq: bad stream");
        for (int i = 0; i < pool->ppseq; ++i) {
            int32_t& e = pool->table[(int64_t)seq_id * pool->ppseq + i];
            if (e >= 0) {
                drop(pool, e);
                e = -1;
            }
        }
        upload_table(pool);
    });
}

vkb_status vkb_kv_release_layer(vkb_kv_pool* pool, int32_t layer) {
    return guard([&] {
        if (!pool) fail(VKB_ERROR_INVALID_ARGUMENT, "release_layer: null pool");
        if (pool->d.layout != VKB_KV_LAYOUT_REFERENCE)
            fail(VKB_ERROR_INVALID_ARGUMENT, "release_layer: only the reference layout owns pages per layer");
        if (layer < 0 || layer >= pool->d.n_layer)
            fail(VKB_ERROR_INVALID_ARGUMENT, "release_layer: layer " + std::to_string(layer) + " >= n_layer " +
                                                 std::to_string(pool->d.n_layer));
        for (int i = 0; i < pool->ppl; ++i) {
            int32_t& e = pool->table[(int64_t)layer * pool->ppl + i];
            if (e >= 0) {
                zero_page(pool, e, 0);
                pool->refs[e] = 1;
                drop(pool, e);
                e = -1;
            }
        }
        upload_table(pool);
    });
}

vkb_status vkb_kv_reset(vkb_kv_pool* pool) {
    return guard([&] {
        if (!pool) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_reset: null pool");
        std::fill(pool->table.begin(), pool->table.end(), -1);
        cudaStream_t st = pool->ctx->stream;
        for (DevBuf* b : {&pool->kq, &pool->vq, &pool->kd, &pool->vd, &pool->kh, &pool->vh})
            if (b->n) VKB_CUDA(cudaMemsetAsync(b->p, 0, b->n, st));
        pool->free_list.clear();
        for (int64_t i = pool->n_pages - 1; i >= 0; --i) pool->free_list.push_back((int32_t)i);
        std::fill(pool->refs.begin(), pool->refs.end(), 0);
        pool->n_tok = 0;
        upload_table(pool);
    });
}

vkb_status vkb_kv_set_page_table(vkb_kv_pool* pool, const int32_t* table_host, size_t len) {
    return guard([&] {
        if (!pool || !table_host) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_set_page_table: null argument");
        if (pool->d.layout != VKB_KV_LAYOUT_SEQUENCE)
            fail(VKB_ERROR_INVALID_ARGUMENT, "kv_set_page_table: the reference layout allocates its own pages");
        if ((int64_t)len != pool->table_len) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_set_page_table: wrong length");
        std::vector<char> used(pool->n_pages, 0);
        for (size_t i = 0; i < len; ++i) {
            int32_t e = table_host[i];
            if (e < -1 || e >= pool->n_pages) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_set_page_table: page id out of range");
            if (e >= 0) {
                if (used[e]) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_set_page_table: page listed twice");
                used[e] = 1;
            }
        }
        pool->table.assign(table_host, table_host + len);
        pool->free_list.clear();
        for (int64_t i = pool->n_pages - 1; i >= 0; --i) {
            pool->refs[i] = used[i] ? 1 : 0;
            if (!used[i]) pool->free_list.push_back((int32_t)i);
        }
        upload_table(pool);
    });
}

size_t vkb_kv_table_len(const vkb_kv_pool* pool) { return pool ? (size_t)pool->table_len : 0; }

vkb_status vkb_kv_page_table(const vkb_kv_pool* pool, int64_t* out_host, size_t len) {
    return guard([&] {
        if (!pool || !out_host) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_page_table: null argument");
        if ((int64_t)len != pool->table_len) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_page_table: wrong length");
        for (size_t i = 0; i < len; ++i) out_host[i] = pool->table[i];
    });
}

int32_t vkb_kv_pages_in_use(const vkb_kv_pool* pool) {
    return pool ? (int32_t)(pool->n_pages - (int64_t)pool->free_list.size()) : 0;
}

size_t vkb_kv_page_bytes(const vkb_kv_pool* pool) {
    return pool ? (size_t)pool->rpp * pool->wire_row_bytes() : 0;
}

size_t vkb_kv_on_wire_bytes(const vkb_kv_pool* pool) {
    return pool ? (size_t)pool->n_arena * pool->n_pages * 2 * vkb_kv_page_bytes(pool) : 0;
}

namespace vkb {
// Host copy of rows [row0, row0 + n) of one side (K or V) in the reference's
// on-wire block encoding: Q8_0 34-byte blocks (d, 32 quants), Q4_0 18-byte
// blocks (d, 16 nibble bytes), Q5_0 22-byte blocks (d, 4 qh bytes, 16 nibble
// bytes), FP32 the plain values.
static std::vector<uint8_t> wire_rows(const vkb_kv_pool* p, int side, int64_t row0, int64_t n) {
    const int nb = p->row_blocks, sb = p->srow_bytes();
    std::vector<uint8_t> q((size_t)n * p->qrow), d((size_t)n * sb), h((size_t)n * p->hrow);
    cudaStream_t st = p->ctx->stream;
    VKB_CUDA(cudaMemcpyAsync(q.data(), (side ? p->vq : p->kq).as<uint8_t>() + row0 * p->qrow, q.size(),
                             cudaMemcpyDeviceToHost, st));
    if (sb) VKB_CUDA(cudaMemcpyAsync(d.data(), (side ? p->vd : p->kd).as<uint8_t>() + row0 * sb, d.size(),
                                     cudaMemcpyDeviceToHost, st));
    if (p->hrow) VKB_CUDA(cudaMemcpyAsync(h.data(), (side ? p->vh : p->kh).as<uint8_t>() + row0 * p->hrow, h.size(),
                                          cudaMemcpyDeviceToHost, st));
    VKB_CUDA(cudaStreamSynchronize(st));
    if (p->d.mode == VKB_KV_FP32) return q;
    const int bb = p->wire_row_bytes() / nb, qb = p->qrow / nb;
    std::vector<uint8_t> o((size_t)n * nb * bb);
    for (int64_t r = 0; r < n; ++r)
        for (int b = 0; b < nb; ++b) {
            uint8_t* blk = o.data() + ((size_t)r * nb + b) * bb;
            memcpy(blk, &d[((size_t)r * nb + b) * 2], 2);
            int off = 2;
            if (p->hrow) {
                memcpy(blk + 2, &h[(size_t)r * p->hrow + b * 4], 4);
                off = 6;
            }
            memcpy(blk + off, &q[(size_t)r * p->qrow + b * qb], qb);
        }
    return o;
}
}  // namespace vkb

vkb_status vkb_kv_read_page(const vkb_kv_pool* pool, int32_t layer, int32_t page, void* k_host, void* v_host) {
    return guard([&] {
        if (!pool || !k_host || !v_host) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_read_page: null argument");
        if (page < 0 || page >= pool->n_pages) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_read_page: page out of range");
        int arena = pool->d.layout == VKB_KV_LAYOUT_SEQUENCE ? layer : 0;
        if (arena < 0 || arena >= pool->n_arena) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_read_page: layer out of range");
        const int64_t row0 = ((int64_t)arena * pool->n_pages + page) * pool->rpp;
        for (int side = 0; side < 2; ++side) {
            std::vector<uint8_t> o = wire_rows(pool, side, row0, pool->rpp);
            memcpy(side ? v_host : k_host, o.data(), o.size());
        }
    });
}

vkb_status vkb_kv_read_step(const vkb_kv_pool* pool, int32_t layer, int32_t t, int32_t s, float* k_host,
                            float* v_host) {
    return guard([&] {
        if (!pool || !k_host || !v_host) fail(VKB_ERROR_INVALID_ARGUMENT, "kv_read_step: null argument");
        const auto& d = pool->d;
        if (layer < 0 || layer >= d.n_layer || t < 0 || t >= d.max_time || s < 0 || s >= d.n_stream)
            fail(VKB_ERROR_INVALID_ARGUMENT, "kv_read_step: out of range");
        int64_t row = row_of(pool, layer, t, s);
        if (row < 0) fail(VKB_ERROR_OTHER, "kv_read_step: slot was never written");
        const int W = pool->W, nb = pool->row_blocks;
        for (int side = 0; side < 2; ++side) {
            std::vector<uint8_t> o = wire_rows(pool, side, row, 1);
            float* out = side ? v_host : k_host;
            if (d.mode == VKB_KV_FP32) {
                memcpy(out, o.data(), (size_t)W * 4);
                continue;
            }
            // BlockQ8_0 / BlockQ4_0 / BlockQ5_0 ::unpack (q8_0.rs:69, q4_0.rs:73, q5_0.rs:84)
            const int bb = pool->wire_row_bytes() / nb;
            for (int b = 0; b < nb; ++b) {
                const uint8_t* blk = o.data() + (size_t)b * bb;
                const float sc = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
                for (int i = 0; i < 32; ++i) {
                    int q;
                    if (d.mode == VKB_KV_Q8_0) {
                        q = (int8_t)blk[2 + i];
                    } else if (d.mode == VKB_KV_Q4_0) {
                        q = (int)((blk[2 + i / 2] >> (4 * (i & 1))) & 0xf) - 8;
                    } else {
                        const int lo = (blk[6 + i / 2] >> (4 * (i & 1))) & 0xf, hi = (blk[2 + i / 8] >> (i % 8)) & 1;
                        q = (lo | (hi << 4)) - 16;
                    }
                    out[b * 32 + i] = (float)q * sc;
                }
            }
        }
    });
}

vkb_status vkb_attention_dense(vkb_context* ctx, int32_t n_tok, int32_t n_head, int32_t d_head, const float* q_dev,
                               const int32_t* seq_of_tok_dev, const void* k_dev, const void* v_dev,
                               const void* k_scale_dev, const void* v_scale_dev, int32_t n_ctx, int32_t kv_dtype,
                               void* ctx_out_dev, int32_t out_dtype) {
    return guard([&] {
        if (!ctx || !q_dev || !seq_of_tok_dev || !k_dev || !v_dev || !ctx_out_dev)
            fail(VKB_ERROR_INVALID_ARGUMENT, "attention_dense: null argument");
        if (n_tok <= 0 || n_ctx <= 0) fail(VKB_ERROR_INVALID_ARGUMENT, "attention_dense: empty shape");
        if (kv_dtype != VKB_DT_F16 && kv_dtype != VKB_KV_Q8_0)
            fail(VKB_ERROR_UNSUPPORTED_OP, "attention_dense: kv dtype must be F16 or Q8_0");
        if (kv_dtype == VKB_KV_Q8_0 && (!k_scale_dev || !v_scale_dev))
            fail(VKB_ERROR_INVALID_ARGUMENT, "attention_dense: Q8_0 needs scale planes");
        if (out_dtype != VKB_DT_F32 && out_dtype != VKB_DT_F16 && out_dtype != VKB_DT_F16X2)
            fail(VKB_ERROR_INVALID_ARGUMENT, "attention_dense: bad out dtype");
        run_dense_attention(ctx, n_tok, n_head, d_head, q_dev, seq_of_tok_dev, k_dev, v_dev, k_scale_dev, v_scale_dev,
                            n_ctx, kv_dtype == VKB_DT_F16 ? VKB_DT_F16 : VKB_KV_Q8_0, ctx_out_dev, out_dtype, nullptr);
    });
}

vkb_status vkb_quantize_rows_q8_0(vkb_context* ctx, const float* x_dev, int64_t n_rows, int32_t width, void* q_dev,
                                  void* d_dev) {
    return guard([&] {
        if (!ctx || !x_dev || !q_dev || !d_dev) fail(VKB_ERROR_INVALID_ARGUMENT, "quantize_rows: null argument");
        if (n_rows <= 0 || width <= 0) fail(VKB_ERROR_INVALID_ARGUMENT, "quantize_rows: empty shape");
        run_quantize_rows(ctx, x_dev, width, n_rows, width, reinterpret_cast<int8_t*>(q_dev),
                          reinterpret_cast<__half*>(d_dev), nullptr, 1);
    });
}

vkb_status vkb_kv_dequant_gemv(vkb_context* ctx, int mode, const void* blocks_dev, size_t n_bytes, size_t n_rows,
                               size_t nbpr, const float* x_dev, size_t x_len, float* y_dev) {
    return guard([&] {
        if (!ctx) fail(VKB_ERROR_INVALID_ARGUMENT, "dequant_gemv: null context");
        validate_dequant_gemv(mode, n_bytes, n_rows, nbpr, x_len);
        if (n_rows && (!blocks_dev || !x_dev || !y_dev)) fail(VKB_ERROR_INVALID_ARGUMENT, "dequant_gemv: null buffer");
        run_dequant_gemv(ctx, mode, blocks_dev, n_rows, nbpr, x_dev, y_dev);
    });
}

vkb_status vkb_kv_dequant_gemv_host(vkb_context* ctx, int mode, const void* blocks_host, size_t n_bytes, size_t n_rows,
                                    size_t nbpr, const float* x_host, size_t x_len, float* y_host) {
    return guard([&] {
        if (!ctx) fail(VKB_ERROR_INVALID_ARGUMENT, "dequant_gemv: null context");
        validate_dequant_gemv(mode, n_bytes, n_rows, nbpr, x_len);
        if (n_rows == 0) return;
        if (!blocks_host || !x_host || !y_host) fail(VKB_ERROR_INVALID_ARGUMENT, "dequant_gemv: null buffer");
        DevBuf b(n_bytes), x(x_len * 4), y(n_rows * 4);
        cudaStream_t st = ctx->stream;
        VKB_CUDA(cudaMemcpyAsync(b.p, blocks_host, n_bytes, cudaMemcpyHostToDevice, st));
        VKB_CUDA(cudaMemcpyAsync(x.p, x_host, x_len * 4, cudaMemcpyHostToDevice, st));
        run_dequant_gemv(ctx, mode, b.p, n_rows, nbpr, x.as<float>(), y.as<float>());
        VKB_CUDA(cudaMemcpyAsync(y_host, y.p, n_rows * 4, cudaMemcpyDeviceToHost, st));
        VKB_CUDA(cudaStreamSynchronize(st));
    });
}

}  // extern "C"
