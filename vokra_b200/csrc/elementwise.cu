// elementwise.cu — layer norm, token embedding, conv stem im2col, positional
// add and argmax for the Whisper forward.
#include "common.cuh"
#include "weights.cuh"
#include "elementwise.cuh"

namespace vkb {

// One warp per row; two passes over the row held in registers (cols <= 2048,
// a multiple of 4). All of a lane's float4 loads are issued before the first
// use, so a row costs one memory round trip even when there are few rows (the
// decode step normalizes one row per stream).
template <int PER4>
__global__ void layer_norm_kernel(const float* __restrict__ x, int64_t rows, int cols, const float* __restrict__ g,
                                  const float* __restrict__ b, float eps, void* out, int out_fmt) {
    pdl_entry();
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int n4 = cols >> 2;
    const float4* xr = reinterpret_cast<const float4*>(x + row * cols);
    float4 v[PER4];
#pragma unroll
    for (int i = 0; i < PER4; ++i) {
        const int c = lane + 32 * i;
        v[i] = c < n4 ? __ldg(xr + c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < PER4; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    s = warp_sum(s);
    const float inv_cols = 1.0f / (float)cols;
    const float mean = s * inv_cols;
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < PER4; ++i) {
        const int c = lane + 32 * i;
        if (c < n4) {
            const float d0 = v[i].x - mean, d1 = v[i].y - mean, d2 = v[i].z - mean, d3 = v[i].w - mean;
            q += (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3);
        }
    }
    q = warp_sum(q);
    const float inv_std = 1.0f / sqrtf(q * inv_cols + eps);
    const float4* g4 = reinterpret_cast<const float4*>(g);
    const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
    for (int i = 0; i < PER4; ++i) {
        const int c = lane + 32 * i;
        if (c >= n4) break;
        const float4 gg = __ldg(g4 + c), bb = __ldg(b4 + c);
        const float y[4] = {(v[i].x - mean) * inv_std * gg.x + bb.x, (v[i].y - mean) * inv_std * gg.y + bb.y,
                            (v[i].z - mean) * inv_std * gg.z + bb.z, (v[i].w - mean) * inv_std * gg.w + bb.w};
        const int64_t o = row * cols + 4 * c;
        if (out_fmt == 0) {
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + o) = make_float4(y[0], y[1], y[2], y[3]);
        } else {
            __half* oh = reinterpret_cast<__half*>(out);
            const __half2 h01 = __floats2half2_rn(y[0], y[1]), h23 = __floats2half2_rn(y[2], y[3]);
            uint2 hv;
            hv.x = *reinterpret_cast<const uint32_t*>(&h01);
            hv.y = *reinterpret_cast<const uint32_t*>(&h23);
            *reinterpret_cast<uint2*>(oh + o) = hv;
            if (out_fmt == 2) {
                const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
                const __half2 l01 = __floats2half2_rn(y[0] - f01.x, y[1] - f01.y);
                const __half2 l23 = __floats2half2_rn(y[2] - f23.x, y[3] - f23.y);
                uint2 lv;
                lv.x = *reinterpret_cast<const uint32_t*>(&l01);
                lv.y = *reinterpret_cast<const uint32_t*>(&l23);
                *reinterpret_cast<uint2*>(oh + rows * cols + o) = lv;
            }
        }
    }
}

// Few rows (a decode step): one CTA per row, one float4 of x, g and b per
// thread, all loaded before the two block reductions.
__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = l < nw ? red[l] : 0.0f;
    return warp_sum(t);
}

__global__ void layer_norm_row_kernel(const float* __restrict__ x, int64_t rows, int cols, const float* __restrict__ g,
                                      const float* __restrict__ b, float eps, void* out, int out_fmt) {
    pdl_launch();
    __shared__ float red[32];
    const int64_t row = blockIdx.x;
    const int c = threadIdx.x, n4 = cols >> 2;
    const bool on = c < n4;
    const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    // LayerNorm parameters are model weights: read before the wait, x after it
    const float4 gg = on ? __ldg(reinterpret_cast<const float4*>(g) + c) : z;
    const float4 bb = on ? __ldg(reinterpret_cast<const float4*>(b) + c) : z;
    pdl_wait();
    const float4 v = on ? __ldg(reinterpret_cast<const float4*>(x + row * cols) + c) : z;
    const float inv_cols = 1.0f / (float)cols;
    const float mean = block_sum((v.x + v.y) + (v.z + v.w), red) * inv_cols;
    const float d0 = v.x - mean, d1 = v.y - mean, d2 = v.z - mean, d3 = v.w - mean;
    const float q = block_sum(on ? (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3) : 0.0f, red);
    const float inv_std = 1.0f / sqrtf(q * inv_cols + eps);
    if (!on) return;
    const float y[4] = {d0 * inv_std * gg.x + bb.x, d1 * inv_std * gg.y + bb.y, d2 * inv_std * gg.z + bb.z,
                        d3 * inv_std * gg.w + bb.w};
    const int64_t o = row * cols + 4 * c;
    if (out_fmt == 0) {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + o) = make_float4(y[0], y[1], y[2], y[3]);
    } else {
        __half* oh = reinterpret_cast<__half*>(out);
        const __half2 h01 = __floats2half2_rn(y[0], y[1]), h23 = __floats2half2_rn(y[2], y[3]);
        uint2 hv;
        hv.x = *reinterpret_cast<const uint32_t*>(&h01);
        hv.y = *reinterpret_cast<const uint32_t*>(&h23);
        *reinterpret_cast<uint2*>(oh + o) = hv;
        if (out_fmt == 2) {
            const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
            const __half2 l01 = __floats2half2_rn(y[0] - f01.x, y[1] - f01.y);
            const __half2 l23 = __floats2half2_rn(y[2] - f23.x, y[3] - f23.y);
            uint2 lv;
            lv.x = *reinterpret_cast<const uint32_t*>(&l01);
            lv.y = *reinterpret_cast<const uint32_t*>(&l23);
            *reinterpret_cast<uint2*>(oh + rows * cols + o) = lv;
        }
    }
}

// One CTA per row, one float4 of the row per thread: sums the split-K partials
// of a residual projection (split order, as splitk_reduce_kernel), adds bias
// and the residual, writes h, then normalizes the new row like
// layer_norm_row_kernel.
__global__ void reduce_residual_ln_kernel(const float* __restrict__ part, int splits, int64_t rows, int cols,
                                          const float* __restrict__ bias, float* __restrict__ h,
                                          const float* __restrict__ g, const float* __restrict__ b, float eps,
                                          void* out, int out_fmt) {
    pdl_launch();
    __shared__ float red[32];
    const int64_t row = blockIdx.x;
    const int c = threadIdx.x, n4 = cols >> 2;
    const bool on = c < n4;
    const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float4 v = z, gg = z, bb = z, bi = z;
    // the layer's bias and LayerNorm parameters are model weights (no kernel
    // writes them): loaded while the projection that produced the partials ends
    if (on) {
        if (bias) bi = __ldg(reinterpret_cast<const float4*>(bias) + c);
        gg = __ldg(reinterpret_cast<const float4*>(g) + c);
        bb = __ldg(reinterpret_cast<const float4*>(b) + c);
    }
    pdl_wait();
    if (on) {
        const int64_t o4 = row * n4 + c;
        // the residual row with the first partials: one round of loads
        const float4 r = reinterpret_cast<const float4*>(h)[o4];
        float4 acc = z;
        constexpr int U = 8;
        for (int s0 = 0; s0 < splits; s0 += U) {
            float4 t[U];
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (s0 + u < splits) t[u] = __ldcg(reinterpret_cast<const float4*>(part) + (int64_t)(s0 + u) * rows * n4 + o4);
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (s0 + u < splits) {
                    acc.x += t[u].x; acc.y += t[u].y; acc.z += t[u].z; acc.w += t[u].w;
                }
        }
        v = make_float4(r.x + (acc.x + bi.x), r.y + (acc.y + bi.y), r.z + (acc.z + bi.z), r.w + (acc.w + bi.w));
        reinterpret_cast<float4*>(h)[o4] = v;
    }
    const float inv_cols = 1.0f / (float)cols;
    const float mean = block_sum((v.x + v.y) + (v.z + v.w), red) * inv_cols;
    const float d0 = v.x - mean, d1 = v.y - mean, d2 = v.z - mean, d3 = v.w - mean;
    const float q = block_sum(on ? (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3) : 0.0f, red);
    const float inv_std = 1.0f / sqrtf(q * inv_cols + eps);
    if (!on) return;
    const float y[4] = {d0 * inv_std * gg.x + bb.x, d1 * inv_std * gg.y + bb.y, d2 * inv_std * gg.z + bb.z,
                        d3 * inv_std * gg.w + bb.w};
    const int64_t o = row * cols + 4 * c;
    if (out_fmt == 0) {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + o) = make_float4(y[0], y[1], y[2], y[3]);
    } else {
        __half* oh = reinterpret_cast<__half*>(out);
        const __half2 h01 = __floats2half2_rn(y[0], y[1]), h23 = __floats2half2_rn(y[2], y[3]);
        uint2 hv;
        hv.x = *reinterpret_cast<const uint32_t*>(&h01);
        hv.y = *reinterpret_cast<const uint32_t*>(&h23);
        *reinterpret_cast<uint2*>(oh + o) = hv;
        if (out_fmt == 2) {
            const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
            const __half2 l01 = __floats2half2_rn(y[0] - f01.x, y[1] - f01.y);
            const __half2 l23 = __floats2half2_rn(y[2] - f23.x, y[3] - f23.y);
            uint2 lv;
            lv.x = *reinterpret_cast<const uint32_t*>(&l01);
            lv.y = *reinterpret_cast<const uint32_t*>(&l23);
            *reinterpret_cast<uint2*>(oh + rows * cols + o) = lv;
        }
    }
}

void run_reduce_residual_ln(vkb_context* ctx, const float* part, int splits, int64_t rows, int cols, const float* bias,
                            float* h, const float* g, const float* b, float eps, void* out, int out_fmt) {
    if (cols % 4 || cols / 4 > 1024) fail(VKB_ERROR_UNSUPPORTED_OP, "reduce_residual_ln: row width");
    const int threads = ((cols / 4 + 31) / 32) * 32;
    launch_pdl(ctx, reduce_residual_ln_kernel, (unsigned)rows, threads, 0, part, splits, rows, cols, bias, h, g, b,
               eps, out, out_fmt);
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}

void run_layer_norm(vkb_context* ctx, const float* x, int64_t rows, int cols, const float* g, const float* b, float eps,
                    void* out, int out_fmt) {
    if (cols > 2048) fail(VKB_ERROR_UNSUPPORTED_OP, "layer_norm: row width above 2048");
    if (cols % 4) fail(VKB_ERROR_UNSUPPORTED_OP, "layer_norm: row width must be a multiple of 4");
    if (rows <= 4 * (int64_t)ctx->sm_count) {
        const int threads = ((cols / 4 + 31) / 32) * 32;
        launch_pdl(ctx, layer_norm_row_kernel, (unsigned)rows, threads, 0, x, rows, cols, g, b, eps, out, out_fmt);
        VKB_CUDA(cudaGetLastError());
        ctx->count();
        return;
    }
    unsigned grid = (unsigned)((rows * 32 + 255) / 256);
    if (cols <= 512) launch_pdl(ctx, layer_norm_kernel<4>, grid, 256, 0, x, rows, cols, g, b, eps, out, out_fmt);
    else if (cols <= 1280) launch_pdl(ctx, layer_norm_kernel<10>, grid, 256, 0, x, rows, cols, g, b, eps, out, out_fmt);
    else launch_pdl(ctx, layer_norm_kernel<16>, grid, 256, 0, x, rows, cols, g, b, eps, out, out_fmt);
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}

// One thread per (token, 64-wide stage) of the embedding row.
template <int FMT>
__global__ void embed_kernel(const uint8_t* __restrict__ qs, const uint8_t* __restrict__ sc, int64_t K,
                             const int32_t* __restrict__ tokens, const int32_t* __restrict__ positions, int n_tok,
                             const float* __restrict__ pos, float* __restrict__ h) {
    pdl_entry();
    const int stages = (int)(K / STAGE_K);
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)n_tok * stages) return;
    const int t = (int)(i / stages), s = (int)(i % stages);
    const int64_t row = tokens[t];
    StagePtrs p = stage_ptrs(FMT, qs, sc, K, row / TILE_N, s);
    float w[64];
    dequant_row_stage<FMT>(p.qs, p.sc, (int)(row % TILE_N), s, w);
    const float* pe = pos + (int64_t)positions[t] * K + s * 64;
    float* dst = h + (int64_t)t * K + s * 64;
#pragma unroll
    for (int e = 0; e < 64; ++e) dst[e] = w[e] + pe[e];
}

void run_embed(vkb_context* ctx, const vkb_weight* w, const int32_t* tokens, const int32_t* positions, int n_tok,
               const float* pos, float* h) {
    int64_t n = (int64_t)n_tok * (w->k / STAGE_K);
    unsigned grid = (unsigned)((n + 127) / 128);
    const uint8_t* qs = w->qs.as<uint8_t>();
    const uint8_t* sc = w->sc.as<uint8_t>();
    with_fmt(w->fmt, [&](auto F) {
        launch_pdl(ctx, embed_kernel<decltype(F)::value>, grid, 128, 0, qs, sc, w->k, tokens, positions, n_tok, pos, h);
    });
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}

// col[b*To + t][c*3 + kk] = x[b][c][t*stride + kk - 1]; columns C*3 .. ldc-1 are zero
__global__ void im2col_ct_kernel(const float* __restrict__ x, int B, int C, int T, int To, int stride, int ldc,
                                 __half* __restrict__ col, int split) {
    pdl_entry();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t total = (int64_t)B * To * ldc;
    if (i >= total) return;
    const int64_t r = i / ldc;
    const int cc = (int)(i % ldc);
    if (cc >= C * 3) {
        col[i] = __float2half_rn(0.0f);
        if (split) col[total + i] = __float2half_rn(0.0f);
        return;
    }
    const int c = cc / 3, kk = cc % 3;
    const int b = (int)(r / To), t = (int)(r % To);
    const int p = t * stride + kk - 1;
    float v = (p >= 0 && p < T) ? x[((int64_t)b * C + c) * T + p] : 0.0f;
    __half hi = __float2half_rn(v);
    col[i] = hi;
    if (split) col[total + i] = __float2half_rn(v - __half2float(hi));
}

// col[b*To + t][c*3 + kk] = x[b*T + t*stride + kk - 1][c]; one thread per
// (output row, 8 channels): three 16-byte tap loads, interleaved in registers
// into 24 contiguous halves (48 bytes).
__global__ void im2col_tc_kernel(const __half* __restrict__ x, int B, int C, int T, int To, int stride,
                                 __half* __restrict__ col, int planes) {
    pdl_entry();
    const int nchunk = C >> 3;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * To * nchunk) return;
    const int r = i / nchunk, ch = i - r * nchunk;
    const int b = r / To, t = r - b * To;
    const int64_t in_plane = (int64_t)B * T * C, out_plane = (int64_t)B * To * C * 3;
    for (int pl = 0; pl < planes; ++pl) {
        uint4 tap[3];
#pragma unroll
        for (int kk = 0; kk < 3; ++kk) {
            const int p = t * stride + kk - 1;
            tap[kk] = (p >= 0 && p < T)
                          ? __ldg(reinterpret_cast<const uint4*>(x + pl * in_plane + ((int64_t)b * T + p) * C) + ch)
                          : make_uint4(0, 0, 0, 0);
        }
        const uint16_t* h0 = reinterpret_cast<const uint16_t*>(&tap[0]);
        const uint16_t* h1 = reinterpret_cast<const uint16_t*>(&tap[1]);
        const uint16_t* h2 = reinterpret_cast<const uint16_t*>(&tap[2]);
        uint32_t o[12];
#pragma unroll
        for (int q = 0; q < 12; ++q) {
            // output halves 2q and 2q+1: channel (2q)/3 tap (2q)%3, channel (2q+1)/3 tap (2q+1)%3
            const int e0 = 2 * q, e1 = 2 * q + 1;
            const uint16_t* s0 = (e0 % 3 == 0) ? h0 : (e0 % 3 == 1) ? h1 : h2;
            const uint16_t* s1 = (e1 % 3 == 0) ? h0 : (e1 % 3 == 1) ? h1 : h2;
            o[q] = (uint32_t)s0[e0 / 3] | ((uint32_t)s1[e1 / 3] << 16);
        }
        uint4* dst = reinterpret_cast<uint4*>(col + pl * out_plane + (int64_t)r * C * 3 + ch * 24);
        dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
        dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
        dst[2] = make_uint4(o[8], o[9], o[10], o[11]);
    }
}

static int conv_out(int T, int stride) { return (T + 2 - 3) / stride + 1; }

void run_im2col_ct(vkb_context* ctx, const float* x, int B, int C, int T, int stride, int ldc, __half* col,
                   bool split) {
    int To = conv_out(T, stride);
    int64_t total = (int64_t)B * To * ldc;
    launch_pdl(ctx, im2col_ct_kernel, (unsigned)((total + 255) / 256), 256, 0, x, B, C, T, To, stride, ldc, col,
                                                                              split ? 1 : 0);
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}

void run_im2col_tc(vkb_context* ctx, const __half* x, int B, int C, int T, int stride, __half* col, int planes) {
    int To = conv_out(T, stride);
    if (C % 8 || ((uintptr_t)x & 15) || ((uintptr_t)col & 15))
        fail(VKB_ERROR_UNSUPPORTED_OP, "im2col: channels must be a multiple of 8 with 16-byte aligned buffers");
    const int64_t total = (int64_t)B * To * (C / 8);
    if (total >= (int64_t(1) << 31)) fail(VKB_ERROR_UNSUPPORTED_OP, "im2col: too many rows");
    launch_pdl(ctx, im2col_tc_kernel, (unsigned)((total + 255) / 256), 256, 0, x, B, C, T, To, stride, col, planes);
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}

// 4 channels per thread (C % 4 == 0).
__global__ void add_pos_kernel(const __half* __restrict__ y, const float* __restrict__ pos, int B, int T, int C,
                               float* __restrict__ h, int planes) {
    pdl_entry();
    const int i4 = blockIdx.x * blockDim.x + threadIdx.x;  // float4 index
    const int total4 = B * T * C / 4;
    if (i4 >= total4) return;
    const int tc4 = i4 % (T * C / 4);
    const uint2 hv = __ldg(reinterpret_cast<const uint2*>(y) + i4);
    float2 a = __half22float2(*reinterpret_cast<const __half2*>(&hv.x));
    float2 c = __half22float2(*reinterpret_cast<const __half2*>(&hv.y));
    if (planes == 2) {
        const uint2 lv = __ldg(reinterpret_cast<const uint2*>(y + (int64_t)total4 * 4) + i4);
        const float2 la = __half22float2(*reinterpret_cast<const __half2*>(&lv.x));
        const float2 lc = __half22float2(*reinterpret_cast<const __half2*>(&lv.y));
        a.x += la.x; a.y += la.y; c.x += lc.x; c.y += lc.y;
    }
    const float4 p = __ldg(reinterpret_cast<const float4*>(pos) + tc4);
    reinterpret_cast<float4*>(h)[i4] = make_float4(a.x + p.x, a.y + p.y, c.x + p.z, c.y + p.w);
}

void run_add_pos(vkb_context* ctx, const __half* y, const float* pos, int B, int T, int C, float* h, int planes) {
    const int64_t total4 = (int64_t)B * T * C / 4;
    if (C % 4 || total4 >= (int64_t(1) << 31)) fail(VKB_ERROR_UNSUPPORTED_OP, "add_pos: shape");
    launch_pdl(ctx, add_pos_kernel, (unsigned)((total4 + 255) / 256), 256, 0, y, pos, B, T, C, h, planes);
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}

// One CTA per row; first index of the maximum wins ties. Each thread loads
// 8 values before comparing any, so a row costs a few memory round trips.
__global__ void argmax_kernel(const float* __restrict__ logits, int n_cols, int32_t* __restrict__ ids) {
    pdl_entry();
    const float* r = logits + (int64_t)blockIdx.x * n_cols;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    constexpr int U = 8;
    for (int j0 = threadIdx.x; j0 < n_cols; j0 += U * blockDim.x) {
        float v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = j0 + u * blockDim.x;
            v[u] = j < n_cols ? __ldg(r + j) : -INFINITY;
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = j0 + u * blockDim.x;
            if (j < n_cols && (v[u] > best || (v[u] == best && j < bi))) { best = v[u]; bi = j; }
        }
    }
    __shared__ float sv[32];
    __shared__ int si[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, best, o);
        int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) { sv[w] = best; si[w] = bi; }
    __syncthreads();
    if (w == 0) {
        const int nw = blockDim.x >> 5;
        best = l < nw ? sv[l] : -INFINITY;
        bi = l < nw ? si[l] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, best, o);
            int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
        }
        if (l == 0) ids[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
    }
}

void run_argmax(vkb_context* ctx, const float* logits, int n_rows, int n_cols, int32_t* ids) {
    launch_pdl(ctx, argmax_kernel, n_rows, 1024, 0, logits, n_cols, ids);
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}

}  // namespace vkb
