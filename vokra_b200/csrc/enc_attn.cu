// enc_attn.cu — non-causal multi-head attention over a whole window (the
// Whisper encoder's 1500x1500 self-attention, whisper/nn.rs:209-300 with
// causal=false), FlashAttention-2 style: 128 queries per CTA (16 per warp),
// K/V tiles of 64 keys double-buffered in shared memory with cp.async,
// S = Q K^T and O += P V on m16n8k16 f16 tensor-core MMAs with fp32
// accumulators, online softmax in fp32 registers.
//
// Layout: qkv is [rows][ld] f16 with q at column h*64, k at kcol + h*64 and v
// at vcol + h*64 (the fused QKV projection writes q|k|v per row, q already
// scaled by d_head^-0.5); ctx is [rows][ctx_ld] f16 at column h*64. Rows of
// window b are b*T .. b*T+T-1.
#include "common.cuh"
#include "enc_attn.cuh"
#include <cstdlib>

namespace vkb {

namespace {
constexpr int HD = 64;       // head dim
constexpr int BQ = 128;      // queries per CTA (8 warps)
constexpr int NT = 256;      // threads
constexpr int BK = 64;       // keys per tile
constexpr int LDS = HD + 8;  // padded smem row (halves)

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
    uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    int sz = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
    uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
    uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(a));
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Loads a [ROWS rows][64 halves] tile (rows r0.., column col) into padded smem.
template <int ROWS>
__device__ __forceinline__ void load_tile(__half* dst, const __half* base, int64_t row0, int rows_valid, int64_t ld,
                                          int col) {
    const int tid = threadIdx.x;
#pragma unroll
    for (int i = 0; i < ROWS * 8 / NT; ++i) {
        int chunk = tid + i * NT;  // ROWS * 8 chunks of 8 halves
        int r = chunk >> 3, c8 = (chunk & 7) * 8;
        bool valid = r < rows_valid;
        const __half* src = base + (row0 + (valid ? r : 0)) * ld + col + c8;
        cp_async16(dst + r * LDS + c8, src, valid);
    }
}
}  // namespace

__global__ void __launch_bounds__(NT) enc_attn_kernel(const __half* __restrict__ qkv, int64_t ld, int kcol, int vcol,
                                                      int T, int n_head, __half* __restrict__ ctx, int64_t ctx_ld,
                                                      __half* __restrict__ ctx_lo) {
    pdl_entry();
    extern __shared__ __align__(128) __half enc_smem[];
    __half* sQ = enc_smem;                             // [BQ][LDS]
    auto sK = [&](int i) { return sQ + (BQ + i * BK) * LDS; };        // 2 x [BK][LDS]
    auto sV = [&](int i) { return sQ + (BQ + (2 + i) * BK) * LDS; };  // 2 x [BK][LDS]
    const int qt = blockIdx.x;
    const int bh = blockIdx.y;
    const int b = bh / n_head, h = bh % n_head;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row_base = (int64_t)b * T;
    const int q0 = qt * BQ;

    load_tile<BQ>(sQ, qkv, row_base + q0, min(BQ, T - q0), ld, h * HD);
    load_tile<BK>(sK(0), qkv, row_base, min(BK, T), ld, kcol + h * HD);
    load_tile<BK>(sV(0), qkv, row_base, min(BK, T), ld, vcol + h * HD);
    cp_async_commit();

    // Q fragments: 16 rows of this warp x 64 dims = 4 k-steps.
    uint32_t qa[4][4];
    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[j][e] = 0.0f;
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.0f, 0.0f};

    const int n_tiles = (T + BK - 1) / BK;
    for (int kt = 0; kt < n_tiles; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < n_tiles) {
            int k0 = (kt + 1) * BK;
            load_tile<BK>(sK(buf ^ 1), qkv, row_base + k0, min(BK, T - k0), ld, kcol + h * HD);
            load_tile<BK>(sV(buf ^ 1), qkv, row_base + k0, min(BK, T - k0), ld, vcol + h * HD);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (kt == 0) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
                int c = kk * 16 + (lane >> 4) * 8;
                ldsm_x4(qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], sQ + r * LDS + c);
            }
        }
        // S = Q K^T : 16 x 64 per warp
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) s[j][e] = 0.0f;
        const __half* K = sK(buf);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int jp = 0; jp < 4; ++jp) {  // pairs of 8-key n-tiles
                uint32_t b0, b1, b2, b3;
                int key = jp * 16 + (lane & 7) + (lane >> 4) * 8;
                int dim = kk * 16 + ((lane >> 3) & 1) * 8;
                ldsm_x4(b0, b1, b2, b3, K + key * LDS + dim);
                mma16816(s[2 * jp], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
                mma16816(s[2 * jp + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
            }
        }
        // mask keys past the window
        const int kbase = kt * BK;
        if (kbase + BK > T) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                int key = kbase + j * 8 + (lane & 3) * 2;
                if (key >= T) { s[j][0] = -INFINITY; s[j][2] = -INFINITY; }
                if (key + 1 >= T) { s[j][1] = -INFINITY; s[j][3] = -INFINITY; }
            }
        }
        // online softmax for rows r0 = lane/4 (elements 0,1) and r1 = r0+8 (2,3)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fmaxf(s[j][2 * hr], s[j][2 * hr + 1]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            // scores are in natural-log units; exp(x - m) = exp2((x - m) * log2 e)
            constexpr float L2E = 1.4426950408889634f;
            float mn = fmaxf(m_r[hr], mx);
            float corr = exp2f((m_r[hr] - mn) * L2E);
            const float mb = mn * L2E;
            float rs = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float p0 = exp2f(fmaf(s[j][2 * hr], L2E, -mb));
                float p1 = exp2f(fmaf(s[j][2 * hr + 1], L2E, -mb));
                s[j][2 * hr] = p0;
                s[j][2 * hr + 1] = p1;
                rs += p0 + p1;
            }
            rs += __shfl_xor_sync(0xffffffffu, rs, 1);
            rs += __shfl_xor_sync(0xffffffffu, rs, 2);
            l_r[hr] = l_r[hr] * corr + rs;
            m_r[hr] = mn;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                o[j][2 * hr] *= corr;
                o[j][2 * hr + 1] *= corr;
            }
        }
        // O += P V : P (16 x 64 keys) from the S accumulators, V via ldmatrix.trans
        const __half* V = sV(buf);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {  // 16 keys per k-step
            uint32_t a0 = pack_h2(s[2 * kk][0], s[2 * kk][1]);
            uint32_t a1 = pack_h2(s[2 * kk][2], s[2 * kk][3]);
            uint32_t a2 = pack_h2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            uint32_t a3 = pack_h2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int dp = 0; dp < 4; ++dp) {  // pairs of 8-dim n-tiles
                uint32_t b0, b1, b2, b3;
                int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
                int dim = dp * 16 + (lane >> 4) * 8;
                ldsm_x4_t(b0, b1, b2, b3, V + key * LDS + dim);
                mma16816(o[2 * dp], a0, a1, a2, a3, b0, b1);
                mma16816(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
            }
        }
        __syncthreads();
    }
    // normalise and store
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
        int q = q0 + warp * 16 + (lane >> 2) + hr * 8;
        if (q >= T) continue;
        float inv = 1.0f / l_r[hr];
        const int64_t off = (row_base + q) * ctx_ld + h * HD;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            int d = j * 8 + (lane & 3) * 2;
            float v0 = o[j][2 * hr] * inv, v1 = o[j][2 * hr + 1] * inv;
            __half2 hi = __floats2half2_rn(v0, v1);
            *reinterpret_cast<__half2*>(ctx + off + d) = hi;
            if (ctx_lo) {
                float2 hf = __half22float2(hi);
                *reinterpret_cast<__half2*>(ctx_lo + off + d) = __floats2half2_rn(v0 - hf.x, v1 - hf.y);
            }
        }
    }
}

void run_encoder_attention(vkb_context* ctx, const __half* qkv, int64_t ld, int kcol, int vcol, int n_windows, int T,
                           int n_head, int d_head, __half* out, int64_t out_ld, __half* out_lo, __half* vt_scratch,
                           size_t scratch_halves) {
    if (d_head != HD) fail(VKB_ERROR_UNSUPPORTED_OP, "encoder attention: d_head must be 64");
    static const bool legacy = std::getenv("VKB_ENC_ATTN_MMA_SYNC") != nullptr;
    if (!legacy && run_encoder_attention_tc(ctx, qkv, ld, kcol, vcol, n_windows, T, n_head, out, out_ld, out_lo,
                                            vt_scratch, scratch_halves))
        return;
    if (ld % 8 || kcol % 8 || vcol % 8 || out_ld % 2)
        fail(VKB_ERROR_INVALID_ARGUMENT, "encoder attention: rows must be 16-byte aligned");
    dim3 grid((unsigned)((T + BQ - 1) / BQ), (unsigned)(n_windows * n_head));
    const size_t smem = (size_t)(BQ + 4 * BK) * LDS * sizeof(__half);
    smem_optin(enc_attn_kernel, (int)smem);
    launch_pdl(ctx, enc_attn_kernel, grid, NT, smem, qkv, ld, kcol, vcol, T, n_head, out, out_ld, out_lo);
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}

}  // namespace vkb
