// enc_attn_tc.cu — the encoder's whole-window attention on the 5th-generation
// tensor cores (tcgen05, accumulators in tensor memory).
//
// Same result as enc_attn_kernel (whisper/nn.rs:209-300, causal=false; q
// pre-scaled by d_head^-0.5 in the QKV projection; P rounded to f16 for the
// P.V product, fp32 row sums). One CTA per (window, head, 128 queries):
//   S  = Q K^T   128 x 128 keys, A = Q and B = K from shared memory (TMA,
//                128-byte swizzle), accumulator in TMEM columns [0, 128)
//   softmax      4 warps, thread = query row = TMEM lane: the whole score row
//                is in the thread's own TMEM lane, so row max and sum need no
//                shuffles; P (f16 pairs) is written back to TMEM columns
//                [128, 192) and is the A operand of
//   O += P V     128 x 64, B = V^T tile from shared memory (V is transposed
//                once per layer so that it is K-major), accumulator O in TMEM
//                columns [192, 256).
// The running max is only raised (and O, l rescaled) when a tile's max exceeds
// it by more than 2^8, so most tiles skip the O rescale; P stays below 2^8.
// Warps: 0 producer (TMA), 1 TMEM owner + MMA issuer, 2..5 softmax/epilogue.
// 256 TMEM columns and ~81 KB of shared memory per CTA: two CTAs per SM, so
// one CTA's softmax overlaps the other's MMAs. Every wait is bounded.
#include "common.cuh"
#include "tc_ptx.cuh"
#include "enc_attn.cuh"
#include <cudaTypedefs.h>

namespace vkb {

void make_tmap_f16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows);

namespace {
constexpr int HD = 64;
constexpr int BQ = 128;       // queries per CTA
constexpr int BKEY = 128;     // keys per tile
constexpr int TILE_BYTES = BQ * HD * 2;        // 16 KB: Q tile, K tile, or V^T tile (2 x 8 KB)
constexpr int SMEM = 1024 + 3 * TILE_BYTES + 2 * TILE_BYTES + 512;  // Q + 2 x (K + V^T) + barriers
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t S_COL = 0, P_COL = 128, O_COL = 192;
constexpr float L2E = 1.4426950408889634f;
constexpr float RESCALE_LOG2 = 8.0f;

// 2^x on the special-function unit (ex2.approx; relative error ~2^-22, -inf -> 0).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
}  // namespace

// vt[(w*H + h)*64 + d][t] = qkv[w*T + t][vcol + h*64 + d]; columns t in [T, Tp) are zero.
__global__ void v_transpose_kernel(const __half* __restrict__ qkv, int64_t ld, int vcol, int T, int Tp, int n_head,
                                   __half* __restrict__ vt) {
    pdl_entry();
    __shared__ __half tile[64][72];
    const int t0 = blockIdx.x * 64, wh = blockIdx.y;
    const int w = wh / n_head, h = wh % n_head;
    const int tid = threadIdx.x;
    // load 64 rows (t) x 64 halves (d): 8 threads per row, 16 bytes each
    for (int i = tid; i < 64 * 8; i += blockDim.x) {
        const int r = i >> 3, c8 = (i & 7) * 8;
        const int t = t0 + r;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (t < T) v = __ldg(reinterpret_cast<const uint4*>(qkv + ((int64_t)w * T + t) * ld + vcol + h * HD + c8));
        const __half* hv = reinterpret_cast<const __half*>(&v);
#pragma unroll
        for (int e = 0; e < 8; ++e) tile[r][c8 + e] = hv[e];
    }
    __syncthreads();
    // write 64 rows (d) x 64 halves (t)
    for (int i = tid; i < 64 * 8; i += blockDim.x) {
        const int d = i >> 3, c8 = (i & 7) * 8;
        if (t0 + c8 >= Tp) continue;
        __align__(16) __half o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = tile[c8 + e][d];
        *reinterpret_cast<uint4*>(vt + ((int64_t)wh * HD + d) * Tp + t0 + c8) = *reinterpret_cast<const uint4*>(o);
    }
}

__global__ void __launch_bounds__(192, 2)
    enc_attn_tc_kernel(const __grid_constant__ CUtensorMap qk_map, const __grid_constant__ CUtensorMap vt_map, int kcol,
                       int T, int n_head, __half* __restrict__ ctx, int64_t ctx_ld, __half* __restrict__ ctx_lo,
                       int* err) {
    pdl_launch();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* sK = smem + TILE_BYTES;          // 2 stages
    uint8_t* sV = smem + 3 * TILE_BYTES;      // 2 stages (each 2 x 8 KB key blocks)
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 5 * TILE_BYTES);
    uint64_t* q_full = bars;
    uint64_t* kv_full = bars + 1;   // [2]
    uint64_t* kv_empty = bars + 3;  // [2]
    uint64_t* s_full = bars + 5;
    uint64_t* p_full = bars + 6;
    uint64_t* o_full = bars + 7;
    uint64_t* s_free = bars + 8;   // softmax(j) holds S(j) in registers: S may be overwritten
    uint64_t* pv_done = bars + 9;  // O += P(j) V(j) completed: P may be overwritten, O rescaled
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * BQ;
    const int wh = blockIdx.y;
    const int w = wh / n_head, h = wh % n_head;
    const int n_tiles = (T + BKEY - 1) / BKEY;

    if (threadIdx.x == 0) {
        ptx::mbar_init(q_full, 1);
        for (int i = 0; i < 2; ++i) {
            ptx::mbar_init(&kv_full[i], 1);
            ptx::mbar_init(&kv_empty[i], 1);
        }
        ptx::mbar_init(s_full, 1);
        ptx::mbar_init(p_full, 128);
        ptx::mbar_init(o_full, 1);
        ptx::mbar_init(s_free, 128);
        ptx::mbar_init(pv_done, 1);
        ptx::fence_mbar_init();
    }
    if (warp == 1) {
        ptx::tmem_alloc(tmem_slot, TMEM_COLS);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            pdl_wait();
            const int row0 = w * T;
            ptx::mbar_expect_tx(q_full, TILE_BYTES);
            ptx::tma_load_2d(sQ, &qk_map, q_full, h * HD, row0 + q0);
            for (int j = 0; j < n_tiles && ok; ++j) {
                const int s = j & 1;
                if (!ptx::mbar_wait(&kv_empty[s], ((j >> 1) & 1) ^ 1)) { ok = false; break; }
                ptx::mbar_expect_tx(&kv_full[s], 2 * TILE_BYTES);
                ptx::tma_load_2d(sK + s * TILE_BYTES, &qk_map, &kv_full[s], kcol + h * HD, row0 + j * BKEY);
                uint8_t* v = sV + s * TILE_BYTES;
                ptx::tma_load_2d(v, &vt_map, &kv_full[s], j * BKEY, wh * HD);
                ptx::tma_load_2d(v + TILE_BYTES / 2, &vt_map, &kv_full[s], j * BKEY + 64, wh * HD);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_s = ptx::idesc_f16_f32(BQ, BKEY);
            constexpr uint32_t idesc_o = ptx::idesc_f16_f32(BQ, HD);
            const uint32_t q_addr = ptx::smem_u32(sQ);
            auto issue_pv = [&](int j) {
                const uint32_t v_addr = ptx::smem_u32(sV + (j & 1) * TILE_BYTES);
#pragma unroll
                for (int kk = 0; kk < BKEY / 16; ++kk) {
                    const uint64_t bd = ptx::sdesc_sw128(v_addr + (kk >> 2) * (TILE_BYTES / 2) + (kk & 3) * 32);
                    ptx::mma_f16_ts(tmem + O_COL, tmem + P_COL + kk * 8, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
                }
                ptx::mma_commit(&kv_empty[j & 1]);
                ptx::mma_commit(pv_done);
            };
            auto issue_s = [&](int j) {
                const uint32_t k_addr = ptx::smem_u32(sK + (j & 1) * TILE_BYTES);
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk)
                    ptx::mma_f16_ss(tmem + S_COL, ptx::sdesc_sw128(q_addr + kk * 32),
                                    ptx::sdesc_sw128(k_addr + kk * 32), idesc_s, kk > 0 ? 1u : 0u);
                ptx::mma_commit(s_full);
            };
            // S(j+1) is issued as soon as softmax(j) has S(j) in registers, so it
            // runs while softmax(j) computes; O += P(j) V(j) follows P(j).
            if (!ptx::mbar_wait(q_full, 0) || !ptx::mbar_wait(&kv_full[0], 0)) ok = false;
            if (ok) issue_s(0);
            for (int j = 0; j < n_tiles && ok; ++j) {
                if (j + 1 < n_tiles) {
                    if (!ptx::mbar_wait(&kv_full[(j + 1) & 1], ((j + 1) >> 1) & 1)) { ok = false; break; }
                    if (!ptx::mbar_wait(s_free, j & 1)) { ok = false; break; }
                    ptx::tc_fence_after();
                    issue_s(j + 1);
                }
                if (!ptx::mbar_wait(p_full, j & 1)) { ok = false; break; }
                ptx::tc_fence_after();
                issue_pv(j);
            }
            if (ok) ptx::mma_commit(o_full);
        }
    } else {
        // softmax + epilogue: thread = query row r = TMEM lane r
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        float m_used = -INFINITY;  // running max, log2 units
        float l = 0.0f;
        for (int j = 0; j < n_tiles && ok; ++j) {
            if (!ptx::mbar_wait(s_full, j & 1)) { ok = false; break; }
            ptx::tc_fence_after();
            const int kvalid = min(BKEY, T - j * BKEY);
            // the whole score row of this tile in registers: four loads, one wait
            uint32_t sv[BKEY];
            ptx::tmem_ld32(tmem + lane_off + S_COL + 0, *reinterpret_cast<uint32_t(*)[32]>(sv + 0));
            ptx::tmem_ld32(tmem + lane_off + S_COL + 32, *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
            ptx::tmem_ld32(tmem + lane_off + S_COL + 64, *reinterpret_cast<uint32_t(*)[32]>(sv + 64));
            ptx::tmem_ld32(tmem + lane_off + S_COL + 96, *reinterpret_cast<uint32_t(*)[32]>(sv + 96));
            ptx::tmem_ld_wait();
            ptx::tc_fence_before();
            ptx::mbar_arrive(s_free);  // S(j+1) may now be computed into the same columns
            if (kvalid < BKEY) {
#pragma unroll
                for (int c = 0; c < BKEY; ++c)
                    if (c >= kvalid) sv[c] = __float_as_uint(-INFINITY);
            }
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < BKEY; ++c) mx = fmaxf(mx, __uint_as_float(sv[c]));
            const float mt = mx * L2E;
            // raise the running max only when this tile would overflow P's range
            const bool raise = mt > m_used + RESCALE_LOG2;
            const float m_new = raise ? mt : m_used;
            const float corr = raise ? ex2_approx(m_used - m_new) : 1.0f;  // 0 on the first tile
            // O += P(j-1) V(j-1) must be complete before O is rescaled or P rewritten
            if (j > 0 && !ptx::mbar_wait(pv_done, (j - 1) & 1)) { ok = false; break; }
            ptx::tc_fence_after();
            if (__any_sync(0xffffffffu, raise && j > 0)) {
                // rescale O
                uint32_t o[32];
#pragma unroll
                for (int c0 = 0; c0 < HD; c0 += 32) {
                    ptx::tmem_ld32(tmem + lane_off + O_COL + c0, o);
                    ptx::tmem_ld_wait();
#pragma unroll
                    for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * corr);
                    ptx::tmem_st32(tmem + lane_off + O_COL + c0, o);
                }
            }
            l *= corr;
            m_used = m_new;
            // P = exp2(s*log2e - m) as f16 pairs into TMEM, row sum in fp32
#pragma unroll
            for (int c0 = 0; c0 < BKEY; c0 += 32) {
                uint32_t pk[16];
#pragma unroll
                for (int c = 0; c < 32; c += 2) {
                    const float p0 = ex2_approx(fmaf(__uint_as_float(sv[c0 + c]), L2E, -m_used));
                    const float p1 = ex2_approx(fmaf(__uint_as_float(sv[c0 + c + 1]), L2E, -m_used));
                    const __half2 hp = __floats2half2_rn(p0, p1);
                    const float2 hf = __half22float2(hp);
                    l += hf.x + hf.y;
                    pk[c >> 1] = *reinterpret_cast<const uint32_t*>(&hp);
                }
                ptx::tmem_st16(tmem + lane_off + P_COL + (c0 >> 1), pk);
            }
            ptx::tmem_st_wait();
            ptx::tc_fence_before();
            ptx::mbar_arrive(p_full);
        }
        // epilogue: ctx[row] = O / l as f16 hi (+ lo) planes
        pdl_wait();
        if (ok && ptx::mbar_wait(o_full, 0)) {
            ptx::tc_fence_after();
            const int q = q0 + r;
            const float inv = 1.0f / l;
#pragma unroll
            for (int c0 = 0; c0 < HD; c0 += 32) {
                uint32_t o[32];
                ptx::tmem_ld32(tmem + lane_off + O_COL + c0, o);
                ptx::tmem_ld_wait();
                if (q < T) {
                    const int64_t off = ((int64_t)w * T + q) * ctx_ld + h * HD + c0;
                    __align__(16) __half hi[32], lo[32];
#pragma unroll
                    for (int c = 0; c < 32; ++c) {
                        const float x = __uint_as_float(o[c]) * inv;
                        hi[c] = __float2half_rn(x);
                        lo[c] = __float2half_rn(x - __half2float(hi[c]));
                    }
#pragma unroll
                    for (int c = 0; c < 32; c += 8) {
                        *reinterpret_cast<uint4*>(ctx + off + c) = *reinterpret_cast<const uint4*>(hi + c);
                        if (ctx_lo) *reinterpret_cast<uint4*>(ctx_lo + off + c) = *reinterpret_cast<const uint4*>(lo + c);
                    }
                }
            }
        } else {
            ok = false;
        }
    }
    if (!ok && err) atomicExch(err, 1);
    __syncwarp();
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, TMEM_COLS);
    }
}

bool run_encoder_attention_tc(vkb_context* ctx, const __half* qkv, int64_t ld, int kcol, int vcol, int n_windows,
                              int T, int n_head, __half* out, int64_t out_ld, __half* out_lo, __half* vt_scratch,
                              size_t scratch_halves) {
    const int Tp = (T + 7) / 8 * 8;
    if (!vt_scratch || scratch_halves < (size_t)n_windows * n_head * HD * Tp) return false;
    if ((ld * 2) % 16 || kcol % 8 || ((uintptr_t)qkv & 15) || ((uintptr_t)vt_scratch & 15) || out_ld % 8 ||
        ((uintptr_t)out & 15) || (out_lo && ((uintptr_t)out_lo & 15)))
        return false;
    {
        dim3 grid((unsigned)((Tp + 63) / 64), (unsigned)(n_windows * n_head));
        launch_pdl(ctx, v_transpose_kernel, grid, 256, 0, qkv, ld, vcol, T, Tp, n_head, vt_scratch);
        VKB_CUDA(cudaGetLastError());
        ctx->count();
    }
    CUtensorMap qk_map, vt_map;
    make_tmap_f16(&qk_map, qkv, (int64_t)n_windows * T, ld, BQ);
    make_tmap_f16(&vt_map, vt_scratch, (int64_t)n_windows * n_head * HD, Tp, HD);
    smem_optin(enc_attn_tc_kernel, SMEM);
    dim3 grid((unsigned)((T + BQ - 1) / BQ), (unsigned)(n_windows * n_head));
    launch_pdl(ctx, enc_attn_tc_kernel, grid, 192, SMEM, qk_map, vt_map, kcol, T, n_head, out, out_ld, out_lo,
               ctx->err_flag.as<int>());
    VKB_CUDA(cudaGetLastError());
    ctx->count();
    return true;
}

}  // namespace vkb
