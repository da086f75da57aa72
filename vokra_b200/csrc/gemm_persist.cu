// gemm_persist.cu — persistent tcgen05 GEMM for the large-M Linear layers of
// the encoder (M = clips x 1500 tokens), split precision (W_hi/W_lo x X_hi/X_lo)
// or, with SPLIT = false, single f16 operands (one MMA per K=16 step).
//
// Same product as tc_gemm_kernel's non-stacked split mode (three MMAs per
// K=16 step: W_hi.X_hi + W_hi.X_lo + W_lo.X_hi, weights dequantized into
// tensor memory as the A operand, activations by TMA as the B operand), but
// one CTA per SM walks a static list of output tiles (tile t, t + grid, ...)
// and the accumulator is double-buffered in tensor memory:
//   columns [0, 192)    accumulator 0      (128 weight rows x 192 tokens, f32)
//   columns [192, 384)  accumulator 1
//   columns [384, 512)  two A stages of W_hi | W_lo (64 K each), or four of a
//                       single f16 W plane
// so the epilogue of tile i (its own 8 warps: tensor-memory load, bias, GELU /
// scale / residual, stores) runs while the MMAs of tile i+1 fill the other
// buffer, and the TMA ring never drains between tiles. The non-persistent
// kernel pays CTA setup, pipeline fill and the epilogue with the tensor pipe
// idle, once per tile.
//
// Warp roles (448 or 576 threads): warp 0 producer (one lane: weight bulk copies +
// activation TMA), warp 1 MMA issuer (one lane), warps 2-5 dequantization
// (thread = weight row = tensor-memory lane), then the epilogue: EG groups of
// four warps (two in split mode, three with single-f16 operands); a group
// covers the 128 lanes and 192 / EG of the columns.
// The epilogue needs both groups to stay shorter than a tile's MMAs at K = 1280
// (measured: one group of four made fc1's GELU epilogue the bottleneck).
// Every mbarrier wait is bounded; a timeout flags the context error.
#include "common.cuh"
#include "weights.cuh"
#include "tc_ptx.cuh"
#include "linear.cuh"

namespace vkb {

// SS = true: the weight tile arrives by TMA as f16 from a plane that
// dequant_plane_kernel wrote just before (single-f16 operands only); both MMA
// operands come from shared memory, there are no dequantization warps, and
// tensor memory holds two 256-token accumulators.
template <int FMT, bool SPLIT = true, int EG = 2, bool SS = false>
struct PCfg {
    static_assert(!(SS && SPLIT), "the f16 weight plane carries no low part");
    static constexpr int BN = SS ? 256 : 192;               // tokens per tile
    static constexpr int NP = SPLIT ? 2 : 1;                // activation planes (hi, lo)
    static constexpr int B_BYTES = BN * 128;                // one activation plane per stage
    static constexpr int RAW_Q = SS ? TILE_N * 128 : stage_qs_bytes(FMT);
    static constexpr int RAW_S = SS ? 0 : stage_sc_bytes(FMT);
    static constexpr int RAW_BYTES = ((RAW_Q + RAW_S) + 1023) / 1024 * 1024;
    static constexpr int STAGE_BYTES = NP * B_BYTES + RAW_BYTES;
    static constexpr int S0 = (225 * 1024 - 2048) / STAGE_BYTES;
    static constexpr int SMAX = SPLIT ? 4 : (SS ? 4 : 6);
    static constexpr int S = S0 > SMAX ? SMAX : S0;
    static constexpr int SMEM = 1024 + S * STAGE_BYTES + 1024;
    // A stages in tensor memory: W_hi | W_lo take 64 columns, a single f16 plane
    // 32, so the single-f16 kernel keeps four stages in the same 128 columns
    // (the dequant warps run two stages further ahead of the MMAs)
    static constexpr int A_STRIDE = SPLIT ? 64 : 32;
    static constexpr int AS = SS ? 1 : (SPLIT ? 2 : 4);  // (unused with SS)
    static constexpr int A_COL0 = 2 * BN;
    static constexpr int DEQ_WARPS = SS ? 0 : 4;
    static constexpr int EPI_WARPS = 4 * EG;  // EG groups of four warps, BN / EG columns each
    static_assert((BN / EG) % 32 == 0, "epilogue column share");
    static constexpr int THREADS = 32 * (2 + DEQ_WARPS + EPI_WARPS);
    static_assert(SS ? 2 * BN <= 512 : A_COL0 + AS * A_STRIDE <= 512, "tensor memory budget");
    static_assert(S >= 2, "pipeline needs at least two stages");
    static_assert(B_BYTES % 1024 == 0, "128-byte swizzle atoms");
};

// Two outputs (tokens m and m + 1 of one feature, ldo apart): f32 stores, or
// one paired f32 -> f16 conversion (a packing ALU instruction, where a single
// __float2half_rn is a conversion on the XU pipe, which the epilogue otherwise
// saturates) and two 2-byte stores; same round-to-nearest values.
__device__ __forceinline__ void pstore2(const PEpi& e, int64_t i, float2 x, bool v0, bool v1) {
    if (e.out_fmt == VKB_DT_F32) {
        if (v0) reinterpret_cast<float*>(e.out)[i] = x.x;
        if (v1) reinterpret_cast<float*>(e.out)[i + e.ldo] = x.y;
        return;
    }
    const __half2 h = __floats2half2_rn(x.x, x.y);
    __half* o = reinterpret_cast<__half*>(e.out);
    if (v0) o[i] = __low2half(h);
    if (v1) o[i + e.ldo] = __high2half(h);
    if (e.out_fmt == VKB_DT_F16X2) {
        const float2 hf = __half22float2(h);
        const __half2 l = __floats2half2_rn(x.x - hf.x, x.y - hf.y);
        if (v0) o[e.plane + i] = __low2half(l);
        if (v1) o[e.plane + i + e.ldo] = __high2half(l);
    }
}

// Max over the warp's 32 lanes of each of 32 values, transposed: lane l returns
// the maximum of x[l] over all lanes. A butterfly that halves the values each
// lane carries (16 + 8 + 4 + 2 + 1 shuffles, all independent within a step);
// fmaxf drops NaN as the reference's f32::max does.
__device__ __forceinline__ float transpose_max32(const float (&x)[32], int lane) {
    float a[16], b[8], c[4], d[2];
    {
        const bool hi = lane & 16;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const float keep = fabsf(hi ? x[k + 16] : x[k]), send = fabsf(hi ? x[k] : x[k + 16]);
            a[k] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 16));
        }
    }
    {
        const bool hi = lane & 8;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float keep = hi ? a[k + 8] : a[k], send = hi ? a[k] : a[k + 8];
            b[k] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 8));
        }
    }
    {
        const bool hi = lane & 4;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float keep = hi ? b[k + 4] : b[k], send = hi ? b[k] : b[k + 4];
            c[k] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 4));
        }
    }
    {
        const bool hi = lane & 2;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const float keep = hi ? c[k + 2] : c[k], send = hi ? c[k] : c[k + 2];
            d[k] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 2));
        }
    }
    const bool hi = lane & 1;
    const float keep = hi ? d[1] : d[0], send = hi ? d[0] : d[1];
    return fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 1));
}

// Store row of token m under the Q8 pair output's row-group map.
__device__ __forceinline__ int64_t q8_row(const PEpi& e, int64_t m) {
    if (!e.row_map) return m;
    const unsigned g = (unsigned)m / (unsigned)e.row_group;
    return (int64_t)e.row_map[g] * e.row_group + ((unsigned)m - g * (unsigned)e.row_group);
}

// The epilogue of one output tile for one thread: row r of the 128-row weight
// tile n_tile (tensor-memory lane r), the CG token columns from cb of the
// accumulator at column acc_col (BN tokens from m_tile * BN): bias, GELU /
// scale / residual, stores; or the Q8_0 pair output of the cross K/V store.
template <int BN, int CG>
__device__ __forceinline__ void persist_epilogue_tile(const PEpi& e, uint32_t lane_base, uint32_t acc_col, int n_tile,
                                                      int m_tile, int r, int cb, int lane, int64_t N, int64_t M) {
                const int64_t n = (int64_t)n_tile * TILE_N + r;
                const bool nv = n < N;
                if (e.q8_width > 0) {
                    // Q8_0 pair output: this warp's 32 rows (features) are one 32-channel block of the
                    // K or V store row of each token (BlockQ8_0::pack, q8_0.rs:40-66), 32 tokens at a time
                    const int half = n_tile * TILE_N >= e.q8_width;
                    const int64_t c = n - half * e.q8_width;
                    const int blk = (int)(c >> 5), nb = (int)(e.q8_width >> 5);
                    int8_t* qb = half ? e.q8[1] : e.q8[0];
                    __half* db = half ? e.q8d[1] : e.q8d[0];
                    const float bias_q = e.bias ? e.bias[n] : 0.0f;
    #pragma unroll 1
                    for (int c0 = cb; c0 < cb + CG; c0 += 32) {
                        uint32_t v[32];
                        ptx::tmem_ld32(lane_base + acc_col + c0, v);
                        ptx::tmem_ld_wait();
                        const int64_t m0 = (int64_t)m_tile * BN + c0;
                        float x[32];
    #pragma unroll
                        for (int j = 0; j < 32; ++j) x[j] = __uint_as_float(v[j]) + bias_q;
                        // lane l ends with the block amax of token m0 + l, then its scale and inverse
                        const float amax = fmaxf(0.0f, transpose_max32(x, lane));
                        const float dq = amax == 0.0f ? 0.0f : amax / 127.0f;
                        const float inv = dq == 0.0f ? 0.0f : 1.0f / dq;
                        const int64_t my_m = m0 + lane;
                        if (my_m < M)
                            *reinterpret_cast<uint16_t*>(db + q8_row(e, my_m) * nb + blk) = f32_to_f16_bits(dq);
    #pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const float inv_j = __shfl_sync(0xffffffffu, inv, j);
                            if (m0 + j >= M) continue;  // uniform across the warp
                            const float sq = x[j] * inv_j;
                            const float c = sq < -127.0f ? -127.0f : (sq > 127.0f ? 127.0f : sq);
                            qb[q8_row(e, m0 + j) * e.q8_width + blk * 32 + lane] = isnan(c) ? (int8_t)0 : (int8_t)(int)roundf(c);
                        }
                    }
                    return;
                }
                const float bias_n = (nv && e.bias) ? e.bias[n] : 0.0f;
                const float scl = (e.kind == VKB_EPI_SCALE && n < e.n_scaled) ? e.scale : 1.0f;
    #pragma unroll 1
                for (int c0 = cb; c0 < cb + CG; c0 += 32) {
                    uint32_t v[32];
                    ptx::tmem_ld32(lane_base + acc_col + c0, v);
                    ptx::tmem_ld_wait();
                    const int64_t m0 = (int64_t)m_tile * BN + c0;
                    if (nv) {
                        if (e.kind == VKB_EPI_RESIDUAL) {
                            // all 32 residual loads in flight before any store (out may alias residual)
                            float res[32];
    #pragma unroll
                            for (int j = 0; j < 32; ++j)
                                res[j] = (m0 + j < M) ? e.residual[(m0 + j) * e.ldo + n] : 0.0f;
    #pragma unroll
                            for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + res[j]);
                        }
    #pragma unroll
                        for (int j = 0; j < 32; j += 2) {
                            float2 x = make_float2(__uint_as_float(v[j]) + bias_n, __uint_as_float(v[j + 1]) + bias_n);
                            if (e.kind == VKB_EPI_GELU) {
                                x = gelu_as_fast2(x);
                            } else {
                                x.x *= scl;
                                x.y *= scl;
                            }
                            pstore2(e, (m0 + j) * e.ldo + n, x, m0 + j < M, m0 + j + 1 < M);
                        }
                    }
                }
}

template <int FMT, bool SPLIT, int EG, bool SS>
__global__ void __launch_bounds__(PCfg<FMT, SPLIT, EG, SS>::THREADS, 1)
    tc_gemm_persist_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap xmap_lo,
                           const __grid_constant__ CUtensorMap wmap, const uint8_t* __restrict__ qs,
                           const uint8_t* __restrict__ sc, int64_t K, int64_t N, int64_t M, int n_tiles,
                           int total_tiles, PEpi e, int* err) {
    using C = PCfg<FMT, SPLIT, EG, SS>;
    constexpr int BN = C::BN, S = C::S, AS = C::AS;
    constexpr int CG = BN / EG;  // columns per epilogue group
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + S * C::STAGE_BYTES);
    uint64_t* empty = full + S;
    uint64_t* a_full = empty + S;
    uint64_t* a_empty = a_full + AS;
    uint64_t* acc_full = a_empty + AS;   // [2]
    uint64_t* acc_empty = acc_full + 2;  // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nst = (int)(K / STAGE_K);
    const int first = blockIdx.x, stride = gridDim.x;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            ptx::mbar_init(&full[i], 1);
            ptx::mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < AS; ++i) {
            ptx::mbar_init(&a_full[i], 32 * C::DEQ_WARPS);
            ptx::mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            ptx::mbar_init(&acc_full[i], 1);
            ptx::mbar_init(&acc_empty[i], C::EPI_WARPS);
        }
        ptx::fence_mbar_init();
    }
    if (warp == 1) {
        ptx::tmem_alloc(tmem_slot, 512);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;
    // Programmatic dependent launch: weights are never written by a kernel, so
    // the first ring stages' weights are fetched before waiting for the
    // previous kernel; activations (producer) and outputs (epilogue) wait.
    pdl_launch();

    if (warp == 0) {
        if (lane == 0) {
            auto load_weights = [&](int s, int n_tile, int i) {
                uint8_t* raw_dst = ring + s * C::STAGE_BYTES + C::NP * C::B_BYTES;
                if constexpr (SS) {
                    ptx::mbar_expect_tx(&full[s], C::NP * C::B_BYTES + C::RAW_Q);
                    ptx::tma_load_2d(raw_dst, &wmap, &full[s], i * STAGE_K, n_tile * TILE_N);
                    return;
                }
                StagePtrs p = stage_ptrs(FMT, qs, sc, K, n_tile, i);
                ptx::mbar_expect_tx(&full[s], C::NP * C::B_BYTES + C::RAW_Q + C::RAW_S);
                ptx::bulk_load(raw_dst, p.qs, C::RAW_Q, &full[s]);
                if (C::RAW_S) ptx::bulk_load(raw_dst + C::RAW_Q, p.sc, C::RAW_S, &full[s]);
            };
            const int pre = nst < S ? nst : S;
            // the f16 weight plane is written by the kernel before this one
            if (SS) pdl_wait();
            for (int i = 0; i < pre; ++i) load_weights(i, first % n_tiles, i);
            if (!SS) pdl_wait();
            int g = 0;
            for (int t = first; t < total_tiles && ok; t += stride) {
                const int n_tile = t % n_tiles, m_tile = t / n_tiles;
                for (int i = 0; i < nst; ++i, ++g) {
                    const int s = g % S;
                    if (g >= pre) {
                        if (!ptx::mbar_wait(&empty[s], ((g / S) & 1) ^ 1)) {
                            ok = false;
                            break;
                        }
                        load_weights(s, n_tile, i);
                    }
                    uint8_t* b_dst = ring + s * C::STAGE_BYTES;
                    ptx::tma_load_2d(b_dst, &xmap, &full[s], i * STAGE_K, m_tile * BN);
                    if (SPLIT) ptx::tma_load_2d(b_dst + C::B_BYTES, &xmap_lo, &full[s], i * STAGE_K, m_tile * BN);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = ptx::idesc_f16_f32(TILE_N, BN);
            int g = 0, tt = 0;
            for (int t = first; t < total_tiles && ok; t += stride, ++tt) {
                const int b = tt & 1;
                if (!ptx::mbar_wait(&acc_empty[b], ((tt >> 1) & 1) ^ 1)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t d_t = tmem + b * BN;
                for (int i = 0; i < nst; ++i, ++g) {
                    const int s = g % S;
                    if constexpr (SS) {
                        if (!ptx::mbar_wait(&full[s], (g / S) & 1)) {
                            ok = false;
                            break;
                        }
                        ptx::tc_fence_after();
                        const uint32_t b_addr = ptx::smem_u32(ring + s * C::STAGE_BYTES);
                        const uint32_t w_addr = b_addr + C::NP * C::B_BYTES;
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            ptx::mma_f16_ss(d_t, ptx::sdesc_sw128(w_addr + kk * 32), ptx::sdesc_sw128(b_addr + kk * 32),
                                            idesc, (i > 0 || kk > 0) ? 1u : 0u);
                        ptx::mma_commit(&empty[s]);
                        continue;
                    }
                    const int a = g % AS;
                    if (!ptx::mbar_wait(&full[s], (g / S) & 1) || !ptx::mbar_wait(&a_full[a], (g / AS) & 1)) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    const uint32_t a_t = tmem + C::A_COL0 + a * C::A_STRIDE;
                    const uint32_t b_addr = ptx::smem_u32(ring + s * C::STAGE_BYTES);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t bd = ptx::sdesc_sw128(b_addr + kk * 32);
                        ptx::mma_f16_ts(d_t, a_t + kk * 8, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
                        if (SPLIT) {
                            const uint64_t bd_lo = ptx::sdesc_sw128(b_addr + C::B_BYTES + kk * 32);
                            ptx::mma_f16_ts(d_t, a_t + kk * 8, bd_lo, idesc, 1u);
                            ptx::mma_f16_ts(d_t, a_t + 32 + kk * 8, bd, idesc, 1u);
                        }
                    }
                    ptx::mma_commit(&empty[s]);
                    ptx::mma_commit(&a_empty[a]);
                }
                if (!ok) break;
                ptx::mma_commit(&acc_full[b]);
            }
        }
    } else if (!SS && warp < 2 + C::DEQ_WARPS) {
        // dequantization: row r of the 128-row weight tile = tensor-memory lane r
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        int g = 0;
        for (int t = first; t < total_tiles && ok; t += stride) {
            for (int i = 0; i < nst; ++i, ++g) {
                const int s = g % S, a = g % AS;
                if (!ptx::mbar_wait(&full[s], (g / S) & 1) || !ptx::mbar_wait(&a_empty[a], ((g / AS) & 1) ^ 1)) {
                    ok = false;
                    break;
                }
                const uint8_t* raw = ring + s * C::STAGE_BYTES + C::NP * C::B_BYTES;
                const uint32_t a_t = tmem + ((uint32_t)(quarter * 32) << 16) + C::A_COL0 + a * C::A_STRIDE;
                uint32_t hi[32], lo[32];
                dequant_row_stage_h<FMT, SPLIT>(raw, raw + C::RAW_Q, r, i, hi, lo);
                ptx::tc_fence_after();
                ptx::tmem_st32(a_t, hi);
                if (SPLIT) ptx::tmem_st32(a_t + 32, lo);
                ptx::tmem_st_wait();
                ptx::tc_fence_before();
                ptx::mbar_arrive(&a_full[a]);
            }
        }
    } else {
        // epilogue: warp w reads lane quarter w % 4; group (w - 6) / 4 takes half the columns
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const int cb = ((warp - 2 - C::DEQ_WARPS) >> 2) * CG;
        const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
        pdl_wait();
        int tt = 0;
        for (int t = first; t < total_tiles && ok; t += stride, ++tt) {
            const int b = tt & 1;
            const int n_tile = t % n_tiles, m_tile = t / n_tiles;
            if (!ptx::mbar_wait(&acc_full[b], (tt >> 1) & 1)) {
                ok = false;
                break;
            }
            ptx::tc_fence_after();
            persist_epilogue_tile<BN, CG>(e, lane_base, (uint32_t)(b * BN), n_tile, m_tile, r, cb, lane, N, M);
            // accumulator buffer b may be overwritten by the MMAs of tile tt + 2
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&acc_empty[b]);
        }
    }
    if (!ok && err) atomicExch(err, 1);
    __syncwarp();
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, 512);
    }
}

int persist_bn() { return PCfg<W_Q4_0>::BN; }

// The f16 weight plane of the SS kernel: row n of the (padded) weight, K
// halves, row-major, each value the f16 the TMEM path's dequantization warps
// would produce (dequant_row_stage_h, single f16). One CTA per (stage, tile),
// thread = weight row: 64 halves = 128 contiguous bytes per thread.
template <int FMT>
__global__ void __launch_bounds__(TILE_N) dequant_plane_kernel(const uint8_t* __restrict__ qs,
                                                               const uint8_t* __restrict__ sc, int64_t K,
                                                               __half* __restrict__ plane) {
    // the plane may still be read by the GEMM launched before this kernel
    pdl_entry();
    const int i = blockIdx.x, n_tile = blockIdx.y, r = threadIdx.x;
    const StagePtrs p = stage_ptrs(FMT, qs, sc, K, n_tile, i);
    uint32_t hi[32], lo[32];
    dequant_row_stage_h<FMT, false>(p.qs, p.sc, r, i, hi, lo);
    uint4* dst = reinterpret_cast<uint4*>(plane + ((int64_t)n_tile * TILE_N + r) * K + (int64_t)i * STAGE_K);
#pragma unroll
    for (int j = 0; j < 8; ++j) dst[j] = make_uint4(hi[4 * j], hi[4 * j + 1], hi[4 * j + 2], hi[4 * j + 3]);
}

// ---------------------------------------------------------------------------
// The same single-f16 GEMM on CTA pairs (tcgen05 cta_group::2): a cluster of
// two CTAs on two SMs computes a 256 weight rows x 256 tokens tile with one
// M = 256 MMA issued by the even CTA. Each CTA loads its own 128 weight rows
// and half of the token tile (128 tokens) into the same shared-memory offsets
// and holds its 128 weight rows x 256 tokens of the accumulator in its own
// tensor memory, so a CTA reads 32 KB per 64-K stage (16 KB weights + 16 KB
// tokens) for the product the single-CTA kernel reads 48 KB for, and six
// stages fit. No multicast loads: each CTA's TMA load lands in its own shared
// memory and signals the even CTA's barrier (the cta_group::2 form).
//   barriers  full[s] (even CTA: arrive + expect_tx of both CTAs' bytes),
//             empty[s] / acc_full[b] in both CTAs (one tcgen05.commit
//             multicast to the pair), acc_empty[b] (even CTA: every epilogue
//             warp of both CTAs arrives)
//   TMEM      512 columns per CTA (cta_group::2 allocation): two 256-token
//             accumulators
// Every wait is bounded; both CTAs meet at a cluster barrier before the
// tensor memory is freed.
// ---------------------------------------------------------------------------
namespace pairx {
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t n_clusters() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// shared::cluster address of the same shared-memory object in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_to(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(ptx::smem_u32(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void arrive_remote(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
// 2-D tiled load into this CTA's shared memory whose completion is counted on
// the barrier at bar_cluster (the even CTA's), no multicast
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int32_t x,
                                                 int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(ptx::smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc2(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(ptx::smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void mma_f16_ss2(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// arrives once on the barrier at the same offset in both CTAs of the pair when
// the MMAs issued so far complete
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            ptx::smem_u32(bar)),
        "h"((uint16_t)0x3)
        : "memory");
}
}  // namespace pairx

template <int EG>
struct PairCfg {
    static constexpr int BN = 256;                // tokens per pair tile (128 loaded by each CTA)
    static constexpr int A_BYTES = TILE_N * 128;  // this CTA's 128 weight rows x 64 halves
    static constexpr int B_BYTES = 128 * 128;     // this CTA's 128 tokens x 64 halves
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int S = 6;
    static constexpr int SMEM = 1024 + S * STAGE_BYTES + 1024;
    static constexpr int CG = BN / EG;
    static constexpr int EPI_WARPS = 4 * EG;
    static constexpr int THREADS = 32 * (2 + EPI_WARPS);
    static_assert(SMEM <= 227 * 1024, "shared memory");
};

template <int EG>
__global__ void __launch_bounds__(PairCfg<EG>::THREADS, 1)
    tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap, int64_t K,
                        int64_t N, int64_t M, int n_pairs, int total_tiles, PEpi e, int* err) {
    using C = PairCfg<EG>;
    constexpr int BN = C::BN, S = C::S, CG = C::CG;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + S * C::STAGE_BYTES);
    uint64_t* empty = full + S;
    uint64_t* acc_full = empty + S;      // [2]
    uint64_t* acc_empty = acc_full + 2;  // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = pairx::cluster_rank();
    const bool lead = rank == 0;
    const int nst = (int)(K / STAGE_K);
    const int first = (int)pairx::cluster_id(), stride = (int)pairx::n_clusters();

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            ptx::mbar_init(&full[i], 1);
            ptx::mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            ptx::mbar_init(&acc_full[i], 1);
            ptx::mbar_init(&acc_empty[i], 2 * C::EPI_WARPS);
        }
        ptx::fence_mbar_init();
    }
    if (warp == 1) {
        pairx::tmem_alloc2(tmem_slot, 512);
        pairx::tmem_relinquish2();
    }
    ptx::tc_fence_before();
    // both CTAs' barriers are initialized before either CTA's loads or commits reach them
    pairx::cluster_sync();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;
    pdl_launch();
    // the activations and the f16 weight plane are written by earlier kernels
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            int g = 0;
            for (int t = first; t < total_tiles && ok; t += stride) {
                const int pr = t % n_pairs, m_tile = t / n_pairs;
                for (int i = 0; i < nst; ++i, ++g) {
                    const int s = g % S;
                    if (g >= S && !ptx::mbar_wait(&empty[s], ((g / S) & 1) ^ 1)) {
                        ok = false;
                        break;
                    }
                    const uint32_t bar = pairx::map_to(&full[s], 0);
                    if (lead) ptx::mbar_expect_tx(&full[s], 2 * C::STAGE_BYTES);
                    uint8_t* dst = ring + s * C::STAGE_BYTES;
                    pairx::tma_load_2d_pair(dst, &wmap, bar, i * STAGE_K, (2 * pr + (int)rank) * TILE_N);
                    pairx::tma_load_2d_pair(dst + C::A_BYTES, &xmap, bar, i * STAGE_K, m_tile * BN + (int)rank * 128);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && lead) {
            constexpr uint32_t idesc = ptx::idesc_f16_f32(2 * TILE_N, BN);
            int g = 0, tt = 0;
            for (int t = first; t < total_tiles && ok; t += stride, ++tt) {
                const int b = tt & 1;
                if (!ptx::mbar_wait(&acc_empty[b], ((tt >> 1) & 1) ^ 1)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t d_t = tmem + b * BN;
                for (int i = 0; i < nst; ++i, ++g) {
                    const int s = g % S;
                    if (!ptx::mbar_wait(&full[s], (g / S) & 1)) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    const uint32_t w_addr = ptx::smem_u32(ring + s * C::STAGE_BYTES);
                    const uint32_t x_addr = w_addr + C::A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        pairx::mma_f16_ss2(d_t, ptx::sdesc_sw128(w_addr + kk * 32), ptx::sdesc_sw128(x_addr + kk * 32),
                                           idesc, (i > 0 || kk > 0) ? 1u : 0u);
                    pairx::mma_commit_pair(&empty[s]);
                }
                if (!ok) break;
                pairx::mma_commit_pair(&acc_full[b]);
            }
        }
    } else {
        // epilogue: this CTA's 128 weight rows (tile 2 * pair + rank) x the pair tile's 256 tokens
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const int cb = ((warp - 2) >> 2) * CG;
        const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
        int tt = 0;
        for (int t = first; t < total_tiles && ok; t += stride, ++tt) {
            const int b = tt & 1;
            const int pr = t % n_pairs, m_tile = t / n_pairs;
            if (!ptx::mbar_wait(&acc_full[b], (tt >> 1) & 1)) {
                ok = false;
                break;
            }
            ptx::tc_fence_after();
            persist_epilogue_tile<BN, CG>(e, lane_base, (uint32_t)(b * BN), 2 * pr + (int)rank, m_tile, r, cb, lane, N,
                                          M);
            // accumulator buffer b of both CTAs may be overwritten by the MMAs of tile tt + 2
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) pairx::arrive_remote(pairx::map_to(&acc_empty[b], 0));
        }
    }
    if (!ok && err) atomicExch(err, 1);
    __syncwarp();
    ptx::tc_fence_before();
    __syncthreads();
    // the even CTA's MMAs read this CTA's shared memory and write its tensor memory
    pairx::cluster_sync();
    if (warp == 1) {
        ptx::tc_fence_after();
        pairx::tmem_dealloc2(tmem, 512);
    }
}

template <int FMT, int EG>
static void launch_pair(vkb_context* ctx, const vkb_weight* w, int64_t m, const __half* a16, const PEpi& e, int* err) {
    using C = PairCfg<EG>;
    const size_t bytes = (size_t)w->n_pad * w->k * sizeof(__half);
    if (ctx->wplane.n < bytes) {
        VKB_CUDA(cudaStreamSynchronize(ctx->stream));
        ctx->wplane.alloc(bytes);
    }
    launch_pdl(ctx, dequant_plane_kernel<FMT>, dim3((unsigned)(w->k / STAGE_K), (unsigned)(w->n_pad / TILE_N)), TILE_N, 0,
               w->qs.as<uint8_t>(), w->sc.as<uint8_t>(), w->k, ctx->wplane.as<__half>());
    VKB_CUDA(cudaGetLastError());
    ctx->count();
    smem_optin(tc_gemm_pair_kernel<EG>, C::SMEM);
    CUtensorMap xmap, wmap;
    make_tmap_f16(&xmap, a16, m, w->k, 128);
    make_tmap_f16(&wmap, ctx->wplane.p, w->n_pad, w->k, TILE_N);
    const int n_pairs = (int)((w->n_pad / TILE_N + 1) / 2);
    const int m_tiles = (int)((m + C::BN - 1) / C::BN);
    const int total = n_pairs * m_tiles;
    const int clusters = std::min(total, ctx->sm_count / 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * clusters));
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = ctx->pdl ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    VKB_CUDA(cudaLaunchKernelEx(&cfg, tc_gemm_pair_kernel<EG>, xmap, wmap, (int64_t)w->k, (int64_t)w->n, m, n_pairs,
                                total, e, err));
    ctx->count();
}

template <int FMT, bool SPLIT, int EG, bool SS>
static void launch_persist(vkb_context* ctx, const vkb_weight* w, int64_t m, const __half* a16, const PEpi& e,
                           int* err) {
    using C = PCfg<FMT, SPLIT, EG, SS>;
    smem_optin(tc_gemm_persist_kernel<FMT, SPLIT, EG, SS>, C::SMEM);
    CUtensorMap map, map_lo, wmap;
    make_tmap_f16(&map, a16, m, w->k, C::BN);
    if (SPLIT) make_tmap_f16(&map_lo, a16 + m * w->k, m, w->k, C::BN);
    else map_lo = map;
    const int n_tiles = (int)(w->n_pad / TILE_N);
    if (SS) {
        const size_t bytes = (size_t)w->n_pad * w->k * sizeof(__half);
        if (ctx->wplane.n < bytes) {
            VKB_CUDA(cudaStreamSynchronize(ctx->stream));
            ctx->wplane.alloc(bytes);
        }
        launch_pdl(ctx, dequant_plane_kernel<FMT>, dim3((unsigned)(w->k / STAGE_K), (unsigned)n_tiles), TILE_N, 0,
                   w->qs.as<uint8_t>(), w->sc.as<uint8_t>(), w->k, ctx->wplane.as<__half>());
        VKB_CUDA(cudaGetLastError());
        ctx->count();
        make_tmap_f16(&wmap, ctx->wplane.p, w->n_pad, w->k, TILE_N);
    } else {
        wmap = map;
    }
    const int m_tiles = (int)((m + C::BN - 1) / C::BN);
    const int total = n_tiles * m_tiles;
    const int grid = std::min(total, ctx->sm_count);
    launch_pdl(ctx, tc_gemm_persist_kernel<FMT, SPLIT, EG, SS>, grid, C::THREADS, C::SMEM, map, map_lo, wmap,
               w->qs.as<uint8_t>(), w->sc.as<uint8_t>(), w->k, w->n, m, n_tiles, total, e, err);
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}

// Whether single-f16 GEMMs of large M run on the SS kernel (VKB_GEMM_SS=0: the
// TMEM-operand kernel with in-kernel dequantization).
// Read at every call (a host-side getenv per large GEMM), so one process can compare both kernels.
bool persist_ss_enabled() {
    const char* v = std::getenv("VKB_GEMM_SS");
    return !v || v[0] != '0';
}

// Whether single-f16 large-M GEMMs run on CTA pairs (tc_gemm_pair_kernel, the default: fc1 at
// M = 96000 1.073 ms against 1.098 ms on one CTA per tile); VKB_GEMM_PAIR=0 selects the single-CTA
// kernel. Read at every call, like persist_ss_enabled.
bool persist_pair_enabled() {
    const char* v = std::getenv("VKB_GEMM_PAIR");
    return !v || v[0] != '0';
}

void run_tc_persistent(vkb_context* ctx, const vkb_weight* w, int64_t m, const __half* a16, const PEpi& e, int* err,
                       bool split) {
    // single-f16 operands: three epilogue groups (the MMAs of a tile are a third of the split
    // mode's, so fc1's GELU epilogue is the longer phase with two; measured 812 vs 819 ms per
    // bench step); VKB_PERSIST_EPI_GROUPS=2 selects two
    static const int groups = [] { const char* v = std::getenv("VKB_PERSIST_EPI_GROUPS"); return v ? std::atoi(v) : 3; }();
    // shared-memory operands: four epilogue groups of four warps (fc1 1.056 ms against 1.170 ms with two:
    // with no dequantization warps the epilogue is the longer phase of a tile); VKB_SS_EPI_GROUPS=2 selects two
    static const int ss_groups = [] { const char* v = std::getenv("VKB_SS_EPI_GROUPS"); return v ? std::atoi(v) : 4; }();
    with_fmt(w->fmt, [&](auto F) {
        constexpr int FM = decltype(F)::value;
        if (split) launch_persist<FM, true, 2, false>(ctx, w, m, a16, e, err);
        else if (persist_ss_enabled() && persist_pair_enabled()) launch_pair<FM, 4>(ctx, w, m, a16, e, err);
        else if (persist_ss_enabled() && ss_groups == 2) launch_persist<FM, false, 2, true>(ctx, w, m, a16, e, err);
        else if (persist_ss_enabled()) launch_persist<FM, false, 4, true>(ctx, w, m, a16, e, err);
        else if (groups == 3) launch_persist<FM, false, 3, false>(ctx, w, m, a16, e, err);
        else launch_persist<FM, false, 2, false>(ctx, w, m, a16, e, err);
    });
}

}  // namespace vkb
