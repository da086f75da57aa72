// common.cuh — shared host/device helpers of libvkb200 (sm_100a only).
#pragma once
#include <utility>
#include <mutex>
#include <set>
#include <tuple>

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <cstddef>
#include <cstring>
#include <string>
#include <vector>
#include <stdexcept>

#include "../../include/vkb200.h"
#include <nvtx3/nvToolsExt.h>

namespace vkb {

// Error carried through the C++ layer and converted to vkb_status at the ABI.
struct Error : std::runtime_error {
    vkb_status code;
    Error(vkb_status c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] inline void fail(vkb_status c, const std::string& m) { throw Error(c, m); }

inline void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess)
        fail(VKB_ERROR_BACKEND_UNAVAILABLE, std::string(what) + ": " + cudaGetErrorString(e));
}
#define VKB_CUDA(x) ::vkb::cuda_check((x), #x)

// Opts a kernel into `bytes` of dynamic shared memory on the current device.
// The attribute belongs to the device's context, so it is recorded per
// (kernel, device, bytes) and set once for each device a process uses.
template <class F>
inline void smem_optin(F* kernel, int bytes) {
    static std::mutex mu;
    static std::set<std::tuple<const void*, int, int>> done;
    int dev = 0;
    VKB_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> g(mu);
    auto key = std::make_tuple((const void*)kernel, dev, bytes);
    if (done.count(key)) return;
    VKB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done.insert(key);
}

void set_last_error(const std::string& m);

// Runs `f` and converts every exception into a status (the ffi_guard firewall).
template <class F>
vkb_status guard(F&& f) {
    try {
        f();
        return VKB_OK;
    } catch (const Error& e) {
        set_last_error(e.what());
        return e.code;
    } catch (const std::exception& e) {
        set_last_error(std::string("internal error: ") + e.what());
        return VKB_ERROR_PANIC;
    } catch (...) {
        set_last_error("internal error: unknown exception");
        return VKB_ERROR_PANIC;
    }
}

// Device-memory buffer owned by RAII (allocated only at set-up time).
struct DevBuf {
    void* p = nullptr;
    size_t n = 0;
    DevBuf() = default;
    explicit DevBuf(size_t bytes) { alloc(bytes); }
    void alloc(size_t bytes) {
        release();
        if (bytes) VKB_CUDA(cudaMalloc(&p, bytes));
        n = bytes;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
    ~DevBuf() { release(); }
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : p(o.p), n(o.n) { o.p = nullptr; o.n = 0; }
    DevBuf& operator=(DevBuf&& o) noexcept {
        release();
        p = o.p; n = o.n; o.p = nullptr; o.n = 0;
        return *this;
    }
    template <class T> T* as() const { return reinterpret_cast<T*>(p); }
};

}  // namespace vkb

// The context: one per GPU. Owns a stream and a grow-at-setup workspace that
// kernels with split reductions use for their partial sums.
struct vkb_context {
    int device = 0;
    int sm_count = 148;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    uint64_t launches = 0;
    int precision = VKB_PREC_SPLIT;  // tensor-core operand precision (vkb_context_set_precision)
    vkb::DevBuf workspace;
    vkb::DevBuf err_flag;  // int set by a kernel whose bounded wait gave up
    vkb::DevBuf tile_ctr;  // per-tile arrival counters of in-kernel split-K reductions (each returns to 0)
    vkb::DevBuf frontend;  // log-mel tables (window, twiddles, mel bank) + per-clip maxima
    int frontend_mels = 0; // mel count the tables were built for
    vkb::DevBuf wplane;    // f16 weight plane of the SS encoder GEMM (n_pad x k halves, grown on first use)
    // Programmatic dependent launch: each kernel may start while the previous
    // one in the stream drains; it waits (griddepcontrol.wait) before touching
    // anything that kernel wrote (VKB_PDL=0 turns it off).
    bool pdl = true;
    void ensure_workspace(size_t bytes) {
        if (workspace.n < bytes) {
            VKB_CUDA(cudaStreamSynchronize(stream));
            workspace.alloc(bytes);
        }
    }
    void count(int n = 1) { launches += (uint64_t)n; }
};

namespace vkb {

// NVTX range for the duration of a scope (header-only NVTX 3: a no-op unless a
// profiler attaches): one per kernel family at the entry points, so a timeline
// shows the log-mel frontend, the encoder, the decode step and each Linear.
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

constexpr int kTileCounters = 1 << 16;  // weight tiles a split-K GEMV launch may count (N <= 8M rows)

// Launch with programmatic stream serialization (see vkb_context::pdl). Every
// kernel launched this way calls pdl_wait() before reading or writing memory
// that an earlier kernel in the stream may still be using.
template <typename... KArgs, typename... Args>
inline void launch_pdl(vkb_context* ctx, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = ctx->pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    VKB_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

// Lets the next kernel in the stream be scheduled (it still waits for this
// one's memory in its own pdl_wait()).
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Waits until the previous kernel in the stream has completed and its memory
// operations are visible.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_entry() {
    pdl_launch();
    pdl_wait();
}

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Exact half -> single on the host (every f16 value is an f32 value).
inline float f16_bits_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31, ex = (h >> 10) & 0x1f, mant = h & 0x3ff;
    uint32_t bits;
    if (ex == 0) {
        if (mant == 0) {
            bits = sign;
        } else {  // subnormal: normalise
            int e = -1;
            uint32_t m = mant;
            do { m <<= 1; ++e; } while (!(m & 0x400));
            bits = sign | (uint32_t)(127 - 15 - e) << 23 | (m & 0x3ff) << 13;
        }
    } else if (ex == 31) {
        bits = sign | 0x7f800000u | mant << 13;
    } else {
        bits = sign | (ex + 112) << 23 | mant << 13;
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

// IEEE single -> half, round to nearest even; restates the reference encoder
// f32_to_f16_bits (crates/vokra-core/src/kv_quant/half.rs:80-155) so that the
// stored scale bits match it exactly, including NaN canonicalisation.
__host__ __device__ __forceinline__ uint16_t f32_to_f16_bits(float x) {
    uint32_t bits;
#ifdef __CUDA_ARCH__
    bits = __float_as_uint(x);
#else
    memcpy(&bits, &x, 4);
#endif
    uint32_t sign = (bits >> 31) & 1u;
    int exp_f32 = (int)((bits >> 23) & 0xffu);
    uint32_t mant = bits & 0x7fffffu;
    if (exp_f32 == 0xff) {
        if (mant == 0) return (uint16_t)((sign << 15) | (0x1fu << 10));
        return (uint16_t)((sign << 15) | (0x1fu << 10) | 0x200u);
    }
    if (exp_f32 == 0 && mant == 0) return (uint16_t)(sign << 15);
    int e16 = exp_f32 - 127 + 15;
    if (e16 >= 0x1f) return (uint16_t)((sign << 15) | (0x1fu << 10));
    if (e16 >= 1) {
        uint32_t rb = (mant >> 12) & 1u;
        bool sticky = (mant & 0xfffu) != 0;
        uint32_t tr = mant >> 13;
        uint32_t r = tr + ((rb && (sticky || (tr & 1u))) ? 1u : 0u);
        uint32_t e = (uint32_t)e16;
        if (r == 0x400u) {
            r = 0;
            e += 1;
            if (e >= 0x1fu) return (uint16_t)((sign << 15) | (0x1fu << 10));
        }
        return (uint16_t)((sign << 15) | (e << 10) | (r & 0x3ffu));
    }
    if (e16 < -10) return (uint16_t)(sign << 15);
    uint32_t mi = mant | 0x800000u;
    uint32_t sh = (uint32_t)(1 - e16) + 13u;
    uint32_t rb = (mi >> (sh - 1)) & 1u;
    bool sticky = (mi & ((1u << (sh - 1)) - 1u)) != 0;
    uint32_t tr = mi >> sh;
    uint32_t r = tr + ((rb && (sticky || (tr & 1u))) ? 1u : 0u);
    if (r >= 0x400u) return (uint16_t)((sign << 15) | (1u << 10));
    return (uint16_t)((sign << 15) | (r & 0x3ffu));
}

// Abramowitz & Stegun 7.1.26 erf with the reference's constants
// (crates/vokra-backend-cpu/src/kernels/scalar.rs:127-157) and exact GELU
// (scalar.rs:166). expf is CUDA's own.
__device__ __forceinline__ float gelu_as(float v) {
    const float P = 0.3275911f, A1 = 0.254829592f, A2 = -0.284496736f, A3 = 1.421413741f,
                A4 = -1.453152027f, A5 = 1.061405429f;
    float x = v * 0.70710678118654752f;
    float sign = x < 0.0f ? -1.0f : 1.0f;
    x = fabsf(x);
    float t = 1.0f / (1.0f + P * x);
    float poly = ((((A5 * t + A4) * t + A3) * t + A2) * t + A1) * t;
    float y = 1.0f - poly * expf(-x * x);
    return 0.5f * v * (1.0f + sign * y);
}

// The same formula and constants evaluated with CUDA's fast exponential and
// division intrinsics (a few ulp from gelu_as; used in GEMM epilogues, where
// the full-precision version dominated the tile's epilogue time).
__device__ __forceinline__ float gelu_as_fast(float v) {
    const float P = 0.3275911f, A1 = 0.254829592f, A2 = -0.284496736f, A3 = 1.421413741f,
                A4 = -1.453152027f, A5 = 1.061405429f;
    const float x = fabsf(v * 0.70710678118654752f);
    const float t = __fdividef(1.0f, 1.0f + P * x);
    const float poly = ((((A5 * t + A4) * t + A3) * t + A2) * t + A1) * t;
    const float y = 1.0f - poly * __expf(-x * x);
    return 0.5f * v * (1.0f + copysignf(y, v));
}

// gelu_as_fast on two values with packed f32x2 arithmetic (same operations
// and rounding per element; half the floating-point instructions).
__device__ __forceinline__ float2 gelu_as_fast2(float2 v) {
    const float2 P = make_float2(0.3275911f, 0.3275911f), one = make_float2(1.0f, 1.0f);
    const float2 A1 = make_float2(0.254829592f, 0.254829592f), A2 = make_float2(-0.284496736f, -0.284496736f),
                 A3 = make_float2(1.421413741f, 1.421413741f), A4 = make_float2(-1.453152027f, -1.453152027f),
                 A5 = make_float2(1.061405429f, 1.061405429f);
    float2 x = __fmul2_rn(v, make_float2(0.70710678118654752f, 0.70710678118654752f));
    x.x = fabsf(x.x);
    x.y = fabsf(x.y);
    const float2 den = __ffma2_rn(P, x, one);
    const float2 t = make_float2(__fdividef(1.0f, den.x), __fdividef(1.0f, den.y));
    float2 poly = __ffma2_rn(A5, t, A4);
    poly = __ffma2_rn(poly, t, A3);
    poly = __ffma2_rn(poly, t, A2);
    poly = __ffma2_rn(poly, t, A1);
    poly = __fmul2_rn(poly, t);
    const float2 xx = __fmul2_rn(x, x);
    const float2 ex = make_float2(__expf(-xx.x), __expf(-xx.y));
    const float2 y = __ffma2_rn(make_float2(-poly.x, -poly.y), ex, one);
    const float2 hv = __fmul2_rn(make_float2(0.5f, 0.5f), v);
    return __fmul2_rn(hv, __fadd2_rn(one, make_float2(copysignf(y.x, v.x), copysignf(y.y, v.y))));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// One Q8_0 block of 32 values held by the 32 lanes of a warp: the arithmetic
// of BlockQ8_0::pack (crates/vokra-core/src/kv_quant/q8_0.rs:40-66) in IEEE
// fp32 with Rust's NaN rules (max ignores NaN, clamp keeps NaN, NaN casts to
// 0); lane i writes quant i, lane 0 the f16 scale.
__device__ __forceinline__ void q8_0_block_warp(float x, int lane, int8_t* q_out, __half* d_out) {
    float a = fabsf(x);
    a = warp_max(a);
    float amax = fmaxf(0.0f, a);
    float d = amax == 0.0f ? 0.0f : amax / 127.0f;
    float inv = d == 0.0f ? 0.0f : 1.0f / d;
    float s = x * inv;
    float c = s < -127.0f ? -127.0f : (s > 127.0f ? 127.0f : s);
    int8_t qv = isnan(c) ? (int8_t)0 : (int8_t)(int)roundf(c);
    q_out[lane] = qv;
    if (lane == 0) *reinterpret_cast<uint16_t*>(d_out) = f32_to_f16_bits(d);
}

// The BlockQ4_0::pack / BlockQ5_0::pack arithmetic (kv_quant/q4_0.rs:44-66 with
// quantize_nibble :100, q5_0.rs:47-80 with quantize_5bit_biased :116), one
// warp per 32-element block, lane = element: d = amax/7 (/15), scaled = x/d
// clamped to [-8, 7] ([-16, 15]), rounded half away from zero, NaN to 0,
// biased by 8 (16). Channel 2i / 2i+1 go to the low / high nibble of byte i;
// Q5_0's 5th bits form the little-endian 32-bit qh word (bit i = channel i).
template <int LEVELS_POS, int BIAS>
__device__ __forceinline__ uint32_t kv_nibble_quant(float x, int lane, float& d_out) {
    float amax = fmaxf(0.0f, warp_max(fabsf(x)));
    const float d = amax == 0.0f ? 0.0f : amax / (float)LEVELS_POS;
    const float inv = d == 0.0f ? 0.0f : 1.0f / d;
    const float sc = x * inv;
    const float c = sc < -(float)BIAS ? -(float)BIAS : (sc > (float)LEVELS_POS ? (float)LEVELS_POS : sc);
    const int r = isnan(c) ? 0 : (int)roundf(c);
    const int b = r + BIAS;
    d_out = d;
    return (uint32_t)(b < 0 ? 0 : (b > 2 * BIAS - 1 ? 2 * BIAS - 1 : b));
}

__device__ __forceinline__ void q4_0_block_warp(float x, int lane, uint8_t* qs_out, __half* d_out) {
    float d;
    const uint32_t q = kv_nibble_quant<7, 8>(x, lane, d);
    const uint32_t odd = __shfl_down_sync(0xffffffffu, q, 1);
    if (!(lane & 1)) qs_out[lane >> 1] = (uint8_t)((q & 0xfu) | ((odd & 0xfu) << 4));
    if (lane == 0) *reinterpret_cast<uint16_t*>(d_out) = f32_to_f16_bits(d);
}

__device__ __forceinline__ void q5_0_block_warp(float x, int lane, uint8_t* qs_out, uint8_t* qh_out, __half* d_out) {
    float d;
    const uint32_t q = kv_nibble_quant<15, 16>(x, lane, d);
    const uint32_t odd = __shfl_down_sync(0xffffffffu, q, 1);
    const uint32_t hi = __ballot_sync(0xffffffffu, (q >> 4) & 1u);
    if (!(lane & 1)) qs_out[lane >> 1] = (uint8_t)((q & 0xfu) | ((odd & 0xfu) << 4));
    if (lane == 0) {
        *reinterpret_cast<uint32_t*>(qh_out) = hi;
        *reinterpret_cast<uint16_t*>(d_out) = f32_to_f16_bits(d);
    }
}

// Calls f(std::integral_constant<int, MODE>{}) for a KV mode (vkb_kv_quant).
template <class F>
inline void with_kv_mode(int mode, F&& f) {
    switch (mode) {
        case VKB_KV_FP32: f(std::integral_constant<int, VKB_KV_FP32>{}); break;
        case VKB_KV_Q4_0: f(std::integral_constant<int, VKB_KV_Q4_0>{}); break;
        case VKB_KV_Q5_0: f(std::integral_constant<int, VKB_KV_Q5_0>{}); break;
        case VKB_KV_Q8_0: f(std::integral_constant<int, VKB_KV_Q8_0>{}); break;
        default: fail(VKB_ERROR_INVALID_ARGUMENT, "kv: unknown mode " + std::to_string(mode));
    }
}

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

}  // namespace vkb
