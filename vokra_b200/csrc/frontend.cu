// frontend.cu — Whisper's log-mel frontend on the device (PCM -> [n_mels, 3000]).
//
// Semantics: crates/vokra-models/src/whisper/mel.rs:123 (log_mel) ->
// crates/vokra-ops/src/fused_logmel.rs:80 (fused_log_mel_scalar) with the
// Whisper spec: every clip zero-padded or trimmed to 30 s (480000 samples),
// center reflect padding by 200, 3001 frames of 400 samples at hop 160 of
// which the last is dropped, periodic Hann, |X|^2 of the 201 real-DFT bins,
// Slaney mel projection, log10(max(., 1e-10)), then per clip
// (max(l, gmax - 8) + 4) / 4 with gmax the clip's largest log10 energy.
//
// Kernels:
//   logmel_frames_kernel  one CTA per (32 frames, clip): builds the windowed
//       frames in shared memory, the 400-point DFT as a direct sum
//       accumulated in f64 (twiddle index k*n mod 400 from a 400-entry table;
//       8 frames per thread share each twiddle load), the f32 power spectrum,
//       the mel sums over each filter's non-zero bins (the reference adds
//       w * p over all 201 bins; the zero weights add exactly 0), log10, and
//       the clip maximum (atomicMax on an order-preserving integer key).
//   logmel_norm_kernel    the dynamic-range step, in place.
// The DFT is ~31 G f64 FMAs for 64 clips (~2 ms); it runs once per clip.
#include "common.cuh"
#include <cmath>
#include <vector>

namespace vkb {

constexpr int LM_NFFT = 400, LM_HOP = 160, LM_BINS = 201, LM_FRAMES = 3000;
constexpr int64_t LM_SAMPLES = 480000;
constexpr int LM_FT = 32;       // frames per CTA
constexpr int LM_FG = 8;        // frames per DFT work item
constexpr int LM_PSTRIDE = 204; // power row stride (floats)

struct LmTables {
    const float* win;      // [400]
    const double2* tw;     // [400] (cos, -sin)(2 pi j / 400)
    const float* fb;       // [n_mels][201]
    const int2* range;     // [n_mels] first and one-past-last non-zero bin
};

__device__ __forceinline__ unsigned lm_key(float f) {
    const unsigned u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float lm_unkey(unsigned k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Sample i of the reflect-padded 30 s buffer of a clip with `len` valid samples.
__device__ __forceinline__ float lm_sample(const float* pcm, int64_t len, int64_t i) {
    int64_t j = i - LM_NFFT / 2;
    if (j < 0) j = -j;
    else if (j >= LM_SAMPLES) j = 2 * (LM_SAMPLES - 1) - j;
    return j < len ? pcm[j] : 0.0f;
}

__global__ void __launch_bounds__(256, 2) logmel_frames_kernel(const float* __restrict__ pcm, int64_t stride,
                                                              const int32_t* __restrict__ lengths, int n_mels,
                                                              LmTables tb, float* __restrict__ out,
                                                              unsigned* __restrict__ gmax) {
    pdl_entry();
    extern __shared__ __align__(16) uint8_t lm_smem[];
    double2* tw = reinterpret_cast<double2*>(lm_smem);                                    // [400]
    float* frames = reinterpret_cast<float*>(lm_smem + LM_NFFT * sizeof(double2));       // [FT][400]
    float* power = frames + LM_FT * LM_NFFT;                                              // [FT][PSTRIDE]
    __shared__ unsigned s_max;
    const int clip = blockIdx.y, t0 = blockIdx.x * LM_FT, tid = threadIdx.x;
    const float* x = pcm + (int64_t)clip * stride;
    int64_t len = lengths ? (int64_t)lengths[clip] : stride;
    len = len < 0 ? 0 : (len > stride ? stride : len);
    if (tid == 0) s_max = 0u;
    for (int i = tid; i < LM_NFFT; i += blockDim.x) tw[i] = tb.tw[i];
    for (int i = tid; i < LM_FT * LM_NFFT; i += blockDim.x) {
        const int f = i / LM_NFFT, n = i - f * LM_NFFT;
        const int t = t0 + f;
        frames[i] = t < LM_FRAMES ? __fmul_rn(lm_sample(x, len, (int64_t)t * LM_HOP + n), tb.win[n]) : 0.0f;
    }
    __syncthreads();
    // DFT: item = (bin k, group of LM_FG frames)
    for (int item = tid; item < LM_BINS * (LM_FT / LM_FG); item += blockDim.x) {
        const int k = item % LM_BINS, g = item / LM_BINS;
        const float* fr = frames + g * LM_FG * LM_NFFT;
        double re[LM_FG], im[LM_FG];
#pragma unroll
        for (int f = 0; f < LM_FG; ++f) re[f] = im[f] = 0.0;
        int idx = 0;
#pragma unroll 4
        for (int n = 0; n < LM_NFFT; ++n) {
            const double2 c = tw[idx];
#pragma unroll
            for (int f = 0; f < LM_FG; ++f) {
                const double v = (double)fr[f * LM_NFFT + n];
                re[f] = fma(v, c.x, re[f]);
                im[f] = fma(v, c.y, im[f]);
            }
            idx += k;
            if (idx >= LM_NFFT) idx -= LM_NFFT;
        }
#pragma unroll
        for (int f = 0; f < LM_FG; ++f) {
            const float r = (float)re[f], q = (float)im[f];
            power[(g * LM_FG + f) * LM_PSTRIDE + k] = __fadd_rn(__fmul_rn(r, r), __fmul_rn(q, q));
        }
    }
    __syncthreads();
    // mel sums: item = (mel m, frame f), frames fastest so a warp writes 32 consecutive frames
    float local_max = -INFINITY;
    for (int item = tid; item < n_mels * LM_FT; item += blockDim.x) {
        const int m = item / LM_FT, f = item - m * LM_FT;
        const int t = t0 + f;
        if (t >= LM_FRAMES) continue;
        const int2 rg = tb.range[m];
        const float* w = tb.fb + (size_t)m * LM_BINS;
        const float* p = power + f * LM_PSTRIDE;
        float acc = 0.0f;
        for (int kk = rg.x; kk < rg.y; ++kk) acc = __fadd_rn(acc, __fmul_rn(w[kk], p[kk]));
        const float l = log10f(fmaxf(acc, 1e-10f));
        out[((int64_t)clip * n_mels + m) * LM_FRAMES + t] = l;
        local_max = fmaxf(local_max, l);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) local_max = fmaxf(local_max, __shfl_xor_sync(0xffffffffu, local_max, o));
    if ((tid & 31) == 0 && local_max > -INFINITY) atomicMax(&s_max, lm_key(local_max));
    __syncthreads();
    if (tid == 0 && s_max) atomicMax(&gmax[clip], s_max);
}

__global__ void logmel_norm_kernel(float* __restrict__ out, const unsigned* __restrict__ gmax, int64_t per_clip,
                                   int64_t total) {
    pdl_entry();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const unsigned key = gmax[i / per_clip];
        if (!key) continue;  // no frame produced (cannot happen with the fixed 30 s grid)
        const float floor_ = lm_unkey(key) - 8.0f;
        out[i] = (fmaxf(out[i], floor_) + 4.0f) / 4.0f;
    }
}

// Host-side tables, built exactly as the reference builds them.
// Slaney mel warp: crates/vokra-ops/src/mel.rs:162-199.
static double lm_hz_to_mel(double f) {
    const double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp;
    const double logstep = std::log(6.4) / 27.0;
    return f >= min_log_hz ? min_log_mel + std::log(f / min_log_hz) / logstep : f / f_sp;
}
static double lm_mel_to_hz(double m) {
    const double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp;
    const double logstep = std::log(6.4) / 27.0;
    return m >= min_log_mel ? min_log_hz * std::exp(logstep * (m - min_log_mel)) : f_sp * m;
}

struct LmHost {
    std::vector<float> win, fb;
    std::vector<double> tw;  // interleaved cos, -sin
    std::vector<int> range;  // interleaved lo, hi
};

static LmHost lm_build_tables(int n_mels) {
    LmHost h;
    const double PI_ = 3.14159265358979323846, sr = 16000.0;
    h.win.resize(LM_NFFT);
    // periodic Hann, cosine_sum with [0.5, 0.5] (crates/vokra-ops/src/window.rs:19-56)
    for (int i = 0; i < LM_NFFT; ++i) {
        const double x = 2.0 * PI_ * (double)i / (double)LM_NFFT;
        double acc = 0.0;
        acc += 0.5 * std::cos(0.0 * x);
        acc += -0.5 * std::cos(1.0 * x);
        h.win[i] = (float)acc;
    }
    h.tw.resize(2 * LM_NFFT);
    for (int j = 0; j < LM_NFFT; ++j) {
        h.tw[2 * j] = std::cos(2.0 * PI_ * (double)j / (double)LM_NFFT);
        h.tw[2 * j + 1] = -std::sin(2.0 * PI_ * (double)j / (double)LM_NFFT);
    }
    // MelFilterbank::new, Hz interpolation + Slaney norm (crates/vokra-ops/src/mel.rs:30-124)
    std::vector<double> fft_f(LM_BINS), band_hz(n_mels + 2);
    for (int k = 0; k < LM_BINS; ++k) fft_f[k] = (double)k * sr / (double)LM_NFFT;
    const double lo = lm_hz_to_mel(0.0), hi = lm_hz_to_mel(sr / 2.0);
    for (int i = 0; i < n_mels + 2; ++i) band_hz[i] = lm_mel_to_hz(lo + (hi - lo) * (double)i / (double)(n_mels + 1));
    h.fb.assign((size_t)n_mels * LM_BINS, 0.0f);
    h.range.assign(2 * n_mels, 0);
    for (int m = 0; m < n_mels; ++m) {
        const double left = band_hz[m], center = band_hz[m + 1], right = band_hz[m + 2];
        const double dl = center - left, dh = right - center, enorm = 2.0 / (right - left);
        int first = LM_BINS, last = 0;
        for (int k = 0; k < LM_BINS; ++k) {
            const double lower = dl > 0.0 ? (fft_f[k] - left) / dl : 0.0;
            const double upper = dh > 0.0 ? (right - fft_f[k]) / dh : 0.0;
            const float w = (float)std::max(std::min(lower, upper), 0.0);
            const float wn = (float)((double)w * enorm);
            h.fb[(size_t)m * LM_BINS + k] = wn;
            if (wn != 0.0f) {
                first = std::min(first, k);
                last = k + 1;
            }
        }
        h.range[2 * m] = first < last ? first : 0;
        h.range[2 * m + 1] = first < last ? last : 0;
    }
    return h;
}

static size_t lm_align(size_t x) { return (x + 255) / 256 * 256; }

void run_log_mel(vkb_context* ctx, const float* pcm, int64_t n_clips, int64_t stride, const int32_t* lengths,
                 int n_mels, float* out) {
    // tables (built once per mel count) + per-clip maxima, in one context-owned buffer
    const size_t o_tw = 0, o_win = o_tw + lm_align(LM_NFFT * 16), o_fb = o_win + lm_align(LM_NFFT * 4);
    const size_t o_rg = o_fb + lm_align((size_t)n_mels * LM_BINS * 4), o_max = o_rg + lm_align((size_t)n_mels * 8);
    const size_t need = o_max + lm_align((size_t)n_clips * 4);
    if (ctx->frontend_mels != n_mels || ctx->frontend.n < need) {
        VKB_CUDA(cudaStreamSynchronize(ctx->stream));
        if (ctx->frontend.n < need) ctx->frontend.alloc(need);
        LmHost h = lm_build_tables(n_mels);
        uint8_t* b = ctx->frontend.as<uint8_t>();
        VKB_CUDA(cudaMemcpy(b + o_tw, h.tw.data(), h.tw.size() * 8, cudaMemcpyHostToDevice));
        VKB_CUDA(cudaMemcpy(b + o_win, h.win.data(), h.win.size() * 4, cudaMemcpyHostToDevice));
        VKB_CUDA(cudaMemcpy(b + o_fb, h.fb.data(), h.fb.size() * 4, cudaMemcpyHostToDevice));
        VKB_CUDA(cudaMemcpy(b + o_rg, h.range.data(), h.range.size() * 4, cudaMemcpyHostToDevice));
        ctx->frontend_mels = n_mels;
    }
    uint8_t* b = ctx->frontend.as<uint8_t>();
    LmTables tb{reinterpret_cast<const float*>(b + o_win), reinterpret_cast<const double2*>(b + o_tw),
                reinterpret_cast<const float*>(b + o_fb), reinterpret_cast<const int2*>(b + o_rg)};
    unsigned* gmax = reinterpret_cast<unsigned*>(b + o_max);
    VKB_CUDA(cudaMemsetAsync(gmax, 0, (size_t)n_clips * 4, ctx->stream));
    const size_t smem = LM_NFFT * sizeof(double2) + (size_t)LM_FT * (LM_NFFT + LM_PSTRIDE) * 4;
    smem_optin(logmel_frames_kernel, (int)smem);
    dim3 grid((LM_FRAMES + LM_FT - 1) / LM_FT, (unsigned)n_clips);
    launch_pdl(ctx, logmel_frames_kernel, grid, 256, smem, pcm, stride, lengths, n_mels, tb, out, gmax);
    VKB_CUDA(cudaGetLastError());
    ctx->count();
    const int64_t per = (int64_t)n_mels * LM_FRAMES, total = per * n_clips;
    const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, (int64_t)ctx->sm_count * 8);
    launch_pdl(ctx, logmel_norm_kernel, blocks, 256, 0, out, (const unsigned*)gmax, per, total);
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}

}  // namespace vkb

using namespace vkb;

extern "C" {

vkb_status vkb_log_mel(vkb_context* ctx, const float* pcm_dev, int64_t n_clips, int64_t stride,
                       const int32_t* lengths_dev, int32_t n_mels, float* out_dev) {
    return guard([&] {
        NvtxRange nvtx_range("vkb.log_mel");
        if (!ctx || !out_dev) fail(VKB_ERROR_INVALID_ARGUMENT, "log_mel: null context or output");
        if (n_clips <= 0 || n_clips > 65535) fail(VKB_ERROR_INVALID_ARGUMENT, "log_mel: n_clips must be in 1..65535");
        if (stride < 0) fail(VKB_ERROR_INVALID_ARGUMENT, "log_mel: negative stride");
        if (stride > 0 && !pcm_dev) fail(VKB_ERROR_INVALID_ARGUMENT, "log_mel: null pcm");
        if (n_mels <= 0 || n_mels > 256) fail(VKB_ERROR_INVALID_ARGUMENT, "log_mel: n_mels must be in 1..256");
        run_log_mel(ctx, pcm_dev, n_clips, stride, lengths_dev, n_mels, out_dev);
    });
}

}  // extern "C"
