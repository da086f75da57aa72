// noalloc.cu — cross-attention with a fixed, library-owned scratch area.
//
// vkb_attention_dense may grow the context workspace with cudaMalloc the first
// time a call needs more room for its split partials. Some callers cannot let a
// library allocate device memory at call time: hosts that own a fixed device
// memory budget and hand out every byte themselves, real-time audio paths
// whose latency budget forbids driver allocation calls, and engines that must
// not let a callee allocate while they record work. For them,
// vkb_attention_dense_noalloc keeps its partials in the file-scope device array
// below instead. It never calls cudaMalloc or cudaFree.
#include "common.cuh"
#include "kv.cuh"
#include <mutex>

namespace {

// 16 MiB of split partials. Every GPU that loads the library holds this array
// until the process exits.
constexpr size_t kScratchFloats = (size_t)VKB_NOALLOC_ATTN_SCRATCH_FLOATS;
static __device__ __align__(256) float g_attn_scratch[kScratchFloats];

// Host code may not use g_attn_scratch's name as a device address; the device
// address is looked up once per device with that device current.
constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_scratch_ptr[kMaxDevices] = {};

float* scratch_for(int device) {
    if (device < 0 || device >= kMaxDevices) vkb::fail(VKB_ERROR_INVALID_ARGUMENT, "noalloc: device index out of range");
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_ptr[device]) {
        int prev = 0;
        VKB_CUDA(cudaGetDevice(&prev));
        VKB_CUDA(cudaSetDevice(device));
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
        cudaSetDevice(prev);
        if (e != cudaSuccess || !p)
            vkb::fail(VKB_ERROR_BACKEND_UNAVAILABLE,
                      std::string("noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
        g_scratch_ptr[device] = static_cast<float*>(p);
    }
    return g_scratch_ptr[device];
}

}  // namespace

using namespace vkb;

extern "C" {

vkb_status vkb_attention_dense_noalloc(vkb_context* ctx, int32_t n_tok, int32_t n_head, int32_t d_head,
                                       const float* q_dev, const int32_t* seq_of_tok_dev, const void* k_dev,
                                       const void* v_dev, const void* k_scale_dev, const void* v_scale_dev,
                                       int32_t n_ctx, int32_t kv_dtype, void* ctx_out_dev, int32_t out_dtype) {
    return guard([&] {
        if (!ctx || !q_dev || !seq_of_tok_dev || !k_dev || !v_dev || !ctx_out_dev)
            fail(VKB_ERROR_INVALID_ARGUMENT, "attention_dense_noalloc: null argument");
        if (n_tok <= 0 || n_ctx <= 0 || n_head <= 0 || d_head <= 0)
            fail(VKB_ERROR_INVALID_ARGUMENT, "attention_dense_noalloc: empty shape");
        if (kv_dtype != VKB_DT_F16 && kv_dtype != VKB_KV_Q8_0)
            fail(VKB_ERROR_UNSUPPORTED_OP, "attention_dense_noalloc: kv dtype must be F16 or Q8_0");
        if (kv_dtype == VKB_KV_Q8_0 && (!k_scale_dev || !v_scale_dev))
            fail(VKB_ERROR_INVALID_ARGUMENT, "attention_dense_noalloc: Q8_0 needs scale planes");
        if (out_dtype != VKB_DT_F32 && out_dtype != VKB_DT_F16 && out_dtype != VKB_DT_F16X2)
            fail(VKB_ERROR_INVALID_ARGUMENT, "attention_dense_noalloc: bad out dtype");
        // One split partial per query row must fit: n_tok * (n_head*d_head + 2*n_head) floats.
        const size_t per_split = (size_t)n_tok * ((size_t)n_head * d_head + 2 * (size_t)n_head);
        if (per_split > kScratchFloats)
            fail(VKB_ERROR_INVALID_ARGUMENT,
                 "attention_dense_noalloc: n_tok * (n_head*d_head + 2*n_head) = " + std::to_string(per_split) +
                     " floats exceeds the fixed scratch of " + std::to_string(kScratchFloats) + " floats (max n_tok = " +
                     std::to_string(kScratchFloats / ((size_t)n_head * d_head + 2 * (size_t)n_head)) + ")");
        float* scratch = scratch_for(ctx->device);
        run_dense_attention(ctx, n_tok, n_head, d_head, q_dev, seq_of_tok_dev, k_dev, v_dev, k_scale_dev, v_scale_dev,
                            n_ctx, kv_dtype == VKB_DT_F16 ? VKB_DT_F16 : VKB_KV_Q8_0, ctx_out_dev, out_dtype, scratch,
                            kScratchFloats);
    });
}

}  // extern "C"
