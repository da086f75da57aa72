// context.cu — library-level entry points: last error, ABI version, context.
#include "common.cuh"
#include <cstdlib>
#include <cstdio>

namespace vkb {
static thread_local std::string g_last_error;
void set_last_error(const std::string& m) { g_last_error = m; }
}  // namespace vkb

using namespace vkb;

extern "C" {

const char* vkb_last_error(void) { return g_last_error.c_str(); }

int vkb_abi_version(void) { return 1; }

vkb_status vkb_context_create(int device, vkb_context** out) {
    return guard([&] {
        if (!out) fail(VKB_ERROR_INVALID_ARGUMENT, "context_create: null out");
        *out = nullptr;
        int n = 0;
        cudaError_t e = cudaGetDeviceCount(&n);
        if (e != cudaSuccess || n == 0)
            fail(VKB_ERROR_BACKEND_UNAVAILABLE, std::string("no CUDA device: ") + cudaGetErrorString(e));
        if (device < 0 || device >= n) fail(VKB_ERROR_INVALID_ARGUMENT, "context_create: device out of range");
        cudaDeviceProp prop;
        VKB_CUDA(cudaGetDeviceProperties(&prop, device));
        if (prop.major != 10 || prop.minor != 0)
            fail(VKB_ERROR_BACKEND_UNAVAILABLE, "this library is built for sm_100a (B200); device is sm_" +
                                                    std::to_string(prop.major) + std::to_string(prop.minor));
        VKB_CUDA(cudaSetDevice(device));
        auto* c = new vkb_context();
        try {
            c->device = device;
            c->sm_count = prop.multiProcessorCount;
            VKB_CUDA(cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking));
            c->stream = c->own_stream;
            c->err_flag.alloc(sizeof(int));
            c->tile_ctr.alloc(vkb::kTileCounters * sizeof(unsigned));
            VKB_CUDA(cudaMemset(c->tile_ctr.p, 0, c->tile_ctr.n));
            const char* pdl = getenv("VKB_PDL");
            c->pdl = !(pdl && pdl[0] == '0');
            VKB_CUDA(cudaMemset(c->err_flag.p, 0, sizeof(int)));
        } catch (...) {
            delete c;
            throw;
        }
        *out = c;
    });
}

vkb_status vkb_context_destroy(vkb_context* ctx) {
    return guard([&] {
        if (!ctx) return;
        cudaSetDevice(ctx->device);
        cudaStreamSynchronize(ctx->stream);
        if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
        delete ctx;
    });
}

vkb_status vkb_context_set_stream(vkb_context* ctx, void* stream) {
    return guard([&] {
        if (!ctx) fail(VKB_ERROR_INVALID_ARGUMENT, "set_stream: null context");
        ctx->stream = stream ? reinterpret_cast<cudaStream_t>(stream) : ctx->own_stream;
    });
}

vkb_status vkb_context_synchronize(vkb_context* ctx) {
    return guard([&] {
        if (!ctx) fail(VKB_ERROR_INVALID_ARGUMENT, "synchronize: null context");
        VKB_CUDA(cudaStreamSynchronize(ctx->stream));
        VKB_CUDA(cudaGetLastError());
    });
}

vkb_status vkb_context_set_precision(vkb_context* ctx, int precision) {
    return guard([&] {
        if (!ctx) fail(VKB_ERROR_INVALID_ARGUMENT, "set_precision: null context");
        if (precision != VKB_PREC_SPLIT && precision != VKB_PREC_F16 && precision != VKB_PREC_ENCODER_F16)
            fail(VKB_ERROR_INVALID_ARGUMENT, "set_precision: unknown precision");
        ctx->precision = precision;
    });
}

uint64_t vkb_context_launch_count(const vkb_context* ctx) { return ctx ? ctx->launches : 0; }
size_t vkb_context_workspace_bytes(const vkb_context* ctx) { return ctx ? ctx->workspace.n : 0; }

}  // extern "C"
