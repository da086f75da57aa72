// xattn.cuh — the bandwidth-oriented decode cross-attention over a dense Q8_0
// store (xattn.cu).
#pragma once
#include "common.cuh"
namespace vkb {
struct XaPlan {
    bool ok = false;     // false: the shape / alignment is not one this kernel takes
    bool f16 = false;    // the store holds f16 K/V rows (no scales) instead of Q8_0
    int G = 0;           // CTAs (one per SM at most)
    int max_seg = 0;     // partial slots per CTA
    size_t ws_floats = 0;
};
XaPlan xattn_q8_plan(const vkb_context* ctx, int n_tok, int n_head, int d_head, int n_ctx, const float* q,
                     const void* k, const void* v, const void* ks, const void* vs, size_t ws_cap_floats,
                     bool f16 = false);
void run_xattn_q8(vkb_context* ctx, const XaPlan& plan, int n_tok, int n_head, int n_ctx, const float* q,
                  const int32_t* seq_of_tok, const void* k, const void* v, const void* ks, const void* vs, void* out,
                  int out_fmt, float* ws, bool kv_ready = false);
}  // namespace vkb
