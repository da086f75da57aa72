// enc_attn.cuh — encoder (whole-window, non-causal) attention.
#pragma once
#include "common.cuh"
namespace vkb {
void run_encoder_attention(vkb_context* ctx, const __half* qkv, int64_t ld, int kcol, int vcol, int n_windows, int T,
                           int n_head, int d_head, __half* out, int64_t out_ld, __half* out_lo = nullptr);
}
