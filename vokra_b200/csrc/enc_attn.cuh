// enc_attn.cuh — encoder (whole-window, non-causal) attention.
#pragma once
#include "common.cuh"
namespace vkb {
// vt_scratch (n_windows * n_head * 64 * round_up(T, 8) halves) lets the tensor-core
// kernel run; without it (or for shapes it does not take) the mma.sync kernel runs.
void run_encoder_attention(vkb_context* ctx, const __half* qkv, int64_t ld, int kcol, int vcol, int n_windows, int T,
                           int n_head, int d_head, __half* out, int64_t out_ld, __half* out_lo = nullptr,
                           __half* vt_scratch = nullptr, size_t scratch_halves = 0);
bool run_encoder_attention_tc(vkb_context* ctx, const __half* qkv, int64_t ld, int kcol, int vcol, int n_windows,
                              int T, int n_head, __half* out, int64_t out_ld, __half* out_lo, __half* vt_scratch,
                              size_t scratch_halves);
}
