// elementwise.cuh — the small kernels around the hot path (layer norm, token
// embedding, conv stem im2col, positional add, argmax).
#pragma once
#include "common.cuh"
struct vkb_weight;
namespace vkb {
// out = (x - mean) / sqrt(var + eps) * g + b per row (kernels/scalar.rs:201), f32 in, f32 or f16 out.
// out_fmt 0 f32, 1 f16, 2 f16 hi + lo planes.
void run_layer_norm(vkb_context* ctx, const float* x, int64_t rows, int cols, const float* g, const float* b, float eps,
                    void* out, int out_fmt);
// The residual update of a split-K projection fused with the next LayerNorm:
// h[r] += bias + sum_s part[s][r] (partials summed in split order), then
// out = LayerNorm(h[r]) as run_layer_norm. rows * cols floats per partial.
void run_reduce_residual_ln(vkb_context* ctx, const float* part, int splits, int64_t rows, int cols, const float* bias,
                            float* h, const float* g, const float* b, float eps, void* out, int out_fmt);
// h[i] = dequant(tok_emb[tokens[i]]) + pos[positions[i]]  (whisper/decoder.rs:440-452)
void run_embed(vkb_context* ctx, const vkb_weight* tok_emb, const int32_t* tokens, const int32_t* positions, int n_tok,
               const float* pos, float* h);
// conv1 im2col: x [B][C][T] f32 -> col [B*T_out][ldc] f16 (kernel 3, pad 1, stride s;
// columns C*3 .. ldc-1 zero)
void run_im2col_ct(vkb_context* ctx, const float* x, int B, int C, int T, int stride, int ldc, __half* col,
                   bool split);
// conv2 im2col from a [B*T][C] f16 (time-major) input
void run_im2col_tc(vkb_context* ctx, const __half* x, int B, int C, int T, int stride, __half* col, int planes);
// h[b*T+t][c] = y[b*T+t][c] + pos[t][c]
void run_add_pos(vkb_context* ctx, const __half* y, const float* pos, int B, int T, int C, float* h, int planes);
// ids[i] = argmax_j logits[i][j] (first index of the maximum)
void run_argmax(vkb_context* ctx, const float* logits, int n_rows, int n_cols, int32_t* ids);
}  // namespace vkb
