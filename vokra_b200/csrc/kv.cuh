// kv.cuh — internal interface of the paged KV cache and the attention launchers (kv.cu).
#pragma once
#include "common.cuh"
namespace vkb {
vkb_kv_pool* kv_pool_create(vkb_context* ctx, const vkb_kv_pool_desc* desc);
void kv_pool_destroy(vkb_kv_pool* p);
void kv_begin_step(vkb_kv_pool* p, int n_tok, const int32_t* seq, const int32_t* pos);
// k / v rows have stride ld floats (e.g. the fused q|k|v projection output).
// Shape of the step begun last (what a recorded step's launches depend on).
int pool_groups(const vkb_kv_pool* p);
int pool_maxq(const vkb_kv_pool* p);
int pool_splits(const vkb_kv_pool* p);
void kv_append_ex(vkb_kv_pool* p, int layer, const float* k, const float* v, int64_t ld);
// The decode step's append + attention for one layer (fused when
// kv_decode_fused; only then may the q|k|v rows come as split-K partials).
bool kv_decode_fused(const vkb_kv_pool* p);
void kv_append_attention_ex(vkb_kv_pool* p, int layer, const float* qkv, int64_t ld, void* out, int out_dtype,
                            const float* part = nullptr, int splits = 0, const float* bias = nullptr,
                            float qscale = 1.0f);
void kv_copy_stream(vkb_kv_pool* p, int src, int dst, int n_pos);
void kv_attention_ex(vkb_kv_pool* p, int layer, const float* q, int64_t q_ld, void* out, int out_dtype);
void run_dense_attention(vkb_context* ctx, int n_tok, int n_head, int d_head, const float* q, const int32_t* seq_of_tok,
                         const void* k, const void* v, const void* k_scale, const void* v_scale, int n_ctx,
                         int kv_fmt, void* out, int out_dtype, float* ws_override, size_t ws_cap_floats = 0,
                         bool kv_ready = false);
void run_quantize_rows(vkb_context* ctx, const float* x, int64_t ld, int64_t n_rows, int W, int8_t* q, __half* d,
                       const int32_t* map, int group);
}  // namespace vkb
