// linear.cuh — internal interface of the quantized Linear (linear.cu).
#pragma once
#include "common.cuh"
#include "weights.cuh"
#include <cuda.h>

namespace vkb {

struct LinearPlan {
    bool tc = false;     // tcgen05 GEMM (else the streaming GEMV)
    bool gv2 = false;    // the small-m GEMV with the in-kernel split-K reduction (Q4_0, Q8_0, Q4_K)
    int bn = 0;          // token tile of the GEMM
    int m_tiles = 0;
    int splits = 1;      // K splits (partials reduced by splitk_reduce_kernel)
    int sps = 0;         // stages per split
    bool split = false;  // high-precision (hi+lo) tensor-core mode
    size_t ws_bytes = 0; // fp32 partials
};

// Epilogue extensions used by the model runner (fused projections).
struct LinearExtra {
    int64_t n_scaled = -1;        // EPI_SCALE applies to columns [0, n_scaled); -1 = all
    int64_t col_block = 0;        // write column blocks as separate [out_rows][col_block] planes
    int64_t out_rows = 0;         // rows per plane (default m)
    const int32_t* row_map = nullptr;  // device map of row groups to destination groups
    int row_group = 1;
    // Split-K GEMMs: leave the fp32 partials [splits][m][n] in the workspace
    // instead of reducing them (the caller's next kernel reduces them and
    // applies bias / residual); *splits_out = number of partials (1 = the
    // output was written with its epilogue as usual).
    int* splits_out = nullptr;
};

vkb_weight* upload_weight(vkb_context* ctx, uint32_t tag, int64_t n, int64_t k, const void* bytes, size_t len);
LinearPlan plan_linear(const vkb_context* ctx, const vkb_weight* w, int64_t m);
LinearPlan plan_linear(const vkb_context* ctx, const vkb_weight* w, int64_t m, bool split);
// x (f32, n elements) -> f16 plane (or hi then lo planes when split).
void run_split_f16(vkb_context* ctx, const float* x, int64_t n, __half* y, bool split);
// Runs out = epilogue(a . W^T + bias). ws_override / a16_override let a caller
// that pre-sized its own scratch avoid the context workspace.
void run_linear(vkb_context* ctx, const vkb_weight* w, int64_t m, const void* a, int a_dtype, const float* bias,
                void* out, int out_dtype, int epilogue, const float* residual, float scale, float* ws_override,
                __half* a16_override);
void run_linear_ex(vkb_context* ctx, const vkb_weight* w, int64_t m, const void* a, int a_dtype, const float* bias,
                   void* out, int out_dtype, int epilogue, const float* residual, float scale, float* ws_override,
                   __half* a16_override, const LinearExtra& x);
void make_tmap_f16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows);
int read_and_clear_err_flag(vkb_context* ctx);

// Epilogue of the persistent encoder GEMM (gemm_persist.cu): out[m][n] =
// op(acc + bias[n]) with op = GELU, scale (columns < n_scaled) or + residual.
struct PEpi {
    const float* bias;
    const float* residual;
    void* out;
    int out_fmt;
    int kind;
    float scale;
    int64_t ldo;
    int64_t n_scaled;
    int64_t plane;  // elements per plane of an F16X2 output
    // Q8_0 pair output (the cross K/V projection): when q8_width > 0, columns
    // [0, q8_width) are packed as Q8_0 rows into q8[0] / q8d[0] and columns
    // [q8_width, 2 q8_width) into q8[1] / q8d[1] (BlockQ8_0::pack per 32
    // columns); token m lands in row row_map[m / row_group] * row_group +
    // m % row_group. out / out_fmt are unused then.
    int64_t q8_width = 0;
    int8_t* q8[2] = {nullptr, nullptr};
    __half* q8d[2] = {nullptr, nullptr};
    const int32_t* row_map = nullptr;
    int row_group = 1;
};
// Split-precision (hi+lo) GEMM over f16 activation planes a16 [2][m][k], one
// CTA per SM over a static tile list; token tile persist_bn().
// Whether single-f16 large-M GEMMs take the shared-operand kernels (tc_gemm_pair_kernel, or
// tc_gemm_persist_kernel with SS; weights as a once-per-call f16 plane, both operands in shared memory).
bool persist_ss_enabled();
void run_tc_persistent(vkb_context* ctx, const vkb_weight* w, int64_t m, const __half* a16, const PEpi& e, int* err,
                       bool split = true);
int persist_bn();
// out = Q8_0(a . W^T + bias) split into a K and a V store (see PEpi::q8_width)
// on the persistent kernel; false (nothing launched) when the shape or
// precision does not take it.
bool run_linear_q8_pair(vkb_context* ctx, const vkb_weight* w, int64_t m, const __half* a16, const float* bias,
                        int64_t width, int8_t* kq, __half* kd, int8_t* vq, __half* vd, const int32_t* row_map,
                        int row_group, bool split = true);
int gemv_max_m();

}  // namespace vkb
