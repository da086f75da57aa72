/*
 * vkb200.h — C ABI of the B200 (sm_100a) quantized-Whisper hot path.
 *
 * A drop-in for the seams of ayutaz/vokra that a Rust backend crate would bind
 * with `extern "C"`. Every function
 * takes plain pointers and sizes; no C++ or torch type crosses this boundary
 * and no C++ exception escapes it (each entry point catches and converts, like
 * the reference's panic firewall crates/vokra-capi/src/ffi_guard.rs:27).
 *
 * Conventions
 *  - Functions return vkb_status; on error vkb_last_error() holds a message
 *    for the calling thread (vokra_last_error, include/vokra.h).
 *  - "_dev" pointers are device pointers on the context's GPU; "_host"
 *    pointers are host memory. Device-pointer calls are asynchronous on the
 *    context's stream; host-pointer calls are synchronous.
 *  - There is no CPU fallback: an unsupported dtype, shape or mode returns
 *    VKB_ERROR_UNSUPPORTED_OP or VKB_ERROR_INVALID_ARGUMENT, as the reference's
 *    Compute seam does (crates/vokra-models/src/compute.rs:589-600).
 *  - A context is used by one thread at a time (CudaContext is thread-affine,
 *    crates/vokra-backend-cuda/src/context.rs:1071-1076).
 */
#ifndef VKB200_H
#define VKB200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VKB_API __attribute__((visibility("default")))
#else
#define VKB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: the numbering of vokra_status_t (include/vokra.h:58-78),
 * plus KV_CACHE_EXHAUSTED for VokraError::KvCacheExhausted
 * (crates/vokra-core/src/error.rs:170), which vokra's C ABI folds into OTHER. */
typedef enum vkb_status {
    VKB_OK = 0,
    VKB_ERROR_IO = 1,
    VKB_ERROR_MODEL_LOAD = 2,
    VKB_ERROR_UNSUPPORTED_OP = 3,
    VKB_ERROR_BACKEND_UNAVAILABLE = 4,
    VKB_ERROR_INVALID_ARGUMENT = 5,
    VKB_ERROR_GRAPH_VALIDATION = 6,
    VKB_ERROR_NOT_IMPLEMENTED = 7,
    VKB_ERROR_PANIC = 8,
    VKB_ERROR_OTHER = 9,
    VKB_ERROR_KV_CACHE_EXHAUSTED = 10
} vkb_status;

/* GGUF dtype tags (GgmlType, crates/vokra-core/src/gguf/tensor.rs:59-97) plus
 * the loader extension of this library: Q4_0 (2) and Q8_0 (8) in the public
 * ggml block layout. */
enum vkb_ggml_type {
    VKB_GGML_F32 = 0,
    VKB_GGML_F16 = 1,
    VKB_GGML_Q4_0 = 2,
    VKB_GGML_Q8_0 = 8,
    VKB_GGML_Q4_K = 12,
    VKB_GGML_Q5_K = 13,
    VKB_GGML_Q6_K = 14,
    VKB_GGML_BF16 = 30
};

/* KV quantization modes, numbered like KvQuant (crates/vokra-core/src/kv_quant/mod.rs:88). */
enum vkb_kv_quant { VKB_KV_FP32 = 0, VKB_KV_Q4_0 = 1, VKB_KV_Q5_0 = 2, VKB_KV_Q8_0 = 3 };

/* Activation / output element types of the device-pointer entry points.
 * F16X2 is a value stored as two f16 planes, hi = f16(x) then lo = f16(x - hi)
 * (a buffer of 2 * rows * cols halves); the tensor-core GEMM consumes it at
 * about fp32 accuracy. */
enum vkb_dtype { VKB_DT_F32 = 0, VKB_DT_F16 = 1, VKB_DT_F16X2 = 2 };

/* Tensor-core operand precision of a context.
 * SPLIT (default): weights and activations enter the MMA as hi + lo f16
 *   pairs (three MMAs per step), products accurate to about 2^-21 relative;
 *   this is the mode the parity tolerances are stated for.
 * F16: one f16 MMA per step (weights and activations rounded to f16).
 * ENCODER_F16: vkb_session_encode (conv stem, encoder, cross K/V projection)
 *   runs F16, everything else SPLIT. Measured against the reference decoder
 *   (f32 caches) at full Whisper-large-v3 depth: logits 7.5e-4 relative RMS,
 *   2.8e-3 max-abs, identical argmax ids, inside the 1e-3 / 1e-2 budget of a
 *   bf16/fp32-accumulate path, at a third of the encoder's MMAs. */
enum vkb_precision { VKB_PREC_SPLIT = 0, VKB_PREC_F16 = 1, VKB_PREC_ENCODER_F16 = 2 };

/* Fused epilogues of vkb_linear. */
enum vkb_epilogue {
    VKB_EPI_NONE = 0,       /* out = a.W^T + bias                      */
    VKB_EPI_GELU = 1,       /* out = gelu(a.W^T + bias)  (erf form)    */
    VKB_EPI_RESIDUAL = 2,   /* out = residual + a.W^T + bias (f32 out) */
    VKB_EPI_SCALE = 3       /* out = (a.W^T + bias) * scale            */
};

typedef struct vkb_context vkb_context;
typedef struct vkb_weight vkb_weight;
typedef struct vkb_kv_pool vkb_kv_pool;
typedef struct vkb_whisper vkb_whisper;
typedef struct vkb_session vkb_session;

/* ---- library / context --------------------------------------------------- */

/* Thread-local message of the last failed call (vokra_last_error). */
VKB_API const char* vkb_last_error(void);
/* ABI version, bumped on incompatible change. */
VKB_API int vkb_abi_version(void);

/* Creates a context on `device` (one per GPU). Fails with
 * VKB_ERROR_BACKEND_UNAVAILABLE when the device is absent or not sm_100. */
VKB_API vkb_status vkb_context_create(int device, vkb_context** out);
VKB_API vkb_status vkb_context_destroy(vkb_context* ctx);
/* Launch subsequent device-pointer work on `stream` (a cudaStream_t of the
 * same device, or cudaStreamLegacy = (void*)0x1 for the legacy default stream;
 * NULL = the context's own stream). */
VKB_API vkb_status vkb_context_set_stream(vkb_context* ctx, void* stream);
VKB_API vkb_status vkb_context_synchronize(vkb_context* ctx);
/* Selects the tensor-core operand precision (vkb_precision). */
VKB_API vkb_status vkb_context_set_precision(vkb_context* ctx, int precision);
/* Number of kernels this context has launched (CudaContext::submission_count,
 * crates/vokra-backend-cuda/src/context.rs:3152). */
VKB_API uint64_t vkb_context_launch_count(const vkb_context* ctx);
/* Bytes of device scratch the context holds for calls that size their own
 * workspace (it only grows); vkb_attention_dense_noalloc never touches it.
 * No counterpart in the reference (a diagnostics accessor). */
VKB_API size_t vkb_context_workspace_bytes(const vkb_context* ctx);

/* Failure-path self-test (no counterpart in the reference): launches one
 * kernel whose mbarrier wait can never complete, bounded by `polls` polls
 * (1..2^20), the same bounded wait every tensor-core pipeline stage of this
 * library uses. The wait gives up, the kernel records the device error flag
 * and returns; the call then reports VKB_ERROR_OTHER and clears the flag, and
 * the context remains usable. No GPU fault, trap or hang is involved. */
VKB_API vkb_status vkb_context_selftest_bounded_wait(vkb_context* ctx, uint32_t polls);

/* ---- quantized Linear: Compute::gemm_q_f32 (compute.rs:943) ---------------- */

/* Uploads an untransposed [n][k] GGUF weight payload (`bytes`, `len` host
 * bytes) and repacks it once into the device tile layout. Accepted tags:
 * Q4_0, Q8_0, Q4_K (quantized) and F32/F16 (dense). Replaces the load-time
 * binding of whisper::weights::linear_with (whisper/weights.rs:439). */
VKB_API vkb_status vkb_weight_upload(vkb_context* ctx, uint32_t ggml_type, int64_t n, int64_t k,
                             const void* bytes, size_t len, vkb_weight** out);
VKB_API vkb_status vkb_weight_destroy(vkb_weight* w);
/* Device bytes the repacked weight occupies. */
VKB_API size_t vkb_weight_device_bytes(const vkb_weight* w);

/* out[m][n] = epilogue(a[m][k] . dequant(W)[n][k]^T + bias[n]), all device
 * pointers. a is F32 or F16; out is F32 or F16 (EPI_RESIDUAL requires F32 and
 * may alias residual). bias_dev may be NULL (Whisper k_proj). `scale` is used
 * by EPI_SCALE only. Small m runs the streaming GEMV kernel, larger m the
 * tcgen05 tensor-core GEMM. */
VKB_API vkb_status vkb_linear(vkb_context* ctx, const vkb_weight* w, int64_t m,
                      const void* a_dev, int a_dtype, const float* bias_dev,
                      void* out_dev, int out_dtype, int epilogue,
                      const float* residual_dev, float scale);

/* The exact gemm_q_f32 contract with host buffers: uploads `wq` ([n][k] GGUF
 * bytes of `ggml_type`), a[m][k] and bias, runs the GPU kernel, downloads
 * out[m][n]. Synchronous. The reference returns UnsupportedOp on every GPU
 * arm (compute.rs:589-600); this is the B200 arm. */
VKB_API vkb_status vkb_gemm_q_f32(vkb_context* ctx, int64_t m, int64_t n, int64_t k,
                          const float* a_host, const void* wq_host, size_t wq_len,
                          uint32_t ggml_type, const float* bias_host, float* out_host);

/* ---- KvQuantDequantGemvOps::fused_dequant_gemv (kv_quant/gpu_ops.rs:70) ----- */

/* y[n_rows] = dequant(blocks)[n_rows][nbpr*32] . x. Same rejection rules as
 * validate_dequant_gemv (gpu_ops.rs:95): FP32 mode, x_len != nbpr*32 or
 * n_bytes != n_rows*nbpr*block_bytes give VKB_ERROR_INVALID_ARGUMENT. */
VKB_API vkb_status vkb_kv_dequant_gemv(vkb_context* ctx, int mode, const void* blocks_dev, size_t n_bytes,
                               size_t n_rows, size_t nbpr, const float* x_dev, size_t x_len,
                               float* y_dev);
/* Host-buffer form of the same (the trait's exact signature). Synchronous. */
VKB_API vkb_status vkb_kv_dequant_gemv_host(vkb_context* ctx, int mode, const void* blocks_host,
                                    size_t n_bytes, size_t n_rows, size_t nbpr,
                                    const float* x_host, size_t x_len, float* y_host);

/* ---- paged quantized KV cache: QuantizedPagedKvCache (cache/paged_quant.rs)
 *      and GpuPagedKvCacheOps (cache/paged.rs:956) --------------------------- */

enum vkb_kv_layout {
    /* The reference layout (paged_quant.rs:100-130): one page per
     * (layer, time-block) holding every stream, page table indexed by
     * layer * pages_per_layer + t / page_tokens, LIFO allocation.
     * page_tokens 2 or 4 (BlockSize, cache/paged.rs:110) or 16. */
    VKB_KV_LAYOUT_REFERENCE = 0,
    /* Per-sequence pages: one page holds page_tokens tokens of one sequence;
     * the table [n_stream][max_time/page_tokens] is shared by every layer
     * (each layer has its own arena indexed by the same page id). Pages of a
     * sequence are returned by vkb_kv_release_seq (continuous batching). */
    VKB_KV_LAYOUT_SEQUENCE = 1
};

typedef struct vkb_kv_pool_desc {
    int32_t n_layer;
    int32_t n_head;
    int32_t d_head;
    int32_t n_stream;    /* concurrent sequences (KvDims::n_stream) */
    int32_t n_codebook;  /* 1 for Whisper (KvDims::n_codebook) */
    int32_t max_time;    /* KvDims::max_time */
    int32_t page_tokens; /* 2, 4 or 16 */
    int32_t mode;        /* vkb_kv_quant: Q8_0, Q4_0 or Q5_0 (bit-exact block packs);
                          * FP32 (dense f32 rows) in the SEQUENCE layout only */
    int32_t layout;      /* vkb_kv_layout */
    int32_t n_pages;     /* arena pages; 0 = enough for every stream at max_time */
} vkb_kv_pool_desc;

/* Allocates the whole arena up front (no allocation on the hot path,
 * paged_quant.rs:30-36). */
VKB_API vkb_status vkb_kv_pool_create(vkb_context* ctx, const vkb_kv_pool_desc* desc, vkb_kv_pool** out);
VKB_API vkb_status vkb_kv_pool_destroy(vkb_kv_pool* pool);

/* Declares the tokens of the next decode step: token i belongs to stream
 * seq_ids[i] at absolute position positions[i] (host arrays). Acquires pages
 * in the reference's order (layer-major, then token), uploads the table and
 * the step's slot list. VKB_ERROR_KV_CACHE_EXHAUSTED when the free list runs
 * out (QuantPageAllocator::acquire, paged_quant.rs:193). Tokens of one stream
 * must be contiguous and in increasing position. */
VKB_API vkb_status vkb_kv_begin_step(vkb_kv_pool* pool, int32_t n_tok, const int32_t* seq_ids_host,
                             const int32_t* positions_host);
/* Quantizes and stores the step's K and V rows ([n_tok][n_head*d_head] f32,
 * device) for `layer`, bit-exact to BlockQ8_0::pack (kv_quant/q8_0.rs:40). */
VKB_API vkb_status vkb_kv_append(vkb_kv_pool* pool, int32_t layer, const float* k_dev, const float* v_dev);
/* Causal self-attention of the step's queries (q_dev [n_tok][n_head*d_head]
 * f32, already scaled by d_head^-0.5) over their own stream's cached keys
 * 0..position; ctx_out_dev [n_tok][n_head*d_head] in out_dtype. Online
 * softmax in fp32 over the int8 pages gathered through the page table. */
VKB_API vkb_status vkb_kv_attention(vkb_kv_pool* pool, int32_t layer, const float* q_dev,
                            void* ctx_out_dev, int out_dtype);
/* The decode step's append + attention of one layer in one call: row i of
 * qkv_dev ([n_tok][ld] f32, device) holds token i's q (already scaled by
 * d_head^-0.5) in columns [0, W), its k in [W, 2W) and its v in [2W, 3W),
 * W = n_head*d_head. K and V are stored exactly as vkb_kv_append stores them
 * (bit-exact BlockQ8_0::pack), then the queries attend as in
 * vkb_kv_attention. When every stream of the step has one token (a decode
 * step), the pool is in the SEQUENCE layout, d_head is 64 and n_head a
 * multiple of 4, this is one fused kernel (the one vkb_session_step runs);
 * otherwise it is vkb_kv_append followed by vkb_kv_attention. The
 * reference's decoder does the same pair per layer (cache append, then
 * nn::attention_from_kv_into, crates/vokra-models/src/whisper/decoder.rs:455-470,
 * nn.rs:209-300). */
VKB_API vkb_status vkb_kv_append_attention(vkb_kv_pool* pool, int32_t layer, const float* qkv_dev, int64_t ld,
                                           void* ctx_out_dev, int out_dtype);
/* 1 when the step begun last runs vkb_kv_append_attention as the fused kernel. */
VKB_API int32_t vkb_kv_decode_fused(const vkb_kv_pool* pool);
/* Branches a stream (SEQUENCE layout): dst becomes the first n_pos positions
 * of src. dst's pages are let go; src's completely filled pages are shared by
 * reference count (no copy), a partly filled last page is copied on the
 * device. A later step that writes into a shared page gives the writing
 * stream its own copy first (copy on write, in vkb_kv_begin_step). The
 * reference deep-copies its host cache per beam (selfkv_snapshot /
 * selfkv_restore, whisper/decoder.rs:343-368). */
VKB_API vkb_status vkb_kv_copy_stream(vkb_kv_pool* pool, int32_t src, int32_t dst, int32_t n_pos);
/* Frees every page of one stream (SEQUENCE layout); a page shared with other
 * streams stays in use until its last holder lets go. */
VKB_API vkb_status vkb_kv_release_seq(vkb_kv_pool* pool, int32_t seq_id);
/* release_layer (paged_quant.rs:500): REFERENCE layout only. */
VKB_API vkb_status vkb_kv_release_layer(vkb_kv_pool* pool, int32_t layer);
/* reset (paged_quant.rs:489): empties the table, zeroes pages, rebuilds the free list. */
VKB_API vkb_status vkb_kv_reset(vkb_kv_pool* pool);
/* GpuPagedKvCacheOps::upload_page_table: installs an explicit page table
 * (SEQUENCE layout, [n_stream][pages_per_stream] int32, -1 = empty) and marks
 * the listed pages in use. */
VKB_API vkb_status vkb_kv_set_page_table(vkb_kv_pool* pool, const int32_t* table_host, size_t len);
/* Introspection for parity tests (synchronous). */
VKB_API size_t vkb_kv_table_len(const vkb_kv_pool* pool);
VKB_API vkb_status vkb_kv_page_table(const vkb_kv_pool* pool, int64_t* out_host, size_t len);
VKB_API int32_t vkb_kv_pages_in_use(const vkb_kv_pool* pool);
VKB_API size_t vkb_kv_page_bytes(const vkb_kv_pool* pool);      /* on-wire bytes of one K (or V) page */
VKB_API size_t vkb_kv_on_wire_bytes(const vkb_kv_pool* pool);   /* on_wire_storage_bytes, paged_quant.rs:382 */
/* On-wire bytes (reference block order, 34-byte Q8_0 blocks) of one page of
 * `layer` (SEQUENCE layout; the layer is ignored for REFERENCE layout). */
VKB_API vkb_status vkb_kv_read_page(const vkb_kv_pool* pool, int32_t layer, int32_t page,
                            void* k_host, void* v_host);
/* read_step (paged_quant.rs:448): dequantized K and V rows; VKB_ERROR_INVALID_ARGUMENT
 * when out of range, VKB_ERROR_OTHER when the slot was never written. */
VKB_API vkb_status vkb_kv_read_step(const vkb_kv_pool* pool, int32_t layer, int32_t t, int32_t s,
                            float* k_host, float* v_host);

/* ---- dense attention (cross-attention and the encoder) ------------------- */

/* ctx[i] = softmax(q[i] . K_s^T) V_s per head, for n_tok query rows where row
 * i belongs to stream seq_of_tok_dev[i] (device int32). K_s / V_s are the
 * stream's dense rows s*n_ctx .. s*n_ctx+n_ctx-1 of [*][n_head*d_head]:
 *   kv_dtype VKB_DT_F16   : k_dev / v_dev are f16 rows, scales unused (NULL);
 *   kv_dtype VKB_KV_Q8_0  : k_dev / v_dev are int8 quants, k_scale_dev /
 *                           v_scale_dev the f16 scale per 32 channels
 *                           (the layout vkb_quantize_rows_q8_0 writes).
 * q is f32 and already scaled by d_head^-0.5; no mask (cross-attention,
 * whisper/nn.rs:209 with causal=false). ctx_out is f32 or f16. */
VKB_API vkb_status vkb_attention_dense(vkb_context* ctx, int32_t n_tok, int32_t n_head, int32_t d_head,
                               const float* q_dev, const int32_t* seq_of_tok_dev,
                               const void* k_dev, const void* v_dev,
                               const void* k_scale_dev, const void* v_scale_dev,
                               int32_t n_ctx, int32_t kv_dtype, void* ctx_out_dev, int32_t out_dtype);

/* Same computation as vkb_attention_dense, for callers that cannot let the
 * library allocate device memory during a call (a host that owns a fixed
 * device-memory budget, a real-time audio path, an engine recording work that
 * a callee must not interrupt with an allocation). This entry point has no
 * counterpart in the reference. Its split partials live in a fixed array
 * inside the library (VKB_NOALLOC_ATTN_SCRATCH_FLOATS floats = 16 MiB, held by
 * every GPU that loads the library until the process exits); it never calls
 * cudaMalloc or cudaFree. The first call on a device looks up that array's
 * device address (cudaGetSymbolAddress) with the device current; make that
 * first call before any stream capture. Calls that need more than
 * n_tok * (n_head*d_head + 2*n_head) <= VKB_NOALLOC_ATTN_SCRATCH_FLOATS are
 * rejected with VKB_ERROR_INVALID_ARGUMENT. Every call on a device shares the
 * array and it keeps the last call's partials (each call overwrites the slots
 * it reads, nothing needs to start at zero): calls that overlap on the GPU,
 * on any streams or contexts of the same device, race and must be ordered by
 * the caller. */
#define VKB_NOALLOC_ATTN_SCRATCH_FLOATS (4u * 1024u * 1024u)
VKB_API vkb_status vkb_attention_dense_noalloc(vkb_context* ctx, int32_t n_tok, int32_t n_head, int32_t d_head,
                                               const float* q_dev, const int32_t* seq_of_tok_dev,
                                               const void* k_dev, const void* v_dev,
                                               const void* k_scale_dev, const void* v_scale_dev,
                                               int32_t n_ctx, int32_t kv_dtype, void* ctx_out_dev,
                                               int32_t out_dtype);

/* Quantizes f32 rows [n_rows][width] (width % 32 == 0) into int8 quants
 * q_dev [n_rows][width] and f16 scales d_dev [n_rows][width/32] with the
 * arithmetic of BlockQ8_0::pack (crates/vokra-core/src/kv_quant/q8_0.rs:40),
 * bit-exact. Used for the cross-attention K/V store. */
VKB_API vkb_status vkb_quantize_rows_q8_0(vkb_context* ctx, const float* x_dev, int64_t n_rows, int32_t width,
                                  void* q_dev, void* d_dev);


/* ---- GGUF reader (GgufFile::parse, crates/vokra-core/src/gguf/reader.rs:132) */

/* Parses a GGUF v3 image held in host memory with the checks the model
 * loader applies (host only, no device work): magic, version 3, counts
 * bounded by the file size, metadata values, general.alignment a power of
 * two, at most 8 dimensions, known dtype tags (the reference's F32, F16,
 * BF16, Q4_K, Q5_K, Q6_K plus Q4_0 and Q8_0), unique names, whole blocks,
 * aligned offsets, every tensor inside the file. Malformed input returns
 * VKB_ERROR_MODEL_LOAD with the reference's GgufError variant named in
 * vkb_last_error() (e.g. "(BadMagic)", "(UnsupportedVersion)",
 * "(Truncated)"). On success the counts are written where non-NULL. */
VKB_API vkb_status vkb_gguf_inspect(const void* bytes, size_t len, int64_t* n_tensors, int64_t* n_metadata);

/* ---- Whisper model and decode session ------------------------------------ */

/* Model hyper-parameters read from the GGUF metadata (vokra.whisper.*,
 * crates/vokra-models/src/whisper/config.rs:19-50). */
typedef struct vkb_whisper_dims {
    int32_t n_mels, n_audio_ctx, d_model, n_audio_head, n_audio_layer;
    int32_t n_text_ctx, n_text_head, n_text_layer, n_vocab, ffn_dim, eot;
    int32_t n_start_ids;
    int32_t start_ids[8];
} vkb_whisper_dims;

/* Loads a Whisper GGUF (tensor names of crates/vokra-models/src/whisper/weights.rs:302-360)
 * and repacks every Linear once into the device tile layout. Linear weights
 * may be Q4_0, Q8_0, Q4_K, F16 or F32; conv / positional / LayerNorm tensors
 * F32, F16 or BF16. The file is read once and not kept. */
VKB_API vkb_status vkb_whisper_load(vkb_context* ctx, const char* gguf_path, vkb_whisper** out);
VKB_API vkb_status vkb_whisper_get_dims(const vkb_whisper* m, vkb_whisper_dims* out);
VKB_API vkb_status vkb_whisper_destroy(vkb_whisper* m);

typedef struct vkb_session_options {
    int32_t max_streams;      /* concurrent utterances (KV streams, cross-store slots) */
    int32_t max_step_tokens;  /* tokens per decode step (e.g. 4 * max_streams for prefixes) */
    int32_t max_clips;        /* clips per vkb_session_encode call (0 = no encoder buffers) */
    int32_t cross_kv_q8;      /* 1: cross K/V stored as Q8_0 int8 + f16 scales; 0: f16 */
    int32_t kv_page_tokens;   /* self-attention page size (0 = 16) */
    int32_t self_kv_mode;     /* vkb_self_kv: how the self-attention K/V pages are stored */
} vkb_session_options;

/* Self-attention KV storage of a session.
 * Q8_0 (default): int8 pages, bit-exact BlockQ8_0 (the reference's
 *   QuantizedPagedKvCache in KvQuant::Q8_0), decoded by the fused decode kernel.
 * F32: dense f32 pages, the numerics of the KvCache the reference's Whisper
 *   decoder keeps (whisper/decoder.rs:183-200, 455-470).
 * Q4_0 / Q5_0: the reference's 4- and 5-bit KV blocks. */
enum vkb_self_kv { VKB_SELF_KV_Q8_0 = 0, VKB_SELF_KV_F32 = 1, VKB_SELF_KV_Q4_0 = 2, VKB_SELF_KV_Q5_0 = 3 };

/* A batched decoding session (the DecoderStepSession / CudaDecodeSession seam,
 * crates/vokra-models/src/compute.rs:2892-3140): owns the paged self-attention
 * cache (sequence layout, Q8_0 unless self_kv_mode says otherwise), the cross-attention store and every
 * device buffer; nothing is allocated per step. */
VKB_API vkb_status vkb_session_create(vkb_whisper* m, const vkb_session_options* opt, vkb_session** out);
VKB_API vkb_status vkb_session_destroy(vkb_session* s);
/* Runs the encoder on n_clips log-mels ([n_clips][n_mels][2*n_audio_ctx] f32,
 * device) and projects every decoder layer's cross K/V into the stream slots
 * streams_host[i] (once per utterance, decoder.rs:205-216). */
VKB_API vkb_status vkb_session_encode(vkb_session* s, int32_t n_clips, const float* logmel_dev,
                                      const int32_t* streams_host);
/* Device pointer to the last encoder output [n_clips][n_audio_ctx][d_model] f32 (after ln_post). */
VKB_API const float* vkb_session_encoder_output(const vkb_session* s);
/* Synchronous copy of the first n_floats of that output to host memory. */
VKB_API vkb_status vkb_session_read_encoder_output(const vkb_session* s, float* host, size_t n_floats);
/* Device pointers to decoder layer `layer`'s cross-attention K/V store, rows
 * stream*n_audio_ctx + t of d_model channels: Q8_0 quants (int8) with one f16
 * scale per 32 channels when the session was created with cross_kv_q8 (the
 * scale pointers are NULL for the f16 store). Rows of a stream are valid after
 * vkb_session_encode wrote it. The counterpart of the reference's
 * project_kv_into result (whisper/nn.rs:185, decoder.rs:205-216). */
VKB_API vkb_status vkb_session_cross_kv(const vkb_session* s, int32_t layer, const void** k, const void** v,
                                        const void** k_scale, const void** v_scale);
/* One decoder step over n_tok tokens (token i of stream streams_host[i] at
 * position positions_host[i]; tokens of one stream contiguous and
 * consecutive): appends their self-attention K/V, writes logits
 * [n_tok][n_vocab] f32 (logits_dev, or the session's buffer when NULL) and the
 * greedy argmax ids (ids_dev, or the session's buffer when NULL). Asynchronous
 * on the context stream. */
VKB_API vkb_status vkb_session_step(vkb_session* s, int32_t n_tok, const int32_t* streams_host,
                                    const int32_t* positions_host, const int32_t* tokens_host,
                                    float* logits_dev, int32_t* ids_dev);
/* vkb_session_step whose tokens may come from the device: where
 * feed_rows_host[i] >= 0, token i is feed_ids_dev[feed_rows_host[i]] (e.g.
 * the greedy id a previous step wrote for that stream into its ids_dev),
 * read on the device when the step runs; elsewhere tokens_host[i] is used.
 * A greedy loop can so launch step t+1 before reading step t's ids back
 * (the reference's loop reads each id on the host first, whisper/greedy.rs:32). */
VKB_API vkb_status vkb_session_step_feed(vkb_session* s, int32_t n_tok, const int32_t* streams_host,
                                         const int32_t* positions_host, const int32_t* tokens_host,
                                         const int32_t* feed_rows_host, const int32_t* feed_ids_dev,
                                         float* logits_dev, int32_t* ids_dev);
VKB_API const float* vkb_session_logits(const vkb_session* s);
VKB_API const int32_t* vkb_session_ids(const vkb_session* s);
/* Returns a finished stream's KV pages to the pool (continuous batching). */
VKB_API vkb_status vkb_session_release(vkb_session* s, int32_t stream);
/* Branches a decode stream: stream dst becomes a copy of the first n_pos
 * positions of stream src's self-attention cache (dst's own pages are
 * released first), so dst continues at position n_pos exactly as src would.
 * With copy_cross != 0 dst's cross-attention K/V rows are also copied from
 * src (once per clip: beams of one clip share them afterwards). This is the
 * per-beam branch of beam search: the reference deep-copies the host cache
 * (selfkv_snapshot / selfkv_restore, whisper/decoder.rs:343-368); here the
 * filled pages are shared (copy on write, as vkb_kv_copy_stream) and at most
 * one partly filled page is copied on the device. Asynchronous on the
 * context's stream. */
VKB_API vkb_status vkb_session_copy_stream(vkb_session* s, int32_t src, int32_t dst, int32_t n_pos,
                                           int32_t copy_cross);

/* ---- Whisper log-mel frontend --------------------------------------------
 * Replaces vokra_models::whisper::mel::log_mel(pcm, n_mels)
 * (crates/vokra-models/src/whisper/mel.rs:123, via
 * crates/vokra-ops/src/fused_logmel.rs:80) for a batch of clips.
 * pcm_dev: n_clips rows of `stride` f32 samples at 16 kHz (row c starts at
 * pcm_dev + c*stride); lengths_dev (device int32, may be NULL = all `stride`)
 * gives each clip's valid samples, the rest reads as zeros. Every clip is
 * zero-padded or trimmed to 30 s as the reference does. out_dev: f32
 * [n_clips][n_mels][3000], the layout vkb_session_encode takes. n_mels in
 * 1..256 (80 or 128 for Whisper). Asynchronous on the context's stream. */
VKB_API vkb_status vkb_log_mel(vkb_context* ctx, const float* pcm_dev, int64_t n_clips, int64_t stride,
                               const int32_t* lengths_dev, int32_t n_mels, float* out_dev);

#ifdef __cplusplus
}
#endif
#endif /* VKB200_H */
