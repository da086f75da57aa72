// whisper.cu — the Whisper model on the B200: GGUF load (weights repacked once
// into the device tile layout), batched encoder forward, once-per-utterance
// cross-attention K/V projection into the int8 (Q8_0) or f16 cross store, and
// the batched decoder step over the paged Q8_0 self-attention KV cache.
//
// Forward semantics follow the reference CPU path:
//   encoder  crates/vokra-models/src/whisper/encoder.rs:41-110 (conv1 -> GELU ->
//            conv2(s2) -> GELU -> + pos) and :180-236 (pre-norm blocks), ln_post;
//   decoder  crates/vokra-models/src/whisper/decoder.rs:413-566 (token + pos
//            embedding, causal self-attention over the cache, cross-attention
//            over the encoder output, MLP, final LayerNorm, tied logits);
//   nn       whisper/nn.rs:62-300 (q scaled by d_head^-0.5 after its bias,
//            k_proj without bias, exact-erf GELU).
// The q|k|v projections of a block run as one fused GEMM (weights concatenated
// along the output dimension at load time); the cross K/V projections of all
// decoder layers run once per utterance.
#include "common.cuh"
#include "weights.cuh"
#include "linear.cuh"
#include "kv.cuh"
#include "gguf.cuh"
#include "elementwise.cuh"
#include "enc_attn.cuh"
#include <memory>
#include <algorithm>
#include <cstdlib>
#include <map>
#include <tuple>

using namespace vkb;

namespace vkb {
// f32 rows -> f16 rows with the stream remap (the f16 cross store)
__global__ void copy_rows_f16_kernel(const float* __restrict__ x, int64_t ld, int64_t n_rows, int W,
                                     __half* __restrict__ y, const int32_t* __restrict__ map, int group) {
    pdl_entry();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_rows * W) return;
    const int64_t r = i / W;
    const int c = (int)(i % W);
    const int64_t dst = map ? (int64_t)map[r / group] * group + r % group : r;
    y[dst * W + c] = __float2half_rn(x[r * ld + c]);
}
static void run_copy_rows_f16(vkb_context* ctx, const float* x, int64_t ld, int64_t n_rows, int W, __half* y,
                              const int32_t* map, int group) {
    int64_t tot = n_rows * W;
    launch_pdl(ctx, copy_rows_f16_kernel, (unsigned)((tot + 255) / 256), 256, 0, x, ld, n_rows, W, y, map, group);
    VKB_CUDA(cudaGetLastError());
    ctx->count();
}
}  // namespace vkb

namespace {

struct WDel {
    void operator()(vkb_weight* w) const { delete w; }
};
using WPtr = std::unique_ptr<vkb_weight, WDel>;

struct EncLayer {
    DevBuf ln1g, ln1b, ln2g, ln2b, qkv_b, o_b, fc1_b, fc2_b;
    WPtr qkv, o, fc1, fc2;
};
struct DecLayer {
    DevBuf ln1g, ln1b, ln2g, ln2b, ln3g, ln3b, qkv_b, o_b, cq_b, co_b, fc1_b, fc2_b, ckv_b;
    WPtr qkv, o, cq, co, fc1, fc2, ckv;
};

DevBuf upload_f32(const std::vector<float>& v) {
    DevBuf b(v.size() * 4);
    VKB_CUDA(cudaMemcpy(b.p, v.data(), v.size() * 4, cudaMemcpyHostToDevice));
    return b;
}

}  // namespace

struct vkb_whisper {
    vkb_context* ctx = nullptr;
    vkb_whisper_dims dims{};
    uint32_t wtag = 0;
    int k1 = 0, k1p = 0;  // conv1 im2col width and its 64-multiple padding
    WPtr conv1, conv2, tok_emb;
    DevBuf conv1_b, conv2_b, enc_pos, enc_lng, enc_lnb, dec_pos, dec_lng, dec_lnb;
    std::vector<EncLayer> enc;
    std::vector<DecLayer> dec;
};

struct vkb_session {
    vkb_whisper* m = nullptr;
    vkb_context* ctx = nullptr;
    vkb_session_options opt{};
    vkb_kv_pool* pool = nullptr;
    int max_tok = 0;
    // decoder step buffers
    DevBuf h, xln, qkv, ctxb, qc, ffn, logits, ids, tok, pos, seq, ws, feed;
    int32_t* h_tok = nullptr;  // pinned staging: tokens | positions | streams | feed rows
    cudaEvent_t staged = nullptr;
    bool staged_pending = false;
    // cross-attention store: per layer K and V planes for n_stream * n_audio_ctx rows
    DevBuf ck, cv, cks, cvs;
    // encoder buffers (max_clips)
    DevBuf col1, bufA, bufB, eh, exln, ectx, eout, emap;
    int32_t* h_map = nullptr;
    int last_clips = 0;
    // cross-attention partials of a step (session-owned, so a recorded step
    // never points into a context workspace that a later call regrows)
    DevBuf xws;
    size_t xws_floats = 0;
    // Recorded decode steps, keyed by everything that shapes their launches:
    // (n_tok, query groups, queries per group, key splits, logits, ids, precision).
    struct StepGraph {
        cudaGraphExec_t exec = nullptr;
        uint64_t launches = 0;
        bool seen = false;    // ran once eagerly (buffers sized, attributes set)
        bool failed = false;  // recording was refused: run eagerly
    };
    std::map<std::tuple<int, int, int, int, uintptr_t, uintptr_t, int>, StepGraph> graphs;
    bool use_graphs = true;
    cudaStream_t rec_stream = nullptr;  // private stream the step is recorded on
    ~vkb_session() {
        if (rec_stream) cudaStreamDestroy(rec_stream);
        for (auto& kv : graphs)
            if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
        if (pool) kv_pool_destroy(pool);
        if (h_tok) cudaFreeHost(h_tok);
        if (h_map) cudaFreeHost(h_map);
        if (staged) cudaEventDestroy(staged);
    }
};

namespace {

// Concatenates GGUF Linear payloads (same dtype, same k) along the output dim.
WPtr fused_linear(vkb_context* ctx, const GgufFile& g, const std::vector<std::string>& names, int64_t k,
                  uint32_t& tag_out) {
    std::vector<uint8_t> bytes;
    int64_t n_total = 0;
    uint32_t tag = 0;
    for (size_t i = 0; i < names.size(); ++i) {
        const GgufTensor& t = g.tensor(names[i]);
        if (t.dims.size() != 2 || t.dims[1] != k) fail(VKB_ERROR_MODEL_LOAD, "whisper: " + names[i] + " has the wrong shape");
        if (i == 0) tag = t.tag;
        else if (t.tag != tag) fail(VKB_ERROR_MODEL_LOAD, "whisper: fused projections need one dtype (" + names[i] + ")");
        const uint8_t* p = g.data(t);
        bytes.insert(bytes.end(), p, p + t.nbytes);
        n_total += t.dims[0];
    }
    tag_out = tag;
    return WPtr(upload_weight(ctx, tag, n_total, k, bytes.data(), bytes.size()));
}

std::vector<float> bias_or_zero(const GgufFile& g, const std::string& name, int64_t n) {
    if (g.has(name)) return g.f32(name, {n});
    return std::vector<float>((size_t)n, 0.0f);
}

std::vector<float> cat(std::initializer_list<std::vector<float>> parts) {
    std::vector<float> r;
    for (auto& p : parts) r.insert(r.end(), p.begin(), p.end());
    return r;
}

// conv weight [d][c][3] F32/F16 -> dense f16 [d][k_pad] (zero columns past c*3)
WPtr conv_weight(vkb_context* ctx, const GgufFile& g, const std::string& name, int64_t d, int64_t c, int k_pad) {
    std::vector<float> w = g.f32(name, {d, c, 3});
    std::vector<float> p((size_t)d * k_pad, 0.0f);
    for (int64_t o = 0; o < d; ++o) memcpy(&p[(size_t)o * k_pad], &w[(size_t)o * c * 3], (size_t)c * 3 * 4);
    return WPtr(upload_weight(ctx, VKB_GGML_F32, d, k_pad, p.data(), p.size() * 4));
}

vkb_whisper* load_whisper(vkb_context* ctx, const char* path) {
    if (!ctx || !path) fail(VKB_ERROR_INVALID_ARGUMENT, "whisper_load: null argument");
    std::unique_ptr<GgufFile> g(gguf_open(path));
    auto it = g->meta.find("general.architecture");
    if (it == g->meta.end() || it->second.s != "whisper")
        fail(VKB_ERROR_MODEL_LOAD, "whisper_load: general.architecture is not 'whisper'");
    auto m = std::make_unique<vkb_whisper>();
    m->ctx = ctx;
    auto& D = m->dims;
    D.n_mels = (int32_t)g->u32("vokra.whisper.n_mels");
    D.n_audio_ctx = (int32_t)g->u32("vokra.whisper.n_audio_ctx");
    D.d_model = (int32_t)g->u32("vokra.whisper.n_audio_state");
    D.n_audio_head = (int32_t)g->u32("vokra.whisper.n_audio_head");
    D.n_audio_layer = (int32_t)g->u32("vokra.whisper.n_audio_layer");
    D.n_text_ctx = (int32_t)g->u32("vokra.whisper.n_text_ctx");
    D.n_text_head = (int32_t)g->u32("vokra.whisper.n_text_head");
    D.n_text_layer = (int32_t)g->u32("vokra.whisper.n_text_layer");
    D.n_vocab = (int32_t)g->u32("vokra.whisper.n_vocab");
    D.ffn_dim = (int32_t)g->u32("vokra.whisper.ffn_dim");
    D.eot = (int32_t)g->u32("vokra.whisper.eot");
    if ((int32_t)g->u32("vokra.whisper.n_text_state") != D.d_model)
        fail(VKB_ERROR_MODEL_LOAD, "whisper_load: n_text_state != n_audio_state");
    auto sit = g->meta.find("vokra.whisper.decoder_start_ids");
    if (sit != g->meta.end()) {
        D.n_start_ids = (int32_t)std::min<size_t>(8, sit->second.arr.size());
        for (int i = 0; i < D.n_start_ids; ++i) D.start_ids[i] = (int32_t)sit->second.arr[i].u;
    }
    const int64_t d = D.d_model, f = D.ffn_dim;
    if (d % 64 || d / D.n_audio_head != 64 || d / D.n_text_head != 64)
        fail(VKB_ERROR_UNSUPPORTED_OP, "whisper_load: the B200 kernels need d_head = 64");
    VKB_CUDA(cudaSetDevice(ctx->device));
    m->k1 = D.n_mels * 3;
    m->k1p = (m->k1 + 63) / 64 * 64;
    m->conv1 = conv_weight(ctx, *g, "model.encoder.conv1.weight", d, D.n_mels, m->k1p);
    m->conv1_b = upload_f32(g->f32("model.encoder.conv1.bias", {d}));
    m->conv2 = conv_weight(ctx, *g, "model.encoder.conv2.weight", d, d, (int)(d * 3));
    m->conv2_b = upload_f32(g->f32("model.encoder.conv2.bias", {d}));
    m->enc_pos = upload_f32(g->f32("model.encoder.embed_positions.weight", {D.n_audio_ctx, d}));
    for (int i = 0; i < D.n_audio_layer; ++i) {
        std::string p = "model.encoder.layers." + std::to_string(i);
        EncLayer L;
        L.ln1g = upload_f32(g->f32(p + ".self_attn_layer_norm.weight", {d}));
        L.ln1b = upload_f32(g->f32(p + ".self_attn_layer_norm.bias", {d}));
        L.ln2g = upload_f32(g->f32(p + ".final_layer_norm.weight", {d}));
        L.ln2b = upload_f32(g->f32(p + ".final_layer_norm.bias", {d}));
        L.qkv = fused_linear(ctx, *g, {p + ".self_attn.q_proj.weight", p + ".self_attn.k_proj.weight", p + ".self_attn.v_proj.weight"}, d, m->wtag);
        L.qkv_b = upload_f32(cat({g->f32(p + ".self_attn.q_proj.bias", {d}), bias_or_zero(*g, p + ".self_attn.k_proj.bias", d),
                                  g->f32(p + ".self_attn.v_proj.bias", {d})}));
        uint32_t t;
        L.o = fused_linear(ctx, *g, {p + ".self_attn.out_proj.weight"}, d, t);
        L.o_b = upload_f32(g->f32(p + ".self_attn.out_proj.bias", {d}));
        L.fc1 = fused_linear(ctx, *g, {p + ".fc1.weight"}, d, t);
        L.fc1_b = upload_f32(g->f32(p + ".fc1.bias", {f}));
        L.fc2 = fused_linear(ctx, *g, {p + ".fc2.weight"}, f, t);
        L.fc2_b = upload_f32(g->f32(p + ".fc2.bias", {d}));
        m->enc.push_back(std::move(L));
    }
    m->enc_lng = upload_f32(g->f32("model.encoder.layer_norm.weight", {d}));
    m->enc_lnb = upload_f32(g->f32("model.encoder.layer_norm.bias", {d}));
    uint32_t t;
    m->tok_emb = fused_linear(ctx, *g, {"model.decoder.embed_tokens.weight"}, d, t);
    if (m->tok_emb->n != D.n_vocab) fail(VKB_ERROR_MODEL_LOAD, "whisper_load: embed_tokens rows != n_vocab");
    m->dec_pos = upload_f32(g->f32("model.decoder.embed_positions.weight", {D.n_text_ctx, d}));
    for (int i = 0; i < D.n_text_layer; ++i) {
        std::string p = "model.decoder.layers." + std::to_string(i);
        DecLayer L;
        L.ln1g = upload_f32(g->f32(p + ".self_attn_layer_norm.weight", {d}));
        L.ln1b = upload_f32(g->f32(p + ".self_attn_layer_norm.bias", {d}));
        L.ln2g = upload_f32(g->f32(p + ".encoder_attn_layer_norm.weight", {d}));
        L.ln2b = upload_f32(g->f32(p + ".encoder_attn_layer_norm.bias", {d}));
        L.ln3g = upload_f32(g->f32(p + ".final_layer_norm.weight", {d}));
        L.ln3b = upload_f32(g->f32(p + ".final_layer_norm.bias", {d}));
        L.qkv = fused_linear(ctx, *g, {p + ".self_attn.q_proj.weight", p + ".self_attn.k_proj.weight", p + ".self_attn.v_proj.weight"}, d, t);
        L.qkv_b = upload_f32(cat({g->f32(p + ".self_attn.q_proj.bias", {d}), bias_or_zero(*g, p + ".self_attn.k_proj.bias", d),
                                  g->f32(p + ".self_attn.v_proj.bias", {d})}));
        L.o = fused_linear(ctx, *g, {p + ".self_attn.out_proj.weight"}, d, t);
        L.o_b = upload_f32(g->f32(p + ".self_attn.out_proj.bias", {d}));
        L.cq = fused_linear(ctx, *g, {p + ".encoder_attn.q_proj.weight"}, d, t);
        L.cq_b = upload_f32(g->f32(p + ".encoder_attn.q_proj.bias", {d}));
        L.ckv = fused_linear(ctx, *g, {p + ".encoder_attn.k_proj.weight", p + ".encoder_attn.v_proj.weight"}, d, t);
        L.ckv_b = upload_f32(cat({bias_or_zero(*g, p + ".encoder_attn.k_proj.bias", d), g->f32(p + ".encoder_attn.v_proj.bias", {d})}));
        L.co = fused_linear(ctx, *g, {p + ".encoder_attn.out_proj.weight"}, d, t);
        L.co_b = upload_f32(g->f32(p + ".encoder_attn.out_proj.bias", {d}));
        L.fc1 = fused_linear(ctx, *g, {p + ".fc1.weight"}, d, t);
        L.fc1_b = upload_f32(g->f32(p + ".fc1.bias", {f}));
        L.fc2 = fused_linear(ctx, *g, {p + ".fc2.weight"}, f, t);
        L.fc2_b = upload_f32(g->f32(p + ".fc2.bias", {d}));
        m->dec.push_back(std::move(L));
    }
    m->dec_lng = upload_f32(g->f32("model.decoder.layer_norm.weight", {d}));
    m->dec_lnb = upload_f32(g->f32("model.decoder.layer_norm.bias", {d}));
    return m.release();
}

constexpr float LN_EPS = 1e-5f;  // LAYER_NORM_DEFAULT_EPS, crates/vokra-backend-cpu/src/kernels/mod.rs:218

size_t ws_need(const vkb_context* ctx, const vkb_weight* w, int64_t m) {
    return plan_linear(ctx, w, m).ws_bytes;
}

vkb_session* create_session(vkb_whisper* m, const vkb_session_options* o) {
    if (!m || !o) fail(VKB_ERROR_INVALID_ARGUMENT, "session_create: null argument");
    if (o->max_streams <= 0 || o->max_clips < 0 || o->max_step_tokens <= 0)
        fail(VKB_ERROR_INVALID_ARGUMENT, "session_create: max_streams and max_step_tokens must be positive");
    auto s = std::make_unique<vkb_session>();
    s->m = m;
    s->ctx = m->ctx;
    s->opt = *o;
    const auto& D = m->dims;
    const int64_t d = D.d_model, f = D.ffn_dim, V = D.n_vocab, S = o->max_streams, T = D.n_audio_ctx;
    VKB_CUDA(cudaSetDevice(s->ctx->device));
    vkb_kv_pool_desc kd{};
    kd.n_layer = D.n_text_layer;
    kd.n_head = D.n_text_head;
    kd.d_head = (int32_t)(d / D.n_text_head);
    kd.n_stream = (int32_t)S;
    kd.n_codebook = 1;
    kd.max_time = D.n_text_ctx;
    kd.page_tokens = o->kv_page_tokens ? o->kv_page_tokens : 16;
    switch (o->self_kv_mode) {
        case VKB_SELF_KV_Q8_0: kd.mode = VKB_KV_Q8_0; break;
        case VKB_SELF_KV_F32: kd.mode = VKB_KV_FP32; break;
        case VKB_SELF_KV_Q4_0: kd.mode = VKB_KV_Q4_0; break;
        case VKB_SELF_KV_Q5_0: kd.mode = VKB_KV_Q5_0; break;
        default: fail(VKB_ERROR_INVALID_ARGUMENT, "session_create: bad self_kv_mode");
    }
    kd.layout = VKB_KV_LAYOUT_SEQUENCE;
    kd.n_pages = 0;
    s->pool = kv_pool_create(s->ctx, &kd);
    const int64_t mt = o->max_step_tokens;
    s->max_tok = (int)mt;
    s->h.alloc(mt * d * 4);
    // activations that feed a GEMM are f16 hi + lo planes (VKB_DT_F16X2)
    s->xln.alloc(mt * d * 4);
    s->qkv.alloc(mt * 3 * d * 4);
    s->ctxb.alloc(mt * d * 4);
    s->qc.alloc(mt * d * 4);
    s->ffn.alloc(mt * f * 4);
    s->logits.alloc(mt * V * 4);
    s->ids.alloc(mt * 4);
    s->tok.alloc(mt * 4);
    s->pos.alloc(mt * 4);
    s->seq.alloc(mt * 4);
    VKB_CUDA(cudaMallocHost(&s->h_tok, (size_t)mt * 4 * 4));
    s->feed.alloc(mt * 4);
    VKB_CUDA(cudaEventCreateWithFlags(&s->staged, cudaEventDisableTiming));
    // cross store
    const int64_t rows = S * T;
    const int64_t L = D.n_text_layer;
    if (o->cross_kv_q8) {
        s->ck.alloc(L * rows * d);
        s->cv.alloc(L * rows * d);
        s->cks.alloc(L * rows * (d / 32) * 2);
        s->cvs.alloc(L * rows * (d / 32) * 2);
    } else {
        s->ck.alloc(L * rows * d * 2);
        s->cv.alloc(L * rows * d * 2);
    }
    // encoder buffers
    const int64_t C = o->max_clips;
    if (C > 0) {
        const int64_t Tin = 2 * T, M = C * T;
        s->col1.alloc(C * Tin * m->k1p * 4);
        // bufA holds the conv1 output [C*Tin][d], the MLP hidden [M][ffn] and the
        // cross K/V projection [M][2d] f32 in turn.
        s->bufA.alloc(std::max({M * f * 4, C * Tin * d * 4, M * 2 * d * 4}));
        s->bufB.alloc(M * 3 * d * 4);
        s->eh.alloc(M * d * 4);
        s->exln.alloc(M * d * 4);
        s->ectx.alloc(M * d * 4);
        s->eout.alloc(M * d * 4);
        s->emap.alloc(C * 4);
        VKB_CUDA(cudaMallocHost(&s->h_map, (size_t)C * 4));
    }
    // split-K workspace for the largest step-size linears (sized once here)
    size_t ws = 0;
    const DecLayer& l0 = m->dec[0];
    for (const vkb_weight* w : {l0.qkv.get(), l0.o.get(), l0.cq.get(), l0.co.get(), l0.fc1.get(), l0.fc2.get(),
                                m->tok_emb.get()})
        for (int64_t mm = 1; mm <= mt; ++mm) ws = std::max(ws, ws_need(s->ctx, w, mm));
    if (C > 0) {
        const int64_t M = C * T;
        const EncLayer& e0 = m->enc[0];
        for (const vkb_weight* w : {e0.qkv.get(), e0.o.get(), e0.fc1.get(), e0.fc2.get(), m->conv1.get(), m->conv2.get(),
                                    l0.ckv.get()})
            for (int64_t mm = T; mm <= 2 * M; mm *= 2) ws = std::max(ws, ws_need(s->ctx, w, mm));
    }
    s->ws.alloc(std::max<size_t>(ws, 256));
    // Cross-attention partials: the balanced kernel keeps at most
    // sm_count * (ceil(n_tok / sm_count) + 2) row partials; the row-group
    // kernel (f16 store) at most (8 * sm_count + n_tok) split partials.
    {
        const int64_t H = D.n_text_head, sms = s->ctx->sm_count;
        const int64_t per = d + 2 * H;
        s->xws_floats = (size_t)std::max(sms * ((mt + sms - 1) / sms + 2), 8 * sms + mt) * per;
        s->xws.alloc(s->xws_floats * sizeof(float));
    }
    const char* g = std::getenv("VKB_STEP_GRAPHS");
    s->use_graphs = !(g && g[0] == '0');
    return s.release();
}

// Encoder forward of n clips plus the cross K/V projection into stream slots.
void session_encode(vkb_session* s, int n, const float* logmel, const int32_t* streams) {
    NvtxRange nvtx_range("vkb.session_encode");
    vkb_whisper* m = s->m;
    vkb_context* ctx = s->ctx;
    const auto& D = m->dims;
    if (n <= 0 || n > s->opt.max_clips) fail(VKB_ERROR_INVALID_ARGUMENT, "session_encode: n_clips out of range");
    if (!logmel || !streams) fail(VKB_ERROR_INVALID_ARGUMENT, "session_encode: null argument");
    for (int i = 0; i < n; ++i)
        if (streams[i] < 0 || streams[i] >= s->opt.max_streams)
            fail(VKB_ERROR_INVALID_ARGUMENT, "session_encode: stream id out of range");
    const int64_t d = D.d_model, f = D.ffn_dim, T = D.n_audio_ctx, Tin = 2 * T, M = (int64_t)n * T;
    // VKB_PREC_ENCODER_F16: the whole encode (conv stem, encoder, cross K/V
    // projections) runs single-f16 operands; the context's mode comes back after
    struct PrecisionScope {
        vkb_context* c;
        int saved;
        ~PrecisionScope() { c->precision = saved; }
    } scope{ctx, ctx->precision};
    if (ctx->precision == VKB_PREC_ENCODER_F16) ctx->precision = VKB_PREC_F16;
    float* ws = s->ws.as<float>();
    __half* bufA = s->bufA.as<__half>();
    __half* bufB = s->bufB.as<__half>();
    float* h = s->eh.as<float>();
    __half* xln = s->exln.as<__half>();
    __half* ectx = s->ectx.as<__half>();
    // GEMM inputs are f16 hi + lo planes in the default (split) precision
    const bool split = ctx->precision == VKB_PREC_SPLIT;
    const int AF = split ? VKB_DT_F16X2 : VKB_DT_F16;
    const int planes = split ? 2 : 1;
    // conv stem: conv1 (k3 s1 p1) + GELU, conv2 (k3 s2 p1) + GELU, + positions
    run_im2col_ct(ctx, logmel, n, D.n_mels, (int)Tin, 1, m->k1p, s->col1.as<__half>(), split);
    run_linear(ctx, m->conv1.get(), n * Tin, s->col1.p, AF, m->conv1_b.as<float>(), bufA, AF, VKB_EPI_GELU, nullptr,
               1.0f, ws, nullptr);
    run_im2col_tc(ctx, bufA, n, (int)d, (int)Tin, 2, bufB, planes);
    run_linear(ctx, m->conv2.get(), M, bufB, AF, m->conv2_b.as<float>(), xln, AF, VKB_EPI_GELU, nullptr, 1.0f, ws,
               nullptr);
    run_add_pos(ctx, xln, m->enc_pos.as<float>(), n, (int)T, (int)d, h, planes);
    const float scale = 1.0f / sqrtf((float)(d / D.n_audio_head));
    for (const EncLayer& L : m->enc) {
        run_layer_norm(ctx, h, M, (int)d, L.ln1g.as<float>(), L.ln1b.as<float>(), LN_EPS, xln, AF);
        LinearExtra x;
        x.n_scaled = d;
        run_linear_ex(ctx, L.qkv.get(), M, xln, AF, L.qkv_b.as<float>(), bufB, VKB_DT_F16, VKB_EPI_SCALE, nullptr,
                      scale, ws, nullptr, x);
        // bufA (the MLP hidden) is idle here: it holds the transposed V of the tensor-core attention
        run_encoder_attention(ctx, bufB, 3 * d, (int)d, (int)(2 * d), n, (int)T, D.n_audio_head, 64, ectx, d,
                              split ? ectx + M * d : nullptr, reinterpret_cast<__half*>(s->bufA.p), s->bufA.n / 2);
        run_linear(ctx, L.o.get(), M, ectx, AF, L.o_b.as<float>(), h, VKB_DT_F32, VKB_EPI_RESIDUAL, h, 1.0f, ws,
                   nullptr);
        run_layer_norm(ctx, h, M, (int)d, L.ln2g.as<float>(), L.ln2b.as<float>(), LN_EPS, xln, AF);
        run_linear(ctx, L.fc1.get(), M, xln, AF, L.fc1_b.as<float>(), bufA, AF, VKB_EPI_GELU, nullptr, 1.0f, ws,
                   nullptr);
        run_linear(ctx, L.fc2.get(), M, bufA, AF, L.fc2_b.as<float>(), h, VKB_DT_F32, VKB_EPI_RESIDUAL, h, 1.0f, ws,
                   nullptr);
    }
    (void)f;
    run_layer_norm(ctx, h, M, (int)d, m->enc_lng.as<float>(), m->enc_lnb.as<float>(), LN_EPS, s->eout.p, 0);
    run_layer_norm(ctx, h, M, (int)d, m->enc_lng.as<float>(), m->enc_lnb.as<float>(), LN_EPS, xln, AF);
    // cross K/V for every decoder layer, rows remapped to the stream slots
    if (s->staged_pending) VKB_CUDA(cudaEventSynchronize(s->staged));
    memcpy(s->h_map, streams, (size_t)n * 4);
    VKB_CUDA(cudaMemcpyAsync(s->emap.p, s->h_map, (size_t)n * 4, cudaMemcpyHostToDevice, ctx->stream));
    VKB_CUDA(cudaEventRecord(s->staged, ctx->stream));
    s->staged_pending = true;
    const int32_t* map = s->emap.as<int32_t>();
    const int64_t rows = (int64_t)s->opt.max_streams * T;
    for (int l = 0; l < D.n_text_layer; ++l) {
        const DecLayer& L = m->dec[l];
        if (s->opt.cross_kv_q8) {
            int8_t* kq = s->ck.as<int8_t>() + (size_t)l * rows * d;
            int8_t* vq = s->cv.as<int8_t>() + (size_t)l * rows * d;
            __half* ks = s->cks.as<__half>() + (size_t)l * rows * (d / 32);
            __half* vs = s->cvs.as<__half>() + (size_t)l * rows * (d / 32);
            // the projection's epilogue packs Q8_0 rows straight into the store (no f32 round trip)
            if (run_linear_q8_pair(ctx, L.ckv.get(), M, xln, L.ckv_b.as<float>(), d, kq, ks, vq, vs, map, (int)T,
                                   split))
                continue;
            float* tmp = reinterpret_cast<float*>(bufA);  // [M][2d] f32
            run_linear(ctx, L.ckv.get(), M, xln, AF, L.ckv_b.as<float>(), tmp, VKB_DT_F32, VKB_EPI_NONE,
                       nullptr, 1.0f, ws, nullptr);
            run_quantize_rows(ctx, tmp, 2 * d, M, (int)d, kq, ks, map, (int)T);
            run_quantize_rows(ctx, tmp + d, 2 * d, M, (int)d, vq, vs, map, (int)T);
        } else {
            float* tmp = reinterpret_cast<float*>(bufA);  // [M][2d] f32
            run_linear(ctx, L.ckv.get(), M, xln, AF, L.ckv_b.as<float>(), tmp, VKB_DT_F32, VKB_EPI_NONE,
                       nullptr, 1.0f, ws, nullptr);
            run_copy_rows_f16(ctx, tmp, 2 * d, M, (int)d, s->ck.as<__half>() + (size_t)l * rows * d, map, (int)T);
            run_copy_rows_f16(ctx, tmp + d, 2 * d, M, (int)d, s->cv.as<__half>() + (size_t)l * rows * d, map, (int)T);
        }
    }
    s->last_clips = n;
}

// Tokens fed from the device: token i = feed_ids[rows[i]] where rows[i] >= 0
// (a previous step's greedy ids, never seen by the host); elsewhere the host
// value already copied stays.
__global__ void feed_tokens_kernel(int32_t* tok, const int32_t* __restrict__ rows, const int32_t* __restrict__ feed_ids,
                                   int n_tok) {
    pdl_entry();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n_tok && rows[i] >= 0) tok[i] = feed_ids[rows[i]];
}

void session_step(vkb_session* s, int n_tok, const int32_t* streams, const int32_t* positions, const int32_t* tokens,
                  float* logits_out, int32_t* ids_out, const int32_t* feed_rows = nullptr,
                  const int32_t* feed_ids = nullptr) {
    NvtxRange nvtx_range("vkb.session_step");
    vkb_whisper* m = s->m;
    vkb_context* ctx = s->ctx;
    const auto& D = m->dims;
    if (n_tok <= 0 || n_tok > s->max_tok) fail(VKB_ERROR_INVALID_ARGUMENT, "session_step: n_tok out of range");
    if (!streams || !positions || !tokens) fail(VKB_ERROR_INVALID_ARGUMENT, "session_step: null argument");
    if ((feed_rows == nullptr) != (feed_ids == nullptr))
        fail(VKB_ERROR_INVALID_ARGUMENT, "session_step: feed rows and feed ids go together");
    for (int i = 0; i < n_tok; ++i) {
        if (feed_rows && feed_rows[i] >= 0) {
            if (feed_rows[i] >= s->max_tok) fail(VKB_ERROR_INVALID_ARGUMENT, "session_step: feed row out of range");
            if (positions[i] < 0 || positions[i] >= D.n_text_ctx)
                fail(VKB_ERROR_INVALID_ARGUMENT, "whisper decoder: position " + std::to_string(positions[i] + 1) +
                                                     " exceeds n_text_ctx " + std::to_string(D.n_text_ctx));
            continue;
        }
        if (tokens[i] < 0 || tokens[i] >= D.n_vocab)
            fail(VKB_ERROR_INVALID_ARGUMENT, "whisper decoder: token id " + std::to_string(tokens[i]) + " >= n_vocab " +
                                                 std::to_string(D.n_vocab));
        if (positions[i] < 0 || positions[i] >= D.n_text_ctx)
            fail(VKB_ERROR_INVALID_ARGUMENT, "whisper decoder: position " + std::to_string(positions[i] + 1) +
                                                 " exceeds n_text_ctx " + std::to_string(D.n_text_ctx));
    }
    const int64_t d = D.d_model, T = D.n_audio_ctx;
    kv_begin_step(s->pool, n_tok, streams, positions);
    if (s->staged_pending) VKB_CUDA(cudaEventSynchronize(s->staged));
    memcpy(s->h_tok, tokens, (size_t)n_tok * 4);
    memcpy(s->h_tok + n_tok, positions, (size_t)n_tok * 4);
    memcpy(s->h_tok + 2 * n_tok, streams, (size_t)n_tok * 4);
    VKB_CUDA(cudaMemcpyAsync(s->tok.p, s->h_tok, (size_t)n_tok * 4, cudaMemcpyHostToDevice, ctx->stream));
    VKB_CUDA(cudaMemcpyAsync(s->pos.p, s->h_tok + n_tok, (size_t)n_tok * 4, cudaMemcpyHostToDevice, ctx->stream));
    VKB_CUDA(cudaMemcpyAsync(s->seq.p, s->h_tok + 2 * n_tok, (size_t)n_tok * 4, cudaMemcpyHostToDevice, ctx->stream));
    if (feed_rows) {
        int32_t* hf = s->h_tok + 3 * n_tok;
        for (int i = 0; i < n_tok; ++i) hf[i] = feed_rows[i] >= 0 ? feed_rows[i] : -1;
        VKB_CUDA(cudaMemcpyAsync(s->feed.p, hf, (size_t)n_tok * 4, cudaMemcpyHostToDevice, ctx->stream));
        launch_pdl(ctx, feed_tokens_kernel, (unsigned)((n_tok + 127) / 128), 128, 0, s->tok.as<int32_t>(),
                   s->feed.as<int32_t>(), feed_ids, n_tok);
        VKB_CUDA(cudaGetLastError());
        ctx->count();
    }
    VKB_CUDA(cudaEventRecord(s->staged, ctx->stream));
    s->staged_pending = true;

    // Launch sequence of the step. Every pointer and shape it uses is fixed
    // for a given key, and the per-step inputs (tokens, positions, streams,
    // page table, rows, query groups) were copied into fixed device buffers
    // above, so after one eager run the sequence is recorded once into a CUDA
    // graph and replayed with a single launch (host cost per step: one graph
    // launch instead of ~600 kernel launches).
    float* lg = logits_out ? logits_out : s->logits.as<float>();
    int32_t* ids = ids_out ? ids_out : s->ids.as<int32_t>();
    auto launch_all = [&]() {
        float* h = s->h.as<float>();
        __half* xln = s->xln.as<__half>();
        float* qkv = s->qkv.as<float>();
        __half* ctxb = s->ctxb.as<__half>();
        float* qc = s->qc.as<float>();
        __half* ffn = s->ffn.as<__half>();
        float* ws = s->ws.as<float>();
        const int AF = ctx->precision != VKB_PREC_F16 ? VKB_DT_F16X2 : VKB_DT_F16;
        run_embed(ctx, m->tok_emb.get(), s->tok.as<int32_t>(), s->pos.as<int32_t>(), n_tok, m->dec_pos.as<float>(), h);
        const float scale = 1.0f / sqrtf((float)(d / D.n_text_head));
        const int64_t rows = (int64_t)s->opt.max_streams * T;
        // A residual projection (h += x.W^T + bias) followed by the next
        // LayerNorm: with split-K, the partials are reduced inside the fused
        // residual + LayerNorm kernel instead of a separate reduce kernel.
        auto residual_ln = [&](const vkb_weight* w, const void* x_in, const float* bias, const float* g,
                               const float* b) {
            int sp = 1;
            LinearExtra rx;
            rx.splits_out = &sp;
            run_linear_ex(ctx, w, n_tok, x_in, AF, bias, h, VKB_DT_F32, VKB_EPI_RESIDUAL, h, 1.0f, ws, nullptr, rx);
            if (sp > 1) run_reduce_residual_ln(ctx, ws, sp, n_tok, (int)d, bias, h, g, b, LN_EPS, xln, AF);
            else run_layer_norm(ctx, h, n_tok, (int)d, g, b, LN_EPS, xln, AF);
        };
        run_layer_norm(ctx, h, n_tok, (int)d, m->dec[0].ln1g.as<float>(), m->dec[0].ln1b.as<float>(), LN_EPS, xln,
                       AF);
        // the cross store is written by the encoder and the step starts with host copies (a full
        // barrier), so the cross-attention may fill its ring before the query projection ends
        static const bool xa_early = [] { const char* v = std::getenv("VKB_XA_EARLY"); return !v || v[0] != '0'; }();
        for (int l = 0; l < D.n_text_layer; ++l) {
            const DecLayer& L = m->dec[l];
            LinearExtra x;
            x.n_scaled = d;
            // with the fused decode attention the split-K partials are summed there
            int qkv_splits = 1;
            const bool fused = kv_decode_fused(s->pool);
            if (fused) x.splits_out = &qkv_splits;
            run_linear_ex(ctx, L.qkv.get(), n_tok, xln, AF, L.qkv_b.as<float>(), qkv, VKB_DT_F32, VKB_EPI_SCALE,
                          nullptr, scale, ws, nullptr, x);
            if (fused && qkv_splits > 1)
                kv_append_attention_ex(s->pool, l, qkv, 3 * d, ctxb, AF, ws, qkv_splits, L.qkv_b.as<float>(), scale);
            else
                kv_append_attention_ex(s->pool, l, qkv, 3 * d, ctxb, AF);
            residual_ln(L.o.get(), ctxb, L.o_b.as<float>(), L.ln2g.as<float>(), L.ln2b.as<float>());
            run_linear(ctx, L.cq.get(), n_tok, xln, AF, L.cq_b.as<float>(), qc, VKB_DT_F32, VKB_EPI_SCALE, nullptr,
                       scale, ws, nullptr);
            if (s->opt.cross_kv_q8) {
                run_dense_attention(ctx, n_tok, D.n_text_head, 64, qc, s->seq.as<int32_t>(),
                                    s->ck.as<int8_t>() + (size_t)l * rows * d, s->cv.as<int8_t>() + (size_t)l * rows * d,
                                    s->cks.as<__half>() + (size_t)l * rows * (d / 32),
                                    s->cvs.as<__half>() + (size_t)l * rows * (d / 32), (int)T, VKB_KV_Q8_0, ctxb,
                                    AF, s->xws.as<float>(), s->xws_floats, xa_early);
            } else {
                run_dense_attention(ctx, n_tok, D.n_text_head, 64, qc, s->seq.as<int32_t>(),
                                    s->ck.as<__half>() + (size_t)l * rows * d, s->cv.as<__half>() + (size_t)l * rows * d,
                                    nullptr, nullptr, (int)T, VKB_DT_F16, ctxb, AF, s->xws.as<float>(), s->xws_floats);
            }
            residual_ln(L.co.get(), ctxb, L.co_b.as<float>(), L.ln3g.as<float>(), L.ln3b.as<float>());
            run_linear(ctx, L.fc1.get(), n_tok, xln, AF, L.fc1_b.as<float>(), ffn, AF, VKB_EPI_GELU,
                       nullptr, 1.0f, ws, nullptr);
            const bool last = l + 1 == D.n_text_layer;
            residual_ln(L.fc2.get(), ffn, L.fc2_b.as<float>(),
                        last ? m->dec_lng.as<float>() : m->dec[l + 1].ln1g.as<float>(),
                        last ? m->dec_lnb.as<float>() : m->dec[l + 1].ln1b.as<float>());
        }
        run_linear(ctx, m->tok_emb.get(), n_tok, xln, AF, nullptr, lg, VKB_DT_F32, VKB_EPI_NONE, nullptr, 1.0f, ws,
                   nullptr);
        run_argmax(ctx, lg, n_tok, D.n_vocab, ids);
    };
    const auto key = std::make_tuple(n_tok, pool_groups(s->pool), pool_maxq(s->pool), pool_splits(s->pool),
                                     (uintptr_t)lg, (uintptr_t)ids, ctx->precision);
    vkb_session::StepGraph& sg = s->graphs[key];
    if (!s->use_graphs || sg.failed || !sg.seen) {
        launch_all();
        sg.seen = true;
        return;
    }
    if (!sg.exec) {
        // Record on the session's private stream (the context's stream may be
        // the legacy default stream, which cannot be recorded); nothing runs
        // while recording, and the graph is then launched on the context's stream.
        if (!s->rec_stream) VKB_CUDA(cudaStreamCreateWithFlags(&s->rec_stream, cudaStreamNonBlocking));
        const uint64_t l0 = ctx->launches;
        cudaStream_t user = ctx->stream;
        cudaGraph_t graph = nullptr;
        VKB_CUDA(cudaStreamBeginCapture(s->rec_stream, cudaStreamCaptureModeThreadLocal));
        ctx->stream = s->rec_stream;
        try {
            launch_all();
        } catch (...) {
            ctx->stream = user;
            cudaStreamEndCapture(s->rec_stream, &graph);
            if (graph) cudaGraphDestroy(graph);
            throw;
        }
        ctx->stream = user;
        cudaError_t e = cudaStreamEndCapture(s->rec_stream, &graph);
        if (e == cudaSuccess) e = cudaGraphInstantiate(&sg.exec, graph, 0);
        if (graph) cudaGraphDestroy(graph);
        sg.launches = ctx->launches - l0;  // recorded, not yet run: counted at each replay
        ctx->launches = l0;
        if (e != cudaSuccess) {
            (void)cudaGetLastError();
            sg.exec = nullptr;
            sg.failed = true;
            launch_all();
            return;
        }
    }
    VKB_CUDA(cudaGraphLaunch(sg.exec, ctx->stream));
    ctx->count((int)sg.launches);
}

}  // namespace

extern "C" {

vkb_status vkb_whisper_load(vkb_context* ctx, const char* gguf_path, vkb_whisper** out) {
    return guard([&] {
        if (!out) fail(VKB_ERROR_INVALID_ARGUMENT, "whisper_load: null out");
        *out = load_whisper(ctx, gguf_path);
    });
}

vkb_status vkb_whisper_get_dims(const vkb_whisper* m, vkb_whisper_dims* out) {
    return guard([&] {
        if (!m || !out) fail(VKB_ERROR_INVALID_ARGUMENT, "whisper_get_dims: null argument");
        *out = m->dims;
    });
}

vkb_status vkb_whisper_destroy(vkb_whisper* m) {
    return guard([&] {
        if (m && m->ctx) cudaStreamSynchronize(m->ctx->stream);
        delete m;
    });
}

vkb_status vkb_session_create(vkb_whisper* m, const vkb_session_options* opt, vkb_session** out) {
    return guard([&] {
        if (!out) fail(VKB_ERROR_INVALID_ARGUMENT, "session_create: null out");
        *out = create_session(m, opt);
    });
}

vkb_status vkb_session_destroy(vkb_session* s) {
    return guard([&] {
        if (s && s->ctx) cudaStreamSynchronize(s->ctx->stream);
        delete s;
    });
}

vkb_status vkb_session_encode(vkb_session* s, int32_t n_clips, const float* logmel_dev, const int32_t* streams_host) {
    return guard([&] {
        if (!s) fail(VKB_ERROR_INVALID_ARGUMENT, "session_encode: null session");
        session_encode(s, n_clips, logmel_dev, streams_host);
    });
}

const float* vkb_session_encoder_output(const vkb_session* s) { return s ? s->eout.as<float>() : nullptr; }

vkb_status vkb_session_cross_kv(const vkb_session* s, int32_t layer, const void** k, const void** v,
                                const void** k_scale, const void** v_scale) {
    return guard([&] {
        if (!s || !k || !v || !k_scale || !v_scale) fail(VKB_ERROR_INVALID_ARGUMENT, "cross_kv: null argument");
        if (layer < 0 || layer >= s->m->dims.n_text_layer) fail(VKB_ERROR_INVALID_ARGUMENT, "cross_kv: bad layer");
        const int64_t d = s->m->dims.d_model;
        const size_t rows = (size_t)s->opt.max_streams * s->m->dims.n_audio_ctx;
        if (s->opt.cross_kv_q8) {
            *k = s->ck.as<int8_t>() + (size_t)layer * rows * d;
            *v = s->cv.as<int8_t>() + (size_t)layer * rows * d;
            *k_scale = s->cks.as<__half>() + (size_t)layer * rows * (d / 32);
            *v_scale = s->cvs.as<__half>() + (size_t)layer * rows * (d / 32);
        } else {
            *k = s->ck.as<__half>() + (size_t)layer * rows * d;
            *v = s->cv.as<__half>() + (size_t)layer * rows * d;
            *k_scale = *v_scale = nullptr;
        }
    });
}

vkb_status vkb_session_read_encoder_output(const vkb_session* s, float* host, size_t n_floats) {
    return guard([&] {
        if (!s || !host) fail(VKB_ERROR_INVALID_ARGUMENT, "read_encoder_output: null argument");
        if (n_floats * 4 > s->eout.n) fail(VKB_ERROR_INVALID_ARGUMENT, "read_encoder_output: too many floats");
        VKB_CUDA(cudaMemcpyAsync(host, s->eout.p, n_floats * 4, cudaMemcpyDeviceToHost, s->ctx->stream));
        VKB_CUDA(cudaStreamSynchronize(s->ctx->stream));
    });
}

vkb_status vkb_session_step(vkb_session* s, int32_t n_tok, const int32_t* streams_host, const int32_t* positions_host,
                            const int32_t* tokens_host, float* logits_dev, int32_t* ids_dev) {
    return guard([&] {
        if (!s) fail(VKB_ERROR_INVALID_ARGUMENT, "session_step: null session");
        session_step(s, n_tok, streams_host, positions_host, tokens_host, logits_dev, ids_dev);
    });
}

vkb_status vkb_session_step_feed(vkb_session* s, int32_t n_tok, const int32_t* streams_host,
                                 const int32_t* positions_host, const int32_t* tokens_host,
                                 const int32_t* feed_rows_host, const int32_t* feed_ids_dev, float* logits_dev,
                                 int32_t* ids_dev) {
    return guard([&] {
        if (!s) fail(VKB_ERROR_INVALID_ARGUMENT, "session_step: null session");
        if (!feed_rows_host || !feed_ids_dev) fail(VKB_ERROR_INVALID_ARGUMENT, "session_step_feed: null feed");
        session_step(s, n_tok, streams_host, positions_host, tokens_host, logits_dev, ids_dev, feed_rows_host,
                     feed_ids_dev);
    });
}

const float* vkb_session_logits(const vkb_session* s) { return s ? s->logits.as<float>() : nullptr; }
const int32_t* vkb_session_ids(const vkb_session* s) { return s ? s->ids.as<int32_t>() : nullptr; }

vkb_status vkb_session_copy_stream(vkb_session* s, int32_t src, int32_t dst, int32_t n_pos, int32_t copy_cross) {
    return guard([&] {
        if (!s) fail(VKB_ERROR_INVALID_ARGUMENT, "session_copy_stream: null session");
        if (src < 0 || src >= s->opt.max_streams || dst < 0 || dst >= s->opt.max_streams)
            fail(VKB_ERROR_INVALID_ARGUMENT, "session_copy_stream: stream out of range");
        if (n_pos < 0 || n_pos > s->m->dims.n_text_ctx)
            fail(VKB_ERROR_INVALID_ARGUMENT, "session_copy_stream: n_pos out of range");
        kv_copy_stream(s->pool, src, dst, n_pos);
        if (copy_cross && src != dst) {
            const auto& D = s->m->dims;
            const int64_t d = D.d_model, T = D.n_audio_ctx, rows = (int64_t)s->opt.max_streams * T;
            const size_t qb = s->opt.cross_kv_q8 ? 1 : 2;  // bytes per element of the store
            for (int l = 0; l < D.n_text_layer; ++l) {
                const size_t layer0 = (size_t)l * rows, sz = (size_t)T * d * qb;
                uint8_t* ck = s->ck.as<uint8_t>() + layer0 * d * qb;
                uint8_t* cv = s->cv.as<uint8_t>() + layer0 * d * qb;
                VKB_CUDA(cudaMemcpyAsync(ck + (size_t)dst * sz, ck + (size_t)src * sz, sz, cudaMemcpyDeviceToDevice,
                                         s->ctx->stream));
                VKB_CUDA(cudaMemcpyAsync(cv + (size_t)dst * sz, cv + (size_t)src * sz, sz, cudaMemcpyDeviceToDevice,
                                         s->ctx->stream));
                if (s->opt.cross_kv_q8) {
                    const size_t ssz = (size_t)T * (d / 32) * 2;
                    uint8_t* ks = s->cks.as<uint8_t>() + layer0 * (d / 32) * 2;
                    uint8_t* vs = s->cvs.as<uint8_t>() + layer0 * (d / 32) * 2;
                    VKB_CUDA(cudaMemcpyAsync(ks + (size_t)dst * ssz, ks + (size_t)src * ssz, ssz,
                                             cudaMemcpyDeviceToDevice, s->ctx->stream));
                    VKB_CUDA(cudaMemcpyAsync(vs + (size_t)dst * ssz, vs + (size_t)src * ssz, ssz,
                                             cudaMemcpyDeviceToDevice, s->ctx->stream));
                }
            }
        }
    });
}

vkb_status vkb_session_release(vkb_session* s, int32_t stream) {
    return guard([&] {
        if (!s) fail(VKB_ERROR_INVALID_ARGUMENT, "session_release: null session");
        vkb_kv_release_seq(s->pool, stream) == VKB_OK ? void() : fail(VKB_ERROR_INVALID_ARGUMENT, vkb_last_error());
    });
}

}  // extern "C"
