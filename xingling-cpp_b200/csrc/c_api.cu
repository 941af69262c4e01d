// extern "C" surface of libxl_engine.so (declared in include/xl_engine.h).
#include <nccl.h>

#include <cstring>
#include <string>
#include <vector>

#include "engine.h"

using xl::Engine;

struct xl_engine {
    Engine* impl;
};
struct xl_batch {
    xl::BatchDecoder* impl;
};

namespace {

int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return XL_OK;
    xl::set_error(std::string("CUDA error in ") + what + ": " + cudaGetErrorString(e));
    return XL_ERR_CUDA;
}

int bad(const char* msg) {
    xl::set_error(msg);
    return XL_ERR_ARG;
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// Op-level workspaces that carry a DevState.
struct OpState {
    xl::DevState st;
};

}  // namespace

extern "C" {

const char* xl_last_error(void) { return xl::last_error(); }

void xl_config_default(xl_config* cfg) {
    if (!cfg) return;
    cfg->layers = 16;
    cfg->hidden = 1536;
    cfg->heads = 24;
    cfg->ffn = 4096;
    cfg->vocab = 151669;
    cfg->max_ctx = 768;
    cfg->rope_base = 10000.0f;
}

int xl_nccl_unique_id(void* out, int nbytes) {
    if (!out || nbytes < static_cast<int>(sizeof(ncclUniqueId))) return bad("xl_nccl_unique_id: buffer too small");
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) {
        xl::set_error(std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
        return XL_ERR_NCCL;
    }
    std::memcpy(out, &id, sizeof(id));
    return XL_OK;
}

int xl_engine_create(const xl_config* cfg, int device, int tp_size, int tp_rank, const void* nccl_id,
                     xl_engine** out) {
    xl::clear_error();
    if (!cfg || !out) return bad("xl_engine_create: null argument");
    *out = nullptr;
    Engine* impl = nullptr;
    const int rc = Engine::create(*cfg, device, tp_size, tp_rank, nccl_id, &impl);
    if (rc != XL_OK) return rc;
    *out = new xl_engine{impl};
    return XL_OK;
}

int xl_batch_create(xl_engine* e, xl_batch** out) {
    xl::clear_error();
    if (!e || !out) return bad("null argument");
    static_assert(XL_BATCH == xl::kBatch, "batch size of the ABI");
    xl::BatchDecoder* b = nullptr;
    const int rc = xl::BatchDecoder::create(e->impl, &b);
    if (rc != XL_OK) return rc;
    *out = new xl_batch{b};
    return XL_OK;
}

void xl_batch_destroy(xl_batch* b) {
    if (!b) return;
    delete b->impl;
    delete b;
}

int xl_batch_seed(xl_batch* b, int seq, unsigned long long seed) {
    xl::clear_error();
    if (!b) return bad("null batch decoder");
    return b->impl->seed(seq, seed);
}

int xl_batch_prefill(xl_batch* b, int seq, const int* ids, int n, float temperature, float top_p,
                     float repetition_penalty, int* token_out) {
    xl::clear_error();
    if (!b || !token_out) return bad("null argument");
    return b->impl->prefill(seq, ids, n, temperature, top_p, repetition_penalty, token_out);
}

int xl_batch_decode(xl_batch* b, const int* tokens, float temperature, float top_p, float repetition_penalty,
                    int* tokens_out) {
    xl::clear_error();
    if (!b) return bad("null batch decoder");
    return b->impl->decode(tokens, temperature, top_p, repetition_penalty, tokens_out);
}

int xl_batch_last_logits(xl_batch* b, int seq, float* out, int n) {
    xl::clear_error();
    if (!b) return bad("null batch decoder");
    return b->impl->last_logits(seq, out, n);
}

int xl_batch_ctx_len(const xl_batch* b, int seq) { return b ? b->impl->ctx_len(seq) : -1; }

int xl_batch_last_device_ms(const xl_batch* b, float* ms) {
    if (!b || !ms) return bad("null argument");
    *ms = b->impl->last_device_ms();
    return XL_OK;
}

void xl_engine_destroy(xl_engine* e) {
    if (!e) return;
    delete e->impl;
    delete e;
}

int xl_engine_load(xl_engine* e, const char* dir) {
    xl::clear_error();
    if (!e) return bad("null engine");
    return e->impl->load(dir);
}

int xl_engine_prefill(xl_engine* e, const int* ids, int n, float temperature, float top_p, float repetition_penalty,
                      int* token_out) {
    xl::clear_error();
    if (!e || !token_out) return bad("null argument");
    return e->impl->prefill(ids, n, temperature, top_p, repetition_penalty, token_out);
}

int xl_engine_decode(xl_engine* e, int token, float temperature, float top_p, float repetition_penalty,
                     int* token_out) {
    xl::clear_error();
    if (!e || !token_out) return bad("null argument");
    return e->impl->decode(token, temperature, top_p, repetition_penalty, token_out);
}

int xl_engine_extend(xl_engine* e, const int* ids, int n, float temperature, float top_p, float repetition_penalty,
                     int* token_out) {
    xl::clear_error();
    if (!e || !token_out) return bad("null argument");
    return e->impl->prefill(ids, n, temperature, top_p, repetition_penalty, token_out, true);
}

int xl_engine_generate(xl_engine* e, int token, int n, float temperature, float top_p, float repetition_penalty,
                       int stop_id, int* tokens_out, int* n_out) {
    xl::clear_error();
    if (!e || !n_out) return bad("null argument");
    return e->impl->generate(token, n, temperature, top_p, repetition_penalty, stop_id, tokens_out, n_out);
}

int xl_engine_set_uniforms(xl_engine* e, const float* u, int n) {
    xl::clear_error();
    if (!e) return bad("null engine");
    return e->impl->set_uniforms(u, n);
}

int xl_engine_seed(xl_engine* e, uint64_t seed) {
    xl::clear_error();
    if (!e) return bad("null engine");
    return e->impl->seed(seed);
}

int xl_engine_last_logits(xl_engine* e, float* out, int n) {
    xl::clear_error();
    if (!e) return bad("null engine");
    return e->impl->last_logits(out, n);
}

int xl_engine_vocab_shard(const xl_engine* e, int* begin, int* count) {
    if (!e || !begin || !count) return bad("null argument");
    *begin = e->impl->vocab_begin();
    *count = e->impl->vocab_count();
    return XL_OK;
}

int xl_engine_ctx_len(const xl_engine* e) { return e ? e->impl->ctx_len() : -1; }

int xl_engine_kv_copy(xl_engine* e, int layer, int npos, float* k_out, float* v_out) {
    xl::clear_error();
    if (!e || !k_out || !v_out) return bad("null argument");
    return e->impl->kv_copy(layer, npos, k_out, v_out);
}

int xl_engine_last_device_ms(const xl_engine* e, float* ms) {
    if (!e || !ms) return bad("null argument");
    *ms = e->impl->last_device_ms();
    return XL_OK;
}

int xl_engine_last_kernel_ms(const xl_engine* e, float* ms) {
    if (!e || !ms) return bad("null argument");
    *ms = e->impl->last_kernel_ms();
    return XL_OK;
}

int xl_engine_last_load_s(const xl_engine* e, float* s) {
    if (!e || !s) return bad("null argument");
    *s = e->impl->last_load_s();
    return XL_OK;
}

long long xl_kernel_launches(void) { return xl::launch_count(); }

int xl_engine_set_option(xl_engine* e, const char* key, int value) {
    xl::clear_error();
    if (!e) return bad("null engine");
    return e->impl->set_option(key, value);
}

int xl_engine_phase_trace(xl_engine* e, unsigned long long* out, int n) {
    xl::clear_error();
    if (!e) return bad("null engine");
    return e->impl->phase_trace(out, n);
}

int xl_philox_uniforms(uint64_t seed, uint64_t start, int n, float* out) {
    if (n < 0 || (n > 0 && !out)) return bad("xl_philox_uniforms: bad arguments");
    for (int i = 0; i < n; ++i) out[i] = xl::philox_uniform(start + static_cast<uint64_t>(i), seed);
    return XL_OK;
}

int xl_tp_plan(const xl_config* cfg, int tp, int rank, int* out) {
    xl::clear_error();
    if (!cfg || !out) return bad("xl_tp_plan: null argument");
    xl::TpPlan p;
    const int rc = xl::make_tp_plan(*cfg, tp, rank, &p);
    if (rc != XL_OK) return rc;
    out[0] = p.heads;
    out[1] = p.hidden;
    out[2] = p.ffn;
    out[3] = p.vocab_begin;
    out[4] = p.vocab_count;
    return XL_OK;
}

int xl_engine_profile_lm_head(xl_engine* e, int iters, float* avg_ms) {
    xl::clear_error();
    if (!e) return bad("null engine");
    return e->impl->profile_lm_head(iters, avg_ms);
}

// ---------------------------------------------------------------------------
int xl_op_norm_gemv(int mode, const float* x, const float* gamma, const float* w, const float* b, float* y, int m,
                    int k, void* stream) {
    xl::clear_error();
    if (!x || !w || !y || m <= 0 || k <= 0 || k % 4) return bad("xl_op_norm_gemv: bad arguments");
    if (mode != xl::kGemvPlain && mode != xl::kGemvSwiGLU && mode != xl::kGemvResidual)
        return bad("xl_op_norm_gemv: mode must be 0, 1 or 2");
    if (mode == xl::kGemvSwiGLU && (m % 2 || !b)) return bad("xl_op_norm_gemv: SwiGLU needs even m and a bias");
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    xl::NormGemvParams p{};
    p.x = x;
    p.gamma = gamma;
    p.eps = 1e-6;
    p.W = w;
    p.bias = b;
    p.y = y;
    p.M = m;
    p.K = k;
    return cuda_status(xl::launch_norm_gemv(mode, p, sms, false, as_stream(stream)), "xl_op_norm_gemv");
}

int xl_rope_table(float base, int max_ctx, float* out) {
    if (!out || max_ctx <= 0) return bad("xl_rope_table: bad arguments");
    xl::fill_rope_table(base, max_ctx, out);
    return XL_OK;
}

size_t xl_op_attn_decode_workspace_bytes(int heads, int max_ctx) {
    const size_t part = static_cast<size_t>(heads) * xl::attn_max_splits(max_ctx) * (xl::kHeadDim + 2) * 4;
    return (part + 255) / 256 * 256 + static_cast<size_t>(heads) * 4;
}

int xl_op_attn_decode(const float* qkv, const float* rope, float* kc, float* vc, float* out, const int* pos, int heads,
                      int max_ctx, void* workspace, void* stream) {
    xl::clear_error();
    if (!qkv || !rope || !kc || !vc || !out || !pos || !workspace || heads <= 0 || max_ctx <= 0)
        return bad("xl_op_attn_decode: bad arguments");
    const size_t part = static_cast<size_t>(heads) * xl::attn_max_splits(max_ctx) * (xl::kHeadDim + 2) * 4;
    xl::AttnDecodeParams a{};
    a.qkv = qkv;
    a.rope = reinterpret_cast<const float2*>(rope);
    a.kc = kc;
    a.vc = vc;
    a.out = out;
    a.part = static_cast<float*>(workspace);
    a.counters = reinterpret_cast<int*>(static_cast<char*>(workspace) + (part + 255) / 256 * 256);
    a.pos = pos;
    a.heads = heads;
    a.max_ctx = max_ctx;
    return cuda_status(xl::launch_attn_decode(a, false, as_stream(stream)), "xl_op_attn_decode");
}

size_t xl_op_lm_head_workspace_bytes(void) { return sizeof(OpState); }

int xl_op_lm_head(const float* x, const float* gamma, const float* table, float* logits, const uint8_t* rep_flags,
                  float repetition_penalty, int vocab, int k, int* argmax_out, void* workspace, void* stream) {
    xl::clear_error();
    if (!x || !table || !logits || !rep_flags || !workspace || vocab <= 0 || k <= 0 || k % 4)
        return bad("xl_op_lm_head: bad arguments");
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaStream_t s = as_stream(stream);
    xl::DevState* st = static_cast<xl::DevState*>(workspace);
    xl::DevState hs{};
    hs.in.rp = repetition_penalty;
    int rc = cuda_status(cudaMemcpyAsync(st, &hs, sizeof(hs), cudaMemcpyHostToDevice, s), "xl_op_lm_head copy");
    if (rc != XL_OK) return rc;
    xl::NormGemvParams p{};
    p.x = x;
    p.gamma = gamma;
    p.eps = 1e-6;
    p.W = table;
    p.y = logits;
    p.M = vocab;
    p.K = k;
    p.rep_flags = rep_flags;
    p.st = st;
    p.row_offset = 0;
    rc = cuda_status(xl::launch_norm_gemv(xl::kGemvLogits, p, sms, false, s), "xl_op_lm_head");
    if (rc != XL_OK) return rc;
    if (argmax_out) {
        rc = cuda_status(cudaMemcpyAsync(&hs, st, sizeof(hs), cudaMemcpyDeviceToHost, s), "xl_op_lm_head copy");
        if (rc != XL_OK) return rc;
        rc = cuda_status(cudaStreamSynchronize(s), "xl_op_lm_head sync");
        if (rc != XL_OK) return rc;
        *argmax_out = hs.greedy_token;
    }
    return XL_OK;
}

namespace {
// The sampler chain of xl_op_sample runs on as many vocab slices as a B200 has SMs.
constexpr int kOpSampleSms = 148;
size_t op_flags_bytes(int vocab) { return (static_cast<size_t>(vocab) + 255) / 256 * 256; }
}  // namespace

size_t xl_op_sample_workspace_bytes(int vocab) {
    if (vocab <= 0) return 0;
    return (sizeof(OpState) + 255) / 256 * 256 + op_flags_bytes(vocab) +
           xl::sample_work_bytes(vocab, xl::sample_grid(vocab, kOpSampleSms, 1));
}

int xl_op_sample(const float* logits, int vocab, float temperature, float top_p, float r, int* token_out,
                 void* workspace, void* stream) {
    xl::clear_error();
    if (!logits || vocab <= 0 || !token_out || !workspace) return bad("xl_op_sample: bad arguments");
    cudaStream_t s = as_stream(stream);
    xl::DevState* st = static_cast<xl::DevState*>(workspace);
    uint8_t* flags = static_cast<uint8_t*>(workspace) + (sizeof(OpState) + 255) / 256 * 256;
    void* work = flags + op_flags_bytes(vocab);
    const int grid = xl::sample_grid(vocab, kOpSampleSms, 1);
    xl::DevState hs{};
    hs.in.temperature = temperature;
    hs.in.top_p = top_p;
    hs.in.rp = 1.0f;
    hs.in.uniform = r;
    int rc = cuda_status(cudaMemcpyAsync(st, &hs, sizeof(hs), cudaMemcpyHostToDevice, s), "xl_op_sample copy");
    if (rc != XL_OK) return rc;
    // The chain leaves its work area zeroed; clearing it here also covers a workspace never used before.
    rc = cuda_status(cudaMemsetAsync(work, 0, xl::sample_work_bytes(vocab, grid), s), "xl_op_sample clear");
    if (rc != XL_OK) return rc;
    xl::SampleParams sp{};
    sp.logits = logits;
    sp.V = vocab;
    sp.v0 = 0;
    sp.st = st;
    sp.rep_flags = flags;
    sp.full = 1;
    sp.work = work;
    sp.work_stride = xl::sample_work_bytes(vocab, grid);
    sp.stride = vocab;
    sp.grid = grid;
    rc = cuda_status(xl::launch_sample_chain(sp, 1, false, s), "xl_op_sample");
    if (rc != XL_OK) return rc;
    rc = cuda_status(cudaMemcpyAsync(&hs, st, sizeof(hs), cudaMemcpyDeviceToHost, s), "xl_op_sample copy");
    if (rc != XL_OK) return rc;
    rc = cuda_status(cudaStreamSynchronize(s), "xl_op_sample sync");
    if (rc != XL_OK) return rc;
    if (hs.err != 0) {
        xl::set_error("xl_op_sample: device error word " + std::to_string(hs.err));
        return XL_ERR_DEVICE;
    }
    *token_out = hs.token_out;
    return XL_OK;
}

int xl_op_linear(int mode, const float* x, const float* x_lo, const float* w, const float* w_lo, const float* b,
                 float* y, float* y_lo, int n, int m, int k, void* stream) {
    xl::clear_error();
    if (!x || !w || !y || n <= 0 || m <= 0 || k <= 0 || k % 8) return bad("xl_op_linear: bad arguments");
    if (mode != xl::kGemvPlain && mode != xl::kGemvSwiGLU && mode != xl::kGemvResidual)
        return bad("xl_op_linear: mode must be 0, 1 or 2");
    if (mode == xl::kGemvSwiGLU && (m % 2 || !b)) return bad("xl_op_linear: SwiGLU needs even m and a bias");
    cudaStream_t s = as_stream(stream);
    if (!x_lo || !w_lo)
        return cuda_status(xl::launch_linear_prefill(mode, x, w, b, y, n, m, k, s), "xl_op_linear");
    if (k % 32) return bad("xl_op_linear: the tensor-core path needs k % 32 == 0");
    if (mode == xl::kGemvSwiGLU && !y_lo) return bad("xl_op_linear: the tensor-core SwiGLU path writes y_lo");
    xl::TcOperands o;
    int rc = cuda_status(xl::make_tile_map(&o.w, w, m, k), "make_tile_map");
    if (rc == XL_OK) rc = cuda_status(xl::make_tile_map(&o.w_lo, w_lo, m, k), "make_tile_map");
    if (rc == XL_OK) rc = cuda_status(xl::make_tile_map(&o.x, x, n, k), "make_tile_map");
    if (rc == XL_OK) rc = cuda_status(xl::make_tile_map(&o.x_lo, x_lo, n, k), "make_tile_map");
    if (rc != XL_OK) return rc;
    return cuda_status(xl::launch_gemm_tc(mode, o, b, y, y_lo, n, m, k, nullptr, s), "xl_op_linear (tcgen05)");
}

int xl_op_split_lo(const float* x, float* lo, size_t n, void* stream) {
    xl::clear_error();
    if (!x || !lo) return bad("xl_op_split_lo: null pointer");
    return cuda_status(xl::launch_split_lo(x, lo, n, as_stream(stream)), "xl_op_split_lo");
}

int xl_op_rmsnorm(const float* x, const float* gamma, float* out, int n, int k, void* stream) {
    xl::clear_error();
    if (!x || !gamma || !out || n <= 0 || k <= 0 || k % 4) return bad("xl_op_rmsnorm: bad arguments");
    return cuda_status(xl::launch_rmsnorm_rows(x, gamma, out, nullptr, n, k, as_stream(stream)), "xl_op_rmsnorm");
}

int xl_op_embedding(const float* table, const int* ids, float* out, int n, int k, void* stream) {
    xl::clear_error();
    if (!table || !ids || !out || n <= 0 || k <= 0 || k % 4) return bad("xl_op_embedding: bad arguments");
    return cuda_status(xl::launch_embed_gather(table, ids, out, n, k, as_stream(stream)), "xl_op_embedding");
}

int xl_op_attn_prefill(float* qkv, const float* rope, float* kc, float* vc, float* out, int n, int heads, int max_ctx,
                       void* stream) {
    xl::clear_error();
    if (!qkv || !rope || !kc || !vc || !out || n <= 0 || n > max_ctx || heads <= 0)
        return bad("xl_op_attn_prefill: bad arguments");
    cudaStream_t s = as_stream(stream);
    const float2* r2 = reinterpret_cast<const float2*>(rope);
    int rc = cuda_status(xl::launch_rope_kv_prefill(qkv, r2, kc, vc, n, heads, max_ctx, s), "rope_kv_prefill");
    if (rc != XL_OK) return rc;
    return cuda_status(xl::launch_attn_prefill(qkv, kc, vc, out, nullptr, n, heads, max_ctx, s), "attn_prefill");
}

}  // extern "C"
