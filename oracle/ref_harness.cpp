// Test infrastructure only: a C-ABI harness around the reference engine's own
// CPU (AVX2 + OpenMP) path, compiled from the reference sources by
// oracle/Makefile into oracle/_ref/libxlref.so.  Only the tests, smoke() and
// bench.py's CPU-baseline / reference arm load it, as the checker or as the
// timed CPU baseline.  Nothing in the product links it.
//
// Every function drives a reference class on the "cpu" device:
//   Transformer            include/ops.h:174-201, src/transformer.cu:107-186
//   sample_cpu             src/inference.cu:69-114
//   Linear                 src/linear.cu:170-195, 284-307
//   RMSNorm                src/rmsnorm.cu:82-110
//   RoPE                   src/rope.cu:47-68, 108-128
//   MultiHeadAttention     src/attn.cu:201-239, 449-486
//   Embedding              src/embedding.cu:63-73, 156-171
//
// Objects holding an Embedding are never destroyed: Embedding::~Embedding
// calls cudaFree(nullptr) under CHECK_CUDA and exits the process on hosts
// without a GPU (src/embedding.cu:24-27).  Run processes that use this
// library with CUDA_VISIBLE_DEVICES="" so that the reference's Tensor
// constructor does not mirror every buffer on GPU 0 (src/tensor.cu:23-26).
#include <cstring>
#include <cstdint>
#include <random>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

#include "ops.h"
#include "tensor.h"

// Defined with external linkage in the reference's src/inference.cu.
int sample_cpu(float* logits, int n, float temperature, float top_p, float repetition_penalty,
               std::mt19937& gen, std::set<int>& repetition_set);

namespace {
struct RefModel {
    Transformer tr;
    int vocab;
    int hidden;
    int heads;
    int max_len;
    int layers;
    Tensor logits;
    RefModel(int max_len_, int hidden_, int heads_, float base, int ffn, int vocab_, int layers_)
        : tr(max_len_, hidden_, heads_, base, ffn, vocab_, layers_, "cpu"),
          vocab(vocab_), hidden(hidden_), heads(heads_), max_len(max_len_), layers(layers_),
          logits({vocab_}, "cpu") {}
};

void copy_in(Tensor& t, const float* src) { std::memcpy(t.h_ptr, src, sizeof(float) * t.size()); }
void copy_out(const Tensor& t, float* dst) { std::memcpy(dst, t.h_ptr, sizeof(float) * t.size()); }
}  // namespace

extern "C" {

void* xlref_model_create(int max_len, int hidden, int heads, float base, int ffn, int vocab, int layers) {
    return new RefModel(max_len, hidden, heads, base, ffn, vocab, layers);
}

int xlref_model_load(void* h, const char* dir) {
    try {
        static_cast<RefModel*>(h)->tr.load(dir);
    } catch (const std::exception&) {
        return -1;
    }
    return 0;
}

// Transformer::forward(vector) — prefill; resets every layer's KV counter to n.
int xlref_model_prefill(void* h, const int* ids, int n, float* logits_out) {
    RefModel* m = static_cast<RefModel*>(h);
    if (n <= 0 || n > m->max_len) return -2;
    for (int i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= m->vocab) return -3;
    std::vector<int> tokens(ids, ids + n);
    m->tr.forward(tokens, m->logits);
    copy_out(m->logits, logits_out);
    return 0;
}

// Transformer::forward(int) — one decode step; appends at KV.n then n++.
int xlref_model_decode(void* h, int id, float* logits_out) {
    RefModel* m = static_cast<RefModel*>(h);
    if (id < 0 || id >= m->vocab) return -3;
    if (m->tr.blocks_[0]->attn_.KV.n >= m->max_len) return -4;
    m->tr.forward(id, m->logits);
    copy_out(m->logits, logits_out);
    return 0;
}

int xlref_model_kv_n(void* h, int layer) {
    return static_cast<RefModel*>(h)->tr.blocks_[layer]->attn_.KV.n;
}

// Position-major [npos][heads][64] copies of one layer's cache.
void xlref_model_kv_copy(void* h, int layer, int npos, float* k_out, float* v_out) {
    RefModel* m = static_cast<RefModel*>(h);
    const KVcache& kv = m->tr.blocks_[layer]->attn_.KV;
    size_t count = static_cast<size_t>(npos) * m->hidden;
    std::memcpy(k_out, kv.K_.h_ptr, count * sizeof(float));
    std::memcpy(v_out, kv.V_.h_ptr, count * sizeof(float));
}

// sample_cpu with a std::mt19937 seeded by `seed` and the given repetition set.
// `logits` is modified in place exactly as the reference does.
int xlref_sample(float* logits, int n, float temperature, float top_p, float rp,
                 uint32_t seed, const int* rep, int nrep) {
    std::mt19937 gen(seed);
    std::set<int> rs(rep, rep + nrep);
    return sample_cpu(logits, n, temperature, top_p, rp, gen, rs);
}

// The uniform that sample_cpu draws first from std::mt19937(seed)
// (src/inference.cu:105).
float xlref_mt_uniform(uint32_t seed) {
    std::mt19937 gen(seed);
    return std::uniform_real_distribution<float>(0.0f, 1.0f)(gen);
}

// Linear::forward (N rows) or Linear::forward_vec (vec != 0, N must be 1).
void xlref_linear(const float* in, const float* w, const float* b, float* out, int n, int k, int mdim,
                  int vec) {
    Linear lin(k, mdim, "cpu");
    copy_in(lin.weight_, w);
    copy_in(lin.bias_, b);
    if (vec) {
        Tensor x({k}, "cpu"), y({mdim}, "cpu");
        copy_in(x, in);
        lin.forward_vec(x, y);
        copy_out(y, out);
    } else {
        Tensor x({n, k}, "cpu"), y({n, mdim}, "cpu");
        copy_in(x, in);
        lin.forward(x, y);
        copy_out(y, out);
    }
}

void xlref_rmsnorm(float* x, const float* gamma, int n, int k) {
    RMSNorm norm(k, "cpu");
    copy_in(norm.gamma_, gamma);
    Tensor t({n, k}, "cpu");
    copy_in(t, x);
    norm.forward(t);
    copy_out(t, x);
}

// RoPE::forward (pos = row index) when pos < 0, else RoPE::forward_vec at pos.
void xlref_rope(float* x, int n, int heads, int c, int pos, float base) {
    if (pos < 0) {
        Tensor t({n, heads, c}, "cpu");
        copy_in(t, x);
        RoPE::forward(t, base);
        copy_out(t, x);
    } else {
        Tensor t({heads, c}, "cpu");
        copy_in(t, x);
        RoPE::forward_vec(t, pos, base);
        copy_out(t, x);
    }
}

// MultiHeadAttention::prefill over [n][heads][c]; fills kv_k/kv_v ([max_len][heads][c]).
void xlref_attn_prefill(const float* q, const float* k, const float* v, float* out, float* kv_k,
                        float* kv_v, int n, int heads, int c, int max_len) {
    Tensor Q({n, heads, c}, "cpu"), K({n, heads, c}, "cpu"), V({n, heads, c}, "cpu"),
        O({n, heads, c}, "cpu");
    copy_in(Q, q);
    copy_in(K, k);
    copy_in(V, v);
    KVcache kv(max_len, c, heads, "cpu");
    MultiHeadAttention::prefill(Q, K, V, O, kv);
    copy_out(O, out);
    copy_out(kv.K_, kv_k);
    copy_out(kv.V_, kv_v);
}

// MultiHeadAttention::forward: appends q/k/v ([heads][c]) at position n of the
// given cache (in/out, [max_len][heads][c]) and attends over 0..n.
void xlref_attn_decode(const float* q, const float* k, const float* v, float* out, float* kv_k,
                       float* kv_v, int n, int heads, int c, int max_len) {
    Tensor Q({heads, c}, "cpu"), K({heads, c}, "cpu"), V({heads, c}, "cpu"), O({heads, c}, "cpu");
    copy_in(Q, q);
    copy_in(K, k);
    copy_in(V, v);
    KVcache kv(max_len, c, heads, "cpu");
    copy_in(kv.K_, kv_k);
    copy_in(kv.V_, kv_v);
    kv.n = n;
    MultiHeadAttention::forward(Q, K, V, O, kv);
    copy_out(O, out);
    copy_out(kv.K_, kv_k);
    copy_out(kv.V_, kv_v);
}

// Embedding::forward (row gather) and Embedding::inverse (tied LM head).
// The Embedding object is intentionally leaked (see the file header).
void xlref_embedding(const float* table, int vocab, int k, const int* ids, int n, float* rows_out,
                     const float* h, float* logits_out) {
    Embedding* emb = new Embedding(vocab, k, "cpu");
    copy_in(emb->weight_, table);
    if (n > 0) {
        std::vector<int> tokens(ids, ids + n);
        Tensor out({n, k}, "cpu");
        emb->forward(tokens, out);
        copy_out(out, rows_out);
    }
    if (h != nullptr) {
        Tensor x({k}, "cpu"), y({vocab}, "cpu");
        copy_in(x, h);
        emb->inverse(x, y);
        copy_out(y, logits_out);
    }
}

// SwishGLU::forward on [n][in_dim] (in place), the reference FFN.
void xlref_swiglu(float* x, const float* w1, const float* b1, const float* v, const float* bv,
                  const float* w2, const float* b2, int n, int in_dim, int hidden) {
    SwishGLU ffn(in_dim, hidden, "cpu");
    copy_in(ffn.W1_.weight_, w1);
    copy_in(ffn.W1_.bias_, b1);
    copy_in(ffn.V_.weight_, v);
    copy_in(ffn.V_.bias_, bv);
    copy_in(ffn.W2_.weight_, w2);
    copy_in(ffn.W2_.bias_, b2);
    Tensor t({n, in_dim}, "cpu");
    copy_in(t, x);
    if (n == 1) {
        Tensor tv({in_dim}, "cpu");
        copy_in(tv, x);
        ffn.forward_vec(tv);
        copy_out(tv, x);
    } else {
        ffn.forward(t);
        copy_out(t, x);
    }
}

}  // extern "C"
