/*
 * Test infrastructure only: the CPU oracle for the XingLing token loop.
 *
 * A plain-C restatement of the reference engine's fp32 CPU path
 * (fancyovo/XingLing-cpp), used by the tests, smoke() and bench.py's CPU
 * baseline as the checker.  The product never links or calls it.  Each
 * function cites the reference file:line it restates.  Accumulations follow
 * the reference's 8-lane AVX2 FMA pattern (lane partial sums, then a
 * sequential float sum of the 8 lanes) so that results agree with the
 * reference to a few ulps; the pin against the reference build itself
 * (oracle/_ref) is in tests/test_oracle_pin.py and tests/golden/.
 *
 * Layouts follow the reference: Linear weight [out][in] row-major
 * (include/ops.h:9-25), KV cache position-major [max_len][heads][64]
 * (src/attn.cu:11-16), embedding [vocab][hidden] (src/embedding.cu:13-17).
 */
#include <errno.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* Dot product with the reference's 8-lane FMA pattern:
 * src/linear.cu:180-192 (and attn.cu __scale_dot, rmsnorm.cu:80-90).   */
static float dot8(const float* a, const float* b, int n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int k = 0;
    for (; k + 8 <= n; k += 8)
        for (int l = 0; l < 8; ++l) acc[l] = fmaf(a[k + l], b[k + l], acc[l]);
    float s = 0.0f;
    for (int l = 0; l < 8; ++l) s += acc[l];
    for (; k < n; ++k) s = fmaf(a[k], b[k], s);
    return s;
}

/* Linear::forward / forward_vec CPU path, src/linear.cu:170-195 and 284-307:
 * out[i][j] = bias[j] + sum_k in[i][k] * W[j][k].                          */
void xlo_linear(const float* in, const float* w, const float* b, float* out, int n, int k, int m) {
#pragma omp parallel for schedule(static)
    for (int j = 0; j < m; ++j)
        for (int i = 0; i < n; ++i) out[(size_t)i * m + j] = b[j] + dot8(in + (size_t)i * k, w + (size_t)j * k, k);
}

/* RMSNorm CPU path, src/rmsnorm.cu:82-110 (in place):
 * x * (1 / sqrt(mean(x^2) + 1e-6)) * gamma, sqrt and reciprocal in double.  */
void xlo_rmsnorm(float* x, const float* gamma, int n, int k) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) {
        float* row = x + (size_t)i * k;
        float sum = dot8(row, row, k);
        float sqrt_mean = (float)sqrt((double)(sum / k) + 1e-6);
        float inv = (float)(1.0 / sqrt_mean);
        for (int j = 0; j < k; ++j) row[j] = row[j] * inv * gamma[j];
    }
}

/* RoPE CPU path, src/rope.cu:47-68 (prefill, position = start + row) and
 * src/rope.cu:108-128 (decode).  Rotate-half pairs (j, j + c/2):
 * o0 = x0 cos + x1 sin, o1 = -x0 sin + x1 cos, theta = base^(-2j/c) * pos.  */
void xlo_rope(float* x, int n, int heads, int c, int start_pos, float base) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) {
        float pos = (float)(start_pos + i);
        for (int h = 0; h < heads; ++h) {
            float* v = x + ((size_t)i * heads + h) * c;
            for (int j = 0; j < c / 2; ++j) {
                float theta = powf(base, -2.0f * j / c) * pos;
                float cp = cosf(theta), sp = sinf(theta);
                float i0 = v[j], i1 = v[j + c / 2];
                v[j] = i0 * cp + i1 * sp;
                v[j + c / 2] = -i0 * sp + i1 * cp;
            }
        }
    }
}

/* __scale_add of src/attn.cu:186-198: a = a * m + k * b (fma).              */
static void scale_add(float* a, const float* b, float m, float k, int n) {
    for (int j = 0; j < n; ++j) a[j] = fmaf(k, b[j], a[j] * m);
}

/* One query's online softmax over cache rows 0..last (inclusive), the loop
 * body shared by src/attn.cu:210-235 (prefill) and :466-483 (decode).       */
static void attend_one(const float* q, const float* kc, const float* vc, float* out, int last,
                       int stride, int c) {
    float inv_sqrt_c = (float)(1.0f / sqrt((double)c));
    float max_val = -1e6f, sum_exp = 0.0f;
    memset(out, 0, sizeof(float) * c);
    for (int t = 0; t <= last; ++t) {
        const float* kr = kc + (size_t)t * stride;
        const float* vr = vc + (size_t)t * stride;
        float d = dot8(q, kr, c) * inv_sqrt_c;
        if (d > max_val) {
            float s = expf(max_val - d);
            scale_add(out, vr, s, 1.0f, c);
            max_val = d;
            sum_exp = sum_exp * s + 1.0f;
        } else {
            float e = expf(d - max_val);
            sum_exp += e;
            scale_add(out, vr, 1.0f, e, c);
        }
    }
    float inv = 1.0f / sum_exp;
    for (int j = 0; j < c; ++j) out[j] = out[j] * inv;
}

/* MultiHeadAttention::prefill CPU path, src/attn.cu:201-239 and :319-365:
 * causal attention over q/k/v [n][heads][c]; copies k/v to the cache rows
 * 0..n-1 ([max_len][heads][c]).  The caller sets the cache counter to n.    */
void xlo_attn_prefill(const float* q, const float* k, const float* v, float* out, float* kv_k,
                      float* kv_v, int n, int heads, int c) {
    int stride = heads * c;
    memcpy(kv_k, k, sizeof(float) * (size_t)n * stride);
    memcpy(kv_v, v, sizeof(float) * (size_t)n * stride);
#pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < heads; ++h)
        for (int t = 0; t < n; ++t)
            attend_one(q + (size_t)t * stride + h * c, kv_k + h * c, kv_v + h * c,
                       out + (size_t)t * stride + h * c, t, stride, c);
}

/* MultiHeadAttention::forward CPU path, src/attn.cu:449-486 and :490-547:
 * appends k/v ([heads][c]) at position pos, attends over 0..pos.  The caller
 * increments the counter.                                                    */
void xlo_attn_decode(const float* q, const float* k, const float* v, float* out, float* kv_k,
                     float* kv_v, int pos, int heads, int c) {
    int stride = heads * c;
    memcpy(kv_k + (size_t)pos * stride, k, sizeof(float) * stride);
    memcpy(kv_v + (size_t)pos * stride, v, sizeof(float) * stride);
#pragma omp parallel for schedule(static)
    for (int h = 0; h < heads; ++h)
        attend_one(q + h * c, kv_k + h * c, kv_v + h * c, out + h * c, pos, stride, c);
}

/* silu(a) * b, src/ffn.cu:67-69 and :78-88 (in place on a).                 */
void xlo_silu_mul(float* a, const float* b, size_t n) {
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; ++i) a[i] = a[i] / (1.0f + expf(-a[i])) * b[i];
}

/* Embedding::forward, src/embedding.cu:63-73 (row gather).                  */
void xlo_embedding(const float* table, int k, const int* ids, int n, float* out) {
    for (int i = 0; i < n; ++i) memcpy(out + (size_t)i * k, table + (size_t)ids[i] * k, sizeof(float) * k);
}

/* Embedding::inverse, src/embedding.cu:156-171: logits[v] = E[v] . h        */
void xlo_lm_head(const float* table, const float* h, float* logits, int vocab, int k) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < vocab; ++r) {
        const float* row = table + (size_t)r * k;
        float d = 0.0f;
        for (int j = 0; j < k; ++j) d += h[j] * row[j];
        logits[r] = d;
    }
}

/* ------------------------------------------------------------------ */
/* sample_cpu, src/inference.cu:58-114, with the uniform r supplied.
 * (1) repetition penalty on the ids in rep[] (in place on logits),
 * (2) top 1024 by value, descending (ties: lower index first; the
 *     reference's nth_element + sort leaves tie order unspecified),
 * (3) v / (T + 0.001) and a sequential online max / sum of exp,
 * (4) smallest prefix whose float cumsum >= top_p,
 * (5) first i whose cumsum > r * total, else the 1024th.                    */
typedef struct {
    int idx;
    float val;
} xlo_cand;

static int cand_cmp(const void* a, const void* b) {
    const xlo_cand* x = (const xlo_cand*)a;
    const xlo_cand* y = (const xlo_cand*)b;
    if (x->val > y->val) return -1;
    if (x->val < y->val) return 1;
    return (x->idx > y->idx) - (x->idx < y->idx);
}

#define XLO_TOPK 1024

int xlo_sample(float* logits, int n, float temperature, float top_p, float rp, const int* rep,
               int nrep, float r) {
    for (int i = 0; i < nrep; ++i) {
        int x = rep[i];
        if (logits[x] > 0) logits[x] /= rp;
        else logits[x] *= rp;
    }
    xlo_cand* p = (xlo_cand*)malloc(sizeof(xlo_cand) * (size_t)n);
    if (!p) return -1;
    for (int i = 0; i < n; ++i) {
        p[i].idx = i;
        p[i].val = logits[i];
    }
    qsort(p, (size_t)n, sizeof(xlo_cand), cand_cmp);
    int k = n < XLO_TOPK ? n : XLO_TOPK;
    float max_val = -1e6f, sum_exp = 0.0f;
    for (int i = 0; i < k; ++i) {
        float val = p[i].val / (temperature + 0.001f);
        p[i].val = val;
        if (val > max_val) {
            sum_exp = sum_exp * expf(max_val - val) + 1.0f;
            max_val = val;
        } else {
            sum_exp += expf(val - max_val);
        }
    }
    float total = 0.0f;
    for (int i = 0; i < k; ++i) {
        total += expf(p[i].val - max_val) / sum_exp;
        if (total >= top_p) break;
    }
    float acc = 0.0f;
    int tok = p[k - 1].idx;
    for (int i = 0; i < k; ++i) {
        acc += expf(p[i].val - max_val) / sum_exp;
        if (acc > r * total) {
            tok = p[i].idx;
            break;
        }
    }
    free(p);
    return tok;
}

/* ------------------------------------------------------------------ */
/* The model: Transformer / TransformerBlock / AttentionBlock / SwishGLU,
 * src/transformer.cu:68-105 and :163-186, src/attn.cu:622-665,
 * src/ffn.cu:92-139.                                                        */
typedef struct {
    float *wq, *bq, *wk, *bk, *wv, *bv, *wo, *bo;
    float *w1, *b1, *wvf, *bvf, *w2, *b2;
    float *g1, *g2;
    float *kv_k, *kv_v; /* [max_len][heads][64] */
} xlo_layer;

typedef struct {
    int layers, hidden, heads, ffn, vocab, max_len;
    float base;
    float *emb, *gnorm;
    xlo_layer* L;
    int n; /* positions in the cache (KV.n, identical in every layer) */
    /* work buffers sized for max_len rows */
    float *x, *res, *q, *k, *v, *att, *h1, *h2, *last;
} xlo_model;

static float* xlo_alloc(size_t count) { return (float*)calloc(count, sizeof(float)); }

xlo_model* xlo_model_create(int layers, int hidden, int heads, int ffn, int vocab, int max_len, float base) {
    xlo_model* m = (xlo_model*)calloc(1, sizeof(xlo_model));
    m->layers = layers;
    m->hidden = hidden;
    m->heads = heads;
    m->ffn = ffn;
    m->vocab = vocab;
    m->max_len = max_len;
    m->base = base;
    size_t H = hidden, F = ffn, T = max_len;
    m->emb = xlo_alloc((size_t)vocab * H);
    m->gnorm = xlo_alloc(H);
    m->L = (xlo_layer*)calloc(layers, sizeof(xlo_layer));
    for (int l = 0; l < layers; ++l) {
        xlo_layer* y = &m->L[l];
        y->wq = xlo_alloc(H * H); y->bq = xlo_alloc(H);
        y->wk = xlo_alloc(H * H); y->bk = xlo_alloc(H);
        y->wv = xlo_alloc(H * H); y->bv = xlo_alloc(H);
        y->wo = xlo_alloc(H * H); y->bo = xlo_alloc(H);
        y->w1 = xlo_alloc(F * H); y->b1 = xlo_alloc(F);
        y->wvf = xlo_alloc(F * H); y->bvf = xlo_alloc(F);
        y->w2 = xlo_alloc(H * F); y->b2 = xlo_alloc(H);
        y->g1 = xlo_alloc(H); y->g2 = xlo_alloc(H);
        y->kv_k = xlo_alloc(T * H); y->kv_v = xlo_alloc(T * H);
    }
    m->x = xlo_alloc(T * H); m->res = xlo_alloc(T * H);
    m->q = xlo_alloc(T * H); m->k = xlo_alloc(T * H); m->v = xlo_alloc(T * H);
    m->att = xlo_alloc(T * H);
    m->h1 = xlo_alloc(T * F); m->h2 = xlo_alloc(T * F);
    m->last = xlo_alloc(H);
    return m;
}

void xlo_model_free(xlo_model* m) {
    if (!m) return;
    for (int l = 0; l < m->layers; ++l) {
        xlo_layer* y = &m->L[l];
        float* ps[] = {y->wq, y->bq, y->wk, y->bk, y->wv, y->bv, y->wo, y->bo, y->w1, y->b1, y->wvf,
                       y->bvf, y->w2, y->b2, y->g1, y->g2, y->kv_k, y->kv_v};
        for (size_t i = 0; i < sizeof(ps) / sizeof(ps[0]); ++i) free(ps[i]);
    }
    free(m->L);
    float* ps[] = {m->emb, m->gnorm, m->x, m->res, m->q, m->k, m->v, m->att, m->h1, m->h2, m->last};
    for (size_t i = 0; i < sizeof(ps) / sizeof(ps[0]); ++i) free(ps[i]);
    free(m);
}

/* Tensor::load, src/tensor.cu:113-126: raw little-endian fp32, exactly
 * count floats must be readable (a short file is an error).                */
static int read_raw(const char* dir, const char* rel, float* dst, size_t count) {
    char path[4096];
    snprintf(path, sizeof(path), "%s/%s", dir, rel);
    FILE* f = fopen(path, "rb");
    if (!f) return -1;
    size_t got = fread(dst, sizeof(float), count, f);
    fclose(f);
    return got == count ? 0 : -2;
}

/* The weight tree of src/transformer.cu:139-146, :32-37, src/attn.cu:572-577,
 * src/ffn.cu:27-31, src/linear.cu:68-72.                                    */
int xlo_model_load(xlo_model* m, const char* dir) {
    size_t H = m->hidden, F = m->ffn;
    char rel[256];
    int rc = 0;
    rc |= read_raw(dir, "embedding/weight.bin", m->emb, (size_t)m->vocab * H);
    rc |= read_raw(dir, "norm/weight.bin", m->gnorm, H);
    for (int l = 0; l < m->layers && rc == 0; ++l) {
        xlo_layer* y = &m->L[l];
        struct { const char* name; float* w; float* b; size_t rows, cols; } lin[] = {
            {"attn/Q", y->wq, y->bq, H, H},  {"attn/K", y->wk, y->bk, H, H},
            {"attn/V", y->wv, y->bv, H, H},  {"attn/W", y->wo, y->bo, H, H},
            {"ffn/W1", y->w1, y->b1, F, H},  {"ffn/V", y->wvf, y->bvf, F, H},
            {"ffn/W2", y->w2, y->b2, H, F},
        };
        for (size_t i = 0; i < sizeof(lin) / sizeof(lin[0]); ++i) {
            snprintf(rel, sizeof(rel), "blocks/%d/%s/weight.bin", l, lin[i].name);
            rc |= read_raw(dir, rel, lin[i].w, lin[i].rows * lin[i].cols);
            snprintf(rel, sizeof(rel), "blocks/%d/%s/bias.bin", l, lin[i].name);
            rc |= read_raw(dir, rel, lin[i].b, lin[i].rows);
        }
        snprintf(rel, sizeof(rel), "blocks/%d/norm1/weight.bin", l);
        rc |= read_raw(dir, rel, y->g1, H);
        snprintf(rel, sizeof(rel), "blocks/%d/norm2/weight.bin", l);
        rc |= read_raw(dir, rel, y->g2, H);
    }
    return rc == 0 ? 0 : -1;
}

/* TransformerBlock::forward, src/transformer.cu:68-105, for n rows starting
 * at cache position pos0 (prefill: pos0 = 0; decode: n = 1, pos0 = KV.n).  */
static void block_forward(xlo_model* m, xlo_layer* y, int n, int pos0, int prefill) {
    size_t H = m->hidden, F = m->ffn;
    int c = (int)(H / m->heads);
    memcpy(m->res, m->x, sizeof(float) * n * H);
    xlo_rmsnorm(m->x, y->g1, n, (int)H);
    /* AttentionBlock::forward, src/attn.cu:622-665 */
    xlo_linear(m->x, y->wq, y->bq, m->q, n, (int)H, (int)H);
    xlo_linear(m->x, y->wk, y->bk, m->k, n, (int)H, (int)H);
    xlo_linear(m->x, y->wv, y->bv, m->v, n, (int)H, (int)H);
    xlo_rope(m->q, n, m->heads, c, pos0, m->base);
    xlo_rope(m->k, n, m->heads, c, pos0, m->base);
    if (prefill)
        xlo_attn_prefill(m->q, m->k, m->v, m->att, y->kv_k, y->kv_v, n, m->heads, c);
    else
        xlo_attn_decode(m->q, m->k, m->v, m->att, y->kv_k, y->kv_v, pos0, m->heads, c);
    xlo_linear(m->att, y->wo, y->bo, m->x, n, (int)H, (int)H);
    for (size_t i = 0; i < n * H; ++i) m->x[i] += m->res[i];
    memcpy(m->res, m->x, sizeof(float) * n * H);
    xlo_rmsnorm(m->x, y->g2, n, (int)H);
    /* SwishGLU::forward, src/ffn.cu:92-109 */
    xlo_linear(m->x, y->w1, y->b1, m->h1, n, (int)H, (int)F);
    xlo_linear(m->x, y->wvf, y->bvf, m->h2, n, (int)H, (int)F);
    xlo_silu_mul(m->h1, m->h2, (size_t)n * F);
    xlo_linear(m->h1, y->w2, y->b2, m->x, n, (int)F, (int)H);
    for (size_t i = 0; i < n * H; ++i) m->x[i] += m->res[i];
}

/* Transformer::forward(vector), src/transformer.cu:163-178: prefill resets
 * the cache to the n prompt positions and returns last-row logits.         */
int xlo_model_prefill(xlo_model* m, const int* ids, int n, float* logits) {
    if (n <= 0 || n > m->max_len) return -2;
    for (int i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= m->vocab) return -3;
    size_t H = m->hidden;
    xlo_embedding(m->emb, (int)H, ids, n, m->x);
    for (int l = 0; l < m->layers; ++l) block_forward(m, &m->L[l], n, 0, 1);
    m->n = n;
    xlo_rmsnorm(m->x, m->gnorm, n, (int)H);
    memcpy(m->last, m->x + (size_t)(n - 1) * H, sizeof(float) * H);
    xlo_lm_head(m->emb, m->last, logits, m->vocab, (int)H);
    return 0;
}

/* Transformer::forward(int), src/transformer.cu:180-186: one decode step at
 * position KV.n; the reference exits when the cache is full
 * (src/attn.cu:506-515), here that is error -4.                             */
int xlo_model_decode(xlo_model* m, int id, float* logits) {
    if (id < 0 || id >= m->vocab) return -3;
    if (m->n >= m->max_len) return -4;
    size_t H = m->hidden;
    xlo_embedding(m->emb, (int)H, &id, 1, m->x);
    for (int l = 0; l < m->layers; ++l) block_forward(m, &m->L[l], 1, m->n, 0);
    m->n += 1;
    xlo_rmsnorm(m->x, m->gnorm, 1, (int)H);
    xlo_lm_head(m->emb, m->x, logits, m->vocab, (int)H);
    return 0;
}

int xlo_model_n(const xlo_model* m) { return m->n; }

/* Position-major copies of one layer's cache rows 0..npos-1. */
void xlo_model_kv_copy(const xlo_model* m, int layer, int npos, float* k_out, float* v_out) {
    size_t count = (size_t)npos * m->hidden;
    memcpy(k_out, m->L[layer].kv_k, sizeof(float) * count);
    memcpy(v_out, m->L[layer].kv_v, sizeof(float) * count);
}
