// Decode-step kernels for sm_100a (batch 1, fp32, HBM-bound).
//
//  norm_gemv_kernel   fused [embedding gather] + [residual add] + RMSNorm +
//                     GEMV + epilogue (bias / SwiGLU / residual / logits).
//                     Replaces Linear::forward_vec (src/linear.cu:260-282,
//                     309-357), RMSNorm::forward (src/rmsnorm.cu:46-80),
//                     silu_mul_vec (src/ffn.cu:112-139), add_kernel
//                     (src/transformer.cu:54-59) and Embedding::inverse
//                     (src/embedding.cu:130-154, 173-205).
//  attn_decode_kernel RoPE (src/rope.cu:20-45) + KV append + split-K
//                     attention over the head-major cache, replacing
//                     MultiHeadAttention::forward (src/attn.cu:372-447, 490-547).
//  sample_kernel      repetition-penalised top-1024 / temperature / top-p
//                     sampling on the device, replacing sample_cpu
//                     (src/inference.cu:58-114).
#include <math.h>

#include <atomic>

#include <mutex>
#include <string>

#include "xl_device.cuh"
#include "xl_engine.h"
#include "xl_kernels.h"

namespace xl {

namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvU = 4;         // float4 per lane per row per batch (8 KB in flight per warp)
constexpr int kGemvPrefetch = 2;  // row groups a warp keeps in flight as L2 bulk prefetches

// One warp computes a group of two consecutive rows per iteration (a W1/V
// pair in SwiGLU mode).  Weights stream once from HBM with 128-bit loads;
// x sits in shared memory, already normalised.
template <int MODE>
__global__ void __launch_bounds__(kGemvThreads) norm_gemv_kernel(const NormGemvParams p) {
    extern __shared__ float4 xs4[];
    __shared__ float red[kGemvWarps];
    __shared__ unsigned long long best_s[kGemvWarps];

    const int K4 = p.K >> 2;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int gw = blockIdx.x * kGemvWarps + warp;
    const int GW = gridDim.x * kGemvWarps;
    const int G = (p.M + 1) >> 1;
    const size_t group_floats = 2 * static_cast<size_t>(p.K);

    // Weights do not depend on the previous kernel: start pulling them into
    // L2 before waiting on it.
    if (lane == 0) {
        for (int d = 0; d < kGemvPrefetch; ++d) {
            const int g = gw + d * GW;
            if (g < G) {
                const int rows = min(2, p.M - 2 * g);
                prefetch_l2_bulk(p.W + g * group_floats, static_cast<uint32_t>(rows * p.K * 4));
            }
        }
    }
    pdl_launch_dependents();
    pdl_wait();

    const float4* src4 = p.table ? reinterpret_cast<const float4*>(p.table + static_cast<size_t>(*p.token) * p.K)
                                 : reinterpret_cast<const float4*>(p.x);
    const float4* d4 = reinterpret_cast<const float4*>(p.delta);
    float4* xo4 = (p.x_out != nullptr && blockIdx.x == 0) ? reinterpret_cast<float4*>(p.x_out) : nullptr;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < K4; i += kGemvThreads) {
        float4 v = src4[i];
        if (d4) {
            const float4 d = d4[i];
            v.x += d.x;
            v.y += d.y;
            v.z += d.z;
            v.w += d.w;
        }
        if (xo4) xo4[i] = v;
        xs4[i] = v;
        ss = dot4(v, v, ss);
    }
    if (p.gamma) {
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < kGemvWarps; ++w) tot += red[w];
        // RMSNorm of src/rmsnorm.cu:99-101: 1 / sqrt(mean + eps) in double.
        const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(tot / static_cast<float>(p.K)) + p.eps));
        const float4* g4 = reinterpret_cast<const float4*>(p.gamma);
        for (int i = threadIdx.x; i < K4; i += kGemvThreads) {
            float4 v = xs4[i];
            const float4 g = g4[i];
            v.x = v.x * inv * g.x;
            v.y = v.y * inv * g.y;
            v.z = v.z * inv * g.z;
            v.w = v.w * inv * g.w;
            xs4[i] = v;
        }
    }
    __syncthreads();

    float rp = 1.0f;
    if (MODE == kGemvLogits) rp = p.st->in.rp;
    float best_v = -INFINITY;
    int best_i = -1;

    const float4* W4 = reinterpret_cast<const float4*>(p.W);
    for (int g = gw; g < G; g += GW) {
        if (lane == 0) {
            const int gp = g + kGemvPrefetch * GW;
            if (gp < G) {
                const int rows = min(2, p.M - 2 * gp);
                prefetch_l2_bulk(p.W + gp * group_floats, static_cast<uint32_t>(rows * p.K * 4));
            }
        }
        const int r0 = 2 * g;
        const bool has1 = (r0 + 1) < p.M;
        const float4* w0 = W4 + static_cast<size_t>(r0) * K4;
        const float4* w1 = w0 + K4;
        float acc0 = 0.0f, acc1 = 0.0f;
        for (int base = 0; base < K4; base += 32 * kGemvU) {
            float4 a[kGemvU], b[kGemvU];
#pragma unroll
            for (int u = 0; u < kGemvU; ++u) {
                const int i = base + u * 32 + lane;
                a[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                b[u] = a[u];
                if (i < K4) {
                    a[u] = ld_stream(w0 + i);
                    if (has1) b[u] = ld_stream(w1 + i);
                }
            }
#pragma unroll
            for (int u = 0; u < kGemvU; ++u) {
                const int i = base + u * 32 + lane;
                if (i < K4) {
                    const float4 xv = xs4[i];
                    acc0 = dot4(a[u], xv, acc0);
                    acc1 = dot4(b[u], xv, acc1);
                }
            }
        }
        acc0 = warp_sum(acc0);
        acc1 = warp_sum(acc1);
        if (MODE == kGemvPlain) {
            if (lane == 0) p.y[r0] = acc0 + (p.bias ? p.bias[r0] : 0.0f);
            if (lane == 1 && has1) p.y[r0 + 1] = acc1 + (p.bias ? p.bias[r0 + 1] : 0.0f);
        } else if (MODE == kGemvResidual) {
            if (lane == 0) p.y[r0] += acc0 + (p.bias ? p.bias[r0] : 0.0f);
            if (lane == 1 && has1) p.y[r0 + 1] += acc1 + (p.bias ? p.bias[r0 + 1] : 0.0f);
        } else if (MODE == kGemvSwiGLU) {
            if (lane == 0) {
                const float a = acc0 + p.bias[r0];
                const float c = acc1 + p.bias[r0 + 1];
                p.y[g] = silu(a) * c;
            }
        } else {  // kGemvLogits
            float v0 = acc0;
            if (p.rep_flags[r0]) v0 = rep_penalty(v0, rp);
            if (v0 > best_v) {
                best_v = v0;
                best_i = r0;
            }
            if (lane == 0) p.y[r0] = v0;
            if (has1) {
                float v1 = acc1;
                if (p.rep_flags[r0 + 1]) v1 = rep_penalty(v1, rp);
                if (v1 > best_v) {
                    best_v = v1;
                    best_i = r0 + 1;
                }
                if (lane == 1) p.y[r0 + 1] = v1;
            }
        }
    }

    if (MODE == kGemvLogits) {
        // All lanes hold identical warp sums, so best_v / best_i are warp-uniform.
        if (lane == 0) best_s[warp] = best_i >= 0 ? pack_argmax(best_v, p.row_offset + best_i) : 0ull;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long k = 0;
#pragma unroll
            for (int w = 0; w < kGemvWarps; ++w) k = best_s[w] > k ? best_s[w] : k;
            if (k) atomicMax(&p.st->argmax_key, k);
            __threadfence();
            const int t = atomicAdd(&p.st->lm_done, 1);
            if (t == static_cast<int>(gridDim.x) - 1) {
                __threadfence();
                const unsigned long long fin = atomicExch(&p.st->argmax_key, 0ull);
                p.st->argmax_final = fin;
                p.st->greedy_token = unpack_argmax_index(fin);
                p.st->lm_done = 0;
            }
        }
    }
}

// RoPE + KV append + one split of the decode attention for one head.
// grid (heads, max_splits), 128 threads.  The split owning the new slot n
// rotates k and writes k, v into the cache; every split rotates q.  The last
// split of a head to finish merges the (max, sum, o) partials.
__global__ void __launch_bounds__(128) attn_decode_kernel(const AttnDecodeParams p) {
    __shared__ float qs[kHeadDim];
    __shared__ float sc[kAttnChunk];
    __shared__ float ored[2][kHeadDim];
    __shared__ float stat[2];
    __shared__ int is_last;

    const int h = blockIdx.x;
    const int s = blockIdx.y;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;

    pdl_launch_dependents();
    pdl_wait();

    const int n = *p.pos;
    const int total = n + 1;
    const int nsplit = (total + kAttnChunk - 1) / kAttnChunk;
    if (s >= nsplit) return;
    const int t0 = s * kAttnChunk;
    const int cnt = min(kAttnChunk, total - t0);
    const int HL = p.heads * kHeadDim;
    const float* q = p.qkv + h * kHeadDim;
    const float* kn = p.qkv + HL + h * kHeadDim;
    const float* vn = p.qkv + 2 * HL + h * kHeadDim;
    float* kc = p.kc + static_cast<size_t>(h) * p.max_ctx * kHeadDim;
    float* vc = p.vc + static_cast<size_t>(h) * p.max_ctx * kHeadDim;

    if (tid < kHalfHead) {
        const float2 cs = p.rope[n * kHalfHead + tid];
        const float a = q[tid], b = q[tid + kHalfHead];
        // 1/sqrt(64) = 2^-3 applied to q is exact.
        qs[tid] = (a * cs.x + b * cs.y) * 0.125f;
        qs[tid + kHalfHead] = (-a * cs.y + b * cs.x) * 0.125f;
        if (n >= t0 && n < t0 + cnt) {
            const float ka = kn[tid], kb = kn[tid + kHalfHead];
            kc[n * kHeadDim + tid] = ka * cs.x + kb * cs.y;
            kc[n * kHeadDim + tid + kHalfHead] = -ka * cs.y + kb * cs.x;
            vc[n * kHeadDim + tid] = vn[tid];
            vc[n * kHeadDim + tid + kHalfHead] = vn[tid + kHalfHead];
        }
    }
    __syncthreads();

    const float2 qv = reinterpret_cast<const float2*>(qs)[lane];
#pragma unroll 4
    for (int j = warp; j < cnt; j += 4) {
        const float2 kv = reinterpret_cast<const float2*>(kc + static_cast<size_t>(t0 + j) * kHeadDim)[lane];
        const float d = warp_sum(fmaf(kv.x, qv.x, kv.y * qv.y));
        if (lane == 0) sc[j] = d;
    }
    __syncthreads();
    if (warp == 0) {
        float m = -INFINITY;
        for (int j = lane; j < cnt; j += 32) m = fmaxf(m, sc[j]);
        m = warp_max(m);
        float l = 0.0f;
        for (int j = lane; j < cnt; j += 32) {
            const float e = expf(sc[j] - m);
            sc[j] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
            stat[0] = m;
            stat[1] = l;
        }
    }
    __syncthreads();
    {
        const int d = tid & (kHeadDim - 1);
        const int half = tid >> 6;
        float o = 0.0f;
        for (int j = half; j < cnt; j += 2) o = fmaf(sc[j], vc[static_cast<size_t>(t0 + j) * kHeadDim + d], o);
        ored[half][d] = o;
    }
    __syncthreads();
    if (nsplit == 1) {
        if (tid < kHeadDim) p.out[h * kHeadDim + tid] = (ored[0][tid] + ored[1][tid]) / stat[1];
        return;
    }
    const int maxs = attn_max_splits(p.max_ctx);
    float* pp = p.part + (static_cast<size_t>(h) * maxs + s) * (kHeadDim + 2);
    if (tid < kHeadDim) pp[2 + tid] = ored[0][tid] + ored[1][tid];
    if (tid == 0) {
        pp[0] = stat[0];
        pp[1] = stat[1];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const int t = atomicAdd(&p.counters[h], 1);
        is_last = (t == nsplit - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    if (tid < kHeadDim) {
        const float* base = p.part + static_cast<size_t>(h) * maxs * (kHeadDim + 2);
        float M = -INFINITY;
        for (int k = 0; k < nsplit; ++k) M = fmaxf(M, __ldcg(base + k * (kHeadDim + 2)));
        float L = 0.0f, O = 0.0f;
        for (int k = 0; k < nsplit; ++k) {
            const float* pk = base + k * (kHeadDim + 2);
            const float w = expf(__ldcg(pk) - M);
            L = fmaf(__ldcg(pk + 1), w, L);
            O = fmaf(__ldcg(pk + 2 + tid), w, O);
        }
        p.out[h * kHeadDim + tid] = O / L;
    }
    if (tid == 0) p.counters[h] = 0;
}

// ---------------------------------------------------------------------------
// Sampler: one CTA of 1024 threads.
constexpr int kSampThreads = 1024;
constexpr int kSampWarps = kSampThreads / 32;

// Block-wide inclusive scan of one int per thread.
__device__ int block_inclusive_scan(int v, int* warp_tot) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
    }
    if (lane == 31) warp_tot[warp] = v;
    __syncthreads();
    if (warp == 0) {
        int w = warp_tot[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += t;
        }
        warp_tot[lane] = w;
    }
    __syncthreads();
    const int add = warp > 0 ? warp_tot[warp - 1] : 0;
    __syncthreads();
    return v + add;
}

// Temperature, softmax over the kc sorted candidates (packed (key, ~global
// id)), top-p and the draw with the step's uniform: the arithmetic of
// src/inference.cu:87-111, sequential float sums in candidate order on one
// thread.  All threads of the block call it; thread 0 writes *s_token.
__device__ void draw_token(const unsigned long long* cand, int kc, float* prob, const DevState* st, int* s_token) {
    const int tid = threadIdx.x;
    const float top_p = st->in.top_p;
    const float inv_t_den = st->in.temperature + 0.001f;
    const float v0 = key_float(static_cast<uint32_t>(cand[0] >> 32)) / inv_t_den;
    float e = 0.0f;
    if (tid < kc) {
        const float v = key_float(static_cast<uint32_t>(cand[tid] >> 32)) / inv_t_den;
        e = expf(v - v0);
    }
    prob[tid] = e;
    __syncthreads();
    if (tid == 0) {
        float sum_exp = 1.0f;
        for (int i = 1; i < kc; ++i) sum_exp += prob[i];
        prob[0] = prob[0] / sum_exp;
        for (int i = 1; i < kc; ++i) prob[i] = prob[i] / sum_exp;
        float total = 0.0f;
        for (int i = 0; i < kc; ++i) {
            total += prob[i];
            if (total >= top_p) break;
        }
        const float r = st->in.uniform;
        float acc = 0.0f;
        int pick = kc - 1;
        for (int i = 0; i < kc; ++i) {
            acc += prob[i];
            if (acc > r * total) {
                pick = i;
                break;
            }
        }
        *s_token = static_cast<int>(0xffffffffu - static_cast<uint32_t>(cand[pick] & 0xffffffffull));
    }
}

__device__ __forceinline__ void sample_block(const SampleParams& p) {
    __shared__ unsigned int hist[2048];
    __shared__ unsigned long long cand[kTopK];
    __shared__ float prob[kTopK];
    __shared__ int warp_tot[32];
    __shared__ int wcnt[2][kSampWarps];
    __shared__ unsigned int sel_bin;
    __shared__ int sel_need;
    __shared__ int s_token;

    pdl_launch_dependents();
    pdl_wait();

    DevState* st = p.st;
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const float top_p = st->in.top_p;
    if (!(top_p > 0.0f) && !p.full) {
        // top_p <= 0: the prefix loop of src/inference.cu:100-103 stops at the
        // first (largest) candidate and any r in [0,1) returns it.
        if (tid == 0) s_token = unpack_argmax_index(st->argmax_final);
    } else {
        const int V = p.V;
        const int kc = V < kTopK ? V : kTopK;
        // --- radix select of the kc-th largest key: 11 + 11 + 10 bits ---
        uint32_t prefix = 0, pmask = 0;
        int need = kc;
        const int shifts[3] = {21, 10, 0};
        const int bits[3] = {11, 11, 10};
        for (int pass = 0; pass < 3; ++pass) {
            for (int i = tid; i < 2048; i += kSampThreads) hist[i] = 0;
            __syncthreads();
            const int sh = shifts[pass];
            const uint32_t bm = (1u << bits[pass]) - 1u;
            // Warp-aggregated counts: logits crowd into few bins, so lanes that
            // share a bin add once (their leader adds the group's size).
            for (int base = warp * 32; base < V; base += kSampThreads) {
                const int i = base + lane;
                uint32_t bin = 0;
                bool act = false;
                if (i < V) {
                    const uint32_t k = float_key(p.logits[i]);
                    act = (k & pmask) == prefix;
                    bin = (k >> sh) & bm;
                }
                const unsigned amask = __ballot_sync(0xffffffffu, act);
                if (act) {
                    const unsigned peers = __match_any_sync(amask, bin);
                    if (lane == __ffs(peers) - 1) atomicAdd(&hist[bin], static_cast<unsigned>(__popc(peers)));
                }
            }
            __syncthreads();
            // Thread t owns bins (2047 - 2t, 2046 - 2t); scan counts from the top.
            const int bhi = 2047 - 2 * tid, blo = 2046 - 2 * tid;
            const int chi = static_cast<int>(hist[bhi]), clo = static_cast<int>(hist[blo]);
            const int incl = block_inclusive_scan(chi + clo, warp_tot);
            const int excl = incl - chi - clo;
            if (excl < need && need <= excl + chi) {
                sel_bin = static_cast<unsigned>(bhi);
                sel_need = need - excl;
            } else if (excl + chi < need && need <= incl) {
                sel_bin = static_cast<unsigned>(blo);
                sel_need = need - excl - chi;
            }
            __syncthreads();
            prefix |= sel_bin << sh;
            pmask |= bm << sh;
            need = sel_need;
            __syncthreads();
        }
        const uint32_t T = prefix;  // key of the kc-th largest value
        const int need_eq = need;   // how many ids with key == T are taken (lowest ids first)
        const int n_gt = kc - need_eq;
        // --- ordered collection: warp w scans ids [w*per, (w+1)*per) ---
        const int per = ((V + kSampWarps * 32 - 1) / (kSampWarps * 32)) * 32;
        const int lo = warp * per, hi = min(V, lo + per);
        int cgt = 0, ceq = 0;
        for (int b = lo; b < hi; b += 32) {
            const int i = b + lane;
            const uint32_t k = i < hi ? float_key(p.logits[i]) : 0u;
            cgt += __popc(__ballot_sync(0xffffffffu, i < hi && k > T));
            ceq += __popc(__ballot_sync(0xffffffffu, i < hi && k == T));
        }
        if (lane == 0) {
            wcnt[0][warp] = cgt;
            wcnt[1][warp] = ceq;
        }
        __syncthreads();
        int off_gt = 0, off_eq = 0;
        for (int w = 0; w < warp; ++w) {
            off_gt += wcnt[0][w];
            off_eq += wcnt[1][w];
        }
        const unsigned lt = (1u << lane) - 1u;
        for (int b = lo; b < hi; b += 32) {
            const int i = b + lane;
            const uint32_t k = i < hi ? float_key(p.logits[i]) : 0u;
            const bool gt = i < hi && k > T;
            const bool eq = i < hi && k == T;
            const unsigned bg = __ballot_sync(0xffffffffu, gt);
            const unsigned be = __ballot_sync(0xffffffffu, eq);
            const unsigned long long packed =
                (static_cast<unsigned long long>(k) << 32) | (0xffffffffu - static_cast<uint32_t>(p.v0 + i));
            if (gt) {
                const int at = off_gt + __popc(bg & lt);
                if (at < n_gt) cand[at] = packed;
            }
            if (eq) {
                const int r = off_eq + __popc(be & lt);
                if (r < need_eq && n_gt + r < kTopK) cand[n_gt + r] = packed;
            }
            off_gt += __popc(bg);
            off_eq += __popc(be);
        }
        for (int i = kc + tid; i < kTopK; i += kSampThreads) cand[i] = 0ull;
        __syncthreads();
        // --- bitonic sort, descending by (value, then lower id) ---
        for (int k = 2; k <= kTopK; k <<= 1) {
            for (int j = k >> 1; j > 0; j >>= 1) {
                const int i = tid;
                const int ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long a = cand[i], b = cand[ixj];
                    const bool desc = (i & k) == 0;
                    if (desc ? (a < b) : (a > b)) {
                        cand[i] = b;
                        cand[ixj] = a;
                    }
                }
                __syncthreads();
            }
        }
        if (p.cand_out) {
            // Tensor-parallel select: this shard's sorted top-kc, merged across ranks by sample_merge_kernel.
            for (int i = tid; i < kTopK; i += kSampThreads) p.cand_out[i] = cand[i];
            return;
        }
        // --- temperature, softmax over the candidates, top-p, draw ---
        draw_token(cand, kc, prob, st, &s_token);
    }
    __syncthreads();
    if (tid == 0) {
        const int tok = s_token;
        st->token_out = tok;
        const int local = tok - p.v0;
        if (local >= 0 && local < p.V) p.rep_flags[local] = 1;
        if (st->in.decode_mode) st->pos += 1;
    }
}

__global__ void __launch_bounds__(kSampThreads) sample_kernel(const SampleParams p) { sample_block(p); }

// kBatch independent sequences, one CTA each: sequence b's logits at
// logits + b * stride, its flags at rep_flags + b * stride, its state st + b.
__global__ void __launch_bounds__(kSampThreads) sample_batch_kernel(const SampleParams p, int stride) {
    SampleParams q = p;
    const int b = blockIdx.x;
    q.logits = p.logits + static_cast<size_t>(b) * stride;
    q.rep_flags = p.rep_flags + static_cast<size_t>(b) * stride;
    q.st = p.st + b;
    sample_block(q);
}

// Tensor-parallel merge of sample_cpu (src/inference.cu:58-114) over vocab
// shards: every rank holds the same all-gathered candidate lists (each shard's
// sorted top-1024, packed (key, ~global id)), sorts their union by value (ties:
// lower id first), keeps the top min(V, 1024) and draws exactly as the
// single-GPU sampler does, with the same uniform on every rank, so all ranks
// agree on the id.  Greedy steps take the all-reduced argmax instead.
__global__ void __launch_bounds__(kSampThreads) sample_merge_kernel(const SampleMergeParams p) {
    extern __shared__ unsigned long long all[];  // n_pad packed candidates
    __shared__ float prob[kTopK];
    __shared__ int s_token;
    pdl_launch_dependents();
    pdl_wait();
    DevState* st = p.st;
    const int tid = threadIdx.x;
    if (!(st->in.top_p > 0.0f)) {
        if (tid == 0) s_token = unpack_argmax_index(st->argmax_final);
    } else {
        for (int i = tid; i < p.n_pad; i += kSampThreads) all[i] = i < p.n ? p.cand[i] : 0ull;
        __syncthreads();
        for (int k = 2; k <= p.n_pad; k <<= 1) {
            for (int j = k >> 1; j > 0; j >>= 1) {
                for (int i = tid; i < p.n_pad; i += kSampThreads) {
                    const int ixj = i ^ j;
                    if (ixj > i) {
                        const unsigned long long a = all[i], b = all[ixj];
                        const bool desc = (i & k) == 0;
                        if (desc ? (a < b) : (a > b)) {
                            all[i] = b;
                            all[ixj] = a;
                        }
                    }
                }
                __syncthreads();
            }
        }
        draw_token(all, p.V_total < kTopK ? p.V_total : kTopK, prob, st, &s_token);
    }
    __syncthreads();
    if (tid == 0) {
        const int tok = s_token;
        st->token_out = tok;
        const int local = tok - p.v0;
        if (local >= 0 && local < p.V) p.rep_flags[local] = 1;
        if (st->in.decode_mode) st->pos += 1;
    }
}

template <typename Kern, typename... Args>
cudaError_t launch_ex(Kern kern, dim3 grid, dim3 block, size_t smem, bool pdl, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    count_launch();
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

}  // namespace

cudaError_t launch_norm_gemv(int mode, const NormGemvParams& p, int num_sms, bool pdl, cudaStream_t s) {
    if (p.K % 4 != 0 || p.M <= 0) return cudaErrorInvalidValue;
    const int groups = (p.M + 1) / 2;
    int grid = (groups + kGemvWarps - 1) / kGemvWarps;
    const int cap = 2 * num_sms;
    if (grid > cap) grid = cap;
    const size_t smem = static_cast<size_t>(p.K) * sizeof(float);
    switch (mode) {
        case kGemvPlain:
            return launch_ex(norm_gemv_kernel<kGemvPlain>, dim3(grid), dim3(kGemvThreads), smem, pdl, s, p);
        case kGemvSwiGLU:
            return launch_ex(norm_gemv_kernel<kGemvSwiGLU>, dim3(grid), dim3(kGemvThreads), smem, pdl, s, p);
        case kGemvResidual:
            return launch_ex(norm_gemv_kernel<kGemvResidual>, dim3(grid), dim3(kGemvThreads), smem, pdl, s, p);
        case kGemvLogits:
            return launch_ex(norm_gemv_kernel<kGemvLogits>, dim3(grid), dim3(kGemvThreads), smem, pdl, s, p);
        default:
            return cudaErrorInvalidValue;
    }
}

cudaError_t launch_attn_decode(const AttnDecodeParams& p, bool pdl, cudaStream_t s) {
    return launch_ex(attn_decode_kernel, dim3(p.heads, attn_max_splits(p.max_ctx)), dim3(128), 0, pdl, s, p);
}

cudaError_t launch_sample(const SampleParams& p, bool pdl, cudaStream_t s) {
    return launch_ex(sample_kernel, dim3(1), dim3(kSampThreads), 0, pdl, s, p);
}

cudaError_t launch_sample_batch(const SampleParams& p, int batch, int stride, bool pdl, cudaStream_t s) {
    if (batch <= 0) return cudaErrorInvalidValue;
    return launch_ex(sample_batch_kernel, dim3(batch), dim3(kSampThreads), 0, pdl, s, p, stride);
}

cudaError_t launch_sample_merge(const SampleMergeParams& p, bool pdl, cudaStream_t s) {
    if (p.n <= 0 || p.n_pad < p.n || p.n_pad > kMaxMergeCandidates || (p.n_pad & (p.n_pad - 1))) {
        return cudaErrorInvalidValue;
    }
    const size_t smem = static_cast<size_t>(p.n_pad) * sizeof(unsigned long long);
    cudaError_t e = cudaFuncSetAttribute(sample_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    return launch_ex(sample_merge_kernel, dim3(1), dim3(kSampThreads), smem, pdl, s, p);
}

void set_error(const std::string& msg);

// ---------------------------------------------------------------------------
// Decode attention without a caller workspace.
//
// The split-K partials and the per-head split counters live in this
// file-scope device array instead of caller memory.  Every GPU that loads the
// library holds the array until the process exits.  Its device address is
// looked up once per device (cudaGetSymbolAddress with that device current)
// by the first call on that device; in host code the symbol itself is only a
// host-side stand-in and is never passed to a kernel.
namespace {
constexpr int kStaticMaxHeads = 32;
constexpr int kStaticMaxCtx = 1024;
constexpr size_t kStaticPartBytes =
    static_cast<size_t>(kStaticMaxHeads) * ((kStaticMaxCtx + kAttnChunk - 1) / kAttnChunk) * (kHeadDim + 2) * 4;
constexpr size_t kStaticScratchBytes = kStaticPartBytes + kStaticMaxHeads * 4;  // partials, then counters
static __device__ __align__(256) unsigned char g_attn_scratch[kStaticScratchBytes];
constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;
}  // namespace

namespace {
std::atomic<long long> g_launches{0};  // kernels enqueued or recorded by the launchers
std::atomic<long long> g_graphs{0};    // kernels run by graph replays, less those recorded at capture
}  // namespace
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
void count_graph_kernels(long long n) { g_graphs.fetch_add(n, std::memory_order_relaxed); }
long long launch_count() {
    return g_launches.load(std::memory_order_relaxed) + g_graphs.load(std::memory_order_relaxed);
}

}  // namespace xl

extern "C" XL_API int xl_op_attn_decode_noalloc(const float* qkv, const float* rope, float* kc, float* vc, float* out,
                                                const int* pos, int heads, int max_ctx, void* stream) {
    if (!qkv || !rope || !kc || !vc || !out || !pos || heads <= 0 || max_ctx <= 0) {
        xl::set_error("xl_op_attn_decode_noalloc: bad arguments");
        return XL_ERR_ARG;
    }
    if (heads > xl::kStaticMaxHeads || max_ctx > xl::kStaticMaxCtx) {
        xl::set_error("xl_op_attn_decode_noalloc: heads must be <= 32 and max_ctx <= 1024 (the static scratch limit); "
                      "use xl_op_attn_decode with a workspace for larger sizes");
        return XL_ERR_ARG;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= xl::kMaxDevices) {
        xl::set_error(std::string("xl_op_attn_decode_noalloc: no usable current device: ") + cudaGetErrorString(e));
        return XL_ERR_CUDA;
    }
    void* base = nullptr;
    {
        std::lock_guard<std::mutex> lock(xl::g_scratch_mu);
        if (!xl::g_scratch_addr[dev]) {
            e = cudaGetSymbolAddress(&xl::g_scratch_addr[dev], xl::g_attn_scratch);
            if (e != cudaSuccess) {
                xl::g_scratch_addr[dev] = nullptr;
                xl::set_error(std::string("xl_op_attn_decode_noalloc: cudaGetSymbolAddress failed: ") +
                              cudaGetErrorString(e));
                return XL_ERR_CUDA;
            }
        }
        base = xl::g_scratch_addr[dev];
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The counters must start at zero; the partials need no clearing.
    int* counters = reinterpret_cast<int*>(static_cast<unsigned char*>(base) + xl::kStaticPartBytes);
    e = cudaMemsetAsync(counters, 0, sizeof(int) * heads, s);
    if (e != cudaSuccess) {
        xl::set_error(std::string("xl_op_attn_decode_noalloc: clearing the counters failed: ") + cudaGetErrorString(e));
        return XL_ERR_CUDA;
    }
    xl::AttnDecodeParams a{};
    a.qkv = qkv;
    a.rope = reinterpret_cast<const float2*>(rope);
    a.kc = kc;
    a.vc = vc;
    a.out = out;
    a.part = static_cast<float*>(base);  // laid out for max_ctx up to kStaticMaxCtx
    a.counters = counters;
    a.pos = pos;
    a.heads = heads;
    a.max_ctx = max_ctx;
    e = xl::launch_attn_decode(a, false, s);
    if (e != cudaSuccess) {
        xl::set_error(std::string("xl_op_attn_decode_noalloc: ") + cudaGetErrorString(e));
        return XL_ERR_CUDA;
    }
    return XL_OK;
}
