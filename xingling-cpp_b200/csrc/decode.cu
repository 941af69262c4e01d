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
//  sample_*_kernel    repetition-penalised top-1024 / temperature / top-p
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
    // A position outside [0, max_ctx) would write the caches, read the RoPE
    // table and index the split partials out of range: nothing is touched,
    // and the head's output is NaN so that the caller sees the error.
    if (n < 0 || n >= p.max_ctx) {
        if (s == 0 && tid < kHeadDim) p.out[h * kHeadDim + tid] = __int_as_float(0x7fc00000);
        return;
    }
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
// Sampler: the histogram / gather chain declared with SampleWorkHdr.
constexpr int kSampWarps = kSampThreads / 32;
constexpr int kSampLoads = 4;      // keys per thread loaded before any is used
constexpr int kErrSample = 8;      // DevState::err bit: the chain found inconsistent counts

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
// src/inference.cu:87-111.  The two float sums (the softmax denominator and
// the running probability, which stops at the top-p cut) are sequential in
// candidate order on one thread, as in the reference; the exponentials, the
// divides and the search for the drawn index run across the block, which
// gives the reference's index because the running sums never decrease and
// r * total < total.  prob: 1024 floats, 16-byte aligned.  All threads of
// the block call it; thread 0 writes *s_token.
__device__ void draw_token(const unsigned long long* cand, int kc, float* prob, const DevState* st, int* s_token) {
    __shared__ float s_sum;
    __shared__ int s_cut, s_pick, s_done;
    const int tid = threadIdx.x, lane = tid & 31;
    const float top_p = st->in.top_p;
    const float inv_t_den = st->in.temperature + 0.001f;
    const float v0 = key_float(static_cast<uint32_t>(cand[0] >> 32)) / inv_t_den;
    float e = 0.0f;
    if (tid < kc) {
        const float v = key_float(static_cast<uint32_t>(cand[tid] >> 32)) / inv_t_den;
        e = expf(v - v0);
    }
    prob[tid] = e;
    if (tid == 0) {
        s_cut = kc - 1;
        s_pick = kc - 1;
    }
    __syncthreads();
    float4* p4 = reinterpret_cast<float4*>(prob);
    constexpr int nq = kTopK / 4;
    if (tid == 0) {
        // 1 + e_1 + ... (prob[0] = exp(0) = 1; entries past kc are 0 and add nothing)
        float4 q = p4[0];
        float sum = 1.0f;
        sum += q.y;
        sum += q.z;
        sum += q.w;
#pragma unroll 8
        for (int i = 1; i < nq; ++i) {
            q = p4[i];
            sum += q.x;
            sum += q.y;
            sum += q.z;
            sum += q.w;
        }
        s_sum = sum;
    }
    __syncthreads();
    if (tid < kc) prob[tid] = prob[tid] / s_sum;
    __syncthreads();
    if (tid == 0) {
        // running sums, in place, up to the group of 16 where one reaches top_p
        // (the next group's loads are issued before this group's adds)
        float acc = 0.0f;
        int q = 0;
        float4 c[4], n[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) c[u] = p4[u];
        for (; q < nq; q += 4) {
            if (q + 4 < nq) {
#pragma unroll
                for (int u = 0; u < 4; ++u) n[u] = p4[q + 4 + u];
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                float4 x = c[u];
                acc += x.x;
                x.x = acc;
                acc += x.y;
                x.y = acc;
                acc += x.z;
                x.z = acc;
                acc += x.w;
                x.w = acc;
                p4[q + u] = x;
            }
            if (acc >= top_p) {
                q += 4;
                break;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) c[u] = n[u];
        }
        s_done = 4 * q;
    }
    __syncthreads();
    // top-p cut: the first running sum reaching top_p, else the last candidate
    const int lim = min(s_done, kc);
    const unsigned hc = __ballot_sync(0xffffffffu, tid < lim && prob[tid] >= top_p);
    if (lane == 0 && hc) atomicMin(&s_cut, (tid & ~31) + __ffs(hc) - 1);
    __syncthreads();
    // the draw: the first running sum above r * total (total = the sum at the cut)
    const int cut = s_cut;
    const float thr = st->in.uniform * prob[cut];
    const unsigned hit = __ballot_sync(0xffffffffu, tid <= cut && prob[tid] > thr);
    if (lane == 0 && hit) atomicMin(&s_pick, (tid & ~31) + __ffs(hit) - 1);
    __syncthreads();
    if (tid == 0) *s_token = static_cast<int>(0xffffffffu - static_cast<uint32_t>(cand[s_pick] & 0xffffffffull));
}

// Device view of one sequence's work area (layout of sample_work_bytes).
struct SampleWork {
    SampleWorkHdr* h;
    unsigned int* hist;        // [2048]
    unsigned long long* cand;  // [kCandCap]
    int* tie_cnt;              // [grid]
    unsigned int* tie_ids;     // [grid][slice]
};
constexpr size_t kWorkHdrBytes = 256;
constexpr size_t kWorkHistBytes = 2048 * sizeof(unsigned int);
constexpr size_t kWorkCandBytes = static_cast<size_t>(kCandCap) * sizeof(unsigned long long);
__host__ __device__ inline size_t align256(size_t n) { return (n + 255) / 256 * 256; }
__host__ __device__ inline int sample_slice(int V, int grid) { return (V + grid - 1) / grid; }

__device__ __forceinline__ SampleWork work_of(const SampleParams& p, int b) {
    char* base = static_cast<char*>(p.work) + static_cast<size_t>(b) * p.work_stride;
    SampleWork w;
    w.h = reinterpret_cast<SampleWorkHdr*>(base);
    base += kWorkHdrBytes;
    w.hist = reinterpret_cast<unsigned int*>(base);
    base += kWorkHistBytes;
    w.cand = reinterpret_cast<unsigned long long*>(base);
    base += kWorkCandBytes;
    w.tie_cnt = reinterpret_cast<int*>(base);
    base += align256(static_cast<size_t>(p.grid) * sizeof(int));
    w.tie_ids = reinterpret_cast<unsigned int*>(base);
    return w;
}

__device__ __forceinline__ bool greedy_step(const SampleParams& p, const DevState* st) {
    return !(st->in.top_p > 0.0f) && !p.full;
}
__device__ __forceinline__ bool skipped(const DevState* st) { return st->in.skip != 0; }

// The step's id: state, repetition flag, KV position (src/inference.cu:113 and
// the caller's history update).
__device__ __forceinline__ void finish_token(const SampleParams& p, int b, DevState* st, int tok) {
    st->token_out = tok;
    const int local = tok - p.v0;
    if (local >= 0 && local < p.V) p.rep_flags[static_cast<size_t>(b) * p.stride + local] = 1;
    if (st->in.decode_mode) st->pos += 1;
}

// One radix pass over this CTA's vocab slice (grid (p.grid, batch)):
// pass 0 counts the top 11 key bits of every id (shared-memory histogram,
// then one global add per non-empty bin); passes 1 and 2 count the next 11 /
// 10 bits of the few ids inside the chosen prefix straight into the global
// histogram.  The last CTA to finish picks the bin that holds the kc-th
// largest key, extends the prefix and zeroes the histogram; the selection is
// done when exactly kc ids are at or above the prefix, or after pass 2.
__global__ void __launch_bounds__(kSampThreads) sample_hist_kernel(const SampleParams p, int pass) {
    __shared__ unsigned int hist[2048];
    __shared__ int warp_tot[32];
    __shared__ int s_last;
    __shared__ unsigned int s_bin, s_cnt;
    __shared__ int s_excl;

    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.y;
    DevState* st = p.st + b;
    if (greedy_step(p, st) || skipped(st)) return;
    const SampleWork w = work_of(p, b);
    const int tid = threadIdx.x;
    const int V = p.V;
    const int kc = V < kTopK ? V : kTopK;
    if (pass == 0 && V <= kCandCap) {  // every id is a candidate
        if (blockIdx.x == 0 && tid == 0) {
            w.h->n_ge = V;
            w.h->done = 1;
        }
        return;
    }
    if (w.h->done) return;
    const uint32_t prefix = w.h->prefix, pmask = w.h->pmask;
    const int sh = pass == 0 ? 21 : pass == 1 ? 10 : 0;
    const uint32_t bm = pass == 2 ? 0x3ffu : 0x7ffu;
    const int S = sample_slice(V, p.grid);
    const int lo = blockIdx.x * S, hi = min(V, lo + S);
    const float* x = p.logits + static_cast<size_t>(b) * p.stride;
    if (pass == 0) {
        for (int i = tid; i < 2048; i += kSampThreads) hist[i] = 0;
        __syncthreads();
    }
    for (int base = lo; base < hi; base += kSampThreads * kSampLoads) {
        uint32_t k[kSampLoads];
#pragma unroll
        for (int j = 0; j < kSampLoads; ++j) {
            const int i = base + j * kSampThreads + tid;
            k[j] = i < hi ? float_key(__ldcg(x + i)) : 0u;
        }
#pragma unroll
        for (int j = 0; j < kSampLoads; ++j) {
            const int i = base + j * kSampThreads + tid;
            if (i >= hi) continue;
            if (pass == 0) {
                atomicAdd(&hist[k[j] >> 21], 1u);
            } else if ((k[j] & pmask) == prefix) {
                atomicAdd(&w.hist[(k[j] >> sh) & bm], 1u);
            }
        }
    }
    if (pass == 0) {
        __syncthreads();
        for (int i = tid; i < 2048; i += kSampThreads) {
            const unsigned int c = hist[i];
            if (c) atomicAdd(&w.hist[i], c);
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        s_last = atomicAdd(&w.h->ticket, 1) == static_cast<int>(gridDim.x) - 1;
        s_bin = 0;
        s_cnt = 0;
        s_excl = -1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int need = kc - w.h->n_above;
    // Thread t owns bins (2047 - 2t, 2046 - 2t); scan counts from the top.
    const int bhi = 2047 - 2 * tid, blo = 2046 - 2 * tid;
    const int chi = static_cast<int>(__ldcg(w.hist + bhi)), clo = static_cast<int>(__ldcg(w.hist + blo));
    const int incl = block_inclusive_scan(chi + clo, warp_tot);
    const int excl = incl - chi - clo;
    if (excl < need && need <= excl + chi) {
        s_bin = static_cast<unsigned>(bhi);
        s_cnt = static_cast<unsigned>(chi);
        s_excl = excl;
    } else if (excl + chi < need && need <= incl) {
        s_bin = static_cast<unsigned>(blo);
        s_cnt = static_cast<unsigned>(clo);
        s_excl = excl + chi;
    }
    w.hist[bhi] = 0;
    w.hist[blo] = 0;
    __syncthreads();
    if (tid == 0) {
        if (s_excl < 0) {
            atomicOr(&st->err, kErrSample);
            w.h->done = 1;  // the gather reports the error and resets the work area
            w.h->exact = 0;
            w.h->n_ge = -1;
        } else {
            const int n_above = w.h->n_above + s_excl;
            const int n_ge = n_above + static_cast<int>(s_cnt);
            w.h->prefix = prefix | (s_bin << sh);
            w.h->pmask = pmask | (bm << sh);
            w.h->n_above = n_above;
            w.h->n_ge = n_ge;
            w.h->passes = pass + 1;
            // Stop once exactly kc ids are at or above the prefix; after the last
            // pass the prefix is the full threshold key and a wider count is a tie
            // there, resolved by id order.
            w.h->exact = pass == 2 && n_ge > kc;
            w.h->done = n_ge == kc || pass == 2;
        }
        w.h->ticket = 0;
    }
}

// One compare-exchange of a descending bitonic stage of size k at distance
// j: element i keeps the larger value when it is the lower index of a
// descending pair or the upper index of an ascending one.
__device__ __forceinline__ unsigned long long bitonic_pick(unsigned long long v, unsigned long long y, int i, int j,
                                                           int k) {
    const bool keep_max = ((i & j) == 0) == ((i & k) == 0);
    return (v < y) == keep_max ? y : v;
}

// Descending bitonic sort of M x 1024 packed candidates, element i at a[i]
// (thread t holds elements t, 1024 + t, ...), unrolled: distances of 1024 and
// more compare registers of one thread, 32 .. 512 go through shared memory
// (for M = 1 alternating between a[0, 1024) and a[1024, 2048), one barrier a
// stage), below 32 through warp shuffles.
template <int M>
__device__ void bitonic_sort_desc(unsigned long long* a) {
    constexpr int n = M * kSampThreads;
    const int tid = threadIdx.x;
    unsigned long long v[M];
#pragma unroll
    for (int m = 0; m < M; ++m) v[m] = a[m * kSampThreads + tid];
    __syncthreads();
    int half = 0;
#pragma unroll
    for (int k = 2; k <= n; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (j >= kSampThreads) {
#pragma unroll
                for (int m = 0; m < M; ++m) {
#pragma unroll
                    for (int m2 = m + 1; m2 < M; ++m2) {
                        if ((m ^ m2) * kSampThreads != j) continue;
                        const unsigned long long x = v[m], y = v[m2];
                        const bool desc = ((m * kSampThreads + tid) & k) == 0;
                        if (desc ? (x < y) : (x > y)) {
                            v[m] = y;
                            v[m2] = x;
                        }
                    }
                }
            } else if (j >= 32) {
                if (M == 1) {
                    unsigned long long* t = a + half * kSampThreads;
                    t[tid] = v[0];
                    __syncthreads();
                    v[0] = bitonic_pick(v[0], t[tid ^ j], tid, j, k);
                    half ^= 1;
                } else {
                    __syncthreads();
#pragma unroll
                    for (int m = 0; m < M; ++m) a[m * kSampThreads + tid] = v[m];
                    __syncthreads();
#pragma unroll
                    for (int m = 0; m < M; ++m)
                        v[m] = bitonic_pick(v[m], a[m * kSampThreads + (tid ^ j)], m * kSampThreads + tid, j, k);
                }
            } else {
#pragma unroll
                for (int m = 0; m < M; ++m)
                    v[m] = bitonic_pick(v[m], __shfl_xor_sync(0xffffffffu, v[m], j), m * kSampThreads + tid, j, k);
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < M; ++m) a[m * kSampThreads + tid] = v[m];
    __syncthreads();
}

// Gather and draw (grid (p.grid, batch)).  Each CTA adds the ids of its slice
// whose key is at or above the chosen prefix (above it, when the prefix is an
// exact threshold with a wide tie) to the candidate list, packed (key, ~global
// id), and, for an exact threshold, lists its tied ids in id order.  The last
// CTA loads the list, appends the lowest tied ids the count still needs,
// sorts (value, then lower id) so that the first kc are sample_cpu's candidate
// list, then draws (or, tensor parallel, writes the list out) and leaves the
// work area zeroed.
__global__ void __launch_bounds__(kSampThreads) sample_gather_kernel(const SampleParams p) {
    __shared__ unsigned long long s_cand[kCandCap];  // M = 1 sorts use [1024, 2048) as the second buffer
    __shared__ __align__(16) float prob[kTopK];
    __shared__ int tie_pre[kSampThreads + 1];
    __shared__ int warp_tot[32];
    __shared__ int s_last, s_token, s_run;

    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.y;
    DevState* st = p.st + b;
    const int tid = threadIdx.x, lane = tid & 31;
    if (skipped(st)) return;
    if (greedy_step(p, st)) {
        if (blockIdx.x == 0 && tid == 0) finish_token(p, b, st, unpack_argmax_index(st->argmax_final));
        return;
    }
    const SampleWork w = work_of(p, b);
    const int V = p.V;
    const int kc = V < kTopK ? V : kTopK;
    const uint32_t prefix = w.h->prefix;
    const int exact = w.h->exact;
    const int n_ge = w.h->n_ge;
    const bool ok = w.h->done && n_ge >= 0;
    const int S = sample_slice(V, p.grid);
    const int lo = blockIdx.x * S, hi = min(V, lo + S);
    const float* x = p.logits + static_cast<size_t>(b) * p.stride;
    const unsigned lt = (1u << lane) - 1u;
    if (tid == 0) s_run = 0;
    if (ok) {
        for (int base = lo; base < hi; base += kSampThreads * kSampLoads) {
            uint32_t k[kSampLoads];
#pragma unroll
            for (int j = 0; j < kSampLoads; ++j) {
                const int i = base + j * kSampThreads + tid;
                k[j] = i < hi ? float_key(__ldcg(x + i)) : 0u;
            }
#pragma unroll
            for (int j = 0; j < kSampLoads; ++j) {
                const int i = base + j * kSampThreads + tid;
                const bool take = i < hi && (exact ? k[j] > prefix : k[j] >= prefix);
                const unsigned bt = __ballot_sync(0xffffffffu, take);
                if (bt) {
                    const int leader = __ffs(bt) - 1;
                    int slot = 0;
                    if (lane == leader) slot = atomicAdd(&w.h->n_gt, __popc(bt));
                    slot = __shfl_sync(0xffffffffu, slot, leader) + __popc(bt & lt);
                    if (take && slot < kCandCap)
                        w.cand[slot] = (static_cast<unsigned long long>(k[j]) << 32) |
                                       (0xffffffffu - static_cast<uint32_t>(p.v0 + i));
                }
                if (exact) {  // block-uniform: list this slice's tied ids in id order
                    const int tie = i < hi && k[j] == prefix;
                    const int incl = block_inclusive_scan(tie, warp_tot);
                    if (tie) w.tie_ids[static_cast<size_t>(blockIdx.x) * S + s_run + incl - 1] = static_cast<unsigned>(i);
                    __syncthreads();
                    if (tid == kSampThreads - 1) s_run += incl;
                    __syncthreads();
                }
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        if (exact) w.tie_cnt[blockIdx.x] = s_run;
        __threadfence();
        s_last = atomicAdd(&w.h->ticket, 1) == static_cast<int>(gridDim.x) - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // --- last CTA: candidate list, sort, draw ---
    const int n_gt = exact ? w.h->n_above : n_ge;
    const bool counts_ok = ok && __ldcg(&w.h->n_gt) == n_gt && n_gt <= kCandCap;
    if (!counts_ok) {
        if (tid == 0) {
            atomicOr(&st->err, kErrSample);
            finish_token(p, b, st, unpack_argmax_index(st->argmax_final));
        }
    } else {
        int n_sort = kTopK;
        while (n_sort < n_gt) n_sort <<= 1;
        for (int i = tid; i < n_sort; i += kSampThreads) s_cand[i] = i < n_gt ? __ldcg(w.cand + i) : 0ull;
        if (exact) {
            // the need_eq lowest tied ids: slices in order, each slice's list in id order
            const int need_eq = kc - n_gt;
            const int c = tid < p.grid ? __ldcg(w.tie_cnt + tid) : 0;
            const int incl = block_inclusive_scan(c, warp_tot);
            tie_pre[tid + 1] = incl;
            if (tid == 0) tie_pre[0] = 0;
            __syncthreads();
            for (int r = tid; r < need_eq; r += kSampThreads) {
                int a = 0, z = p.grid - 1;  // the last slice whose first tie index is <= r
                while (a < z) {
                    const int mid = (a + z + 1) >> 1;
                    if (tie_pre[mid] <= r) a = mid;
                    else z = mid - 1;
                }
                const unsigned id = __ldcg(w.tie_ids + static_cast<size_t>(a) * S + (r - tie_pre[a]));
                s_cand[n_gt + r] = (static_cast<unsigned long long>(prefix) << 32) | (0xffffffffu - (p.v0 + id));
            }
        }
        __syncthreads();
        if (n_sort == kTopK) bitonic_sort_desc<1>(s_cand);
        else if (n_sort == 2 * kTopK) bitonic_sort_desc<2>(s_cand);
        else bitonic_sort_desc<4>(s_cand);
        if (p.cand_out) {
            // Tensor-parallel select: this shard's sorted top-kc, merged across ranks by sample_merge_kernel.
            p.cand_out[tid] = tid < kc ? s_cand[tid] : 0ull;
        } else {
            draw_token(s_cand, kc, prob, st, &s_token);
            if (tid == 0) finish_token(p, b, st, s_token);
        }
    }
    __syncthreads();
    if (tid < static_cast<int>(sizeof(SampleWorkHdr) / sizeof(int))) reinterpret_cast<int*>(w.h)[tid] = 0;
}

// Greedy steps: the LM head's argmax is the step's id (grid (1, batch)).
__global__ void __launch_bounds__(32) sample_finish_kernel(const SampleParams p) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.y;
    if (threadIdx.x == 0 && !skipped(p.st + b)) finish_token(p, b, p.st + b, unpack_argmax_index(p.st[b].argmax_final));
}

// Step input of a device-side generation: the previous step's id (or the
// first id), the sampling arguments and the step's uniform; a run that has
// produced its stop id, done its steps or filled the cache skips the step.
__global__ void __launch_bounds__(32) gen_feed_kernel(const GenParams p) {
    if (threadIdx.x != 0) return;
    GenCtl* c = p.ctl;
    DevState* st = p.st;
    const int i = c->step;
    if (c->stopped || i >= c->n || st->pos >= c->max_ctx) {
        st->in.skip = 1;
        return;
    }
    st->in.skip = 0;
    st->in.token_in = i == 0 ? c->first : st->token_out;
    st->in.temperature = c->temperature;
    st->in.top_p = c->top_p;
    st->in.rp = c->rp;
    st->in.uniform = p.uniforms[i];
    st->in.decode_mode = 1;
}

// Records the step's id; the stop id ends the run (it is returned).
__global__ void __launch_bounds__(32) gen_collect_kernel(const GenParams p) {
    if (threadIdx.x != 0) return;
    GenCtl* c = p.ctl;
    DevState* st = p.st;
    if (st->in.skip) return;
    const int tok = st->token_out;
    p.out[c->step] = tok;
    c->step += 1;
    if (tok == c->stop_id) c->stopped = 1;
}

// Tensor-parallel merge of sample_cpu (src/inference.cu:58-114) over vocab
// shards: every rank holds the same all-gathered candidate lists (each shard's
// sorted top-1024, packed (key, ~global id)), sorts their union by value (ties:
// lower id first), keeps the top min(V, 1024) and draws exactly as the
// single-GPU sampler does, with the same uniform on every rank, so all ranks
// agree on the id.  Greedy steps take the all-reduced argmax instead.
__global__ void __launch_bounds__(kSampThreads) sample_merge_kernel(const SampleMergeParams p) {
    extern __shared__ unsigned long long all[];  // n_pad packed candidates
    __shared__ __align__(16) float prob[kTopK];
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

size_t sample_work_bytes(int V, int grid) {
    if (V <= 0 || grid <= 0) return 0;
    return kWorkHdrBytes + kWorkHistBytes + kWorkCandBytes + align256(static_cast<size_t>(grid) * sizeof(int)) +
           align256(static_cast<size_t>(grid) * sample_slice(V, grid) * sizeof(unsigned int));
}

int sample_grid(int V, int num_sms, int batch) {
    int g = num_sms / (batch > 0 ? batch : 1);
    const int by_size = (V + 255) / 256;  // at least 256 ids per slice
    if (g > by_size) g = by_size;
    if (g > kSampThreads) g = kSampThreads;
    return g > 0 ? g : 1;
}

cudaError_t launch_sample_chain(const SampleParams& p, int batch, bool pdl, cudaStream_t s) {
    if (batch <= 0 || batch > 65535 || p.grid <= 0 || p.grid > kSampThreads || !p.work || p.V <= 0 ||
        (batch > 1 && (p.stride < p.V || p.work_stride < sample_work_bytes(p.V, p.grid))) ||
        (p.cand_out && batch != 1)) {
        return cudaErrorInvalidValue;
    }
    const dim3 grid(p.grid, batch);
    for (int pass = 0; pass < 3; ++pass) {
        const cudaError_t e = launch_ex(sample_hist_kernel, grid, dim3(kSampThreads), 0, pass > 0 || pdl, s, p, pass);
        if (e != cudaSuccess) return e;
    }
    return launch_ex(sample_gather_kernel, grid, dim3(kSampThreads), 0, true, s, p);
}

cudaError_t launch_gen_feed(const GenParams& p, cudaStream_t s) {
    return launch_ex(gen_feed_kernel, dim3(1), dim3(32), 0, false, s, p);
}

cudaError_t launch_gen_collect(const GenParams& p, cudaStream_t s) {
    return launch_ex(gen_collect_kernel, dim3(1), dim3(32), 0, false, s, p);
}

cudaError_t launch_sample_finish(const SampleParams& p, int batch, bool pdl, cudaStream_t s) {
    if (batch <= 0 || batch > 65535 || (batch > 1 && p.stride < p.V)) return cudaErrorInvalidValue;
    return launch_ex(sample_finish_kernel, dim3(1, batch), dim3(32), 0, pdl, s, p);
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
