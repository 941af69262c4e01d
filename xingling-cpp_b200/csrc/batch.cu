// Batched decode: kBatch independent sequences advance one token per step on
// one GPU, sharing a single pass over the weights (an extension; the
// reference decodes one sequence at a time, src/attn.cu:372-447).
//
// A BatchDecoder borrows a loaded single-GPU Engine: its weights, RoPE table
// and prefill path.  Each sequence has its own KV cache ([kBatch][heads][T][64]
// per layer), repetition flags, logits and DevState (position, sampler
// inputs).  One decode step is a CUDA graph of per-op kernels chained with
// programmatic dependent launch:
//   16 x [RMSNorm + QKV GEMV (x kBatch), RoPE + KV append, attention,
//         out-proj GEMV + residual, RMSNorm + W1/V GEMV + SwiGLU,
//         W2 GEMV + residual]
//   -> final RMSNorm + LM head with per-sequence penalty and argmax
//   -> the single-sequence sampler once per sequence.
// The GEMVs are exact fp32 FMA: decode is HBM-bound, and the 3xTF32 tensor
// path would stream every weight twice (W and its lo half).  A warp owns 4
// rows and keeps 4 x kBatch = 32 accumulators; one 32-value butterfly leaves
// lane l with the sum for (row l / 8, sequence l % 8).
#include <math.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "engine.h"
#include "xl_device.cuh"
#include "xl_kernels.h"

namespace xl {

namespace {

constexpr int kBgThreads = 512;
constexpr int kBgWarps = kBgThreads / 32;
constexpr int kBgRows = 4;  // rows per warp-group
constexpr int kBgU = 2;     // float4 per lane per row in flight
constexpr int kBgPrefetch = 2;
static_assert(kBgRows * kBatch == 32, "one (row, sequence) sum per lane");

struct BatchGemvParams {
    const float* x;       // [kBatch][ldx] inputs, or nullptr with table
    const float* table;   // layer 0: x_b = table[tokens[b]]
    const int* tokens;    // [kBatch]
    int ldx;
    const float* gamma;   // RMSNorm gain or nullptr
    float eps;
    const float* W;       // [M][K]
    const float* bias;    // [M] or nullptr
    float* y;             // [kBatch][ldy]
    int ldy;
    float* x_out;         // table mode: the gathered rows (written by CTA 0) [kBatch][ldx]
    int M, K;
    const uint8_t* rep_flags;  // logits: [kBatch][M]
    DevState* st;              // logits: [kBatch]
    int* ticket;               // logits: CTAs finished (the last one resets it)
    int wpg;                   // warps per row group (each a K slice; 1 = a warp owns its groups)
};

// Butterfly reduce-scatter of 32 values held by every lane: afterwards lane l
// holds the warp-wide sum of value l.
__device__ __forceinline__ float reduce_scatter32(float (&v)[32]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int half = 16; half > 0; half >>= 1) {
        const bool upper = (lane & half) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, half);
        }
    }
    return v[0];
}

template <int MODE>
__global__ void __launch_bounds__(kBgThreads) batch_gemv_kernel(const BatchGemvParams p) {
    extern __shared__ float4 xs4[];  // [kBatch][K/4]
    __shared__ float red[kBatch][kBgWarps];
    __shared__ unsigned long long best_s[kBatch][kBgWarps];
    __shared__ float part[kBgWarps][32];
    const int K4 = p.K >> 2;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;  // 1 .. kBgWarps
    // Teams of wpg warps share a row group, each warp one K slice.
    const int wpg = p.wpg, teams = nwarps / wpg, team = warp / wpg, ks = warp % wpg;
    const int gw = blockIdx.x * teams + team, GW = gridDim.x * teams;
    const int G = (p.M + kBgRows - 1) / kBgRows;
    const int k_lo = K4 * ks / wpg, k_hi = K4 * (ks + 1) / wpg;
    const size_t group_floats = static_cast<size_t>(kBgRows) * p.K;

    if (lane == 0 && ks == 0 && warp < teams * wpg) {
        for (int d = 0; d < kBgPrefetch; ++d) {
            const int g = gw + d * GW;
            if (g < G) {
                const int rows = min(kBgRows, p.M - kBgRows * g);
                prefetch_l2_bulk(p.W + g * group_floats, static_cast<uint32_t>(rows * p.K * 4));
            }
        }
    }
    pdl_launch_dependents();
    pdl_wait();

    // Stage the kBatch input rows (RMSNorm of src/rmsnorm.cu:99-101 per row).
    for (int b = 0; b < kBatch; ++b) {
        const float4* src4 = p.table ? reinterpret_cast<const float4*>(p.table + static_cast<size_t>(p.tokens[b]) * p.K)
                                     : reinterpret_cast<const float4*>(p.x + static_cast<size_t>(b) * p.ldx);
        float4* xo4 = (p.x_out && blockIdx.x == 0) ? reinterpret_cast<float4*>(p.x_out + static_cast<size_t>(b) * p.ldx)
                                                   : nullptr;
        float ss = 0.0f;
        for (int i = threadIdx.x; i < K4; i += blockDim.x) {
            const float4 v = src4[i];
            if (xo4) xo4[i] = v;
            xs4[b * K4 + i] = v;
            ss = dot4(v, v, ss);
        }
        if (p.gamma) {
            ss = warp_sum(ss);
            if (lane == 0) red[b][warp] = ss;
        }
    }
    if (p.gamma) {
        __syncthreads();
        const float4* g4 = reinterpret_cast<const float4*>(p.gamma);
        for (int b = 0; b < kBatch; ++b) {
            float tot = 0.0f;
            for (int w = 0; w < nwarps; ++w) tot += red[b][w];
            const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(tot / static_cast<float>(p.K)) + p.eps));
            for (int i = threadIdx.x; i < K4; i += blockDim.x) {
                float4 v = xs4[b * K4 + i];
                const float4 g = g4[i];
                v.x = v.x * inv * g.x;
                v.y = v.y * inv * g.y;
                v.z = v.z * inv * g.z;
                v.w = v.w * inv * g.w;
                xs4[b * K4 + i] = v;
            }
        }
    }
    __syncthreads();

    const int my_r = lane >> 3, my_b = lane & 7;  // the (row, sequence) this lane finishes
    float rp = 1.0f;
    if (MODE == kGemvLogits) rp = p.st[my_b].in.rp;
    float best_v = -INFINITY;
    int best_i = -1;
    const float4* W4 = reinterpret_cast<const float4*>(p.W);
    const bool in_team = warp < teams * wpg;
    const int iters = (G + GW - 1) / GW;  // the same trip count for every warp (block barriers inside)
    for (int it = 0; it < iters; ++it) {
        const int g = gw + it * GW;
        const bool has = in_team && g < G;
        if (has && lane == 0 && ks == 0) {
            const int gp = g + kBgPrefetch * GW;
            if (gp < G) {
                const int rows = min(kBgRows, p.M - kBgRows * gp);
                prefetch_l2_bulk(p.W + gp * group_floats, static_cast<uint32_t>(rows * p.K * 4));
            }
        }
        const int r0 = kBgRows * g;
        float acc[kBgRows * kBatch];
#pragma unroll
        for (int i = 0; i < kBgRows * kBatch; ++i) acc[i] = 0.0f;
        for (int base = has ? k_lo : k_hi; base < k_hi; base += 32 * kBgU) {
            float4 w[kBgRows][kBgU];
#pragma unroll
            for (int r = 0; r < kBgRows; ++r)
#pragma unroll
                for (int u = 0; u < kBgU; ++u) {
                    const int i = base + u * 32 + lane;
                    w[r][u] = (i < k_hi && r0 + r < p.M) ? ld_stream(W4 + static_cast<size_t>(r0 + r) * K4 + i)
                                                         : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
            for (int u = 0; u < kBgU; ++u) {
                const int i = base + u * 32 + lane;
                if (i < k_hi) {
#pragma unroll
                    for (int b = 0; b < kBatch; ++b) {
                        const float4 xv = xs4[b * K4 + i];
#pragma unroll
                        for (int r = 0; r < kBgRows; ++r) acc[r * kBatch + b] = dot4(w[r][u], xv, acc[r * kBatch + b]);
                    }
                }
            }
        }
        float v = reduce_scatter32(acc);
        if (wpg > 1) {
            // the team's K slices, summed in slice order by the team's first warp
            part[warp][lane] = v;
            __syncthreads();
            if (ks == 0) {
                v = part[warp][lane];
                for (int q = 1; q < wpg; ++q) v += part[warp + q][lane];
            }
            __syncthreads();
        }
        if (!has || ks != 0) continue;
        const int row = r0 + my_r;
        const bool ok = row < p.M;
        if (MODE == kGemvSwiGLU) {
            // rows (4g + 2j, 4g + 2j + 1) = (W1 row, V row) of hidden unit 2g + j
            const float partner = __shfl_down_sync(0xffffffffu, v, kBatch);
            if ((my_r & 1) == 0 && row + 1 < p.M) {
                const float h = silu(v + p.bias[row]) * (partner + p.bias[row + 1]);
                p.y[static_cast<size_t>(my_b) * p.ldy + (row >> 1)] = h;
            }
        } else if (MODE == kGemvLogits) {
            if (ok) {
                float lv = v;
                if (p.rep_flags[static_cast<size_t>(my_b) * p.M + row]) lv = rep_penalty(lv, rp);
                p.y[static_cast<size_t>(my_b) * p.ldy + row] = lv;
                if (lv > best_v) best_v = lv, best_i = row;
            }
        } else if (ok) {
            const float out = v + (p.bias ? p.bias[row] : 0.0f);
            float* dst = p.y + static_cast<size_t>(my_b) * p.ldy + row;
            if (MODE == kGemvResidual) *dst += out;
            else *dst = out;
        }
    }
    if (MODE == kGemvLogits) {
        // per sequence: warp max over the lanes of that sequence, then the CTA, then atomically the grid
        unsigned long long k = best_i >= 0 ? pack_argmax(best_v, best_i) : 0ull;
#pragma unroll
        for (int off = 8; off < 32; off <<= 1) {
            const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, off);
            k = o > k ? o : k;
        }
        if (lane < kBatch) best_s[lane][warp] = k;
        __syncthreads();
        if (threadIdx.x < kBatch) {
            unsigned long long c = 0;
            for (int w = 0; w < nwarps; ++w) c = best_s[threadIdx.x][w] > c ? best_s[threadIdx.x][w] : c;
            if (c) atomicMax(&p.st[threadIdx.x].argmax_key, c);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            const int t = atomicAdd(p.ticket, 1);
            if (t == static_cast<int>(gridDim.x) - 1) {
                __threadfence();
                for (int b = 0; b < kBatch; ++b) {
                    const unsigned long long fin = atomicExch(&p.st[b].argmax_key, 0ull);
                    p.st[b].argmax_final = fin;
                    p.st[b].greedy_token = unpack_argmax_index(fin);
                }
                *p.ticket = 0;
            }
        }
    }
}

// Step inputs: in[b] -> st[b].in, token ids for the layer-0 gather.
__global__ void batch_in_kernel(const StepIn* __restrict__ in, DevState* st, int* tokens) {
    const int b = threadIdx.x;
    if (b < kBatch) {
        st[b].in = in[b];
        tokens[b] = in[b].token_in;
    }
}

// One (sequence, head): RoPE of q (in place) and k at the sequence's position
// (src/rope.cu:20-45), k and v appended to that sequence's cache.
__global__ void __launch_bounds__(32) batch_rope_kv_kernel(float* __restrict__ qkv, const float2* __restrict__ rope,
                                                           float* __restrict__ kc, float* __restrict__ vc,
                                                           const DevState* __restrict__ st, int heads, int max_ctx) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x, h = blockIdx.y, j = threadIdx.x;
    const int HL = heads * kHeadDim;
    const int t = st[b].pos;
    float* row = qkv + static_cast<size_t>(b) * 3 * HL;
    const float2 cs = rope[t * kHalfHead + j];
    float* q = row + h * kHeadDim;
    const float qa = q[j], qb = q[j + kHalfHead];
    q[j] = qa * cs.x + qb * cs.y;
    q[j + kHalfHead] = -qa * cs.y + qb * cs.x;
    const float* k = row + HL + h * kHeadDim;
    const float* v = row + 2 * HL + h * kHeadDim;
    const size_t c = ((static_cast<size_t>(b) * heads + h) * max_ctx + t) * kHeadDim;
    const float ka = k[j], kb = k[j + kHalfHead];
    kc[c + j] = ka * cs.x + kb * cs.y;
    kc[c + j + kHalfHead] = -ka * cs.y + kb * cs.x;
    vc[c + j] = v[j];
    vc[c + j + kHalfHead] = v[j + kHalfHead];
}

// One (head, sequence) per CTA, 8 warps: warp w takes the 32-position chunks
// w, w + 8, w + 16 of positions 0..pos with an online softmax (lane = position
// for the scores, lane = output-dimension pair for P.V); the warps merge in
// shared memory (src/attn.cu:490-547 for one sequence).
constexpr int kBaWarps = 8;
__global__ void __launch_bounds__(32 * kBaWarps) batch_attn_kernel(const float* __restrict__ qkv,
                                                                   const float* __restrict__ kc,
                                                                   const float* __restrict__ vc, float* __restrict__ att,
                                                                   const DevState* __restrict__ st, int heads,
                                                                   int max_ctx) {
    __shared__ __align__(16) float qsh[kHeadDim];
    __shared__ float part[kBaWarps][kHeadDim + 4];
    pdl_launch_dependents();
    pdl_wait();
    const int h = blockIdx.x, b = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int HL = heads * kHeadDim;
    const int n = st[b].pos;  // the token's own position (already appended)
    if (threadIdx.x < kHeadDim)
        qsh[threadIdx.x] = qkv[static_cast<size_t>(b) * 3 * HL + h * kHeadDim + threadIdx.x] * 0.125f;
    __syncthreads();
    const float* kh = kc + (static_cast<size_t>(b) * heads + h) * max_ctx * kHeadDim;
    const float* vh = vc + (static_cast<size_t>(b) * heads + h) * max_ctx * kHeadDim;
    const int nsplit = n / 32 + 1;
    float m = -INFINITY, l = 0.0f;
    float2 o = make_float2(0.0f, 0.0f);
    const float4* q4 = reinterpret_cast<const float4*>(qsh);
    for (int s = warp; s < nsplit; s += kBaWarps) {
        const int t0 = s * 32, pos = t0 + lane;
        const bool mine = pos <= n;
        const float4* kr = reinterpret_cast<const float4*>(kh + static_cast<size_t>(mine ? pos : t0) * kHeadDim);
        float4 kv[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) kv[i] = __ldcg(kr + i);
        const int cnt = min(32, n + 1 - t0);
        const float2* vr = reinterpret_cast<const float2*>(vh + static_cast<size_t>(t0) * kHeadDim) + lane;
        float2 vrow[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) vrow[j] = j < cnt ? __ldcg(vr + j * (kHeadDim / 2)) : make_float2(0.f, 0.f);
        float d = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) d = dot4(kv[i], q4[i], d);
        const float sc = mine ? d : -INFINITY;
        const float mc = warp_max(sc);
        const float e = mine ? expf(sc - mc) : 0.0f;
        const float lc = warp_sum(e);
        float2 oc = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const float ej = __shfl_sync(0xffffffffu, e, j);
            oc.x = fmaf(ej, vrow[j].x, oc.x);
            oc.y = fmaf(ej, vrow[j].y, oc.y);
        }
        const float M = fmaxf(m, mc);
        const float a = m == -INFINITY ? 0.0f : expf(m - M), c = expf(mc - M);
        o.x = o.x * a + oc.x * c;
        o.y = o.y * a + oc.y * c;
        l = l * a + lc * c;
        m = M;
    }
    reinterpret_cast<float2*>(&part[warp][4])[lane] = o;
    if (lane == 0) {
        part[warp][0] = m;
        part[warp][1] = l;
    }
    __syncthreads();
    if (warp != 0) return;
    const int nw = min(kBaWarps, nsplit);
    const float mk = lane < nw ? part[lane][0] : -INFINITY;
    const float lk = lane < nw ? part[lane][1] : 0.0f;
    const float M = warp_max(mk);
    const float wk = lane < nw ? expf(mk - M) : 0.0f;
    const float L = warp_sum(lk * wk);
    float2 acc = make_float2(0.0f, 0.0f);
    for (int k = 0; k < nw; ++k) {
        const float wt = __shfl_sync(0xffffffffu, wk, k);
        const float2 ok = reinterpret_cast<const float2*>(&part[k][4])[lane];
        acc.x = fmaf(wt, ok.x, acc.x);
        acc.y = fmaf(wt, ok.y, acc.y);
    }
    reinterpret_cast<float2*>(att + static_cast<size_t>(b) * HL + h * kHeadDim)[lane] =
        make_float2(acc.x / L, acc.y / L);
}

template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

cudaError_t launch_batch_gemv(int mode, const BatchGemvParams& p, int num_sms, cudaStream_t s) {
    if (p.K % 4 || p.M <= 0) return cudaErrorInvalidValue;
    const size_t smem = static_cast<size_t>(kBatch) * p.K * 4;
    const int groups = (p.M + kBgRows - 1) / kBgRows;
    // Small matrices: fewer warps per CTA so that every SM streams part of the
    // weights; large ones (the LM head): full CTAs looping over the groups.
    // Row groups per CTA needed to cover the matrix with one CTA per SM; the
    // spare warps split each group's K range (teams of wpg warps).
    const int per_cta = (groups + num_sms - 1) / num_sms;
    BatchGemvParams q = p;
    q.wpg = std::max(1, kBgWarps / std::min(per_cta, kBgWarps));
    const int teams = kBgWarps / q.wpg;
    const int grid = std::min((groups + teams - 1) / teams, num_sms);
    const dim3 block(kBgThreads);
    cudaError_t e;
    switch (mode) {
        case kGemvPlain:
            e = cudaFuncSetAttribute(batch_gemv_kernel<kGemvPlain>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem));
            return e != cudaSuccess ? e : launch_pdl(batch_gemv_kernel<kGemvPlain>, dim3(grid), block, smem, s, q);
        case kGemvSwiGLU:
            e = cudaFuncSetAttribute(batch_gemv_kernel<kGemvSwiGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem));
            return e != cudaSuccess ? e
                                    : launch_pdl(batch_gemv_kernel<kGemvSwiGLU>, dim3(grid), block, smem, s, q);
        case kGemvResidual:
            e = cudaFuncSetAttribute(batch_gemv_kernel<kGemvResidual>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem));
            return e != cudaSuccess ? e
                                    : launch_pdl(batch_gemv_kernel<kGemvResidual>, dim3(grid), block, smem, s, q);
        case kGemvLogits:
            e = cudaFuncSetAttribute(batch_gemv_kernel<kGemvLogits>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem));
            return e != cudaSuccess ? e
                                    : launch_pdl(batch_gemv_kernel<kGemvLogits>, dim3(grid), block, smem, s, q);
        default:
            return cudaErrorInvalidValue;
    }
}

}  // namespace

// ---------------------------------------------------------------------------
BatchDecoder::~BatchDecoder() {
    if (!eng_) return;
    cudaSetDevice(eng_->device_);
    if (exec_) cudaGraphExecDestroy(exec_);
    if (exec_s_) cudaGraphExecDestroy(exec_s_);
    if (arena_) cudaFree(arena_);
    if (h_in_) cudaFreeHost(h_in_);
    if (h_st_) cudaFreeHost(h_st_);
    if (ev0_) cudaEventDestroy(ev0_);
    if (ev1_) cudaEventDestroy(ev1_);
}

int BatchDecoder::create(Engine* eng, BatchDecoder** out) {
    if (!eng || !out) {
        set_error("batch decoder: null argument");
        return XL_ERR_ARG;
    }
    if (!eng->loaded_ || eng->tp_ != 1) {
        set_error("batch decoder: needs a loaded single-GPU engine");
        return XL_ERR_STATE;
    }
    if (eng->H_ > 4096 || eng->Hl_ > 4096 || eng->Fl_ > 4096) {
        set_error("batch decoder: hidden and FFN widths up to 4096");
        return XL_ERR_ARG;
    }
    BatchDecoder* b = new BatchDecoder();
    b->eng_ = eng;
    const int rc = b->init();
    if (rc != XL_OK) {
        delete b;
        return rc;
    }
    *out = b;
    return XL_OK;
}

int BatchDecoder::cuda_fail(cudaError_t e, const char* what) {
    set_error(std::string("CUDA error in ") + what + ": " + cudaGetErrorString(e));
    return XL_ERR_CUDA;
}
#define XB_CUDA(call)                                   \
    do {                                                \
        cudaError_t e_ = (call);                        \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
    } while (0)

int BatchDecoder::init() {
    Engine& E = *eng_;
    XB_CUDA(cudaSetDevice(E.device_));
    const size_t L = E.cfg_.layers, H = E.H_, Hl = E.Hl_, Fl = E.Fl_, T = E.T_, V = E.V_, heads = E.heads_l_;
    const size_t kv = static_cast<size_t>(kBatch) * heads * T * kHeadDim * 4;
    std::vector<std::pair<void**, size_t>> plan;
    auto add = [&](void* slot, size_t bytes) { plan.emplace_back(reinterpret_cast<void**>(slot), bytes); };
    kc_.assign(L, nullptr);
    vc_.assign(L, nullptr);
    for (size_t l = 0; l < L; ++l) {
        add(&kc_[l], kv);
        add(&vc_[l], kv);
    }
    add(&x_, kBatch * H * 4);
    // batched persistent kernel: the second residual stream, the split projections' partial sums,
    // the attention partials and the phase counters / merge tickets
    add(&xb_, kBatch * H * 4);
    add(&cres_, kBatch * (H / kPersistTileRows) * kPersistMaxContrib * kPersistTileRows * 4);
    add(&part_, kBatch * heads * static_cast<size_t>(persistent_max_splits(E.T_)) * (kHeadDim + 2) * 4);
    add(&done_, done_words() * 4);
    add(&tick_, tick_words() * 4);
    add(&qkv_, kBatch * 3 * Hl * 4);
    add(&att_, kBatch * Hl * 4);
    add(&ffh_, kBatch * Fl * 4);
    add(&logits_, kBatch * V * 4);
    add(&rep_, kBatch * V);
    add(&st_, kBatch * sizeof(DevState));
    add(&in_, kBatch * sizeof(StepIn));
    add(&tokens_, kBatch * 4);
    add(&ticket_, 256);
    samp_grid_ = sample_grid(E.V_, E.num_sms_, kBatch);
    samp_stride_ = sample_work_bytes(E.V_, samp_grid_);
    add(&samp_work_, kBatch * samp_stride_);
    size_t total = 0;
    for (auto& pr : plan) total += (pr.second + 255) / 256 * 256;
    XB_CUDA(cudaMalloc(reinterpret_cast<void**>(&arena_), total));
    XB_CUDA(cudaMemset(arena_, 0, total));
    size_t off = 0;
    for (auto& pr : plan) {
        *pr.first = arena_ + off;
        off += (pr.second + 255) / 256 * 256;
    }
    XB_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h_in_), kBatch * sizeof(StepIn), cudaHostAllocDefault));
    XB_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h_st_), kBatch * sizeof(DevState), cudaHostAllocDefault));
    XB_CUDA(cudaEventCreate(&ev0_));
    XB_CUDA(cudaEventCreate(&ev1_));
    for (int b = 0; b < kBatch; ++b) {
        seed_[b] = E.philox_seed_ + 0x9E3779B97F4A7C15ull * static_cast<uint64_t>(b + 1);
        ctr_[b] = 0;
        n_[b] = -1;
    }
    return capture();
}

// The batched persistent kernel serves when the engine uses the persistent
// decode path, its option batch_persistent is 1, and the shape fits it (one GPU, widths multiples of 64 up to
// kBatchPersistMaxK, at most 32 CTAs per attention item, at most
// kPersistMaxContrib CTAs per row group of the split projections).
bool BatchDecoder::persistent_fits() const {
    const Engine& E = *eng_;
    return E.decode_path_ == 0 && E.batch_persistent_ && E.tp_ == 1 && E.cfg_.layers <= kMaxLayers && E.H_ % kPersistKAlign == 0 &&
           E.Hl_ % kPersistKAlign == 0 && E.Fl_ % kPersistKAlign == 0 && E.H_ <= kBatchPersistMaxK &&
           E.Hl_ <= kBatchPersistMaxK && E.Fl_ <= kBatchPersistMaxK && persist_attn_ctas_per_head(E.T_) <= 32 &&
           persist_max_contrib(E.H_, E.Hl_, E.num_sms_) <= kPersistMaxContrib &&
           persist_max_contrib(E.H_, E.Fl_, E.num_sms_) <= kPersistMaxContrib;
}

// One step as a single cooperative launch (after the step inputs): every
// weight box is streamed once and dotted with all kBatch sequences' inputs.
int BatchDecoder::enqueue_persistent(cudaStream_t s, bool sampled) {
    Engine& E = *eng_;
    BatchPersistParams bp{};
    PersistentParams& p = bp.base;
    for (int l = 0; l < E.cfg_.layers; ++l) {
        const LayerWeights& L = E.layers_[l];
        p.layer[l] = LayerPtrs{L.wqkv, L.bqkv, L.wo, L.bo, L.w13, L.b13, L.w2, L.b2, L.g1, L.g2, L.kc, L.vc};
        XB_CUDA(make_stream_map(&p.maps[4 * l + 0], L.wqkv, 3 * E.Hl_, E.H_));
        XB_CUDA(make_stream_map(&p.maps[4 * l + 1], L.wo, E.H_, E.Hl_));
        XB_CUDA(make_stream_map(&p.maps[4 * l + 2], L.w13, 2 * E.Fl_, E.H_));
        XB_CUDA(make_stream_map(&p.maps[4 * l + 3], L.w2, E.H_, E.Fl_));
        bp.kc[l] = kc_[l];
        bp.vc[l] = vc_[l];
    }
    XB_CUDA(make_stream_map(&p.maps[kPersistMaps - 1], E.emb_, E.V_, E.H_));
    p.layers = E.cfg_.layers;
    p.emb = E.emb_;
    p.gnorm = E.gnorm_;
    p.rope = E.rope_;
    p.st = st_;
    p.done = done_;
    p.trace = E.trace_;  // the engine's phase_trace option, when on before the decoder was created
    p.inflight = std::min(E.inflight_, 3);
    p.tma_evict_first = E.tma_evict_first_;
    p.H = E.H_;
    p.Hl = E.Hl_;
    p.heads = E.heads_l_;
    p.Fl = E.Fl_;
    p.V = E.V_;
    p.v0 = 0;
    p.T = E.T_;
    p.tp = 1;
    p.rank = 0;
    bp.xa = x_;
    bp.xb = xb_;
    bp.cres = cres_;
    bp.tickets = tick_;
    bp.qkv = qkv_;
    bp.att = att_;
    bp.ffh = ffh_;
    bp.logits = logits_;
    bp.rep = rep_;
    bp.st = st_;
    bp.part = part_;
    bp.done = done_;
    bp.head_done = done_ + 5 * E.cfg_.layers + 1;
    bp.finish_greedy = sampled ? 0 : 1;
    count_launch();
    batch_in_kernel<<<1, 32, 0, s>>>(in_, st_, tokens_);
    XB_CUDA(cudaGetLastError());
    XB_CUDA(cudaMemsetAsync(done_, 0, done_words() * sizeof(int), s));
    XB_CUDA(cudaMemsetAsync(tick_, 0, tick_words() * sizeof(int), s));
    XB_CUDA(launch_decode_batch_persistent(bp, E.num_sms_, s));
    if (!sampled) return XL_OK;  // the kernel wrote every sequence's greedy id
    SampleParams sp{};
    sp.logits = logits_;
    sp.V = E.V_;
    sp.v0 = 0;
    sp.st = st_;
    sp.rep_flags = rep_;
    sp.full = 0;
    sp.work = samp_work_;
    sp.work_stride = samp_stride_;
    sp.stride = E.V_;
    sp.grid = samp_grid_;
    XB_CUDA(launch_sample_chain(sp, kBatch, false, s));
    return XL_OK;
}

int BatchDecoder::enqueue(cudaStream_t s, bool sampled) {
    Engine& E = *eng_;
    if (persistent_fits()) return enqueue_persistent(s, sampled);
    const int H = E.H_, Hl = E.Hl_, Fl = E.Fl_, T = E.T_, V = E.V_, heads = E.heads_l_;
    count_launch();
    batch_in_kernel<<<1, 32, 0, s>>>(in_, st_, tokens_);
    XB_CUDA(cudaGetLastError());
    for (int l = 0; l < E.cfg_.layers; ++l) {
        const LayerWeights& W = E.layers_[l];
        BatchGemvParams q{};
        if (l == 0) {
            q.table = E.emb_;
            q.tokens = tokens_;
            q.x_out = x_;
        } else {
            q.x = x_;
        }
        q.ldx = H;
        q.gamma = W.g1;
        q.eps = 1e-6f;
        q.W = W.wqkv;
        q.bias = W.bqkv;
        q.y = qkv_;
        q.ldy = 3 * Hl;
        q.M = 3 * Hl;
        q.K = H;
        XB_CUDA(launch_batch_gemv(kGemvPlain, q, E.num_sms_, s));
        XB_CUDA(launch_pdl(batch_rope_kv_kernel, dim3(kBatch, heads), dim3(32), 0, s, qkv_,
                           static_cast<const float2*>(E.rope_), kc_[l], vc_[l], static_cast<const DevState*>(st_),
                           heads, T));
        XB_CUDA(launch_pdl(batch_attn_kernel, dim3(heads, kBatch), dim3(32 * kBaWarps), 0, s,
                           static_cast<const float*>(qkv_), static_cast<const float*>(kc_[l]),
                           static_cast<const float*>(vc_[l]), att_, static_cast<const DevState*>(st_), heads, T));
        BatchGemvParams o{};
        o.x = att_;
        o.ldx = Hl;
        o.W = W.wo;
        o.bias = W.bo;
        o.y = x_;
        o.ldy = H;
        o.M = H;
        o.K = Hl;
        XB_CUDA(launch_batch_gemv(kGemvResidual, o, E.num_sms_, s));
        BatchGemvParams f{};
        f.x = x_;
        f.ldx = H;
        f.gamma = W.g2;
        f.eps = 1e-6f;
        f.W = W.w13;
        f.bias = W.b13;
        f.y = ffh_;
        f.ldy = Fl;
        f.M = 2 * Fl;
        f.K = H;
        XB_CUDA(launch_batch_gemv(kGemvSwiGLU, f, E.num_sms_, s));
        BatchGemvParams d{};
        d.x = ffh_;
        d.ldx = Fl;
        d.W = W.w2;
        d.bias = W.b2;
        d.y = x_;
        d.ldy = H;
        d.M = H;
        d.K = Fl;
        XB_CUDA(launch_batch_gemv(kGemvResidual, d, E.num_sms_, s));
    }
    BatchGemvParams h{};
    h.x = x_;
    h.ldx = H;
    h.gamma = E.gnorm_;
    h.eps = 1e-6f;
    h.W = E.emb_;
    h.y = logits_;
    h.ldy = V;
    h.M = V;
    h.K = H;
    h.rep_flags = rep_;
    h.st = st_;
    h.ticket = ticket_;
    XB_CUDA(launch_batch_gemv(kGemvLogits, h, E.num_sms_, s));
    SampleParams sp{};
    sp.logits = logits_;
    sp.V = V;
    sp.v0 = 0;
    sp.st = st_;
    sp.rep_flags = rep_;
    sp.full = 0;
    sp.work = samp_work_;
    sp.work_stride = samp_stride_;
    sp.stride = V;
    sp.grid = samp_grid_;
    if (sampled) XB_CUDA(launch_sample_chain(sp, kBatch, true, s));
    else XB_CUDA(launch_sample_finish(sp, kBatch, true, s));
    return XL_OK;
}

int BatchDecoder::capture() {
    cudaStream_t s = eng_->stream_;
    for (int sampled = 0; sampled < 2; ++sampled) {
        cudaGraphExec_t& exec = sampled ? exec_s_ : exec_;
        long long& kernels = sampled ? graph_kernels_s_ : graph_kernels_;
        cudaGraph_t g = nullptr;
        XB_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        const long long recorded0 = launch_count();
        const int rc = enqueue(s, sampled != 0);
        kernels = launch_count() - recorded0;
        count_graph_kernels(-kernels);
        const cudaError_t ce = cudaStreamEndCapture(s, &g);
        if (rc != XL_OK) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamEndCapture");
        const cudaError_t ie = cudaGraphInstantiate(&exec, g, 0);
        cudaGraphDestroy(g);
        if (ie != cudaSuccess) return cuda_fail(ie, "cudaGraphInstantiate");
    }
    return XL_OK;
}

int BatchDecoder::seed(int seq, uint64_t s) {
    if (seq < 0 || seq >= kBatch) {
        set_error("batch decoder: sequence index out of range");
        return XL_ERR_ARG;
    }
    seed_[seq] = s;
    ctr_[seq] = 0;
    return XL_OK;
}

float BatchDecoder::next_uniform(int seq) { return philox_uniform(ctr_[seq]++, seed_[seq]); }

int BatchDecoder::prefill(int seq, const int* ids, int n, float temperature, float top_p, float rp, int* token_out) {
    if (seq < 0 || seq >= kBatch || token_out == nullptr) {
        set_error("batch decoder: sequence index out of range");
        return XL_ERR_ARG;
    }
    Engine& E = *eng_;
    XB_CUDA(cudaSetDevice(E.device_));
    const float u = next_uniform(seq);
    int rc = E.set_uniforms(&u, 1);
    if (rc != XL_OK) return rc;
    rc = E.prefill(ids, n, temperature, top_p, rp, token_out);
    if (rc != XL_OK) return rc;
    // The engine's cache rows [0, n), repetition flags and state become this sequence's.
    cudaStream_t s = E.stream_;
    const size_t row = static_cast<size_t>(E.T_) * kHeadDim * 4;
    for (int l = 0; l < E.cfg_.layers; ++l) {
        const size_t dst = static_cast<size_t>(seq) * E.heads_l_ * E.T_ * kHeadDim;
        XB_CUDA(cudaMemcpy2DAsync(kc_[l] + dst, row, E.layers_[l].kc, row, static_cast<size_t>(n) * kHeadDim * 4,
                                  E.heads_l_, cudaMemcpyDeviceToDevice, s));
        XB_CUDA(cudaMemcpy2DAsync(vc_[l] + dst, row, E.layers_[l].vc, row, static_cast<size_t>(n) * kHeadDim * 4,
                                  E.heads_l_, cudaMemcpyDeviceToDevice, s));
    }
    XB_CUDA(cudaMemcpyAsync(rep_ + static_cast<size_t>(seq) * E.V_, E.rep_flags_, E.V_, cudaMemcpyDeviceToDevice, s));
    XB_CUDA(cudaMemcpyAsync(st_ + seq, E.st_, sizeof(DevState), cudaMemcpyDeviceToDevice, s));
    XB_CUDA(cudaStreamSynchronize(s));
    n_[seq] = n;
    return XL_OK;
}

int BatchDecoder::decode(const int* tokens, float temperature, float top_p, float rp, int* tokens_out) {
    if (tokens == nullptr || tokens_out == nullptr) {
        set_error("batch decoder: null argument");
        return XL_ERR_ARG;
    }
    Engine& E = *eng_;
    XB_CUDA(cudaSetDevice(E.device_));
    for (int b = 0; b < kBatch; ++b) {
        if (n_[b] < 0) {
            set_error("batch decoder: sequence " + std::to_string(b) + " has no prompt (prefill it first)");
            return XL_ERR_STATE;
        }
        if (n_[b] >= E.T_) {
            set_error("batch decoder: KV cache of sequence " + std::to_string(b) + " is full");
            return XL_ERR_CTX;
        }
        if (tokens[b] < 0 || tokens[b] >= E.V_) {
            set_error("Embedding : Invalid token: " + std::to_string(tokens[b]));
            return XL_ERR_TOKEN;
        }
    }
    for (int b = 0; b < kBatch; ++b) {
        StepIn& in = h_in_[b];
        std::memset(&in, 0, sizeof(StepIn));
        in.token_in = tokens[b];
        in.temperature = temperature;
        in.top_p = top_p;
        in.rp = rp;
        in.uniform = next_uniform(b);
        in.decode_mode = 1;
    }
    cudaStream_t s = E.stream_;
    XB_CUDA(cudaMemcpyAsync(in_, h_in_, kBatch * sizeof(StepIn), cudaMemcpyHostToDevice, s));
    XB_CUDA(cudaEventRecord(ev0_, s));
    const bool sampled = top_p > 0.0f;
    XB_CUDA(cudaGraphLaunch(sampled ? exec_s_ : exec_, s));
    count_graph_kernels(sampled ? graph_kernels_s_ : graph_kernels_);
    XB_CUDA(cudaEventRecord(ev1_, s));
    XB_CUDA(cudaMemcpyAsync(h_st_, st_, kBatch * sizeof(DevState), cudaMemcpyDeviceToHost, s));
    XB_CUDA(cudaStreamSynchronize(s));
    XB_CUDA(cudaEventElapsedTime(&last_ms_, ev0_, ev1_));
    for (int b = 0; b < kBatch; ++b) {
        if (h_st_[b].err != 0) {
            set_error("device error word " + std::to_string(h_st_[b].err));
            return XL_ERR_DEVICE;
        }
        tokens_out[b] = h_st_[b].token_out;
        n_[b] += 1;
    }
    return XL_OK;
}

int BatchDecoder::last_logits(int seq, float* out, int n) {
    if (seq < 0 || seq >= kBatch || out == nullptr || n < eng_->V_) {
        set_error("batch decoder: bad logits request");
        return XL_ERR_ARG;
    }
    XB_CUDA(cudaSetDevice(eng_->device_));
    XB_CUDA(cudaMemcpy(out, logits_ + static_cast<size_t>(seq) * eng_->V_, eng_->V_ * sizeof(float),
                       cudaMemcpyDeviceToHost));
    return XL_OK;
}

}  // namespace xl
