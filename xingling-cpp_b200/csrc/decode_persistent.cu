// Persistent decode-step kernel for sm_100a: one launch per token.
//
// One CTA per SM (cooperative launch, so every CTA is resident).  Warp 0 is a
// producer: one lane streams every weight tile this CTA needs for the whole
// token (16 x [QKV, out-proj, W1/V, W2] and the tied LM head) from HBM into a
// shared-memory ring with cp.async.bulk (TMA engine), gated only by free ring
// slots.  Warps 1..8 consume: per phase they wait for the previous phase of
// every CTA (a global counter), stage the phase's input vector in shared
// memory (residual update, RMSNorm, attention combine or SwiGLU input), take
// ring tiles, reduce with warp shuffles and apply the epilogue.  Because the
// producer never waits on activations, HBM keeps streaming across phase
// boundaries; the only per-phase cost is the consumers' barrier latency,
// hidden behind the ring.
//
// Replaces, for one decode token, the reference's Transformer::forward(int)
// (src/transformer.cu:180-186) with TransformerBlock::forward
// (src/transformer.cu:68-105), AttentionBlock::forward decode branch
// (src/attn.cu:648-664), MultiHeadAttention::forward (src/attn.cu:372-447,
// 490-547), SwishGLU::forward_vec (src/ffn.cu:126-139), Linear::forward_vec
// (src/linear.cu:260-282) and Embedding::inverse (src/embedding.cu:130-205).
//
// Every wait is bounded: a timed-out wait sets a bit in DevState::err, makes
// the other CTAs leave at their next wait, and the producer drains its
// in-flight copies before returning.
#include <math.h>

#include "xl_device.cuh"
#include "xl_kernels.h"

namespace xl {

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = 32 * kConsumerWarps;
constexpr int kThreads = kConsumerThreads + 32;
constexpr int kTileRows = 2 * kConsumerWarps;   // each consumer warp owns two rows of a tile
constexpr int kTileK = 384;                     // floats of a row per tile
constexpr int kSlotBytes = kTileRows * kTileK * 4;  // 24 KB
constexpr int kSlots = 8;                       // 192 KB ring
constexpr int kMaxK = 4096;
constexpr size_t kSmemBytes =
    static_cast<size_t>(kSlots) * kSlotBytes + kMaxK * 4 + 2 * kSlots * 8 + 256 + kConsumerWarps * 64 * 4;
constexpr uint32_t kMbarSpinLimit = 1u << 24;
constexpr uint32_t kFlagSpinLimit = 1u << 23;
constexpr int kErrMbar = 1, kErrFlag = 2;

enum PhaseKind : int { kQKV = 0, kAttn = 1, kWo = 2, kW13 = 3, kW2 = 4, kLM = 5 };

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Global -> shared bulk copy (no multicast) completing on a CTA-local mbarrier.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumerThreads) : "memory"); }
__device__ __forceinline__ int ld_acquire(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ bool aborted(const DevState* st) { return *reinterpret_cast<const volatile int*>(&st->err); }

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// Optional phase timeline: trace[(cta * phases + ph) * kTraceFields + field] (ns).
enum TraceField : int { kTrConsStart = 0, kTrConsStaged = 1, kTrConsEnd = 2, kTrProdFirst = 3, kTrProdLast = 4 };
__device__ __forceinline__ void trace_at(const PersistentParams& p, int ph, int field) {
    if (p.trace) p.trace[(static_cast<size_t>(blockIdx.x) * (5 * p.layers + 1) + ph) * kTraceFields + field] = globaltimer();
}

// Bounded wait on an mbarrier phase; false (and the error bit) on timeout or abort.
__device__ bool wait_parity(uint64_t* bar, uint32_t parity, DevState* st) {
    uint32_t it = 0;
    while (!mbar_try_wait(bar, parity)) {
        if (++it >= kMbarSpinLimit || ((it & 1023u) == 0 && aborted(st))) {
            atomicOr(&st->err, kErrMbar);
            return false;
        }
    }
    return true;
}

struct Gemv {
    const float* W;
    const float* bias;
    int M, K, kind;
};

__device__ __forceinline__ int phase_kind(int ph, int L) { return ph == 5 * L ? kLM : ph % 5; }

__device__ __forceinline__ Gemv gemv_of(const PersistentParams& p, int ph) {
    Gemv g{};
    const int L = p.layers;
    if (ph == 5 * L) {
        g.W = p.emb;
        g.bias = nullptr;
        g.M = p.V;
        g.K = p.H;
        g.kind = kLM;
        return g;
    }
    const LayerPtrs& y = p.layer[ph / 5];
    g.kind = ph % 5;
    switch (g.kind) {
        case kQKV:
            g.W = y.wqkv, g.bias = y.bqkv, g.M = 3 * p.Hl, g.K = p.H;
            break;
        case kWo:
            g.W = y.wo, g.bias = y.bo, g.M = p.H, g.K = p.Hl;
            break;
        case kW13:
            g.W = y.w13, g.bias = y.b13, g.M = 2 * p.Fl, g.K = p.H;
            break;
        case kW2:
            g.W = y.w2, g.bias = y.b2, g.M = p.H, g.K = p.Fl;
            break;
        default:
            break;
    }
    return g;
}

// This CTA's row groups (16 rows each) of an M-row matrix: a balanced split.
__device__ __forceinline__ void my_groups(int M, int& g0, int& g1) {
    const int groups = (M + kTileRows - 1) / kTileRows;
    g0 = static_cast<int>((static_cast<long long>(blockIdx.x) * groups) / gridDim.x);
    g1 = static_cast<int>((static_cast<long long>(blockIdx.x + 1) * groups) / gridDim.x);
}

// ---------------------------------------------------------------------------
// Producer: the whole token's weight stream for this CTA.
//
// A unit is one 16-row group of one GEMV phase; its rows are contiguous in
// HBM.  Besides the ring copies, the producer keeps an L2 prefetch cursor
// kPrefetchUnits units ahead, so that HBM keeps streaming into L2 while the
// ring is full (consumers waiting at a phase boundary or in attention); the
// ring copies then hit L2.
constexpr int kPrefetchUnits = 4;
constexpr uint32_t kPrefetchPiece = 32768;

struct Unit {
    int ph, g, g1;
};

// First unit at or after phase ph (ph beyond the schedule: none).
__device__ bool unit_first(const PersistentParams& p, int ph, Unit& u) {
    const int last = 5 * p.layers;
    for (; ph <= last; ++ph) {
        if (phase_kind(ph, p.layers) == kAttn) continue;
        int g0, g1;
        my_groups(gemv_of(p, ph).M, g0, g1);
        if (g0 < g1) {
            u = Unit{ph, g0, g1};
            return true;
        }
    }
    return false;
}

__device__ bool unit_next(const PersistentParams& p, Unit& u) {
    if (++u.g < u.g1) return true;
    return unit_first(p, u.ph + 1, u);
}

__device__ __forceinline__ int cu_first_group(const PersistentParams& p, const Unit& u) {
    int g0, g1;
    my_groups(gemv_of(p, u.ph).M, g0, g1);
    return g0;
}

__device__ void prefetch_unit(const PersistentParams& p, const Unit& u) {
    const Gemv d = gemv_of(p, u.ph);
    const int rows = min(kTileRows, d.M - u.g * kTileRows);
    const char* src = reinterpret_cast<const char*>(d.W + static_cast<size_t>(u.g) * kTileRows * d.K);
    uint32_t bytes = static_cast<uint32_t>(rows) * d.K * 4;
    for (uint32_t off = 0; off < bytes; off += kPrefetchPiece)
        prefetch_l2_bulk(src + off, min(kPrefetchPiece, bytes - off));
}

__device__ void producer(const PersistentParams& p, char* ring, uint64_t* full, uint64_t* empty) {
    DevState* st = p.st;
    int slot = 0;
    uint32_t par = 0;
    int issued = 0;
    bool ok = true;
    Unit cu, pu;
    bool have = unit_first(p, 0, cu);
    bool pf = unit_first(p, 0, pu);
    for (int i = 0; i < kPrefetchUnits && pf; ++i) {
        prefetch_unit(p, pu);
        pf = unit_next(p, pu);
    }
    for (; have && ok; have = unit_next(p, cu)) {
        if (pf) {
            prefetch_unit(p, pu);
            pf = unit_next(p, pu);
        }
        const Gemv d = gemv_of(p, cu.ph);
        const int nkt = (d.K + kTileK - 1) / kTileK;
        const int g = cu.g;
        if (g == cu_first_group(p, cu)) trace_at(p, cu.ph, kTrProdFirst);
        {
            const int rows = min(kTileRows, d.M - g * kTileRows);
            for (int kt = 0; kt < nkt; ++kt) {
                if (!wait_parity(&empty[slot], par ^ 1u, st)) {
                    ok = false;
                    break;
                }
                const int k0 = kt * kTileK;
                const int kc = min(kTileK, d.K - k0);
                mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(rows * kc * 4));
                char* dst = ring + static_cast<size_t>(slot) * kSlotBytes;
                const float* src = d.W + static_cast<size_t>(g) * kTileRows * d.K + k0;
                for (int r = 0; r < rows; ++r)
                    bulk_g2s(dst + r * kTileK * 4, src + static_cast<size_t>(r) * d.K, static_cast<uint32_t>(kc * 4),
                             &full[slot]);
                ++issued;
                if (++slot == kSlots) {
                    slot = 0;
                    par ^= 1u;
                }
            }
        }
        if (g + 1 == cu.g1) trace_at(p, cu.ph, kTrProdLast);
    }
    if (!ok) {
        // Drain: every copy already issued must land before this CTA exits.
        const int pending = issued < kSlots ? issued : kSlots;
        for (int i = 1; i <= pending; ++i) {
            const int k = issued - i;  // tile index k went to slot k % kSlots with parity (k / kSlots) & 1
            const int s = k % kSlots;
            const uint32_t pp = static_cast<uint32_t>((k / kSlots) & 1);
            uint32_t it = 0;
            while (!mbar_try_wait(&full[s], pp) && ++it < kMbarSpinLimit) {
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Consumer helpers (256 threads, named barrier 1).

// Wait until every CTA finished phase ph (counter == gridDim.x).
__device__ bool wait_phase(const PersistentParams& p, int ph) {
    __shared__ int s_ok;
    if (threadIdx.x == 32) {
        const int* c = p.done + ph;
        uint32_t it = 0;
        int ok = 1;
        while (ld_acquire(c) < static_cast<int>(gridDim.x)) {
            if (++it >= kFlagSpinLimit || ((it & 255u) == 0 && aborted(p.st))) {
                atomicOr(&p.st->err, kErrFlag);
                ok = 0;
                break;
            }
            __nanosleep(32);
        }
        __threadfence();
        s_ok = ok;
    }
    consumer_sync();
    return s_ok != 0;
}

__device__ void signal_phase(const PersistentParams& p, int ph) {
    consumer_sync();
    if (threadIdx.x == 32) {
        __threadfence();
        atomicAdd(p.done + ph, 1);
    }
}

// Block-wide (consumers) sum of one float per thread.
__device__ float consumer_sum(float v, float* red) {
    const int t = threadIdx.x - 32;
    v = warp_sum(v);
    if ((t & 31) == 0) red[t >> 5] = v;
    consumer_sync();
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) s += red[w];
    consumer_sync();
    return s;
}

// xs = rmsnorm(src) * gamma (src read through L2); optionally store src to x_out.
__device__ void stage_norm(const float* src, const float* gamma, int K, float* xs, float* red, float* x_out) {
    const int t = threadIdx.x - 32;
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4* x4 = reinterpret_cast<float4*>(xs);
    float ss = 0.0f;
    for (int i = t; i < (K >> 2); i += kConsumerThreads) {
        const float4 v = __ldcg(s4 + i);
        x4[i] = v;
        if (x_out) reinterpret_cast<float4*>(x_out)[i] = v;
        ss = dot4(v, v, ss);
    }
    const float tot = consumer_sum(ss, red);
    // RMSNorm of src/rmsnorm.cu:99-101: 1 / sqrt(mean + 1e-6), in double.
    const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(tot / static_cast<float>(K)) + 1e-6));
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
    for (int i = t; i < (K >> 2); i += kConsumerThreads) {
        float4 v = x4[i];
        const float4 g = g4[i];
        v.x = v.x * inv * g.x;
        v.y = v.y * inv * g.y;
        v.z = v.z * inv * g.z;
        v.w = v.w * inv * g.w;
        x4[i] = v;
    }
}

__device__ void stage_copy(const float* src, int K, float* xs) {
    const int t = threadIdx.x - 32;
    for (int i = t; i < (K >> 2); i += kConsumerThreads)
        reinterpret_cast<float4*>(xs)[i] = __ldcg(reinterpret_cast<const float4*>(src) + i);
}

// Merge the split-K attention partials (m, l, o[64]) of every head into xs.
__device__ void stage_attn_combine(const PersistentParams& p, int nsplit, float* xs) {
    const int t = threadIdx.x - 32;
    const int maxs = persistent_max_splits(p.T);
    for (int i = t; i < p.Hl; i += kConsumerThreads) {
        const int h = i >> 6, d = i & 63;
        const float* base = p.part + static_cast<size_t>(h) * maxs * (kHeadDim + 2);
        if (nsplit == 1) {
            xs[i] = __ldcg(base + 2 + d) / __ldcg(base + 1);
            continue;
        }
        float M = -INFINITY;
        for (int s = 0; s < nsplit; ++s) M = fmaxf(M, __ldcg(base + s * (kHeadDim + 2)));
        float Ls = 0.0f, O = 0.0f;
        for (int s = 0; s < nsplit; ++s) {
            const float* ps = base + s * (kHeadDim + 2);
            const float w = expf(__ldcg(ps) - M);
            Ls = fmaf(__ldcg(ps + 1), w, Ls);
            O = fmaf(__ldcg(ps + 2 + d), w, O);
        }
        xs[i] = O / Ls;
    }
}

// One (head, 32-position chunk) of the decode attention on one warp, lane j
// owning position t0 + j: RoPE at position n (src/rope.cu:20-45), KV append
// when the chunk holds n, scores, softmax and P.V; writes the (max, sum, o)
// partial.  All 16 K-row loads of a lane are in flight together.
__device__ void attend_chunk(const PersistentParams& p, const LayerPtrs& y, int h, int s, int n, float* qsh) {
    const int lane = threadIdx.x & 31;
    const int t0 = s * kPersistChunk;
    const int cnt = min(kPersistChunk, n + 1 - t0);
    const float* q = p.qkv + h * kHeadDim;
    const float* kn = p.qkv + p.Hl + h * kHeadDim;
    const float* vn = p.qkv + 2 * p.Hl + h * kHeadDim;
    float* kc = y.kc + static_cast<size_t>(h) * p.T * kHeadDim;
    float* vc = y.vc + static_cast<size_t>(h) * p.T * kHeadDim;
    const float2 cs = p.rope[n * kHalfHead + lane];
    const float qa = __ldcg(q + lane), qb = __ldcg(q + lane + kHalfHead);
    qsh[lane] = (qa * cs.x + qb * cs.y) * 0.125f;  // 1/sqrt(64) is exact
    qsh[lane + kHalfHead] = (-qa * cs.y + qb * cs.x) * 0.125f;
    if (n >= t0 && n < t0 + cnt) {
        const float ka = __ldcg(kn + lane), kb = __ldcg(kn + lane + kHalfHead);
        kc[n * kHeadDim + lane] = ka * cs.x + kb * cs.y;
        kc[n * kHeadDim + lane + kHalfHead] = -ka * cs.y + kb * cs.x;
        vc[n * kHeadDim + lane] = __ldcg(vn + lane);
        vc[n * kHeadDim + lane + kHalfHead] = __ldcg(vn + lane + kHalfHead);
    }
    __syncwarp();
    float sc = -INFINITY;
    if (lane < cnt) {
        const float4* kr = reinterpret_cast<const float4*>(kc + static_cast<size_t>(t0 + lane) * kHeadDim);
        float4 kv[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) kv[i] = __ldcg(kr + i);
        const float4* q4 = reinterpret_cast<const float4*>(qsh);
        float d = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) d = dot4(kv[i], q4[i], d);
        sc = d;
    }
    const float m = warp_max(sc);
    const float e = lane < cnt ? expf(sc - m) : 0.0f;
    const float l = warp_sum(e);
    float oa = 0.0f, ob = 0.0f;
#pragma unroll 8
    for (int j = 0; j < cnt; ++j) {
        const float pj = __shfl_sync(0xffffffffu, e, j);
        const float* vr = vc + static_cast<size_t>(t0 + j) * kHeadDim;
        oa = fmaf(pj, __ldcg(vr + lane), oa);
        ob = fmaf(pj, __ldcg(vr + lane + kHalfHead), ob);
    }
    float* pp = p.part + (static_cast<size_t>(h) * persistent_max_splits(p.T) + s) * (kHeadDim + 2);
    pp[2 + lane] = oa;
    pp[2 + lane + kHalfHead] = ob;
    if (lane == 0) {
        pp[0] = m;
        pp[1] = l;
    }
    __syncwarp();
}

__device__ void consumers(const PersistentParams& p, char* ring, float* xs, uint64_t* full, uint64_t* empty,
                          float* red, unsigned long long* best_s, float* qbuf) {
    DevState* st = p.st;
    const int t = threadIdx.x - 32;
    const int warp = t >> 5, lane = t & 31;
    const int n = st->pos;
    const int nsplit = (n + kPersistChunk) / kPersistChunk;  // chunks of positions 0..n
    const float rp = st->in.rp;
    int slot = 0;
    uint32_t par = 0;
    float best_v = -INFINITY;
    int best_i = -1;
    bool ok = true;
    const int last = 5 * p.layers;
    for (int ph = 0; ph <= last; ++ph) {
        if (ph > 0 && !wait_phase(p, ph - 1)) return;
        if (t == 0) trace_at(p, ph, kTrConsStart);
        const int kind = phase_kind(ph, p.layers);
        const LayerPtrs* y = ph < last ? &p.layer[ph / 5] : nullptr;
        if (kind == kAttn) {
            const int items = p.heads * nsplit;
            for (int it = blockIdx.x + gridDim.x * warp; it < items; it += gridDim.x * kConsumerWarps)
                attend_chunk(p, *y, it / nsplit, it % nsplit, n, qbuf + warp * kHeadDim);
            if (t == 0) trace_at(p, ph, kTrConsStaged);
            signal_phase(p, ph);
            if (t == 0) trace_at(p, ph, kTrConsEnd);
            continue;
        }
        const Gemv d = gemv_of(p, ph);
        // stage this phase's input vector
        if (kind == kQKV) {
            if (ph == 0) {
                const float* row = p.emb + static_cast<size_t>(st->in.token_in) * p.H;
                stage_norm(row, y->g1, p.H, xs, red, blockIdx.x == 0 ? p.x : nullptr);
            } else {
                stage_norm(p.x, y->g1, p.H, xs, red, nullptr);
            }
        } else if (kind == kWo) {
            stage_attn_combine(p, nsplit, xs);
        } else if (kind == kW13) {
            stage_norm(p.x, y->g2, p.H, xs, red, nullptr);
        } else if (kind == kW2) {
            stage_copy(p.ffh, p.Fl, xs);
        } else {  // kLM
            stage_norm(p.x, p.gnorm, p.H, xs, red, nullptr);
        }
        consumer_sync();
        if (t == 0) trace_at(p, ph, kTrConsStaged);
        int g0, g1;
        my_groups(d.M, g0, g1);
        const int nkt = (d.K + kTileK - 1) / kTileK;
        const float4* x4 = reinterpret_cast<const float4*>(xs);
        for (int g = g0; g < g1; ++g) {
            const int rows = min(kTileRows, d.M - g * kTileRows);
            const int ra = 2 * warp, rb = 2 * warp + 1;
            const bool va = ra < rows, vb = rb < rows;
            float acc_a = 0.0f, acc_b = 0.0f;
            for (int kt = 0; kt < nkt; ++kt) {
                // After a failed wait this warp only walks the schedule so that it
                // meets the other consumer warps at every named barrier.
                if (ok && !wait_parity(&full[slot], par, st)) ok = false;
                if (!ok) {
                    if (++slot == kSlots) {
                        slot = 0;
                        par ^= 1u;
                    }
                    continue;
                }
                const int k0 = kt * kTileK;
                const int kc4 = min(kTileK, d.K - k0) >> 2;
                const float4* tile = reinterpret_cast<const float4*>(ring + static_cast<size_t>(slot) * kSlotBytes);
                const float4* wa = tile + ra * (kTileK / 4);
                const float4* wb = tile + rb * (kTileK / 4);
                const float4* xk = x4 + (k0 >> 2);
#pragma unroll
                for (int j0 = 0; j0 < kTileK / 4; j0 += 32) {
                    const int j = j0 + lane;
                    if (j < kc4) {
                        const float4 xv = xk[j];
                        if (va) acc_a = dot4(wa[j], xv, acc_a);
                        if (vb) acc_b = dot4(wb[j], xv, acc_b);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
                if (++slot == kSlots) {
                    slot = 0;
                    par ^= 1u;
                }
            }
            acc_a = warp_sum(acc_a);
            acc_b = warp_sum(acc_b);
            const int Ra = g * kTileRows + ra, Rb = Ra + 1;
            switch (kind) {
                case kQKV:
                    if (lane == 0 && va) p.qkv[Ra] = acc_a + d.bias[Ra];
                    if (lane == 1 && vb) p.qkv[Rb] = acc_b + d.bias[Rb];
                    break;
                case kWo:
                case kW2:
                    if (lane == 0 && va) p.x[Ra] = __ldcg(p.x + Ra) + (acc_a + d.bias[Ra]);
                    if (lane == 1 && vb) p.x[Rb] = __ldcg(p.x + Rb) + (acc_b + d.bias[Rb]);
                    break;
                case kW13:
                    if (lane == 0 && vb) p.ffh[Ra >> 1] = silu(acc_a + d.bias[Ra]) * (acc_b + d.bias[Rb]);
                    break;
                default: {  // kLM: logits with the repetition penalty, running argmax
                    if (va) {
                        float v = acc_a;
                        if (p.rep_flags[Ra]) v = rep_penalty(v, rp);
                        if (lane == 0) p.logits[Ra] = v;
                        if (v > best_v) best_v = v, best_i = Ra;
                    }
                    if (vb) {
                        float v = acc_b;
                        if (p.rep_flags[Rb]) v = rep_penalty(v, rp);
                        if (lane == 1) p.logits[Rb] = v;
                        if (v > best_v) best_v = v, best_i = Rb;
                    }
                }
            }
        }
        if (kind != kLM) signal_phase(p, ph);
        if (t == 0) trace_at(p, ph, kTrConsEnd);
    }
    // LM head: CTA argmax -> global max; the last CTA publishes the winner.
    if (lane == 0) best_s[warp] = best_i >= 0 ? pack_argmax(best_v, best_i) : 0ull;
    consumer_sync();
    if (t == 0) {
        unsigned long long k = 0;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) k = best_s[w] > k ? best_s[w] : k;
        if (k) atomicMax(&st->argmax_key, k);
        __threadfence();
        const int ticket = atomicAdd(p.done + last, 1);
        if (ticket == static_cast<int>(gridDim.x) - 1) {
            __threadfence();
            const unsigned long long fin = atomicExch(&st->argmax_key, 0ull);
            st->argmax_final = fin;
            st->greedy_token = unpack_argmax_index(fin);
        }
    }
}

__global__ void __launch_bounds__(kThreads, 1) decode_persistent_kernel(const __grid_constant__ PersistentParams p) {
    extern __shared__ __align__(128) char smem[];
    char* ring = smem;
    float* xs = reinterpret_cast<float*>(smem + static_cast<size_t>(kSlots) * kSlotBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(xs + kMaxK);
    uint64_t* empty = full + kSlots;
    float* red = reinterpret_cast<float*>(empty + kSlots);
    unsigned long long* best_s = reinterpret_cast<unsigned long long*>(red + 16);
    float* qbuf = reinterpret_cast<float*>(best_s + kConsumerWarps + 8);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x < 32) {
        if (threadIdx.x == 0) producer(p, ring, full, empty);
    } else {
        consumers(p, ring, xs, full, empty, red, best_s, qbuf);
    }
}

}  // namespace

size_t persistent_smem_bytes() { return kSmemBytes; }

cudaError_t launch_decode_persistent(const PersistentParams& p, int num_sms, cudaStream_t s) {
    if (p.H > kMaxK || p.Hl > kMaxK || p.Fl > kMaxK || p.H % 4 || p.Hl % 4 || p.Fl % 4) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(decode_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_persistent_kernel, p);
}

}  // namespace xl
