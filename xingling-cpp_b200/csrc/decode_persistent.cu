// Persistent decode-step kernel for sm_100a: one launch per token.
//
// One CTA per SM (cooperative launch, so every CTA is resident).  Warp 0 is a
// producer: one lane streams every weight tile this CTA needs for the whole
// token (16 x [QKV, out-proj, W1/V, W2] and the tied LM head) from HBM into a
// shared-memory ring with 2D TMA tile loads (cp.async.bulk.tensor, one 16 KB
// [16 rows][256 floats] box per instruction), gated only by free ring slots,
// and keeps an L2 bulk-prefetch cursor a few row groups ahead.  Warps 1..8
// consume: per phase they wait for the previous phase of every CTA (a global
// counter), stage the phase's input vector in shared memory (embedding
// gather, residual stream, RMSNorm, attention combine or SwiGLU input), take
// ring tiles (two rows per warp), reduce with warp shuffles and apply the
// epilogue, whose operands (bias, residual, repetition flags) are loaded
// before the unit's tiles so their latency overlaps the stream.  Because the
// producer never waits on activations, HBM keeps streaming across phase
// boundaries.
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
constexpr int kSlotBytes = kPersistTileRows * kPersistTileK * 4;  // 16 KB
constexpr int kSlots = 12;                                       // 192 KB ring
constexpr int kMaxK = 4096;
constexpr size_t kSmemBytes =
    static_cast<size_t>(kSlots) * kSlotBytes + kMaxK * 4 + 2 * kSlots * 8 + 512 + kConsumerWarps * 64 * 4;
constexpr uint32_t kMbarSpinLimit = 1u << 24;
constexpr uint32_t kFlagSpinLimit = 1u << 24;
constexpr int kErrMbar = 1, kErrFlag = 2;
constexpr uint32_t kPrefetchPiece = 32768;

static_assert(kPersistTileRows == 2 * kConsumerWarps, "each consumer warp owns two rows of a tile");

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
// 2D TMA tile load (no multicast) of one [16 rows][256 floats] box at (x, y).
__device__ __forceinline__ void tma_tile(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
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
    const CUtensorMap* map;
    int M, K, kind;
};

__device__ __forceinline__ int phase_kind(int ph, int L) { return ph == 5 * L ? kLM : ph % 5; }

__device__ __forceinline__ Gemv gemv_of(const PersistentParams& p, int ph) {
    Gemv g{};
    const int L = p.layers;
    if (ph == 5 * L) {
        g.W = p.emb, g.bias = nullptr, g.map = &p.maps[kPersistMaps - 1], g.M = p.V, g.K = p.H, g.kind = kLM;
        return g;
    }
    const int l = ph / 5;
    const LayerPtrs& y = p.layer[l];
    g.kind = ph % 5;
    switch (g.kind) {
        case kQKV:
            g.W = y.wqkv, g.bias = y.bqkv, g.map = &p.maps[4 * l + 0], g.M = 3 * p.Hl, g.K = p.H;
            break;
        case kWo:
            g.W = y.wo, g.bias = y.bo, g.map = &p.maps[4 * l + 1], g.M = p.H, g.K = p.Hl;
            break;
        case kW13:
            g.W = y.w13, g.bias = y.b13, g.map = &p.maps[4 * l + 2], g.M = 2 * p.Fl, g.K = p.H;
            break;
        case kW2:
            g.W = y.w2, g.bias = y.b2, g.map = &p.maps[4 * l + 3], g.M = p.H, g.K = p.Fl;
            break;
        default:
            break;
    }
    return g;
}

// This CTA's row groups (16 rows each) of an M-row matrix: a balanced split.
__device__ __forceinline__ void my_groups(int M, int& g0, int& g1) {
    const int groups = (M + kPersistTileRows - 1) / kPersistTileRows;
    g0 = static_cast<int>((static_cast<long long>(blockIdx.x) * groups) / gridDim.x);
    g1 = static_cast<int>((static_cast<long long>(blockIdx.x + 1) * groups) / gridDim.x);
}

// ---------------------------------------------------------------------------
// Producer.  A unit is one 16-row group of one GEMV phase; its rows are
// contiguous in HBM, which the L2 prefetch cursor (p.prefetch_units units
// ahead of the ring copies, 0 = off) uses.
struct Unit {
    int ph, g, g0, g1;
};

__device__ bool unit_first(const PersistentParams& p, int ph, Unit& u) {
    const int last = 5 * p.layers;
    for (; ph <= last; ++ph) {
        if (phase_kind(ph, p.layers) == kAttn) continue;
        int g0, g1;
        my_groups(gemv_of(p, ph).M, g0, g1);
        if (g0 < g1) {
            u = Unit{ph, g0, g0, g1};
            return true;
        }
    }
    return false;
}

__device__ bool unit_next(const PersistentParams& p, Unit& u) {
    if (++u.g < u.g1) return true;
    return unit_first(p, u.ph + 1, u);
}

__device__ void prefetch_unit(const PersistentParams& p, const Unit& u) {
    const Gemv d = gemv_of(p, u.ph);
    const int rows = min(kPersistTileRows, d.M - u.g * kPersistTileRows);
    const char* src = reinterpret_cast<const char*>(d.W + static_cast<size_t>(u.g) * kPersistTileRows * d.K);
    const uint32_t bytes = static_cast<uint32_t>(rows) * d.K * 4;
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
    for (int i = 0; i < p.prefetch_units && pf; ++i) {
        prefetch_unit(p, pu);
        pf = unit_next(p, pu);
    }
    for (; have && ok; have = unit_next(p, cu)) {
        if (pf && p.prefetch_units > 0) {
            prefetch_unit(p, pu);
            pf = unit_next(p, pu);
        }
        const Gemv d = gemv_of(p, cu.ph);
        const int nkt = (d.K + kPersistTileK - 1) / kPersistTileK;
        if (cu.g == cu.g0) trace_at(p, cu.ph, kTrProdFirst);
        for (int kt = 0; kt < nkt; ++kt) {
            if (!wait_parity(&empty[slot], par ^ 1u, st)) {
                ok = false;
                break;
            }
            // Rows past M and columns past K of the box are zero-filled by TMA and
            // still counted in the transaction bytes.
            mbar_arrive_expect_tx(&full[slot], kSlotBytes);
            tma_tile(ring + static_cast<size_t>(slot) * kSlotBytes, d.map, kt * kPersistTileK,
                     cu.g * kPersistTileRows, &full[slot]);
            ++issued;
            if (++slot == kSlots) {
                slot = 0;
                par ^= 1u;
            }
        }
        if (cu.g + 1 == cu.g1) trace_at(p, cu.ph, kTrProdLast);
    }
    if (!ok) {
        // Drain: every copy already issued must land before this CTA exits.
        const int pending = issued < kSlots ? issued : kSlots;
        for (int i = 1; i <= pending; ++i) {
            const int k = issued - i;  // tile k went to slot k % kSlots with parity (k / kSlots) & 1
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
__device__ bool wait_phase(const PersistentParams& p, int ph, int* s_ok) {
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
        }
        *s_ok = ok;
    }
    consumer_sync();
    return *s_ok != 0;
}

__device__ void signal_phase(const PersistentParams& p, int ph) {
    consumer_sync();
    if (threadIdx.x == 32) asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(p.done + ph) : "memory");
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
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
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

// Butterfly reduce-scatter of a 64-float vector held by every lane: afterwards
// lane l holds the warp-wide sums of elements 2l and 2l+1.
__device__ __forceinline__ float2 warp_reduce_scatter64(float (&v)[64]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int half = 32, off = 16; off > 0; half >>= 1, off >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
    return make_float2(v[0], v[1]);
}

// One (head, 32-position chunk) of the decode attention on one warp, lane j
// owning position t0 + j: RoPE at position n (src/rope.cu:20-45), KV append
// when the chunk holds n, scores, softmax and P.V.  Each lane's K and V rows
// (32 x 16 B loads) are in flight together.  With one chunk the warp writes the
// head's output; otherwise it writes its (max, sum, o) partial and the last
// chunk of the head to finish (a per-head ticket) merges the partials.
__device__ void attend_chunk(const PersistentParams& p, const LayerPtrs& y, int layer, int h, int s, int nsplit, int n,
                             float* qsh) {
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
    const bool mine = lane < cnt;
    const float4* kr = reinterpret_cast<const float4*>(kc + static_cast<size_t>(t0 + (mine ? lane : 0)) * kHeadDim);
    const float4* vr = reinterpret_cast<const float4*>(vc + static_cast<size_t>(t0 + (mine ? lane : 0)) * kHeadDim);
    float4 kv[16], vv[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) kv[i] = __ldcg(kr + i);
#pragma unroll
    for (int i = 0; i < 16; ++i) vv[i] = __ldcg(vr + i);
    const float4* q4 = reinterpret_cast<const float4*>(qsh);
    float d = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) d = dot4(kv[i], q4[i], d);
    const float sc = mine ? d : -INFINITY;
    const float m = warp_max(sc);
    const float e = mine ? expf(sc - m) : 0.0f;
    const float l = warp_sum(e);
    float w[64];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        w[4 * i + 0] = e * vv[i].x;
        w[4 * i + 1] = e * vv[i].y;
        w[4 * i + 2] = e * vv[i].z;
        w[4 * i + 3] = e * vv[i].w;
    }
    const float2 o = warp_reduce_scatter64(w);
    float2* out = reinterpret_cast<float2*>(p.att + h * kHeadDim);
    if (nsplit == 1) {
        out[lane] = make_float2(o.x / l, o.y / l);
        return;
    }
    const int maxs = persistent_max_splits(p.T);
    float* base = p.part + static_cast<size_t>(h) * maxs * (kHeadDim + 2);
    float* pp = base + s * (kHeadDim + 2);
    reinterpret_cast<float2*>(pp + 2)[lane] = o;
    if (lane == 0) {
        pp[0] = m;
        pp[1] = l;
    }
    __syncwarp();
    int ticket = 0;
    if (lane == 0) {
        __threadfence();
        ticket = atomicAdd(p.head_done + layer * p.heads + h, 1);
    }
    ticket = __shfl_sync(0xffffffffu, ticket, 0);
    if (ticket != nsplit - 1) return;
    __threadfence();
    // Merge: lane s holds split s's (max, sum); every lane its two output dims.
    const float ms = lane < nsplit ? __ldcg(base + lane * (kHeadDim + 2)) : -INFINITY;
    const float ls = lane < nsplit ? __ldcg(base + lane * (kHeadDim + 2) + 1) : 0.0f;
    const float M = warp_max(ms);
    const float ws = lane < nsplit ? expf(ms - M) : 0.0f;
    const float L = warp_sum(ls * ws);
    float2 acc = make_float2(0.0f, 0.0f);
    for (int k = 0; k < nsplit; ++k) {
        const float wk = __shfl_sync(0xffffffffu, ws, k);
        const float2 ok = __ldcg(reinterpret_cast<const float2*>(base + k * (kHeadDim + 2) + 2) + lane);
        acc.x = fmaf(wk, ok.x, acc.x);
        acc.y = fmaf(wk, ok.y, acc.y);
    }
    out[lane] = make_float2(acc.x / L, acc.y / L);
}

__device__ void consumers(const PersistentParams& p, char* ring, float* xs, uint64_t* full, uint64_t* empty,
                          float* red, unsigned long long* best_s, float* qbuf, int* s_ok) {
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
        if (ph > 0 && !wait_phase(p, ph - 1, s_ok)) return;
        if (t == 0) trace_at(p, ph, kTrConsStart);
        const int kind = phase_kind(ph, p.layers);
        const LayerPtrs* y = ph < last ? &p.layer[ph / 5] : nullptr;
        if (kind == kAttn) {
            const int items = p.heads * nsplit;
            for (int it = blockIdx.x + gridDim.x * warp; it < items; it += gridDim.x * kConsumerWarps)
                attend_chunk(p, *y, ph / 5, it / nsplit, it % nsplit, nsplit, n, qbuf + warp * kHeadDim);
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
            stage_copy(p.att, p.Hl, xs);
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
        const int nkt = (d.K + kPersistTileK - 1) / kPersistTileK;
        const float4* x4 = reinterpret_cast<const float4*>(xs);
        const int ra = 2 * warp, rb = ra + 1;
        for (int g = g0; g < g1; ++g) {
            const int rows = min(kPersistTileRows, d.M - g * kPersistTileRows);
            const bool va = ra < rows, vb = rb < rows;
            const int Ra = g * kPersistTileRows + ra, Rb = Ra + 1;
            // Epilogue operands, loaded now so that their latency overlaps the tiles.
            float ea = 0.0f, eb = 0.0f;  // bias, or the repetition flag in the LM head
            float xa = 0.0f, xb = 0.0f;  // residual stream
            if (kind == kLM) {
                if (va) ea = p.rep_flags[Ra] ? 1.0f : 0.0f;
                if (vb) eb = p.rep_flags[Rb] ? 1.0f : 0.0f;
            } else {
                if (va) ea = d.bias[Ra];
                if (vb) eb = d.bias[Rb];
                if (kind == kWo || kind == kW2) {
                    if (va) xa = __ldcg(p.x + Ra);
                    if (vb) xb = __ldcg(p.x + Rb);
                }
            }
            float acc_a = 0.0f, acc_b = 0.0f;
            for (int kt = 0; kt < nkt; ++kt) {
                // After a failed wait this warp only walks the schedule so that it
                // meets the other consumer warps at every named barrier.
                if (ok && !wait_parity(&full[slot], par, st)) ok = false;
                if (ok) {
                    const int k0 = kt * kPersistTileK;
                    const int kc4 = min(kPersistTileK, d.K - k0) >> 2;
                    const float4* tile =
                        reinterpret_cast<const float4*>(ring + static_cast<size_t>(slot) * kSlotBytes);
                    const float4* wa = tile + ra * (kPersistTileK / 4);
                    const float4* wb = tile + rb * (kPersistTileK / 4);
                    const float4* xk = x4 + (k0 >> 2);
#pragma unroll
                    for (int j0 = 0; j0 < kPersistTileK / 4; j0 += 32) {
                        const int j = j0 + lane;
                        if (j < kc4) {
                            const float4 xv = xk[j];
                            acc_a = dot4(wa[j], xv, acc_a);
                            acc_b = dot4(wb[j], xv, acc_b);
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[slot]);
                }
                if (++slot == kSlots) {
                    slot = 0;
                    par ^= 1u;
                }
            }
            acc_a = warp_sum(acc_a);
            acc_b = warp_sum(acc_b);
            switch (kind) {
                case kQKV:
                    if (lane == 0 && va) p.qkv[Ra] = acc_a + ea;
                    if (lane == 1 && vb) p.qkv[Rb] = acc_b + eb;
                    break;
                case kWo:
                case kW2:
                    if (lane == 0 && va) p.x[Ra] = xa + (acc_a + ea);
                    if (lane == 1 && vb) p.x[Rb] = xb + (acc_b + eb);
                    break;
                case kW13:
                    if (lane == 0 && vb) p.ffh[Ra >> 1] = silu(acc_a + ea) * (acc_b + eb);
                    break;
                default: {  // kLM: logits with the repetition penalty, running argmax
                    if (va) {
                        float v = acc_a;
                        if (ea != 0.0f) v = rep_penalty(v, rp);
                        if (lane == 0) p.logits[Ra] = v;
                        if (v > best_v) best_v = v, best_i = Ra;
                    }
                    if (vb) {
                        float v = acc_b;
                        if (eb != 0.0f) v = rep_penalty(v, rp);
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
    float* red = reinterpret_cast<float*>(empty + kSlots);                  // 16 floats
    unsigned long long* best_s = reinterpret_cast<unsigned long long*>(red + 16);  // 8
    int* s_ok = reinterpret_cast<int*>(best_s + kConsumerWarps);            // 1 (+pad)
    float* qbuf = reinterpret_cast<float*>(smem + static_cast<size_t>(kSlots) * kSlotBytes + kMaxK * 4 +
                                           2 * kSlots * 8 + 512);           // 8 x 64

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
        consumers(p, ring, xs, full, empty, red, best_s, qbuf, s_ok);
    }
}

}  // namespace

size_t persistent_smem_bytes() { return kSmemBytes; }

cudaError_t launch_decode_persistent(const PersistentParams& p, int num_sms, cudaStream_t s) {
    if (p.H > kMaxK || p.Hl > kMaxK || p.Fl > kMaxK || p.H % 4 || p.Hl % 4 || p.Fl % 4) return cudaErrorInvalidValue;
    if (persistent_max_splits(p.T) > 32) return cudaErrorInvalidValue;  // one lane per split in the merge
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
