// Persistent decode-step kernel for sm_100a: one launch per token.
//
// One CTA per SM (cooperative launch, so every CTA is resident).  Warp 0 is a
// producer: one lane streams every weight box this CTA needs for the whole
// token (16 x [QKV, out-proj, W1/V, W2] and the tied LM head) from HBM into a
// shared-memory ring with 3D TMA loads (cp.async.bulk.tensor, one 32 KB
// [16 rows][512 floats] box per instruction: a single SM sustains ~70 GB/s
// with 16 KB boxes and ~90 GB/s with 32 KB ones), gated by free ring slots and
// by a cap on boxes in flight (requested, not landed), so HBM keeps streaming
// across phase boundaries without queueing more requests than it needs to
// stay busy.  The boxes are loaded with an L2 evict-first policy: a weight
// line is dead once read, and the 113 MB a layer streams would otherwise push
// the activations, partial sums and cached K/V rows that the stagings and the
// attention wait on out of L2.  Between the landing of a phase's last box and
// the staging of the next phase's input the producer pauses: the phase's
// release signal, the grid-counter polls and the staging loads would
// otherwise wait behind the SM's in-flight weight data.  Warps 1..8 consume: per phase they wait for the previous phase
// of every CTA (a global counter), stage the phase's input vector in shared
// memory, take ring boxes (two rows per warp) and reduce with warp shuffles.
//
// Work split.  QKV, W1/V and the LM head go to the CTAs in whole 16-row
// groups (bias / SwiGLU / penalty epilogues in place).  The out-projection and
// W2 (1536 rows = 96 groups, fewer than the 148 SMs) are split evenly by
// boxes instead; each CTA writes the partial row sums of the groups it
// touches, and the next RMSNorm staging, which reads the residual stream
// anyway, adds x + bias + the partials in CTA order (deterministic).  The
// residual stream ping-pongs between xa (entering a layer) and xb (after the
// out-projection); each CTA stores one slice of it.
//
// Attention.  Head h runs on one CTA (six at most, at 768 positions); its
// warps take one 16-position chunk each and load the chunk's cached K/V rows
// into registers before the wait for the QKV phase, so only the new
// position's q / k / v is read after it; the chunks merge in shared memory,
// and only a head split over several CTAs merges through global memory
// (ticket).
//
// Replaces, for one decode token, the reference's Transformer::forward(int)
// (src/transformer.cu:180-186) with TransformerBlock::forward
// (src/transformer.cu:68-105), AttentionBlock::forward decode branch
// (src/attn.cu:648-664), MultiHeadAttention::forward (src/attn.cu:372-447,
// 490-547), SwishGLU::forward_vec (src/ffn.cu:126-139), Linear::forward_vec
// (src/linear.cu:260-282) and Embedding::inverse (src/embedding.cu:130-205).
//
// Tensor parallel (one kernel per rank, each on its own GPU, same grid): each
// rank runs its heads, FFN columns and vocab shard; the out-projection and W2
// partial row sums of every CTA are stored, each as one 64-bit word of value
// and tag (step, layer, projection), into this rank's exchange buffer before
// the phase signal and into every peer's (NVLink) after it, so the next
// staging on each rank waits for its own CTAs on the usual counter and for
// the peers' words by their tags, and sums all ranks' partials in the same
// (rank, CTA) order everywhere: no collective launch and no system-scope
// fence.
//
// Every wait is bounded: a timed-out wait sets a bit in DevState::err, makes
// the other CTAs leave at their next wait, and the producer drains its
// in-flight copies before returning.
#include <math.h>

#include "xl_device.cuh"
#include "xl_kernels.h"

namespace xl {

namespace {

constexpr int kConsumerWarps = kPersistWarps;
constexpr int kConsumerThreads = 32 * kConsumerWarps;
constexpr int kThreads = kConsumerThreads + 32;
constexpr int kBoxK = kPersistBoxK;                             // 512 floats of K per box at most
constexpr int kSlotBytes = kPersistTileRows * kBoxK * 4;         // 32 KB
constexpr int kSlots = kPersistSlots;                            // 192 KB ring
constexpr int kMaxK = 4096;
constexpr size_t kSmemBytes = static_cast<size_t>(kSlots) * kSlotBytes + kMaxK * 4 + 2 * kSlots * 8 + 512;
constexpr size_t kMaxSmemPerBlock = 232448;  // sm_100: 227 KB of dynamic shared memory per block
// Every wait is bounded twice: by polls and by wall-clock time (an mbarrier
// try_wait may suspend the thread for a while, so a poll count alone can last
// far longer than intended).  A decode step takes under a millisecond.
constexpr uint32_t kMbarSpinLimit = 1u << 24;
constexpr uint32_t kFlagSpinLimit = 1u << 24;
constexpr unsigned long long kWaitLimitNs = 200ull * 1000 * 1000;
constexpr int kErrMbar = 1, kErrFlag = 2;
// Tensor parallel: the step-start liveness sum (every rank adds 1) did not
// reach tp, so a peer never joined this step (its all-reduce was aborted).
constexpr int kErrPeer = 16;
// Attention scratch inside the staging buffer xs (free between the QKV and
// out-projection stagings): per warp the rotated q (64 floats), then per warp
// (max, sum, o[64]) partials, then per warp the rotated k of the new position.
constexpr int kAttnWarpScratch = kHeadDim;
constexpr int kAttnPartStride = kHeadDim + 4;
constexpr int kStageQuads = kMaxK / 4 / kConsumerThreads;  // float4 of a staged vector per consumer thread
constexpr int kStageBatch = 2;  // quads of an RMSNorm staging whose loads are issued together
constexpr int kPreGroups = 4;  // row groups per CTA whose biases are loaded before the phase wait

static_assert(kPersistTileRows == 2 * kConsumerWarps, "each consumer warp owns two rows of a box");
static_assert(kConsumerWarps * (kAttnWarpScratch + kAttnPartStride + kHeadDim) <= kMaxK, "attention scratch fits in xs");
static_assert(kPersistChunk == 16, "attention lanes: two per position of a 16-position chunk");

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
// 3D TMA load (no multicast) of one [16 rows][kd k-tiles][tw floats] box whose
// first k-tile is kt and first row is row; the map views W[rows][K] as
// [rows][K/tw][tw].
__device__ __forceinline__ void tma_box(void* dst, const CUtensorMap* map, int kt, int row, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(0), "r"(kt), "r"(row), "r"(smem_u32(bar))
        : "memory");
}
// The same load with an L2 cache policy (evict-first: a weight line is dead once read).
__device__ __forceinline__ void tma_box_hint(void* dst, const CUtensorMap* map, int kt, int row, uint64_t* bar,
                                             uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(0), "r"(kt), "r"(row), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
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
    unsigned long long t0 = 0;
    while (!mbar_try_wait(bar, parity)) {
        ++it;
        if ((it & 63u) == 0) {
            const unsigned long long now = globaltimer();
            if (t0 == 0) t0 = now;
            if (it >= kMbarSpinLimit || now - t0 > kWaitLimitNs || aborted(st)) {
                atomicOr(&st->err, kErrMbar);
                return false;
            }
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

// Index arithmetic is 32-bit: every product below is at most 148 SMs x 28,440
// boxes (the LM head), far inside int range.
// This CTA's boxes [t0, t1) of a phase, nb boxes of kd k-tiles per 16-row
// group, T boxes in all: whole groups (a balanced split of the groups) for
// QKV, W1/V and the LM head; an even split of the boxes for the residual
// projections.
struct Boxes {
    int t0, t1, nb, kd, bw, T;  // kd k-tiles, bw floats of K per box
};
__device__ __forceinline__ Boxes boxes_of(const Gemv& d) {
    Boxes r;
    r.kd = persist_box_tiles(d.K);
    r.bw = persist_box_width(d.K);
    r.nb = persist_boxes_per_group(d.K);
    const int groups = (d.M + kPersistTileRows - 1) / kPersistTileRows;
    r.T = groups * r.nb;
    if (d.kind == kWo || d.kind == kW2) {
        r.t0 = static_cast<int>(blockIdx.x) * r.T / static_cast<int>(gridDim.x);
        r.t1 = static_cast<int>(blockIdx.x + 1) * r.T / static_cast<int>(gridDim.x);
    } else {
        r.t0 = static_cast<int>(blockIdx.x) * groups / static_cast<int>(gridDim.x) * r.nb;
        r.t1 = static_cast<int>(blockIdx.x + 1) * groups / static_cast<int>(gridDim.x) * r.nb;
    }
    return r;
}

// Tensor parallel: rank r's exchange slot for the partial row sums that rank
// src's CTA c computed for 16-row group g of a split projection (w2 = 0: the
// out-projection, 1: W2).  A slot holds one word per row: the float's bits
// in the low half, the tag of the step, layer and projection in the high half,
// stored and loaded as one 64-bit access, so a reader that sees the tag it
// expects holds that word's value (no fence on either side).
__device__ __forceinline__ unsigned long long* xc_part(const PersistentParams& p, int r, int w2, int src, int g,
                                                       int c) {
    const int groups = p.H / kPersistTileRows;
    return p.xc[r] +
           ((static_cast<size_t>(w2 * p.tp + src) * groups + g) * kPersistMaxContrib + c) * kPersistTileRows;
}
// Tag of layer l's split projection w2 in this step: grows with every use, and
// the buffers start zeroed, so a stale word never carries it.
__device__ __forceinline__ unsigned xtag(const PersistentParams& p, int l, int w2) {
    return static_cast<unsigned>(p.st->epoch) * (2u * static_cast<unsigned>(p.layers)) + 2u * l + w2 + 1u;
}
// The tag a staging waits for: xtag shifted by tag_skew (0 in service; a test
// sets it to a tag nobody writes, so that the bounded wait runs out).
__device__ __forceinline__ unsigned rtag(const PersistentParams& p, int l, int w2) {
    return xtag(p, l, w2) + static_cast<unsigned>(p.tag_skew);
}
__device__ __forceinline__ unsigned long long xword(float v, unsigned tag) {
    return (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
}
// This rank's partial sum of row `row` of group g (slot c) of layer l's split
// projection w2, tagged, into its own exchange buffer.
__device__ __noinline__ void store_own_tp(const PersistentParams& p, int l, int w2, int g, int c, int row, float v) {
    xc_part(p, p.rank, w2, p.rank, g, c)[row] = xword(v, xtag(p, l, w2));
}
// tag_split: this CTA's partial sum of row `row` of group g (slot c) of layer
// l's split projection w2 goes, tagged, straight to every rank's exchange
// buffer (this rank's own included): the next staging waits for the tags
// alone, so the phase needs neither a release fence nor a grid counter.  The
// stores are relaxed and single-copy atomic (one aligned 64-bit word each):
// a reader that sees the expected tag holds the value stored with it.
__device__ __noinline__ void store_all_tp(const PersistentParams& p, int l, int w2, int g, int c, int row, float v) {
    const unsigned long long w = xword(v, xtag(p, l, w2));
    for (int r = 0; r < p.tp; ++r) {
        unsigned long long* a = xc_part(p, r, w2, p.rank, g, c) + row;
        if (r == p.rank)
            asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(a), "l"(w) : "memory");
        else
            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(w) : "memory");
    }
}
// After this warp's phase signal: its partial sums of the phase (row `row` of
// each group of boxes [r.t0, r.t1), already in this rank's own slots) go to
// the same slots on every other rank (stores to peer memory over NVLink).
__device__ __noinline__ void forward_partials_tp(const PersistentParams& p, int t0, int t1, int nb, int T, int w2,
                                                 int row) {
    for (int tau = t0; tau < t1;) {
        const int g = tau / nb, bi0 = tau % nb, bi1 = min(nb, bi0 + (t1 - tau));
        const int c = persist_contrib_slot(blockIdx.x, g, bi0, nb, T, gridDim.x);
        const unsigned long long w = xc_part(p, p.rank, w2, p.rank, g, c)[row];  // this thread's own store
        for (int r = 0; r < p.tp; ++r)
            if (r != p.rank)
                asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(xc_part(p, r, w2, p.rank, g, c) + row), "l"(w)
                             : "memory");
        tau += bi1 - bi0;
    }
}
// Tensor parallel, greedy steps: the merge area after the partial-sum slots of
// rank r's exchange buffer holds one (key, tag) pair of 64-bit words per rank.
__device__ __forceinline__ unsigned long long* xmerge(const PersistentParams& p, int r) {
    const int groups = p.H / kPersistTileRows;
    return p.xc[r] + static_cast<size_t>(2 * p.tp) * groups * kPersistMaxContrib * kPersistTileRows;
}
// This rank's packed argmax key (value key, ~global id) goes to slot [rank]
// of every rank's merge area: the key word, one system-scope fence, then the
// step's tag word (every slot then holds this step's key before its tag).
// The step's winner is the largest key of all ranks, read back from this
// rank's own area once every tag is there.  Slot reuse is safe: a rank
// overwrites its slots only in the next step, which starts with an NCCL
// barrier that every rank joins after this kernel.  Returns 0 (and sets the
// error bit) if a peer's tag does not arrive within the wait limit.
__device__ unsigned long long merge_argmax_tp(const PersistentParams& p, unsigned long long key) {
    const unsigned long long tag = static_cast<unsigned long long>(static_cast<unsigned>(p.st->epoch)) + 1ull;
    for (int r = 0; r < p.tp; ++r)
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(xmerge(p, r) + 2 * p.rank), "l"(key) : "memory");
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int r = 0; r < p.tp; ++r)
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(xmerge(p, r) + 2 * p.rank + 1), "l"(tag) : "memory");
    const unsigned long long* mine = xmerge(p, p.rank);
    unsigned long long best = 0;
    for (int src = 0; src < p.tp; ++src) {
        uint32_t it = 0;
        unsigned long long t0 = 0, tg = 0;
        for (;;) {
            asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(tg) : "l"(mine + 2 * src + 1) : "memory");
            if (tg == tag) break;
            if ((++it & 63u) == 0) {
                const unsigned long long now = globaltimer();
                if (t0 == 0) t0 = now;
                if (it >= kFlagSpinLimit || now - t0 > kWaitLimitNs || aborted(p.st)) {
                    atomicOr(&p.st->err, kErrFlag);
                    return 0ull;
                }
            }
        }
        unsigned long long k;
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(k) : "l"(mine + 2 * src) : "memory");
        best = k > best ? k : best;
    }
    return best;
}

// ---------------------------------------------------------------------------
// Producer: walks this CTA's boxes of every GEMV phase in order.
struct Cursor {
    const CUtensorMap* map;
    int ph, tau, t1, t0, nb, kd, bw;
    bool valid;
};

__device__ void cursor_first(const PersistentParams& p, int ph, Cursor& c) {
    const int last = 5 * p.layers;
    for (; ph <= last; ++ph) {
        if (phase_kind(ph, p.layers) == kAttn) continue;
        const Gemv d = gemv_of(p, ph);
        const Boxes r = boxes_of(d);
        if (r.t0 < r.t1) {
            c.map = d.map;
            c.ph = ph, c.tau = r.t0, c.t0 = r.t0, c.t1 = r.t1, c.nb = r.nb, c.kd = r.kd, c.bw = r.bw;
            c.valid = true;
            return;
        }
    }
    c.valid = false;
}

template <int SLOTS>
__device__ void producer(const PersistentParams& p, char* ring, uint64_t* full, uint64_t* empty,
                         const volatile int* quiet) {
    DevState* st = p.st;
    int slot = 0;
    uint32_t par = 0;
    int issued = 0;
    bool ok = true;
    const int inflight = p.inflight;
    const uint64_t policy = evict_first_policy();
    Cursor c;
    for (cursor_first(p, 0, c); c.valid;) {
        if (!wait_parity(&empty[slot], par ^ 1u, st)) {
            ok = false;
            break;
        }
        // Quiet window (set by the consumers from the moment the last box of a
        // phase has landed until the next phase's input is staged): issue
        // nothing, so that the result stores' acknowledgements the phase
        // signal waits for, the grid-counter polls and the staging loads do not
        // queue behind this SM's weight stream.
        if (*quiet) {
            uint32_t it = 0;
            const unsigned long long t0 = globaltimer();
            while (*quiet) {
                if ((++it & 63u) == 0 && (globaltimer() - t0 > kWaitLimitNs || aborted(st))) break;
            }
        }
        // At most `inflight` boxes requested but not landed: a deeper queue only
        // adds latency to every other memory access once HBM is saturated.
        if (issued >= inflight) {
            const int k = issued - inflight;
            if (!wait_parity(&full[k % SLOTS], static_cast<uint32_t>((k / SLOTS) & 1), st)) {
                ok = false;
                break;
            }
        }
        if (c.tau == c.t0) trace_at(p, c.ph, kTrProdFirst);
        const int g = c.tau / c.nb, bi = c.tau % c.nb;
        // Rows past M and k-tiles past K of the box are zero-filled by TMA and
        // still counted in the transaction bytes.
        mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(kPersistTileRows * c.bw * 4));
        if (p.tma_evict_first)
            tma_box_hint(ring + static_cast<size_t>(slot) * kSlotBytes, c.map, bi * c.kd, g * kPersistTileRows,
                         &full[slot], policy);
        else
            tma_box(ring + static_cast<size_t>(slot) * kSlotBytes, c.map, bi * c.kd, g * kPersistTileRows, &full[slot]);
        ++issued;
        if (++slot == SLOTS) {
            slot = 0;
            par ^= 1u;
        }
        if (++c.tau == c.t1) {
            trace_at(p, c.ph, kTrProdLast);
            cursor_first(p, c.ph + 1, c);
        }
    }
    if (!ok) {
        // Drain: every copy already issued must land before this CTA exits.
        const int pending = issued < SLOTS ? issued : SLOTS;
        for (int i = 1; i <= pending; ++i) {
            const int k = issued - i;  // box k went to slot k % SLOTS with parity (k / SLOTS) & 1
            const int s = k % SLOTS;
            const uint32_t pp = static_cast<uint32_t>((k / SLOTS) & 1);
            uint32_t it = 0;
            unsigned long long t0 = 0;
            while (!mbar_try_wait(&full[s], pp) && ++it < kMbarSpinLimit) {
                if ((it & 63u) == 0) {
                    const unsigned long long now = globaltimer();
                    if (t0 == 0) t0 = now;
                    if (now - t0 > kWaitLimitNs) break;
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Consumer helpers (256 threads, named barrier 1).

// Wait until phase ph is complete (its counter reaches its target).
__device__ bool wait_phase(const PersistentParams& p, int ph, int* s_ok) {
    const int kind = phase_kind(ph, p.layers);
    // An attention phase is signalled once per head (by the warp that writes
    // the head's output); every other phase by every consumer warp of every CTA.
    const int target = kind == kAttn ? p.heads : static_cast<int>(gridDim.x) * (p.sig_cta ? 1 : kConsumerWarps);
    if (threadIdx.x == 32) {
        const int* c = p.done + ph;
        uint32_t it = 0;
        unsigned long long t0 = 0;
        int ok = 1;
        while (ld_acquire(c) < target) {
            ++it;
            if ((it & 255u) == 0) {
                const unsigned long long now = globaltimer();
                if (t0 == 0) t0 = now;
                if (it >= kFlagSpinLimit || now - t0 > kWaitLimitNs || aborted(p.st)) {
                    atomicOr(&p.st->err, kErrFlag);
                    ok = 0;
                    break;
                }
            }
        }
        *s_ok = ok;
    }
    consumer_sync();
    return *s_ok != 0;
}

// One warp publishes its own stores of phase ph as soon as it has issued
// them: lane 0 releases (cumulative over the warp's lanes, ordered by the
// __syncwarp) and adds 1 to the counter.
__device__ void signal_warp(const PersistentParams& p, int ph) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(p.done + ph) : "memory");
}
// A GEMV phase's signal, from every consumer warp: per warp (no warp waits
// for its CTA), or with sig_cta one release per CTA after a consumer barrier
// (the barrier orders the other warps' stores before the first consumer
// thread's release, which is cumulative over them): 8x fewer reductions on
// the phase counter's line.
__device__ void signal_phase(const PersistentParams& p, int ph) {
    if (!p.sig_cta) {
        signal_warp(p, ph);
        return;
    }
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

// Residual rows 4q .. 4q+3 (within one 16-row group) after a split
// projection: x_old + (the partial row sums of the CTAs that own the group's
// boxes, in CTA order, + bias).
__device__ __forceinline__ float4 residual_quad(float4 xo, const float* bias, const float* cres, int q, int nb,
                                                int T) {
    const int g = (4 * q) / kPersistTileRows;
    const int G = gridDim.x;
    const int nc = persist_group_contrib(g, nb, T, G);
    const float4* part = reinterpret_cast<const float4*>(cres + g * (kPersistMaxContrib * kPersistTileRows)) +
                         (q % (kPersistTileRows / 4));
    float4 v[kPersistMaxContrib];
#pragma unroll
    for (int c = 0; c < kPersistMaxContrib; ++c)
        v[c] = c < nc ? __ldcg(part + c * (kPersistTileRows / 4)) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const float4 b = reinterpret_cast<const float4*>(bias)[q];
    float4 s = v[0];
#pragma unroll
    for (int c = 1; c < kPersistMaxContrib; ++c) {
        if (c < nc) {
            s.x += v[c].x;
            s.y += v[c].y;
            s.z += v[c].z;
            s.w += v[c].w;
        }
    }
    return make_float4(xo.x + (s.x + b.x), xo.y + (s.y + b.y), xo.z + (s.z + b.z), xo.w + (s.w + b.w));
}

// xs = rmsnorm(x) * gamma, where x is the embedding row (cres == nullptr) or
// the residual after a split projection of nb boxes per group; this CTA stores
// its slice of x to x_out.  float4 accesses; every load of a batch of quads
// (x, partial sums, bias, gamma) is issued before the first store, so a
// staging costs one L2 round trip per batch (one in all at K <= 2048).
// With xr (resid_smem), the residual before the projection is this CTA's own
// copy in shared memory (every CTA computes the same x in the same order) and
// x is written back there; x_out then gets its slice only when out_too is set
// (the LM head's input, read back by the host's LM-head profile).
__device__ __noinline__ void stage_norm(const PersistentParams& p, const float* x_old, const float* bias, const float* cres,
                           int nb, const float* gamma, float* xs, float* red, float* x_out, float* xr, bool out_too) {
    const int t = threadIdx.x - 32;
    const int K = p.H;
    const int T = (K / kPersistTileRows) * nb;
    const int s0 = static_cast<int>(blockIdx.x) * K / static_cast<int>(gridDim.x);
    const int s1 = static_cast<int>(blockIdx.x + 1) * K / static_cast<int>(gridDim.x);
    float4* x4 = reinterpret_cast<float4*>(xs);
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
    float4 gk[kStageQuads];
    float ss = 0.0f;
#pragma unroll
    for (int k0 = 0; k0 < kStageQuads; k0 += kStageBatch) {
        if (k0 * kConsumerThreads >= (K >> 2)) break;
        float4 v[kStageBatch];
#pragma unroll
        for (int u = 0; u < kStageBatch; ++u) {
            const int q = t + (k0 + u) * kConsumerThreads;
            if (q < (K >> 2)) {
                gk[k0 + u] = g4[q];
                // the residual before the projection: this CTA's copy in shared
                // memory, or global memory written by other CTAs (L2, not L1)
                const float4 xo = xr && cres ? reinterpret_cast<const float4*>(xr)[q]
                                             : __ldcg(reinterpret_cast<const float4*>(x_old) + q);
                v[u] = cres ? residual_quad(xo, bias, cres, q, nb, T) : xo;
            }
        }
#pragma unroll
        for (int u = 0; u < kStageBatch; ++u) {
            const int q = t + (k0 + u) * kConsumerThreads;
            if (q < (K >> 2)) {
                x4[q] = v[u];
                if (xr) reinterpret_cast<float4*>(xr)[q] = v[u];
                if (!xr || out_too) {
                    const float e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        if (4 * q + c >= s0 && 4 * q + c < s1) x_out[4 * q + c] = e[c];
                }
                ss = dot4(v[u], v[u], ss);
            }
        }
    }
    const float tot = consumer_sum(ss, red);
    // RMSNorm of src/rmsnorm.cu:99-101: 1 / sqrt(mean + 1e-6), in double.
    const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(tot / static_cast<float>(K)) + 1e-6));
#pragma unroll
    for (int k = 0; k < kStageQuads; ++k) {
        const int q = t + k * kConsumerThreads;
        if (q < (K >> 2)) {
            float4 v = x4[q];
            v.x = v.x * inv * gk[k].x;
            v.y = v.y * inv * gk[k].y;
            v.z = v.z * inv * gk[k].z;
            v.w = v.w * inv * gk[k].w;
            x4[q] = v;
        }
    }
}

// Tensor parallel: as residual_quad, with the partial row sums of every rank
// (already in this rank's exchange buffer) added in (rank, CTA) order, so that
// every rank computes the same residual.
__device__ __forceinline__ void ld_words(const unsigned long long* a, unsigned long long& x, unsigned long long& y) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(x), "=l"(y) : "l"(a) : "memory");
}
__device__ __forceinline__ float4 residual_quad_tp(const PersistentParams& p, float4 xo, const float* bias,
                                                   int w2, int q, int nb, int T, unsigned tag) {
    const int g = (4 * q) / kPersistTileRows;
    const int G = gridDim.x;
    const int nc = persist_group_contrib(g, nb, T, G);
    const int qq = q % (kPersistTileRows / 4);
    float4 s = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int src = 0; src < p.tp; ++src) {
        const unsigned long long* part = xc_part(p, p.rank, w2, src, g, 0) + 4 * qq;
        unsigned long long w[kPersistMaxContrib][4];
        // Spin until every word carries this use's tag (bounded like every wait).
        uint32_t it = 0;
        unsigned long long t0 = 0;
        for (;;) {
#pragma unroll
            for (int c = 0; c < kPersistMaxContrib; ++c) {
                if (c < nc) {
                    ld_words(part + c * kPersistTileRows, w[c][0], w[c][1]);
                    ld_words(part + c * kPersistTileRows + 2, w[c][2], w[c][3]);
                }
            }
            bool ok = true;
#pragma unroll
            for (int c = 0; c < kPersistMaxContrib; ++c)
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (c < nc && static_cast<unsigned>(w[c][k] >> 32) != tag) ok = false;
            if (ok) break;
            ++it;
            if ((it & 15u) == 0) {
                const unsigned long long now = globaltimer();
                if (t0 == 0) t0 = now;
                if (it >= kFlagSpinLimit || now - t0 > kWaitLimitNs || aborted(p.st)) {
                    atomicOr(&p.st->err, kErrFlag);
                    break;
                }
            }
        }
#pragma unroll
        for (int c = 0; c < kPersistMaxContrib; ++c) {
            if (c < nc) {
                const float4 v = make_float4(__uint_as_float(static_cast<unsigned>(w[c][0])),
                                             __uint_as_float(static_cast<unsigned>(w[c][1])),
                                             __uint_as_float(static_cast<unsigned>(w[c][2])),
                                             __uint_as_float(static_cast<unsigned>(w[c][3])));
                if (src == 0 && c == 0) {
                    s = v;
                } else {
                    s.x += v.x;
                    s.y += v.y;
                    s.z += v.z;
                    s.w += v.w;
                }
            }
        }
    }
    const float4 b = reinterpret_cast<const float4*>(bias)[q];
    return make_float4(xo.x + (s.x + b.x), xo.y + (s.y + b.y), xo.z + (s.z + b.z), xo.w + (s.w + b.w));
}

// stage_norm for tensor parallel: the residual after a split projection whose
// partial sums all ranks exchanged (w2: which projection; tag: its use).
__device__ __noinline__ void stage_norm_tp(const PersistentParams& p, const float* x_old, const float* bias, int w2,
                                           unsigned tag, int nb, const float* gamma, float* xs, float* red,
                                           float* x_out, float* xr, bool out_too) {
    const int t = threadIdx.x - 32;
    const int K = p.H;
    const int T = (K / kPersistTileRows) * nb;
    const int s0 = static_cast<int>(blockIdx.x) * K / static_cast<int>(gridDim.x);
    const int s1 = static_cast<int>(blockIdx.x + 1) * K / static_cast<int>(gridDim.x);
    float4* x4 = reinterpret_cast<float4*>(xs);
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
    float4 gk[kStageQuads];
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < kStageQuads; ++k) {
        const int q = t + k * kConsumerThreads;
        if (q < (K >> 2)) {
            gk[k] = g4[q];
            const float4 xo = xr ? reinterpret_cast<const float4*>(xr)[q]
                                 : __ldcg(reinterpret_cast<const float4*>(x_old) + q);
            const float4 v = residual_quad_tp(p, xo, bias, w2, q, nb, T, tag);
            x4[q] = v;
            if (xr) reinterpret_cast<float4*>(xr)[q] = v;
            if (!xr || out_too) {
                const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (4 * q + u >= s0 && 4 * q + u < s1) x_out[4 * q + u] = e[u];
            }
            ss = dot4(v, v, ss);
        }
    }
    const float tot = consumer_sum(ss, red);
    const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(tot / static_cast<float>(K)) + 1e-6));
#pragma unroll
    for (int k = 0; k < kStageQuads; ++k) {
        const int q = t + k * kConsumerThreads;
        if (q < (K >> 2)) {
            float4 v = x4[q];
            v.x = v.x * inv * gk[k].x;
            v.y = v.y * inv * gk[k].y;
            v.z = v.z * inv * gk[k].z;
            v.w = v.w * inv * gk[k].w;
            x4[q] = v;
        }
    }
}

// xs = src[0, K): all of a thread's loads before its shared-memory stores.
__device__ void stage_copy(const float* src, int K, float* xs) {
    const int t = threadIdx.x - 32;
    float4 v[kStageQuads];
#pragma unroll
    for (int k = 0; k < kStageQuads; ++k) {
        const int q = t + k * kConsumerThreads;
        if (q < (K >> 2)) v[k] = __ldcg(reinterpret_cast<const float4*>(src) + q);
    }
#pragma unroll
    for (int k = 0; k < kStageQuads; ++k) {
        const int q = t + k * kConsumerThreads;
        if (q < (K >> 2)) reinterpret_cast<float4*>(xs)[q] = v[k];
    }
}

// This CTA's attention item of the token: head h, CTA j of the head's nct;
// the heads * nct items are spread evenly over the grid, one per CTA at most.
__device__ __forceinline__ bool attn_item(int heads, int nct, int& h, int& j) {
    const int items = heads * nct, G = gridDim.x, b = blockIdx.x;
    const int i = (b * items + G - 1) / G;
    if (i >= items || (i * G) / items != b) return false;
    h = i / nct;
    j = i % nct;
    return true;
}

// The attention phase of one layer on this CTA (all consumer warps enter).
// Per warp: chunk s = j * 8 + warp of positions [32 s, 32 s + 32) ∩ [0, n],
// lane l owning position 32 s + l: RoPE at position n (src/rope.cu:20-45), KV
// append, scores, softmax and P.V (src/attn.cu:490-547).  Returns false if the
// wait for the QKV phase failed.
__device__ bool attention_phase(const PersistentParams& p, int layer, int ph, int n, float* xs, int* s_ok) {
    const int t = threadIdx.x - 32;
    const int warp = t >> 5, lane = t & 31;
    const int nsplit = n / kPersistChunk + 1;
    const int nct = (nsplit + kConsumerWarps - 1) / kConsumerWarps;
    int h = 0, j = 0;
    const bool has = attn_item(p.heads, nct, h, j);
    const LayerPtrs& y = p.layer[layer];
    const int s = j * kConsumerWarps + warp;
    const bool active = has && s < nsplit;
    const int t0 = s * kPersistChunk;
    float* kc = y.kc + static_cast<size_t>(h) * p.T * kHeadDim;
    float* vc = y.vc + static_cast<size_t>(h) * p.T * kHeadDim;
    // The chunk's cached rows (positions t0 .. min(t0 + 16, n) - 1) do not depend
    // on this token's QKV phase: load them before its wait, so the only L2 round
    // trip after it is q / k / v of the new position.  Scores: lane pair
    // (2 kp, 2 kp + 1) owns position t0 + kp, half kh of its 64 dims (8 float4
    // of K).  P.V: lane owns output dims (2 lane, 2 lane + 1) of every row.
    const int kp = lane >> 1, kh = lane & 1;
    const int posk = t0 + kp;
    const int cached = active ? min(kPersistChunk, n - t0) : 0;
    float4 kv[8];
    float2 vrow[kPersistChunk];
    const float4* kr = reinterpret_cast<const float4*>(kc + static_cast<size_t>(kp < cached ? posk : 0) * kHeadDim) +
                       8 * kh;
#pragma unroll
    for (int i = 0; i < 8; ++i) kv[i] = kp < cached ? __ldcg(kr + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const float2* vr = reinterpret_cast<const float2*>(vc + static_cast<size_t>(t0) * kHeadDim) + lane;
#pragma unroll
    for (int jp = 0; jp < kPersistChunk; ++jp)
        vrow[jp] = jp < cached ? __ldcg(vr + jp * (kHeadDim / 2)) : make_float2(0.0f, 0.0f);
    const float2 cs = active ? p.rope[n * kHalfHead + lane] : make_float2(0.0f, 0.0f);
    // A CTA without an attention item neither waits nor signals: the next
    // phase waits for the heads' outputs, which imply the QKV phase.
    if (!has) return true;
    if (!wait_phase(p, ph - 1, s_ok)) return false;
    if (t == 0) trace_at(p, ph, kTrConsStart);
    float* qsh = xs + warp * kAttnWarpScratch;
    float* apart = xs + kConsumerWarps * kAttnWarpScratch;  // [8][68]
    float* knew = xs + kConsumerWarps * (kAttnWarpScratch + kAttnPartStride) + warp * kHeadDim;  // rotated k of row n
    if (active) {
        const bool has_n = n >= t0 && n < t0 + kPersistChunk;
        const float* q = p.qkv + h * kHeadDim;
        const float* kn = p.qkv + p.Hl + h * kHeadDim;
        const float* vn = p.qkv + 2 * p.Hl + h * kHeadDim;
        const float qa = __ldcg(q + lane), qb = __ldcg(q + lane + kHalfHead);
        float ka = 0.0f, kb = 0.0f;
        float2 vnew = make_float2(0.0f, 0.0f);
        if (has_n) {
            ka = __ldcg(kn + lane);
            kb = __ldcg(kn + lane + kHalfHead);
            vnew = __ldcg(reinterpret_cast<const float2*>(vn) + lane);
        }
        qsh[lane] = (qa * cs.x + qb * cs.y) * 0.125f;  // 1/sqrt(64) is exact
        qsh[lane + kHalfHead] = (-qa * cs.y + qb * cs.x) * 0.125f;
        if (has_n) {
            // RoPE of k at position n and the KV append (read back from the cache by later tokens).
            const float k0 = ka * cs.x + kb * cs.y, k1 = -ka * cs.y + kb * cs.x;
            knew[lane] = k0;
            knew[lane + kHalfHead] = k1;
            kc[n * kHeadDim + lane] = k0;
            kc[n * kHeadDim + lane + kHalfHead] = k1;
            reinterpret_cast<float2*>(vc + n * kHeadDim)[lane] = vnew;
        }
        __syncwarp();
        const float4* q4 = reinterpret_cast<const float4*>(qsh) + 8 * kh;
        if (posk == n) {
            const float4* k4 = reinterpret_cast<const float4*>(knew) + 8 * kh;
#pragma unroll
            for (int i = 0; i < 8; ++i) kv[i] = k4[i];
        }
        float d = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) d = dot4(kv[i], q4[i], d);
        d += __shfl_xor_sync(0xffffffffu, d, 1);
        const bool mine = posk <= n;
        const float sc = mine ? d : -INFINITY;
        const float m = warp_max(sc);
        const float e = mine ? expf(sc - m) : 0.0f;
        const float l = warp_sum(kh == 0 ? e : 0.0f);  // each position counted once
        // P.V over the chunk's rows; row n comes from this token's v.
        float2 o = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int jp = 0; jp < kPersistChunk; ++jp) {
            const float ej = __shfl_sync(0xffffffffu, e, 2 * jp);
            const float2 v = t0 + jp == n ? vnew : vrow[jp];
            o.x = fmaf(ej, v.x, o.x);
            o.y = fmaf(ej, v.y, o.y);
        }
        float* ap = apart + warp * kAttnPartStride;
        reinterpret_cast<float2*>(ap + 4)[lane] = o;
        if (lane == 0) {
            ap[0] = m;
            ap[1] = l;
        }
    }
    consumer_sync();
    if (warp != 0) return true;
    // Merge this CTA's chunks: lane k holds chunk k's (max, sum); every lane
    // two output dims.
    const int nw = min(kConsumerWarps, nsplit - j * kConsumerWarps);
    const float mk = lane < nw ? apart[lane * kAttnPartStride] : -INFINITY;
    const float lk = lane < nw ? apart[lane * kAttnPartStride + 1] : 0.0f;
    const float M = warp_max(mk);
    const float wk = lane < nw ? expf(mk - M) : 0.0f;
    const float L = warp_sum(lk * wk);
    float2 acc = make_float2(0.0f, 0.0f);
    for (int k = 0; k < nw; ++k) {
        const float wt = __shfl_sync(0xffffffffu, wk, k);
        const float2 ok = reinterpret_cast<const float2*>(apart + k * kAttnPartStride + 4)[lane];
        acc.x = fmaf(wt, ok.x, acc.x);
        acc.y = fmaf(wt, ok.y, acc.y);
    }
    float2* out = reinterpret_cast<float2*>(p.att + h * kHeadDim);
    if (nct == 1) {
        out[lane] = make_float2(acc.x / L, acc.y / L);
        signal_warp(p, ph);
        return true;
    }
    // A head split over nct CTAs: the last CTA to finish merges their partials.
    float* base = p.part + static_cast<size_t>(h) * persistent_max_splits(p.T) * (kHeadDim + 2);
    float* pp = base + j * (kHeadDim + 2);
    reinterpret_cast<float2*>(pp + 2)[lane] = acc;
    if (lane == 0) {
        pp[0] = M;
        pp[1] = L;
    }
    __syncwarp();
    int ticket = 0;
    if (lane == 0) {
        __threadfence();
        ticket = atomicAdd(p.head_done + layer * p.heads + h, 1);
    }
    ticket = __shfl_sync(0xffffffffu, ticket, 0);
    if (ticket != nct - 1) return true;
    __threadfence();
    const float mc = lane < nct ? __ldcg(base + lane * (kHeadDim + 2)) : -INFINITY;
    const float lc = lane < nct ? __ldcg(base + lane * (kHeadDim + 2) + 1) : 0.0f;
    const float M2 = warp_max(mc);
    const float wc = lane < nct ? expf(mc - M2) : 0.0f;
    const float L2 = warp_sum(lc * wc);
    float2 acc2 = make_float2(0.0f, 0.0f);
    for (int k = 0; k < nct; ++k) {
        const float wt = __shfl_sync(0xffffffffu, wc, k);
        const float2 ok = __ldcg(reinterpret_cast<const float2*>(base + k * (kHeadDim + 2) + 2) + lane);
        acc2.x = fmaf(wt, ok.x, acc2.x);
        acc2.y = fmaf(wt, ok.y, acc2.y);
    }
    out[lane] = make_float2(acc2.x / L2, acc2.y / L2);
    signal_warp(p, ph);
    return true;
}

template <bool TP>
__device__ void consumers(const PersistentParams& p, char* ring, float* xs, uint64_t* full, uint64_t* empty,
                          float* red, unsigned long long* best_s, int* s_ok, volatile int* quiet, float* xr) {
    DevState* st = p.st;
    const int t = threadIdx.x - 32;
    const int warp = t >> 5, lane = t & 31;
    const int n = st->pos;
    const float rp = st->in.rp;
    const int nb_wo = persist_boxes_per_group(p.Hl), nb_w2 = persist_boxes_per_group(p.Fl);
    int slot = 0;
    uint32_t par = 0;
    float best_v = -INFINITY;
    int best_i = -1;
    bool ok = true;
    const int last = 5 * p.layers;
    for (int ph = 0; ph <= last; ++ph) {
        const int kind = phase_kind(ph, p.layers);
        if (kind == kAttn) {
            // Head outputs are signalled inside; the pause that began with the
            // QKV phase's last box lasts through this CTA's attention.
            if (!attention_phase(p, ph / 5, ph, n, xs, s_ok)) return;
            if (t == 0) *quiet = 0;
            if (t == 0) trace_at(p, ph, kTrConsEnd);
            continue;
        }
        const int l = ph / 5;
        const LayerPtrs* y = ph < last ? &p.layer[l] : nullptr;
        const Gemv d = gemv_of(p, ph);
        const Boxes r = boxes_of(d);
        const int ra = 2 * warp, rb = ra + 1;
        // Biases of this CTA's first groups (QKV, W1/V), loaded before the wait so
        // that their latency hides behind it.
        const int g_first = r.t0 / r.nb;
        float pre_a[kPreGroups], pre_b[kPreGroups];
        if (kind == kQKV || kind == kW13) {
#pragma unroll
            for (int i = 0; i < kPreGroups; ++i) {
                const int g = g_first + i;
                if (g * r.nb < r.t1) {
                    pre_a[i] = d.bias[g * kPersistTileRows + ra];
                    pre_b[i] = d.bias[g * kPersistTileRows + rb];
                }
            }
        }
        // tag_split: a staging after a split projection (W1/V after the
        // out-projection, QKV and the LM head after W2) waits for the tags of
        // the partial sums it reads, not for the phase counter; the residual it
        // adds them to is the CTA's own copy in shared memory.
        const bool by_tags = TP && p.tag_split && (kind == kW13 || (kind == kQKV && l > 0) || kind == kLM);
        if (ph > 0 && !by_tags && !wait_phase(p, ph - 1, s_ok)) return;
        if (t == 0) trace_at(p, ph, kTrConsStart);
        // Stage this phase's input vector.
        if (kind == kQKV) {
            if (l == 0)
                stage_norm(p, p.emb + static_cast<size_t>(st->in.token_in) * p.H, nullptr, nullptr, 0, y->g1, xs, red,
                           p.xa, xr, false);
            else if (TP)
                stage_norm_tp(p, p.xb, p.layer[l - 1].b2, 1, rtag(p, l - 1, 1), nb_w2, y->g1, xs, red, p.xa, xr,
                              false);
            else
                stage_norm(p, p.xb, p.layer[l - 1].b2, p.cres, nb_w2, y->g1, xs, red, p.xa, xr, false);
        } else if (kind == kWo) {
            stage_copy(p.att, p.Hl, xs);
        } else if (kind == kW13) {
            if (TP)
                stage_norm_tp(p, p.xa, y->bo, 0, rtag(p, l, 0), nb_wo, y->g2, xs, red, p.xb, xr, false);
            else
                stage_norm(p, p.xa, y->bo, p.cres, nb_wo, y->g2, xs, red, p.xb, xr, false);
        } else if (kind == kW2) {
            stage_copy(p.ffh, p.Fl, xs);
        } else {  // kLM: the final residual also goes to xa (the LM head's input in global memory)
            if (TP)
                stage_norm_tp(p, p.xb, p.layer[l - 1].b2, 1, rtag(p, l - 1, 1), nb_w2, p.gnorm, xs, red, p.xa, xr,
                              true);
            else
                stage_norm(p, p.xb, p.layer[l - 1].b2, p.cres, nb_w2, p.gnorm, xs, red, p.xa, xr, true);
        }
        consumer_sync();
        if (t == 0) *quiet = 0;
        if (t == 0) trace_at(p, ph, kTrConsStaged);
        const int rs4 = r.bw / 4;  // float4 per row of a box
        const float4* x4 = reinterpret_cast<const float4*>(xs);
        const bool split = kind == kWo || kind == kW2;
        for (int tau = r.t0; tau < r.t1;) {
            const int g = tau / r.nb;
            const int bi0 = tau % r.nb, bi1 = min(r.nb, bi0 + (r.t1 - tau));
            const int rows = min(kPersistTileRows, d.M - g * kPersistTileRows);
            const bool va = ra < rows, vb = rb < rows;
            const int Ra = g * kPersistTileRows + ra, Rb = Ra + 1;
            // Epilogue operands, loaded now so that their latency overlaps the boxes.
            float ea = 0.0f, eb = 0.0f;  // bias, or the repetition flag in the LM head
            if (kind == kLM) {
                if (va) ea = p.rep_flags[Ra] ? 1.0f : 0.0f;
                if (vb) eb = p.rep_flags[Rb] ? 1.0f : 0.0f;
            } else if (!split) {
                const int gi = g - g_first;
                if (gi < kPreGroups) {
                    ea = pre_a[gi];
                    eb = pre_b[gi];
                } else {
                    if (va) ea = d.bias[Ra];
                    if (vb) eb = d.bias[Rb];
                }
            }
            float acc_a = 0.0f, acc_b = 0.0f;
            for (int bi = bi0; bi < bi1; ++bi) {
                // After a failed wait this warp only walks the schedule so that it
                // meets the other consumer warps at every named barrier.
                if (ok && !wait_parity(&full[slot], par, st)) ok = false;
                // Every box of this phase has landed: quiet window until the next staging.
                if (t == 0 && kind != kLM && tau + (bi - bi0) == r.t1 - 1) *quiet = 1;
                if (ok) {
                    const int k0 = bi * r.bw;
                    const int kc4 = min(r.bw, d.K - k0) >> 2;
                    const float4* tile =
                        reinterpret_cast<const float4*>(ring + static_cast<size_t>(slot) * kSlotBytes);
                    const float4* wa = tile + ra * rs4;
                    const float4* wb = tile + rb * rs4;
                    const float4* xk = x4 + (k0 >> 2);
#pragma unroll
                    for (int j0 = 0; j0 < kBoxK / 4; j0 += 32) {
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
            tau += bi1 - bi0;
            acc_a = warp_sum(acc_a);
            acc_b = warp_sum(acc_b);
            switch (kind) {
                case kQKV:
                    if (lane == 0 && va) p.qkv[Ra] = acc_a + ea;
                    if (lane == 1 && vb) p.qkv[Rb] = acc_b + eb;
                    break;
                case kWo:
                case kW2: {  // partial row sums of this CTA's boxes of group g (c: this CTA's rank among its owners)
                    const int c = persist_contrib_slot(blockIdx.x, g, bi0, r.nb, r.T, gridDim.x);
                    if (!TP) {
                        float* q = p.cres + (static_cast<size_t>(g) * kPersistMaxContrib + c) * kPersistTileRows;
                        if (lane == 0) q[ra] = acc_a;
                        if (lane == 1) q[rb] = acc_b;
                    } else if (lane < 2 && p.tag_split) {  // every rank's slot now
                        store_all_tp(p, l, kind == kW2, g, c, lane == 0 ? ra : rb, lane == 0 ? acc_a : acc_b);
                    } else if (lane < 2) {  // this rank's own slot; forwarded to the peers after the signal
                        store_own_tp(p, l, kind == kW2, g, c, lane == 0 ? ra : rb, lane == 0 ? acc_a : acc_b);
                    }
                    break;
                }
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
        if (kind != kLM && !(TP && p.tag_split && split)) signal_phase(p, ph);
        if (TP && split && !p.tag_split && lane < 2)
            forward_partials_tp(p, r.t0, r.t1, r.nb, r.T, kind == kW2, lane == 0 ? ra : rb);
        if (t == 0) trace_at(p, ph, kTrConsEnd);
    }
    // LM head: CTA argmax -> global max; the last CTA publishes the winner.
    if (lane == 0) best_s[warp] = best_i >= 0 ? pack_argmax(best_v, p.v0 + best_i) : 0ull;
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
            unsigned long long fin = atomicExch(&st->argmax_key, 0ull);
            // Tensor-parallel greedy step: the maximum over every rank's vocab shard.
            if (TP && p.tp > 1 && p.finish_greedy) fin = merge_argmax_tp(p, fin);
            const int tok = unpack_argmax_index(fin);
            st->argmax_final = fin;
            st->greedy_token = tok;
            st->epoch += 1;  // every CTA has read it for this step's cross-rank targets
            if (p.finish_greedy) {
                // Greedy step: the argmax is the step's id (no sampler launch follows).
                st->token_out = tok;
                const int local = tok - p.v0;
                if (local >= 0 && local < p.V) p.rep_flags[local] = 1;
                if (st->in.decode_mode) st->pos += 1;
            }
        }
    }
}

template <bool TP>
__global__ void __launch_bounds__(kThreads, 1) decode_persistent_kernel(const __grid_constant__ PersistentParams p) {
    extern __shared__ __align__(128) char smem[];
    char* ring = smem;
    float* xs = reinterpret_cast<float*>(smem + static_cast<size_t>(kSlots) * kSlotBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(xs + kMaxK);
    uint64_t* empty = full + kSlots;
    float* red = reinterpret_cast<float*>(empty + kSlots);                  // 16 floats
    unsigned long long* best_s = reinterpret_cast<unsigned long long*>(red + 16);  // 8
    int* s_ok = reinterpret_cast<int*>(best_s + kConsumerWarps);            // 1 (+pad)
    volatile int* quiet = s_ok + 8;                                           // producer pause flag
    // resid_smem: this CTA's copy of the residual stream [H], after the fixed layout
    float* xr = p.resid_smem ? reinterpret_cast<float*>(smem + kSmemBytes) : nullptr;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *quiet = 0;
    }
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait();
    // A stopped device-side generation: nothing to do this step (every CTA reads the same flag).
    if (p.st->in.skip) return;
    // Tensor parallel: every rank adds 1 to tp_sync in the step-start
    // all-reduce.  A smaller sum means a peer did not join (the host aborted
    // the communicator after its step timeout): leave before any load or any
    // store to peer memory.  Every CTA reads the same word.
    if (TP && p.tp > 1 && *reinterpret_cast<const volatile int*>(&p.st->tp_sync) != p.tp) {
        if (threadIdx.x == 0) atomicOr(&p.st->err, kErrPeer);
        return;
    }
    if (threadIdx.x < 32) {
        if (threadIdx.x == 0) producer<kSlots>(p, ring, full, empty, quiet);
    } else {
        consumers<TP>(p, ring, xs, full, empty, red, best_s, s_ok, quiet, xr);
    }
}


// ===========================================================================
// Batched persistent decode: kBatch sequences over one pass of the weights.
//
// The same weight stream as decode_persistent_kernel (producer, ring of TMA
// boxes, quiet window), with a 3-slot ring: shared memory holds every
// sequence's staged input instead ([kBatch][4096] floats, 128 KB).  Each box
// is dotted with all kBatch inputs: warp w owns rows 4 (w % 4) .. + 3 of the box
// over half of its K and keeps 4 x kBatch accumulators; one 32-value
// butterfly leaves lane l with (row l / 8, sequence l % 8), and the two halves
// meet in shared memory (a double-buffered hand-over).  The residual streams
// ping-pong in global memory (no room for them in shared memory): the last
// contributor of each row quad of a split projection finishes it (a ticket),
// and the next RMSNorm staging bulk-copies the eight finished vectors into
// shared memory.  Attention runs per (sequence, head, 128-position part) item,
// spread over the grid, four at once per CTA, with the cached K and V rows
// prefetched into L2 before the wait.  The LM head applies each sequence's
// penalty and keeps each sequence's argmax; a greedy step ends in the kernel.
constexpr int kSlotsB = 3;
constexpr size_t kSmemBytesB = static_cast<size_t>(kSlotsB) * kSlotBytes +
                               static_cast<size_t>(kBatch) * kBatchPersistMaxK * 4 + 2 * kSlotsB * 8 +
                               256 * 4 + kBatch * kConsumerWarps * 8 + 64;
static_assert(kSmemBytesB <= kMaxSmemPerBlock, "batched persistent kernel fits in 227 KB of shared memory");
static_assert(4 * kBatch == 32, "one (row, sequence) sum per lane of a row quad");
static_assert(kConsumerWarps == kBatch, "the RMSNorm staging gives each sequence one warp");

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

// Wait until phase ph's counter reaches target (bounded like every wait).
__device__ bool wait_count(const PersistentParams& p, int ph, int target, int* s_ok) {
    if (threadIdx.x == 32) {
        const int* c = p.done + ph;
        uint32_t it = 0;
        unsigned long long t0 = 0;
        int ok = 1;
        while (ld_acquire(c) < target) {
            ++it;
            if ((it & 255u) == 0) {
                const unsigned long long now = globaltimer();
                if (t0 == 0) t0 = now;
                if (it >= kFlagSpinLimit || now - t0 > kWaitLimitNs || aborted(p.st)) {
                    atomicOr(&p.st->err, kErrFlag);
                    ok = 0;
                    break;
                }
            }
        }
        *s_ok = ok;
    }
    consumer_sync();
    return *s_ok != 0;
}

// xs8[b] = rmsnorm(x_b) * gamma for every sequence b (src/rmsnorm.cu:99-101).
// Either x_b is the embedding row of b's input id (gather: loaded here, six
// quads of a lane per L2 round trip; this CTA also stores its slice of x_b to
// x_out), or it is the residual the previous split projection finished,
// already copied into xs8 by stage_copy8.  Warp w normalises sequence w alone
// (sum of squares reduced in the warp); the gains were prefetched into L1
// before the phase's wait.
__device__ __noinline__ void stage_norm8(const BatchPersistParams& bp, const float* gamma, float* xs8, float* x_out,
                                         bool gather) {
    const PersistentParams& p = bp.base;
    const int t = threadIdx.x - 32;
    const int b = t >> 5, lane = t & 31;  // kConsumerWarps == kBatch
    const int K = p.H, K4 = K >> 2;
    const int s0 = static_cast<int>(blockIdx.x) * K / static_cast<int>(gridDim.x);
    const int s1 = static_cast<int>(blockIdx.x + 1) * K / static_cast<int>(gridDim.x);
    float4* x4 = reinterpret_cast<float4*>(xs8 + static_cast<size_t>(b) * kBatchPersistMaxK);
    float ss = 0.0f;
    if (!gather)
        for (int q = lane; q < K4; q += 32) ss = dot4(x4[q], x4[q], ss);
    const float* src = gather ? p.emb + static_cast<size_t>(bp.st[b].in.token_in) * K : nullptr;
    constexpr int kU = 6;  // quads of a lane whose loads are issued together (two batches at H = 1536)
    for (int q0 = lane; gather && q0 < K4; q0 += 32 * kU) {
        float4 v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int q = q0 + 32 * u;
            if (q < K4) v[u] = __ldcg(reinterpret_cast<const float4*>(src) + q);
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int q = q0 + 32 * u;
            if (q < K4) {
                x4[q] = v[u];
                if (gather) {
                    const float e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        if (4 * q + c >= s0 && 4 * q + c < s1) x_out[static_cast<size_t>(b) * K + 4 * q + c] = e[c];
                    ss = dot4(v[u], v[u], ss);
                }
            }
        }
    }
    const float tot = warp_sum(ss);
    const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(tot / static_cast<float>(K)) + 1e-6));
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
    for (int q = lane; q < K4; q += 32) {
        const float4 g = __ldg(g4 + q);
        float4 v = x4[q];
        v.x = v.x * inv * g.x;
        v.y = v.y * inv * g.y;
        v.z = v.z * inv * g.z;
        v.w = v.w * inv * g.w;
        x4[q] = v;
    }
}

// A split projection's group g (16 rows, nc contributing CTAs): each
// contributor's lower-half warp for row quad `quad` stores its partial sums,
// then takes a ticket; the last one finishes the quad's rows for every
// sequence: x_new = x_old + (partials in CTA order + bias), as the
// single-sequence staging forms it, stored to x_out.  Lane l holds row
// r0 + l / 8 of sequence l % 8.  The tickets are zeroed before each launch.
__device__ void finish_quad(const BatchPersistParams& bp, int* ticket, int nc, int g, int my_r, int my_b,
                            const float* x_old, const float* bias, float* x_out) {
    const PersistentParams& p = bp.base;
    const int lane = threadIdx.x & 31;
    const size_t cstride = static_cast<size_t>(p.H / kPersistTileRows) * kPersistMaxContrib * kPersistTileRows;
    __threadfence();
    __syncwarp();
    int tk = 0;
    if (lane == 0) tk = atomicAdd(ticket, 1);
    tk = __shfl_sync(0xffffffffu, tk, 0);
    if (tk != nc - 1) return;
    __threadfence();
    const float* part = bp.cres + my_b * cstride + static_cast<size_t>(g) * kPersistMaxContrib * kPersistTileRows + my_r;
    float sp = __ldcg(part);
    for (int c = 1; c < nc; ++c) sp += __ldcg(part + c * kPersistTileRows);
    const int R = g * kPersistTileRows + my_r;
    const float x = __ldcg(x_old + static_cast<size_t>(my_b) * p.H + R) + (sp + bias[R]);
    x_out[static_cast<size_t>(my_b) * p.H + R] = x;
}

// xs8[b] = src_b[0, K) for every sequence b (src_b = src + b * K), by bulk
// copies of the tensor memory accelerator: the first consumer thread issues
// one cp.async.bulk per sequence onto an mbarrier that every consumer waits
// for.  The rows were written by other CTAs in the previous phase (generic
// proxy, ordered by that phase's counter): a proxy fence makes them visible
// to the copies.  Bounded wait; false on a timeout.
__device__ bool stage_copy8(const PersistentParams& p, const float* src, int K, float* xs8, uint64_t* bar,
                            uint32_t& bar_par) {
    const int t = threadIdx.x - 32;
    const uint32_t bytes = static_cast<uint32_t>(K) * 4u;
    if (t == 0) {
        asm volatile("fence.proxy.async.global;" ::: "memory");
        mbar_arrive_expect_tx(bar, bytes * kBatch);
        for (int b = 0; b < kBatch; ++b)
            asm volatile(
                "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                    smem_u32(xs8 + static_cast<size_t>(b) * kBatchPersistMaxK)),
                "l"(src + static_cast<size_t>(b) * K), "r"(bytes), "r"(smem_u32(bar))
                : "memory");
    }
    const bool ok = wait_parity(bar, bar_par, p.st);
    bar_par ^= 1u;
    return ok;
}

// The attention phase of one layer for every sequence.  Items (sequence b,
// head h, part j of nct_b): an item covers 128 positions, eight 16-position
// chunks.  Items are enumerated sequence by sequence and dealt to the CTAs
// round robin; a CTA runs four items at once, one per warp pair (slot), so
// that their load latencies overlap.  Each warp of a pair takes four chunks of
// the item in turn (RoPE at position n_b, the KV append by the chunk holding
// n_b, scores, softmax, P.V, src/attn.cu:490-547), keeping a running (max,
// sum, output); the pair merges in shared memory behind a named barrier of
// its own, and an item split over several CTAs merges through global memory
// (last-CTA ticket).  Every (sequence, head)'s final writer signals once: the
// phase's target is kBatch x heads.  Returns false if the wait for the QKV
// phase failed.
constexpr int kBAttnSlots = kConsumerWarps / 2;  // items in flight per CTA
constexpr int kBAttnChunks = 4;                  // chunks per warp of an item
static_assert(2 * kBAttnChunks == kConsumerWarps, "an item covers as many chunks as the single-sequence CTA");

__device__ __forceinline__ void pair_sync(int slot) {
    asm volatile("bar.sync %0, 64;" ::"r"(2 + slot) : "memory");
}

__device__ __noinline__ bool attention_batch(const BatchPersistParams& bp, int layer, int ph, float* xs, int* s_ok) {
    const PersistentParams& p = bp.base;
    const int t = threadIdx.x - 32;
    const int warp = t >> 5, lane = t & 31;
    const int slot = warp >> 1, half = warp & 1;
    const int G = gridDim.x;
    int nct[kBatch], ustart[kBatch + 1];
    ustart[0] = 0;
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
        const int nsplit = bp.st[b].pos / kPersistChunk + 1;
        nct[b] = (nsplit + kConsumerWarps - 1) / kConsumerWarps;
        ustart[b + 1] = ustart[b] + p.heads * nct[b];
    }
    const int U = ustart[kBatch];
    if (static_cast<int>(blockIdx.x) >= U) return true;  // no item: neither waits nor signals
    // The cached K and V rows of this warp's chunks (positions before n_b, which the QKV phase does not
    // touch) into L2 while that phase still runs: a lane pair takes the two 128-byte lines of one row.
    for (int k = slot;; k += kBAttnSlots) {
        const int u = static_cast<int>(blockIdx.x) + k * G;
        if (u >= U) break;
        int b = 0;
#pragma unroll
        for (int i = 1; i < kBatch; ++i)
            if (u >= ustart[i]) b = i;
        const int h = (u - ustart[b]) / nct[b], j = (u - ustart[b]) % nct[b];
        const int n = bp.st[b].pos;
        const size_t head_off = (static_cast<size_t>(b) * p.heads + h) * p.T * kHeadDim;
        const float* kc = bp.kc[layer] + head_off;
        const float* vc = bp.vc[layer] + head_off;
        for (int c = 0; c < kBAttnChunks; ++c) {
            const int row = (j * kConsumerWarps + half * kBAttnChunks + c) * kPersistChunk + (lane >> 1);
            if (row - (lane >> 1) > n) break;  // chunk past the new position
            if (row < n) {
                const size_t off = static_cast<size_t>(row) * kHeadDim + (lane & 1) * 32;
                asm volatile("prefetch.global.L2 [%0];" ::"l"(kc + off));
                asm volatile("prefetch.global.L2 [%0];" ::"l"(vc + off));
            }
        }
    }
    if (!wait_count(p, ph - 1, static_cast<int>(gridDim.x), s_ok)) return false;
    if (t == 0) trace_at(p, ph, kTrConsStart);
    float* qsh = xs + warp * kAttnWarpScratch;
    float* apart = xs + kConsumerWarps * kAttnWarpScratch;  // [8][68]
    float* knew = xs + kConsumerWarps * (kAttnWarpScratch + kAttnPartStride) + warp * kHeadDim;
    const int maxs = persistent_max_splits(p.T);
    const int kp = lane >> 1, kh = lane & 1;
    for (int k = slot;; k += kBAttnSlots) {
        const int u = static_cast<int>(blockIdx.x) + k * G;
        if (u >= U) break;
        int b = 0;
#pragma unroll
        for (int i = 1; i < kBatch; ++i)
            if (u >= ustart[i]) b = i;
        const int nb = nct[b];
        const int h = (u - ustart[b]) / nb, j = (u - ustart[b]) % nb;
        const int n = bp.st[b].pos;
        const int nsplit = n / kPersistChunk + 1;
        const size_t head_off = (static_cast<size_t>(b) * p.heads + h) * p.T * kHeadDim;
        float* kc = bp.kc[layer] + head_off;
        float* vc = bp.vc[layer] + head_off;
        const float* qkv = bp.qkv + static_cast<size_t>(b) * 3 * p.Hl;
        const float2 cs = p.rope[n * kHalfHead + lane];
        {
            const float* q = qkv + h * kHeadDim;
            const float qa = __ldcg(q + lane), qb = __ldcg(q + lane + kHalfHead);
            qsh[lane] = (qa * cs.x + qb * cs.y) * 0.125f;  // 1/sqrt(64) is exact
            qsh[lane + kHalfHead] = (-qa * cs.y + qb * cs.x) * 0.125f;
        }
        __syncwarp();
        const float4* q4 = reinterpret_cast<const float4*>(qsh) + 8 * kh;
        float m_run = -INFINITY, l_run = 0.0f;
        float2 o_run = make_float2(0.0f, 0.0f);
        for (int c = 0; c < kBAttnChunks; ++c) {
            const int s = j * kConsumerWarps + half * kBAttnChunks + c;
            if (s >= nsplit) break;
            const int t0 = s * kPersistChunk;
            const int posk = t0 + kp;
            const int cached = min(kPersistChunk, n - t0);
            const bool has_n = n >= t0 && n < t0 + kPersistChunk;
            // the chunk's cached K and V rows, all loads issued together (one memory round trip)
            float4 kv[8];
            float2 vrow[kPersistChunk];
            const float4* kr =
                reinterpret_cast<const float4*>(kc + static_cast<size_t>(kp < cached ? posk : 0) * kHeadDim) + 8 * kh;
#pragma unroll
            for (int i = 0; i < 8; ++i) kv[i] = kp < cached ? __ldcg(kr + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            const float2* vr = reinterpret_cast<const float2*>(vc + static_cast<size_t>(t0) * kHeadDim) + lane;
#pragma unroll
            for (int jp = 0; jp < kPersistChunk; ++jp)
                vrow[jp] = jp < cached ? __ldcg(vr + jp * (kHeadDim / 2)) : make_float2(0.0f, 0.0f);
            float2 vnew = make_float2(0.0f, 0.0f);
            if (has_n) {
                const float* kn = qkv + p.Hl + h * kHeadDim;
                const float* vn = qkv + 2 * p.Hl + h * kHeadDim;
                const float ka = __ldcg(kn + lane), kb = __ldcg(kn + lane + kHalfHead);
                vnew = __ldcg(reinterpret_cast<const float2*>(vn) + lane);
                const float k0 = ka * cs.x + kb * cs.y, k1 = -ka * cs.y + kb * cs.x;
                knew[lane] = k0;
                knew[lane + kHalfHead] = k1;
                kc[n * kHeadDim + lane] = k0;
                kc[n * kHeadDim + lane + kHalfHead] = k1;
                reinterpret_cast<float2*>(vc + n * kHeadDim)[lane] = vnew;
                __syncwarp();
                if (posk == n) {
                    const float4* k4 = reinterpret_cast<const float4*>(knew) + 8 * kh;
#pragma unroll
                    for (int i = 0; i < 8; ++i) kv[i] = k4[i];
                }
            }
            float d = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) d = dot4(kv[i], q4[i], d);
            d += __shfl_xor_sync(0xffffffffu, d, 1);
            const bool mine = posk <= n;
            const float sc = mine ? d : -INFINITY;
            const float m = warp_max(sc);
            const float e = mine ? expf(sc - m) : 0.0f;
            const float l = warp_sum(kh == 0 ? e : 0.0f);
            float2 o = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int jp = 0; jp < kPersistChunk; ++jp) {
                const float ej = __shfl_sync(0xffffffffu, e, 2 * jp);
                const float2 v = t0 + jp == n ? vnew : vrow[jp];
                o.x = fmaf(ej, v.x, o.x);
                o.y = fmaf(ej, v.y, o.y);
            }
            // running merge over this warp's chunks
            const float mn = fmaxf(m_run, m);
            const float sa = expf(m_run - mn), sb = expf(m - mn);
            l_run = l_run * sa + l * sb;
            o_run = make_float2(o_run.x * sa + o.x * sb, o_run.y * sa + o.y * sb);
            m_run = mn;
        }
        float* ap = apart + warp * kAttnPartStride;
        reinterpret_cast<float2*>(ap + 4)[lane] = o_run;
        if (lane == 0) {
            ap[0] = m_run;
            ap[1] = l_run;
        }
        pair_sync(slot);
        if (half == 0) {
            const float* a0 = apart + warp * kAttnPartStride;
            const float* a1 = a0 + kAttnPartStride;
            const float m0 = a0[0], m1 = a1[0];
            const float M = fmaxf(m0, m1);
            const float w0 = expf(m0 - M), w1 = expf(m1 - M);  // a warp without a chunk holds (-inf, 0, 0)
            const float L = a0[1] * w0 + a1[1] * w1;
            const float2 o0 = reinterpret_cast<const float2*>(a0 + 4)[lane];
            const float2 o1 = reinterpret_cast<const float2*>(a1 + 4)[lane];
            const float2 acc = make_float2(o0.x * w0 + o1.x * w1, o0.y * w0 + o1.y * w1);
            float2* out = reinterpret_cast<float2*>(bp.att + static_cast<size_t>(b) * p.Hl + h * kHeadDim);
            if (nb == 1) {
                out[lane] = make_float2(acc.x / L, acc.y / L);
                signal_warp(p, ph);
            } else {
                float* base = bp.part + (static_cast<size_t>(b) * p.heads + h) * maxs * (kHeadDim + 2);
                float* pp = base + j * (kHeadDim + 2);
                reinterpret_cast<float2*>(pp + 2)[lane] = acc;
                if (lane == 0) {
                    pp[0] = M;
                    pp[1] = L;
                }
                __syncwarp();
                int ticket = 0;
                if (lane == 0) {
                    __threadfence();
                    ticket = atomicAdd(bp.head_done + (layer * kBatch + b) * p.heads + h, 1);
                }
                ticket = __shfl_sync(0xffffffffu, ticket, 0);
                if (ticket == nb - 1) {
                    __threadfence();
                    const float mc = lane < nb ? __ldcg(base + lane * (kHeadDim + 2)) : -INFINITY;
                    const float lc = lane < nb ? __ldcg(base + lane * (kHeadDim + 2) + 1) : 0.0f;
                    const float M2 = warp_max(mc);
                    const float wc = lane < nb ? expf(mc - M2) : 0.0f;
                    const float L2 = warp_sum(lc * wc);
                    float2 acc2 = make_float2(0.0f, 0.0f);
                    for (int q = 0; q < nb; ++q) {
                        const float wt = __shfl_sync(0xffffffffu, wc, q);
                        const float2 ok = __ldcg(reinterpret_cast<const float2*>(base + q * (kHeadDim + 2) + 2) + lane);
                        acc2.x = fmaf(wt, ok.x, acc2.x);
                        acc2.y = fmaf(wt, ok.y, acc2.y);
                    }
                    out[lane] = make_float2(acc2.x / L2, acc2.y / L2);
                    signal_warp(p, ph);
                }
            }
        }
        pair_sync(slot);  // the pair's scratch is reused by its next item
    }
    return true;
}

__device__ void consumers_batch(const BatchPersistParams& bp, char* ring, float* xs8, uint64_t* full, uint64_t* empty,
                                float* red8, unsigned long long* best8, int* s_ok, volatile int* quiet,
                                uint64_t* copy_bar) {
    uint32_t copy_par = 0;  // phase parity of the staging copies' mbarrier
    const PersistentParams& p = bp.base;
    DevState* st0 = bp.st;  // sequence 0's state holds the step's error word
    const int t = threadIdx.x - 32;
    const int warp = t >> 5, lane = t & 31;
    const int G = gridDim.x;
    const size_t cstride = static_cast<size_t>(p.H / kPersistTileRows) * kPersistMaxContrib * kPersistTileRows;
    int slot = 0;
    uint32_t par = 0;
    bool ok = true;
    // LM head: lane l of a lower-half warp keeps the running argmax of sequence l % 8 over the rows it finishes.
    float best_v = -INFINITY;
    int best_i = -1;
    const int last = 5 * p.layers;
    for (int ph = 0; ph <= last; ++ph) {
        const int kind = phase_kind(ph, p.layers);
        const int l = ph / 5;
        if (kind == kAttn) {
            if (!attention_batch(bp, l, ph, xs8, s_ok)) return;
            if (t == 0) *quiet = 0;
            if (t == 0) trace_at(p, ph, kTrConsEnd);
            continue;
        }
        const LayerPtrs* y = ph < last ? &p.layer[l] : nullptr;
        const Gemv d = gemv_of(p, ph);
        const Boxes r = boxes_of(d);
        if (ph > 0) {
            if (kind == kQKV || kind == kW13 || kind == kLM) {  // the staging's gains into L1 during the wait
                const float* gm = kind == kQKV ? y->g1 : kind == kW13 ? y->g2 : p.gnorm;
                for (int i = t; i < (p.H >> 5); i += kConsumerWarps * 32)
                    asm volatile("prefetch.global.L1 [%0];" ::"l"(gm + 32 * i));
            }
            // the attention phase is signalled once per (sequence, head) item; the others once per CTA
            const int target = phase_kind(ph - 1, p.layers) == kAttn ? kBatch * p.heads : G;
            if (!wait_count(p, ph - 1, target, s_ok)) return;
        }
        if (t == 0) trace_at(p, ph, kTrConsStart);
        // The residual streams: the W2 phase finishes xa (from xb), the out-projection finishes xb (from xa).
        if (kind == kQKV && l == 0) {
            stage_norm8(bp, y->g1, xs8, bp.xa, true);
        } else if (kind == kWo) {
            if (!stage_copy8(p, bp.att, p.Hl, xs8, copy_bar, copy_par)) ok = false;
        } else if (kind == kW2) {
            if (!stage_copy8(p, bp.ffh, p.Fl, xs8, copy_bar, copy_par)) ok = false;
        } else {  // QKV (layers past the first), W1/V, LM head: the finished residual copied in, then normalised
            const bool xa = kind != kW13;
            if (!stage_copy8(p, xa ? bp.xa : bp.xb, p.H, xs8, copy_bar, copy_par)) ok = false;
            else stage_norm8(bp, kind == kQKV ? y->g1 : kind == kW13 ? y->g2 : p.gnorm, xs8, nullptr, false);
        }
        consumer_sync();
        if (t == 0) *quiet = 0;
        if (t == 0) trace_at(p, ph, kTrConsStaged);
        const int rs4 = r.bw / 4;
        // Warp w owns rows 4 (w % 4) .. 4 (w % 4) + 3 of each box over half of its K (w / 4); after a group's
        // boxes, a 32-value butterfly leaves lane l with (row l / 8, sequence l % 8) of that half, the upper
        // half's warp hands its sums over in shared memory, and the lower half's warp finishes the group.
        const int quad = warp & 3, khalf = warp >> 2;
        const int r0 = 4 * quad;
        const int my_r = r0 + (lane >> 3), my_b = lane & 7;
        const float my_rp = bp.st[my_b].in.rp;
        int xbuf = 0;  // hand-over buffer of the current group: [2][4 quads][32 lanes], alternating
        for (int tau = r.t0; tau < r.t1;) {
            const int g = tau / r.nb;
            const int bi0 = tau % r.nb, bi1 = min(r.nb, bi0 + (r.t1 - tau));
            const int rows = min(kPersistTileRows, d.M - g * kPersistTileRows);
            const int Rl = g * kPersistTileRows + my_r;
            const bool vl = my_r < rows;
            float el = 0.0f;  // bias of the lane's row, or its sequence's repetition flag in the LM head
            if (khalf == 0) {
                if (kind == kLM) {
                    if (vl) el = bp.rep[static_cast<size_t>(my_b) * p.V + Rl] ? 1.0f : 0.0f;
                } else if (kind == kQKV || kind == kW13) {
                    if (vl) el = d.bias[Rl];
                }
            }
            float acc[32];
#pragma unroll
            for (int i2 = 0; i2 < 32; ++i2) acc[i2] = 0.0f;
            for (int bi = bi0; bi < bi1; ++bi) {
                if (ok && !wait_parity(&full[slot], par, st0)) ok = false;
                if (t == 0 && kind != kLM && tau + (bi - bi0) == r.t1 - 1) *quiet = 1;
                if (ok) {
                    const int k0 = bi * r.bw;
                    const int kc4 = min(r.bw, d.K - k0) >> 2;
                    const int hq = rs4 >> 1;  // float4 per half row
                    const float4* tile = reinterpret_cast<const float4*>(ring + static_cast<size_t>(slot) * kSlotBytes);
#pragma unroll
                    for (int j0 = 0; j0 < kBoxK / 8; j0 += 32) {
                        const int j = khalf * hq + j0 + lane;
                        if (j0 + lane < hq && j < kc4) {
                            float4 w4[4];
#pragma unroll
                            for (int rr = 0; rr < 4; ++rr) w4[rr] = tile[(r0 + rr) * rs4 + j];
#pragma unroll
                            for (int b = 0; b < kBatch; ++b) {
                                const float4 xv = reinterpret_cast<const float4*>(
                                    xs8 + static_cast<size_t>(b) * kBatchPersistMaxK)[(k0 >> 2) + j];
#pragma unroll
                                for (int rr = 0; rr < 4; ++rr) acc[rr * 8 + b] = dot4(w4[rr], xv, acc[rr * 8 + b]);
                            }
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[slot]);
                }
                if (++slot == kSlotsB) {
                    slot = 0;
                    par ^= 1u;
                }
            }
            tau += bi1 - bi0;
            float sum = reduce_scatter32(acc);  // lane l: row r0 + l / 8, sequence l % 8, this half of K
            // Two buffers: the upper warp writes group i + 2's sums only after the barrier of group i + 1, which
            // the lower warp reaches after reading group i's.
            float* xch = red8 + (xbuf * 4 + quad) * 32;
            xbuf ^= 1;
            if (khalf == 1) xch[lane] = sum;
            pair_sync(4 + quad);  // warps quad and quad + 4
            if (khalf == 0) {
                sum += xch[lane];
                switch (kind) {
                    case kQKV:
                        if (vl) bp.qkv[static_cast<size_t>(my_b) * 3 * p.Hl + Rl] = sum + el;
                        break;
                    case kWo:
                    case kW2: {
                        const int c = persist_contrib_slot(blockIdx.x, g, bi0, r.nb, r.T, G);
                        bp.cres[my_b * cstride + (static_cast<size_t>(g) * kPersistMaxContrib + c) * kPersistTileRows +
                                my_r] = sum;
                        const bool w2 = kind == kW2;
                        int* tk = bp.tickets + ((static_cast<size_t>(w2) * p.layers + l) * (p.H / kPersistTileRows) + g) * 4 +
                                  quad;
                        finish_quad(bp, tk, persist_group_contrib(g, r.nb, r.T, G), g, my_r, my_b,
                                    w2 ? bp.xb : bp.xa, w2 ? y->b2 : y->bo, w2 ? bp.xa : bp.xb);
                        break;
                    }
                    case kW13: {
                        // rows (2i, 2i + 1) = (W1 row i, V row i) sit in lanes l and l + 8 (same sequence)
                        const float gate = __shfl_xor_sync(0xffffffffu, sum + el, 8);
                        if ((my_r & 1) == 1 && vl)
                            bp.ffh[static_cast<size_t>(my_b) * p.Fl + (Rl >> 1)] = silu(gate) * (sum + el);
                        break;
                    }
                    default: {  // kLM: logits with the sequence's repetition penalty, running argmax
                        if (vl) {
                            float v = sum;
                            if (el != 0.0f) v = rep_penalty(v, my_rp);
                            bp.logits[static_cast<size_t>(my_b) * p.V + Rl] = v;
                            if (v > best_v) best_v = v, best_i = Rl;
                        }
                    }
                }
            }
        }
        if (kind != kLM) {
            consumer_sync();  // every warp's stores of the phase, then one release per CTA
            if (t == 0) asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(p.done + ph) : "memory");
        }
        if (t == 0) trace_at(p, ph, kTrConsEnd);
    }
    // LM head: per sequence, the lanes of a warp -> the warp -> the CTA -> the grid maximum; the last CTA
    // finishes the step.  Lane l of a lower-half warp holds sequence l % 8.
    unsigned long long k = best_i >= 0 ? pack_argmax(best_v, best_i) : 0ull;
#pragma unroll
    for (int off = 8; off < 32; off <<= 1) {
        const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, k, off);
        k = k2 > k ? k2 : k;
    }
    if (lane < kBatch) best8[warp * kBatch + lane] = k;
    consumer_sync();
    if (t < kBatch) {
        unsigned long long m = 0;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) m = best8[w * kBatch + t] > m ? best8[w * kBatch + t] : m;
        if (m) atomicMax(&bp.st[t].argmax_key, m);
    }
    consumer_sync();
    if (t == 0) {
        __threadfence();
        const int ticket = atomicAdd(p.done + last, 1);
        if (ticket == G - 1) {
            __threadfence();
            for (int b = 0; b < kBatch; ++b) {
                DevState* sb = bp.st + b;
                const unsigned long long fin = atomicExch(&sb->argmax_key, 0ull);
                const int tok = unpack_argmax_index(fin);
                sb->argmax_final = fin;
                sb->greedy_token = tok;
                if (bp.finish_greedy) {
                    sb->token_out = tok;
                    if (tok >= 0 && tok < p.V) bp.rep[static_cast<size_t>(b) * p.V + tok] = 1;
                    if (sb->in.decode_mode) sb->pos += 1;
                }
            }
        }
    }
}

__global__ void __launch_bounds__(kThreads, 1) decode_batch_persistent_kernel(const __grid_constant__ BatchPersistParams bp) {
    extern __shared__ __align__(128) char smem[];
    char* ring = smem;
    float* xs8 = reinterpret_cast<float*>(smem + static_cast<size_t>(kSlotsB) * kSlotBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(xs8 + static_cast<size_t>(kBatch) * kBatchPersistMaxK);
    uint64_t* empty = full + kSlotsB;
    float* red8 = reinterpret_cast<float*>(empty + kSlotsB);  // [2][4 row quads][32]: K-half hand-over
    unsigned long long* best8 = reinterpret_cast<unsigned long long*>(red8 + 256);  // [8 warps][kBatch]
    int* s_ok = reinterpret_cast<int*>(best8 + kBatch * kConsumerWarps);
    volatile int* quiet = s_ok + 8;
    uint64_t* copy_bar = reinterpret_cast<uint64_t*>(s_ok + 12);  // 8-byte aligned: s_ok is
    if (threadIdx.x == 0) {
        for (int s = 0; s < kSlotsB; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        mbar_init(copy_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *quiet = 0;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        if (threadIdx.x == 0) producer<kSlotsB>(bp.base, ring, full, empty, quiet);
    } else {
        consumers_batch(bp, ring, xs8, full, empty, red8, best8, s_ok, quiet, copy_bar);
    }
}

}  // namespace

size_t persistent_smem_bytes(int H, int resid_smem) {
    return kSmemBytes + (resid_smem ? static_cast<size_t>(H) * sizeof(float) : 0);
}

cudaError_t launch_decode_persistent(const PersistentParams& p, int num_sms, cudaStream_t s) {
    if (p.H <= 0 || p.Hl <= 0 || p.Fl <= 0 || p.H > kMaxK || p.Hl > kMaxK || p.Fl > kMaxK ||
        p.H % kPersistKAlign || p.Hl % kPersistKAlign || p.Fl % kPersistKAlign)
        return cudaErrorInvalidValue;
    // Attention: at most one item per CTA, at most 32 CTAs per head (one lane each in the merge).
    const int nct = persist_attn_ctas_per_head(p.T);
    if (p.heads * nct > num_sms || nct > 32) return cudaErrorInvalidValue;
    if (p.inflight < 1 || p.inflight > kSlots) return cudaErrorInvalidValue;
    if (p.tp < 1 || p.tp > kMaxTp || p.rank < 0 || p.rank >= p.tp) return cudaErrorInvalidValue;
    const bool exchange = p.tp > 1 || p.tag_split;  // the instantiation with tagged partial sums
    for (int r = 0; r < p.tp && exchange; ++r)
        if (!p.xc[r]) return cudaErrorInvalidValue;
    if (p.tag_split && !p.resid_smem) return cudaErrorInvalidValue;  // tag-ordered stagings read no global residual
    if (persist_max_contrib(p.H, p.Hl, num_sms) > kPersistMaxContrib ||
        persist_max_contrib(p.H, p.Fl, num_sms) > kPersistMaxContrib)
        return cudaErrorInvalidValue;
    const size_t smem = persistent_smem_bytes(p.H, p.resid_smem);
    if (smem > kMaxSmemPerBlock) return cudaErrorInvalidValue;
    auto kern = exchange ? decode_persistent_kernel<true> : decode_persistent_kernel<false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    return cudaLaunchKernelEx(&cfg, kern, p);
}

size_t batch_persistent_smem_bytes() { return kSmemBytesB; }

cudaError_t launch_decode_batch_persistent(const BatchPersistParams& bp, int num_sms, cudaStream_t s) {
    const PersistentParams& p = bp.base;
    if (p.H <= 0 || p.Hl <= 0 || p.Fl <= 0 || p.H > kBatchPersistMaxK || p.Hl > kBatchPersistMaxK ||
        p.Fl > kBatchPersistMaxK || p.H % kPersistKAlign || p.Hl % kPersistKAlign || p.Fl % kPersistKAlign)
        return cudaErrorInvalidValue;
    // one GPU; the error word and the producer's state are sequence 0's; at most 32 CTAs per attention item
    if (p.tp != 1 || p.st != bp.st || persist_attn_ctas_per_head(p.T) > 32) return cudaErrorInvalidValue;
    if (p.inflight < 1 || p.inflight > kSlotsB) return cudaErrorInvalidValue;
    if (persist_max_contrib(p.H, p.Hl, num_sms) > kPersistMaxContrib ||
        persist_max_contrib(p.H, p.Fl, num_sms) > kPersistMaxContrib)
        return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(decode_batch_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmemBytesB));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytesB;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    return cudaLaunchKernelEx(&cfg, decode_batch_persistent_kernel, bp);
}

}  // namespace xl
