// Host side of the XingLing engine: weights and KV cache resident in HBM,
// one CUDA graph per decode step, direct launches for prefill, NCCL for
// tensor parallelism.  Mirrors the reference's InferenceEngine / Transformer
// (src/inference.cu:18-151, src/transformer.cu:107-186) with status codes
// instead of exit(1).
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <memory>
#include <mutex>
#include <thread>
#include <utility>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "engine.h"

namespace xl {

namespace {
thread_local std::string g_err;
constexpr double kEps = 1e-6;  // RMSNorm eps, src/rmsnorm.cu:72,100
constexpr size_t kLoadChunkBytes = 8u << 20;  // weight-file bytes per staging chunk of the loader

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// NVTX ranges (domain "xingling") around every public call, so that an
// nsys / ncu timeline lines up with the engine's steps: "load", "prefill",
// "extend", "decode", "generate"; the payload is the call's first position
// (prefill: the prompt length).  Without an attached tool each push / pop is
// a branch on a null function pointer.
nvtxDomainHandle_t nvtx_domain() {
    static nvtxDomainHandle_t d = nvtxDomainCreateA("xingling");
    return d;
}
struct NvtxRange {
    NvtxRange(const char* name, long long payload) {
        nvtxEventAttributes_t a{};
        a.version = NVTX_VERSION;
        a.size = NVTX_EVENT_ATTRIB_STRUCT_SIZE;
        a.messageType = NVTX_MESSAGE_TYPE_ASCII;
        a.message.ascii = name;
        a.payloadType = NVTX_PAYLOAD_TYPE_INT64;
        a.payload.llValue = payload;
        nvtxDomainRangePushEx(nvtx_domain(), &a);
    }
    ~NvtxRange() { nvtxDomainRangePop(nvtx_domain()); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};
}  // namespace

void set_error(const std::string& msg) { g_err = msg; }
const char* last_error() { return g_err.c_str(); }
void clear_error() { g_err.clear(); }

// ---------------------------------------------------------------------------
uint32_t philox4x32_10_x0(uint64_t ctr, uint64_t seed) {
    uint32_t c0 = static_cast<uint32_t>(ctr), c1 = static_cast<uint32_t>(ctr >> 32), c2 = 0, c3 = 0;
    uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
    for (int round = 0; round < 10; ++round) {
        const uint64_t p0 = static_cast<uint64_t>(0xD2511F53u) * c0;
        const uint64_t p1 = static_cast<uint64_t>(0xCD9E8D57u) * c2;
        const uint32_t hi0 = static_cast<uint32_t>(p0 >> 32), lo0 = static_cast<uint32_t>(p0);
        const uint32_t hi1 = static_cast<uint32_t>(p1 >> 32), lo1 = static_cast<uint32_t>(p1);
        c0 = hi1 ^ c1 ^ k0;
        c1 = lo1;
        c2 = hi0 ^ c3 ^ k1;
        c3 = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c0;
}

float philox_uniform(uint64_t ctr, uint64_t seed) {
    return static_cast<float>(philox4x32_10_x0(ctr, seed) >> 8) * (1.0f / 16777216.0f);
}

void fill_rope_table(float base, int max_ctx, float* out) {
    for (int pos = 0; pos < max_ctx; ++pos) {
        for (int j = 0; j < kHalfHead; ++j) {
            // theta formed in fp32 as src/rope.cu:57 (powf, then * pos).
            const float theta = std::pow(base, -2.0f * j / 64) * static_cast<float>(pos);
            out[(pos * kHalfHead + j) * 2 + 0] = std::cos(theta);
            out[(pos * kHalfHead + j) * 2 + 1] = std::sin(theta);
        }
    }
}

// ---------------------------------------------------------------------------
int Engine::cuda_fail(cudaError_t e, const char* what) {
    set_error(std::string("CUDA error in ") + what + ": " + cudaGetErrorString(e));
    return XL_ERR_CUDA;
}

int Engine::nccl_fail(ncclResult_t r, const char* what) {
    set_error(std::string("NCCL error in ") + what + ": " + ncclGetErrorString(r));
    return XL_ERR_NCCL;
}

#define XL_CUDA(call)                                        \
    do {                                                     \
        cudaError_t e_ = (call);                             \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call);  \
    } while (0)

#define XL_NCCL(call)                                        \
    do {                                                     \
        ncclResult_t r_ = (call);                            \
        if (r_ != ncclSuccess) return nccl_fail(r_, #call);  \
    } while (0)

int make_tp_plan(const xl_config& cfg, int tp, int rank, TpPlan* out) {
    if (tp < 1 || rank < 0 || rank >= tp || cfg.heads % tp || cfg.ffn % tp) {
        set_error("tensor parallel: tp_size must divide heads and ffn, 0 <= rank < tp_size");
        return XL_ERR_ARG;
    }
    if (cfg.hidden % 8 || (cfg.ffn / tp) % 8) {
        set_error("config: hidden and the per-rank ffn width must be multiples of 8");
        return XL_ERR_ARG;
    }
    const int vper = (cfg.vocab + tp - 1) / tp;
    out->heads = cfg.heads / tp;
    out->hidden = out->heads * kHeadDim;
    out->ffn = cfg.ffn / tp;
    out->vocab_begin = rank * vper;
    out->vocab_count = std::max(0, std::min(vper, cfg.vocab - rank * vper));
    if (out->vocab_count <= 0) {
        set_error("tensor parallel: empty vocab shard");
        return XL_ERR_ARG;
    }
    return XL_OK;
}

int Engine::create(const xl_config& cfg, int device, int tp_size, int tp_rank, const void* nccl_id, Engine** out) {
    *out = nullptr;
    Engine* e = new Engine();
    int rc = e->init(cfg, device, tp_size, tp_rank, nccl_id);
    if (rc != XL_OK) {
        delete e;
        return rc;
    }
    *out = e;
    return XL_OK;
}

int Engine::init(const xl_config& cfg, int device, int tp_size, int tp_rank, const void* nccl_id) {
    if (cfg.layers <= 0 || cfg.hidden <= 0 || cfg.heads <= 0 || cfg.ffn <= 0 || cfg.vocab <= 0 || cfg.max_ctx <= 0) {
        set_error("config: every size must be positive");
        return XL_ERR_ARG;
    }
    if (cfg.hidden != cfg.heads * kHeadDim) {
        set_error("config: hidden must equal heads * 64");
        return XL_ERR_ARG;
    }
    TpPlan plan;
    const int prc = make_tp_plan(cfg, tp_size, tp_rank, &plan);
    if (prc != XL_OK) return prc;
    cfg_ = cfg;
    device_ = device;
    tp_ = tp_size;
    rank_ = tp_rank;
    H_ = cfg.hidden;
    heads_l_ = plan.heads;
    Hl_ = plan.hidden;
    F_ = cfg.ffn;
    Fl_ = plan.ffn;
    V_ = cfg.vocab;
    T_ = cfg.max_ctx;
    v0_ = plan.vocab_begin;
    vl_ = plan.vocab_count;
    int ndev = 0;
    XL_CUDA(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) {
        set_error("device ordinal out of range");
        return XL_ERR_ARG;
    }
    XL_CUDA(cudaSetDevice(device_));
    XL_CUDA(cudaDeviceGetAttribute(&num_sms_, cudaDevAttrMultiProcessorCount, device_));
    XL_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    XL_CUDA(cudaEventCreate(&ev0_));
    XL_CUDA(cudaEventCreate(&ev1_));
    XL_CUDA(cudaEventCreate(&kev0_));
    XL_CUDA(cudaEventCreate(&kev1_));
    XL_CUDA(cudaEventCreateWithFlags(&ev_sync_, cudaEventDisableTiming));
    XL_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h_in_), sizeof(DevState), cudaHostAllocDefault));
    XL_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h_out_), sizeof(DevState), cudaHostAllocDefault));
    XL_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h_gen_), sizeof(GenCtl) + 2 * static_cast<size_t>(T_) * 4,
                          cudaHostAllocDefault));
    XL_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h_ids_), sizeof(int) * (T_ + 1), cudaHostAllocDefault));
    std::random_device rd;
    philox_seed_ = (static_cast<uint64_t>(rd()) << 32) ^ rd();
    int rc = alloc_all();
    if (rc != XL_OK) return rc;
    const int one = 1;  // this rank's share of the step-start liveness sum
    XL_CUDA(cudaMemcpy(&st_->tp_one, &one, sizeof(int), cudaMemcpyHostToDevice));
    if (tp_ > 1) {
        if (nccl_id == nullptr) {
            set_error("tensor parallel: nccl_id is required when tp_size > 1");
            return XL_ERR_ARG;
        }
        ncclUniqueId id;
        std::memcpy(&id, nccl_id, sizeof(id));
        // Every rank must draw the same uniforms: seed Philox from the shared id (FNV-1a).
        uint64_t h = 1469598103934665603ull;
        for (size_t i = 0; i < sizeof(id); ++i) h = (h ^ static_cast<unsigned char>(id.internal[i])) * 1099511628211ull;
        philox_seed_ = h;
        XL_NCCL(ncclCommInitRank(&comm_, tp_, id, rank_));
        if (xbuf_) {
            rc = setup_peers();
            if (rc != XL_OK) return rc;
        }
    }
    return XL_OK;
}

// Every rank exports its exchange buffer (CUDA IPC) and maps every other
// rank's; the handles are all-gathered over the engine's NCCL communicator
// together with each rank's kernel geometry.  The persistent kernel's
// exchange slots are laid out by the grid (one CTA per SM) and the shard
// widths, and a reader sums the slots its own grid implies: ranks whose SM
// counts or shapes differ would silently drop or misread contributions, so
// creation fails instead.
namespace {
struct PeerInfo {
    cudaIpcMemHandle_t handle;
    int sms, hidden, hidden_local, ffn_local, layers, max_ctx, tp, rank;
};
}  // namespace

int Engine::setup_peers() {
    PeerInfo mine{};
    XL_CUDA(cudaIpcGetMemHandle(&mine.handle, xbuf_));
    mine.sms = num_sms_;
    mine.hidden = H_;
    mine.hidden_local = Hl_;
    mine.ffn_local = Fl_;
    mine.layers = cfg_.layers;
    mine.max_ctx = T_;
    mine.tp = tp_;
    mine.rank = rank_;
    constexpr size_t kH = sizeof(PeerInfo);
    char* dev = nullptr;
    XL_CUDA(cudaMalloc(reinterpret_cast<void**>(&dev), kH * tp_));
    std::vector<PeerInfo> all(tp_);
    cudaError_t ce = cudaMemcpy(dev + kH * rank_, &mine, kH, cudaMemcpyHostToDevice);
    ncclResult_t nr = ncclSuccess;
    if (ce == cudaSuccess) nr = ncclAllGather(dev + kH * rank_, dev, kH, ncclUint8, comm_, stream_);
    if (ce == cudaSuccess && nr == ncclSuccess) ce = cudaStreamSynchronize(stream_);
    if (ce == cudaSuccess && nr == ncclSuccess) ce = cudaMemcpy(all.data(), dev, kH * tp_, cudaMemcpyDeviceToHost);
    cudaFree(dev);
    if (nr != ncclSuccess) return nccl_fail(nr, "ncclAllGather (exchange buffer handles)");
    if (ce != cudaSuccess) return cuda_fail(ce, "exchange buffer handles");
    for (int r = 0; r < tp_; ++r) {
        const PeerInfo& q = all[r];
        if (q.sms != mine.sms || q.hidden != mine.hidden || q.hidden_local != mine.hidden_local ||
            q.ffn_local != mine.ffn_local || q.layers != mine.layers || q.max_ctx != mine.max_ctx ||
            q.tp != mine.tp || q.rank != r) {
            set_error("tensor parallel: rank " + std::to_string(r) + " has " + std::to_string(q.sms) + " SMs, hidden " +
                      std::to_string(q.hidden) + "/" + std::to_string(q.hidden_local) + ", ffn shard " +
                      std::to_string(q.ffn_local) + ", " + std::to_string(q.layers) + " layers, context " +
                      std::to_string(q.max_ctx) + " (rank " + std::to_string(q.rank) + " of " + std::to_string(q.tp) +
                      "); rank " + std::to_string(rank_) + " has " + std::to_string(mine.sms) + " SMs, hidden " +
                      std::to_string(mine.hidden) + "/" + std::to_string(mine.hidden_local) + ", ffn shard " +
                      std::to_string(mine.ffn_local) + ", " + std::to_string(mine.layers) + " layers, context " +
                      std::to_string(mine.max_ctx) + ": every rank needs the same GPU model and the same shape");
            return XL_ERR_ARG;
        }
    }
    for (int r = 0; r < tp_; ++r) {
        if (r == rank_) {
            xpeer_[r] = xbuf_;
            continue;
        }
        void* ptr = nullptr;
        XL_CUDA(cudaIpcOpenMemHandle(&ptr, all[r].handle, cudaIpcMemLazyEnablePeerAccess));
        xpeer_[r] = static_cast<char*>(ptr);
    }
    peers_ = true;
    return XL_OK;
}

int Engine::alloc_all() {
    const size_t H = H_, Hl = Hl_, Fl = Fl_, T = T_, V = V_, vl = vl_;
    const int maxs = std::max(attn_max_splits(T_), persistent_max_splits(T_));
    std::vector<std::pair<void**, size_t>> plan;
    auto add = [&](void* slot, size_t bytes) { plan.emplace_back(reinterpret_cast<void**>(slot), bytes); };
    add(&emb_, V * H * 4);
    add(&gnorm_, H * 4);
    add(&rope_, T * kHalfHead * 8);
    layers_.assign(cfg_.layers, LayerWeights{});
    for (auto& L : layers_) {
        add(&L.wqkv, 3 * Hl * H * 4);
        add(&L.bqkv, 3 * Hl * 4);
        add(&L.wo, H * Hl * 4);
        add(&L.bo, H * 4);
        add(&L.w13, 2 * Fl * H * 4);
        add(&L.b13, 2 * Fl * 4);
        add(&L.w2, H * Fl * 4);
        add(&L.b2, H * 4);
        add(&L.g1, H * 4);
        add(&L.g2, H * 4);
        add(&L.kc, heads_l_ * T * kHeadDim * 4);
        add(&L.vc, heads_l_ * T * kHeadDim * 4);
        add(&L.wqkv_lo, 3 * Hl * H * 4);
        add(&L.wo_lo, H * Hl * 4);
        add(&L.w13_lo, 2 * Fl * H * 4);
        add(&L.w2_lo, H * Fl * 4);
        add(&L.bo_full, tp_ > 1 ? H * 4 : 0);
        add(&L.b2_full, tp_ > 1 ? H * 4 : 0);
    }
    add(&xa_, H * 4);
    add(&xb_, H * 4);
    add(&qkv_, 3 * Hl * 4);
    add(&att_, Hl * 4);
    add(&ffh_, Fl * 4);
    add(&part_, H * 4);
    add(&cand_local_, kTopK * 8);
    add(&gen_ctl_, sizeof(GenCtl));
    add(&gen_u_, T * 4);
    add(&gen_out_, T * 4);
    add(&cand_all_, static_cast<size_t>(tp_) * kTopK * 8);
    add(&cres_, H / kPersistTileRows * kPersistMaxContrib * kPersistTileRows * 4);
    add(&logits_, vl * 4);
    add(&attn_ws_, static_cast<size_t>(heads_l_) * maxs * (kHeadDim + 2) * 4);
    add(&attn_cnt_, heads_l_ * 4);
    add(&done_, done_words() * 4);
    add(&rep_flags_, vl);
    add(&st_, sizeof(DevState));
    samp_grid_ = sample_grid(vl_, num_sms_, 1);
    add(&samp_work_, sample_work_bytes(vl_, samp_grid_));
    add(&px_, T * H * 4);
    add(&pxn_, T * H * 4);
    add(&pqkv_, T * 3 * Hl * 4);
    add(&patt_, T * H * 4);
    add(&pffh_, T * Fl * 4);
    splitk_floats_ = static_cast<size_t>(16) << 20;  // 64 MB
    add(&splitk_ws_, splitk_floats_ * 4);
    add(&pxn_lo_, T * H * 4);
    add(&patt_lo_, T * H * 4);
    add(&pffh_lo_, T * Fl * 4);
    add(&pids_, T * 4);
    // tensor-core prefill attention (transient, shared by the layers)
    add(&aq_, T * Hl * 4);
    add(&aq_lo_, T * Hl * 4);
    add(&ak_, T * Hl * 4);
    add(&ak_lo_, T * Hl * 4);
    add(&avt_, T * Hl * 4);
    add(&avt_lo_, T * Hl * 4);
    add(&ap_, static_cast<size_t>(heads_l_) * T * T * 4);  // S / P, or the fused kernel's split rows
    add(&ap_lo_, static_cast<size_t>(heads_l_) * T * T * 4);
    add(&fa_tickets_, static_cast<size_t>(heads_l_) * ((T + 127) / 128) * 4 * 4);
    size_t total = 0;
    for (auto& pr : plan) total += align_up(pr.second, 256);
    XL_CUDA(cudaMalloc(reinterpret_cast<void**>(&arena_), total));
    arena_bytes_ = total;
    XL_CUDA(cudaMemset(arena_, 0, total));
    if (tp_ <= kMaxTp) {
        // Its own allocation, so that the peers can map it (an IPC handle covers a whole allocation);
        // one GPU uses it too when the split projections' partial sums are ordered by tags (tag_split).
        // the partial-sum slots, then the greedy merge area: (key, tag) per rank
        const size_t xc = 2 * static_cast<size_t>(tp_) * (H / kPersistTileRows) * kPersistMaxContrib *
                              kPersistTileRows * 8 +
                          2 * kMaxTp * 8;
        XL_CUDA(cudaMalloc(reinterpret_cast<void**>(&xbuf_), xc));
        XL_CUDA(cudaMemset(xbuf_, 0, xc));  // tag 0: no use has written a word yet
    }
    size_t off = 0;
    for (auto& pr : plan) {
        *pr.first = arena_ + off;
        off += align_up(pr.second, 256);
    }
    std::vector<float> table(static_cast<size_t>(T_) * kHalfHead * 2);
    fill_rope_table(cfg_.rope_base, T_, table.data());
    XL_CUDA(cudaMemcpy(rope_, table.data(), table.size() * 4, cudaMemcpyHostToDevice));
    return XL_OK;
}

Engine::~Engine() {
    cudaSetDevice(device_);
    // A tensor-parallel stream may still wait on a peer that never joined:
    // wait a bounded time, abort the communicator if it is still busy, and
    // leak the device memory rather than block in cudaFree if it never drains.
    if (stream_ && tp_ > 1 && stream_idle_ && !drain_stream(failed_ ? 10000 : 60000)) {
        if (comm_)
            abort_tp("engine destroyed while a step was still running");  // drains again, sets stream_idle_
        else
            stream_idle_ = false;
    }
    if (!stream_idle_) {
        for (int r = 0; r < kMaxTp; ++r)
            if (xpeer_[r] && xpeer_[r] != xbuf_) cudaIpcCloseMemHandle(xpeer_[r]);
        return;
    }
    if (stream_) cudaStreamSynchronize(stream_);
    if (decode_exec_) cudaGraphExecDestroy(decode_exec_);
    if (decode_exec_s_) cudaGraphExecDestroy(decode_exec_s_);
    if (gen_exec_) cudaGraphExecDestroy(gen_exec_);
    if (gen_exec_s_) cudaGraphExecDestroy(gen_exec_s_);
    for (int r = 0; r < kMaxTp; ++r)
        if (xpeer_[r] && xpeer_[r] != xbuf_) cudaIpcCloseMemHandle(xpeer_[r]);
    if (comm_) ncclCommDestroy(comm_);
    if (ev_sync_) cudaEventDestroy(ev_sync_);
    if (xbuf_) cudaFree(xbuf_);
    if (arena_) cudaFree(arena_);
    if (h_in_) cudaFreeHost(h_in_);
    if (h_out_) cudaFreeHost(h_out_);
    if (h_gen_) cudaFreeHost(h_gen_);
    if (h_ids_) cudaFreeHost(h_ids_);
    if (trace_) cudaFree(trace_);
    if (ev0_) cudaEventDestroy(ev0_);
    if (ev1_) cudaEventDestroy(ev1_);
    if (kev0_) cudaEventDestroy(kev0_);
    if (kev1_) cudaEventDestroy(kev1_);
    if (stream_) cudaStreamDestroy(stream_);
}

// ---------------------------------------------------------------------------
// Weight loading: Tensor::load (src/tensor.cu:113-126) reads raw fp32 and
// fails on a short file.  Rows [r0, r1) x columns [c0, c1) of a [rows][cols]
// file go to dst with a destination pitch, through pinned staging.
namespace {
// The raw-fp32 weight tree (scripts/export_weights.py:13-25, one file per
// tensor, [rows][cols] row-major) to device memory.  Each job copies rows
// [r0, r1) and columns [c0, c1) of one file (a tensor-parallel shard is read
// straight from its rows / columns) to dst with a row pitch, or, with
// elem_pitch > 0, single elements of one row with that pitch (bias
// interleave).  Jobs are cut into chunks of whole rows; worker threads each
// pread chunks into two pinned staging buffers of their own and copy them to
// the device on their own stream, so file reads, host-to-device copies and
// the other workers overlap.
struct LoadJob {
    std::string rel;
    size_t rows, cols, r0, r1, c0, c1;
    void* dst;
    size_t dpitch, elem_pitch;
};

struct Loader {
    std::string dir;
    std::vector<LoadJob> jobs;
    std::string err;

    void copy(const std::string& rel, size_t rows, size_t cols, size_t r0, size_t r1, size_t c0, size_t c1, void* dst,
              size_t dpitch_bytes, size_t elem_pitch_bytes = 0) {
        jobs.push_back({rel, rows, cols, r0, r1, c0, c1, dst, dpitch_bytes, elem_pitch_bytes});
    }

    int run(int threads, int device) {
        for (const LoadJob& j : jobs) {  // existence and size first, in job order
            const std::string path = dir + "/" + j.rel;
            struct stat sb;
            if (stat(path.c_str(), &sb) != 0) {
                err = "cannot open weight file " + path;
                return XL_ERR_IO;
            }
            if (static_cast<size_t>(sb.st_size) < j.rows * j.cols * 4) {
                err = "weight file too short: " + path + " (" + std::to_string(sb.st_size) + " bytes, need " +
                      std::to_string(j.rows * j.cols * 4) + ")";
                return XL_ERR_IO;
            }
        }
        struct Chunk {
            int job;
            size_t r, nr;
        };
        std::vector<Chunk> chunks;
        for (size_t i = 0; i < jobs.size(); ++i) {
            const size_t row_bytes = jobs[i].cols * 4;
            const size_t per = std::max<size_t>(1, kLoadChunkBytes / row_bytes);
            for (size_t r = jobs[i].r0; r < jobs[i].r1; r += per)
                chunks.push_back({static_cast<int>(i), r, std::min(per, jobs[i].r1 - r)});
        }
        size_t max_chunk = 0;
        for (const Chunk& c : chunks) max_chunk = std::max(max_chunk, c.nr * jobs[c.job].cols * 4);
        std::atomic<size_t> next{0};
        std::atomic<int> rc{XL_OK};
        std::mutex mu;
        auto fail = [&](int code, const std::string& msg) {
            std::lock_guard<std::mutex> g(mu);
            if (rc.load() == XL_OK) {
                err = msg;
                rc = code;
            }
        };
        auto worker = [&]() {
            if (cudaSetDevice(device) != cudaSuccess) return fail(XL_ERR_CUDA, "load: cudaSetDevice failed");
            cudaStream_t s = nullptr;
            cudaEvent_t ev[2] = {nullptr, nullptr};
            void* buf[2] = {nullptr, nullptr};
            std::vector<std::pair<int, int>> fds;  // (job's file index, fd), small per-thread cache
            cudaError_t ce = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
            for (int b = 0; b < 2 && ce == cudaSuccess; ++b) {
                ce = cudaHostAlloc(&buf[b], max_chunk, cudaHostAllocDefault);
                if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&ev[b], cudaEventDisableTiming);
            }
            if (ce != cudaSuccess) fail(XL_ERR_CUDA, std::string("load: ") + cudaGetErrorString(ce));
            int use = 0;
            while (rc.load() == XL_OK) {
                const size_t i = next.fetch_add(1);
                if (i >= chunks.size()) break;
                const Chunk& c = chunks[i];
                const LoadJob& j = jobs[c.job];
                const std::string path = dir + "/" + j.rel;
                int fd = -1;
                for (auto& kv : fds)
                    if (kv.first == c.job) fd = kv.second;
                if (fd < 0) {
                    fd = open(path.c_str(), O_RDONLY);
                    if (fd < 0) {
                        fail(XL_ERR_IO, "cannot open weight file " + path);
                        break;
                    }
                    fds.emplace_back(c.job, fd);
                }
                const int b = use++ & 1;
                ce = cudaEventSynchronize(ev[b]);  // the copy that last used this buffer has finished
                const size_t row_bytes = j.cols * 4, want = c.nr * row_bytes;
                size_t got = 0;
                while (ce == cudaSuccess && got < want) {
                    const ssize_t k = pread(fd, static_cast<char*>(buf[b]) + got, want - got,
                                            static_cast<off_t>(c.r * row_bytes + got));
                    if (k <= 0) break;
                    got += static_cast<size_t>(k);
                }
                if (ce == cudaSuccess && got != want) {
                    fail(XL_ERR_IO, "read failed: " + path);
                    break;
                }
                char* d = static_cast<char*>(j.dst) + (c.r - j.r0) * j.dpitch;
                const char* src = static_cast<const char*>(buf[b]) + j.c0 * 4;
                if (ce == cudaSuccess) {
                    ce = j.elem_pitch ? cudaMemcpy2DAsync(d, j.elem_pitch, src, 4, 4, j.c1 - j.c0,
                                                          cudaMemcpyHostToDevice, s)
                                      : cudaMemcpy2DAsync(d, j.dpitch, src, row_bytes, (j.c1 - j.c0) * 4, c.nr,
                                                          cudaMemcpyHostToDevice, s);
                }
                if (ce == cudaSuccess) ce = cudaEventRecord(ev[b], s);
                if (ce != cudaSuccess) {
                    fail(XL_ERR_CUDA, std::string("H2D copy failed for ") + path + ": " + cudaGetErrorString(ce));
                    break;
                }
            }
            if (s) {
                ce = cudaStreamSynchronize(s);
                if (ce != cudaSuccess) fail(XL_ERR_CUDA, std::string("load: ") + cudaGetErrorString(ce));
                cudaStreamDestroy(s);
            }
            for (int b = 0; b < 2; ++b) {
                if (ev[b]) cudaEventDestroy(ev[b]);
                if (buf[b]) cudaFreeHost(buf[b]);
            }
            for (auto& kv : fds) close(kv.second);
        };
        const int n = std::max(1, std::min(threads, static_cast<int>(chunks.size())));
        std::vector<std::thread> pool;
        for (int t = 1; t < n; ++t) pool.emplace_back(worker);
        worker();
        for (auto& th : pool) th.join();
        return rc.load();
    }
};
}  // namespace

int Engine::load(const char* dir) {
    NvtxRange range("load", 0);
    XL_CUDA(cudaSetDevice(device_));
    if (dir == nullptr) {
        set_error("load: null path");
        return XL_ERR_ARG;
    }
    Loader ld;
    ld.dir = dir;
    const size_t H = H_, Hl = Hl_, Fl = Fl_, F = F_;
    const size_t hq0 = static_cast<size_t>(rank_) * Hl, hq1 = hq0 + Hl;
    const size_t f0 = static_cast<size_t>(rank_) * Fl, f1 = f0 + Fl;
    // Embedding (full table: the decode gather may need any row) and final norm.
    ld.copy("embedding/weight.bin", V_, H, 0, V_, 0, H, emb_, H * 4);
    ld.copy("norm/weight.bin", 1, H, 0, 1, 0, H, gnorm_, H * 4);
    for (int l = 0; l < cfg_.layers; ++l) {
        const std::string b = "blocks/" + std::to_string(l) + "/";
        LayerWeights& L = layers_[l];
        const char* qkv_names[3] = {"attn/Q", "attn/K", "attn/V"};
        for (int i = 0; i < 3; ++i) {
            ld.copy(b + qkv_names[i] + "/weight.bin", H, H, hq0, hq1, 0, H, L.wqkv + i * Hl * H, H * 4);
            ld.copy(b + qkv_names[i] + "/bias.bin", 1, H, 0, 1, hq0, hq1, L.bqkv + i * Hl, Hl * 4);
        }
        ld.copy(b + "attn/W/weight.bin", H, H, 0, H, hq0, hq1, L.wo, Hl * 4);
        if (rank_ == 0) ld.copy(b + "attn/W/bias.bin", 1, H, 0, 1, 0, H, L.bo, H * 4);
        if (tp_ > 1) ld.copy(b + "attn/W/bias.bin", 1, H, 0, 1, 0, H, L.bo_full, H * 4);
        ld.copy(b + "ffn/W1/weight.bin", F, H, f0, f1, 0, H, L.w13, 2 * H * 4);
        ld.copy(b + "ffn/V/weight.bin", F, H, f0, f1, 0, H, L.w13 + H, 2 * H * 4);
        ld.copy(b + "ffn/W1/bias.bin", 1, F, 0, 1, f0, f1, L.b13, 0, 8);
        ld.copy(b + "ffn/V/bias.bin", 1, F, 0, 1, f0, f1, L.b13 + 1, 0, 8);
        ld.copy(b + "ffn/W2/weight.bin", H, F, 0, H, f0, f1, L.w2, Fl * 4);
        if (rank_ == 0) ld.copy(b + "ffn/W2/bias.bin", 1, H, 0, 1, 0, H, L.b2, H * 4);
        if (tp_ > 1) ld.copy(b + "ffn/W2/bias.bin", 1, H, 0, 1, 0, H, L.b2_full, H * 4);
        ld.copy(b + "norm1/weight.bin", 1, H, 0, 1, 0, H, L.g1, H * 4);
        ld.copy(b + "norm2/weight.bin", 1, H, 0, 1, 0, H, L.g2, H * 4);
    }
    // The device is idle while loading: nothing else may use the destination buffers.
    XL_CUDA(cudaStreamSynchronize(stream_));
    const auto t0 = std::chrono::steady_clock::now();
    int rc = ld.run(load_threads_, device_);
    last_load_s_ = std::chrono::duration<float>(std::chrono::steady_clock::now() - t0).count();
    if (rc != XL_OK) {
        set_error(ld.err);
        return rc;
    }
    rc = prepare_prefill_operands();
    if (rc != XL_OK) return rc;
    loaded_ = true;
    has_seq_ = false;
    n_ = 0;
    rc = capture_decode_graph();
    return rc;
}

// TF32 residuals of the projection weights and the TMA maps of every prefill
// GEMM operand (weights, their residuals, the fixed activation buffers).
int Engine::prepare_prefill_operands() {
    const size_t H = H_, Hl = Hl_, Fl = Fl_;
    for (auto& L : layers_) {
        XL_CUDA(launch_split_lo(L.wqkv, L.wqkv_lo, 3 * Hl * H, stream_));
        XL_CUDA(launch_split_lo(L.wo, L.wo_lo, H * Hl, stream_));
        XL_CUDA(launch_split_lo(L.w13, L.w13_lo, 2 * Fl * H, stream_));
        XL_CUDA(launch_split_lo(L.w2, L.w2_lo, H * Fl, stream_));
        XL_CUDA(make_tile_map(&L.tc_qkv.w, L.wqkv, 3 * Hl_, H_));
        XL_CUDA(make_tile_map(&L.tc_qkv.w_lo, L.wqkv_lo, 3 * Hl_, H_));
        XL_CUDA(make_tile_map(&L.tc_qkv.x, pxn_, T_, H_));
        XL_CUDA(make_tile_map(&L.tc_qkv.x_lo, pxn_lo_, T_, H_));
        XL_CUDA(make_tile_map(&L.tc_qkv.x_wide, pxn_, T_, H_, 256));
        XL_CUDA(make_tile_map(&L.tc_qkv.x_lo_wide, pxn_lo_, T_, H_, 256));
        L.tc_qkv.wide = true;
        XL_CUDA(make_tile_map(&L.tc_wo.w, L.wo, H_, Hl_));
        XL_CUDA(make_tile_map(&L.tc_wo.w_lo, L.wo_lo, H_, Hl_));
        XL_CUDA(make_tile_map(&L.tc_wo.x, patt_, T_, Hl_));
        XL_CUDA(make_tile_map(&L.tc_wo.x_lo, patt_lo_, T_, Hl_));
        XL_CUDA(make_tile_map(&L.tc_w13.w, L.w13, 2 * Fl_, H_));
        XL_CUDA(make_tile_map(&L.tc_w13.w_lo, L.w13_lo, 2 * Fl_, H_));
        XL_CUDA(make_tile_map(&L.tc_w13.x, pxn_, T_, H_));
        XL_CUDA(make_tile_map(&L.tc_w13.x_lo, pxn_lo_, T_, H_));
        XL_CUDA(make_tile_map(&L.tc_w13.x_wide, pxn_, T_, H_, 256));
        XL_CUDA(make_tile_map(&L.tc_w13.x_lo_wide, pxn_lo_, T_, H_, 256));
        L.tc_w13.wide = true;
        XL_CUDA(make_tile_map(&L.tc_w2.w, L.w2, H_, Fl_));
        XL_CUDA(make_tile_map(&L.tc_w2.w_lo, L.w2_lo, H_, Fl_));
        XL_CUDA(make_tile_map(&L.tc_w2.x, pffh_, T_, Fl_));
        XL_CUDA(make_tile_map(&L.tc_w2.x_lo, pffh_lo_, T_, Fl_));
    }
    // tensor-core prefill attention: S = (q/8) k^T, then P v (its key blocks need T % 32 == 0)
    if (T_ % 32 == 0) {
        XL_CUDA(make_tile_map(&tc_attn_s_.x, aq_, T_, Hl_));
        XL_CUDA(make_tile_map(&tc_attn_s_.x_lo, aq_lo_, T_, Hl_));
        XL_CUDA(make_tile_map(&tc_attn_s_.w, ak_, heads_l_ * T_, kHeadDim));
        XL_CUDA(make_tile_map(&tc_attn_s_.w_lo, ak_lo_, heads_l_ * T_, kHeadDim));
        XL_CUDA(make_tile_map(&tc_attn_pv_.x, ap_, heads_l_ * T_, T_));
        XL_CUDA(make_tile_map(&tc_attn_pv_.x_lo, ap_lo_, heads_l_ * T_, T_));
        XL_CUDA(make_tile_map(&tc_attn_pv_.w, avt_, heads_l_ * kHeadDim, T_));
        XL_CUDA(make_tile_map(&tc_attn_pv_.w_lo, avt_lo_, heads_l_ * kHeadDim, T_));
        XL_CUDA(make_tile_map(&flash_.q, aq_, T_, Hl_));
        XL_CUDA(make_tile_map(&flash_.q_lo, aq_lo_, T_, Hl_));
        XL_CUDA(make_tile_map(&flash_.k, ak_, heads_l_ * T_, kHeadDim, 64));
        XL_CUDA(make_tile_map(&flash_.k_lo, ak_lo_, heads_l_ * T_, kHeadDim, 64));
        XL_CUDA(make_tile_map(&flash_.v, avt_, heads_l_ * kHeadDim, T_, 64));
        XL_CUDA(make_tile_map(&flash_.v_lo, avt_lo_, heads_l_ * kHeadDim, T_, 64));
    }
    XL_CUDA(cudaStreamSynchronize(stream_));
    return XL_OK;
}

int Engine::prefill_linear(int mode, const TcOperands& o, const float* x, const float* w, const float* b, float* y,
                           float* y_lo, int n, int m, int k, cudaStream_t s) {
    if (prefill_gemm_ == 0) {
        XL_CUDA(launch_gemm_tc(mode, o, b, y, y_lo, n, m, k, &st_->err, s, splitk_ws_, splitk_floats_, num_sms_));
    } else {
        XL_CUDA(launch_linear_prefill(mode, x, w, b, y, n, m, k, s));
        if (y_lo) XL_CUDA(launch_split_lo(y, y_lo, static_cast<size_t>(n) * (mode == kGemvSwiGLU ? m / 2 : m), s));
    }
    return XL_OK;
}

// ---------------------------------------------------------------------------
// One decode step, Transformer::forward(int) (src/transformer.cu:180-186):
// gather -> 16 x [norm1+QKV, RoPE+KV append+attention, out-proj+residual,
// norm2+W1/V+SwiGLU, W2+residual] -> final norm + LM head -> sampler.
// Single-GPU decode step: zero the phase counters, one persistent kernel for
// all 16 layers and the LM head, then the sampler.
int Engine::enqueue_decode_persistent(cudaStream_t s, bool sampled) {
    PersistentParams p{};
    const bool tpk = tp_ > 1;
    if (cfg_.layers > kMaxLayers) {
        set_error("persistent decode supports at most 32 layers");
        return XL_ERR_ARG;
    }
    for (int l = 0; l < cfg_.layers; ++l) {
        const LayerWeights& L = layers_[l];
        // Tensor parallel: the stagings add the whole biases once (the exchanged partial sums carry none).
        p.layer[l] = LayerPtrs{L.wqkv, L.bqkv, L.wo, tpk ? L.bo_full : L.bo, L.w13, L.b13, L.w2,
                               tpk ? L.b2_full : L.b2, L.g1, L.g2, L.kc, L.vc};
        XL_CUDA(make_stream_map(&p.maps[4 * l + 0], L.wqkv, 3 * Hl_, H_));
        XL_CUDA(make_stream_map(&p.maps[4 * l + 1], L.wo, H_, Hl_));
        XL_CUDA(make_stream_map(&p.maps[4 * l + 2], L.w13, 2 * Fl_, H_));
        XL_CUDA(make_stream_map(&p.maps[4 * l + 3], L.w2, H_, Fl_));
    }
    XL_CUDA(make_stream_map(&p.maps[kPersistMaps - 1], emb_ + static_cast<size_t>(v0_) * H_, vl_, H_));
    p.layers = cfg_.layers;
    p.emb = emb_;
    p.gnorm = gnorm_;
    p.rope = rope_;
    p.xa = xa_;
    p.xb = xb_;
    p.cres = cres_;
    p.qkv = qkv_;
    p.part = attn_ws_;
    p.ffh = ffh_;
    p.logits = logits_;
    p.rep_flags = rep_flags_;
    p.st = st_;
    p.done = done_;
    p.head_done = done_ + 5 * cfg_.layers + 1;
    p.att = att_;
    p.trace = trace_;
    p.inflight = inflight_;
    p.H = H_;
    p.Hl = Hl_;
    p.heads = heads_l_;
    p.Fl = Fl_;
    p.V = vl_;
    p.v0 = v0_;
    p.T = T_;
    // Greedy steps end in the kernel; tensor parallel merges the ranks' argmax keys there too (tp_merge).
    p.finish_greedy = sampled || (tpk && !tp_merge_) ? 0 : 1;
    p.tma_evict_first = tma_evict_first_;
    p.sig_cta = sig_cta_;
    const bool tag_split = tag_split_ < 0 ? tpk : tag_split_ != 0;
    p.resid_smem = (resid_smem_ || tag_split) && persistent_smem_bytes(H_, 1) <= 232448 ? 1 : 0;
    p.tag_split = tag_split && p.resid_smem ? 1 : 0;
    p.tag_skew = tag_skew_;
    p.tp = tp_;
    p.rank = rank_;
    if (tpk) {
        for (int r = 0; r < tp_; ++r) p.xc[r] = reinterpret_cast<unsigned long long*>(xpeer_[r]);
        // The ranks' kernels wait on one another (with a time limit), so they
        // start together, after a one-word NCCL barrier: the hosts may launch
        // a step at very different times.  The barrier is a liveness sum:
        // every rank adds 1, and the kernel runs only if the sum is tp.  When a
        // peer never joins, the host aborts the communicator after its step
        // timeout; the aborted all-reduce leaves the sum short, and the kernel
        // leaves before touching any peer's memory.
        XL_CUDA(cudaMemsetAsync(&st_->tp_sync, 0, sizeof(int), s));
        XL_NCCL(ncclAllReduce(&st_->tp_one, &st_->tp_sync, 1, ncclInt32, ncclSum, comm_, s));
    } else {
        p.xc[0] = reinterpret_cast<unsigned long long*>(xbuf_);  // tag_split on one GPU: this engine's own slots
    }
    XL_CUDA(cudaMemsetAsync(done_, 0, done_words() * sizeof(int), s));
    // Optional event-record nodes around the kernel (kernel_events): its own
    // duration, read back by last_kernel_ms.
    if (kernel_events_) XL_CUDA(cudaEventRecordWithFlags(kev0_, s, cudaEventRecordExternal));
    XL_CUDA(launch_decode_persistent(p, num_sms_, s));
    if (kernel_events_) XL_CUDA(cudaEventRecordWithFlags(kev1_, s, cudaEventRecordExternal));
    lm_x_ = xa_;
    if (tpk && !p.finish_greedy) return lm_tail(s, sampled);
    if (sampled) XL_CUDA(launch_sample_chain(sample_params(), 1, true, s));
    return XL_OK;
}

SampleParams Engine::sample_params() const {
    SampleParams sp{};
    sp.logits = logits_;
    sp.V = vl_;
    sp.v0 = v0_;
    sp.st = st_;
    sp.rep_flags = rep_flags_;
    sp.full = 0;
    sp.work = samp_work_;
    sp.work_stride = sample_work_bytes(vl_, samp_grid_);
    sp.stride = vl_;
    sp.grid = samp_grid_;
    return sp;
}

int Engine::enqueue_decode(cudaStream_t s, bool sampled) {
    persistent_graph_ = decode_path_ == 0 && persistent_fits();
    if (persistent_graph_) return enqueue_decode_persistent(s, sampled);
    float* cur = xa_;
    float* other = xb_;
    bool pending = false;  // TP: part_ holds a reduced delta not yet added to cur
    for (int l = 0; l < cfg_.layers; ++l) {
        const LayerWeights& L = layers_[l];
        NormGemvParams p{};
        p.gamma = L.g1;
        p.eps = kEps;
        p.W = L.wqkv;
        p.bias = L.bqkv;
        p.y = qkv_;
        p.M = 3 * Hl_;
        p.K = H_;
        if (l == 0) {
            p.table = emb_;
            p.token = &st_->in.token_in;
            p.x_out = cur;
        } else if (pending) {
            p.x = cur;
            p.delta = part_;
            p.x_out = other;
            std::swap(cur, other);
            pending = false;
        } else {
            p.x = cur;
        }
        XL_CUDA(launch_norm_gemv(kGemvPlain, p, num_sms_, true, s));

        AttnDecodeParams a{};
        a.qkv = qkv_;
        a.rope = rope_;
        a.kc = L.kc;
        a.vc = L.vc;
        a.out = att_;
        a.part = attn_ws_;
        a.counters = attn_cnt_;
        a.pos = &st_->pos;
        a.heads = heads_l_;
        a.max_ctx = T_;
        XL_CUDA(launch_attn_decode(a, true, s));

        NormGemvParams o{};
        o.x = att_;
        o.W = L.wo;
        o.bias = L.bo;
        o.M = H_;
        o.K = Hl_;
        if (tp_ == 1) {
            o.y = cur;
            XL_CUDA(launch_norm_gemv(kGemvResidual, o, num_sms_, true, s));
        } else {
            o.y = part_;
            XL_CUDA(launch_norm_gemv(kGemvPlain, o, num_sms_, true, s));
            XL_NCCL(ncclAllReduce(part_, part_, H_, ncclFloat, ncclSum, comm_, s));
            pending = true;
        }

        NormGemvParams f{};
        f.gamma = L.g2;
        f.eps = kEps;
        f.W = L.w13;
        f.bias = L.b13;
        f.y = ffh_;
        f.M = 2 * Fl_;
        f.K = H_;
        f.x = cur;
        if (pending) {
            f.delta = part_;
            f.x_out = other;
            std::swap(cur, other);
            pending = false;
        }
        XL_CUDA(launch_norm_gemv(kGemvSwiGLU, f, num_sms_, true, s));

        NormGemvParams d{};
        d.x = ffh_;
        d.W = L.w2;
        d.bias = L.b2;
        d.M = H_;
        d.K = Fl_;
        if (tp_ == 1) {
            d.y = cur;
            XL_CUDA(launch_norm_gemv(kGemvResidual, d, num_sms_, true, s));
        } else {
            d.y = part_;
            XL_CUDA(launch_norm_gemv(kGemvPlain, d, num_sms_, true, s));
            XL_NCCL(ncclAllReduce(part_, part_, H_, ncclFloat, ncclSum, comm_, s));
            pending = true;
        }
    }
    lm_x_ = cur;
    return run_lm_head_and_sample(cur, pending ? part_ : nullptr, s, sampled);
}

// Final norm + tied LM head (Embedding::inverse, src/embedding.cu:173-205)
// over this rank's vocab shard, argmax merge across ranks, then the sampler.
int Engine::launch_lm_head(const float* x_last, const float* delta, bool pdl, cudaStream_t s) {
    NormGemvParams h{};
    h.x = x_last;
    h.delta = delta;
    h.gamma = gnorm_;
    h.eps = kEps;
    h.W = emb_ + static_cast<size_t>(v0_) * H_;
    h.y = logits_;
    h.M = vl_;
    h.K = H_;
    h.rep_flags = rep_flags_;
    h.st = st_;
    h.row_offset = v0_;
    XL_CUDA(launch_norm_gemv(kGemvLogits, h, num_sms_, pdl, s));
    return XL_OK;
}

int Engine::run_lm_head_and_sample(const float* x_last, const float* delta, cudaStream_t s, bool sampled) {
    const int rc = launch_lm_head(x_last, delta, true, s);
    if (rc != XL_OK) return rc;
    return lm_tail(s, sampled);
}

// After the LM head: the argmax merge across vocab shards (tensor parallel),
// then the greedy id or the sampler.
int Engine::lm_tail(cudaStream_t s, bool sampled) {
    if (tp_ > 1) XL_NCCL(ncclAllReduce(&st_->argmax_final, &st_->argmax_final, 1, ncclUint64, ncclMax, comm_, s));
    SampleParams sp = sample_params();
    if (!sampled) {
        XL_CUDA(launch_sample_finish(sp, 1, true, s));
        return XL_OK;
    }
    if (tp_ > 1) {
        // Sampling merge across vocab shards: local top-1024, all-gather, one draw on every rank.
        sp.full = 1;
        sp.cand_out = cand_local_;
        XL_CUDA(launch_sample_chain(sp, 1, true, s));
        XL_NCCL(ncclAllGather(cand_local_, cand_all_, kTopK, ncclUint64, comm_, s));
        SampleMergeParams mp{};
        mp.cand = cand_all_;
        mp.n = tp_ * kTopK;
        mp.n_pad = kTopK;
        while (mp.n_pad < mp.n) mp.n_pad <<= 1;
        mp.V_total = V_;
        mp.st = st_;
        mp.rep_flags = rep_flags_;
        mp.V = vl_;
        mp.v0 = v0_;
        XL_CUDA(launch_sample_merge(mp, false, s));
        return XL_OK;
    }
    XL_CUDA(launch_sample_chain(sp, 1, true, s));
    return XL_OK;
}

int Engine::capture_decode_graph() {
    for (int sampled = 0; sampled < 2; ++sampled) {
        cudaGraphExec_t& exec = sampled ? decode_exec_s_ : decode_exec_;
        long long& kernels = sampled ? decode_graph_kernels_s_ : decode_graph_kernels_;
        if (exec) {
            cudaGraphExecDestroy(exec);
            exec = nullptr;
        }
        cudaGraph_t g = nullptr;
        XL_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
        const long long recorded0 = launch_count();
        int rc = enqueue_decode(stream_, sampled != 0);
        kernels = launch_count() - recorded0;
        count_graph_kernels(-kernels);  // recorded, not run; each replay adds them
        cudaError_t ce = cudaStreamEndCapture(stream_, &g);
        if (rc != XL_OK) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamEndCapture");
        ce = cudaGraphInstantiate(&exec, g, 0);
        cudaGraphDestroy(g);
        if (ce != cudaSuccess) return cuda_fail(ce, "cudaGraphInstantiate");
    }
    return capture_gen_graphs();
}

// Device-side generation graphs: gen_feed, the persistent decode step and
// gen_collect (persistent path only: its kernels skip a step once the run has
// stopped).  Tensor parallel: greedy steps whose argmax merges inside the
// kernel (tp_merge), the step-start all-reduce included, so that every rank
// runs the same collectives whether a step is skipped or not; sampled
// tensor-parallel steps keep the host loop.
int Engine::capture_gen_graphs() {
    for (int sampled = 0; sampled < 2; ++sampled) {
        cudaGraphExec_t& exec = sampled ? gen_exec_s_ : gen_exec_;
        if (exec) {
            cudaGraphExecDestroy(exec);
            exec = nullptr;
        }
    }
    if (!persistent_graph_) return XL_OK;
    GenParams gp{};
    gp.ctl = gen_ctl_;
    gp.uniforms = gen_u_;
    gp.out = gen_out_;
    gp.st = st_;
    for (int sampled = 0; sampled < 2; ++sampled) {
        if (tp_ > 1 && (sampled || !tp_merge_)) continue;
        cudaGraphExec_t& exec = sampled ? gen_exec_s_ : gen_exec_;
        long long& kernels = sampled ? gen_graph_kernels_s_ : gen_graph_kernels_;
        cudaGraph_t g = nullptr;
        XL_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
        const long long recorded0 = launch_count();
        cudaError_t le = launch_gen_feed(gp, stream_);
        int rc = le == cudaSuccess ? enqueue_decode(stream_, sampled != 0) : XL_OK;
        if (le == cudaSuccess && rc == XL_OK) le = launch_gen_collect(gp, stream_);
        kernels = launch_count() - recorded0;
        count_graph_kernels(-kernels);
        cudaError_t ce = cudaStreamEndCapture(stream_, &g);
        if (rc != XL_OK || le != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            return rc != XL_OK ? rc : cuda_fail(le, "generation graph capture");
        }
        if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamEndCapture");
        ce = cudaGraphInstantiate(&exec, g, 0);
        cudaGraphDestroy(g);
        if (ce != cudaSuccess) return cuda_fail(ce, "cudaGraphInstantiate");
    }
    return XL_OK;
}

float Engine::next_uniform() {
    if (!uniforms_.empty()) {
        const float u = uniforms_.front();
        uniforms_.pop_front();
        return u;
    }
    return philox_uniform(philox_ctr_++, philox_seed_);
}

int Engine::finish_step(int* token_out) {
    XL_CUDA(cudaEventRecord(ev1_, stream_));
    XL_CUDA(cudaMemcpyAsync(h_out_, st_, sizeof(DevState), cudaMemcpyDeviceToHost, stream_));
    int rc = wait_stream("step");
    if (rc != XL_OK) return rc;
    XL_CUDA(cudaEventElapsedTime(&last_ms_, ev0_, ev1_));
    const DevState* hs = reinterpret_cast<const DevState*>(h_out_);
    if (hs->err != 0) return device_error(hs->err);
    *token_out = hs->token_out;
    return XL_OK;
}

// A kernel reported an error through DevState::err (a bounded wait ran out).
// One GPU: the word is cleared and the sequence dropped, so the next prompt
// starts clean.  Tensor parallel: the ranks' step counters (the exchange tags)
// may now disagree, so the engine refuses every further step.
int Engine::device_error(int bits) {
    std::string msg = "device error word " + std::to_string(bits);
    has_seq_ = false;
    n_ = 0;
    if (tp_ > 1) {
        failed_ = true;
        fail_msg_ = "tensor parallel: a step failed on the device (error word " + std::to_string(bits) +
                    "); this engine is unusable: create a new one on every rank";
        msg = fail_msg_;
    } else {
        // The failed step's tagged words carry its step counter, which its last CTA never advanced: move the
        // counter past it, so that the next step's waits never accept one of those words.
        const int epoch = reinterpret_cast<const DevState*>(h_out_)->epoch + 1;
        XL_CUDA(cudaMemsetAsync(&st_->err, 0, sizeof(int), stream_));
        XL_CUDA(cudaMemcpyAsync(&st_->epoch, &epoch, sizeof(int), cudaMemcpyHostToDevice, stream_));
        XL_CUDA(cudaStreamSynchronize(stream_));
        msg += "; the sequence was dropped: prefill a new prompt";
    }
    set_error(msg);
    return XL_ERR_DEVICE;
}

// Waits for the engine stream.  A tensor-parallel step can wait on a peer
// rank that never joins (its host stopped or died between steps): the wait is
// then bounded by the step timeout (option step_timeout_ms) and by NCCL's
// asynchronous error, after which the communicator is aborted.
int Engine::wait_stream(const char* what) {
    if (tp_ == 1) {
        XL_CUDA(cudaStreamSynchronize(stream_));
        return XL_OK;
    }
    XL_CUDA(cudaEventRecord(ev_sync_, stream_));
    const auto t0 = std::chrono::steady_clock::now();
    for (uint32_t it = 0;; ++it) {
        const cudaError_t q = cudaEventQuery(ev_sync_);
        if (q == cudaSuccess) return XL_OK;
        if (q != cudaErrorNotReady) return cuda_fail(q, what);
        if ((it & 255u) != 0) continue;
        ncclResult_t ar = ncclSuccess;
        if (comm_ && ncclCommGetAsyncError(comm_, &ar) != ncclSuccess) ar = ncclInternalError;
        if (ar != ncclSuccess && ar != ncclInProgress)
            return abort_tp(std::string(what) + ": NCCL reported " + ncclGetErrorString(ar));
        const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        if (ms > step_timeout_ms_)
            return abort_tp(std::string(what) + " did not finish within " + std::to_string(step_timeout_ms_) +
                            " ms (a peer rank stopped or died?)");
    }
}

// Polls the engine stream until it is idle or timeout_ms has passed.
bool Engine::drain_stream(int timeout_ms) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t q = cudaStreamQuery(stream_);
        if (q != cudaErrorNotReady) return q == cudaSuccess;
        const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        if (ms > timeout_ms) return false;
        std::this_thread::yield();
    }
}

// Tensor parallel: gives up on the communicator.  The executable graphs that
// hold its collectives go first (one still in flight is released when it
// completes), then ncclCommAbort makes the collectives that wait for the
// missing rank return; the persistent kernel of that step finds the liveness
// sum short and leaves.  The engine refuses every later call.
int Engine::abort_tp(const std::string& why) {
    // XL_TRACE_ABORT=1: each step of the abort on stderr (diagnosis of a stuck abort).
    static const bool trace = std::getenv("XL_TRACE_ABORT") != nullptr;
    auto note = [&](const char* what) {
        if (trace) std::fprintf(stderr, "[xl rank %d] abort: %s\n", rank_, what), std::fflush(stderr);
    };
    note(why.c_str());
    // ncclCommAbort raises the communicator's abort flag first (the collectives
    // waiting for the missing rank return), then waits until no executable
    // graph holds its collectives.  Releasing an executable graph that is still
    // running blocks until it completes, and it completes only once the flag is
    // up: so the abort runs on a helper thread while this one releases the
    // graphs.  Both waits are bounded here; a helper still blocked after them
    // is detached (the engine is unusable either way).
    std::thread aborter;
    auto done = std::make_shared<std::atomic<bool>>(false);
    if (comm_) {
        ncclComm_t c = comm_;
        aborter = std::thread([c, done]() {
            ncclCommAbort(c);
            done->store(true);
        });
    }
    comm_ = nullptr;
    for (cudaGraphExec_t* e : {&decode_exec_, &decode_exec_s_, &gen_exec_, &gen_exec_s_}) {
        if (*e) cudaGraphExecDestroy(*e);
        *e = nullptr;
    }
    note("graphs released");
    if (aborter.joinable()) {
        const auto t0 = std::chrono::steady_clock::now();
        while (!done->load() && std::chrono::steady_clock::now() - t0 < std::chrono::seconds(20))
            std::this_thread::sleep_for(std::chrono::milliseconds(1));
        if (done->load()) {
            aborter.join();
            note("communicator aborted");
        } else {
            aborter.detach();
            note("communicator abort still running after 20 s (detached)");
        }
    }
    failed_ = true;
    fail_msg_ = "tensor parallel: " + why + "; the communicator was aborted and this engine is unusable: create a new "
                "one on every rank";
    const bool idle = drain_stream(10000);
    note(idle ? "stream drained" : "stream still busy after 10 s");
    if (!idle) fail_msg_ += " (its stream did not drain within 10 s)";
    stream_idle_ = idle;
    has_seq_ = false;
    set_error(fail_msg_);
    return XL_ERR_NCCL;
}

int Engine::check_usable() const {
    if (!failed_) return XL_OK;
    set_error(fail_msg_);
    return XL_ERR_STATE;
}

// InferenceEngine::next_token(vector), src/inference.cu:116-136.
int Engine::prefill(const int* ids, int n, float temperature, float top_p, float rp, int* token_out, bool append) {
    NvtxRange range(append ? "extend" : "prefill", n);
    XL_CUDA(cudaSetDevice(device_));
    if (const int u = check_usable()) return u;
    if (!loaded_) {
        set_error("prefill before load");
        return XL_ERR_STATE;
    }
    if (ids == nullptr || n <= 0) {
        set_error("prefill: empty prompt");
        return XL_ERR_ARG;
    }
    if (append && !has_seq_) {
        set_error("extend before any prefill: the KV cache is empty");
        return XL_ERR_STATE;
    }
    const int p0 = append ? n_ : 0;  // position of the first new id
    if (p0 + n > T_) {
        set_error("Input sequence length exceeds max_seq_len (" + std::to_string(p0 + n) + " > " + std::to_string(T_) +
                  ")");
        return XL_ERR_CTX;
    }
    for (int i = 0; i < n; ++i) {
        if (ids[i] < 0 || ids[i] >= V_) {
            set_error("Embedding : Invalid token: " + std::to_string(ids[i]) + " ( i = " + std::to_string(i) +
                      " ), vocabulary size = " + std::to_string(V_));
            return XL_ERR_TOKEN;
        }
    }
    std::memcpy(h_ids_, ids, sizeof(int) * n);
    StepIn in{};
    in.token_in = 0;
    in.temperature = temperature;
    in.top_p = top_p;
    in.rp = rp;
    in.uniform = next_uniform();
    in.decode_mode = 0;
    DevState* hs = reinterpret_cast<DevState*>(h_in_);
    std::memset(hs, 0, sizeof(DevState));
    hs->in = in;
    hs->pos = p0 + n;
    cudaStream_t s = stream_;
    XL_CUDA(cudaMemcpyAsync(pids_, h_ids_, sizeof(int) * n, cudaMemcpyHostToDevice, s));
    // in + pos: the first bytes of DevState
    XL_CUDA(cudaMemcpyAsync(st_, hs, offsetof(DevState, pos) + sizeof(int), cudaMemcpyHostToDevice, s));
    // A new prompt clears the repetition set (src/inference.cu:116-136); an appended one keeps it.
    if (!append) XL_CUDA(cudaMemsetAsync(rep_flags_, 0, vl_, s));
    // the fused attention's merge tickets (left zero by every complete launch; reset after a failed one)
    XL_CUDA(cudaMemsetAsync(fa_tickets_, 0, static_cast<size_t>(heads_l_) * ((T_ + 127) / 128) * 4 * 4, s));
    XL_CUDA(cudaEventRecord(ev0_, s));

    const size_t H = H_;
    XL_CUDA(launch_embed_gather(emb_, pids_, px_, n, H_, s));
    int rc = XL_OK;
    for (int l = 0; l < cfg_.layers && rc == XL_OK; ++l) {
        const LayerWeights& L = layers_[l];
        XL_CUDA(launch_rmsnorm_rows(px_, L.g1, pxn_, pxn_lo_, n, H_, s));
        rc = prefill_linear(kGemvPlain, L.tc_qkv, pxn_, L.wqkv, L.bqkv, pqkv_, nullptr, n, 3 * Hl_, H_, s);
        if (rc != XL_OK) break;
        if (prefill_attn_ != 1 && T_ % 32 == 0 && p0 == 0) {
            XL_CUDA(launch_attn_prep(pqkv_, rope_, L.kc, L.vc, aq_, aq_lo_, ak_, ak_lo_, avt_, avt_lo_, n, heads_l_, T_,
                                     s));
            if (prefill_attn_ == 0) {
                XL_CUDA(launch_attn_flash_tc(flash_, patt_, patt_lo_, n, heads_l_, T_, ap_,
                                             static_cast<size_t>(heads_l_) * T_ * T_, fa_tickets_, &st_->err, s));
            } else {
                XL_CUDA(launch_attn_scores_tc(tc_attn_s_, ap_, n, heads_l_, T_, &st_->err, s));
                XL_CUDA(launch_attn_softmax(ap_, ap_lo_, n, heads_l_, T_, s));
                XL_CUDA(launch_attn_pv_tc(tc_attn_pv_, patt_, patt_lo_, n, heads_l_, T_, &st_->err, s));
            }
        } else {
            XL_CUDA(launch_rope_kv_prefill(pqkv_, rope_, L.kc, L.vc, n, heads_l_, T_, s, p0));
            XL_CUDA(launch_attn_prefill(pqkv_, L.kc, L.vc, patt_, patt_lo_, n, heads_l_, T_, s, p0));
        }
        if (tp_ == 1) {
            rc = prefill_linear(kGemvResidual, L.tc_wo, patt_, L.wo, L.bo, px_, nullptr, n, H_, Hl_, s);
        } else {
            // partial sums into pxn_ (free until the next norm), reduced over ranks, then added
            rc = prefill_linear(kGemvPlain, L.tc_wo, patt_, L.wo, L.bo, pxn_, nullptr, n, H_, Hl_, s);
            if (rc == XL_OK) {
                XL_NCCL(ncclAllReduce(pxn_, pxn_, n * H, ncclFloat, ncclSum, comm_, s));
                XL_CUDA(launch_add_rows(px_, pxn_, n * H_, s));
            }
        }
        if (rc != XL_OK) break;
        XL_CUDA(launch_rmsnorm_rows(px_, L.g2, pxn_, pxn_lo_, n, H_, s));
        rc = prefill_linear(kGemvSwiGLU, L.tc_w13, pxn_, L.w13, L.b13, pffh_, pffh_lo_, n, 2 * Fl_, H_, s);
        if (rc != XL_OK) break;
        if (tp_ == 1) {
            rc = prefill_linear(kGemvResidual, L.tc_w2, pffh_, L.w2, L.b2, px_, nullptr, n, H_, Fl_, s);
        } else {
            rc = prefill_linear(kGemvPlain, L.tc_w2, pffh_, L.w2, L.b2, pxn_, nullptr, n, H_, Fl_, s);
            if (rc == XL_OK) {
                XL_NCCL(ncclAllReduce(pxn_, pxn_, n * H, ncclFloat, ncclSum, comm_, s));
                XL_CUDA(launch_add_rows(px_, pxn_, n * H_, s));
            }
        }
    }
    if (rc != XL_OK) return rc;
    rc = run_lm_head_and_sample(px_ + static_cast<size_t>(n - 1) * H, nullptr, s, top_p > 0.0f);
    if (rc != XL_OK) return rc;
    rc = finish_step(token_out);
    if (rc != XL_OK) return rc;
    n_ = p0 + n;
    has_seq_ = true;
    return XL_OK;
}

// InferenceEngine::next_token(int), src/inference.cu:138-151.
int Engine::decode(int token, float temperature, float top_p, float rp, int* token_out) {
    NvtxRange range("decode", n_);
    XL_CUDA(cudaSetDevice(device_));
    if (const int u = check_usable()) return u;
    if (!loaded_) {
        set_error("decode before load");
        return XL_ERR_STATE;
    }
    if (!has_seq_) {
        set_error("decode before any prefill: the KV cache is empty");
        return XL_ERR_STATE;
    }
    if (token < 0 || token >= V_) {
        set_error("Embedding : Invalid token: " + std::to_string(token));
        return XL_ERR_TOKEN;
    }
    if (n_ >= T_) {
        set_error("KV cache full: position " + std::to_string(n_) + " of max_seq_len " + std::to_string(T_));
        return XL_ERR_CTX;
    }
    StepIn* in = h_in_;
    std::memset(in, 0, sizeof(StepIn));
    in->token_in = token;
    in->temperature = temperature;
    in->top_p = top_p;
    in->rp = rp;
    in->uniform = next_uniform();
    in->decode_mode = 1;
    XL_CUDA(cudaMemcpyAsync(&st_->in, in, sizeof(StepIn), cudaMemcpyHostToDevice, stream_));
    XL_CUDA(cudaEventRecord(ev0_, stream_));
    const bool use_sampled = top_p > 0.0f;
    XL_CUDA(cudaGraphLaunch(use_sampled ? decode_exec_s_ : decode_exec_, stream_));
    count_graph_kernels(use_sampled ? decode_graph_kernels_s_ : decode_graph_kernels_);
    const int rc = finish_step(token_out);
    if (rc != XL_OK) return rc;
    last_kernel_ms_ = -1.0f;
    if (kernel_events_ && persistent_graph_) XL_CUDA(cudaEventElapsedTime(&last_kernel_ms_, kev0_, kev1_));
    n_ += 1;
    return XL_OK;
}

int Engine::generate(int token, int n, float temperature, float top_p, float rp, int stop_id, int* tokens_out,
                     int* n_out) {
    NvtxRange range("generate", n_);
    XL_CUDA(cudaSetDevice(device_));
    *n_out = 0;
    if (const int u = check_usable()) return u;
    if (n < 0 || (n > 0 && tokens_out == nullptr)) {
        set_error("generate: n must be >= 0 and tokens_out non-null");
        return XL_ERR_ARG;
    }
    if (n == 0) return XL_OK;
    if (!loaded_) {
        set_error("decode before load");
        return XL_ERR_STATE;
    }
    if (!has_seq_) {
        set_error("decode before any prefill: the KV cache is empty");
        return XL_ERR_STATE;
    }
    if (token < 0 || token >= V_) {
        set_error("Embedding : Invalid token: " + std::to_string(token));
        return XL_ERR_TOKEN;
    }
    if (n_ >= T_) {
        set_error("KV cache full: position " + std::to_string(n_) + " of max_seq_len " + std::to_string(T_));
        return XL_ERR_CTX;
    }
    const bool sampled = top_p > 0.0f;
    cudaGraphExec_t exec = sampled ? gen_exec_s_ : gen_exec_;
    if (!exec) {
        // Per-op engines and sampled tensor-parallel steps: the same loop on the host.
        int tok = token;
        for (int i = 0; i < n && n_ < T_; ++i) {
            const int rc = decode(tok, temperature, top_p, rp, &tok);
            if (rc != XL_OK) return rc;
            tokens_out[(*n_out)++] = tok;
            if (tok == stop_id) break;
        }
        return XL_OK;
    }
    const int steps = std::min(n, T_ - n_);
    // The draws of successive next_token calls; those of steps that never run are handed back below.
    const size_t queued = uniforms_.size();
    const uint64_t ctr0 = philox_ctr_;
    std::deque<float> queue0 = uniforms_;
    GenCtl* c = reinterpret_cast<GenCtl*>(h_gen_);
    float* hu = reinterpret_cast<float*>(h_gen_ + sizeof(GenCtl));
    int* ho = reinterpret_cast<int*>(hu + T_);
    std::memset(c, 0, sizeof(GenCtl));
    c->n = steps;
    c->first = token;
    c->stop_id = stop_id;
    c->max_ctx = T_;
    c->temperature = temperature;
    c->top_p = top_p;
    c->rp = rp;
    for (int i = 0; i < steps; ++i) hu[i] = next_uniform();
    XL_CUDA(cudaMemcpyAsync(gen_ctl_, c, sizeof(GenCtl), cudaMemcpyHostToDevice, stream_));
    XL_CUDA(cudaMemcpyAsync(gen_u_, hu, static_cast<size_t>(steps) * 4, cudaMemcpyHostToDevice, stream_));
    XL_CUDA(cudaEventRecord(ev0_, stream_));
    for (int i = 0; i < steps; ++i) {
        XL_CUDA(cudaGraphLaunch(exec, stream_));
        count_graph_kernels(sampled ? gen_graph_kernels_s_ : gen_graph_kernels_);
    }
    XL_CUDA(cudaEventRecord(ev1_, stream_));
    XL_CUDA(cudaMemcpyAsync(c, gen_ctl_, sizeof(GenCtl), cudaMemcpyDeviceToHost, stream_));
    XL_CUDA(cudaMemcpyAsync(ho, gen_out_, static_cast<size_t>(steps) * 4, cudaMemcpyDeviceToHost, stream_));
    XL_CUDA(cudaMemcpyAsync(h_out_, st_, sizeof(DevState), cudaMemcpyDeviceToHost, stream_));
    // tensor parallel: bounded by the step timeout and NCCL's asynchronous error (a peer that stops)
    if (const int rc = wait_stream("generate")) return rc;
    XL_CUDA(cudaEventElapsedTime(&last_ms_, ev0_, ev1_));
    const DevState* hs = reinterpret_cast<const DevState*>(h_out_);
    if (hs->err != 0) return device_error(hs->err);
    const int done = c->step;
    if (done < steps) {
        // Return the unused draws: queued values go back in order, the Philox counter rewinds.
        uniforms_ = queue0;
        const size_t from_queue = std::min(static_cast<size_t>(done), queued);
        for (size_t i = 0; i < from_queue; ++i) uniforms_.pop_front();
        philox_ctr_ = ctr0 + (static_cast<size_t>(done) > queued ? static_cast<size_t>(done) - queued : 0);
    }
    for (int i = 0; i < done; ++i) tokens_out[i] = ho[i];
    *n_out = done;
    n_ += done;
    last_kernel_ms_ = -1.0f;
    return XL_OK;
}

int Engine::profile_lm_head(int iters, float* avg_ms) {
    XL_CUDA(cudaSetDevice(device_));
    if (!loaded_ || iters <= 0 || avg_ms == nullptr) {
        set_error("profile_lm_head: needs a loaded engine and iters > 0");
        return XL_ERR_ARG;
    }
    if (tp_ > 1) {
        set_error("profile_lm_head: single-rank engines only");
        return XL_ERR_ARG;
    }
    // Same kernel, same arguments as the decode graph's LM head (its residual
    // stream, final norm, full tied table), without PDL.
    int rc = launch_lm_head(lm_x_, nullptr, false, stream_);
    if (rc != XL_OK) return rc;
    XL_CUDA(cudaEventRecord(ev0_, stream_));
    for (int i = 0; i < iters && rc == XL_OK; ++i) rc = launch_lm_head(lm_x_, nullptr, false, stream_);
    if (rc != XL_OK) return rc;
    XL_CUDA(cudaEventRecord(ev1_, stream_));
    XL_CUDA(cudaEventSynchronize(ev1_));
    float ms = 0.0f;
    XL_CUDA(cudaEventElapsedTime(&ms, ev0_, ev1_));
    *avg_ms = ms / static_cast<float>(iters);
    return XL_OK;
}

int Engine::set_option(const char* key, int value) {
    XL_CUDA(cudaSetDevice(device_));
    const std::string k = key ? key : "";
    if (k == "decode_path") {
        if (value != 0 && value != 1) {
            set_error("decode_path must be 0 (persistent kernel) or 1 (per-op kernels)");
            return XL_ERR_ARG;
        }
        decode_path_ = value;
        return loaded_ ? capture_decode_graph() : XL_OK;
    }
    if (k == "prefill_gemm") {
        if (value != 0 && value != 1) {
            set_error("prefill_gemm must be 0 (tcgen05 3xTF32) or 1 (fp32 SIMT tiles)");
            return XL_ERR_ARG;
        }
        prefill_gemm_ = value;
        return XL_OK;
    }
    if (k == "prefill_attn") {
        if (value < 0 || value > 2) {
            set_error("prefill_attn must be 0 (fused tcgen05), 1 (fp32 FMA tiles) or 2 (tcgen05 S, softmax, P.V)");
            return XL_ERR_ARG;
        }
        prefill_attn_ = value;
        return XL_OK;
    }
    if (k == "tma_inflight") {
        if (value < 1 || value > kPersistSlots) {
            set_error("tma_inflight must be in [1, 6]");
            return XL_ERR_ARG;
        }
        inflight_ = value;
        return loaded_ ? capture_decode_graph() : XL_OK;
    }
    if (k == "step_timeout_ms") {
        if (value < 1) {
            set_error("step_timeout_ms must be >= 1");
            return XL_ERR_ARG;
        }
        step_timeout_ms_ = value;
        return XL_OK;
    }
    if (k == "load_threads") {
        if (value < 1 || value > 64) {
            set_error("load_threads must be in [1, 64]");
            return XL_ERR_ARG;
        }
        load_threads_ = value;
        return XL_OK;
    }
    if (k == "tma_evict_first") {
        if (value != 0 && value != 1) {
            set_error("tma_evict_first must be 0 or 1");
            return XL_ERR_ARG;
        }
        tma_evict_first_ = value;
        return loaded_ ? capture_decode_graph() : XL_OK;
    }
    if (k == "tag_skew") {
        // Test hook: the tagged exchange's stagings wait for a tag shifted by this amount; a tag nobody writes
        // makes their bounded wait run out, and the step reports a device error.
        tag_skew_ = value;
        return loaded_ ? capture_decode_graph() : XL_OK;
    }
    if (k == "batch_persistent") {
        if (value != 0 && value != 1) {
            set_error("batch_persistent must be 0 or 1");
            return XL_ERR_ARG;
        }
        batch_persistent_ = value;  // read when a BatchDecoder is created
        return XL_OK;
    }
    if (k == "tp_merge") {
        if (value != 0 && value != 1) {
            set_error("tp_merge must be 0 or 1");
            return XL_ERR_ARG;
        }
        tp_merge_ = value;
        return loaded_ ? capture_decode_graph() : XL_OK;
    }
    if (k == "sig_cta" || k == "resid_smem" || k == "tag_split") {
        if (value != 0 && value != 1) {
            set_error(k + " must be 0 or 1");
            return XL_ERR_ARG;
        }
        (k == "sig_cta" ? sig_cta_ : k == "resid_smem" ? resid_smem_ : tag_split_) = value;
        return loaded_ ? capture_decode_graph() : XL_OK;
    }
    if (k == "kernel_events") {
        if (value != 0 && value != 1) {
            set_error("kernel_events must be 0 or 1");
            return XL_ERR_ARG;
        }
        kernel_events_ = value != 0;
        return loaded_ ? capture_decode_graph() : XL_OK;
    }
    if (k == "phase_trace") {
        if (value && !trace_) {
            const size_t n = static_cast<size_t>(num_sms_) * (5 * cfg_.layers + 1) * kTraceFields;
            XL_CUDA(cudaMalloc(reinterpret_cast<void**>(&trace_), n * sizeof(unsigned long long)));
            XL_CUDA(cudaMemset(trace_, 0, n * sizeof(unsigned long long)));
        } else if (!value && trace_) {
            XL_CUDA(cudaStreamSynchronize(stream_));
            XL_CUDA(cudaFree(trace_));
            trace_ = nullptr;
        }
        return loaded_ ? capture_decode_graph() : XL_OK;
    }
    set_error("unknown option: " + k);
    return XL_ERR_ARG;
}

int Engine::phase_trace(unsigned long long* out, int n) {
    XL_CUDA(cudaSetDevice(device_));
    const int need = num_sms_ * (5 * cfg_.layers + 1) * kTraceFields;
    if (!trace_ || !out || n != need) {
        set_error("phase_trace: enable the phase_trace option; n must be " + std::to_string(need));
        return XL_ERR_ARG;
    }
    XL_CUDA(cudaMemcpyAsync(out, trace_, sizeof(unsigned long long) * n, cudaMemcpyDeviceToHost, stream_));
    XL_CUDA(cudaStreamSynchronize(stream_));
    return XL_OK;
}

int Engine::set_uniforms(const float* u, int n) {
    if (n < 0 || (n > 0 && u == nullptr)) {
        set_error("set_uniforms: bad array");
        return XL_ERR_ARG;
    }
    uniforms_.assign(u, u + n);
    return XL_OK;
}

int Engine::seed(uint64_t s) {
    philox_seed_ = s;
    philox_ctr_ = 0;
    uniforms_.clear();
    return XL_OK;
}

int Engine::last_logits(float* out, int n) {
    XL_CUDA(cudaSetDevice(device_));
    if (n != vl_ || out == nullptr) {
        set_error("last_logits: n must equal the vocab shard size " + std::to_string(vl_));
        return XL_ERR_ARG;
    }
    XL_CUDA(cudaMemcpyAsync(out, logits_, sizeof(float) * vl_, cudaMemcpyDeviceToHost, stream_));
    XL_CUDA(cudaStreamSynchronize(stream_));
    return XL_OK;
}

int Engine::kv_copy(int layer, int npos, float* k_out, float* v_out) {
    XL_CUDA(cudaSetDevice(device_));
    if (layer < 0 || layer >= cfg_.layers || npos < 0 || npos > T_) {
        set_error("kv_copy: layer or npos out of range");
        return XL_ERR_ARG;
    }
    if (npos == 0) return XL_OK;
    const LayerWeights& L = layers_[layer];
    for (int h = 0; h < heads_l_; ++h) {
        const size_t src_off = static_cast<size_t>(h) * T_ * kHeadDim;
        XL_CUDA(cudaMemcpy2DAsync(k_out + h * kHeadDim, Hl_ * 4, L.kc + src_off, kHeadDim * 4,
                                  kHeadDim * 4, npos, cudaMemcpyDeviceToHost, stream_));
        XL_CUDA(cudaMemcpy2DAsync(v_out + h * kHeadDim, Hl_ * 4, L.vc + src_off, kHeadDim * 4,
                                  kHeadDim * 4, npos, cudaMemcpyDeviceToHost, stream_));
    }
    XL_CUDA(cudaStreamSynchronize(stream_));
    return XL_OK;
}

}  // namespace xl
