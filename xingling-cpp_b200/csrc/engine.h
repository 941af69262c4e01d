// XingLing token-loop engine on one B200 (or one tensor-parallel rank).
#pragma once
#include <cuda_runtime.h>
#include <nccl.h>
#include <stdint.h>

#include <deque>
#include <string>
#include <vector>

#include "../../include/xl_engine.h"
#include "xl_kernels.h"

namespace xl {

// Thread-local last-error message behind xl_last_error().
void set_error(const std::string& msg);
const char* last_error();
void clear_error();

struct LayerWeights {
    float* wqkv;  // [3*Hl][H]: this rank's Q rows, then K rows, then V rows
    float* bqkv;  // [3*Hl]
    float* wo;    // [H][Hl]: columns of this rank's heads
    float* bo;    // [H] (zero on ranks > 0)
    float* w13;   // [2*Fl][H]: rows (W1 j, V j) interleaved
    float* b13;   // [2*Fl]
    float* w2;    // [H][Fl]
    float* b2;    // [H] (zero on ranks > 0)
    float* g1;    // [H]
    float* g2;    // [H]
    float *bo_full, *b2_full;  // [H] the whole biases (tensor parallel only: the persistent kernel's stagings)
    float* kc;    // [heads_l][max_ctx][64]
    float* vc;    // [heads_l][max_ctx][64]
    // TF32 residuals (w - trunc19(w)) of the four projections, for the 3xTF32 prefill GEMMs
    float *wqkv_lo, *wo_lo, *w13_lo, *w2_lo;
    TcOperands tc_qkv, tc_wo, tc_w13, tc_w2;  // TMA maps of the prefill GEMM operands
};

class BatchDecoder;

class Engine {
    friend class BatchDecoder;

   public:
    static int create(const xl_config& cfg, int device, int tp_size, int tp_rank, const void* nccl_id, Engine** out);
    ~Engine();

    int load(const char* dir);
    // append: the ids continue the cached sequence (positions ctx_len ..), and
    // the repetition set is kept; otherwise the cache and the set restart.
    int prefill(const int* ids, int n, float temperature, float top_p, float rp, int* token_out, bool append = false);
    int decode(int token, float temperature, float top_p, float rp, int* token_out);
    // Up to n decode steps fed on the device (each step's input is the previous
    // step's id), stopping after stop_id (>= 0) or a full cache; the ids go to
    // tokens_out, their count to *n_out.  Same ids, draws and state as that many
    // decode calls.
    int generate(int token, int n, float temperature, float top_p, float rp, int stop_id, int* tokens_out, int* n_out);
    int set_uniforms(const float* u, int n);
    int seed(uint64_t s);
    int last_logits(float* out, int n);
    int kv_copy(int layer, int npos, float* k_out, float* v_out);
    int profile_lm_head(int iters, float* avg_ms);
    int set_option(const char* key, int value);
    int phase_trace(unsigned long long* out, int n);
    int ctx_len() const { return n_; }
    float last_device_ms() const { return last_ms_; }
    float last_kernel_ms() const { return last_kernel_ms_; }
    float last_load_s() const { return last_load_s_; }
    int vocab_begin() const { return v0_; }
    int vocab_count() const { return vl_; }

   private:
    Engine() = default;
    int init(const xl_config& cfg, int device, int tp_size, int tp_rank, const void* nccl_id);
    int alloc_all();
    int capture_decode_graph();
    int capture_gen_graphs();
    int enqueue_decode(cudaStream_t s, bool sampled);
    int enqueue_decode_persistent(cudaStream_t s, bool sampled);
    SampleParams sample_params() const;  // this engine's sequence, single-step sampler chain
    // The persistent kernel streams K in tiles of 64 floats or more, at most
    // 4096 floats, runs at most one attention item per SM and lets at most
    // kPersistMaxContrib SMs share a row group of the residual projections;
    // tensor-parallel ranks need every peer's exchange buffer mapped.
    bool persistent_fits() const {
        return cfg_.layers <= kMaxLayers && (tp_ == 1 || (tp_ <= kMaxTp && peers_)) && H_ % kPersistKAlign == 0 &&
               Hl_ % kPersistKAlign == 0 && Fl_ % kPersistKAlign == 0 && H_ <= 4096 && Hl_ <= 4096 && Fl_ <= 4096 &&
               heads_l_ * persist_attn_ctas_per_head(T_) <= num_sms_ &&
               persist_max_contrib(H_, Hl_, num_sms_) <= kPersistMaxContrib &&
               persist_max_contrib(H_, Fl_, num_sms_) <= kPersistMaxContrib;
    }
    int prepare_prefill_operands();
    int prefill_linear(int mode, const TcOperands& o, const float* x, const float* w, const float* b, float* y,
                       float* y_lo, int n, int m, int k, cudaStream_t s);
    int run_lm_head_and_sample(const float* x_last, const float* delta, cudaStream_t s, bool sampled);
    int lm_tail(cudaStream_t s, bool sampled);  // after the LM head: argmax merge across ranks, id or sampler
    int setup_peers();                          // tensor parallel: map every rank's exchange buffer
    int launch_lm_head(const float* x_last, const float* delta, bool pdl, cudaStream_t s);
    const float* lm_x_ = nullptr;  // residual stream the decode graph's LM head reads
    int finish_step(int* token_out);
    int wait_stream(const char* what);       // bounded under tensor parallelism (step_timeout_ms)
    bool drain_stream(int timeout_ms);
    int abort_tp(const std::string& why);    // graphs released, ncclCommAbort, engine unusable
    int device_error(int bits);
    int check_usable() const;
    float next_uniform();
    int cuda_fail(cudaError_t e, const char* what);
    int nccl_fail(ncclResult_t r, const char* what);

    xl_config cfg_{};
    int device_ = 0;
    int num_sms_ = 148;
    int tp_ = 1, rank_ = 0;
    int H_ = 0, Hl_ = 0, heads_l_ = 0, F_ = 0, Fl_ = 0, V_ = 0, v0_ = 0, vl_ = 0, T_ = 0;

    // device memory
    char* arena_ = nullptr;
    size_t arena_bytes_ = 0;
    float* emb_ = nullptr;     // [V][H] (full table: gather needs every row)
    float* gnorm_ = nullptr;   // [H]
    float2* rope_ = nullptr;   // [T][32]
    std::vector<LayerWeights> layers_;
    float* xa_ = nullptr;      // decode residual stream (ping)
    float* xb_ = nullptr;      // decode residual stream (pong)
    float* cres_ = nullptr;    // persistent decode: partial row sums of the residual projections
    float* qkv_ = nullptr;     // [3*Hl]
    float* att_ = nullptr;     // [Hl]
    float* ffh_ = nullptr;     // [Fl]
    float* part_ = nullptr;    // [H] TP partial sums
    float* logits_ = nullptr;  // [vl]
    float* attn_ws_ = nullptr; // split-K partials
    int* attn_cnt_ = nullptr;  // [heads_l] split counters
    int* done_ = nullptr;      // [5*layers + 1] phase counters of the persistent decode kernel
    unsigned long long* trace_ = nullptr;  // optional phase timeline of the persistent kernel
    uint8_t* rep_flags_ = nullptr;  // [vl]
    DevState* st_ = nullptr;
    void* samp_work_ = nullptr;     // sampler chain work area (sample_work_bytes)
    int samp_grid_ = 1;             // CTAs of the sampler kernels
    // prefill buffers [T][...]
    float *px_ = nullptr, *pxn_ = nullptr, *pqkv_ = nullptr, *patt_ = nullptr, *pffh_ = nullptr;
    float *pxn_lo_ = nullptr, *patt_lo_ = nullptr, *pffh_lo_ = nullptr;
    float* splitk_ws_ = nullptr;  // split-K partial sums of the prefill GEMMs
    size_t splitk_floats_ = 0;
    int* pids_ = nullptr;

    // host
    StepIn* h_in_ = nullptr;   // pinned
    int* h_out_ = nullptr;     // pinned: token_out, err
    int* h_ids_ = nullptr;     // pinned prompt staging
    cudaStream_t stream_ = nullptr;
    cudaEvent_t ev0_ = nullptr, ev1_ = nullptr;
    cudaGraphExec_t decode_exec_ = nullptr;    // greedy step (top_p <= 0)
    cudaGraphExec_t decode_exec_s_ = nullptr;  // sampled step (the sampler chain; TP: candidate merge)
    long long decode_graph_kernels_s_ = 0;
    unsigned long long *cand_local_ = nullptr, *cand_all_ = nullptr;  // tensor-parallel sampling merge
    GenCtl* gen_ctl_ = nullptr;    // device-side generation: control block
    float* gen_u_ = nullptr;       // [T] its draws
    int* gen_out_ = nullptr;       // [T] its ids
    char* h_gen_ = nullptr;        // pinned: GenCtl, draws [T], ids [T]
    cudaGraphExec_t gen_exec_ = nullptr, gen_exec_s_ = nullptr;  // gen_feed + decode step + gen_collect
    long long gen_graph_kernels_ = 0, gen_graph_kernels_s_ = 0;
    ncclComm_t comm_ = nullptr;
    // Tensor parallel, persistent decode: this rank's exchange buffer (its own
    // allocation, exported over CUDA IPC): the tagged partial sums
    // [2][tp][H/16][kPersistMaxContrib][16] (u64); and every rank's buffer
    // mapped here (xpeer_[rank_] == xbuf_).
    char* xbuf_ = nullptr;
    char* xpeer_[kMaxTp] = {};
    bool peers_ = false;

    int decode_path_ = 0;      // 0: persistent kernel (where it fits), 1: per-op kernels
    int prefill_gemm_ = 0;     // 0: tcgen05 3xTF32, 1: fp32 SIMT tiles
    int prefill_attn_ = 0;     // 0: one fused tcgen05 kernel (flash-style), 1: fp32 FMA flash tiles,
                               // 2: tcgen05 S GEMM, softmax, P.V GEMM (all 3xTF32)
    // tensor-core prefill attention: q/8 [T][Hl], k [heads][T][64], v^T [heads*64][T], S/P [heads][T][T]
    float *aq_ = nullptr, *aq_lo_ = nullptr, *ak_ = nullptr, *ak_lo_ = nullptr, *avt_ = nullptr, *avt_lo_ = nullptr;
    float *ap_ = nullptr, *ap_lo_ = nullptr;
    int* fa_tickets_ = nullptr;  // the fused prefill attention's merge tickets [heads][T / 128][4]
    TcOperands tc_attn_s_{}, tc_attn_pv_{};
    FlashOperands flash_{};  // TMA maps of the fused prefill attention's operands
    long long decode_graph_kernels_ = 0;  // kernels recorded in the decode graph
    int load_threads_ = 4;      // weight loader worker threads
    float last_load_s_ = 0.0f;  // wall time of the last load's file reads and copies
    int inflight_ = 3;  // persistent decode: weight boxes requested but not landed, per SM
    int tma_evict_first_ = 1;  // persistent decode: weight boxes loaded with an L2 evict-first policy
    int sig_cta_ = 1;          // persistent decode: one phase signal per CTA (else per warp)
    int resid_smem_ = 1;       // persistent decode: the residual stream kept in each CTA's shared memory
    // persistent decode: split-projection partial sums ordered by tags (implies resid_smem); -1: on under
    // tensor parallelism (TP2: 0.742 -> 0.679 ms/token), off on one GPU (where it is 13 % slower)
    int tag_split_ = -1;
    int tp_merge_ = 1;         // tensor parallel, greedy: the ranks' argmax keys merged inside the persistent kernel
    int tag_skew_ = 0;         // test hook: shift of the tag the tagged exchange's stagings wait for
    // BatchDecoder: 1 = the batched persistent kernel (one launch per step; 1.37 against 1.43 ms per greedy
    // 8-token step of the replica workload's prompts), 0 = per-op kernels
    int batch_persistent_ = 1;
    // Persistent kernel counters, zeroed before each launch: phase counters
    // [5*layers + 1], then the attention merge tickets [layers][heads].
    size_t done_words() const {
        return 5 * static_cast<size_t>(cfg_.layers) + 1 + static_cast<size_t>(cfg_.layers) * heads_l_;
    }
    bool loaded_ = false;
    bool failed_ = false;          // tensor parallel: aborted or a device error; every later step is refused
    std::string fail_msg_;
    bool stream_idle_ = true;      // false: an aborted step never drained (device memory is leaked, not freed)
    int step_timeout_ms_ = 30000;  // tensor parallel: longest host wait for one call's work
    cudaEvent_t ev_sync_ = nullptr;
    bool has_seq_ = false;
    int n_ = 0;
    float last_ms_ = 0.0f;
    float last_kernel_ms_ = -1.0f;     // persistent kernel of the last decode step (kernel_events), or -1
    bool kernel_events_ = false;       // event-record nodes around the persistent kernel in the decode graph
    bool persistent_graph_ = false;    // the decode graph runs the persistent kernel
    cudaEvent_t kev0_ = nullptr, kev1_ = nullptr;
    std::deque<float> uniforms_;
    uint64_t philox_seed_ = 0;
    uint64_t philox_ctr_ = 0;
};

// kBatch sequences decoding together on one GPU over a loaded Engine's
// weights (batch.cu).  The Engine's own sequence serves as the prefill
// scratch: prefill(seq) runs the Engine's prefill and copies the result into
// sequence seq.
class BatchDecoder {
   public:
    static int create(Engine* eng, BatchDecoder** out);
    ~BatchDecoder();
    int seed(int seq, uint64_t s);
    int prefill(int seq, const int* ids, int n, float temperature, float top_p, float rp, int* token_out);
    int decode(const int* tokens, float temperature, float top_p, float rp, int* tokens_out);
    int last_logits(int seq, float* out, int n);
    int ctx_len(int seq) const { return seq >= 0 && seq < kBatch ? n_[seq] : -1; }
    float last_device_ms() const { return last_ms_; }

   private:
    BatchDecoder() = default;
    int init();
    int enqueue(cudaStream_t s, bool sampled);
    int enqueue_persistent(cudaStream_t s, bool sampled);  // the batched persistent kernel
    bool persistent_fits() const;
    int capture();
    float next_uniform(int seq);
    int cuda_fail(cudaError_t e, const char* what);

    Engine* eng_ = nullptr;
    char* arena_ = nullptr;
    std::vector<float*> kc_, vc_;  // per layer [kBatch][heads][T][64]
    float *x_ = nullptr, *qkv_ = nullptr, *att_ = nullptr, *ffh_ = nullptr, *logits_ = nullptr;
    // batched persistent kernel: second residual stream [kBatch][H], partial row sums
    // [kBatch][H/16][kPersistMaxContrib][16], attention partials, phase counters + merge tickets
    float *xb_ = nullptr, *cres_ = nullptr, *part_ = nullptr;
    int *done_ = nullptr, *tick_ = nullptr;
    // residual-finishing tickets [2][layers][H/16][4] of the split projections
    size_t tick_words() const { return 2 * static_cast<size_t>(eng_->cfg_.layers) * (eng_->H_ / kPersistTileRows) * 4; }
    size_t done_words() const {
        return 5 * static_cast<size_t>(eng_->cfg_.layers) + 1 +
               static_cast<size_t>(eng_->cfg_.layers) * kBatch * eng_->heads_l_;
    }
    uint8_t* rep_ = nullptr;       // [kBatch][V]
    DevState* st_ = nullptr;       // [kBatch]
    StepIn* in_ = nullptr;         // [kBatch]
    int* tokens_ = nullptr;        // [kBatch]
    int* ticket_ = nullptr;
    StepIn* h_in_ = nullptr;       // pinned
    DevState* h_st_ = nullptr;     // pinned
    cudaGraphExec_t exec_ = nullptr;    // greedy step
    cudaGraphExec_t exec_s_ = nullptr;  // sampled step (sampler chain)
    long long graph_kernels_ = 0, graph_kernels_s_ = 0;
    void* samp_work_ = nullptr;         // [kBatch] sampler work areas
    size_t samp_stride_ = 0;
    int samp_grid_ = 1;
    cudaEvent_t ev0_ = nullptr, ev1_ = nullptr;
    float last_ms_ = 0.0f;
    uint64_t seed_[kBatch] = {};
    uint64_t ctr_[kBatch] = {};
    int n_[kBatch] = {};
};

// Tensor-parallel partition of one rank (see xl_tp_plan in xl_engine.h).
struct TpPlan {
    int heads, hidden, ffn, vocab_begin, vocab_count;
};
int make_tp_plan(const xl_config& cfg, int tp, int rank, TpPlan* out);

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11): counter (ctr, 0, 0, 0),
// key (seed lo, seed hi); returns the first output word.
uint32_t philox4x32_10_x0(uint64_t ctr, uint64_t seed);
float philox_uniform(uint64_t ctr, uint64_t seed);

// RoPE angle table of the reference (src/rope.cu:47-68), (cos, sin) pairs.
void fill_rope_table(float base, int max_ctx, float* out);

}  // namespace xl
