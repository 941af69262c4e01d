/*
 * xl_engine.h — C ABI of the B200-native XingLing token-loop engine
 * (libxl_engine.so).
 *
 * The engine replaces the reference's InferenceEngine / Transformer stack
 * (fancyovo/XingLing-cpp, include/inference.h:16-38, include/ops.h:174-201)
 * behind plain C entry points: opaque handles, plain pointers and sizes, and
 * an int status on every call (XL_OK = 0).  The reference exits the process
 * on almost every error (include/utils.h:7-36); here each failure is a status
 * code plus a message from xl_last_error().  The pybind11 module
 * `llm_cpp_engine` (the reference's Python surface, src/bindings.cpp:7-39)
 * is a thin layer over these calls.
 *
 * The op-level entry points (xl_op_*) run one kernel on device pointers the
 * caller owns, on the caller's CUDA stream; they exist so that each kernel
 * can be checked on its own against the oracle, as the reference's own C++
 * tests check each op (tests/test_*.cu).
 */
#ifndef XL_ENGINE_H
#define XL_ENGINE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define XL_API __attribute__((visibility("default")))

/* Status codes. */
enum {
    XL_OK = 0,
    XL_ERR_ARG = 1,      /* bad argument (sizes, device string, empty prompt) */
    XL_ERR_TOKEN = 2,    /* token id outside [0, vocab): reference exits, src/embedding.cu:77-81,113-116 */
    XL_ERR_CTX = 3,      /* context full: reference exits, src/inference.cu:117-120, src/attn.cu:506-515 */
    XL_ERR_IO = 4,       /* weight file missing or short: reference throws, src/tensor.cu:113-126 */
    XL_ERR_CUDA = 5,     /* CUDA runtime error */
    XL_ERR_NCCL = 6,     /* NCCL error (tensor-parallel engines) */
    XL_ERR_STATE = 7,    /* call out of order (e.g. decode before load / prefill) */
    XL_ERR_DEVICE = 8    /* a kernel reported an error through its status word */
};

/* Model shape.  xl_config_default fills the XingLing-0.68B constants of the
 * reference's engine constructor (src/inference.cu:19-28): 16 layers, hidden
 * 1536, 24 heads of 64, FFN 4096, vocab 151669, context 768, RoPE base 1e4.
 * Smaller shapes (hidden a multiple of 64, ffn a multiple of 8) serve tests. */
typedef struct xl_config {
    int layers;
    int hidden;
    int heads;
    int ffn;
    int vocab;
    int max_ctx;
    float rope_base;
} xl_config;

typedef struct xl_engine xl_engine;

/* Message of the last failed call on this thread ("" if none). */
XL_API const char* xl_last_error(void);

XL_API void xl_config_default(xl_config* cfg);

/* InferenceEngine::InferenceEngine (src/inference.cu:18-40): builds the
 * engine on CUDA device `device` (the reference's device string "cuda" is
 * device 0).  Allocates every weight, the head-major KV cache and the work
 * buffers once.  tp_size / tp_rank / nccl_id select tensor-parallel decode:
 * tp_size 1 ignores the other two; otherwise nccl_id points to the
 * XL_NCCL_ID_BYTES bytes from xl_nccl_unique_id() on rank 0, shared by all
 * ranks, and every rank must create its engine concurrently, one process per
 * GPU of one node: creation also maps every rank's exchange buffer over CUDA
 * IPC (the persistent decode kernel writes its partial sums there) and fails
 * with XL_ERR_CUDA if a mapping cannot be made, or with XL_ERR_ARG if the
 * ranks' SM counts or shapes differ (the exchange slots are laid out by each
 * rank's grid).  Tensor parallel, every later call: the host's wait for the
 * call's GPU work is bounded by the option step_timeout_ms (default 30000)
 * and by NCCL's asynchronous error; past either, the engine aborts its
 * communicator and returns XL_ERR_NCCL, and every later call returns
 * XL_ERR_STATE (the ranks must create new engines).  A device error on a
 * tensor-parallel rank makes the engine unusable the same way; on one GPU it
 * drops the cached sequence instead (the next prefill starts clean). */
#define XL_NCCL_ID_BYTES 128
XL_API int xl_engine_create(const xl_config* cfg, int device, int tp_size, int tp_rank, const void* nccl_id,
                            xl_engine** out);
XL_API int xl_nccl_unique_id(void* out, int nbytes);

/* Releases all device and host memory of the engine. */
XL_API void xl_engine_destroy(xl_engine* e);

/* InferenceEngine::load (src/inference.cu:44-46) -> Transformer::load
 * (src/transformer.cu:139-146): reads the raw little-endian fp32 weight tree
 * (embedding/weight.bin, norm/weight.bin, blocks/{i}/attn/{Q,K,V,W}/{weight,
 * bias}.bin, blocks/{i}/ffn/{W1,V,W2}/{weight,bias}.bin,
 * blocks/{i}/norm{1,2}/weight.bin) into device memory, this rank's shard only. */
XL_API int xl_engine_load(xl_engine* e, const char* dir);

/* InferenceEngine::next_token(vector) (src/inference.cu:116-136): prefill of
 * `n` prompt ids (1 <= n <= max_ctx), resets the KV cache and the repetition
 * set, samples the next id into *token_out and records it in the set. */
XL_API int xl_engine_prefill(xl_engine* e, const int* ids, int n, float temperature, float top_p,
                             float repetition_penalty, int* token_out);

/* Prefill continuation (no reference counterpart: the reference restarts the
 * cache on every prompt, src/attn.cu:350,360): the n ids extend the cached
 * sequence at positions ctx_len .. ctx_len + n - 1, attending to every cached
 * position; the repetition set is kept.  Samples the next id like
 * xl_engine_prefill.  XL_ERR_STATE before any prefill, XL_ERR_CTX past the
 * context. */
XL_API int xl_engine_extend(xl_engine* e, const int* ids, int n, float temperature, float top_p,
                            float repetition_penalty, int* token_out);

/* InferenceEngine::next_token(int) (src/inference.cu:138-151): one decode
 * step at position ctx_len (XL_ERR_CTX when the cache is full). */
XL_API int xl_engine_decode(xl_engine* e, int token, float temperature, float top_p, float repetition_penalty,
                            int* token_out);

/* Device-side multi-token loop (no reference counterpart; replaces the
 * per-token host loop of the reference's main.py:26-27 and
 * test_speed.py:52-57): up to n decode steps, step 0 fed `token`, each later
 * step the previous step's id, all without a host round trip between steps
 * (one CUDA graph launch per step, one synchronisation at the end).  Stops
 * after producing stop_id (when >= 0; it is returned) or when the cache is
 * full.  tokens_out receives the ids (capacity n), *n_out their count.  The
 * ids, the uniforms consumed (one per step taken) and the engine state equal
 * those of *n_out successive xl_engine_decode calls.  With the persistent
 * decode kernel the loop runs on the device: on one GPU for greedy and sampled
 * steps, under tensor parallelism for greedy steps (option tp_merge 1, the
 * default; every rank must make the same call, as for decode).  Otherwise it
 * is that host loop. */
XL_API int xl_engine_generate(xl_engine* e, int token, int n, float temperature, float top_p,
                              float repetition_penalty, int stop_id, int* tokens_out, int* n_out);

/* Sampling-uniform control (no reference counterpart: the reference seeds a
 * std::mt19937 from std::random_device, src/inference.cu:37-38).  Each
 * next-token call consumes one uniform in [0, 1): first the queued values
 * given to xl_engine_set_uniforms (replacing any queue), then the engine's
 * Philox4x32-10 stream, key = seed, counter = draw index, u = (x0 >> 8) / 2^24. */
XL_API int xl_engine_set_uniforms(xl_engine* e, const float* u, int n);
XL_API int xl_engine_seed(xl_engine* e, uint64_t seed);
/* The uniforms draws [start, start + n) of the Philox stream with key seed
 * (host only, no GPU needed). */
XL_API int xl_philox_uniforms(uint64_t seed, uint64_t start, int n, float* out);

/* Tensor-parallel shard plan of rank `rank` of `tp` (host only): out[0] heads
 * on this rank, out[1] its attention width (heads * 64), out[2] its FFN
 * columns, out[3] first vocab id of its LM-head shard, out[4] shard size.
 * Heads and FFN columns split evenly; the vocab splits into tp contiguous
 * shards of ceil(vocab / tp) ids, the last one shorter.  No reference
 * counterpart (the reference runs on one device). */
XL_API int xl_tp_plan(const xl_config* cfg, int tp, int rank, int* out);

/* Copies this rank's logits of the last step (after the repetition penalty,
 * before temperature) to host memory: n must equal xl_engine_vocab_shard(). */
XL_API int xl_engine_last_logits(xl_engine* e, float* out, int n);
XL_API int xl_engine_vocab_shard(const xl_engine* e, int* begin, int* count);

/* KVcache::n of the reference (src/attn.cu:11-16): cached positions. */
XL_API int xl_engine_ctx_len(const xl_engine* e);

/* Copies cache rows [0, npos) of one layer, as the reference's position-major
 * [npos][heads][64] layout, for this rank's heads. */
XL_API int xl_engine_kv_copy(xl_engine* e, int layer, int npos, float* k_out, float* v_out);

/* Engine options (no reference counterpart):
 *   "decode_path" 0  one persistent kernel per decode token (default): a TMA
 *                    weight stream through shared memory across all layers
 *                    and the LM head, phases gated by grid-wide counters;
 *                    tensor-parallel ranks exchange the out-projection and
 *                    W2 partial sums inside it over NVLink peer memory;
 *                 1  one kernel per fused op (NCCL all-reduces under tensor
 *                    parallelism).
 *   "phase_trace" 1  the persistent kernel stamps %globaltimer (ns) per CTA
 *                    and phase: consumer start (after the grid-wide wait),
 *                    input staged, phase done, producer first and last issue;
 *                    read with xl_engine_phase_trace (a profiling aid);
 *   "tma_inflight" n  weight boxes (32 KB) each SM of the persistent kernel
 *                    keeps requested but not landed, in [1, 6] (default 3):
 *                    enough to keep HBM busy, few enough that other memory
 *                    accesses do not queue behind the stream;
 *   "tma_evict_first" 1  the persistent kernel loads weight boxes with an L2
 *                    evict-first policy (default), keeping activations and
 *                    cached K/V in L2; 0  the default L2 policy;
 *   "load_threads" n  worker threads of xl_engine_load, in [1, 64] (default
 *                    4): each preads chunks of the weight files into its own
 *                    pinned buffers and copies them on its own stream;
 *   "kernel_events" 1  event-record nodes around the persistent kernel in the
 *                    decode graph, so xl_engine_last_kernel_ms reports its
 *                    own duration;
 *   "prefill_gemm" 0  prefill projections on tcgen05 with the 3xTF32 split
 *                     (default); 1  fp32 FMA tiles.
 *   "batch_persistent" 1  a batch decoder created afterwards runs each step
 *                    as one batched persistent kernel (default, where the
 *                    shape fits it); 0  per-op batched kernels;
 *   "prefill_attn" 0  prefill attention in one tcgen05 kernel per layer
 *                     (3xTF32, flash-style: scores in TMEM, online softmax,
 *                     P in shared memory; the default);
 *                  1  fp32 FMA flash-style tiles with online softmax;
 *                  2  tcgen05 in three kernels: S = q k^T per head, causal
 *                     row softmax, P v.
 * Changing an option re-captures the decode graph. */
XL_API int xl_engine_set_option(xl_engine* e, const char* key, int value);
/* The last decode step's phase timeline: n = SMs x (5 x layers + 1) x 5
 * values, [cta][phase][field], phases ordered QKV, attention, out-proj,
 * W1/V, W2 per layer, then the LM head. */
XL_API int xl_engine_phase_trace(xl_engine* e, unsigned long long* out, int n);

/* Device time of the last prefill / decode call in milliseconds (CUDA events
 * around the device work, excluding host copies). */
XL_API int xl_engine_last_device_ms(const xl_engine* e, float* ms);

/* Duration of the persistent decode kernel alone in the last decode step
 * (CUDA events in the decode graph; needs option "kernel_events" = 1 and the
 * persistent path), else -1.  No reference counterpart: a profiling aid. */
XL_API int xl_engine_last_kernel_ms(const xl_engine* e, float* ms);

/* Wall time in seconds of the last xl_engine_load's file reads and
 * host-to-device copies (option "load_threads" workers, default 4). */
XL_API int xl_engine_last_load_s(const xl_engine* e, float* s);

/* Kernels this library has run in this process, every engine and op entry
 * point included (a decode graph's kernels count at each replay).  No
 * reference counterpart: lets a caller check that the GPU path ran. */
XL_API long long xl_kernel_launches(void);

/* Launches the engine's fused final-norm + LM-head kernel (the largest single
 * kernel of a decode step: it streams the whole tied embedding table) `iters`
 * times back to back on the engine's stream and returns the mean duration
 * from CUDA events.  Leaves the logits of the last step unchanged in value. */
XL_API int xl_engine_profile_lm_head(xl_engine* e, int iters, float* avg_ms);

/* ---- batched decode (no reference counterpart) -------------------------
 * XL_BATCH sequences decode together on one GPU, sharing one pass over the
 * weights of a loaded single-GPU engine (the reference decodes one sequence at
 * a time).  Each sequence has its own KV cache, repetition set, Philox stream
 * and position.  xl_batch_prefill runs the engine's own prefill (so the
 * engine's single sequence is overwritten) and makes the result sequence seq;
 * xl_batch_decode feeds tokens[b] to every sequence b and returns the next id
 * of each, with the same sampling arguments for all.  The engine must outlive
 * the batch decoder, and the two must not be used from different threads at
 * once (they share the engine's stream). */
#define XL_BATCH 8
typedef struct xl_batch xl_batch;
XL_API int xl_batch_create(xl_engine* e, xl_batch** out);
XL_API void xl_batch_destroy(xl_batch* b);
XL_API int xl_batch_seed(xl_batch* b, int seq, unsigned long long seed);
XL_API int xl_batch_prefill(xl_batch* b, int seq, const int* ids, int n, float temperature, float top_p,
                            float repetition_penalty, int* token_out);
XL_API int xl_batch_decode(xl_batch* b, const int* tokens, float temperature, float top_p,
                           float repetition_penalty, int* tokens_out);
/* Penalised logits of sequence seq after the last decode step (n >= vocab). */
XL_API int xl_batch_last_logits(xl_batch* b, int seq, float* out, int n);
XL_API int xl_batch_ctx_len(const xl_batch* b, int seq);
XL_API int xl_batch_last_device_ms(const xl_batch* b, float* ms);

/* ---- op-level entry points (device pointers, caller's stream) ---------- */

/* RMSNorm::forward (src/rmsnorm.cu:112-147) fused with
 * Linear::forward_vec (src/linear.cu:309-357), plus epilogues:
 * mode 0: y = W.norm(x) + b;  mode 1: SwiGLU over interleaved (W1, V) rows,
 * y[j] = silu(a_j + b_2j) * (c_j + b_2j+1) (src/ffn.cu:126-139);
 * mode 2: y += W.x + b (residual, src/transformer.cu:54-59).
 * gamma may be NULL (no norm).  W is [m][k] row-major, k % 4 == 0. */
XL_API int xl_op_norm_gemv(int mode, const float* x, const float* gamma, const float* w, const float* b, float* y,
                           int m, int k, void* stream);

/* The RoPE angle table of src/rope.cu:47-68 on the host:
 * out[(pos * 32 + j) * 2 + {0, 1}] = {cos, sin}(base^(-2j/64) * pos) for
 * pos < max_ctx, j < 32, each angle formed in fp32 as the reference does.
 * Ops taking `rope` expect this table copied to device memory. */
XL_API int xl_rope_table(float base, int max_ctx, float* out);

/* RoPE::forward_vec (src/rope.cu:130-165) + KV append +
 * MultiHeadAttention::forward (src/attn.cu:490-547) for one token at
 * position pos (device int, 0 <= pos < max_ctx: a position outside that
 * range leaves the caches untouched and writes NaN to every output, since the
 * value is on the device and the call does not synchronize to check it).
 * qkv = [q | k | v] of `heads` heads (pre-RoPE);
 * kc / vc are head-major [heads][max_ctx][64].  workspace: at least
 * xl_op_attn_decode_workspace_bytes(heads, max_ctx) bytes, zero-filled
 * before first use (the kernel leaves it zeroed). */
XL_API size_t xl_op_attn_decode_workspace_bytes(int heads, int max_ctx);
XL_API int xl_op_attn_decode(const float* qkv, const float* rope, float* kc, float* vc, float* out, const int* pos,
                             int heads, int max_ctx, void* workspace, void* stream);

/* xl_op_attn_decode for callers that cannot allocate device memory.  No
 * counterpart in the reference.  Some hosts cannot call cudaMalloc on the
 * decode path: an embedder whose device memory is owned by a pool it must not
 * bypass, or a latency-critical caller for whom a cudaMalloc (which may
 * synchronize the device) is not acceptable.  This entry point needs no
 * workspace: its split-K scratch is a static device array of about 132 KB
 * inside the library, which every GPU that loads the library holds until the
 * process exits.  Limits: heads <= 32, max_ctx <= 1024; larger sizes return
 * XL_ERR_ARG (use xl_op_attn_decode with a workspace).  It allocates nothing
 * and calls no allocating routine.  The first call on each device looks up
 * the array's device address with that device current; make that first call
 * before any stream capture.  All calls share the one array: calls that
 * overlap on the GPU (other streams, other threads) race on it, so order them
 * on one stream.  Same arguments, results and position precondition
 * (0 <= pos < max_ctx, else NaN outputs and untouched caches) as
 * xl_op_attn_decode. */
XL_API int xl_op_attn_decode_noalloc(const float* qkv, const float* rope, float* kc, float* vc, float* out,
                                     const int* pos, int heads, int max_ctx, void* stream);

/* Embedding::inverse (src/embedding.cu:173-205) fused with the final RMSNorm
 * (gamma may be NULL) and the repetition penalty of sample_cpu
 * (src/inference.cu:71-74): logits[v] = E[v].x, penalised where
 * rep_flags[v] != 0; *argmax_out receives the id of the largest logit
 * (lowest id on ties).  workspace: xl_op_lm_head_workspace_bytes() bytes,
 * zero-filled before first use. */
XL_API size_t xl_op_lm_head_workspace_bytes(void);
XL_API int xl_op_lm_head(const float* x, const float* gamma, const float* table, float* logits,
                         const uint8_t* rep_flags, float repetition_penalty, int vocab, int k, int* argmax_out,
                         void* workspace, void* stream);

/* sample_cpu (src/inference.cu:69-114) on the device with the uniform r
 * supplied: top-1024 by value, / (T + 0.001), softmax, top-p prefix, draw.
 * logits must already carry the repetition penalty.  workspace:
 * xl_op_sample_workspace_bytes(vocab) bytes (any contents; cleared on the
 * stream by the call); synchronous (the id is returned in *token_out). */
XL_API size_t xl_op_sample_workspace_bytes(int vocab);
XL_API int xl_op_sample(const float* logits, int vocab, float temperature, float top_p, float r, int* token_out,
                        void* workspace, void* stream);

/* Linear::forward (src/linear.cu:197-253): Y[n][m] = X[n][k] . W[m][k]^T + b
 * with the same three modes as xl_op_norm_gemv (SwiGLU writes [n][m/2]).
 * With x_lo and w_lo (the TF32 residuals from xl_op_split_lo) the product
 * runs on the tcgen05 tensor cores as X.W_hi + X_lo.W_hi + X_hi.W_lo
 * (3xTF32, fp32-level accuracy; k % 32 == 0; SwiGLU also writes y_lo);
 * with x_lo or w_lo NULL it runs as fp32 FMA tiles. */
XL_API int xl_op_linear(int mode, const float* x, const float* x_lo, const float* w, const float* w_lo,
                        const float* b, float* y, float* y_lo, int n, int m, int k, void* stream);

/* lo[i] = x[i] - (x[i] with its 13 low mantissa bits cleared): the part of
 * an fp32 value a TF32 tensor-core operand drops. */
XL_API int xl_op_split_lo(const float* x, float* lo, size_t n, void* stream);

/* RMSNorm::forward on [n][k] rows (out may alias x). */
XL_API int xl_op_rmsnorm(const float* x, const float* gamma, float* out, int n, int k, void* stream);

/* Embedding::forward (src/embedding.cu:75-110): out[i] = table[ids[i]]
 * (ids on the device, validated by the caller). */
XL_API int xl_op_embedding(const float* table, const int* ids, float* out, int n, int k, void* stream);

/* RoPE::forward on q and k (src/rope.cu:70-106) + KV-cache fill +
 * MultiHeadAttention::prefill (src/attn.cu:319-365): qkv is [n][3*heads*64]
 * (q rotated in place), out is [n][heads*64]. */
XL_API int xl_op_attn_prefill(float* qkv, const float* rope, float* kc, float* vc, float* out, int n, int heads,
                              int max_ctx, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* XL_ENGINE_H */
