// Host-side launchers for the XingLing sm_100a kernels.  Every launcher is
// asynchronous on the given stream and returns the launch status.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace xl {

constexpr int kHeadDim = 64;   // XingLing attention head width (src/inference.cu:19-28: 1536 / 24)
constexpr int kHalfHead = 32;  // rotate-half RoPE pairs (j, j + 32), src/rope.cu:20-45
constexpr int kBatch = 8;      // sequences of a batched decode step (batch.cu)
constexpr int kTopK = 1024;    // sampler candidate count, src/inference.cu:66

// Host-written inputs of one step (copied to the device before each call).
struct StepIn {
    int token_in;       // decode input id
    float temperature;  // sample_cpu arguments, src/inference.cu:69-76
    float top_p;
    float rp;
    float uniform;      // the draw r in [0, 1), src/inference.cu:105
    int decode_mode;    // 1: the sampler also advances pos (decode), 0: prefill
    int skip;           // 1: a device-side generation has stopped; every kernel of the step returns at once
    int pad;
};

// Device-resident state of one engine (one sequence per GPU).
struct DevState {
    StepIn in;
    int pos;                          // positions in the KV cache (the reference's KVcache::n)
    int token_out;                    // last sampled id
    int greedy_token;                 // argmax of the penalised logits of the last LM-head pass
    int lm_done;                      // scratch: LM-head CTAs finished (zero between steps)
    unsigned long long argmax_key;    // scratch for the LM-head argmax (zero between steps)
    unsigned long long argmax_final;  // packed (value, id) of the winning logit
    int err;                          // device-side error bits (0 = ok)
    int epoch;                        // persistent decode steps run (tensor parallel: cross-rank counter targets)
    int tp_sync;                      // tensor parallel: step-start liveness sum (tp when every rank joined)
    int tp_one;                       // tensor parallel: the constant 1 each rank adds into tp_sync
};

enum GemvMode : int {
    kGemvPlain = 0,     // y[m] = W[m].x + b[m]
    kGemvSwiGLU = 1,    // rows interleaved (W1 row j, V row j): y[j] = silu(a + b1[j]) * (c + bv[j])
    kGemvResidual = 2,  // y[m] += W[m].x + b[m]   (y is the residual stream)
    kGemvLogits = 3,    // y[m] = E[m].x with repetition penalty; argmax into DevState
};

struct NormGemvParams {
    const float* x;        // input vector [K] (ignored when table != nullptr)
    const float* table;    // gather source: x = table[*token] (decode embedding)
    const int* token;      // device token id for the gather
    const float* delta;    // optional addend: x_eff = x + delta
    float* x_out;          // optional: block 0 stores x_eff here (residual stream)
    const float* gamma;    // optional RMSNorm gain (nullptr: no norm)
    double eps;
    const float* W;        // [M][K] row-major
    const float* bias;     // [M] or nullptr
    float* y;              // output
    int M, K;
    // kGemvLogits only
    const uint8_t* rep_flags;  // [M] 1 = id was sampled since the last prefill
    DevState* st;
    int row_offset;        // global id of row 0 (vocab shard start)
};

cudaError_t launch_norm_gemv(int mode, const NormGemvParams& p, int num_sms, bool pdl, cudaStream_t s);

struct AttnDecodeParams {
    const float* qkv;      // [3 * heads * 64]: q | k | v of this token (pre-RoPE)
    const float2* rope;    // [max_ctx][32] (cos, sin)
    float* kc;             // [heads][max_ctx][64] this layer's key cache
    float* vc;             // [heads][max_ctx][64]
    float* out;            // [heads * 64]
    float* part;           // scratch [heads][max_splits][66]
    int* counters;         // scratch [heads], zero between calls
    const int* pos;        // device position n (the new token's slot)
    int heads, max_ctx;
};
constexpr int kAttnChunk = 64;
__host__ __device__ inline int attn_max_splits(int max_ctx) { return (max_ctx + kAttnChunk - 1) / kAttnChunk; }
cudaError_t launch_attn_decode(const AttnDecodeParams& p, bool pdl, cudaStream_t s);

// Kernels this library ran, process-wide: each launcher counts the kernel it
// enqueues (or records, during a stream capture); a graph's owner subtracts
// the recorded kernels once and adds them back at every replay.
void count_launch();
void count_graph_kernels(long long n);
long long launch_count();

// Persistent decode step (decode_persistent.cu): one cooperative launch per token.
constexpr int kMaxLayers = 32;
constexpr int kPersistChunk = 16;     // attention positions per warp
constexpr int kPersistTileRows = 16;  // weight box streamed per TMA load: 16 rows x up to 512 floats of K
constexpr int kPersistBoxK = 512;     // floats of K per box at most (k-tiles of 256, 128 or 64)
constexpr int kPersistKAlign = 64;    // every streamed K is a multiple of this
constexpr int kPersistSlots = 6;      // 32 KB ring slots per CTA
constexpr int kPersistWarps = 8;      // consumer warps per CTA (attention: one chunk each)
constexpr int kPersistMaxContrib = 4; // CTAs that may share one 16-row group of a residual projection
constexpr int kPersistMaps = 4 * kMaxLayers + 1;  // QKV, Wo, W1/V, W2 per layer, then the LM head
constexpr int kMaxTp = 8;  // tensor-parallel ranks of the persistent decode kernel
__host__ __device__ inline int persistent_max_splits(int max_ctx) {
    return (max_ctx + kPersistChunk - 1) / kPersistChunk;
}
// Geometry of a K-column weight (K % 64 == 0) streamed as 16-row boxes: a
// 3D tensor map of k-tiles of persist_tile_w(K) floats (the widest of 256,
// 128, 64 dividing K; a box dimension holds at most 256 elements), boxes of
// persist_box_tiles(K) tiles (at most 512 floats), persist_boxes_per_group(K)
// boxes per 16-row group (k-tiles past K in the last box are zero-filled).
__host__ __device__ inline int persist_tile_w(int K) { return K % 256 == 0 ? 256 : K % 128 == 0 ? 128 : 64; }
__host__ __device__ inline int persist_box_tiles(int K) {
    const int n = K / persist_tile_w(K), m = kPersistBoxK / persist_tile_w(K);
    return n < m ? n : m;
}
__host__ __device__ inline int persist_box_width(int K) { return persist_tile_w(K) * persist_box_tiles(K); }
__host__ __device__ inline int persist_boxes_per_group(int K) {
    const int kd = persist_box_tiles(K);
    return (K / persist_tile_w(K) + kd - 1) / kd;
}
// The residual projections (out-proj, W2) are split evenly by boxes: CTA b of
// G takes boxes [b*T/G, (b+1)*T/G) of T = (M/16) * nb; box tau belongs to
// persist_owner_cta(tau).  A group's partial row sums come from the CTAs that
// own its boxes, each writing one slot, summed in CTA order: with T >= G every
// CTA owns a box, so they are the CTAs owner(first box) .. owner(last box);
// with T < G a CTA owns at most one box and CTAs without a box lie between,
// so the slot is the box's index within the group.
__host__ __device__ inline int persist_owner_cta(long long tau, long long T, int G) {
    return static_cast<int>(((tau + 1) * G - 1) / T);
}
// Slots (contributing CTAs) of group g.  32-bit arithmetic: the split
// projections have at most 256 groups of 8 boxes, and G is the SM count.
__host__ __device__ inline int persist_group_contrib(int g, int nb, int T, int G) {
    if (T < G) return nb;
    return ((g * nb + nb) * G - 1) / T - ((g * nb + 1) * G - 1) / T + 1;
}
// Slot of CTA b among the contributors of group g, whose first box of the group is bi0.
__host__ __device__ inline int persist_contrib_slot(int b, int g, int bi0, int nb, int T, int G) {
    if (T < G) return bi0;
    return b - ((g * nb + 1) * G - 1) / T;
}
inline int persist_max_contrib(int M, int K, int G) {
    const int nb = persist_boxes_per_group(K), T = (M / kPersistTileRows) * nb;
    int c = 0;
    for (int g = 0; g < M / kPersistTileRows; ++g) {
        const int n = persist_group_contrib(g, nb, T, G);
        c = n > c ? n : c;
    }
    return c;
}
// Attention: CTAs per head, each taking up to kPersistWarps chunks of 32 positions.
__host__ __device__ inline int persist_attn_ctas_per_head(int max_ctx) {
    return (persistent_max_splits(max_ctx) + kPersistWarps - 1) / kPersistWarps;
}
struct LayerPtrs {
    const float *wqkv, *bqkv, *wo, *bo, *w13, *b13, *w2, *b2, *g1, *g2;
    float *kc, *vc;
};
struct PersistentParams {
    CUtensorMap maps[kPersistMaps];  // 3D box maps (make_stream_map) of every streamed matrix
    LayerPtrs layer[kMaxLayers];
    int layers;
    const float* emb;       // [V][H] tied embedding / LM head
    const float* gnorm;     // [H] final RMSNorm gain
    const float2* rope;     // [T][32]
    float* xa;              // [H] residual stream entering a layer (and the LM head's input)
    float* xb;              // [H] residual stream after the out-projection
    float* cres;            // [H/16][kPersistMaxContrib][16] partial row sums of out-proj / W2
    float* qkv;             // [3*Hl]
    float* part;            // attention partials across CTAs [heads][persistent_max_splits][66]
    float* att;             // [Hl] attention output (merged per head)
    int* head_done;         // [layers][heads] CTA tickets of the cross-CTA attention merge
    float* ffh;             // [Fl] SwiGLU activations
    float* logits;          // [V]
    uint8_t* rep_flags;     // [V] ids already generated (penalised; finish_greedy flags the step's id)
    DevState* st;
    int* done;              // [5*layers + 1] phase counters (then head_done), zeroed before each launch
    unsigned long long* trace;  // optional [grid][5*layers + 1][kTraceFields] timestamps (ns), or nullptr
    int inflight;               // weight boxes requested but not landed, per CTA (1 .. kPersistSlots)
    int H, Hl, heads, Fl, V, T;  // V: rows of this rank's vocab shard
    int finish_greedy;          // 1: the LM head's last CTA writes the argmax as the step's id
    int tma_evict_first;        // 1: weight boxes are loaded with an L2 evict-first policy
    int sig_cta;                // 1: one release per CTA signals a phase (after a consumer barrier); 0: one per warp
    int resid_smem;             // 1: every CTA keeps the whole residual stream in shared memory (H floats)
    int tag_skew;               // added to the tag a staging waits for: 0 in service (tests: a tag nobody writes)
    int tag_split;              // 1: out-proj / W2 partial sums go tagged to every rank's xc, the next staging
                                //    waits for the tags (no phase counter); needs resid_smem (also at tp == 1)
    // Tensor parallel (tp > 1): every CTA writes its out-projection / W2 partial
    // row sums into every rank's exchange buffer xc[r] (peer memory over NVLink),
    // laid out [2 (out-proj, W2)][tp][H/16][kPersistMaxContrib][16] words of
    // (tag << 32 | float bits); the tag of layer l's projection w2 in step e is
    // e * 2 * layers + 2 l + w2 + 1 (e = DevState::epoch).
    int tp, rank;
    int v0;                     // global id of this rank's vocab row 0 (argmax keys carry global ids)
    unsigned long long* xc[kMaxTp];
};
constexpr int kTraceFields = 5;

// Batched persistent decode step (decode_persistent.cu): kBatch sequences
// advance one token over a single pass of the weights, in one cooperative
// launch, with the same weight stream and phases as decode_persistent_kernel.
struct BatchPersistParams {
    PersistentParams base;   // weights, maps, geometry, stream options; base.st = st (sequence 0 holds the error word)
    float* xa;               // [kBatch][H] residual streams entering a layer (and the LM head's inputs)
    float* xb;               // [kBatch][H] after the out-projection
    float* cres;             // [kBatch][H/16][kPersistMaxContrib][16] partial row sums of out-proj / W2
    int* tickets;            // [2][layers][H/16][4] per (projection, layer, group, row quad); zeroed before each launch
    float* qkv;              // [kBatch][3*Hl]
    float* att;              // [kBatch][Hl]
    float* ffh;              // [kBatch][Fl]
    float* logits;           // [kBatch][V]
    uint8_t* rep;            // [kBatch][V]
    DevState* st;            // [kBatch]
    float* kc[kMaxLayers];   // per layer [kBatch][heads][T][64]
    float* vc[kMaxLayers];
    float* part;             // [kBatch][heads][persistent_max_splits(T)][66] attention partials across CTAs
    int* head_done;          // [layers][kBatch][heads] CTA tickets of the cross-CTA attention merge
    int* done;               // [5*layers + 1] phase counters; head_done follows; zeroed before each launch
    int finish_greedy;       // 1: the LM head's last CTA writes every sequence's argmax as its id
};
size_t batch_persistent_smem_bytes();
// The batched kernel streams K up to this many floats (every sequence's staged input in shared memory).
constexpr int kBatchPersistMaxK = 4096;
cudaError_t launch_decode_batch_persistent(const BatchPersistParams& p, int num_sms, cudaStream_t s);
size_t persistent_smem_bytes(int H, int resid_smem);
// The TMA map (no swizzle) of a row-major [rows][cols] weight viewed as
// [rows][cols/tw][tw] (tw = persist_tile_w(cols)), box [16 rows]
// [persist_box_tiles(cols) k-tiles][tw floats]; cols must be a multiple of 64.
cudaError_t make_stream_map(CUtensorMap* map, const float* base, int rows, int cols);
cudaError_t launch_decode_persistent(const PersistentParams& p, int num_sms, cudaStream_t s);

// ---- sampler: sample_cpu (src/inference.cu:58-114) over one vocab shard ----
// A chain of grid-wide kernels per step: up to three radix-histogram passes
// over the float keys (11 + 11 + 10 bits from the top), each over vocab
// slices on all SMs, whose last CTA (an atomic ticket) picks the bin holding
// the 1024th largest key; then one gather kernel whose slices collect the
// selected ids and whose last CTA sorts them and draws.  No CTA waits on
// another.  The selection stops as soon as exactly 1024 ids are at or above
// the chosen prefix; a tie at the full threshold key is resolved in id order
// from per-slice lists.  A vocab of at most kCandCap ids is taken whole.
constexpr int kCandCap = 4096;   // candidates sorted by the last CTA
constexpr int kSampThreads = 1024;
struct SampleWorkHdr {
    unsigned int prefix, pmask;  // radix prefix chosen so far and its mask
    int n_above;                 // ids whose masked key is above prefix (all taken)
    int n_ge;                    // ids whose key is at or above prefix
    int passes;                  // histogram passes done this step
    int done;                    // 1: selection finished (gather may run)
    int exact;                   // 1: prefix is the full threshold key and more than kc ids reach it
    int ticket;                  // CTAs finished in the current kernel
    int n_gt;                    // gather: candidate slots taken
    int pad[7];
};
// Per-sequence work area (zeroed once; every step leaves it zeroed):
// header, histogram [2048], candidates [kCandCap], per-slice tie counts
// [grid] and tie ids [grid][slice].
size_t sample_work_bytes(int V, int grid);
// CTAs per sequence of the sampler kernels for `batch` sequences.
int sample_grid(int V, int num_sms, int batch);

struct SampleParams {
    const float* logits;   // [V] penalised logits of this vocab shard
    int V;                 // shard size
    int v0;                // global id of shard row 0
    DevState* st;
    uint8_t* rep_flags;    // [V]
    int full;              // 1: always run the full top-k path (no argmax shortcut)
    unsigned long long* cand_out;  // tensor parallel: write the shard's sorted top-1024 here, draw nothing
    void* work;            // sample_work_bytes(V, grid) per sequence
    size_t work_stride;    // bytes between sequences' work areas
    int stride;            // floats (and flag bytes) between sequences' logits
    int grid;              // CTAs per sequence (sample_grid)
};
// The sampling chain for `batch` sequences (sequence b: logits + b * stride,
// rep_flags + b * stride, st + b, work + b * work_stride): three histogram
// launches and the gather launch.
cudaError_t launch_sample_chain(const SampleParams& p, int batch, bool pdl, cudaStream_t s);
// Greedy steps (top_p <= 0): write the LM head's argmax as the step's id.
cudaError_t launch_sample_finish(const SampleParams& p, int batch, bool pdl, cudaStream_t s);

// Device-side generation (InferenceEngine.generate): each step of a decode
// graph is bracketed by gen_feed (step input from the previous step's id and
// the step's uniform) and gen_collect (record the id; a stop id ends the run).
struct GenCtl {
    int step;      // steps done
    int n;         // steps requested
    int first;     // input id of step 0
    int stop_id;   // -1: none
    int stopped;   // 1 after the stop id was produced
    int max_ctx;
    float temperature, top_p, rp;
    int pad[7];
};
struct GenParams {
    GenCtl* ctl;
    const float* uniforms;  // [n] the draws of the steps, in order
    int* out;               // [n] the ids produced
    DevState* st;
};
cudaError_t launch_gen_feed(const GenParams& p, cudaStream_t s);
cudaError_t launch_gen_collect(const GenParams& p, cudaStream_t s);

// Tensor-parallel sampling merge: the all-gathered per-shard candidate lists
// (packed (value key, ~global id), n = tp x 1024), sorted as one; draws as
// the single-GPU gather kernel does.  n_pad: n rounded up to a power of two.
constexpr int kMaxMergeCandidates = 8 * kTopK;
struct SampleMergeParams {
    const unsigned long long* cand;
    int n, n_pad;
    int V_total;           // full vocabulary (the candidate count is min(V_total, 1024))
    DevState* st;
    uint8_t* rep_flags;    // [V] this rank's shard
    int V;                 // shard size
    int v0;                // global id of shard row 0
};
cudaError_t launch_sample_merge(const SampleMergeParams& p, bool pdl, cudaStream_t s);

// ---- prefill on tcgen05 (gemm_tc.cu) ----
// Operand maps of one projection: W and W_lo ([M][K]), X and X_lo ([rows][K]),
// each a 2D TMA map with {32, 128} boxes and 128B swizzle (make_tile_map);
// with `wide`, X and X_lo also with {32, 256} boxes for 256-token tiles.
struct TcOperands {
    CUtensorMap w, w_lo, x, x_lo;
    CUtensorMap x_wide, x_lo_wide;
    bool wide = false;
};
cudaError_t make_tile_map(CUtensorMap* map, const float* base, int rows, int cols, int box_rows = 128);
// C[N][M] (+)= X[N][K] . W[M][K]^T + b with the 3xTF32 split; SwiGLU writes C and C_lo as [N][M/2].
// With a workspace (ws, ws_floats) and fewer output tiles than SMs, K is split
// into slices whose partial sums are added in slice order by a second kernel.
// Tensor-core prefill attention, around the two GEMMs below: RoPE + KV append
// + the operands (a prompt starting at position 0), and the causal row softmax
// of S in place.
cudaError_t launch_attn_prep(const float* qkv, const float2* rope, float* kc, float* vc, float* q8, float* q8_lo,
                             float* kq, float* kq_lo, float* vt, float* vt_lo, int n, int heads, int max_ctx,
                             cudaStream_t s);
cudaError_t launch_attn_softmax(float* S, float* P_lo, int n, int heads, int max_ctx, cudaStream_t s);
// Prefill attention on tcgen05 (3xTF32), per head z as the grid's third
// dimension: operand tile coordinates advance by (w_x, w_y) and (x_x, x_y) per
// head.  Scores: C = S[z][t][ldc] with c_rows rows per head.  P.V: C, C_lo =
// out[t][ldc] at column z * c_col.
struct GemmBatch {
    int w_x, w_y, x_x, x_y;
    int c_rows, ldc, c_col;
};
// S[h][q][k] = (q/8 . k) for q, k < n (tiles above the diagonal are skipped).
// o.x / o.x_lo: q/8 [T][heads*64]; o.w / o.w_lo: k [heads*T][64] (make_tile_map).
cudaError_t launch_attn_scores_tc(const TcOperands& o, float* S, int n, int heads, int max_ctx, int* err,
                                  cudaStream_t s);
// out[q][h*64 + d] (and its lo half) = sum over keys k <= q of P[h][q][k] v[h][k][d].
// o.x / o.x_lo: P [heads*T][T]; o.w / o.w_lo: v transposed [heads*64][T].
cudaError_t launch_attn_pv_tc(const TcOperands& o, float* out, float* out_lo, int n, int heads, int max_ctx, int* err,
                              cudaStream_t s);
// Causal attention of a prompt starting at position 0 in one kernel per layer
// (flash-style: scores and probabilities stay in TMEM and shared memory):
// out[q][h*64 + d] and its lo half for q < n.  Operand maps ({32, rows}
// boxes, 128B swizzle): q/8 and q_lo [T][heads*64] with 128-row boxes; k and
// k_lo [heads*T][64] and v^T and its lo half [heads*64][T] with 64-row boxes.
struct FlashOperands {
    CUtensorMap q, q_lo, k, k_lo, v, v_lo;
};
// Rows longer than 4 key tiles of 64 are split over CTAs, whose partial rows
// meet in a workspace of attn_flash_ws_floats(heads, max_ctx) floats, merged
// by the last of them (tickets: heads * ceil(max_ctx / 128) * 4 ints, zero
// before the first launch and left zero by every complete launch).
size_t attn_flash_ws_floats(int heads, int max_ctx);
cudaError_t launch_attn_flash_tc(const FlashOperands& o, float* out, float* out_lo, int n, int heads, int max_ctx,
                                 float* ws, size_t ws_floats, int* tickets, int* err, cudaStream_t s);
cudaError_t launch_gemm_tc(int mode, const TcOperands& o, const float* bias, float* C, float* C_lo, int n, int m,
                           int k, int* err, cudaStream_t s, float* ws = nullptr, size_t ws_floats = 0,
                           int num_sms = 148);
// lo[i] = x[i] - (x[i] with its 13 low mantissa bits cleared): the TF32 residual.
cudaError_t launch_split_lo(const float* x, float* lo, size_t n, cudaStream_t s);

// ---- prefill ----
cudaError_t launch_embed_gather(const float* table, const int* ids, float* out, int n, int k, cudaStream_t s);
// out_lo (optional) receives the TF32 residual of out for the 3xTF32 GEMMs.
cudaError_t launch_rmsnorm_rows(const float* x, const float* gamma, float* out, float* out_lo, int n, int k,
                                cudaStream_t s);
// Y[N][M] (+)= X[N][K] . W[M][K]^T + b; mode as GemvMode (Plain / SwiGLU / Residual).
cudaError_t launch_linear_prefill(int mode, const float* X, const float* W, const float* b, float* Y, int n,
                                  int m, int k, cudaStream_t s);
// Rows t < n of qkv are positions p0 + t (p0 > 0: a prompt appended to a cached sequence).
cudaError_t launch_rope_kv_prefill(float* qkv, const float2* rope, float* kc, float* vc, int n, int heads,
                                   int max_ctx, cudaStream_t s, int p0 = 0);
// x[i] += d[i] for i < n (tensor-parallel residual add after an all-reduce).
cudaError_t launch_add_rows(float* x, const float* d, int n, cudaStream_t s);
cudaError_t launch_attn_prefill(const float* qkv, const float* kc, const float* vc, float* out, float* out_lo, int n,
                                int heads, int max_ctx, cudaStream_t s, int p0 = 0);

}  // namespace xl
