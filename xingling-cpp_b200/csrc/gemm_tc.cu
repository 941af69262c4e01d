// Prefill projections on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// C[N][M] (+)= X[N][K] . W[M][K]^T + b for the prefill Linear layers, the
// dense contraction of Linear::forward (src/linear.cu:106-168, 197-253).
//
// Precision: fp32 operands through kind::tf32 with the 3xTF32 split.  The
// tensor core reads the top 19 bits of each fp32 operand (sign, exponent, 10
// mantissa bits), so with lo(v) = v - trunc19(v):
//   X.W ~= X.W_hi + X_lo.W_hi + X_hi.W_lo      (the lo.lo term, ~2^-22
// relative, is dropped), which keeps the fp32 accuracy the reference's CPU
// path has.  A single TF32 product misses the logit tolerance on this model
// (about 1.5e-3 of the logit range after 16 layers), three do not.  W_lo is
// prepared once at load time, X_lo by the kernel that produces X.
//
// Tile: 128 output features (MMA M) x 128 or 256 tokens (MMA N), K-blocks of
// 32 floats (128 B, the SWIZZLE_128B span).  Warp 0 issues TMA loads of the
// four operand tiles of a K-block into a ring (3 stages of 64 KB, or 2 of 96 KB
// for 256 tokens) and prefetches the weight tiles of a later K-block into L2;
// warp 1 (one thread) issues 4 K-steps x 3 tcgen05.mma per K-block into an fp32
// accumulator in TMEM and frees each stage with tcgen05.commit; warps 2..5
// read the accumulator with tcgen05.ld and apply the epilogue (bias; residual
// add; SwiGLU over interleaved (W1 j, V j) feature pairs, which also writes
// the lo half for the next GEMM).
#include <cuda.h>
#include <math.h>

#include <algorithm>

#include "xl_device.cuh"
#include "xl_kernels.h"

namespace xl {

namespace {

constexpr int kBM = 128;               // output features per tile (MMA M)
constexpr int kBN = 128;               // tokens per tile (MMA N; 256-token tiles: TileCfg<256>)
constexpr int kBK = 32;                // floats per K-block (128 B rows)
constexpr int kTileBytes = kBM * kBK * 4;  // 16 KB: one 128-row operand tile of a K-block
constexpr int kGemmThreads = 192;
constexpr uint32_t kSpinLimit = 1u << 26;
constexpr unsigned long long kWaitLimitNs = 200ull * 1000 * 1000;  // a tile's operands land in microseconds
constexpr int kGemmPartial = 4;  // epilogue: raw slice accumulator into the split-K workspace
constexpr int kGemmScores = 5;   // attention: S[z][n][m] = q_n . k_m per head z (tiles above the diagonal skipped)
constexpr int kGemmPV = 6;       // attention: O[n][z*64 + f] (+ lo) = P[z][n][:] . V[:][f], keys up to the tile's last query

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
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
__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// Bounded by polls and by wall-clock time (a try_wait may suspend the thread).
__device__ bool wait_bar(uint64_t* bar, uint32_t parity, int* err) {
    uint32_t it = 0;
    unsigned long long t0 = 0;
    while (!mbar_try_wait(bar, parity)) {
        ++it;
        if ((it & 63u) == 0) {
            const unsigned long long now = globaltimer_ns();
            if (t0 == 0) t0 = now;
            if (it >= kSpinLimit || now - t0 > kWaitLimitNs) {
                if (err) atomicOr(err, 4);
                return false;
            }
        }
    }
    return true;
}
// 2D TMA tile load (no multicast): box {32 floats, 128 rows} at (x, y).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
// A 2D tile of a tensor map into L2 only (no shared memory, no multicast).
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map), "r"(x), "r"(y)
                 : "memory");
}
// Shared-memory matrix descriptor: K-major, SWIZZLE_128B, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);   // start address
    d |= static_cast<uint64_t>(1) << 16;                  // leading byte offset (unused for swizzled K-major)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;          // stride byte offset
    d |= static_cast<uint64_t>(1) << 46;                  // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2) << 61;                  // SWIZZLE_128B
    return d;
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mma_tf32_i(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

// A projection tile of 128 features x BN tokens: the token operand's tile
// (X, X_lo) grows with BN; 128 tokens keep three stages of 64 KB, 256 tokens
// two of 96 KB (the same shared memory, twice the MMA work per byte of W).
template <int BN>
struct TileCfg {
    static_assert(BN == 128 || BN == 256, "tile width");
    static constexpr int kXTile = BN * kBK * 4;
    static constexpr int kStage = 2 * kTileBytes + 2 * kXTile;
    static constexpr int kStages = BN == 128 ? 3 : 2;
    // W and W_lo of K-block kb + kPrefetch go to L2 when K-block kb's loads are issued: the weight tiles come
    // from DRAM, and the stages alone hold too few bytes in flight to cover that latency
    static constexpr int kPrefetch = BN == 128 ? 4 : 2;
    static constexpr size_t kSmem = static_cast<size_t>(kStages) * kStage + 1024 + 256;
    // kind::tf32, fp32 accumulate, K-major A and B, M = 128, N = BN
    static constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
                                       (static_cast<uint32_t>(kBM >> 4) << 24);
};

__device__ __forceinline__ float tf32_lo(float v) { return v - __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }

template <int MODE, int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_wlo,
                   const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_xlo,
                   const float* __restrict__ bias, float* __restrict__ C, float* __restrict__ C_lo, int M, int N,
                   int K, int* err, const GemmBatch bt) {
    extern __shared__ __align__(1024) char smem_raw[];
    constexpr bool kBatched = MODE == kGemmScores || MODE == kGemmPV;
    using Cfg = TileCfg<BN>;
    static_assert(BN == 128 || !kBatched, "the attention modes use 128-token tiles");
    // Scores: a tile whose first key follows its last query is fully masked (causal).
    if (MODE == kGemmScores && static_cast<int>(blockIdx.x) * kBM >= static_cast<int>(blockIdx.y + 1) * BN) return;
    char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kStages * Cfg::kStage);
    uint64_t* empty = full + Cfg::kStages;
    uint64_t* accum = empty + Cfg::kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * BN;
    // split-K: this CTA's K-blocks [kb0, kb1) of blockIdx.z of gridDim.z slices;
    // batched (attention) modes: blockIdx.z is the head and K is whole, or for
    // P.V cut at the tile's last query (P is zero past it).
    const int nkb_all = K / kBK;
    int kb0 = 0, kb1 = nkb_all;
    if (!kBatched) {
        kb0 = static_cast<int>(static_cast<long long>(blockIdx.z) * nkb_all / gridDim.z);
        kb1 = static_cast<int>(static_cast<long long>(blockIdx.z + 1) * nkb_all / gridDim.z);
    } else if (MODE == kGemmPV) {
        kb1 = min(nkb_all, (min(N, n0 + BN) + kBK - 1) / kBK);
    }
    const int nkb = kb1 - kb0;
    const int bz = kBatched ? static_cast<int>(blockIdx.z) : 0;
    const int wx0 = bz * bt.w_x, wy0 = bz * bt.w_y, xx0 = bz * bt.x_x, xy0 = bz * bt.x_y;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % Cfg::kStages;
                const uint32_t ph = static_cast<uint32_t>(kb / Cfg::kStages) & 1u;
                if (!wait_bar(&empty[s], ph ^ 1u, err)) break;
                char* st = smem + s * Cfg::kStage;
                const int kx = (kb0 + kb) * kBK;
                mbar_expect_tx(&full[s], Cfg::kStage);
                tma_load_2d(st, &tm_w, kx + wx0, m0 + wy0, &full[s]);
                tma_load_2d(st + kTileBytes, &tm_wlo, kx + wx0, m0 + wy0, &full[s]);
                tma_load_2d(st + 2 * kTileBytes, &tm_x, kx + xx0, n0 + xy0, &full[s]);
                tma_load_2d(st + 2 * kTileBytes + Cfg::kXTile, &tm_xlo, kx + xx0, n0 + xy0, &full[s]);
                if (!kBatched && kb + Cfg::kPrefetch < nkb) {
                    const int px = (kb0 + kb + Cfg::kPrefetch) * kBK;
                    tma_prefetch_2d(&tm_w, px + wx0, m0 + wy0);
                    tma_prefetch_2d(&tm_wlo, px + wx0, m0 + wy0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % Cfg::kStages;
                const uint32_t ph = static_cast<uint32_t>(kb / Cfg::kStages) & 1u;
                if (!wait_bar(&full[s], ph, err)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t base = smem_u32(smem + s * Cfg::kStage);
                const uint64_t dw = umma_desc(base), dwl = umma_desc(base + kTileBytes);
                const uint64_t dx = umma_desc(base + 2 * kTileBytes);
                const uint64_t dxl = umma_desc(base + 2 * kTileBytes + Cfg::kXTile);
#pragma unroll
                for (int ks = 0; ks < kBK / 8; ++ks) {
                    const uint64_t adv = static_cast<uint64_t>(ks * 32) >> 4;  // 8 tf32 = 32 B per K-step
                    mma_tf32_i(tmem, dw + adv, dx + adv, Cfg::kIdesc, (kb | ks) != 0);
                    mma_tf32_i(tmem, dw + adv, dxl + adv, Cfg::kIdesc, 1u);
                    mma_tf32_i(tmem, dwl + adv, dx + adv, Cfg::kIdesc, 1u);
                }
                mma_commit(&empty[s]);
            }
            mma_commit(accum);
        }
    } else {
        // Epilogue warps 2..5: TMEM lane quarter q = warp % 4 holds features m0 + 32q .. +31.
        const int q = warp & 3;
        const int f = m0 + 32 * q + lane;
        const bool fok = f < M;
        const float bf = (fok && bias && MODE != kGemmPartial && !kBatched) ? bias[f] : 0.0f;
        if (wait_bar(accum, 0, err)) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t r[32];
                const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(c0);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                    "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
                    "[%32];"
                    : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                      "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                      "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                      "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
                      "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int n = n0 + c0 + j;
                    const float v = __uint_as_float(r[j]) + bf;
                    if (MODE == kGemmScores) {
                        if (fok && n < N) C[(static_cast<size_t>(bz) * bt.c_rows + n) * bt.ldc + f] = v;
                    } else if (MODE == kGemmPV) {
                        if (fok && n < N) {
                            const size_t o = static_cast<size_t>(n) * bt.ldc + bz * bt.c_col + f;
                            C[o] = v;
                            C_lo[o] = tf32_lo(v);
                        }
                    } else if (MODE == kGemmPartial) {
                        // raw accumulator of this K slice: C is the workspace [slices][N][M]
                        if (fok && n < N) C[(static_cast<size_t>(blockIdx.z) * N + n) * M + f] = v;
                    } else if (MODE == kGemvSwiGLU) {
                        // features (2i, 2i+1) = (W1 row i, V row i) sit in adjacent lanes
                        const float partner = __shfl_xor_sync(0xffffffffu, v, 1);
                        if ((lane & 1) == 0 && fok && n < N) {
                            const float h = silu(v) * partner;
                            const size_t o = static_cast<size_t>(n) * (M >> 1) + (f >> 1);
                            C[o] = h;
                            C_lo[o] = tf32_lo(h);
                        }
                    } else if (fok && n < N) {
                        float* dst = C + static_cast<size_t>(n) * M + f;
                        if (MODE == kGemvResidual) *dst += v;
                        else *dst = v;
                    }
                }
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN) : "memory");
    }
}

// Sum of the split-K slices in slice order, then the mode's epilogue.  Plain
// and residual rows of a multiple of 4 go 4 at a time (float4), indices in 32
// bits (the launcher checks the sizes).
template <int MODE>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ ws, int slices,
                                                            const float* __restrict__ bias, float* __restrict__ C,
                                                            float* __restrict__ C_lo, int N, int M) {
    const int plane = N * M;
    const int stride = gridDim.x * blockDim.x;
    if (MODE == kGemvSwiGLU) {
        const int half = M / 2, total = N * half;
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
            const int n = i / half, j = i - n * half;
            const int ia = n * M + 2 * j;
            float a = 0.0f, c = 0.0f;
            for (int z = 0; z < slices; ++z) {
                const float2 v = *reinterpret_cast<const float2*>(ws + z * plane + ia);
                a += v.x;
                c += v.y;
            }
            const float h = silu(a + bias[2 * j]) * (c + bias[2 * j + 1]);
            C[i] = h;
            C_lo[i] = tf32_lo(h);
        }
    } else if ((M & 3) == 0) {
        const int total4 = plane >> 2, M4 = M >> 2;
        const float4* w4 = reinterpret_cast<const float4*>(ws);
        float4* c4 = reinterpret_cast<float4*>(C);
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total4; i += stride) {
            float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            for (int z = 0; z < slices; ++z) {
                const float4 v = w4[z * total4 + i];
                a.x += v.x;
                a.y += v.y;
                a.z += v.z;
                a.w += v.w;
            }
            if (bias) {
                const float4 b = reinterpret_cast<const float4*>(bias)[i % M4];
                a.x += b.x;
                a.y += b.y;
                a.z += b.z;
                a.w += b.w;
            }
            if (MODE == kGemvResidual) {
                const float4 y = c4[i];
                a.x += y.x;
                a.y += y.y;
                a.z += y.z;
                a.w += y.w;
            }
            c4[i] = a;
        }
    } else {
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < plane; i += stride) {
            float a = 0.0f;
            for (int z = 0; z < slices; ++z) a += ws[z * plane + i];
            const float v = a + (bias ? bias[i % M] : 0.0f);
            if (MODE == kGemvResidual) C[i] += v;
            else C[i] = v;
        }
    }
}

__global__ void split_lo_kernel(const float* __restrict__ x, float* __restrict__ lo, size_t n) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        lo[i] = tf32_lo(x[i]);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

}  // namespace

// Row-major [rows][cols] fp32 matrix as a 2D TMA map with {32, 128} boxes, 128B swizzle.
cudaError_t make_tile_map(CUtensorMap* map, const float* base, int rows, int cols, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    if (reinterpret_cast<uintptr_t>(base) % 16 || (cols * 4) % 16 || box_rows <= 0 || box_rows > 256)
        return cudaErrorInvalidValue;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 4};
    const cuuint32_t box[2] = {kBK, static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, elem,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t make_stream_map(CUtensorMap* map, const float* base, int rows, int cols) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    if (reinterpret_cast<uintptr_t>(base) % 16 || cols <= 0 || cols % kPersistKAlign) return cudaErrorInvalidValue;
    const int tw = persist_tile_w(cols);
    const int nkt = cols / tw;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(tw), static_cast<cuuint64_t>(nkt),
                                static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(tw) * 4, static_cast<cuuint64_t>(cols) * 4};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(tw),
                               static_cast<cuuint32_t>(persist_box_tiles(cols)),
                               static_cast<cuuint32_t>(kPersistTileRows)};
    const cuuint32_t elem[3] = {1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, elem,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// ---- Causal prefill attention in one kernel (flash-style, tcgen05, 3xTF32) ----
//
// The causal MultiHeadAttention::prefill of src/attn.cu:47-167 for one head,
// 128 queries and a run of key tiles per CTA, with the scores and
// probabilities kept on chip: for each tile of 64 keys, S = (q/8) k^T goes to
// TMEM, the four softmax warps (one thread per query row) read their row of
// S, update the row's running maximum and sum (online softmax; exp as exp2f of
// one FMA), write P = exp(s - max) and its TF32 lo half into TMEM (tcgen05.st)
// as the A operand of the next MMA (tcgen05.mma with A in tensor memory), and
// fold the previous tile's P.V from TMEM into the row's output held in
// registers, rescaled by exp(old max - new max).  The output row is divided by the sum at the end and stored with its
// lo half (the out-projection's operands).
//   warp 0: TMA producer (lane 0: q, then the k tiles through two stages;
//           lane 1: the v^T tiles through two stages);
//   warp 1: one thread issues the MMAs, S one tile ahead of P.V; S and P.V
//           each have two TMEM slots of 64 columns, P and P_lo 64 each;
//   warps 2..5: softmax and output, TMEM lane quarter warp % 4; each thread
//           writes its row of P and signals before it folds the previous
//           tile's P.V, so that the next P.V MMA starts meanwhile.
// A 128-query tile with more than kFaSplit key tiles is cut into balanced runs
// of at most kFaSplit, one CTA each (so that the longest CTA is short and the
// grid covers the SMs); each run stores its rows' (output, max, sum) to a
// workspace and the warp that takes the last ticket of its 32 rows merges
// them (the same online-softmax rule across runs).
// Products use the 3xTF32 split of the projections (hi.hi + hi.lo + lo.hi).
// Keys past a row's query get probability 0; key tiles past the CTA's last
// query are not visited.  Operands come from attn_prep_kernel: q/8 [T][heads
// * 64], k [heads * T][64], v^T [heads * 64][T], each with its lo half.
constexpr int kFaKeys = 64;                        // keys per tile: the scores' MMA N
constexpr int kFaQTile = kBM * kBK * 4;            // 16 KB: 128 rows x 32 floats
constexpr int kFaKTile = kFaKeys * kBK * 4;        // 8 KB: 64 rows x 32 floats
constexpr int kFaQBytes = 4 * kFaQTile;            // q and q_lo, two 32-float K-blocks each
constexpr int kFaKStage = 4 * kFaKTile;            // k and k_lo of one tile
constexpr int kFaVBytes = 4 * kFaKTile;            // v^T and its lo half of one tile
constexpr int kFaKStages = 2;
constexpr int kFaVStages = 2;
constexpr int kFaOffK = kFaQBytes;
constexpr int kFaOffV = kFaOffK + kFaKStages * kFaKStage;
constexpr int kFaOffBar = kFaOffV + kFaVStages * kFaVBytes;
constexpr size_t kFaSmem = static_cast<size_t>(kFaOffBar) + 256 + 1024;
constexpr int kFaThreads = 6 * 32;                 // producer, MMA issuer, four softmax warps
constexpr int kFaSplit = 4;                        // key tiles per CTA at most (longer rows split over CTAs)
constexpr int kFaPart = kHeadDim + 4;              // a run's partial row in the workspace: output, max, sum
constexpr uint32_t kFaTmemCols = 512;  // S slots at 0 and 64, P.V slots at 128 and 192, P at 256, P_lo at 320
constexpr uint32_t kFaTmemP = 256;
constexpr uint32_t kFaTmemPlo = 320;
// kind::tf32, fp32 accumulate, K-major A and B, M = 128, N = 64
constexpr uint32_t kIdescN64 = (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(kFaKeys >> 3) << 17) |
                               (static_cast<uint32_t>(kBM >> 4) << 24);
static_assert(kFaSmem <= 232448, "fused attention shared memory");
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void mma_tf32_n64(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(kIdescN64), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// 32 consecutive TMEM columns of the warp's lane quarter (one row per thread).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
        "[%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32 consecutive TMEM columns of the warp's lane quarter (one row per thread), from registers.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
        "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
        "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])),
        "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
        "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
        "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
        "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])),
        "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// D (=|+=) A . B^T with A in TMEM (M = 128 lanes, one tf32 per column) and B in shared memory.
__device__ __forceinline__ void mma_tf32_ts_n64(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(b), "r"(kIdescN64), "r"(accumulate)
        : "memory");
}

// 3 x 4 K-steps x 2 K-blocks of 32 floats: D (=|+=) A . B^T over 64 columns of K.
__device__ __forceinline__ void mma_3xtf32_k64(uint32_t d, uint32_t a, uint32_t a_lo, uint32_t b, uint32_t b_lo,
                                               int a_tile, int b_tile) {
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) {
        const uint64_t da = umma_desc(a + kb * a_tile), dal = umma_desc(a_lo + kb * a_tile);
        const uint64_t db = umma_desc(b + kb * b_tile), dbl = umma_desc(b_lo + kb * b_tile);
#pragma unroll
        for (int ks = 0; ks < kBK / 8; ++ks) {
            const uint64_t adv = static_cast<uint64_t>(ks * 32) >> 4;  // 8 tf32 = 32 B per K-step
            mma_tf32_n64(d, da + adv, db + adv, (kb | ks) != 0);
            mma_tf32_n64(d, da + adv, dbl + adv, 1u);
            mma_tf32_n64(d, dal + adv, db + adv, 1u);
        }
    }
}

// P.V over one 64-key tile with P (and P_lo) in TMEM columns a, a_lo (key c at column c) and v^T in shared
// memory: 3 x 4 K-steps x 2 K-blocks of 32 keys.
__device__ __forceinline__ void mma_3xtf32_pv_tmem(uint32_t d, uint32_t a, uint32_t a_lo, uint32_t b, uint32_t b_lo,
                                                   int b_tile) {
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) {
        const uint64_t db = umma_desc(b + kb * b_tile), dbl = umma_desc(b_lo + kb * b_tile);
#pragma unroll
        for (int ks = 0; ks < kBK / 8; ++ks) {
            const uint32_t ac = static_cast<uint32_t>(kb * kBK + ks * 8);  // 8 tf32 keys = 8 columns per K-step
            const uint64_t adv = static_cast<uint64_t>(ks * 32) >> 4;      // 8 tf32 = 32 B per K-step
            mma_tf32_ts_n64(d, a + ac, db + adv, (kb | ks) != 0);
            mma_tf32_ts_n64(d, a + ac, dbl + adv, 1u);
            mma_tf32_ts_n64(d, a_lo + ac, db + adv, 1u);
        }
    }
}

__global__ void __launch_bounds__(kFaThreads, 1)
    attn_flash_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_qlo,
                         const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_klo,
                         const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_vlo,
                         float* __restrict__ out, float* __restrict__ out_lo, int n, int max_ctx, int ldo,
                         float* __restrict__ ws, int* __restrict__ tickets, int ws_splits, int* err) {
    extern __shared__ __align__(1024) char smem_raw[];
    char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kFaOffBar);
    uint64_t* q_full = bars;        // q landed
    uint64_t* k_full = bars + 1;    // [kFaKStages] k tile landed
    uint64_t* k_empty = bars + 3;   // [kFaKStages] its scores MMA done
    uint64_t* v_full = bars + 5;    // [kFaVStages] v^T tile landed
    uint64_t* v_empty = bars + 7;   // [kFaVStages] its P.V MMA done
    uint64_t* s_full = bars + 9;    // [2] scores in TMEM
    uint64_t* p_full = bars + 11;   // P written to TMEM (128 arrivals)
    uint64_t* pv_full = bars + 12;  // [2] P.V in TMEM (and the P columns free again)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Work unit blockIdx.x: the query tiles from the last (longest) down, each tile's key tiles cut into
    // `splits` balanced runs of at most kFaSplit; this unit takes run sp, key tiles [kt0, kt0 + nkt).
    const int nqt = (n + kBM - 1) / kBM;
    int qt = nqt - 1, splits = 1, sp = static_cast<int>(blockIdx.x), kt_all = 1;
    for (; qt > 0; --qt) {
        kt_all = (min(n, (qt + 1) * kBM) + kFaKeys - 1) / kFaKeys;
        splits = (kt_all + kFaSplit - 1) / kFaSplit;
        if (sp < splits) break;
        sp -= splits;
    }
    if (qt == 0) {
        kt_all = (min(n, kBM) + kFaKeys - 1) / kFaKeys;
        splits = (kt_all + kFaSplit - 1) / kFaSplit;
    }
    const int q0 = qt * kBM;
    const int h = blockIdx.y;
    const int per = (kt_all + splits - 1) / splits;
    const int kt0 = sp * per;
    const int nkt = min(kt_all, kt0 + per) - kt0;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&pv_full[i], 1);
        }
        mbar_init(p_full, 4 * 32);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kFaTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            mbar_expect_tx(q_full, kFaQBytes);
            for (int kb = 0; kb < 2; ++kb) {
                tma_load_2d(smem + kb * kFaQTile, &tm_q, h * kHeadDim + kb * kBK, q0, q_full);
                tma_load_2d(smem + 2 * kFaQTile + kb * kFaQTile, &tm_qlo, h * kHeadDim + kb * kBK, q0, q_full);
            }
            for (int j = 0; j < nkt; ++j) {
                const int st = j % kFaKStages;
                if (!wait_bar(&k_empty[st], ((j / kFaKStages) & 1) ^ 1u, err)) break;
                char* kst = smem + kFaOffK + st * kFaKStage;
                mbar_expect_tx(&k_full[st], kFaKStage);
                for (int kb = 0; kb < 2; ++kb) {
                    const int y = h * max_ctx + (kt0 + j) * kFaKeys;
                    tma_load_2d(kst + kb * kFaKTile, &tm_k, kb * kBK, y, &k_full[st]);
                    tma_load_2d(kst + 2 * kFaKTile + kb * kFaKTile, &tm_klo, kb * kBK, y, &k_full[st]);
                }
            }
        } else if (lane == 1) {
            for (int j = 0; j < nkt; ++j) {
                const int st = j % kFaVStages;
                if (!wait_bar(&v_empty[st], ((j / kFaVStages) & 1) ^ 1u, err)) break;
                char* vs = smem + kFaOffV + st * kFaVBytes;
                mbar_expect_tx(&v_full[st], kFaVBytes);
                for (int kb = 0; kb < 2; ++kb) {
                    const int x = (kt0 + j) * kFaKeys + kb * kBK;
                    tma_load_2d(vs + kb * kFaKTile, &tm_v, x, h * kHeadDim, &v_full[st]);
                    tma_load_2d(vs + 2 * kFaKTile + kb * kFaKTile, &tm_vlo, x, h * kHeadDim, &v_full[st]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t qa = smem_u32(smem);
            bool ok = wait_bar(q_full, 0, err);
            // scores of key tile j into S slot j % 2 (its previous use, tile j - 2, was read before P_{j-2} was
            // written, which the P.V MMA of tile j - 2 waited for)
            auto scores = [&](int j) -> bool {
                const int st = j & 1;
                const int ks = j % kFaKStages;
                if (!wait_bar(&k_full[ks], (j / kFaKStages) & 1, err)) return false;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t ka = smem_u32(smem + kFaOffK + ks * kFaKStage);
                mma_3xtf32_k64(tmem + st * kFaKeys, qa, qa + 2 * kFaQTile, ka, ka + 2 * kFaKTile, kFaQTile, kFaKTile);
                mma_commit(&k_empty[ks]);
                mma_commit(&s_full[st]);
                return true;
            };
            if (ok) ok = scores(0);
            for (int j = 0; ok && j < nkt; ++j) {
                if (j + 1 < nkt && !scores(j + 1)) break;
                const int vs = j % kFaVStages;
                if (!wait_bar(p_full, j & 1, err) || !wait_bar(&v_full[vs], (j / kFaVStages) & 1, err)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t va = smem_u32(smem + kFaOffV + vs * kFaVBytes);
                mma_3xtf32_pv_tmem(tmem + 2 * kFaKeys + (j & 1) * kFaKeys, tmem + kFaTmemP, tmem + kFaTmemPlo, va,
                                   va + 2 * kFaKTile, kFaKTile);
                mma_commit(&v_empty[vs]);
                mma_commit(&pv_full[j & 1]);
            }
        }
    } else {
        const int qq = warp & 3;  // TMEM lane quarter of this warp: rows 32 qq .. 32 qq + 31
        const int r = 32 * qq + lane;
        const int q = q0 + r;
        const uint32_t trow = tmem + (static_cast<uint32_t>(32 * qq) << 16);
        float o[kHeadDim];
#pragma unroll
        for (int d = 0; d < kHeadDim; ++d) o[d] = 0.0f;
        float m = -INFINITY, l = 0.0f, alpha_prev = 0.0f;
        bool ok = true;
        for (int j = 0; j < nkt; ++j) {
            const int st = j & 1;
            // waits are warp-uniform: tcgen05.ld needs the whole warp
            if (!__all_sync(0xffffffffu, wait_bar(&s_full[st], (j >> 1) & 1, err))) {
                ok = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            float sv[kFaKeys];
            tmem_ld32(trow + st * kFaKeys, sv);
            tmem_ld32(trow + st * kFaKeys + 32, sv + 32);
            tmem_wait_ld();
            const int k0 = (kt0 + j) * kFaKeys;
            if (k0 + kFaKeys - 1 > q0) {  // a tile on the diagonal: keys past the row's query masked
#pragma unroll
                for (int c = 0; c < kFaKeys; ++c)
                    if (k0 + c > q) sv[c] = -INFINITY;
            }
            // the row maximum and sum as eight independent chains
            float mx[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) mx[i] = sv[i];
#pragma unroll
            for (int c = 8; c < kFaKeys; ++c) mx[c & 7] = fmaxf(mx[c & 7], sv[c]);
            const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                   fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
            const float mn = fmaxf(m, mt);
            // exp(x) = 2^(x log2 e): one FMA and one exp2f per key; a masked key (-inf) gives 0
            const float mb = mn * kLog2e;
            const float alpha = exp2f(fmaf(m, kLog2e, -mb));  // 0 at the first tile (m = -inf; key 0 is in every row)
            float ls[8];
#pragma unroll
            for (int c = 0; c < kFaKeys; ++c) {
                const float pc = exp2f(fmaf(sv[c], kLog2e, -mb));
                sv[c] = pc;
                if (c < 8) ls[c] = pc;
                else ls[c & 7] += pc;
            }
            l = fmaf(l, alpha, ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7])));
            m = mn;
            const int pj = j - 1;
            if (j > 0) {  // the previous tile's P.V done: the P columns are free, its result in TMEM
                if (!__all_sync(0xffffffffu, wait_bar(&pv_full[pj & 1], (pj >> 1) & 1, err))) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            }
            // P and its lo half into TMEM, the A operand of the P.V MMA: this thread's row, key c at column c
            tmem_st32(trow + kFaTmemP, sv);
            tmem_st32(trow + kFaTmemP + 32, sv + 32);
#pragma unroll
            for (int c = 0; c < kFaKeys; ++c) sv[c] = tf32_lo(sv[c]);
            tmem_st32(trow + kFaTmemPlo, sv);
            tmem_st32(trow + kFaTmemPlo + 32, sv + 32);
            tmem_wait_st();
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            mbar_arrive(p_full);
            if (j > 0) {  // fold the previous tile's P.V while this tile's runs (another TMEM slot)
                float pv[kHeadDim];
                tmem_ld32(trow + 2 * kFaKeys + (pj & 1) * kFaKeys, pv);
                tmem_ld32(trow + 2 * kFaKeys + (pj & 1) * kFaKeys + 32, pv + 32);
                tmem_wait_ld();
#pragma unroll
                for (int d = 0; d < kHeadDim; ++d) o[d] = fmaf(o[d], alpha_prev, pv[d]);
            }
            alpha_prev = alpha;
        }
        if (ok && nkt > 0) {
            const int pj = nkt - 1;
            if (__all_sync(0xffffffffu, wait_bar(&pv_full[pj & 1], (pj >> 1) & 1, err))) {
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                float pv[kHeadDim];
                tmem_ld32(trow + 2 * kFaKeys + (pj & 1) * kFaKeys, pv);
                tmem_ld32(trow + 2 * kFaKeys + (pj & 1) * kFaKeys + 32, pv + 32);
                tmem_wait_ld();
#pragma unroll
                for (int d = 0; d < kHeadDim; ++d) o[d] = fmaf(o[d], alpha_prev, pv[d]);
                bool write = true;
                if (splits > 1) {
                    // this run's (output, max, sum) of the row to the workspace; the warp that takes the last
                    // ticket of its 32 rows merges every run's (the tickets return to 0 for the next launch)
                    const size_t unit = (static_cast<size_t>(h) * nqt + qt) * ws_splits;
                    float4* mine = reinterpret_cast<float4*>(ws + ((unit + sp) * kBM + r) * kFaPart);
#pragma unroll
                    for (int d = 0; d < kHeadDim; d += 4) mine[d >> 2] = make_float4(o[d], o[d + 1], o[d + 2], o[d + 3]);
                    mine[kHeadDim / 4] = make_float4(m, l, 0.0f, 0.0f);
                    __threadfence();
                    __syncwarp();
                    int* tk = tickets + (static_cast<size_t>(h) * nqt + qt) * 4 + qq;
                    int last = 0;
                    if (lane == 0) last = atomicAdd(tk, 1) == splits - 1;
                    write = __shfl_sync(0xffffffffu, last, 0) != 0;
                    if (write) {
                        __threadfence();
                        if (lane == 0) *tk = 0;
                        float mm = m;
                        for (int s2 = 0; s2 < splits; ++s2)
                            if (s2 != sp) mm = fmaxf(mm, __ldcg(ws + ((unit + s2) * kBM + r) * kFaPart + kHeadDim));
                        const float wm = exp2f((m - mm) * kLog2e);
                        l *= wm;
#pragma unroll
                        for (int d = 0; d < kHeadDim; ++d) o[d] *= wm;
                        for (int s2 = 0; s2 < splits; ++s2) {
                            if (s2 == sp) continue;
                            const float4* th = reinterpret_cast<const float4*>(ws + ((unit + s2) * kBM + r) * kFaPart);
                            const float4 ml = __ldcg(th + kHeadDim / 4);
                            const float w = exp2f((ml.x - mm) * kLog2e);
                            l = fmaf(ml.y, w, l);
#pragma unroll
                            for (int d = 0; d < kHeadDim; d += 4) {
                                const float4 v = __ldcg(th + (d >> 2));
                                o[d] = fmaf(v.x, w, o[d]);
                                o[d + 1] = fmaf(v.y, w, o[d + 1]);
                                o[d + 2] = fmaf(v.z, w, o[d + 2]);
                                o[d + 3] = fmaf(v.w, w, o[d + 3]);
                            }
                        }
                    }
                }
                if (write && q < n) {
                    const float inv = 1.0f / l;
                    float4* dst = reinterpret_cast<float4*>(out + static_cast<size_t>(q) * ldo + h * kHeadDim);
                    float4* dlo = reinterpret_cast<float4*>(out_lo + static_cast<size_t>(q) * ldo + h * kHeadDim);
#pragma unroll
                    for (int d = 0; d < kHeadDim; d += 4) {
                        const float4 v = make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
                        dst[d >> 2] = v;
                        dlo[d >> 2] = make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
                    }
                }
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kFaTmemCols) : "memory");
    }
}

template <int MODE, int BN = kBN>
cudaError_t launch_tc(dim3 grid, const TcOperands& o, const float* bias, float* C, float* C_lo, int m, int n, int k,
                      int* err, cudaStream_t s, const GemmBatch& bt = GemmBatch{}) {
    constexpr size_t smem = TileCfg<BN>::kSmem;
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<MODE, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    count_launch();
    const CUtensorMap& x = BN == kBN ? o.x : o.x_wide;
    const CUtensorMap& x_lo = BN == kBN ? o.x_lo : o.x_lo_wide;
    gemm_tc_kernel<MODE, BN><<<grid, kGemmThreads, smem, s>>>(o.w, o.w_lo, x, x_lo, bias, C, C_lo, m, n, k, err, bt);
    return cudaGetLastError();
}

cudaError_t launch_gemm_tc(int mode, const TcOperands& o, const float* bias, float* C, float* C_lo, int n, int m,
                           int k, int* err, cudaStream_t s, float* ws, size_t ws_floats, int num_sms) {
    if (n <= 0 || m <= 0 || k <= 0 || k % kBK || (mode == kGemvSwiGLU && (m % 2 || !C_lo))) return cudaErrorInvalidValue;
    const int tiles = ((m + kBM - 1) / kBM) * ((n + kBN - 1) / kBN);
    const int nkb = k / kBK;
    // K slices so that the grid covers the SMs, each slice keeping >= 4 K-blocks
    int slices = 1;
    if (ws && tiles < num_sms) {
        slices = std::min(num_sms / tiles, std::max(1, nkb / 4));
        const size_t plane = static_cast<size_t>(n) * m;
        while (slices > 1 && static_cast<size_t>(slices) * plane > ws_floats) --slices;
    }
    dim3 grid((m + kBM - 1) / kBM, (n + kBN - 1) / kBN, slices);
    cudaError_t e;
    if (slices > 1 && static_cast<size_t>(slices) * n * m >= (size_t{1} << 31)) slices = 1;  // 32-bit reduce indices
    grid.z = slices;
    if (slices > 1) {
        e = launch_tc<kGemmPartial>(grid, o, nullptr, ws, nullptr, m, n, k, err, s);
        if (e != cudaSuccess) return e;
        const size_t total = static_cast<size_t>(n) * (mode == kGemvSwiGLU ? m / 2 : m);
        const unsigned blocks = static_cast<unsigned>(std::min<size_t>((total + 255) / 256, 148 * 8));
        count_launch();
        switch (mode) {
            case kGemvPlain:
                splitk_reduce_kernel<kGemvPlain><<<blocks, 256, 0, s>>>(ws, slices, bias, C, C_lo, n, m);
                break;
            case kGemvSwiGLU:
                splitk_reduce_kernel<kGemvSwiGLU><<<blocks, 256, 0, s>>>(ws, slices, bias, C, C_lo, n, m);
                break;
            case kGemvResidual:
                splitk_reduce_kernel<kGemvResidual><<<blocks, 256, 0, s>>>(ws, slices, bias, C, C_lo, n, m);
                break;
            default:
                return cudaErrorInvalidValue;
        }
        return cudaGetLastError();
    }
    // 256-token tiles where the operands have them and they take at most half the waves of 128-token ones
    // (a 512-id W1/V: 128 tiles in one wave against 256 in two)
    const int mt = (m + kBM - 1) / kBM;
    const int w128 = (tiles + num_sms - 1) / num_sms;
    const int w256 = (mt * ((n + 255) / 256) + num_sms - 1) / num_sms;
    if (o.wide && n > kBN && 2 * w256 <= w128) {
        const dim3 g2(mt, (n + 255) / 256, 1);
        switch (mode) {
            case kGemvPlain:
                return launch_tc<kGemvPlain, 256>(g2, o, bias, C, C_lo, m, n, k, err, s);
            case kGemvSwiGLU:
                return launch_tc<kGemvSwiGLU, 256>(g2, o, bias, C, C_lo, m, n, k, err, s);
            case kGemvResidual:
                return launch_tc<kGemvResidual, 256>(g2, o, bias, C, C_lo, m, n, k, err, s);
            default:
                return cudaErrorInvalidValue;
        }
    }
    switch (mode) {
        case kGemvPlain:
            return launch_tc<kGemvPlain>(grid, o, bias, C, C_lo, m, n, k, err, s);
        case kGemvSwiGLU:
            return launch_tc<kGemvSwiGLU>(grid, o, bias, C, C_lo, m, n, k, err, s);
        case kGemvResidual:
            return launch_tc<kGemvResidual>(grid, o, bias, C, C_lo, m, n, k, err, s);
        default:
            return cudaErrorInvalidValue;
    }
}

cudaError_t launch_attn_scores_tc(const TcOperands& o, float* S, int n, int heads, int max_ctx, int* err,
                                  cudaStream_t s) {
    if (n <= 0 || n > max_ctx || heads <= 0) return cudaErrorInvalidValue;
    GemmBatch bt{};
    bt.w_y = max_ctx;
    bt.x_x = kHeadDim;
    bt.c_rows = max_ctx;
    bt.ldc = max_ctx;
    const unsigned t = static_cast<unsigned>((n + kBM - 1) / kBM);
    return launch_tc<kGemmScores>(dim3(t, t, heads), o, nullptr, S, nullptr, n, n, kHeadDim, err, s, bt);
}

cudaError_t launch_attn_pv_tc(const TcOperands& o, float* out, float* out_lo, int n, int heads, int max_ctx, int* err,
                              cudaStream_t s) {
    if (n <= 0 || n > max_ctx || heads <= 0 || max_ctx % kBK) return cudaErrorInvalidValue;
    GemmBatch bt{};
    bt.w_y = kHeadDim;
    bt.x_y = max_ctx;
    bt.ldc = heads * kHeadDim;
    bt.c_col = kHeadDim;
    const int k = ((n + kBK - 1) / kBK) * kBK;
    const unsigned t = static_cast<unsigned>((n + kBN - 1) / kBN);
    return launch_tc<kGemmPV>(dim3(1, t, heads), o, nullptr, out, out_lo, kHeadDim, n, k, err, s, bt);
}

int attn_flash_ws_splits(int max_ctx) {
    return ((max_ctx + kFaKeys - 1) / kFaKeys + kFaSplit - 1) / kFaSplit;
}

size_t attn_flash_ws_floats(int heads, int max_ctx) {
    const int splits = attn_flash_ws_splits(max_ctx);
    if (splits <= 1) return 0;
    return static_cast<size_t>(heads) * ((max_ctx + kBM - 1) / kBM) * splits * kBM * kFaPart;
}

cudaError_t launch_attn_flash_tc(const FlashOperands& o, float* out, float* out_lo, int n, int heads, int max_ctx,
                                 float* ws, size_t ws_floats, int* tickets, int* err, cudaStream_t s) {
    if (n <= 0 || n > max_ctx || heads <= 0 || max_ctx % kBK || ws_floats < attn_flash_ws_floats(heads, max_ctx))
        return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(attn_flash_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kFaSmem));
    if (e != cudaSuccess) return e;
    // one CTA per run of at most kFaSplit key tiles of each 128-query tile
    int units = 0;
    for (int qt = 0; qt * kBM < n; ++qt) {
        const int kt = (std::min(n, (qt + 1) * kBM) + kFaKeys - 1) / kFaKeys;
        units += (kt + kFaSplit - 1) / kFaSplit;
    }
    count_launch();
    const dim3 grid(static_cast<unsigned>(units), static_cast<unsigned>(heads));
    attn_flash_tc_kernel<<<grid, kFaThreads, kFaSmem, s>>>(o.q, o.q_lo, o.k, o.k_lo, o.v, o.v_lo, out, out_lo, n,
                                                             max_ctx, heads * kHeadDim, ws, tickets,
                                                             attn_flash_ws_splits(max_ctx), err);
    return cudaGetLastError();
}

cudaError_t launch_split_lo(const float* x, float* lo, size_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const size_t blocks = std::min<size_t>((n + 255) / 256, 148 * 16);
    count_launch();
    split_lo_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(x, lo, n);
    return cudaGetLastError();
}

}  // namespace xl
