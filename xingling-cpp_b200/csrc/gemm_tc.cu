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
// Tile: 128 output features (MMA M) x 128 tokens (MMA N), K-blocks of 32
// floats (128 B, the SWIZZLE_128B span).  Warp 0 issues TMA loads of the four
// operand tiles of a K-block into a 3-stage ring; warp 1 (one thread) issues
// 4 K-steps x 3 tcgen05.mma per K-block into a 128 x 128 fp32 accumulator in
// TMEM and frees each stage with tcgen05.commit; warps 2..5 read the
// accumulator with tcgen05.ld and apply the epilogue (bias; residual add;
// SwiGLU over interleaved (W1 j, V j) feature pairs, which also writes the
// lo half for the next GEMM).
#include <cuda.h>
#include <math.h>

#include <algorithm>

#include "xl_device.cuh"
#include "xl_kernels.h"

namespace xl {

namespace {

constexpr int kBM = 128;               // output features per tile (MMA M)
constexpr int kBN = 128;               // tokens per tile (MMA N)
constexpr int kBK = 32;                // floats per K-block (128 B rows)
constexpr int kStages = 3;
constexpr int kTileBytes = kBM * kBK * 4;  // 16 KB (kBN == kBM)
constexpr int kStageBytes = 4 * kTileBytes;  // W, W_lo, X, X_lo
constexpr int kGemmThreads = 192;
constexpr size_t kGemmSmem = static_cast<size_t>(kStages) * kStageBytes + 1024 + 256;
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
// Instruction descriptor: kind::tf32, fp32 accumulate, K-major A and B, M = 128, N = 128.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(kBN >> 3) << 17) |
                            (static_cast<uint32_t>(kBM >> 4) << 24);

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ float tf32_lo(float v) { return v - __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }

template <int MODE>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_wlo,
                   const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_xlo,
                   const float* __restrict__ bias, float* __restrict__ C, float* __restrict__ C_lo, int M, int N,
                   int K, int* err, const GemmBatch bt) {
    extern __shared__ __align__(1024) char smem_raw[];
    constexpr bool kBatched = MODE == kGemmScores || MODE == kGemmPV;
    // Scores: a tile whose first key follows its last query is fully masked (causal).
    if (MODE == kGemmScores && static_cast<int>(blockIdx.x) * kBM >= static_cast<int>(blockIdx.y + 1) * kBN) return;
    char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    uint64_t* accum = empty + kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * kBN;
    // split-K: this CTA's K-blocks [kb0, kb1) of blockIdx.z of gridDim.z slices;
    // batched (attention) modes: blockIdx.z is the head and K is whole, or for
    // P.V cut at the tile's last query (P is zero past it).
    const int nkb_all = K / kBK;
    int kb0 = 0, kb1 = nkb_all;
    if (!kBatched) {
        kb0 = static_cast<int>(static_cast<long long>(blockIdx.z) * nkb_all / gridDim.z);
        kb1 = static_cast<int>(static_cast<long long>(blockIdx.z + 1) * nkb_all / gridDim.z);
    } else if (MODE == kGemmPV) {
        kb1 = min(nkb_all, (min(N, n0 + kBN) + kBK - 1) / kBK);
    }
    const int nkb = kb1 - kb0;
    const int bz = kBatched ? static_cast<int>(blockIdx.z) : 0;
    const int wx0 = bz * bt.w_x, wy0 = bz * bt.w_y, xx0 = bz * bt.x_x, xy0 = bz * bt.x_y;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kBN)
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
                const int s = kb % kStages;
                const uint32_t ph = static_cast<uint32_t>(kb / kStages) & 1u;
                if (!wait_bar(&empty[s], ph ^ 1u, err)) break;
                char* st = smem + s * kStageBytes;
                const int kx = (kb0 + kb) * kBK;
                mbar_expect_tx(&full[s], kStageBytes);
                tma_load_2d(st, &tm_w, kx + wx0, m0 + wy0, &full[s]);
                tma_load_2d(st + kTileBytes, &tm_wlo, kx + wx0, m0 + wy0, &full[s]);
                tma_load_2d(st + 2 * kTileBytes, &tm_x, kx + xx0, n0 + xy0, &full[s]);
                tma_load_2d(st + 3 * kTileBytes, &tm_xlo, kx + xx0, n0 + xy0, &full[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % kStages;
                const uint32_t ph = static_cast<uint32_t>(kb / kStages) & 1u;
                if (!wait_bar(&full[s], ph, err)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t base = smem_u32(smem + s * kStageBytes);
                const uint64_t dw = umma_desc(base), dwl = umma_desc(base + kTileBytes);
                const uint64_t dx = umma_desc(base + 2 * kTileBytes), dxl = umma_desc(base + 3 * kTileBytes);
#pragma unroll
                for (int ks = 0; ks < kBK / 8; ++ks) {
                    const uint64_t adv = static_cast<uint64_t>(ks * 32) >> 4;  // 8 tf32 = 32 B per K-step
                    mma_tf32(tmem, dw + adv, dx + adv, (kb | ks) != 0);
                    mma_tf32(tmem, dw + adv, dxl + adv, 1u);
                    mma_tf32(tmem, dwl + adv, dx + adv, 1u);
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
            for (int c0 = 0; c0 < kBN; c0 += 32) {
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kBN) : "memory");
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

size_t gemm_tc_smem_bytes() { return kGemmSmem; }

// Row-major [rows][cols] fp32 matrix as a 2D TMA map with {32, 128} boxes, 128B swizzle.
cudaError_t make_tile_map(CUtensorMap* map, const float* base, int rows, int cols) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    if (reinterpret_cast<uintptr_t>(base) % 16 || (cols * 4) % 16) return cudaErrorInvalidValue;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 4};
    const cuuint32_t box[2] = {kBK, kBM};
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

template <int MODE>
cudaError_t launch_tc(dim3 grid, const TcOperands& o, const float* bias, float* C, float* C_lo, int m, int n, int k,
                      int* err, cudaStream_t s, const GemmBatch& bt = GemmBatch{}) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kGemmSmem));
    if (e != cudaSuccess) return e;
    count_launch();
    gemm_tc_kernel<MODE><<<grid, kGemmThreads, kGemmSmem, s>>>(o.w, o.w_lo, o.x, o.x_lo, bias, C, C_lo, m, n, k, err,
                                                                bt);
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

cudaError_t launch_split_lo(const float* x, float* lo, size_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const size_t blocks = std::min<size_t>((n + 255) / 256, 148 * 16);
    count_launch();
    split_lo_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(x, lo, n);
    return cudaGetLastError();
}

}  // namespace xl
