// Prefill kernels for sm_100a (fp32).
//
//  embed_gather_kernel     Embedding::forward (src/embedding.cu:50-61, 75-110)
//  rmsnorm_rows_kernel     RMSNorm::forward on [N][K] rows (src/rmsnorm.cu:46-80)
//  sgemm_tn_kernel         Linear::forward (src/linear.cu:106-168, 197-253), with
//                          the SwiGLU (src/ffn.cu:70-76) and residual-add
//                          (src/transformer.cu:54-59) epilogues fused
//  rope_kv_prefill_kernel  RoPE::forward on q and k (src/rope.cu:70-106) fused
//                          with the KV-cache fill (src/attn.cu:160-166)
//  attn_prefill_kernel     causal MultiHeadAttention::prefill (src/attn.cu:47-167,
//                          319-365), flash-style online softmax over 64x64 tiles
#include <math.h>

#include "xl_device.cuh"
#include "xl_kernels.h"

namespace xl {

namespace {

__global__ void __launch_bounds__(256) embed_gather_kernel(const float* __restrict__ table, const int* __restrict__ ids,
                                                           float* __restrict__ out, int k) {
    const int row = blockIdx.x;
    const float4* src = reinterpret_cast<const float4*>(table + static_cast<size_t>(ids[row]) * k);
    float4* dst = reinterpret_cast<float4*>(out + static_cast<size_t>(row) * k);
    for (int i = threadIdx.x; i < (k >> 2); i += blockDim.x) dst[i] = src[i];
}

__device__ __forceinline__ float lo19(float v) { return v - __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }

__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                                           float* __restrict__ out, float* __restrict__ out_lo, int k,
                                                           double eps) {
    __shared__ float red[8];
    const int row = blockIdx.x;
    const float4* x4 = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * k);
    float4* o4 = reinterpret_cast<float4*>(out + static_cast<size_t>(row) * k);
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
    float ss = 0.0f;
    for (int i = threadIdx.x; i < (k >> 2); i += 256) ss = dot4(x4[i], x4[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += red[w];
    const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(tot / static_cast<float>(k)) + eps));
    for (int i = threadIdx.x; i < (k >> 2); i += 256) {
        float4 v = x4[i];
        const float4 g = g4[i];
        v.x = v.x * inv * g.x;
        v.y = v.y * inv * g.y;
        v.z = v.z * inv * g.z;
        v.w = v.w * inv * g.w;
        o4[i] = v;
        if (out_lo)
            reinterpret_cast<float4*>(out_lo + static_cast<size_t>(row) * k)[i] =
                make_float4(lo19(v.x), lo19(v.y), lo19(v.z), lo19(v.w));
    }
}

// C[N][M] = A[N][K] . B[M][K]^T (+ bias, epilogue).  128 x 128 tile, BK 8,
// 256 threads with an 8 x 8 register tile, double-buffered shared memory.
constexpr int kBM = 128, kBN = 128, kBK = 8;

template <int MODE>
__global__ void __launch_bounds__(256) sgemm_tn_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                       const float* __restrict__ bias, float* __restrict__ C, int N,
                                                       int M, int K) {
    __shared__ __align__(16) float As[2][kBK][kBM + 4];
    __shared__ __align__(16) float Bs[2][kBK][kBN + 4];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int n0 = blockIdx.y * kBM, m0 = blockIdx.x * kBN;
    const int lrow = tid >> 1, lk = (tid & 1) * 4;
    const float* Ap = A + static_cast<size_t>(n0 + lrow) * K + lk;
    const float* Bp = B + static_cast<size_t>(m0 + lrow) * K + lk;
    const bool a_ok = (n0 + lrow) < N;
    const bool b_ok = (m0 + lrow) < M;

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

    float4 ra = a_ok ? *reinterpret_cast<const float4*>(Ap) : make_float4(0, 0, 0, 0);
    float4 rb = b_ok ? *reinterpret_cast<const float4*>(Bp) : make_float4(0, 0, 0, 0);
    As[0][lk + 0][lrow] = ra.x;
    As[0][lk + 1][lrow] = ra.y;
    As[0][lk + 2][lrow] = ra.z;
    As[0][lk + 3][lrow] = ra.w;
    Bs[0][lk + 0][lrow] = rb.x;
    Bs[0][lk + 1][lrow] = rb.y;
    Bs[0][lk + 2][lrow] = rb.z;
    Bs[0][lk + 3][lrow] = rb.w;
    __syncthreads();

    const int ktiles = K / kBK;
    for (int kt = 0; kt < ktiles; ++kt) {
        const int cur = kt & 1;
        if (kt + 1 < ktiles) {
            ra = a_ok ? *reinterpret_cast<const float4*>(Ap + (kt + 1) * kBK) : make_float4(0, 0, 0, 0);
            rb = b_ok ? *reinterpret_cast<const float4*>(Bp + (kt + 1) * kBK) : make_float4(0, 0, 0, 0);
        }
#pragma unroll
        for (int k = 0; k < kBK; ++k) {
            const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][k][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][k][ty * 4 + 64]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][k][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[cur][k][tx * 4 + 64]);
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        if (kt + 1 < ktiles) {
            const int nxt = cur ^ 1;
            As[nxt][lk + 0][lrow] = ra.x;
            As[nxt][lk + 1][lrow] = ra.y;
            As[nxt][lk + 2][lrow] = ra.z;
            As[nxt][lk + 3][lrow] = ra.w;
            Bs[nxt][lk + 0][lrow] = rb.x;
            Bs[nxt][lk + 1][lrow] = rb.y;
            Bs[nxt][lk + 2][lrow] = rb.z;
            Bs[nxt][lk + 3][lrow] = rb.w;
        }
        __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int n = n0 + ty * 4 + (i & 3) + (i >> 2) * 64;
        if (n >= N) continue;
#pragma unroll
        for (int jh = 0; jh < 2; ++jh) {
            const int mb = m0 + tx * 4 + jh * 64;
            if (MODE == kGemvSwiGLU) {
                // Columns (2j, 2j+1) hold (W1 row j, V row j).
#pragma unroll
                for (int jp = 0; jp < 4; jp += 2) {
                    const int m = mb + jp;
                    if (m + 1 < M) {
                        const float a = acc[i][jh * 4 + jp] + bias[m];
                        const float c = acc[i][jh * 4 + jp + 1] + bias[m + 1];
                        C[static_cast<size_t>(n) * (M >> 1) + (m >> 1)] = silu(a) * c;
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int m = mb + j;
                    if (m < M) {
                        const float v = acc[i][jh * 4 + j] + (bias ? bias[m] : 0.0f);
                        float* dst = C + static_cast<size_t>(n) * M + m;
                        if (MODE == kGemvResidual) *dst += v;
                        else *dst = v;
                    }
                }
            }
        }
    }
}

// One (row, head): rotate q in place and k, copy k / v into the head-major
// cache.  Row t of qkv is position p0 + t (p0 > 0: a prompt appended to a
// cached sequence).
__global__ void __launch_bounds__(32) rope_kv_prefill_kernel(float* __restrict__ qkv, const float2* __restrict__ rope,
                                                             float* __restrict__ kc, float* __restrict__ vc, int heads,
                                                             int max_ctx, int p0) {
    const int t = blockIdx.x, h = blockIdx.y, j = threadIdx.x;
    const int HL = heads * kHeadDim;
    float* row = qkv + static_cast<size_t>(t) * 3 * HL;
    const int pos = p0 + t;
    const float2 cs = rope[pos * kHalfHead + j];
    float* q = row + h * kHeadDim;
    const float qa = q[j], qb = q[j + kHalfHead];
    q[j] = qa * cs.x + qb * cs.y;
    q[j + kHalfHead] = -qa * cs.y + qb * cs.x;
    const float* k = row + HL + h * kHeadDim;
    const float* v = row + 2 * HL + h * kHeadDim;
    const float ka = k[j], kb = k[j + kHalfHead];
    float* kd = kc + (static_cast<size_t>(h) * max_ctx + pos) * kHeadDim;
    float* vd = vc + (static_cast<size_t>(h) * max_ctx + pos) * kHeadDim;
    kd[j] = ka * cs.x + kb * cs.y;
    kd[j + kHalfHead] = -ka * cs.y + kb * cs.x;
    vd[j] = v[j];
    vd[j + kHalfHead] = v[j + kHalfHead];
}

// RoPE, KV append and the operands of the tensor-core attention for a tile of
// 32 rows of one head (prompts that start at position 0): rotates q and k with
// the angle table as rope_kv_prefill does, writes k and v into the
// head-major cache, q/8 (the exact 1/sqrt(64) scale) into q8[t][h*64 + d],
// the rotated k into kq[h][t][d] and v transposed into vt[h*64 + d][t]
// (through shared memory, so that every store is a contiguous row), each
// operand with its tf32 lo half for the 3xTF32 products.
constexpr int kPrepRows = 32;
__global__ void __launch_bounds__(256) attn_prep_kernel(const float* __restrict__ qkv, const float2* __restrict__ rope,
                                                        float* __restrict__ kc, float* __restrict__ vc,
                                                        float* __restrict__ q8, float* __restrict__ q8_lo,
                                                        float* __restrict__ kq, float* __restrict__ kq_lo,
                                                        float* __restrict__ vt, float* __restrict__ vt_lo, int n,
                                                        int heads, int max_ctx) {
    __shared__ float vs[kHeadDim][kPrepRows + 1];
    const int t0 = blockIdx.x * kPrepRows, h = blockIdx.y;
    const int HL = heads * kHeadDim;
    for (int e = threadIdx.x; e < kPrepRows * kHalfHead; e += blockDim.x) {
        const int r = e >> 5, j = e & 31;  // a warp covers the 32 pairs (j, j + 32) of one row
        const int t = t0 + r;
        if (t >= n) continue;
        const float* row = qkv + static_cast<size_t>(t) * 3 * HL + h * kHeadDim;
        const float2 cs = rope[t * kHalfHead + j];
        const float qa = row[j], qb = row[j + kHalfHead];
        const float ka = row[HL + j], kb = row[HL + j + kHalfHead];
        const float va = row[2 * HL + j], vb = row[2 * HL + j + kHalfHead];
        const float qr0 = qa * cs.x + qb * cs.y, qr1 = -qa * cs.y + qb * cs.x;
        const float q0 = qr0 * 0.125f, q1 = qr1 * 0.125f;
        const float k0 = ka * cs.x + kb * cs.y, k1 = -ka * cs.y + kb * cs.x;
        const size_t qi = static_cast<size_t>(t) * HL + h * kHeadDim + j;
        q8[qi] = q0;
        q8[qi + kHalfHead] = q1;
        q8_lo[qi] = lo19(q0);
        q8_lo[qi + kHalfHead] = lo19(q1);
        const size_t ci = (static_cast<size_t>(h) * max_ctx + t) * kHeadDim + j;
        kc[ci] = k0;
        kc[ci + kHalfHead] = k1;
        vc[ci] = va;
        vc[ci + kHalfHead] = vb;
        kq[ci] = k0;
        kq[ci + kHalfHead] = k1;
        kq_lo[ci] = lo19(k0);
        kq_lo[ci + kHalfHead] = lo19(k1);
        vs[j][r] = va;
        vs[j + kHalfHead][r] = vb;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < kHeadDim * kPrepRows; e += blockDim.x) {
        const int d = e >> 5, r = e & 31;  // a warp stores 32 consecutive positions of one dim
        const int t = t0 + r;
        if (t >= n) continue;
        const float v = vs[d][r];
        const size_t vi = (static_cast<size_t>(h) * kHeadDim + d) * max_ctx + t;
        vt[vi] = v;
        vt_lo[vi] = lo19(v);
    }
}

// Causal softmax of one score row per warp: P[h][q][k] = exp(s - max) / sum for
// k <= q (the online-softmax result of src/attn.cu:47-167 written out), zero
// for q < k < kpad (the P.V GEMM reads keys up to kpad), plus the lo half.
// One warp per (head, query) row of S: the row is read once into registers
// (float4, up to kSmRowMax positions; longer rows take three passes over
// memory), the maximum and the sum of exponentials over keys 0 .. q are warp
// reductions, and P = e / sum and its TF32 lo half are written as float4 up to
// kpad (zeros past q).
constexpr int kSmRowMax = 2048;
__global__ void __launch_bounds__(256) attn_softmax_kernel(float* __restrict__ S, float* __restrict__ P_lo, int n,
                                                           int heads, int max_ctx, int kpad) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= n * heads) return;
    const int h = row / n, q = row % n;
    float* s = S + (static_cast<size_t>(h) * max_ctx + q) * max_ctx;
    float* pl = P_lo + (static_cast<size_t>(h) * max_ctx + q) * max_ctx;
    if (kpad <= kSmRowMax) {
        constexpr int kV = kSmRowMax / 128;  // float4 per lane
        float4 v[kV];
        float m = -INFINITY;
#pragma unroll
        for (int i = 0; i < kV; ++i) {
            const int k = 4 * (lane + 32 * i);
            if (k < kpad) {
                v[i] = reinterpret_cast<const float4*>(s)[lane + 32 * i];
                v[i].x = k <= q ? v[i].x : -INFINITY;
                v[i].y = k + 1 <= q ? v[i].y : -INFINITY;
                v[i].z = k + 2 <= q ? v[i].z : -INFINITY;
                v[i].w = k + 3 <= q ? v[i].w : -INFINITY;
                m = fmaxf(m, fmaxf(fmaxf(v[i].x, v[i].y), fmaxf(v[i].z, v[i].w)));
            }
        }
        m = warp_max(m);
        float l = 0.0f;
#pragma unroll
        for (int i = 0; i < kV; ++i) {
            const int k = 4 * (lane + 32 * i);
            if (k < kpad) {  // masked keys hold -inf: expf gives 0
                v[i].x = expf(v[i].x - m);
                v[i].y = expf(v[i].y - m);
                v[i].z = expf(v[i].z - m);
                v[i].w = expf(v[i].w - m);
                l += (v[i].x + v[i].y) + (v[i].z + v[i].w);
            }
        }
        l = warp_sum(l);
        const float inv = 1.0f / l;
#pragma unroll
        for (int i = 0; i < kV; ++i) {
            const int k = 4 * (lane + 32 * i);
            if (k < kpad) {
                const float4 p = make_float4(v[i].x * inv, v[i].y * inv, v[i].z * inv, v[i].w * inv);
                reinterpret_cast<float4*>(s)[lane + 32 * i] = p;
                reinterpret_cast<float4*>(pl)[lane + 32 * i] = make_float4(lo19(p.x), lo19(p.y), lo19(p.z), lo19(p.w));
            }
        }
        return;
    }
    float m = -INFINITY;
    for (int k = lane; k <= q; k += 32) m = fmaxf(m, s[k]);
    m = warp_max(m);
    float l = 0.0f;
    for (int k = lane; k <= q; k += 32) l += expf(s[k] - m);
    l = warp_sum(l);
    const float inv = 1.0f / l;
    for (int k = lane; k < kpad; k += 32) {
        const float p = k <= q ? expf(s[k] - m) * inv : 0.0f;
        s[k] = p;
        pl[k] = lo19(p);
    }
}

// Causal attention for one (64-query tile, head); 256 threads as 16 x 16,
// each owning a 4 x 4 block of the score tile and of the output tile.  Query
// row r is position p0 + r and attends to the cached positions 0 .. p0 + r
// (p0 > 0: a prompt appended to a cached sequence).
constexpr int kAT = 64;
constexpr int kAP = kAT + 4;

__global__ void __launch_bounds__(256) attn_prefill_kernel(const float* __restrict__ qkv, const float* __restrict__ kc,
                                                           const float* __restrict__ vc, float* __restrict__ out,
                                                           float* __restrict__ out_lo, int N, int heads, int max_ctx,
                                                           int p0) {
    extern __shared__ __align__(16) float smem[];
    float* Qt = smem;              // [64 dims][kAP] (q scaled by 1/8, transposed)
    float* Kt = Qt + kAT * kAP;    // [64 dims][kAP] (transposed)
    float* Vs = Kt + kAT * kAP;    // [64 keys][kAP]
    float* Pt = Vs + kAT * kAP;    // [64 keys][kAP] (probabilities, transposed)
    // Causal work grows with the query tile: launch the longest tiles first.
    const int qt = gridDim.x - 1 - blockIdx.x, h = blockIdx.y;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int HL = heads * kHeadDim;
    const int q0 = qt * kAT;
    const float* kh = kc + static_cast<size_t>(h) * max_ctx * kHeadDim;
    const float* vh = vc + static_cast<size_t>(h) * max_ctx * kHeadDim;

    for (int e = tid; e < kAT * kHeadDim; e += 256) {
        const int r = e >> 6, d = e & 63;
        const int t = q0 + r;
        Qt[d * kAP + r] = t < N ? qkv[static_cast<size_t>(t) * 3 * HL + h * kHeadDim + d] * 0.125f : 0.0f;
    }
    float m_run[4], l_run[4], o[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m_run[i] = -INFINITY;
        l_run[i] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) o[i][j] = 0.0f;
    }
    const int nk = p0 + N;  // keys: cached positions 0 .. p0 + N - 1
    const int last_kt = (p0 + min(q0 + kAT, N) - 1) / kAT;  // causal: through the tile's last query position
    for (int kt = 0; kt <= last_kt; ++kt) {
        const int k0 = kt * kAT;
        __syncthreads();
        for (int e = tid; e < kAT * kHeadDim / 4; e += 256) {
            const int r = e >> 4, d4 = (e & 15) * 4;
            const int t = k0 + r;
            const bool ok = t < nk;
            const float4 kv = ok ? *reinterpret_cast<const float4*>(kh + static_cast<size_t>(t) * kHeadDim + d4)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 vv = ok ? *reinterpret_cast<const float4*>(vh + static_cast<size_t>(t) * kHeadDim + d4)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            Kt[(d4 + 0) * kAP + r] = kv.x;
            Kt[(d4 + 1) * kAP + r] = kv.y;
            Kt[(d4 + 2) * kAP + r] = kv.z;
            Kt[(d4 + 3) * kAP + r] = kv.w;
            *reinterpret_cast<float4*>(&Vs[r * kAP + d4]) = vv;
        }
        __syncthreads();
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
#pragma unroll 8
        for (int d = 0; d < kHeadDim; ++d) {
            const float4 a = *reinterpret_cast<const float4*>(&Qt[d * kAP + ty * 4]);
            const float4 b = *reinterpret_cast<const float4*>(&Kt[d * kAP + tx * 4]);
            const float av[4] = {a.x, a.y, a.z, a.w};
            const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) s[i][j] = fmaf(av[i], bv[j], s[i][j]);
        }
        // causal / length mask, online softmax per query row
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int qi = p0 + q0 + ty * 4 + i;  // query position
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int kj = k0 + tx * 4 + j;
                if (kj > qi || kj >= nk) s[i][j] = -INFINITY;
                mx = fmaxf(mx, s[i][j]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_new = fmaxf(m_run[i], mx);
            // Rows past N (or fully masked so far) keep m = -inf; guard the exp.
            const float scale = (m_run[i] == -INFINITY) ? 0.0f : expf(m_run[i] - m_new);
            float rs = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float pj = (s[i][j] == -INFINITY) ? 0.0f : expf(s[i][j] - m_new);
                s[i][j] = pj;
                rs += pj;
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
            l_run[i] = l_run[i] * scale + rs;
            m_run[i] = m_new;
#pragma unroll
            for (int j = 0; j < 4; ++j) o[i][j] *= scale;
#pragma unroll
            for (int j = 0; j < 4; ++j) Pt[(tx * 4 + j) * kAP + ty * 4 + i] = s[i][j];
        }
        __syncthreads();
#pragma unroll 8
        for (int j = 0; j < kAT; ++j) {
            const float4 v = *reinterpret_cast<const float4*>(&Vs[j * kAP + tx * 4]);
            const float4 pq = *reinterpret_cast<const float4*>(&Pt[j * kAP + ty * 4]);
            const float pv[4] = {pq.x, pq.y, pq.z, pq.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                o[i][0] = fmaf(pv[i], v.x, o[i][0]);
                o[i][1] = fmaf(pv[i], v.y, o[i][1]);
                o[i][2] = fmaf(pv[i], v.z, o[i][2]);
                o[i][3] = fmaf(pv[i], v.w, o[i][3]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int qi = q0 + ty * 4 + i;
        if (qi < N) {
            const float inv = 1.0f / l_run[i];
            const float4 r = make_float4(o[i][0] * inv, o[i][1] * inv, o[i][2] * inv, o[i][3] * inv);
            const size_t off = static_cast<size_t>(qi) * HL + h * kHeadDim + tx * 4;
            *reinterpret_cast<float4*>(out + off) = r;
            if (out_lo) *reinterpret_cast<float4*>(out_lo + off) = make_float4(lo19(r.x), lo19(r.y), lo19(r.z), lo19(r.w));
        }
    }
}

__global__ void __launch_bounds__(256) add_rows_kernel(float* __restrict__ x, const float* __restrict__ d, int n) {
    const int i = blockIdx.x * 256 + threadIdx.x;
    if (i < n) x[i] += d[i];
}

constexpr size_t kAttnPrefillSmem = 4 * kAT * kAP * sizeof(float);

}  // namespace

cudaError_t launch_embed_gather(const float* table, const int* ids, float* out, int n, int k, cudaStream_t s) {
    if (n <= 0 || k % 4) return cudaErrorInvalidValue;
    count_launch();
    embed_gather_kernel<<<n, 256, 0, s>>>(table, ids, out, k);
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm_rows(const float* x, const float* gamma, float* out, float* out_lo, int n, int k,
                                cudaStream_t s) {
    if (n <= 0 || k % 4) return cudaErrorInvalidValue;
    count_launch();
    rmsnorm_rows_kernel<<<n, 256, 0, s>>>(x, gamma, out, out_lo, k, 1e-6);
    return cudaGetLastError();
}

cudaError_t launch_linear_prefill(int mode, const float* X, const float* W, const float* b, float* Y, int n, int m,
                                  int k, cudaStream_t s) {
    if (n <= 0 || m <= 0 || k % kBK) return cudaErrorInvalidValue;
    dim3 grid((m + kBN - 1) / kBN, (n + kBM - 1) / kBM);
    count_launch();
    switch (mode) {
        case kGemvPlain:
            sgemm_tn_kernel<kGemvPlain><<<grid, 256, 0, s>>>(X, W, b, Y, n, m, k);
            break;
        case kGemvSwiGLU:
            if (m % 2) return cudaErrorInvalidValue;
            sgemm_tn_kernel<kGemvSwiGLU><<<grid, 256, 0, s>>>(X, W, b, Y, n, m, k);
            break;
        case kGemvResidual:
            sgemm_tn_kernel<kGemvResidual><<<grid, 256, 0, s>>>(X, W, b, Y, n, m, k);
            break;
        default:
            return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_add_rows(float* x, const float* d, int n, cudaStream_t s) {
    if (n <= 0) return cudaErrorInvalidValue;
    count_launch();
    add_rows_kernel<<<(n + 255) / 256, 256, 0, s>>>(x, d, n);
    return cudaGetLastError();
}

cudaError_t launch_rope_kv_prefill(float* qkv, const float2* rope, float* kc, float* vc, int n, int heads,
                                   int max_ctx, cudaStream_t s, int p0) {
    if (n <= 0 || p0 < 0 || p0 + n > max_ctx) return cudaErrorInvalidValue;
    count_launch();
    rope_kv_prefill_kernel<<<dim3(n, heads), 32, 0, s>>>(qkv, rope, kc, vc, heads, max_ctx, p0);
    return cudaGetLastError();
}

cudaError_t launch_attn_prefill(const float* qkv, const float* kc, const float* vc, float* out, float* out_lo, int n,
                                int heads, int max_ctx, cudaStream_t s, int p0) {
    if (n <= 0 || p0 < 0 || p0 + n > max_ctx) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kAttnPrefillSmem));
    if (e != cudaSuccess) return e;
    count_launch();
    attn_prefill_kernel<<<dim3((n + kAT - 1) / kAT, heads), 256, kAttnPrefillSmem, s>>>(qkv, kc, vc, out, out_lo, n,
                                                                                        heads, max_ctx, p0);
    return cudaGetLastError();
}

cudaError_t launch_attn_prep(const float* qkv, const float2* rope, float* kc, float* vc, float* q8, float* q8_lo,
                             float* kq, float* kq_lo, float* vt, float* vt_lo, int n, int heads, int max_ctx,
                             cudaStream_t s) {
    if (n <= 0 || n > max_ctx) return cudaErrorInvalidValue;
    count_launch();
    attn_prep_kernel<<<dim3((n + kPrepRows - 1) / kPrepRows, heads), 256, 0, s>>>(qkv, rope, kc, vc, q8, q8_lo, kq,
                                                                                  kq_lo, vt, vt_lo, n, heads, max_ctx);
    return cudaGetLastError();
}

cudaError_t launch_attn_softmax(float* S, float* P_lo, int n, int heads, int max_ctx, cudaStream_t s) {
    const int kpad = ((n + 31) / 32) * 32;
    if (n <= 0 || n > max_ctx || kpad > max_ctx) return cudaErrorInvalidValue;
    count_launch();
    attn_softmax_kernel<<<(n * heads + 7) / 8, 256, 0, s>>>(S, P_lo, n, heads, max_ctx, kpad);
    return cudaGetLastError();
}

}  // namespace xl
