// Device-side helpers shared by the XingLing sm_100a kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace xl {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue (weight prefetch) early, and wait for the previous kernel's
// results before touching activations.  Both are no-ops without PDL.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Streaming 128-bit load of read-once weights: no L1 allocation.
__device__ __forceinline__ float4 ld_stream(const float4* p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

// Bulk prefetch of a contiguous byte range into L2 (TMA engine, no smem).
// ptr must be 16-byte aligned and bytes a multiple of 16.
__device__ __forceinline__ void prefetch_l2_bulk(const void* ptr, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ptr), "r"(bytes) : "memory");
}

__device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
    acc = fmaf(a.x, b.x, acc);
    acc = fmaf(a.y, b.y, acc);
    acc = fmaf(a.z, b.z, acc);
    acc = fmaf(a.w, b.w, acc);
    return acc;
}

// Order-preserving map of an fp32 value to uint32 (larger float -> larger key).
// -0.0 maps to the key of +0.0: the reference compares floats, so the two
// zeros tie and the lower id wins.
__device__ __forceinline__ uint32_t float_key(float f) {
    uint32_t u = __float_as_uint(f);
    if (u == 0x80000000u) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}

// Argmax packing: value key in the high word, (~index) in the low word so
// that atomicMax prefers the larger value and, on ties, the lower index.
__device__ __forceinline__ unsigned long long pack_argmax(float v, int idx) {
    return (static_cast<unsigned long long>(float_key(v)) << 32) |
           static_cast<unsigned long long>(0xffffffffu - static_cast<uint32_t>(idx));
}
__device__ __forceinline__ int unpack_argmax_index(unsigned long long k) {
    return static_cast<int>(0xffffffffu - static_cast<uint32_t>(k & 0xffffffffull));
}

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

// Repetition penalty of src/inference.cu:71-74.
__device__ __forceinline__ float rep_penalty(float v, float rp) { return v > 0.0f ? v / rp : v * rp; }

}  // namespace xl
