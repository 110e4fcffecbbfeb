// kc_common.cuh -- device helpers shared by the sm_100a decode kernels.
//
// NF4 format (bitsandbytes, as consumed by the reference at
// kernels/common/nf4_device.cuh:29-40): logical row-major [N, K], two codes
// per byte, even logical element in the HIGH nibble, one fp32 absmax per 64
// consecutive logical elements.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kc_launch.h"

namespace kc {

constexpr int kBlocksize = 64;

// The 16 NF4 levels (kernels/common/nf4_device.cuh:10-27).  Kept in
// __constant__ for the bit-exact dequant kernel, which reads one level per
// thread per element; the GEMVs never touch it in their inner loop.
__device__ __constant__ float kNf4Levels[16] = {
    -1.0F,
    -0.6961928009986877F,
    -0.5250730514526367F,
    -0.39491748809814453F,
    -0.28444138169288635F,
    -0.18477343022823334F,
    -0.09105003625154495F,
    0.0F,
    0.07958029955625534F,
    0.16093020141124725F,
    0.24611230194568634F,
    0.33791524171829224F,
    0.44070982933044434F,
    0.5626170039176941F,
    0.7229568362236023F,
    1.0F,
};

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  Every kernel in this library issues
// launch_dependents early and calls wait_on_producer before it touches any
// global memory that an earlier kernel in the stream writes (activations,
// caches, positions) and before it writes anything at all.  Only static data
// (NF4 weights, absmax, tables) may be read before the wait.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_on_producer() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Streaming loads for read-once weights: no L1 allocation.
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ float ld_stream_f32(const float* p) {
    float v;
    asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(p));
}

// ---------------------------------------------------------------------------
// Bulk async copies (TMA, non-tensor) and mbarriers.  Only local-GPU global
// memory is ever a source here and no copy uses cluster multicast.
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// global -> shared bulk copy completing `bytes` of transaction on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
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
// Bounded wait: gives up after `limit` polls (each poll itself may suspend
// for a hardware-defined time) and returns false so the caller can record an
// error and leave instead of hanging the GPU.
constexpr uint32_t kMbarPollLimit = 1u << 22;
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < kMbarPollLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// ---------------------------------------------------------------------------
// fp32 += f16 * f16 with a single rounding into fp32 (sm_100 mixed FMA).
// a and b hold two f16 lanes each; the even/odd lanes go to separate
// accumulators so the two dependency chains interleave.
__device__ __forceinline__ void fma2_f16_into_f32(uint32_t a, uint32_t b, float& even, float& odd) {
    asm("{\n\t.reg .f16 a0, a1, b0, b1;\n\t"
        "mov.b32 {a0, a1}, %2;\n\t"
        "mov.b32 {b0, b1}, %3;\n\t"
        "fma.rn.f32.f16 %0, a0, b0, %0;\n\t"
        "fma.rn.f32.f16 %1, a1, b1, %1;\n\t}"
        : "+f"(even), "+f"(odd)
        : "r"(a), "r"(b));
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
    return __uint_as_float(static_cast<uint32_t>(h) << 16);
}
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float round_bf16(float f) {
    return __bfloat162float(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ uint16_t f32_to_f16_bits(float f) {
    return __half_as_ushort(__float2half_rn(f));
}

// element io by dtype code (DType in kc_launch.h: 0 = f32, 1 = f16, 2 = bf16)
template <int DT>
__device__ __forceinline__ float load_elem(const void* p, int64_t i) {
    if constexpr (DT == kF16) return f16_bits_to_f32(static_cast<const uint16_t*>(p)[i]);
    else if constexpr (DT == kBF16) return bf16_bits_to_f32(static_cast<const uint16_t*>(p)[i]);
    else return static_cast<const float*>(p)[i];
}
template <int DT>
__device__ __forceinline__ void store_elem(void* p, int64_t i, float v) {
    if constexpr (DT == kF16) static_cast<uint16_t*>(p)[i] = f32_to_f16_bits(v);
    else if constexpr (DT == kBF16) static_cast<uint16_t*>(p)[i] = f32_to_bf16_bits(v);
    else static_cast<float*>(p)[i] = v;
}

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

// ---------------------------------------------------------------------------
// Codebook-pair lookup table.
//
// Entry e (a packed byte) holds half2(level[e >> 4], level[e & 15]): the even
// element's level in the low half, the odd element's in the high half, the
// same order as an f16 activation pair in memory.  It is replicated once per
// lane with a 128-byte entry stride, so lane l always reads bank l and a
// warp's 32 data-dependent lookups never conflict: byte offset
// (e << 7) | (lane << 2) in a 32 KB table.
constexpr int kLutWords = 256 * 32;

// `lut` must be 16-byte aligned: each thread writes four replicas of an
// entry with one 16-byte store.
__device__ __forceinline__ void build_pair_lut(uint32_t* lut, int tid, int nthreads) {
    for (int i = tid; i < kLutWords / 4; i += nthreads) {
        const int e = i >> 3;  // 8 x 16 bytes per 128-byte entry
        const __half lo = __float2half_rn(kNf4Levels[e >> 4]);
        const __half hi = __float2half_rn(kNf4Levels[e & 15]);
        const uint32_t w = static_cast<uint32_t>(__half_as_ushort(lo)) |
                           (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
        reinterpret_cast<uint4*>(lut)[i] = make_uint4(w, w, w, w);
    }
}

__device__ __forceinline__ uint32_t lut_at(const uint32_t* lut, uint32_t byte_offset) {
    return *reinterpret_cast<const uint32_t*>(reinterpret_cast<const char*>(lut) + byte_offset);
}

// Dot of 8 NF4 weights (one packed word, 4 bytes) with 4 f16 activation
// pairs.  Byte j of `word` selects LUT entry ((word >> 8j) & 0xff).
__device__ __forceinline__ void nf4_word_dot(const uint32_t* lut, uint32_t lane_off, uint32_t word,
                                             const uint32_t* xpairs, float& even, float& odd) {
    const uint32_t o0 = ((word << 7) & 0x7f80u) | lane_off;
    const uint32_t o1 = ((word >> 1) & 0x7f80u) | lane_off;
    const uint32_t o2 = ((word >> 9) & 0x7f80u) | lane_off;
    const uint32_t o3 = ((word >> 17) & 0x7f80u) | lane_off;
    fma2_f16_into_f32(lut_at(lut, o0), xpairs[0], even, odd);
    fma2_f16_into_f32(lut_at(lut, o1), xpairs[1], even, odd);
    fma2_f16_into_f32(lut_at(lut, o2), xpairs[2], even, odd);
    fma2_f16_into_f32(lut_at(lut, o3), xpairs[3], even, odd);
}

// Activation vector staging: f16 values in shared memory, 16-byte chunks
// swizzled so that lane c reading chunks 4c..4c+3 (the 32 activations that
// match its 16-byte weight chunk) is conflict-free per quarter-warp.
__device__ __forceinline__ int x_chunk_slot(int q) { return (q & ~3) | ((q & 3) ^ ((q >> 3) & 3)); }

__device__ __forceinline__ void load_x32(const uint4* xs, int chunk, uint32_t* out16) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const uint4 v = xs[x_chunk_slot(chunk * 4 + t)];
        out16[4 * t + 0] = v.x;
        out16[4 * t + 1] = v.y;
        out16[4 * t + 2] = v.z;
        out16[4 * t + 3] = v.w;
    }
}

}  // namespace kc
