// gqa_decode.cu -- split-KV flash-decode for grouped-query attention, sm_100a.
//
// Replaces every reference GQA tactic behind its own ABI entry:
//   qwen2_gqa_decode_kernel<bool>       kernels/common/qwen2_gqa_decode.cuh:17-203
//   qwen2_gqa_group_tiled_kernel        kernels/common/qwen2_gqa_group_tiled.cuh:27-145
//   qwen2_gqa_vectorized_kernel         kernels/common/qwen2_gqa_vectorized.cuh:23-112
//   qwen2_gqa_workspace_{partial,reduce} kernels/common/qwen2_gqa_workspace.cuh:13-120
// Arithmetic (tests/qwen2_gqa_smoke.cu:65-93): fp32 scores q.k * scale, fp32
// softmax, fp32 P.V, one rounding to the cache dtype at the output.
//
// Layout: q [B][q_heads][128]; caches [B][kv_heads][stride][128] (token
// contiguous, stride = kv_len for direct calls, = capacity for graph calls);
// out [B][q_heads][128].
//
// One CTA = one (batch, kv head, token chunk): it serves all G = q_heads /
// kv_heads query heads of the group, so each K/V byte is read from HBM once
// (the reference reads each KV head once per query head).  Scores are kept in
// the log2 domain (q pre-scaled by scale * log2 e) and exponentiated with
// exp2.  Each CTA writes (max, sum, acc[128]) per head; the last CTA of a
// (batch, kv head) to finish -- found with a self-resetting atomic ticket --
// combines the partials, or a separate combine kernel does when the caller's
// workspace has no room for tickets (the workspace_v3 ABI).
#include "kc_common.cuh"
#include "kc_launch.h"

namespace kc {

constexpr int kHeadDim = 128;
constexpr int kGqaThreads = 256;
constexpr int kGqaMaxChunk = 256;
constexpr int kPartialStride = kHeadDim + 2;
constexpr float kLog2e = 1.4426950408889634F;

template <int DT>
__device__ __forceinline__ void load_vec8(const void* base, int64_t elem, float* out) {
    const uint4 v = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + elem);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if constexpr (DT == kBF16) {
            out[2 * i] = __uint_as_float(w[i] << 16);
            out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        } else {
            out[2 * i] = __half2float(__ushort_as_half(static_cast<uint16_t>(w[i] & 0xffffu)));
            out[2 * i + 1] = __half2float(__ushort_as_half(static_cast<uint16_t>(w[i] >> 16)));
        }
    }
}

template <int DT>
__device__ __forceinline__ void load_vec4(const void* base, int64_t elem, float* out) {
    const uint2 v = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(base) + elem);
    const uint32_t w[2] = {v.x, v.y};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        if constexpr (DT == kBF16) {
            out[2 * i] = __uint_as_float(w[i] << 16);
            out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        } else {
            out[2 * i] = __half2float(__ushort_as_half(static_cast<uint16_t>(w[i] & 0xffffu)));
            out[2 * i + 1] = __half2float(__ushort_as_half(static_cast<uint16_t>(w[i] >> 16)));
        }
    }
}

// Combine the nsplit partials of the G heads of one (batch, kv head).
template <int DT, int G>
__device__ void gqa_combine_group(const GqaArgs& a, int b, int kvh) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    for (int h = warp; h < G; h += kGqaThreads / 32) {
        const int qh = kvh * G + h;
        const float* base = a.partials + (static_cast<int64_t>(b) * a.q_heads + qh) * a.nsplit * kPartialStride;
        float m = -INFINITY;
        for (int s = 0; s < a.nsplit; ++s) m = fmaxf(m, __ldcg(base + s * kPartialStride));
        float l = 0.0F;
        float acc[4] = {0.0F, 0.0F, 0.0F, 0.0F};
        for (int s = 0; s < a.nsplit; ++s) {
            const float* p = base + s * kPartialStride;
            const float ms = __ldcg(p);
            if (ms == -INFINITY) continue;
            const float w = exp2f(ms - m);
            l += w * __ldcg(p + 1);
            // partials are 130 floats apart, so acc (offset 2) is only 8-byte aligned
            const float2 v0 = __ldcg(reinterpret_cast<const float2*>(p + 2) + 2 * lane);
            const float2 v1 = __ldcg(reinterpret_cast<const float2*>(p + 2) + 2 * lane + 1);
            acc[0] += w * v0.x;
            acc[1] += w * v0.y;
            acc[2] += w * v1.x;
            acc[3] += w * v1.y;
        }
        const float inv = l > 0.0F ? 1.0F / l : 0.0F;
        const int64_t o = (static_cast<int64_t>(b) * a.q_heads + qh) * kHeadDim + 4 * lane;
#pragma unroll
        for (int i = 0; i < 4; ++i) store_elem<DT>(a.out, o + i, acc[i] * inv);
    }
}

template <int DT, int G>
__global__ void __launch_bounds__(kGqaThreads) gqa_split_kernel(const GqaArgs a) {
    constexpr int LPH = 32 / G;          // lanes per head in the score phase
    constexpr int DPL = kHeadDim / LPH;  // dims per lane in the score phase
    __shared__ __align__(16) float s_s[G][kGqaMaxChunk];
    __shared__ float ml_s[G][2];
    __shared__ int last_s;

    pdl_launch_dependents();
    pdl_wait_on_producer();

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int b = blockIdx.x / a.kv_heads;
    const int kvh = blockIdx.x - b * a.kv_heads;
    const int split = blockIdx.y;

    int kv_len = a.kv_len_dev != nullptr ? *a.kv_len_dev : a.kv_len;
    if (kv_len < 1 || kv_len > a.stride) {
        if (a.err != nullptr && tid == 0) atomicOr(a.err, 4);
        kv_len = kv_len < 1 ? 0 : a.stride;
    }
    const int t0 = split * a.chunk;
    int n = kv_len - t0;
    n = n < 0 ? 0 : (n > a.chunk ? a.chunk : n);

    const int64_t kv_base = (static_cast<int64_t>(b) * a.kv_heads + kvh) * a.stride * kHeadDim;

    // ---- scores: lane (h, part) owns DPL dims of query head h ----
    {
        const int h = lane / LPH;
        const int part = lane - h * LPH;
        const int qh = kvh * G + h;
        float qv[DPL];
        const int64_t qoff = (static_cast<int64_t>(b) * a.q_heads + qh) * kHeadDim + part * DPL;
        const float qscale = a.scale * kLog2e;
        if constexpr (DPL >= 8) {
#pragma unroll
            for (int i = 0; i < DPL; i += 8) load_vec8<DT>(a.q, qoff + i, qv + i);
        } else {
            load_vec4<DT>(a.q, qoff, qv);
        }
#pragma unroll
        for (int i = 0; i < DPL; ++i) qv[i] *= qscale;
        for (int j = warp; j < n; j += kGqaThreads / 32) {
            const int64_t koff = kv_base + static_cast<int64_t>(t0 + j) * kHeadDim + part * DPL;
            float dot = 0.0F;
            if constexpr (DPL >= 8) {
#pragma unroll
                for (int i = 0; i < DPL; i += 8) {
                    float kv[8];
                    load_vec8<DT>(a.kcache, koff + i, kv);
#pragma unroll
                    for (int e = 0; e < 8; ++e) dot = fmaf(qv[i + e], kv[e], dot);
                }
            } else {
                float kv[4];
                load_vec4<DT>(a.kcache, koff, kv);
#pragma unroll
                for (int e = 0; e < 4; ++e) dot = fmaf(qv[e], kv[e], dot);
            }
#pragma unroll
            for (int o = LPH / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            if (part == 0) s_s[h][j] = dot;
        }
    }
    __syncthreads();

    // ---- per-head chunk softmax (log2 domain) ----
    for (int h = warp; h < G; h += kGqaThreads / 32) {
        float m = -INFINITY;
        for (int j = lane; j < n; j += 32) m = fmaxf(m, s_s[h][j]);
        m = warp_max(m);
        float l = 0.0F;
        for (int j = lane; j < n; j += 32) {
            const float p = exp2f(s_s[h][j] - m);
            s_s[h][j] = p;
            l += p;
        }
        l = warp_sum(l);
        if (lane == 0) {
            ml_s[h][0] = n > 0 ? m : -INFINITY;
            ml_s[h][1] = l;
        }
    }
    __syncthreads();

    // ---- P.V: warp h accumulates head h, lane owns dims 4*lane..4*lane+3 ----
    for (int h = warp; h < G; h += kGqaThreads / 32) {
        float acc[4] = {0.0F, 0.0F, 0.0F, 0.0F};
        for (int j = 0; j < n; ++j) {
            float v[4];
            load_vec4<DT>(a.vcache, kv_base + static_cast<int64_t>(t0 + j) * kHeadDim + 4 * lane, v);
            const float p = s_s[h][j];
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i] = fmaf(p, v[i], acc[i]);
        }
        const int qh = kvh * G + h;
        float* dst = a.partials + ((static_cast<int64_t>(b) * a.q_heads + qh) * a.nsplit + split) * kPartialStride;
        if (lane == 0) {
            dst[0] = ml_s[h][0];
            dst[1] = ml_s[h][1];
        }
        float2* acc2 = reinterpret_cast<float2*>(dst + 2);  // 8-byte aligned (130-float stride)
        acc2[2 * lane] = make_float2(acc[0], acc[1]);
        acc2[2 * lane + 1] = make_float2(acc[2], acc[3]);
    }

    if (a.counters == nullptr) return;
    // ---- last CTA of this (batch, kv head) combines ----
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        int* ctr = a.counters + blockIdx.x;
        const int ticket = atomicAdd(ctr, 1);
        const int last = ticket == a.nsplit - 1;
        if (last) atomicExch(ctr, 0);  // self-reset for the next launch / graph replay
        last_s = last;
    }
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    gqa_combine_group<DT, G>(a, b, kvh);
}

template <int DT, int G>
__global__ void __launch_bounds__(kGqaThreads) gqa_combine_kernel(const GqaArgs a) {
    pdl_launch_dependents();
    pdl_wait_on_producer();
    const int b = blockIdx.x / a.kv_heads;
    const int kvh = blockIdx.x - b * a.kv_heads;
    gqa_combine_group<DT, G>(a, b, kvh);
}

void gqa_plan_splits(int kv_extent, int batch, int kv_heads, int max_splits, int* chunk, int* nsplit) {
    const int ctas_per_split = batch * kv_heads > 0 ? batch * kv_heads : 1;
    const int target = (2 * device_sm_count() + ctas_per_split - 1) / ctas_per_split;
    int c = (kv_extent + target - 1) / (target > 0 ? target : 1);
    c = ((c + 15) / 16) * 16;
    if (c < 16) c = 16;
    if (c > kGqaMaxChunk) c = kGqaMaxChunk;
    int s = (kv_extent + c - 1) / c;
    if (max_splits > 0 && s > max_splits) {
        c = (kv_extent + max_splits - 1) / max_splits;
        c = ((c + 15) / 16) * 16;
        s = (kv_extent + c - 1) / c;
    }
    *chunk = c;
    *nsplit = s < 1 ? 1 : s;
}

size_t gqa_partials_floats(int batch, int q_heads, int nsplit, int head_dim) {
    return static_cast<size_t>(batch) * q_heads * nsplit * (head_dim + 2);
}

namespace {
template <int DT, int G>
cudaError_t gqa_launch(const GqaArgs& a, cudaStream_t s) {
    const dim3 grid(a.batch * a.kv_heads, a.nsplit);
    cudaError_t st = launch_pdl(gqa_split_kernel<DT, G>, grid, dim3(kGqaThreads), 0, s, a);
    if (st != cudaSuccess || a.counters != nullptr) return st;
    return launch_pdl(gqa_combine_kernel<DT, G>, dim3(a.batch * a.kv_heads), dim3(kGqaThreads), 0, s, a);
}
template <int DT>
cudaError_t gqa_dispatch_group(const GqaArgs& a, cudaStream_t s) {
    switch (a.q_heads / a.kv_heads) {
        case 1: return gqa_launch<DT, 1>(a, s);
        case 2: return gqa_launch<DT, 2>(a, s);
        case 4: return gqa_launch<DT, 4>(a, s);
        case 8: return gqa_launch<DT, 8>(a, s);
        default: return cudaErrorInvalidValue;
    }
}
}  // namespace

cudaError_t gqa_decode(GqaArgs a, int dt, cudaStream_t s) {
    if (a.head_dim != kHeadDim || a.kv_heads <= 0 || a.q_heads % a.kv_heads != 0 || a.batch <= 0 ||
        a.chunk <= 0 || a.chunk > kGqaMaxChunk || a.nsplit <= 0 || a.stride <= 0)
        return cudaErrorInvalidValue;
    if (static_cast<int64_t>(a.chunk) * a.nsplit < (a.kv_len_dev != nullptr ? a.stride : a.kv_len))
        return cudaErrorInvalidValue;
    const uintptr_t align = reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.kcache) |
                            reinterpret_cast<uintptr_t>(a.vcache) | reinterpret_cast<uintptr_t>(a.partials);
    if (align & 15u) return cudaErrorMisalignedAddress;
    if (dt == kBF16) return gqa_dispatch_group<kBF16>(a, s);
    if (dt == kF16) return gqa_dispatch_group<kF16>(a, s);
    return cudaErrorInvalidValue;
}

}  // namespace kc
