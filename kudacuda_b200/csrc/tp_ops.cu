// tp_ops.cu -- the small device ops a tensor-parallel decode step needs
// around the NF4 GEMVs (no reference counterpart: the reference runs one GPU).
//
//   * residual_add_f32: resid = bf16(resid + bf16(partial_sum)) after the
//     allreduce of a row-parallel GEMV's fp32 partials -- the same two
//     roundings the single-GPU fused linear+residual epilogue applies;
//   * argmax_shard: greedy argmax of this rank's vocabulary slice of fp32
//     logits, compared after rounding to bf16 (Transformers computes bf16
//     logits, torch.argmax keeps the lowest index on ties); writes one
//     (value, global index) pair;
//   * select_token: the lowest-index maximum over the gathered pairs of all
//     ranks -> next token.
#include <cstdint>

#include "kc_common.cuh"
#include "kc_launch.h"

namespace kc {

__global__ void residual_add_f32_kernel(const float* partial, uint16_t* resid, int n) {
    pdl_launch_dependents();
    pdl_wait_on_producer();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        resid[i] = f32_to_bf16_bits(bf16_bits_to_f32(resid[i]) + round_bf16(partial[i]));
}

cudaError_t residual_add_f32_bf16(const float* partial, void* resid, int n, cudaStream_t s) {
    if (n <= 0) return cudaErrorInvalidValue;
    const int blocks = (n + 255) / 256 < 64 ? (n + 255) / 256 : 64;
    return launch_pdl(residual_add_f32_kernel, dim3(blocks), dim3(256), 0, s, partial, static_cast<uint16_t*>(resid), n);
}

__device__ __forceinline__ bool pair_better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

constexpr int kArgThreads = 256;
constexpr int kArgBlocks = 64;

// Each CTA scans a slice and leaves its best pair in ws; the last CTA (self-
// resetting ticket) reduces the kArgBlocks candidates.
__global__ void __launch_bounds__(kArgThreads) argmax_shard_kernel(const float* logits, int n, int index_base,
                                                                  float* ws, int* ticket, ArgPair* out) {
    __shared__ float sv[kArgThreads / 32];
    __shared__ int si[kArgThreads / 32];
    __shared__ int last_s;
    pdl_launch_dependents();
    pdl_wait_on_producer();
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = blockIdx.x * kArgThreads + threadIdx.x; i < n; i += gridDim.x * kArgThreads) {
        const float v = round_bf16(logits[i]);
        if (pair_better(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (pair_better(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kArgThreads / 32; ++w)
            if (pair_better(sv[w], si[w], sv[0], si[0])) {
                sv[0] = sv[w];
                si[0] = si[w];
            }
        ws[2 * blockIdx.x] = sv[0];
        ws[2 * blockIdx.x + 1] = __int_as_float(si[0]);
        __threadfence();
        const int t = atomicAdd(ticket, 1);
        last_s = t == gridDim.x - 1;
        if (last_s) atomicExch(ticket, 0);
    }
    __syncthreads();
    if (!last_s || threadIdx.x != 0) return;
    __threadfence();
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int b = 0; b < gridDim.x; ++b) {
        const float cv = __ldcg(ws + 2 * b);
        const int ci = __float_as_int(__ldcg(ws + 2 * b + 1));
        if (pair_better(cv, ci, v, idx)) {
            v = cv;
            idx = ci;
        }
    }
    out->value = v;
    out->index = index_base + idx;
}

cudaError_t argmax_shard_f32(const float* logits, int n, int index_base, float* ws, int* ticket, ArgPair* out,
                             cudaStream_t s) {
    if (n <= 0) return cudaErrorInvalidValue;
    return launch_pdl(argmax_shard_kernel, dim3(kArgBlocks), dim3(kArgThreads), 0, s, logits, n, index_base, ws,
                      ticket, out);
}

int argmax_shard_workspace_floats() { return 2 * kArgBlocks; }

__global__ void select_token_kernel(const ArgPair* pairs, int count, int32_t* next_token) {
    pdl_launch_dependents();
    pdl_wait_on_producer();
    if (threadIdx.x != 0) return;
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int r = 0; r < count; ++r)
        if (pair_better(pairs[r].value, pairs[r].index, v, idx)) {
            v = pairs[r].value;
            idx = pairs[r].index;
        }
    *next_token = idx == 0x7fffffff ? 0 : idx;
}

cudaError_t select_token(const ArgPair* pairs, int count, int32_t* next_token, cudaStream_t s) {
    if (count <= 0) return cudaErrorInvalidValue;
    return launch_pdl(select_token_kernel, dim3(1), dim3(32), 0, s, pairs, count, next_token);
}

}  // namespace kc
