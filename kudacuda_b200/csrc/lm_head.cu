// lm_head.cu -- final RMSNorm + tied bf16 lm_head GEMV + greedy argmax, the
// embedding gather, and the small ABI-compatibility kernels.
//
// The reference leaves these to Transformers (lm_head + torch.argmax at
// tools/benchmark/benchmark_gemma.py:324,350; embedding lookup in the model),
// which forces a host round trip per token.  Here argmax runs on the device:
// every CTA reduces its rows to one (logit, index) candidate, and the last CTA
// to finish (self-resetting atomic ticket) picks the winner, lowest index on
// ties -- torch.argmax's rule over the bf16-rounded logits.
#include "kc_common.cuh"
#include "kc_launch.h"

namespace kc {

constexpr int kLmThreads = 256;
constexpr int kLmMaxH = 8192;

__device__ __forceinline__ void fma2_bf16_into_f32(uint32_t a, uint32_t b, float& even, float& odd) {
    asm("{\n\t.reg .b16 a0, a1, b0, b1;\n\t"
        "mov.b32 {a0, a1}, %2;\n\t"
        "mov.b32 {b0, b1}, %3;\n\t"
        "fma.rn.f32.bf16 %0, a0, b0, %0;\n\t"
        "fma.rn.f32.bf16 %1, a1, b1, %1;\n\t}"
        : "+f"(even), "+f"(odd)
        : "r"(a), "r"(b));
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

__global__ void __launch_bounds__(kLmThreads) lm_head_argmax_kernel(const LmHeadArgs a) {
    __shared__ __align__(16) uint16_t xs[kLmMaxH];
    __shared__ float red[32];
    __shared__ float cand_v[kLmThreads / 32];
    __shared__ int cand_i[kLmThreads / 32];
    __shared__ int last_s;

    pdl_launch_dependents();
    pdl_wait_on_producer();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int H = a.H;

    // final RMSNorm, Transformers' bf16 rounding points
    const uint16_t* x = static_cast<const uint16_t*>(a.hidden);
    const uint16_t* w = static_cast<const uint16_t*>(a.final_norm);
    float ss = 0.0F;
    for (int i = tid; i < H; i += kLmThreads) {
        const float v = bf16_bits_to_f32(x[i]);
        ss += v * v;
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (tid < 32) {
        float v = tid < kLmThreads / 32 ? red[tid] : 0.0F;
        v = warp_sum(v);
        if (tid == 0) red[0] = 1.0F / sqrtf(v / static_cast<float>(H) + a.eps);
    }
    __syncthreads();
    const float inv = red[0];
    for (int i = tid; i < H; i += kLmThreads)
        xs[i] = f32_to_bf16_bits(bf16_bits_to_f32(w[i]) * round_bf16(bf16_bits_to_f32(x[i]) * inv));
    __syncthreads();

    // rows: warp-tasks of two rows; lane streams 16-byte chunks (8 bf16)
    const int nchunks = H >> 3;
    const int ntasks = (a.vocab + 1) / 2;
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    const uint16_t* emb = static_cast<const uint16_t*>(a.emb);
    uint16_t* logits = static_cast<uint16_t*>(a.logits);
    for (int t = blockIdx.x + gridDim.x * warp; t < ntasks; t += gridDim.x * (kLmThreads / 32)) {
        const int r0 = 2 * t;
        const int r1 = r0 + 1 < a.vocab ? r0 + 1 : r0;
        const uint16_t* w0 = emb + static_cast<int64_t>(r0) * H;
        const uint16_t* w1 = emb + static_cast<int64_t>(r1) * H;
        float e0 = 0.0F, o0 = 0.0F, e1 = 0.0F, o1 = 0.0F;
        for (int c0 = lane; c0 < nchunks; c0 += 32 * 4) {
            uint4 wa[4], wb[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int c = c0 + 32 * u;
                if (c < nchunks) {
                    wa[u] = ld_stream_u4(w0 + 8 * c);
                    wb[u] = ld_stream_u4(w1 + 8 * c);
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int c = c0 + 32 * u;
                if (c < nchunks) {
                    const uint4 xv = *reinterpret_cast<const uint4*>(xs + 8 * c);
                    fma2_bf16_into_f32(wa[u].x, xv.x, e0, o0);
                    fma2_bf16_into_f32(wa[u].y, xv.y, e0, o0);
                    fma2_bf16_into_f32(wa[u].z, xv.z, e0, o0);
                    fma2_bf16_into_f32(wa[u].w, xv.w, e0, o0);
                    fma2_bf16_into_f32(wb[u].x, xv.x, e1, o1);
                    fma2_bf16_into_f32(wb[u].y, xv.y, e1, o1);
                    fma2_bf16_into_f32(wb[u].z, xv.z, e1, o1);
                    fma2_bf16_into_f32(wb[u].w, xv.w, e1, o1);
                }
            }
        }
        const float s0 = round_bf16(warp_sum(e0 + o0));
        const float s1 = round_bf16(warp_sum(e1 + o1));
        if (lane == 0) {
            if (logits != nullptr) {
                logits[r0] = f32_to_bf16_bits(s0);
                if (r1 != r0) logits[r1] = f32_to_bf16_bits(s1);
            }
            if (better(s0, r0, best_v, best_i)) { best_v = s0; best_i = r0; }
            if (r1 != r0 && better(s1, r1, best_v, best_i)) { best_v = s1; best_i = r1; }
        }
    }
    if (lane == 0) {
        cand_v[warp] = best_v;
        cand_i[warp] = best_i;
    }
    __syncthreads();
    if (tid == 0) {
        float bv = cand_v[0];
        int bi = cand_i[0];
        for (int i = 1; i < kLmThreads / 32; ++i)
            if (better(cand_v[i], cand_i[i], bv, bi)) { bv = cand_v[i]; bi = cand_i[i]; }
        a.partials[2 * blockIdx.x] = bv;
        a.partials[2 * blockIdx.x + 1] = __int_as_float(bi);
        __threadfence();
        const int ticket = atomicAdd(a.counter, 1);
        const int last = ticket == static_cast<int>(gridDim.x) - 1;
        if (last) atomicExch(a.counter, 0);
        last_s = last;
    }
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    if (warp == 0) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int b = lane; b < static_cast<int>(gridDim.x); b += 32) {
            const float v = __ldcg(a.partials + 2 * b);
            const int i = __float_as_int(__ldcg(a.partials + 2 * b + 1));
            if (better(v, i, bv, bi)) { bv = v; bi = i; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) a.token_out[0] = bi == 0x7fffffff ? 0 : bi;
    }
}

int lm_head_grid() { return device_sm_count() * 2; }

cudaError_t lm_head_argmax_bf16(const LmHeadArgs& a, cudaStream_t s) {
    if (a.H <= 0 || a.H > kLmMaxH || (a.H % 8) != 0 || a.vocab <= 0) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(a.emb) & 15u) != 0) return cudaErrorMisalignedAddress;
    return launch_pdl(lm_head_argmax_kernel, dim3(lm_head_grid()), dim3(kLmThreads), 0, s, a);
}

// ---------------------------------------------------------------------------
// Device-resident decode loop step: state = {token, position, kv_len, -};
// after the lm_head wrote next_token, feed it back as the next input, move
// the position on, and append the token to the history.  This replaces the
// host-side argmax/torch.cat/.item() loop of the reference benchmark
// (tools/benchmark/benchmark_gemma.py:328-352).
__global__ void decode_advance_kernel(int32_t* state, const int32_t* next_token, int32_t* history, int history_len) {
    pdl_launch_dependents();
    pdl_wait_on_producer();
    if (threadIdx.x != 0) return;
    const int32_t tok = *next_token;
    const int32_t pos = state[1] + 1;
    state[0] = tok;
    state[1] = pos;
    state[2] = pos + 1;
    if (history != nullptr && pos >= 0 && pos < history_len) history[pos] = tok;
}

cudaError_t decode_advance(int32_t* state, const int32_t* next_token, int32_t* history, int history_len,
                           cudaStream_t s) {
    return launch_pdl(decode_advance_kernel, dim3(1), dim3(32), 0, s, state, next_token, history, history_len);
}

// ---------------------------------------------------------------------------
__global__ void embedding_gather_kernel(const uint16_t* emb, const int32_t* token_dev, uint16_t* out, int H,
                                        int vocab, int* err) {
    pdl_launch_dependents();
    pdl_wait_on_producer();
    int tok = *token_dev;
    if (tok < 0 || tok >= vocab) {
        if (err != nullptr && threadIdx.x == 0) atomicOr(err, 8);
        tok = 0;
    }
    const uint16_t* row = emb + static_cast<int64_t>(tok) * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) out[i] = row[i];
}

cudaError_t embedding_gather_bf16(const void* emb, const int32_t* token_dev, void* out, int H, int vocab,
                                  int* err, cudaStream_t s) {
    if (H <= 0 || vocab <= 0) return cudaErrorInvalidValue;
    return launch_pdl(embedding_gather_kernel, dim3(1), dim3(256), 0, s, static_cast<const uint16_t*>(emb),
                      token_dev, static_cast<uint16_t*>(out), H, vocab, err);
}

// ---------------------------------------------------------------------------
// ABI-compatibility kernels (kernels/vector_add.cu:11-20, kernels/common/rmsnorm.cuh:11-47,
// kernels/common/rmsnorm_qkv_reference.cuh:12-66).  Same arithmetic, plain
// grid-stride loops; they are not on the decode hot path.

__global__ void vector_add_kernel(const float* a, const float* b, float* out, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = a[i] + b[i];
}

cudaError_t vector_add_f32(const float* a, const float* b, float* out, int64_t n, cudaStream_t s) {
    int64_t blocks = (n + 255) / 256;
    if (blocks > 65535) blocks = 65535;
    vector_add_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(a, b, out, n);
    return cudaGetLastError();
}

__global__ void rmsnorm_f32_kernel(const float* x, const float* w, float* out, int64_t hidden, float eps) {
    __shared__ float red[32];
    const float* xr = x + blockIdx.x * hidden;
    float ss = 0.0F;
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) ss += xr[i] * xr[i];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0F;
        v = warp_sum(v);
        if (threadIdx.x == 0) red[0] = rsqrtf(v / static_cast<float>(hidden) + eps);
    }
    __syncthreads();
    const float inv = red[0];
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) out[blockIdx.x * hidden + i] = xr[i] * inv * w[i];
}

cudaError_t rmsnorm_f32(const float* x, const float* w, float* out, int64_t rows, int64_t hidden, float eps,
                        cudaStream_t s) {
    if (rows <= 0 || rows > 2147483647 || hidden <= 0) return cudaErrorInvalidValue;
    rmsnorm_f32_kernel<<<static_cast<unsigned>(rows), 256, 0, s>>>(x, w, out, hidden, eps);
    return cudaGetLastError();
}

// dense fp16 [3H, H] RMSNorm + QKV: one CTA per input row normalises into
// shared memory, then one warp per output row does a coalesced dot.
__global__ void dense_rmsnorm_qkv_kernel(const __half* x, const __half* nw, const __half* w, const __half* bias,
                                         __half* out, int64_t hidden, float eps) {
    extern __shared__ float nrm[];
    __shared__ float red[32];
    const int64_t row = blockIdx.y;
    const __half* xr = x + row * hidden;
    float ss = 0.0F;
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) {
        const float v = __half2float(xr[i]);
        ss += v * v;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0F;
        v = warp_sum(v);
        if (threadIdx.x == 0) red[0] = rsqrtf(v / static_cast<float>(hidden) + eps);
    }
    __syncthreads();
    const float inv = red[0];
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x)
        nrm[i] = __half2float(xr[i]) * inv * __half2float(nw[i]);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t o = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); o < 3 * hidden;
         o += warps_total) {
        const __half* wr = w + o * hidden;
        float acc = 0.0F;
        for (int64_t i = lane; i < hidden; i += 32) acc += nrm[i] * __half2float(wr[i]);
        acc = warp_sum(acc);
        if (lane == 0) {
            if (bias != nullptr) acc += __half2float(bias[o]);
            out[row * hidden * 3 + o] = __float2half(acc);
        }
    }
}

cudaError_t dense_rmsnorm_qkv_f16(const void* x, const void* norm_w, const void* w, const void* bias, void* out,
                                  int64_t rows, int64_t hidden, float eps, cudaStream_t s) {
    if (rows <= 0 || rows > 65535 || hidden <= 0 || hidden > 12 * 1024) return cudaErrorInvalidValue;
    const size_t smem = static_cast<size_t>(hidden) * sizeof(float);
    if (smem > 48 * 1024) {
        const cudaError_t st = cudaFuncSetAttribute(dense_rmsnorm_qkv_kernel,
                                                    cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (st != cudaSuccess) return st;
    }
    const dim3 grid(static_cast<unsigned>(device_sm_count()), static_cast<unsigned>(rows));
    dense_rmsnorm_qkv_kernel<<<grid, 256, smem, s>>>(static_cast<const __half*>(x), static_cast<const __half*>(norm_w),
                                                     static_cast<const __half*>(w), static_cast<const __half*>(bias),
                                                     static_cast<__half*>(out), hidden, eps);
    return cudaGetLastError();
}

}  // namespace kc
