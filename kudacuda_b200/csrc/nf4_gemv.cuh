// nf4_gemv.cuh -- batch-1 NF4 dequant-GEMV family for sm_100a.
//
// Replaces the reference's per-op GEMV kernels
//   kernels/common/nf4_tiled_gemv.cuh:61-278   (RMSNorm + Q/K/V, v2/v3)
//   kernels/common/nf4_fused_rmsnorm_qkv.cuh:15-102 (RMSNorm + Q/K/V, v1)
//   kernels/common/nf4_swiglu.cuh:65-165, nf4_swiglu_bf16.cuh:65-166 (gate/up SwiGLU)
// and adds the o_proj / down_proj / generic GEMV the reference leaves to
// bitsandbytes (python/kudacuda_sidecar.py:947, :1746).
//
// Design (HBM-bound, 0.5625 B per weight):
//   * one warp owns a task of two weight rows and streams both rows' packed
//     nibbles with 16-byte read-once loads, four chunks per row in flight;
//   * each 16-byte chunk (32 weights) is dequantised through a 32 KB
//     bank-conflict-free codebook-pair table and accumulated with sm_100's
//     mixed f16*f16+f32 FMA, then scaled once by its 64-block absmax;
//   * the activation vector is staged once per CTA as f16 in swizzled shared
//     memory and re-used by both rows of every task;
//   * the two rows of a task are chosen so the epilogue can finish the op in
//     registers: RoPE partners (i, i+64), SwiGLU partners (gate j, up j), or
//     K/V partners (k j, v j);
//   * programmatic dependent launch: the table build overlaps the previous
//     kernel; activations are read only after griddepcontrol.wait.
#pragma once

#include "kc_common.cuh"

namespace kc {

enum InMode : int {
    kInRaw = 0,      // x used as given
    kInNormRef = 1,  // RMSNorm, normalised vector kept in fp32 (reference kernels)
    kInNormHF = 2,   // RMSNorm with Transformers' bf16 rounding points
};

enum EpiMode : int {
    kEpiStore = 0,      // out0[r] = acc (+ bias0[r])            (dtype OT)
    kEpiQkvRef = 1,     // q/k/v rows: out_s[r] = acc + bias_s[r] (dtype OT)
    kEpiQkvRopeHF = 2,  // bf16(bf16(acc)+b), RoPE, q -> out0, k/v -> caches at *pos
    kEpiSwiGluRef = 3,  // out0[j] = silu(g) * u                  (dtype OT)
    kEpiSwiGluHF = 4,   // out0[j] = bf16(bf16(silu(bf16 g)) * bf16 u)
    kEpiResidHF = 5,    // resid[r] = bf16(resid[r] + bf16(acc))
};

struct Nf4Matrix {
    const uint8_t* packed;  // [rows * K / 2]
    const float* absmax;    // [rows * K / 64]
    int rows;
};

struct Nf4GemvArgs {
    Nf4Matrix m[3];
    int K;
    int ntasks;
    const void* x;       // [K]
    const void* norm_w;  // [K]
    float eps;
    float* norm_ws;      // optional fp32 normalised output (reference v2/v3 workspace)
    void* out[3];
    const void* bias[3];
    void* resid;               // bf16 [rows] residual stream (kEpiResidHF)
    const uint16_t* rope_cos;  // bf16 [max_pos][head_dim/2]
    const uint16_t* rope_sin;
    const int32_t* pos_dev;    // device position of the new token
    int head_dim;
    int q_heads;
    int kv_heads;
    int kv_cap;
    int max_pos;
    int* err;  // optional error word; bit 0: f16 range, bit 1: position out of range
    int xvec;    // x and norm_w are 16-byte aligned: stage them with 16-byte vector loads
    int stages;  // TMA kernel: shared-memory ring depth chosen by the host
};

struct RowPair {
    const uint8_t* w0;
    const uint8_t* w1;
    const float* a0;
    const float* a1;
    int kind;  // epilogue-specific selector
    int r0, r1;
};

template <int EPI>
__device__ __forceinline__ RowPair decode_task(const Nf4GemvArgs& a, int t) {
    RowPair p;
    const int64_t rb = a.K / 2;
    const int64_t ab = a.K / kBlocksize;
    auto setrow = [&](int s0, int r0, int s1, int r1) {
        p.w0 = a.m[s0].packed + rb * r0;
        p.a0 = a.m[s0].absmax + ab * r0;
        p.w1 = a.m[s1].packed + rb * r1;
        p.a1 = a.m[s1].absmax + ab * r1;
        p.r0 = r0;
        p.r1 = r1;
    };
    if constexpr (EPI == kEpiStore || EPI == kEpiResidHF) {
        const int r0 = 2 * t;
        const int r1 = r0 + 1 < a.m[0].rows ? r0 + 1 : r0;  // odd tail: duplicate row, skip store
        setrow(0, r0, 0, r1);
        p.kind = r1 == r0 ? 1 : 0;
    } else if constexpr (EPI == kEpiQkvRef) {
        const int qt = (a.m[0].rows + 1) / 2;
        if (t < qt) {
            const int r0 = 2 * t;
            const int r1 = r0 + 1 < a.m[0].rows ? r0 + 1 : r0;
            setrow(0, r0, 0, r1);
            p.kind = r1 == r0 ? 3 : 0;
        } else {
            const int j = t - qt;
            setrow(1, j, 2, j);
            p.kind = 1;
        }
    } else if constexpr (EPI == kEpiQkvRopeHF) {
        const int half = a.head_dim / 2;
        const int qt = a.q_heads * half;
        const int kt = a.kv_heads * half;
        if (t < qt + kt) {
            const int s = t < qt ? 0 : 1;
            const int u = t < qt ? t : t - qt;
            const int head = u / half;
            const int i = u - head * half;
            const int r0 = head * a.head_dim + i;
            setrow(s, r0, s, r0 + half);
            p.kind = s;  // 0 = q, 1 = k
        } else {
            const int j = t - qt - kt;
            setrow(2, 2 * j, 2, 2 * j + 1);
            p.kind = 2;  // v
        }
    } else {  // SwiGLU: gate row j with up row j
        setrow(0, t, 1, t);
        p.kind = 0;
    }
    return p;
}

// Stage the (optionally normalised) activation vector as swizzled f16.
template <int IN, int XT>
__device__ __forceinline__ void stage_x(const Nf4GemvArgs& a, uint4* xs, float* red) {
    const int tid = threadIdx.x;
    const int nthreads = blockDim.x;
    const int K = a.K;
    float inv = 1.0F;
    if constexpr (IN != kInRaw) {
        float ss = 0.0F;
        for (int i = tid; i < K; i += nthreads) {
            const float v = load_elem<XT>(a.x, i);
            ss += v * v;
        }
        ss = warp_sum(ss);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        __syncthreads();
        if (tid < 32) {
            float v = tid < (nthreads >> 5) ? red[tid] : 0.0F;
            v = warp_sum(v);
            if (tid == 0) red[0] = 1.0F / sqrtf(v / static_cast<float>(K) + a.eps);
        }
        __syncthreads();
        inv = red[0];
    }
    bool overflow = false;
    for (int q = tid; q < K / 8; q += nthreads) {
        uint32_t packed[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            float v[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int i = 8 * q + e + h;
                float x = load_elem<XT>(a.x, i);
                if constexpr (IN == kInNormRef) {
                    x = x * inv * load_elem<XT>(a.norm_w, i);
                    if (a.norm_ws != nullptr && blockIdx.x == 0) a.norm_ws[i] = x;
                } else if constexpr (IN == kInNormHF) {
                    x = round_bf16(load_elem<XT>(a.norm_w, i) * round_bf16(x * inv));
                }
                overflow |= !(fabsf(x) <= 65504.0F);
                v[h] = x;
            }
            packed[e / 2] = static_cast<uint32_t>(f32_to_f16_bits(v[0])) |
                            (static_cast<uint32_t>(f32_to_f16_bits(v[1])) << 16);
        }
        xs[x_chunk_slot(q)] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
    if (overflow && a.err != nullptr) atomicOr(a.err, 1);
    __syncthreads();
}

template <int EPI, int OT>
__device__ __forceinline__ void epilogue(const Nf4GemvArgs& a, const RowPair& p, float s0, float s1) {
    if constexpr (EPI == kEpiStore) {
        const float b0 = a.bias[0] ? load_elem<OT>(a.bias[0], p.r0) : 0.0F;
        store_elem<OT>(a.out[0], p.r0, s0 + b0);
        if (p.kind == 0) {
            const float b1 = a.bias[0] ? load_elem<OT>(a.bias[0], p.r1) : 0.0F;
            store_elem<OT>(a.out[0], p.r1, s1 + b1);
        }
    } else if constexpr (EPI == kEpiResidHF) {
        uint16_t* r = static_cast<uint16_t*>(a.resid);
        r[p.r0] = f32_to_bf16_bits(bf16_bits_to_f32(r[p.r0]) + round_bf16(s0));
        if (p.kind == 0) r[p.r1] = f32_to_bf16_bits(bf16_bits_to_f32(r[p.r1]) + round_bf16(s1));
    } else if constexpr (EPI == kEpiQkvRef) {
        if (p.kind == 1) {
            store_elem<OT>(a.out[1], p.r0, s0 + load_elem<OT>(a.bias[1], p.r0));
            store_elem<OT>(a.out[2], p.r1, s1 + load_elem<OT>(a.bias[2], p.r1));
        } else {
            store_elem<OT>(a.out[0], p.r0, s0 + load_elem<OT>(a.bias[0], p.r0));
            if (p.kind == 0) store_elem<OT>(a.out[0], p.r1, s1 + load_elem<OT>(a.bias[0], p.r1));
        }
    } else if constexpr (EPI == kEpiQkvRopeHF) {
        const int s = p.kind;
        float y0 = round_bf16(s0);
        float y1 = round_bf16(s1);
        if (a.bias[s] != nullptr) {
            y0 = round_bf16(y0 + load_elem<kBF16>(a.bias[s], p.r0));
            y1 = round_bf16(y1 + load_elem<kBF16>(a.bias[s], p.r1));
        }
        const int pos = *a.pos_dev;
        if (pos < 0 || pos >= a.kv_cap || pos >= a.max_pos) {
            if (a.err != nullptr) atomicOr(a.err, 2);
            return;
        }
        if (s == 2) {  // V: no rotation, append at pos
            uint16_t* vc = static_cast<uint16_t*>(a.out[2]);
            const int h0 = p.r0 / a.head_dim, d0 = p.r0 - h0 * a.head_dim;
            const int h1 = p.r1 / a.head_dim, d1 = p.r1 - h1 * a.head_dim;
            vc[(static_cast<int64_t>(h0) * a.kv_cap + pos) * a.head_dim + d0] = f32_to_bf16_bits(y0);
            vc[(static_cast<int64_t>(h1) * a.kv_cap + pos) * a.head_dim + d1] = f32_to_bf16_bits(y1);
            return;
        }
        const int half = a.head_dim / 2;
        const int head = p.r0 / a.head_dim;
        const int i = p.r0 - head * a.head_dim;
        const float c = bf16_bits_to_f32(a.rope_cos[static_cast<int64_t>(pos) * half + i]);
        const float sn = bf16_bits_to_f32(a.rope_sin[static_cast<int64_t>(pos) * half + i]);
        const float lo = round_bf16(round_bf16(y0 * c) + round_bf16(-y1 * sn));
        const float hi = round_bf16(round_bf16(y1 * c) + round_bf16(y0 * sn));
        if (s == 0) {
            uint16_t* q = static_cast<uint16_t*>(a.out[0]);
            q[p.r0] = f32_to_bf16_bits(lo);
            q[p.r1] = f32_to_bf16_bits(hi);
        } else {
            uint16_t* kc = static_cast<uint16_t*>(a.out[1]);
            const int64_t base = (static_cast<int64_t>(head) * a.kv_cap + pos) * a.head_dim;
            kc[base + i] = f32_to_bf16_bits(lo);
            kc[base + i + half] = f32_to_bf16_bits(hi);
        }
    } else if constexpr (EPI == kEpiSwiGluRef) {
        store_elem<OT>(a.out[0], p.r0, (s0 / (1.0F + expf(-s0))) * s1);
    } else if constexpr (EPI == kEpiSwiGluHF) {
        const float g = round_bf16(s0);
        const float u = round_bf16(s1);
        const float act = round_bf16(g / (1.0F + expf(-g)));
        store_elem<kBF16>(a.out[0], p.r0, act * u);
    }
}

constexpr int kGemvThreads = 256;
constexpr int kGemvUnroll = 4;  // chunks per row in flight per lane

template <int IN, int XT, int EPI, int OT>
__global__ void __launch_bounds__(kGemvThreads, 2) nf4_gemv_kernel(const Nf4GemvArgs a) {
    __shared__ __align__(16) uint32_t lut[kLutWords];
    __shared__ float red[32];
    extern __shared__ __align__(16) uint4 xs[];

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int nwarps = blockDim.x >> 5;

    build_pair_lut(lut, tid, blockDim.x);
    pdl_launch_dependents();
    pdl_wait_on_producer();
    stage_x<IN, XT>(a, xs, red);  // ends with __syncthreads (also covers the table)

    const uint32_t lane_off = static_cast<uint32_t>(lane) << 2;
    const int nchunks = a.K >> 5;
    for (int t = blockIdx.x + gridDim.x * warp; t < a.ntasks; t += gridDim.x * nwarps) {
        const RowPair p = decode_task<EPI>(a, t);
        float acc0 = 0.0F, acc1 = 0.0F;
        for (int c0 = lane; c0 < nchunks; c0 += 32 * kGemvUnroll) {
            uint4 wa[kGemvUnroll], wb[kGemvUnroll];
            float sa[kGemvUnroll], sb[kGemvUnroll];
#pragma unroll
            for (int u = 0; u < kGemvUnroll; ++u) {
                const int c = c0 + 32 * u;
                if (c < nchunks) {
                    wa[u] = ld_stream_u4(p.w0 + 16 * static_cast<int64_t>(c));
                    wb[u] = ld_stream_u4(p.w1 + 16 * static_cast<int64_t>(c));
                    sa[u] = ld_stream_f32(p.a0 + (c >> 1));
                    sb[u] = ld_stream_f32(p.a1 + (c >> 1));
                }
            }
#pragma unroll
            for (int u = 0; u < kGemvUnroll; ++u) {
                const int c = c0 + 32 * u;
                if (c < nchunks) {
                    uint32_t xr[16];
                    load_x32(xs, c, xr);
                    float e0 = 0.0F, o0 = 0.0F, e1 = 0.0F, o1 = 0.0F;
                    nf4_word_dot(lut, lane_off, wa[u].x, xr + 0, e0, o0);
                    nf4_word_dot(lut, lane_off, wb[u].x, xr + 0, e1, o1);
                    nf4_word_dot(lut, lane_off, wa[u].y, xr + 4, e0, o0);
                    nf4_word_dot(lut, lane_off, wb[u].y, xr + 4, e1, o1);
                    nf4_word_dot(lut, lane_off, wa[u].z, xr + 8, e0, o0);
                    nf4_word_dot(lut, lane_off, wb[u].z, xr + 8, e1, o1);
                    nf4_word_dot(lut, lane_off, wa[u].w, xr + 12, e0, o0);
                    nf4_word_dot(lut, lane_off, wb[u].w, xr + 12, e1, o1);
                    acc0 = fmaf(e0 + o0, sa[u], acc0);
                    acc1 = fmaf(e1 + o1, sb[u], acc1);
                }
            }
        }
        acc0 = warp_sum(acc0);
        acc1 = warp_sum(acc1);
        if (lane == 0) epilogue<EPI, OT>(a, p, acc0, acc1);
    }
}

// Number of two-row tasks for each epilogue.
inline int gemv_tasks(int epi, const Nf4GemvArgs& a) {
    switch (epi) {
        case kEpiStore:
        case kEpiResidHF:
            return (a.m[0].rows + 1) / 2;
        case kEpiQkvRef:
            return (a.m[0].rows + 1) / 2 + a.m[1].rows;
        case kEpiQkvRopeHF:
            return (a.q_heads + a.kv_heads) * (a.head_dim / 2) + a.m[2].rows / 2;
        default:
            return a.m[0].rows;
    }
}

}  // namespace kc
