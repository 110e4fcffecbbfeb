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
//
// Contexts up to 2048 tokens take the cluster kernel instead: the (at most 8)
// chunk CTAs of one (batch, kv head) form a thread-block cluster, keep their
// partial (max, sum, acc) in shared memory and combine them through
// distributed shared memory after a cluster barrier -- no global partials,
// no atomic ticket, no extra L2 round trips on the critical path.
#include <atomic>
#include <cstdlib>

#include "kc_common.cuh"
#include "kc_launch.h"

namespace kc {

constexpr int kHeadDim = 128;
constexpr int kGqaThreads = 256;
constexpr int kGqaMaxChunk = 256;
constexpr int kGqaMinChunk = 64;
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

// The KV length of sequence b (one length for all, or one per sequence),
// clamped to [0, stride]; the split kernel flags a length out of range.
__device__ __forceinline__ int gqa_kv_len(const GqaArgs& a, int b) {
    const int kv_len = a.kv_len_dev != nullptr ? a.kv_len_dev[a.kv_len_per_batch ? b : 0] : a.kv_len;
    return kv_len < 1 ? 0 : kv_len > a.stride ? a.stride : kv_len;
}
// Splits that hold tokens of a sequence of kv_len tokens: ceil(kv_len / chunk),
// at least 1 (an empty length still has split 0 write an empty partial).  Only
// these run past their first lines, write partials and take a ticket.
__device__ __forceinline__ int gqa_live_splits(const GqaArgs& a, int kv_len) {
    const int s = (kv_len + a.chunk - 1) / a.chunk;
    return s < 1 ? 1 : s > a.nsplit ? a.nsplit : s;
}

// Combine the live partials of the G heads of one (batch, kv head).  Lane
// s of a warp owns split s (mod 32) for the max and the softmax weights; the
// weights are then broadcast so every lane accumulates its 4 dims over all
// splits with independent (batched) loads.
template <int DT, int G>
__device__ void gqa_combine_group(const GqaArgs& a, int b, int kvh) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int live = gqa_live_splits(a, gqa_kv_len(a, b));
    for (int h = warp; h < G; h += kGqaThreads / 32) {
        const int qh = kvh * G + h;
        const float* base = a.partials + (static_cast<int64_t>(b) * a.q_heads + qh) * a.nsplit * kPartialStride;
        float m = -INFINITY;
        for (int s = lane; s < live; s += 32) m = fmaxf(m, __ldcg(base + s * kPartialStride));
        m = warp_max(m);
        float l = 0.0F;
        float acc[4] = {0.0F, 0.0F, 0.0F, 0.0F};
        for (int s0 = 0; s0 < live; s0 += 32) {
            const int s = s0 + lane;
            float w = 0.0F;
            if (s < live) {
                const float ms = __ldcg(base + s * kPartialStride);
                if (ms != -INFINITY) {
                    w = exp2f(ms - m);
                    l += w * __ldcg(base + s * kPartialStride + 1);
                }
            }
            const int cnt = min(32, live - s0);
#pragma unroll 4
            for (int i = 0; i < cnt; ++i) {
                const float wi = __shfl_sync(0xffffffffu, w, i);
                // partials are 130 floats apart, so acc (offset 2) is only 8-byte aligned
                const float* p = base + (s0 + i) * kPartialStride + 2;
                const float2 v0 = __ldcg(reinterpret_cast<const float2*>(p) + 2 * lane);
                const float2 v1 = __ldcg(reinterpret_cast<const float2*>(p) + 2 * lane + 1);
                acc[0] = fmaf(wi, v0.x, acc[0]);
                acc[1] = fmaf(wi, v0.y, acc[1]);
                acc[2] = fmaf(wi, v1.x, acc[2]);
                acc[3] = fmaf(wi, v1.y, acc[3]);
            }
        }
        l = warp_sum(l);
        const float inv = l > 0.0F ? 1.0F / l : 0.0F;
        const int64_t o = (static_cast<int64_t>(b) * a.q_heads + qh) * kHeadDim + 4 * lane;
#pragma unroll
        for (int i = 0; i < 4; ++i) store_elem<DT>(a.out, o + i, acc[i] * inv);
    }
}

// One CTA per (batch, kv head, chunk).  Thread 0 stages the chunk's K rows
// and V rows (token-contiguous, so each is ONE bulk copy of n * 256 bytes)
// into shared memory on two mbarriers; scores start as soon as K lands while
// V is still in flight.  Dynamic shared memory: 2 * chunk * 256 bytes.
template <int DT, int G>
__global__ void __launch_bounds__(kGqaThreads) gqa_split_kernel(const GqaArgs a) {
    constexpr int LPH = 32 / G;          // lanes per head in the score phase
    constexpr int DPL = kHeadDim / LPH;  // dims per lane in the score phase
    __shared__ __align__(16) float s_s[G][kGqaMaxChunk];
    __shared__ float ml_s[G][2];
    __shared__ int last_s;
    __shared__ __align__(8) uint64_t kv_bar[2];
    extern __shared__ __align__(16) uint8_t kv_rows[];

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    pdl_launch_dependents();
    pdl_wait_on_producer();

    const int b = blockIdx.x / a.kv_heads;
    const int kvh = blockIdx.x - b * a.kv_heads;
    const int split = blockIdx.y;

    const int kv_raw = a.kv_len_dev != nullptr ? a.kv_len_dev[a.kv_len_per_batch ? b : 0] : a.kv_len;
    if ((kv_raw < 1 || kv_raw > a.stride) && a.err != nullptr && tid == 0 && split == 0) atomicOr(a.err, 4);
    const int kv_len = gqa_kv_len(a, b);
    // splits past the sequence's last token leave at once (a whole CTA: the
    // length is the same for every thread); the combine reads live ones only
    const int live = gqa_live_splits(a, kv_len);
    if (split >= live) return;
    if (tid == 0) {
        mbar_init(&kv_bar[0], 1);
        mbar_init(&kv_bar[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    const int t0 = split * a.chunk;
    int n = kv_len - t0;
    n = n < 0 ? 0 : (n > a.chunk ? a.chunk : n);

    const int64_t kv_base = (static_cast<int64_t>(a.kv_shared ? 0 : b) * a.kv_heads + kvh) * a.stride * kHeadDim;
    const uint16_t* ks = reinterpret_cast<const uint16_t*>(kv_rows);
    const uint16_t* vs = ks + static_cast<int64_t>(a.chunk) * kHeadDim;
    if (tid == 0 && n > 0) {
        const uint32_t bytes = static_cast<uint32_t>(n) * kHeadDim * 2;
        const int64_t row0 = kv_base + static_cast<int64_t>(t0) * kHeadDim;
        mbar_arrive_expect_tx(&kv_bar[0], bytes);
        bulk_g2s(const_cast<uint16_t*>(ks), static_cast<const uint16_t*>(a.kcache) + row0, bytes, &kv_bar[0]);
        mbar_arrive_expect_tx(&kv_bar[1], bytes);
        bulk_g2s(const_cast<uint16_t*>(vs), static_cast<const uint16_t*>(a.vcache) + row0, bytes, &kv_bar[1]);
    }
    // A wait that runs out records bit 16, waits again (bounded, a few times)
    // for the copy still in flight, and leaves the chunk empty.
    // The retries give a late copy time to land before the CTA can exit, so
    // no bulk copy still writes into this CTA's shared memory after it ends.
    auto wait_rows = [&](uint64_t* bar) {
        if (n == 0 || mbar_wait_bounded(bar, 0)) return;
        if (a.err != nullptr) atomicOr(a.err, 16);
        for (int retry = 0; retry < 8 && !mbar_wait_bounded(bar, 0); ++retry) {
        }
        n = 0;
    };

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
        wait_rows(&kv_bar[0]);
        for (int j = warp; j < n; j += kGqaThreads / 32) {
            const int64_t koff = static_cast<int64_t>(j) * kHeadDim + part * DPL;
            float dot = 0.0F;
            if constexpr (DPL >= 8) {
#pragma unroll
                for (int i = 0; i < DPL; i += 8) {
                    float kv[8];
                    load_vec8<DT>(ks, koff + i, kv);
#pragma unroll
                    for (int e = 0; e < 8; ++e) dot = fmaf(qv[i + e], kv[e], dot);
                }
            } else {
                float kv[4];
                load_vec4<DT>(ks, koff, kv);
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
    wait_rows(&kv_bar[1]);
    __syncthreads();

    // ---- P.V: warp h accumulates head h, lane owns dims 4*lane..4*lane+3 ----
    for (int h = warp; h < G; h += kGqaThreads / 32) {
        float acc[4] = {0.0F, 0.0F, 0.0F, 0.0F};
#pragma unroll 4
        for (int j = 0; j < n; ++j) {
            float v[4];
            load_vec4<DT>(vs, static_cast<int64_t>(j) * kHeadDim + 4 * lane, v);
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
        const int last = ticket == live - 1;
        if (last) atomicExch(ctr, 0);  // self-reset for the next launch / graph replay
        last_s = last;
    }
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    gqa_combine_group<DT, G>(a, b, kvh);
}

// ---------------------------------------------------------------------------
// Cluster kernel: grid (batch * kv_heads, S), cluster (1, S, 1), S <= 8.
//
//   * every thread j < n issues the bulk copy of K row j and V row j into
//     shared rows of 272 bytes (256 + 16 padding), so the mma fragment loads
//     below hit 32 distinct banks;
//   * scores = q . K^T on the tensor core (mma.m16n8k16, heads in rows 0..G-1,
//     8 tokens per n-tile, fp32 accumulate, exact bf16/f16 products);
//   * P.V on the tensor core with P split into hi + lo halves of the input
//     type (P = hi + lo to ~16 significant bits), so the product keeps fp32
//     level accuracy while V stays in its storage type; V fragments come from
//     ldmatrix.trans of the padded rows;
//   * each CTA writes (max, sum, acc) into the cluster leader's (rank 0)
//     shared memory, then every CTA of the cluster meets at a closing cluster
//     barrier (arrive.release / wait.acquire); after it the leader combines
//     and stores.  Only the leader's shared memory is written remotely, and
//     no CTA leaves before every remote store into it has completed: the
//     leader cannot exit while a peer still writes into its shared memory.
//     Every CTA reaches the closing barrier (no data-dependent wait precedes
//     it), so it needs no time limit.
constexpr int kGqaClusterThreads = 512;
constexpr int kGqaClusterWarps = kGqaClusterThreads / 32;
constexpr int kGqaMaxCluster = 8;
constexpr int kRowPad = kHeadDim * 2 + 16;  // padded shared row: 272 bytes

template <int DT>
__device__ __forceinline__ void mma_16816_dt(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                             uint32_t b1) {
    if constexpr (DT == kBF16) {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%0, %1, %2, %3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    } else {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%0, %1, %2, %3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
}
// two fp32 -> packed pair of the storage type (round to nearest even)
template <int DT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    if constexpr (DT == kBF16)
        return static_cast<uint32_t>(f32_to_bf16_bits(lo)) | (static_cast<uint32_t>(f32_to_bf16_bits(hi)) << 16);
    else
        return static_cast<uint32_t>(f32_to_f16_bits(lo)) | (static_cast<uint32_t>(f32_to_f16_bits(hi)) << 16);
}
template <int DT>
__device__ __forceinline__ float round_dt(float v) {
    if constexpr (DT == kBF16) return round_bf16(v);
    else return f16_bits_to_f32(f32_to_f16_bits(v));
}
// P pair (p0, p1) -> hi pair and lo pair (p = hi + lo)
template <int DT>
__device__ __forceinline__ void split_pair(float p0, float p1, uint32_t& hi, uint32_t& lo) {
    const float h0 = round_dt<DT>(p0), h1 = round_dt<DT>(p1);
    hi = pack2<DT>(h0, h1);
    lo = pack2<DT>(p0 - h0, p1 - h1);
}
__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t& r0, uint32_t& r1, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
template <int DT, int G>
__global__ void __launch_bounds__(kGqaClusterThreads) gqa_cluster_kernel(const GqaArgs a) {
    __shared__ __align__(16) float s_s[2][8][kGqaMaxChunk];  // score halves (dims 0-63, 64-127); then P in [0]
    __shared__ __align__(8) float gat_ml[kGqaMaxCluster][G][2];  // leader: gathered (max, sum)
    __shared__ float ml_s[G][2];
    extern __shared__ __align__(16) uint8_t kv_rows[];

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int S = a.nsplit;
    const int split = blockIdx.y;  // == rank in the cluster
    // announce this CTA (it has started, so its shared memory exists) to the
    // cluster; the matching wait comes right before the first remote access
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    pdl_launch_dependents();
    pdl_wait_on_producer();

    const int b = blockIdx.x / a.kv_heads;
    const int kvh = blockIdx.x - b * a.kv_heads;
    const int t0 = split * a.chunk;
    const int64_t kv_base = (static_cast<int64_t>(a.kv_shared ? 0 : b) * a.kv_heads + kvh) * a.stride * kHeadDim;
    uint8_t* ks = kv_rows;
    uint8_t* vs = kv_rows + static_cast<size_t>(a.chunk) * kRowPad;
    // leader: gathered partial accumulators [rank][head][dim], after the rows
    // (same offset in every CTA of the launch, so mapa finds the leader's copy)
    float* gat_acc = reinterpret_cast<float*>(kv_rows + 2 * static_cast<size_t>(a.chunk) * kRowPad);
    // rows this CTA may read: the chunk, clipped to the cache's row extent;
    // with per-sequence lengths (batched decode, where most sequences are far
    // shorter than the cache) also clipped to that sequence's length, at the
    // price of one dependent load before the K/V loads
    int row_end = a.stride;
    if (a.kv_len_per_batch && a.kv_len_dev != nullptr) row_end = min(row_end, max(0, a.kv_len_dev[b]));
    const int avail = min(a.chunk, max(0, row_end - t0));

    // ---- one global round trip: q fragments, the device length, and every
    // K/V row of the chunk (16-byte loads, 16 per row, into padded rows)
    uint32_t qa[8][2];
    {
        const uint32_t* qw = static_cast<const uint32_t*>(a.q) +
                             ((static_cast<int64_t>(b) * a.q_heads + kvh * G + (g < G ? g : 0)) * kHeadDim) / 2;
#pragma unroll
        for (int s8 = 0; s8 < 8; ++s8) {
            qa[s8][0] = g < G ? qw[8 * s8 + t] : 0u;
            qa[s8][1] = g < G ? qw[8 * s8 + t + 4] : 0u;
        }
    }
    int kv_len = a.kv_len_dev != nullptr ? a.kv_len_dev[a.kv_len_per_batch ? b : 0] : a.kv_len;
    {
        const uint4* kg = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.kcache) + kv_base +
                                                         static_cast<int64_t>(t0) * kHeadDim);
        const uint4* vg = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.vcache) + kv_base +
                                                         static_cast<int64_t>(t0) * kHeadDim);
        const int nvec = avail * (kHeadDim * 2 / 16);  // 16-byte pieces per cache
        for (int base = tid; base < nvec; base += 4 * kGqaClusterThreads) {
            uint4 kr[4], vr[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = base + u * kGqaClusterThreads;
                if (i < nvec) {
                    kr[u] = kg[i];
                    vr[u] = vg[i];
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = base + u * kGqaClusterThreads;
                if (i < nvec) {
                    const int row = i >> 4, piece = i & 15;
                    *reinterpret_cast<uint4*>(ks + row * kRowPad + 16 * piece) = kr[u];
                    *reinterpret_cast<uint4*>(vs + row * kRowPad + 16 * piece) = vr[u];
                }
            }
        }
    }
    if (kv_len < 1 || kv_len > a.stride) {
        if (a.err != nullptr && tid == 0) atomicOr(a.err, 4);
        kv_len = kv_len < 1 ? 0 : a.stride;
    }
    int n = kv_len - t0;
    n = n < 0 ? 0 : (n > a.chunk ? a.chunk : n);
    const int n16 = (n + 15) & ~15;
    // V rows n..n16-1 take part in the last P.V k-step with P = 0: make them
    // finite (they hold stale cache rows or nothing at all); the barrier orders
    // the row stores above before these
    __syncthreads();
    for (int i = tid; i < (n16 - n) * 16; i += kGqaClusterThreads)
        *reinterpret_cast<uint4*>(vs + (n + (i >> 4)) * kRowPad + 16 * (i & 15)) = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();

    // ---- scores: unit (n-tile of 8 tokens, dim half) per warp; four mma
    // k-steps on two independent accumulators
    const float qscale = a.scale * kLog2e;
    for (int unit = warp; unit < (n16 >> 3) * 2; unit += kGqaClusterWarps) {
        const int nt = unit >> 1, half = unit & 1;
        float c0[4] = {0.0F, 0.0F, 0.0F, 0.0F}, c1[4] = {0.0F, 0.0F, 0.0F, 0.0F};
        const uint8_t* krow = ks + (nt * 8 + g) * kRowPad + 4 * t + 128 * half;
#pragma unroll
        for (int s4 = 0; s4 < 4; s4 += 2) {
            // q fragments of k-steps 4*half + s4 and + 1 (selects keep qa in registers)
            const uint32_t qA0 = half ? qa[4 + s4][0] : qa[s4][0], qA1 = half ? qa[4 + s4][1] : qa[s4][1];
            const uint32_t qB0 = half ? qa[5 + s4][0] : qa[s4 + 1][0], qB1 = half ? qa[5 + s4][1] : qa[s4 + 1][1];
            mma_16816_dt<DT>(c0, qA0, 0u, qA1, 0u, *reinterpret_cast<const uint32_t*>(krow + 32 * s4),
                             *reinterpret_cast<const uint32_t*>(krow + 32 * s4 + 16));
            mma_16816_dt<DT>(c1, qB0, 0u, qB1, 0u, *reinterpret_cast<const uint32_t*>(krow + 32 * s4 + 32),
                             *reinterpret_cast<const uint32_t*>(krow + 32 * s4 + 48));
        }
        if (g < G) {
            *reinterpret_cast<float2*>(&s_s[half][g][nt * 8 + 2 * t]) =
                make_float2((c0[0] + c1[0]) * qscale, (c0[1] + c1[1]) * qscale);
        }
    }
    __syncthreads();

    // ---- per-head chunk softmax (log2 domain); probabilities zero past n
    for (int h = warp; h < G; h += kGqaClusterWarps) {
        float m = -INFINITY;
        for (int j = lane; j < n; j += 32) m = fmaxf(m, s_s[0][h][j] + s_s[1][h][j]);
        m = warp_max(m);
        float l = 0.0F;
        for (int j = lane; j < n16; j += 32) {
            const float p = j < n ? exp2f(s_s[0][h][j] + s_s[1][h][j] - m) : 0.0F;
            s_s[0][h][j] = p;
            l += p;
        }
        l = warp_sum(l);
        if (lane == 0) {
            ml_s[h][0] = n > 0 ? m : -INFINITY;
            ml_s[h][1] = l;
        }
    }
    __syncthreads();

    // ---- P.V: warp w owns dims 8w..8w+7; k-steps of 16 tokens alternate
    // between two accumulators
    float o0[4] = {0.0F, 0.0F, 0.0F, 0.0F}, o1[4] = {0.0F, 0.0F, 0.0F, 0.0F};
    {
        const uint32_t vbase = smem_u32(vs) + static_cast<uint32_t>((lane & 15) * kRowPad + 16 * warp);
        const float* prow = &s_s[0][g < G ? g : 0][2 * t];
        const int nk = n16 >> 4;
        for (int kk = 0; kk < nk; kk += 2) {
            // k-steps kk (accumulator 0) and kk + 1 (accumulator 1, if present)
            const bool two = kk + 1 < nk;
            uint32_t b0, b1, b2 = 0u, b3 = 0u;
            ldmatrix_x2_trans(b0, b1, vbase + static_cast<uint32_t>(kk * 16 * kRowPad));
            if (two) ldmatrix_x2_trans(b2, b3, vbase + static_cast<uint32_t>((kk + 1) * 16 * kRowPad));
            float2 pa = make_float2(0.0F, 0.0F), pb = pa, pc = pa, pd = pa;
            if (g < G) {
                pa = *reinterpret_cast<const float2*>(prow + kk * 16);
                pb = *reinterpret_cast<const float2*>(prow + kk * 16 + 8);
                if (two) {
                    pc = *reinterpret_cast<const float2*>(prow + kk * 16 + 16);
                    pd = *reinterpret_cast<const float2*>(prow + kk * 16 + 24);
                }
            }
            uint32_t ah0, al0, ah2, al2, ch0, cl0, ch2, cl2;
            split_pair<DT>(pa.x, pa.y, ah0, al0);
            split_pair<DT>(pb.x, pb.y, ah2, al2);
            split_pair<DT>(pc.x, pc.y, ch0, cl0);
            split_pair<DT>(pd.x, pd.y, ch2, cl2);
            mma_16816_dt<DT>(o0, ah0, 0u, ah2, 0u, b0, b1);
            if (two) mma_16816_dt<DT>(o1, ch0, 0u, ch2, 0u, b2, b3);
            mma_16816_dt<DT>(o0, al0, 0u, al2, 0u, b0, b1);
            if (two) mma_16816_dt<DT>(o1, cl0, 0u, cl2, 0u, b2, b3);
        }
    }

    // ---- push (acc, max, sum) into the leader's gather slot [split]
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (g < G) {
        const uint32_t dst = mapa_shared(smem_u32(gat_acc + (split * G + g) * kHeadDim + 8 * warp + 2 * t), 0);
        asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(dst), "f"(o0[0] + o1[0]), "f"(o0[1] + o1[1])
                     : "memory");
    }
    if (tid < G) {
        const uint32_t dst = mapa_shared(smem_u32(&gat_ml[split][tid][0]), 0);
        asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(dst), "f"(ml_s[tid][0]), "f"(ml_s[tid][1])
                     : "memory");
    }
    // closing rendezvous: the release orders this CTA's remote stores before
    // its arrival, the acquire makes every peer's stores visible to the leader
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (split != 0) return;

    // ---- leader: combine the S partials (loops unrolled over the cluster bound)
    for (int u = tid; u < G * kHeadDim; u += kGqaClusterThreads) {
        const int h = u / kHeadDim, d = u - h * kHeadDim;
        float mr[kGqaMaxCluster], lr[kGqaMaxCluster], ar[kGqaMaxCluster];
        float m = -INFINITY;
#pragma unroll
        for (int r = 0; r < kGqaMaxCluster; ++r) {
            mr[r] = -INFINITY;
            lr[r] = 0.0F;
            ar[r] = 0.0F;
            if (r < S) {
                const float2 ml = *reinterpret_cast<const float2*>(&gat_ml[r][h][0]);
                mr[r] = ml.x;
                lr[r] = ml.y;
                ar[r] = gat_acc[(r * G + h) * kHeadDim + d];
            }
            m = fmaxf(m, mr[r]);
        }
        float l = 0.0F, acc = 0.0F;
#pragma unroll
        for (int r = 0; r < kGqaMaxCluster; ++r) {
            const float w = mr[r] == -INFINITY ? 0.0F : exp2f(mr[r] - m);
            l = fmaf(w, lr[r], l);
            acc = fmaf(w, ar[r], acc);
        }
        const float inv = l > 0.0F ? 1.0F / l : 0.0F;
        store_elem<DT>(a.out, (static_cast<int64_t>(b) * a.q_heads + kvh * G + h) * kHeadDim + d, acc * inv);
    }
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
    // a chunk is one bulk copy per cache: below 64 tokens the fixed per-CTA
    // latency dominates and the partials to combine grow
    if (c < kGqaMinChunk) c = kGqaMinChunk;
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
// KUDACUDA_GQA_SPLIT_ONLY=1 keeps every call on the split kernel (measurement).
bool cluster_gqa_enabled() {
    static const bool on = std::getenv("KUDACUDA_GQA_SPLIT_ONLY") == nullptr;
    return on;
}

// Cluster plan for extents up to 2048 tokens: S = min(8, ceil(extent / 64))
// CTAs of chunk = ceil(extent / S) rounded up to 16 tokens (<= 256).
bool gqa_cluster_plan(int extent, int* chunk, int* nsplit) {
    if (extent < 1 || extent > kGqaMaxCluster * kGqaMaxChunk) return false;
    int S = (extent + kGqaMinChunk - 1) / kGqaMinChunk;
    if (S > kGqaMaxCluster) S = kGqaMaxCluster;
    int c = (extent + S - 1) / S;
    c = ((c + 15) / 16) * 16;
    if (c > kGqaMaxChunk) return false;
    *chunk = c;
    *nsplit = (extent + c - 1) / c;
    return true;
}

template <int DT, int G>
cudaError_t gqa_cluster_launch(GqaArgs a, cudaStream_t s) {
    auto kernel = gqa_cluster_kernel<DT, G>;
    static std::atomic<bool> attr_set[64];
    const int dev = current_device_index();
    if (!attr_set[dev].load(std::memory_order_acquire)) {
        const cudaError_t st = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                    2 * kGqaMaxChunk * kRowPad + kGqaMaxCluster * G * kHeadDim * 4);
        if (st != cudaSuccess) return st;
        attr_set[dev].store(true, std::memory_order_release);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.batch * a.kv_heads, a.nsplit);
    cfg.blockDim = dim3(kGqaClusterThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(2) * a.chunk * kRowPad + kGqaMaxCluster * G * kHeadDim * 4;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = static_cast<unsigned>(a.nsplit);
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, a);
}

template <int DT, int G>
cudaError_t gqa_launch(const GqaArgs& a, cudaStream_t s) {
    // The fused-combine path (tickets given) may take the cluster kernel; the
    // explicit workspace path (separate combine, the workspace_v3 contract)
    // keeps its partials in the caller's workspace.
    if (a.counters != nullptr && !a.split_only && cluster_gqa_enabled()) {
        GqaArgs c = a;
        if (gqa_cluster_plan(a.kv_len_dev != nullptr ? a.stride : a.kv_len, &c.chunk, &c.nsplit))
            return gqa_cluster_launch<DT, G>(c, s);
    }
    const dim3 grid(a.batch * a.kv_heads, a.nsplit);
    auto kernel = gqa_split_kernel<DT, G>;
    static std::atomic<bool> attr_set[64];
    const int dev = current_device_index();
    if (!attr_set[dev].load(std::memory_order_acquire)) {
        const cudaError_t st = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                    2 * kGqaMaxChunk * kHeadDim * 2);
        if (st != cudaSuccess) return st;
        attr_set[dev].store(true, std::memory_order_release);
    }
    const size_t smem = static_cast<size_t>(2) * a.chunk * kHeadDim * 2;
    cudaError_t st = launch_pdl(kernel, grid, dim3(kGqaThreads), smem, s, a);
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

// ---------------------------------------------------------------------------
// Allocation-free scratch for gqa_decode_static_scratch: split-KV partials
// (at most kStaticGqaPartialFloats floats = 1 MiB, e.g. 16 query heads x 126
// splits x 130 floats) followed by at most kStaticGqaTickets tickets.  A
// file-scope __device__ array is zero-filled when the module loads; the
// tickets must start at zero and self-reset after every call, and the first
// call on each device zeroes them once more on the caller's stream.  Two calls
// that overlap in time (different streams, or graphs replayed concurrently)
// share this array and race; callers serialise them.
constexpr size_t kStaticGqaPartialFloats = 262144;
constexpr int kStaticGqaTickets = 1024;
__device__ __align__(256) float g_static_gqa_scratch[kStaticGqaPartialFloats + kStaticGqaTickets];

namespace {
// Per-device address of the scratch, looked up once (cudaGetSymbolAddress
// does not allocate; the first call on a device must come before any stream
// capture on it).
cudaError_t static_gqa_scratch(cudaStream_t s, float** partials, int** tickets) {
    static std::atomic<float*> cached[64];
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;  // one cached address per device ordinal 0..63
    float* base = cached[dev].load(std::memory_order_acquire);
    if (base == nullptr) {
        void* p = nullptr;
        cudaError_t st = cudaGetSymbolAddress(&p, g_static_gqa_scratch);
        if (st != cudaSuccess) return st;
        base = static_cast<float*>(p);
        st = cudaMemsetAsync(base + kStaticGqaPartialFloats, 0, kStaticGqaTickets * sizeof(int), s);
        if (st != cudaSuccess) return st;
        cached[dev].store(base, std::memory_order_release);
    }
    *partials = base;
    *tickets = reinterpret_cast<int*>(base + kStaticGqaPartialFloats);
    return cudaSuccess;
}
}  // namespace

bool gqa_static_fits(int batch, int q_heads, int kv_heads, int extent) {
    if (batch <= 0 || kv_heads <= 0 || q_heads <= 0 || extent <= 0) return false;
    if (static_cast<int64_t>(batch) * kv_heads > kStaticGqaTickets) return false;
    int chunk = 0, nsplit = 0;
    gqa_plan_splits(extent, batch, kv_heads, 0, &chunk, &nsplit);
    return gqa_partials_floats(batch, q_heads, nsplit, kHeadDim) <= kStaticGqaPartialFloats;
}

cudaError_t gqa_decode_static_scratch(GqaArgs a, int dt, cudaStream_t s) {
    if (a.batch <= 0 || a.kv_heads <= 0 || a.q_heads <= 0 || a.stride <= 0) return cudaErrorInvalidValue;
    const int extent = a.kv_len_dev != nullptr ? a.stride : a.kv_len;
    if (!gqa_static_fits(a.batch, a.q_heads, a.kv_heads, extent)) return cudaErrorInvalidValue;
    gqa_plan_splits(extent, a.batch, a.kv_heads, 0, &a.chunk, &a.nsplit);
    cudaError_t st = static_gqa_scratch(s, &a.partials, &a.counters);
    if (st != cudaSuccess) return st;
    a.split_only = 1;
    return gqa_decode(a, dt, s);
}

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
