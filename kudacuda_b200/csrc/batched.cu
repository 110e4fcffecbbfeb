// batched.cu -- batched decode (B independent sequences per step) on sm_100a:
// NF4 dequant-GEMMs on the 5th-generation tensor cores (tcgen05, accumulator in
// TMEM), plus the per-sequence epilogues, RMSNorm, embedding, lm_head argmax
// and state advance around them.
//
// The reference has no batched path (its GQA contract is batch 1,
// python/kudacuda_sidecar.py:145-153, and its projections run one token at a
// time); the arithmetic follows what Transformers does with bitsandbytes NF4
// weights for a batch: each weight is dequantised to bf16 (level * absmax in
// fp32, rounded once, kernels/common/nf4_device.cuh:29-40), the matmul runs in
// bf16 with fp32 accumulation, and every activation is rounded to bf16 at the
// same points as the batch-1 kernels.
//
// GEMM tiling: one CTA owns 128 weight rows (the MMA's M) x the padded batch N
// (16, 32 or 64) for a range of 64-element K blocks (split-K, so every op has
// enough CTAs).  Per block, 256 threads dequantise the 128 x 64 weight tile into
// shared memory in the canonical K-major no-swizzle UMMA layout (8-row x
// 16-byte core matrices; the two 8-element K halves 128 B apart, 8-row groups
// 256 B apart) and stage the activations' 64-element slice beside it; one
// thread issues four tcgen05.mma (K = 16 each) into a 128 x N fp32 TMEM
// accumulator and commits to an mbarrier.  Two stages: the dequant of block
// i + 1 overlaps the MMAs of block i, and each thread's weight loads for
// block i + 1 are in flight while it dequantises block i.  The accumulator is
// read with tcgen05.ld and written as fp32 split-K partials; small epilogue
// kernels sum the splits in a fixed order (deterministic) and finish each op.
#include <cuda_runtime.h>

#include <cstdint>

#include "kc_common.cuh"
#include "kc_launch.h"

namespace kc {
namespace {

constexpr int kTcThreads = 256;
constexpr int kTcM = 128;
constexpr int kBlockK = 64;
constexpr int kATileBytes = kTcM * kBlockK * 2;  // 16 KB of bf16 per stage

struct TcArgs {
    const uint8_t* packed;  // NF4 [rows][K/2] (weight_type 0) or bf16 [rows][K] (weight_type 1)
    const float* absmax;    // [rows][K/64] (NF4)
    const uint16_t* x;      // bf16 [n_pad][K], rows >= batch are zero
    float* partials;        // [ksplit][total_rows][n_pad]; this matrix's rows start at row_offset
    int rows, K, n_pad, ksplit, weight_type, row_offset, total_rows;
    int* err;
};

// Canonical K-major, no-swizzle UMMA layout of a (rows x 16) K step: element
// (r, k) at (r / 8) * 256 + (k / 8) * 128 + (r % 8) * 16 + (k % 8) * 2 bytes.
__device__ __forceinline__ uint32_t kmajor_chunk(int r, int half) {  // byte offset of the 8-element chunk
    return static_cast<uint32_t>((r >> 3) * 256 + half * 128 + (r & 7) * 16);
}
// Shared-memory matrix descriptor (sm_100): start >> 4, LBO >> 4 (K halves),
// SBO >> 4 (8-row groups), version 1, base offset 0, layout SWIZZLE_NONE.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(128u >> 4) << 16;
    d |= static_cast<uint64_t>(256u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    return d;
}
// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, both
// K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__device__ __forceinline__ uint32_t umma_idesc_bf16(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(kTcM >> 4) << 24);
}
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// bf16 pair (lo = element 2j, hi = element 2j + 1) of a dequantised NF4 byte;
// lut is the 16-level codebook in shared memory (16 words in 16 banks: a warp's
// lookups never conflict, unlike divergent constant-memory reads)
__device__ __forceinline__ uint32_t nf4_pair_bf16(const float* lut, uint32_t byte, float s) {
    const float e = lut[(byte >> 4) & 15u] * s;  // even element: high nibble
    const float o = lut[byte & 15u] * s;
    return static_cast<uint32_t>(f32_to_bf16_bits(e)) | (static_cast<uint32_t>(f32_to_bf16_bits(o)) << 16);
}

// One thread's share of a K block: 32 weights of one row (16 code bytes and
// the block's absmax for NF4, 64 bytes for bf16)
struct WLoad {
    uint4 v[4];
    float s;
};
__device__ __forceinline__ void load_weights(const TcArgs& a, bool row_ok, int grow, int nblk, int kb, int half,
                                             WLoad& w) {
    if (!row_ok) return;
    if (a.weight_type == 0) {
        w.v[0] = *reinterpret_cast<const uint4*>(a.packed + static_cast<int64_t>(grow) * (a.K / 2) + kb * 32 +
                                                 half * 16);
        w.s = a.absmax[static_cast<int64_t>(grow) * nblk + kb];
    } else {
        const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(a.packed) +
                                                          static_cast<int64_t>(grow) * a.K + kb * 64 + half * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) w.v[q] = src[q];
    }
}

__global__ void __launch_bounds__(kTcThreads) nf4_gemm_tc_kernel(const TcArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ __align__(8) uint64_t mma_bar[2];
    __shared__ uint32_t tmem_slot;
    __shared__ float lut[16];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid < 16) lut[tid] = kNf4Levels[tid];
    const int n = a.n_pad;
    const int bstage = n * kBlockK * 2;  // B bytes per stage
    uint8_t* const a_base = smem;
    uint8_t* const b_base = smem + 2 * kATileBytes;
    const int ncols = n <= 32 ? 32 : 64;  // TMEM columns: a power of two >= 32 covering N

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(ncols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        mbar_init(&mma_bar[0], 1);
        mbar_init(&mma_bar[1], 1);
        fence_mbar_init();
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_slot;

    const int tile = blockIdx.x, ks = blockIdx.y;
    const int nblk = a.K / kBlockK;
    const int kb0 = static_cast<int>(static_cast<int64_t>(ks) * nblk / a.ksplit);
    const int kb1 = static_cast<int>(static_cast<int64_t>(ks + 1) * nblk / a.ksplit);
    const int r = tid >> 1, half = tid & 1;  // dequant: row r of the tile, K half `half` of the block
    const int grow = tile * kTcM + r;
    const bool row_ok = grow < a.rows;
    const uint32_t idesc = umma_idesc_bf16(n);
    uint32_t phase0 = 0u, phase1 = 0u;
    bool ok = true;

    pdl_launch_dependents();
    pdl_wait_on_producer();
    WLoad cur, nxt;
#pragma unroll
    for (int q = 0; q < 4; ++q) cur.v[q] = nxt.v[q] = make_uint4(0u, 0u, 0u, 0u);
    cur.s = nxt.s = 0.F;
    if (kb0 < kb1) load_weights(a, row_ok, grow, nblk, kb0, half, cur);
    for (int kb = kb0, it = 0; kb < kb1; ++kb, ++it) {
        const int st = it & 1;
        if (kb + 1 < kb1) load_weights(a, row_ok, grow, nblk, kb + 1, half, nxt);  // in flight during this block
        if (it >= 2) {  // the MMAs that read this stage two blocks ago must be done
            uint32_t& ph = st ? phase1 : phase0;
            if (!mbar_wait_bounded(&mma_bar[st], ph)) ok = false;
            ph ^= 1u;
        }
        // ---- A: 32 weights of row r (K half `half`) -> bf16 into the canonical layout
        uint32_t w[16];
        if (a.weight_type == 0) {
            const uint32_t cw[4] = {cur.v[0].x, cur.v[0].y, cur.v[0].z, cur.v[0].w};
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int bb = 0; bb < 4; ++bb) w[q * 4 + bb] = nf4_pair_bf16(lut, (cw[q] >> (8 * bb)) & 0xFFu, cur.s);
        } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                w[4 * q] = cur.v[q].x;
                w[4 * q + 1] = cur.v[q].y;
                w[4 * q + 2] = cur.v[q].z;
                w[4 * q + 3] = cur.v[q].w;
            }
        }
        // elements [32 half, 32 half + 32): K steps 2 half and 2 half + 1, two 8-element chunks each
        uint8_t* const as = a_base + st * kATileBytes;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int kstep = 2 * half + (c >> 1), kh = c & 1;
            *reinterpret_cast<uint4*>(as + kstep * (kTcM * 32) + kmajor_chunk(r, kh)) =
                make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
        }
        // ---- B: the activations' 64-element slice, n rows
        uint8_t* const bs = b_base + st * bstage;
        for (int i = tid; i < n * 8; i += kTcThreads) {
            const int row = i >> 3, c = i & 7;  // chunk c of 8 elements
            const uint4 v = *reinterpret_cast<const uint4*>(a.x + static_cast<int64_t>(row) * a.K + kb * 64 + c * 8);
            *reinterpret_cast<uint4*>(bs + (c >> 1) * (n * 32) + kmajor_chunk(row, c & 1)) = v;
        }
        fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core (async proxy)
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const uint64_t da = umma_desc(smem_u32(as + s * (kTcM * 32)));
                const uint64_t db = umma_desc(smem_u32(bs + s * (n * 32)));
                umma_bf16(tmem, da, db, idesc, (it > 0 || s > 0) ? 1u : 0u);
            }
            umma_commit(&mma_bar[st]);
        }
        cur = nxt;
    }
    // ---- wait for the last MMAs, then read the 128 x n accumulator
    const int nit = kb1 - kb0;
    if (nit > 0) {
        const int st = (nit - 1) & 1;
        if (!mbar_wait_bounded(&mma_bar[st], st ? phase1 : phase0)) ok = false;
        if (nit >= 2) {  // the other stage's last commit is older and already complete
            if (!mbar_wait_bounded(&mma_bar[st ^ 1], st ? phase0 : phase1)) ok = false;
        }
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!ok && lane == 0 && a.err != nullptr) atomicOr(a.err, 16);
    // warp w reads TMEM lanes 32 (w % 4) .. + 31 (tile rows); the n columns go
    // in 16-column chunks, chunk c to warps 4 (c % 2) .. + 3 (n = 16: one chunk,
    // read by warps 0-3 alone)
    {
        const int lrow = 32 * (warp & 3) + lane;
        const int grow2 = tile * kTcM + lrow;
        for (int c0 = 16 * (warp >> 2); c0 < n; c0 += 32) {
            float v[16];
            const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + static_cast<uint32_t>(c0);
            tmem_ld16(taddr, v);
            if (grow2 < a.rows) {
                float* dst = a.partials + (static_cast<int64_t>(ks) * a.total_rows + a.row_offset + grow2) * n + c0;
                const bool any = nit > 0;
#pragma unroll
                for (int i = 0; i < 16; i += 4)
                    *reinterpret_cast<float4*>(dst + i) = any ? make_float4(v[i], v[i + 1], v[i + 2], v[i + 3])
                                                              : make_float4(0.F, 0.F, 0.F, 0.F);
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
    }
}

// ---- per-sequence staging and epilogues (sum of split-K partials in split order)
__device__ __forceinline__ float split_sum(const float* partials, int ksplit, int rows, int n_pad, int row, int b) {
    float v = 0.F;
    for (int k = 0; k < ksplit; ++k) v += partials[(static_cast<int64_t>(k) * rows + row) * n_pad + b];
    return v;
}

// out[b][:] = bf16(w * bf16(x[b] * rsqrt(mean(x[b]^2) + eps)))  (one CTA per sequence)
__global__ void __launch_bounds__(256) batch_rmsnorm_kernel(const uint16_t* x, const uint16_t* w, uint16_t* out,
                                                            int H, float eps) {
    __shared__ float red[8];
    pdl_launch_dependents();
    pdl_wait_on_producer();
    const int b = blockIdx.x, tid = threadIdx.x;
    const uint16_t* xb = x + static_cast<int64_t>(b) * H;
    float ss = 0.F;
    for (int i = tid; i < H; i += 256) {
        const float v = bf16_bits_to_f32(xb[i]);
        ss += v * v;
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.F;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float inv = 1.0F / sqrtf(tot / static_cast<float>(H) + eps);
    for (int i = tid; i < H; i += 256)
        out[static_cast<int64_t>(b) * H + i] =
            f32_to_bf16_bits(round_bf16(bf16_bits_to_f32(w[i]) * round_bf16(bf16_bits_to_f32(xb[i]) * inv)));
}

// bias + RoPE (Transformers' rotate_half with bf16 rounding) + K/V append at pos[b]
__global__ void __launch_bounds__(256) batch_qkv_epilogue_kernel(const BatchQkv a) {
    pdl_launch_dependents();
    pdl_wait_on_producer();
    const int hd = a.head_dim, half = hd / 2;
    const int rows = (a.q_heads + 2 * a.kv_heads) * hd;
    const int pairs = (a.q_heads + a.kv_heads) * half;  // RoPE pairs of q and k
    const int vrows = a.kv_heads * hd;
    const int per_b = pairs + vrows;
    const int64_t total = static_cast<int64_t>(a.batch) * per_b;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int b = static_cast<int>(idx / per_b), u = static_cast<int>(idx - static_cast<int64_t>(b) * per_b);
        const int pos = a.pos[b];
        if (pos < 0 || pos >= a.cap || pos >= a.max_pos) {
            if (a.err != nullptr) atomicOr(a.err, 2);
            continue;
        }
        if (u < pairs) {
            const bool isq = u < a.q_heads * half;
            const int uu = isq ? u : u - a.q_heads * half;
            const int head = uu / half, i = uu - head * half;
            const int base = (isq ? 0 : a.q_heads * hd) + head * hd;
            float y0 = round_bf16(split_sum(a.partials, a.ksplit, rows, a.n_pad, base + i, b));
            float y1 = round_bf16(split_sum(a.partials, a.ksplit, rows, a.n_pad, base + i + half, b));
            const uint16_t* bias = isq ? a.q_bias : a.k_bias;
            if (bias != nullptr) {
                y0 = round_bf16(y0 + bf16_bits_to_f32(bias[head * hd + i]));
                y1 = round_bf16(y1 + bf16_bits_to_f32(bias[head * hd + i + half]));
            }
            const float c = bf16_bits_to_f32(a.rope_cos[static_cast<int64_t>(pos) * half + i]);
            const float sn = bf16_bits_to_f32(a.rope_sin[static_cast<int64_t>(pos) * half + i]);
            const float lo = round_bf16(round_bf16(y0 * c) + round_bf16(-y1 * sn));
            const float hi = round_bf16(round_bf16(y1 * c) + round_bf16(y0 * sn));
            if (isq) {
                uint16_t* q = a.q_out + (static_cast<int64_t>(b) * a.q_heads + head) * hd;
                q[i] = f32_to_bf16_bits(lo);
                q[i + half] = f32_to_bf16_bits(hi);
            } else {
                uint16_t* kc = a.kcache + ((static_cast<int64_t>(b) * a.kv_heads + head) * a.cap + pos) * hd;
                kc[i] = f32_to_bf16_bits(lo);
                kc[i + half] = f32_to_bf16_bits(hi);
            }
        } else {
            const int vr = u - pairs, head = vr / hd, d = vr - head * hd;
            float y = round_bf16(split_sum(a.partials, a.ksplit, rows, a.n_pad, (a.q_heads + a.kv_heads) * hd + vr, b));
            if (a.v_bias != nullptr) y = round_bf16(y + bf16_bits_to_f32(a.v_bias[vr]));
            a.vcache[((static_cast<int64_t>(b) * a.kv_heads + head) * a.cap + pos) * hd + d] = f32_to_bf16_bits(y);
        }
    }
}

// x[b][r] = bf16(x[b][r] + bf16(sum))   (o_proj, down)
__global__ void __launch_bounds__(256) batch_residual_kernel(const float* partials, int ksplit, int rows, int n_pad,
                                                             int batch, uint16_t* x) {
    pdl_launch_dependents();
    pdl_wait_on_producer();
    const int64_t total = static_cast<int64_t>(batch) * rows;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int b = static_cast<int>(idx / rows), r = static_cast<int>(idx - static_cast<int64_t>(b) * rows);
        uint16_t* xp = x + static_cast<int64_t>(b) * rows + r;
        *xp = f32_to_bf16_bits(bf16_bits_to_f32(*xp) + round_bf16(split_sum(partials, ksplit, rows, n_pad, r, b)));
    }
}

// h[b][j] = bf16(bf16(silu(bf16 gate_j)) * bf16 up_j); rows = gate (inter) | up (inter)
__global__ void __launch_bounds__(256) batch_swiglu_kernel(const float* partials, int ksplit, int inter, int n_pad,
                                                           int batch, uint16_t* h) {
    pdl_launch_dependents();
    pdl_wait_on_producer();
    const int rows = 2 * inter;
    const int64_t total = static_cast<int64_t>(batch) * inter;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int b = static_cast<int>(idx / inter), j = static_cast<int>(idx - static_cast<int64_t>(b) * inter);
        const float g = round_bf16(split_sum(partials, ksplit, rows, n_pad, j, b));
        const float u = round_bf16(split_sum(partials, ksplit, rows, n_pad, inter + j, b));
        const float act = round_bf16(g / (1.0F + expf(-g)));
        h[static_cast<int64_t>(b) * inter + j] = f32_to_bf16_bits(act * u);
    }
}

// Per-sequence greedy argmax over bf16-rounded logits (lowest index on ties):
// stage 1 -- one (value, index) candidate per (CTA, sequence).  Lanes run over
// sequences (coalesced partial reads), warps over vocabulary rows.
constexpr int kArgCtas = 128;
__device__ __forceinline__ void arg_better(float& bv, int& bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}
__global__ void __launch_bounds__(256) batch_argmax_stage1(const float* partials, int ksplit, int vocab, int n_pad,
                                                           int batch, float* cand_v, int* cand_i) {
    __shared__ float sv[8][64];
    __shared__ int si[8][64];
    pdl_launch_dependents();
    pdl_wait_on_producer();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float bv[2] = {-INFINITY, -INFINITY};
    int bi[2] = {0x7fffffff, 0x7fffffff};
    for (int r = blockIdx.x * 8 + warp; r < vocab; r += kArgCtas * 8) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int b = lane + 32 * h;
            if (b < batch) arg_better(bv[h], bi[h], round_bf16(split_sum(partials, ksplit, vocab, n_pad, r, b)), r);
        }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        sv[warp][lane + 32 * h] = bv[h];
        si[warp][lane + 32 * h] = bi[h];
    }
    __syncthreads();
    if (threadIdx.x < batch) {
        const int b = threadIdx.x;
        float v = sv[0][b];
        int ix = si[0][b];
        for (int w = 1; w < 8; ++w) arg_better(v, ix, sv[w][b], si[w][b]);
        cand_v[b * kArgCtas + blockIdx.x] = v;
        cand_i[b * kArgCtas + blockIdx.x] = ix;
    }
}
// stage 2 -- one warp per sequence picks among the candidates; writes the
// token and advances that sequence's state {token, pos, kv_len, pad}
__global__ void __launch_bounds__(32) batch_argmax_stage2(const float* cand_v, const int* cand_i, int32_t* state,
                                                          int32_t* history, int history_len) {
    pdl_launch_dependents();
    pdl_wait_on_producer();
    const int b = blockIdx.x, lane = threadIdx.x;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = lane; c < kArgCtas; c += 32) arg_better(best, bi, cand_v[b * kArgCtas + c], cand_i[b * kArgCtas + c]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        arg_better(best, bi, ov, oi);
    }
    if (lane == 0) {
        int32_t* st = state + 4 * b;
        const int pos = st[1] + 1;
        st[0] = bi;
        st[1] = pos;
        st[2] = pos + 1;
        if (history != nullptr && pos < history_len) history[static_cast<int64_t>(b) * history_len + pos] = bi;
    }
}

// x[b][:] = embedding[state[b].token][:]
__global__ void __launch_bounds__(256) batch_embedding_kernel(const uint16_t* emb, const int32_t* state, uint16_t* x,
                                                              int H, int vocab, int* err) {
    pdl_launch_dependents();
    pdl_wait_on_producer();
    const int b = blockIdx.x;
    int tok = state[4 * b];
    if (tok < 0 || tok >= vocab) {
        if (err != nullptr && threadIdx.x == 0) atomicOr(err, 8);
        tok = 0;
    }
    for (int i = threadIdx.x; i < H / 8; i += 256)
        reinterpret_cast<uint4*>(x + static_cast<int64_t>(b) * H)[i] =
            reinterpret_cast<const uint4*>(emb + static_cast<int64_t>(tok) * H)[i];
}

// kv_len[b] = state[b].kv_len, pos[b] = state[b].pos  (the attention and RoPE views of the state)
__global__ void batch_state_views_kernel(const int32_t* state, int batch, int32_t* pos, int32_t* kv_len) {
    pdl_launch_dependents();
    pdl_wait_on_producer();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < batch) {
        pos[b] = state[4 * b + 1];
        kv_len[b] = state[4 * b + 2];
    }
}

int ew_grid(int64_t total) {
    const int64_t g = (total + 255) / 256;
    const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
    return static_cast<int>(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace

int batch_gemm_ksplit(int rows, int K) {
    const int mtiles = (rows + kTcM - 1) / kTcM;
    const int nblk = K / kBlockK;
    const int target = 2 * device_sm_count();
    int ks = (target + mtiles - 1) / mtiles;
    if (ks > nblk) ks = nblk;
    if (ks > 16) ks = 16;
    return ks < 1 ? 1 : ks;
}

cudaError_t batch_gemm(int weight_type, const void* weight, const float* absmax, int rows, int K, const uint16_t* x,
                       int n_pad, int ksplit, float* partials, int row_offset, int total_rows, int* err,
                       cudaStream_t s) {
    if (rows < 1 || K < kBlockK || K % kBlockK != 0 || !(n_pad == 16 || n_pad == 32 || n_pad == 64) || ksplit < 1 ||
        ksplit > K / kBlockK || row_offset < 0 || row_offset + rows > total_rows)
        return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(x) |
         reinterpret_cast<uintptr_t>(partials)) & 15u)
        return cudaErrorMisalignedAddress;
    TcArgs a;
    a.packed = static_cast<const uint8_t*>(weight);
    a.absmax = absmax;
    a.x = x;
    a.partials = partials;
    a.rows = rows;
    a.K = K;
    a.n_pad = n_pad;
    a.ksplit = ksplit;
    a.weight_type = weight_type;
    a.row_offset = row_offset;
    a.total_rows = total_rows;
    a.err = err;
    const int smem = 2 * kATileBytes + 2 * n_pad * kBlockK * 2;
    cudaError_t st = cudaFuncSetAttribute(nf4_gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (st != cudaSuccess) return st;
    return launch_pdl(nf4_gemm_tc_kernel, dim3((rows + kTcM - 1) / kTcM, ksplit), dim3(kTcThreads),
                      static_cast<size_t>(smem), s, a);
}

cudaError_t batch_rmsnorm(const uint16_t* x, const uint16_t* w, uint16_t* out, int batch, int H, float eps,
                          cudaStream_t s) {
    return launch_pdl(batch_rmsnorm_kernel, dim3(batch), dim3(256), 0, s, x, w, out, H, eps);
}

cudaError_t batch_qkv_epilogue(const BatchQkv& q, cudaStream_t s) {
    const int64_t total =
        static_cast<int64_t>(q.batch) * ((q.q_heads + q.kv_heads) * (q.head_dim / 2) + q.kv_heads * q.head_dim);
    return launch_pdl(batch_qkv_epilogue_kernel, dim3(ew_grid(total)), dim3(256), 0, s, q);
}

cudaError_t batch_residual(const float* partials, int ksplit, int rows, int n_pad, int batch, uint16_t* x,
                           cudaStream_t s) {
    return launch_pdl(batch_residual_kernel, dim3(ew_grid(static_cast<int64_t>(batch) * rows)), dim3(256), 0, s,
                      partials, ksplit, rows, n_pad, batch, x);
}

cudaError_t batch_swiglu(const float* partials, int ksplit, int inter, int n_pad, int batch, uint16_t* h,
                         cudaStream_t s) {
    return launch_pdl(batch_swiglu_kernel, dim3(ew_grid(static_cast<int64_t>(batch) * inter)), dim3(256), 0, s,
                      partials, ksplit, inter, n_pad, batch, h);
}

int batch_argmax_workspace_floats(int batch) { return 2 * batch * kArgCtas; }

cudaError_t batch_argmax_advance(const float* partials, int ksplit, int vocab, int n_pad, int batch, float* ws,
                                 int32_t* state, int32_t* history, int history_len, cudaStream_t s) {
    float* cv = ws;
    int* ci = reinterpret_cast<int*>(ws + batch * kArgCtas);
    cudaError_t st =
        launch_pdl(batch_argmax_stage1, dim3(kArgCtas), dim3(256), 0, s, partials, ksplit, vocab, n_pad, batch, cv, ci);
    if (st != cudaSuccess) return st;
    return launch_pdl(batch_argmax_stage2, dim3(batch), dim3(32), 0, s, static_cast<const float*>(cv),
                      static_cast<const int*>(ci), state, history, history_len);
}

cudaError_t batch_embedding(const uint16_t* emb, const int32_t* state, uint16_t* x, int batch, int H, int vocab,
                            int* err, cudaStream_t s) {
    return launch_pdl(batch_embedding_kernel, dim3(batch), dim3(256), 0, s, emb, state, x, H, vocab, err);
}

cudaError_t batch_state_views(const int32_t* state, int batch, int32_t* pos, int32_t* kv_len, cudaStream_t s) {
    return launch_pdl(batch_state_views_kernel, dim3((batch + 63) / 64), dim3(64), 0, s, state, batch, pos, kv_len);
}

}  // namespace kc
