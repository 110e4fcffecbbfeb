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
// enough CTAs).  A producer warp brings each block's weights and the
// activations' block (2D TMA, 128-byte swizzle) into a shared ring; for NF4,
// eight warps dequantise the 128 x 64 tile into tensor memory (tcgen05.st,
// one row per lane, four tiles in flight beside the accumulator); one thread
// issues four tcgen05.mma (K = 16 each, A from tensor memory or shared
// memory, B from shared memory) into a 128 x N fp32 TMEM accumulator and
// commits to an mbarrier that frees the ring stage and the tile.  bf16 weights (the tied lm_head) skip the
// dequant: TMA places them in the swizzled layout the tensor core reads.  NF4
// comes either in the bitsandbytes layout or re-tiled at load into one
// contiguous record per tile and block (one bulk copy).  The accumulator is
// read with tcgen05.ld and written as fp32 split-K partials; the epilogue
// kernels sum the splits in a fixed order (deterministic) and finish each op.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "kc_common.cuh"
#include "kc_launch.h"
#include "kc_tma.h"

namespace kc {
namespace {

constexpr int kTcM = 128;
constexpr int kBlockK = 64;
constexpr int kATileBytes = kTcM * kBlockK * 2;  // 16 KB of bf16 per stage

struct TcArgs {
    const uint8_t* packed;  // NF4 [rows][K/2] (weight_type 0), bf16 [rows][K] (1), re-tiled records (2)
    const float* absmax;    // [rows][K/64] (weight_type 0)
    const uint16_t* x;      // bf16 [n_pad][K], rows >= batch are zero
    float* partials;        // [ksplit][total_rows][n_pad]; this matrix's rows start at row_offset
    int rows, K, n_pad, ksplit, weight_type, row_offset, total_rows;
    int* err;
    BatchEpilogue e;        // fused epilogue (mode 0: none, the partials are the output)
};

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
// A operand from tensor memory (one row per lane, two bf16 per 32-bit column)
__device__ __forceinline__ void umma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                             uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
          "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
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

// ---- tensor memory access, bounded mbarrier waits, TMA
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// try_wait with a suspend-time hint of 1 us: wakes when the phase completes,
// gives up after ~2^17 tries (~0.1 s) or as soon as another thread of the CTA
// has given up (abort flag), so a protocol error ends the kernel instead of
// hanging the GPU.
__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                         bool honour_abort = true) {
    for (uint32_t i = 0; i < (1u << 17); ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity), "r"(1000u)
            : "memory");
        if (ok) return true;
        if (honour_abort && *abort_flag) return false;
    }
    *abort_flag = 1;
    return false;
}
// Shared-memory matrix descriptor, K-major with the 128-byte swizzle (the
// layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B): rows 128 B apart, 8-row
// groups 1024 B apart (SBO), LBO unused (1), version 1, layout type 2.  A K
// step of 16 bf16 advances the start address by 32 B inside the swizzle atom.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
}
// ---- the tensor-core GEMM
// One CTA = one 128-row tile x one split of K, ten warps:
//   warp 0   TMA producer: per 64-element K block, the weight tile (NF4 codes
//            128 x 32 B row-major, or bf16 128 x 128 B swizzled) and the
//            activations' block (n x 128 B swizzled) into a ring stage;
//   warp 1   MMA issuer: four tcgen05.mma (K = 16) per block into the TMEM
//            accumulator, tcgen05.commit frees the ring stage and the A tile;
//   warps 2-9 (NF4) dequantise: thread (row r, half h) reads its 16 code
//            bytes, looks up byte -> (level[hi], level[lo]) in a pair table
//            (16 lane-indexed copies: conflict-free 64-bit lookups), scales by
//            the block's absmax in fp32, rounds to bf16 and stores the 32
//            weights to its TMEM lane (warp w owns lanes 32 (w % 4) ..); then
//            they read the accumulator out.
// Barriers: raw_full (TMA bytes landed), raw_empty (the MMAs of that stage's
// block are done: frees the stage for the producer and, for the dequant warps,
// the A tile that block read), a_full (256 dequant arrivals), done; one
// tcgen05.commit per block.
constexpr int kGThreads = 320;
constexpr int kPairCopies = 16;
constexpr int kPairTableBytes = 256 * kPairCopies * 8;  // 32 KB
constexpr int kMaxA = 4;
constexpr int kTmemAcc = 64;    // accumulator columns (N <= 64)
constexpr int kTmemATile = 32;  // one dequantised A tile: 128 lanes x 64 bf16 = 32 columns
constexpr int kMaxRaw = 6;  // ring stages: bounds the barrier arrays (raw_stages() <= this, checked on launch)

// Weight forms: WT 0 NF4 in the bitsandbytes layout (codes by 2D TMA, absmax
// by the dequant threads from global memory), WT 1 bf16, WT 2 NF4 re-tiled at
// load (one contiguous 4,608-byte record per 128-row tile and K block: the
// codes [128][32 B] then the absmax [128] fp32, fetched by one bulk copy).
constexpr int kRetileRecord = kTcM * 32 + kTcM * 4;  // 4608

template <int WT>
struct GemmSmem {
    static constexpr bool kNf4 = WT != 1;
    static __host__ __device__ int raw_stages(int n) { return kNf4 ? (n == 64 ? 5 : 6) : 4; }
    // NF4: four dequantised A tiles in tensor memory (after the accumulator)
    static __host__ __device__ int a_stages(int n) { return kNf4 ? kMaxA : 0; }
    static __host__ __device__ int w_bytes() { return WT == 0 ? kTcM * 32 : WT == 1 ? kATileBytes : kRetileRecord; }
    // stage = [weights][activations] (WT 0, 1) or [activations][record] (WT 2); the swizzled tiles start
    // on 1024-byte boundaries
    static __host__ __device__ int b_off(int n) { return WT == 2 ? 0 : w_bytes(); }
    static __host__ __device__ int w_off(int n) { return WT == 2 ? n * kBlockK * 2 : 0; }
    static __host__ __device__ int raw_bytes(int n) { return (w_bytes() + n * kBlockK * 2 + 1023) / 1024 * 1024; }
    static __host__ __device__ int fixed_bytes(int n) { return kNf4 ? kPairTableBytes : 0; }
    // NF4 CTAs take 256 TMEM columns, so at most two may share an SM: at least 80 KB keeps a third off
    static __host__ __device__ int bytes(int n) {
        const int b = 1024 + fixed_bytes(n) + raw_stages(n) * raw_bytes(n);
        return kNf4 && b < 80 * 1024 ? 80 * 1024 : b;
    }
};

// Fused epilogue, run by the last CTA of a tile to finish its split (ticket):
// the tile's split partials summed in split order (the order the separate
// epilogue kernels use, so the results are the same bits) into t[row][b],
// then the op's finish for every sequence.
__device__ void fused_epilogue(const TcArgs& a, int tile, float* t) {
    const BatchEpilogue& e = a.e;
    const int n = a.n_pad, np1 = n + 1, tid = threadIdx.x;
    const int nr = min(kTcM, a.rows - tile * kTcM);
    const int64_t kstride = static_cast<int64_t>(a.total_rows) * n;
    for (int idx = tid; idx < nr * n; idx += kGThreads) {
        const int r = idx / n, b = idx - r * n;
        const float* p = a.partials + static_cast<int64_t>(a.row_offset + tile * kTcM + r) * n + b;
        float v = 0.F;
        for (int k = 0; k < a.ksplit; ++k) v += __ldcg(p + k * kstride);
        t[r * np1 + b] = v;
    }
    __syncthreads();
    if (e.mode == 1) {  // x[b][row] = bf16(x + bf16(sum))
        for (int idx = tid; idx < e.batch * nr; idx += kGThreads) {
            const int b = idx / nr, r = idx - b * nr;
            uint16_t* xp = e.resid + static_cast<int64_t>(b) * a.rows + tile * kTcM + r;
            *xp = f32_to_bf16_bits(bf16_bits_to_f32(*xp) + round_bf16(t[r * np1 + b]));
        }
    } else if (e.mode == 2) {  // tile = 64 gate rows | the same 64 up rows
        const int half = kTcM / 2, inter = a.rows / 2;
        for (int idx = tid; idx < e.batch * half; idx += kGThreads) {
            const int b = idx / half, i = idx - b * half;
            const float g = round_bf16(t[i * np1 + b]);
            const float u = round_bf16(t[(half + i) * np1 + b]);
            const float act = round_bf16(g / (1.0F + expf(-g)));
            e.hout[static_cast<int64_t>(b) * inter + tile * half + i] = f32_to_bf16_bits(act * u);
        }
    } else if (e.mode == 3) {  // tile = one head of q | k | v (head_dim 128)
        const int hd = kTcM, half = hd / 2, head = tile;
        const bool isq = head < e.q_heads, isk = !isq && head < e.q_heads + e.kv_heads;
        if (isq || isk) {
            const uint16_t* bias = isq ? e.q_bias : e.k_bias;
            const int hh = isq ? head : head - e.q_heads;
            for (int idx = tid; idx < e.batch * half; idx += kGThreads) {
                const int b = idx / half, i = idx - b * half;
                const int pos = e.pos[b];
                if (pos < 0 || pos >= e.cap || pos >= e.max_pos) {
                    if (a.err != nullptr) atomicOr(a.err, 2);
                    continue;
                }
                float y0 = round_bf16(t[i * np1 + b]), y1 = round_bf16(t[(i + half) * np1 + b]);
                if (bias != nullptr) {
                    y0 = round_bf16(y0 + bf16_bits_to_f32(bias[hh * hd + i]));
                    y1 = round_bf16(y1 + bf16_bits_to_f32(bias[hh * hd + i + half]));
                }
                const float c = bf16_bits_to_f32(e.rope_cos[static_cast<int64_t>(pos) * half + i]);
                const float sn = bf16_bits_to_f32(e.rope_sin[static_cast<int64_t>(pos) * half + i]);
                const float lo = round_bf16(round_bf16(y0 * c) + round_bf16(-y1 * sn));
                const float hi = round_bf16(round_bf16(y1 * c) + round_bf16(y0 * sn));
                uint16_t* dst = isq ? e.q_out + (static_cast<int64_t>(b) * e.q_heads + hh) * hd
                                    : e.kcache + ((static_cast<int64_t>(e.shared_cache ? 0 : b) * e.kv_heads + hh) * e.cap + pos) * hd;
                dst[i] = f32_to_bf16_bits(lo);
                dst[i + half] = f32_to_bf16_bits(hi);
            }
        } else {
            const int hh = head - e.q_heads - e.kv_heads;
            for (int idx = tid; idx < e.batch * hd; idx += kGThreads) {
                const int b = idx / hd, d = idx - b * hd;
                const int pos = e.pos[b];
                if (pos < 0 || pos >= e.cap || pos >= e.max_pos) {
                    if (a.err != nullptr) atomicOr(a.err, 2);
                    continue;
                }
                float y = round_bf16(t[d * np1 + b]);
                if (e.v_bias != nullptr) y = round_bf16(y + bf16_bits_to_f32(e.v_bias[hh * hd + d]));
                e.vcache[((static_cast<int64_t>(e.shared_cache ? 0 : b) * e.kv_heads + hh) * e.cap + pos) * hd + d] =
                    f32_to_bf16_bits(y);
            }
        }
    }
}

template <int WT>
__global__ void __launch_bounds__(kGThreads, 2) gemm_tc_kernel(const __grid_constant__ CUtensorMap map_w,
                                                            const __grid_constant__ CUtensorMap map_x,
                                                            const TcArgs a) {
    using G = GemmSmem<WT>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t raw_full[kMaxRaw], raw_empty[kMaxRaw], a_full[kMaxA], done_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n = a.n_pad;
    const int R = G::raw_stages(n);
    const int SA = G::a_stages(n);
    const int rb = G::raw_bytes(n);
    // 1024-byte aligned base (the swizzled tiles need it)
    uint8_t* const base = smem_raw + (((smem_u32(smem_raw) + 1023u) & ~1023u) - smem_u32(smem_raw));
    uint8_t* const table = base;                          // NF4: pair table
    uint8_t* const raw = base + G::fixed_bytes(n);        // ring of R stages
    // TMEM: the 128 x N fp32 accumulator at column 0; NF4 adds SA bf16 A tiles from column 64
    const int ncols = G::kNf4 ? 256 : (n <= 32 ? 32 : 64);

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(ncols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 32) {
        for (int i = 0; i < kMaxRaw; ++i) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], 1);
        }
        for (int i = 0; i < kMaxA; ++i) mbar_init(&a_full[i], 256);
        mbar_init(&done_bar, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    if (G::kNf4 && warp >= 2) {  // entry e, copy c: (level[e >> 4], level[e & 15]) at (e * 16 + c) * 8
        for (int i = tid - 64; i < 256 * kPairCopies; i += 256) {
            const int e = i / kPairCopies;
            *reinterpret_cast<float2*>(table + i * 8) = make_float2(kNf4Levels[e >> 4], kNf4Levels[e & 15]);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_slot;

    const int tile = blockIdx.x, ks = blockIdx.y;
    const int nblk = a.K / kBlockK;
    const int kb0 = static_cast<int>(static_cast<int64_t>(ks) * nblk / a.ksplit);
    const int kb1 = static_cast<int>(static_cast<int64_t>(ks + 1) * nblk / a.ksplit);
    const int nit = kb1 - kb0;
    volatile int* const abort_p = &abort_flag;

    pdl_launch_dependents();
    pdl_wait_on_producer();
    if (warp == 0) {
        if (lane == 0) {
            const uint32_t tx = static_cast<uint32_t>(G::w_bytes() + n * kBlockK * 2);
            for (int it = 0; it < nit; ++it) {
                const int j = it % R, m = it / R;
                if (m >= 1) bar_wait(&raw_empty[j], (m - 1) & 1, abort_p);
                uint8_t* stg = raw + j * rb;
                mbar_arrive_expect_tx(&raw_full[j], tx);
                if (WT == 2)
                    bulk_g2s(stg + G::w_off(n),
                             a.packed + (static_cast<int64_t>(tile) * nblk + kb0 + it) * kRetileRecord,
                             kRetileRecord, &raw_full[j]);
                else
                    tma_load_2d(stg, &map_w, WT == 0 ? (kb0 + it) * 32 : (kb0 + it) * kBlockK, tile * kTcM,
                                &raw_full[j]);
                tma_load_2d(stg + G::b_off(n), &map_x, (kb0 + it) * kBlockK, 0, &raw_full[j]);
            }
            // every copy has landed before the CTA may exit (normally already true)
            for (int j = 0; j < R; ++j) {
                const int issued = (nit - j + R - 1) / R;  // loads that went to stage j
                if (issued > 0) bar_wait(&raw_full[j], (issued - 1) & 1, abort_p, false);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_bf16(n);
            for (int it = 0; it < nit; ++it) {
                const int j = it % R, s = G::kNf4 ? it % SA : 0;
                bar_wait(&raw_full[j], (it / R) & 1, abort_p);
                if (G::kNf4) bar_wait(&a_full[s], (it / SA) & 1, abort_p);
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                uint8_t* const stg = raw + j * rb;
                const uint32_t sb = smem_u32(stg + G::b_off(n));
                if (G::kNf4) {  // K step k = columns 8k .. 8k + 7 of the A tile
                    const uint32_t ta = tmem + static_cast<uint32_t>(kTmemAcc + s * kTmemATile);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        umma_bf16_ts(tmem, ta + 8 * k, umma_desc_sw128(sb + 32 * k), idesc,
                                     (it > 0 || k > 0) ? 1u : 0u);
                } else {
                    const uint32_t sa = smem_u32(stg);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        umma_bf16(tmem, umma_desc_sw128(sa + 32 * k), umma_desc_sw128(sb + 32 * k), idesc,
                                  (it > 0 || k > 0) ? 1u : 0u);
                }
                // raw_empty[j] frees the ring stage and, for the dequant warps,
                // the A tile this block read
                umma_commit(&raw_empty[j]);
            }
            umma_commit(&done_bar);
        }
    } else if (G::kNf4) {
        // ---- dequantise: warp w owns TMEM lanes 32 (w % 4) .. + 31 (tile rows) and
        // half (w - 2) / 4 of each block's 64 elements; thread = one row
        const int dq = tid - 64, h = dq >> 7, r = 32 * (warp & 3) + lane;
        const int grow = tile * kTcM + r;
        const bool row_ok = grow < a.rows;
        const float* arow = WT == 0 ? a.absmax + static_cast<int64_t>(row_ok ? grow : 0) * nblk : nullptr;
        const bool vec4 = WT == 0 && (nblk & 3) == 0;
        const uint32_t tl_u32 = smem_u32(table) + static_cast<uint32_t>((lane & (kPairCopies - 1)) * 8);
        const uint32_t raw_u32 = smem_u32(raw);
        const uint32_t t_row = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
        float4 cur4 = make_float4(0.F, 0.F, 0.F, 0.F), nxt4 = cur4;
        int cur_g = -1;
        for (int it = 0; it < nit; ++it) {
            const int kb = kb0 + it, j = it % R, s = it % SA;
            // absmax: float4 of four blocks, the next four prefetched (scalar when rows are not 16-B aligned)
            float sc = 0.F;
            if (WT == 0 && row_ok) {
                if (vec4) {
                    const int g = kb >> 2;
                    if (g != cur_g) {
                        cur4 = cur_g < 0 ? *reinterpret_cast<const float4*>(arow + 4 * g) : nxt4;
                        cur_g = g;
                        if (4 * (g + 1) < kb1) nxt4 = *reinterpret_cast<const float4*>(arow + 4 * (g + 1));
                    }
                    const int q = kb & 3;
                    sc = q == 0 ? cur4.x : q == 1 ? cur4.y : q == 2 ? cur4.z : cur4.w;
                } else {
                    sc = arow[kb];
                }
            }
            bar_wait(&raw_full[j], (it / R) & 1, abort_p);
            uint32_t cw[4];
            const uint32_t rec = raw_u32 + static_cast<uint32_t>(j * rb + G::w_off(n));
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(cw[0]), "=r"(cw[1]), "=r"(cw[2]), "=r"(cw[3])
                         : "r"(rec + static_cast<uint32_t>(r * 32 + h * 16)));
            if (WT == 2) asm volatile("ld.shared.f32 %0, [%1];" : "=f"(sc) : "r"(rec + static_cast<uint32_t>(kTcM * 32 + r * 4)));
            // the MMAs of block it - SA (the last reader of A tile s) are done: they
            // committed to the ring stage of that block.  No phase of that barrier
            // can pass unseen: its next phase needs block it - SA + R's MMAs, which
            // need this thread's dequant of a later block (R >= SA).
            if (it >= SA) {
                const int ib = it - SA;
                bar_wait(&raw_empty[ib % R], (ib / R) & 1, abort_p);
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint64_t ss = (static_cast<uint64_t>(__float_as_uint(sc)) << 32) | __float_as_uint(sc);
            uint32_t o[16];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t w = cw[q];
                // byte bb of w -> table offset byte * 128 (+ this lane's copy)
                const uint32_t off[4] = {(w << 7) & 0x7F80u, (w >> 1) & 0x7F80u, (w >> 9) & 0x7F80u,
                                         (w >> 17) & 0x7F80u};
#pragma unroll
                for (int bb = 0; bb < 4; ++bb) {
                    // (level[hi], level[lo]) * absmax in fp32, rounded to a bf16 pair (even element low)
                    asm("{\n\t.reg .b64 t;\n\t.reg .f32 lo, hi;\n\t"
                        "ld.shared.b64 t, [%1];\n\t"
                        "mul.rn.f32x2 t, t, %2;\n\t"
                        "mov.b64 {lo, hi}, t;\n\t"
                        "cvt.rn.bf16x2.f32 %0, hi, lo;\n\t}"
                        : "=r"(o[4 * q + bb])
                        : "r"(tl_u32 + off[bb]), "l"(ss));
                }
            }
            // columns 16 h .. 16 h + 15 of A tile s, this warp's 32 lanes
            tmem_st16(t_row + static_cast<uint32_t>(kTmemAcc + s * kTmemATile + 16 * h), o);
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            bar_arrive(&a_full[s]);
        }
    }
    // ---- epilogue: warps 2-9 read the 128 x n accumulator (warp w: TMEM lanes 32 (w % 4) ..)
    if (warp >= 2) {
        bar_wait(&done_bar, 0u, abort_p, false);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int lrow = 32 * (warp & 3) + lane;
        const int grow2 = tile * kTcM + lrow;
        for (int c0 = 16 * ((warp - 2) >> 2); c0 < n; c0 += 32) {
            float v[16];
            tmem_ld16(tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + static_cast<uint32_t>(c0), v);
            if (grow2 < a.rows) {
                float* dst = a.partials + (static_cast<int64_t>(ks) * a.total_rows + a.row_offset + grow2) * n + c0;
#pragma unroll
                for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            }
        }
    }
    if (tid == 0 && *abort_p && a.err != nullptr) atomicOr(a.err, 16);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    if (G::kNf4 && a.e.mode != 0) {
        // the last CTA of this tile's splits finishes the op (the tickets reset
        // themselves); its shared memory (table, A tiles: 64 KB, all reads and
        // MMAs done) stages the sums
        __shared__ int last_split;
        __threadfence();  // this thread's partial stores before the ticket
        __syncthreads();
        if (tid == 0) last_split = atomicAdd(a.e.tickets + tile, 1) == a.ksplit - 1 ? 1 : 0;
        __syncthreads();
        if (last_split) {
            __threadfence();
            fused_epilogue(a, tile, reinterpret_cast<float*>(table));
            if (tid == 0) a.e.tickets[tile] = 0;
        }
    }
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

// out[b][:] = bf16(w * bf16(x[b] * rsqrt(mean(x[b]^2) + eps)))  (one CTA per sequence).
// hidden % 8 == 0: each thread holds up to kNormVec uint4 of x (8 bf16 each) and
// the matching weights in registers, so the row is read once.
constexpr int kNormVec = 4;  // hidden <= 256 * 8 * kNormVec in one pass
__global__ void __launch_bounds__(256) batch_rmsnorm_kernel(const uint16_t* x, const uint16_t* w, uint16_t* out,
                                                            int H, float eps) {
    __shared__ float red[8];
    pdl_launch_dependents();
    pdl_wait_on_producer();
    const int b = blockIdx.x, tid = threadIdx.x;
    const uint4* xb = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(b) * H);
    const uint4* wb = reinterpret_cast<const uint4*>(w);
    const int nv = H >> 3;
    uint4 xv[kNormVec], wv[kNormVec];
#pragma unroll
    for (int u = 0; u < kNormVec; ++u) {
        const int i = tid + 256 * u;
        xv[u] = i < nv ? xb[i] : make_uint4(0, 0, 0, 0);
        wv[u] = i < nv ? __ldg(wb + i) : make_uint4(0, 0, 0, 0);
    }
    float ss = 0.F;
#pragma unroll
    for (int u = 0; u < kNormVec; ++u) {
        const uint32_t* e = reinterpret_cast<const uint32_t*>(&xv[u]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float lo = bf16_bits_to_f32(static_cast<uint16_t>(e[j] & 0xFFFFu));
            const float hi = bf16_bits_to_f32(static_cast<uint16_t>(e[j] >> 16));
            ss += lo * lo;
            ss += hi * hi;
        }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.F;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float inv = 1.0F / sqrtf(tot / static_cast<float>(H) + eps);
    uint4* ob = reinterpret_cast<uint4*>(out + static_cast<int64_t>(b) * H);
#pragma unroll
    for (int u = 0; u < kNormVec; ++u) {
        const int i = tid + 256 * u;
        if (i < nv) {
            const uint32_t* e = reinterpret_cast<const uint32_t*>(&xv[u]);
            const uint32_t* g = reinterpret_cast<const uint32_t*>(&wv[u]);
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float lo = round_bf16(bf16_bits_to_f32(static_cast<uint16_t>(g[j] & 0xFFFFu)) *
                                            round_bf16(bf16_bits_to_f32(static_cast<uint16_t>(e[j] & 0xFFFFu)) * inv));
                const float hi = round_bf16(bf16_bits_to_f32(static_cast<uint16_t>(g[j] >> 16)) *
                                            round_bf16(bf16_bits_to_f32(static_cast<uint16_t>(e[j] >> 16)) * inv));
                o[j] = static_cast<uint32_t>(f32_to_bf16_bits(lo)) | (static_cast<uint32_t>(f32_to_bf16_bits(hi)) << 16);
            }
            ob[i] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

// The epilogues work on tiles of consecutive rows x the padded batch: the
// split-K partial sums [split][row][n_pad] (16-byte aligned, as the GEMM
// writes them) are read row-contiguous as float4 (coalesced), summed in split
// order (deterministic), staged in shared memory, and written per sequence
// along the row.  A tile is epi_rows(n_pad) rows = 1,024 floats, one float4 per
// thread, so every load a thread needs can be in flight at once.
constexpr int kEpiFloats = 1024;
__host__ __device__ __forceinline__ int epi_rows(int n_pad) { return kEpiFloats / n_pad; }

// Sums of rows row0[u] .. row0[u] + nrows - 1 (nrows <= PER * kEpiFloats / n_pad)
// of NT tiles into t[u][row * (n_pad + 1) + b]; each thread owns PER float4s
// of a tile.  The loads of up to 16 (one float4 a thread) or 8 / (NT * PER)
// splits are issued together (at most 64 registers of loads in flight);
// the adds run in split order from +0, the order of every other reader of the
// partials (the fused epilogue, split_sum).
template <int NT, int PER>
__device__ __forceinline__ void sum_tiles(const float* partials, int ksplit, int rows, int n_pad, const int (&row0)[NT],
                                          int nrows, float* const (&t)[NT]) {
    constexpr int kB = NT * PER == 1 ? 16 : 8 / (NT * PER) > 0 ? 8 / (NT * PER) : 1;
    const int q = n_pad >> 2;  // float4s per row
    const int total = nrows * q;
    const int64_t kstride4 = static_cast<int64_t>(rows) * q;
    const float4* p[NT][PER];
    bool active[PER];
#pragma unroll
    for (int v = 0; v < PER; ++v) {
        const int f = threadIdx.x + 256 * v;
        active[v] = f < total;
#pragma unroll
        for (int u = 0; u < NT; ++u)
            p[u][v] = reinterpret_cast<const float4*>(partials) + static_cast<int64_t>(row0[u]) * q + (active[v] ? f : 0);
    }
    float4 acc[NT][PER];
#pragma unroll
    for (int u = 0; u < NT; ++u)
#pragma unroll
        for (int v = 0; v < PER; ++v) acc[u][v] = make_float4(0.F, 0.F, 0.F, 0.F);
    for (int k0 = 0; k0 < ksplit; k0 += kB) {
        float4 r[NT][PER][kB];
#pragma unroll
        for (int j = 0; j < kB; ++j)
#pragma unroll
            for (int v = 0; v < PER; ++v) {
                const bool ok = active[v] && k0 + j < ksplit;
#pragma unroll
                for (int u = 0; u < NT; ++u)
                    r[u][v][j] = ok ? __ldg(p[u][v] + static_cast<int64_t>(k0 + j) * kstride4)
                                    : make_float4(0.F, 0.F, 0.F, 0.F);
            }
#pragma unroll
        for (int j = 0; j < kB; ++j) {
            if (k0 + j < ksplit) {
#pragma unroll
                for (int u = 0; u < NT; ++u)
#pragma unroll
                    for (int v = 0; v < PER; ++v) {
                        acc[u][v].x += r[u][v][j].x;
                        acc[u][v].y += r[u][v][j].y;
                        acc[u][v].z += r[u][v][j].z;
                        acc[u][v].w += r[u][v][j].w;
                    }
            }
        }
    }
#pragma unroll
    for (int v = 0; v < PER; ++v) {
        if (active[v]) {
            const int f = threadIdx.x + 256 * v, i = f / q, c = 4 * (f - i * q);
#pragma unroll
            for (int u = 0; u < NT; ++u) {
                float* d = t[u] + i * (n_pad + 1) + c;
                d[0] = acc[u][v].x;
                d[1] = acc[u][v].y;
                d[2] = acc[u][v].z;
                d[3] = acc[u][v].w;
            }
        }
    }
}

// bias + RoPE (Transformers' rotate_half with bf16 rounding) + K/V append at
// pos[b]; one CTA per (head of q | k | v, group of kQkvPairs dimension pairs
// (i, i + head_dim / 2))
constexpr int kQkvPairs = 16;
__global__ void __launch_bounds__(256) batch_qkv_epilogue_kernel(const BatchQkv a) {
    __shared__ float tq[2 * kQkvPairs * 65];  // [2 x kQkvPairs rows][n_pad + 1]
    pdl_launch_dependents();
    pdl_wait_on_producer();
    const int hd = a.head_dim, half = hd / 2, np1 = a.n_pad + 1;
    const int rows = (a.q_heads + 2 * a.kv_heads) * hd;
    const int groups = half / kQkvPairs;
    const int head = blockIdx.x / groups;  // 0 .. q_heads + 2 kv_heads - 1
    const int i0 = (blockIdx.x - head * groups) * kQkvPairs;
    {
        const int r0[2] = {head * hd + i0, head * hd + half + i0};
        float* const tt[2] = {tq, tq + kQkvPairs * np1};
        sum_tiles<2, 1>(a.partials, a.ksplit, rows, a.n_pad, r0, kQkvPairs, tt);
    }
    __syncthreads();
    const bool isq = head < a.q_heads, isk = !isq && head < a.q_heads + a.kv_heads;
    if (isq || isk) {
        const uint16_t* bias = isq ? a.q_bias : a.k_bias;
        const int hh = isq ? head : head - a.q_heads;
        for (int e = threadIdx.x; e < a.batch * kQkvPairs; e += blockDim.x) {
            const int b = e / kQkvPairs, ii = e - b * kQkvPairs, i = i0 + ii;
            const int pos = a.pos[b];
            if (pos < 0 || pos >= a.cap || pos >= a.max_pos) {
                if (a.err != nullptr) atomicOr(a.err, 2);
                continue;
            }
            float y0 = round_bf16(tq[ii * np1 + b]), y1 = round_bf16(tq[(kQkvPairs + ii) * np1 + b]);
            if (bias != nullptr) {
                y0 = round_bf16(y0 + bf16_bits_to_f32(bias[hh * hd + i]));
                y1 = round_bf16(y1 + bf16_bits_to_f32(bias[hh * hd + i + half]));
            }
            const float c = bf16_bits_to_f32(a.rope_cos[static_cast<int64_t>(pos) * half + i]);
            const float sn = bf16_bits_to_f32(a.rope_sin[static_cast<int64_t>(pos) * half + i]);
            const float lo = round_bf16(round_bf16(y0 * c) + round_bf16(-y1 * sn));
            const float hi = round_bf16(round_bf16(y1 * c) + round_bf16(y0 * sn));
            uint16_t* dst = isq ? a.q_out + (static_cast<int64_t>(b) * a.q_heads + hh) * hd
                                : a.kcache + ((static_cast<int64_t>(a.shared_cache ? 0 : b) * a.kv_heads + hh) * a.cap + pos) * hd;
            dst[i] = f32_to_bf16_bits(lo);
            dst[i + half] = f32_to_bf16_bits(hi);
        }
    } else {
        const int hh = head - a.q_heads - a.kv_heads;
        for (int e = threadIdx.x; e < a.batch * 2 * kQkvPairs; e += blockDim.x) {
            const int b = e / (2 * kQkvPairs), q = e - b * 2 * kQkvPairs;
            const int d = q < kQkvPairs ? i0 + q : half + i0 + q - kQkvPairs;
            const int pos = a.pos[b];
            if (pos < 0 || pos >= a.cap || pos >= a.max_pos) {
                if (a.err != nullptr) atomicOr(a.err, 2);
                continue;
            }
            float y = round_bf16(tq[q * np1 + b]);
            if (a.v_bias != nullptr) y = round_bf16(y + bf16_bits_to_f32(a.v_bias[hh * hd + d]));
            a.vcache[((static_cast<int64_t>(a.shared_cache ? 0 : b) * a.kv_heads + hh) * a.cap + pos) * hd + d] =
                f32_to_bf16_bits(y);
        }
    }
}

// x[b][r] = bf16(x[b][r] + bf16(sum))   (o_proj, down); epi_rows(n_pad) rows per CTA.
// Each thread reads its (at most four) residual elements before any store.
__global__ void __launch_bounds__(256) batch_residual_kernel(const float* partials, int ksplit, int rows, int n_pad,
                                                             int batch, uint16_t* x) {
    __shared__ float t[kEpiFloats + 64];  // [er][n_pad + 1]
    pdl_launch_dependents();
    pdl_wait_on_producer();
    const int er = epi_rows(n_pad);
    const int row0 = blockIdx.x * er;
    const int nr = min(er, rows - row0);
    {
        const int r0[1] = {row0};
        float* const tt[1] = {t};
        sum_tiles<1, 1>(partials, ksplit, rows, n_pad, r0, nr, tt);
    }
    __syncthreads();
    constexpr int kPer = kEpiFloats / 256;  // batch * er <= n_pad * er = 1,024 elements
    uint16_t* xp[kPer];
    uint16_t xv[kPer];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
        const int e = threadIdx.x + 256 * u, b = e / er, i = e - b * er;
        xp[u] = (b < batch && i < nr) ? x + static_cast<int64_t>(b) * rows + row0 + i : nullptr;
        xv[u] = xp[u] != nullptr ? *xp[u] : static_cast<uint16_t>(0);
    }
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
        const int e = threadIdx.x + 256 * u, b = e / er, i = e - b * er;
        if (xp[u] != nullptr) *xp[u] = f32_to_bf16_bits(bf16_bits_to_f32(xv[u]) + round_bf16(t[i * (n_pad + 1) + b]));
    }
}

// h[b][j] = bf16(bf16(silu(bf16 gate_j)) * bf16 up_j); rows = gate (inter) | up (inter);
// 2 * epi_rows(n_pad) j per CTA (grid within one wave at n_pad 64), gate and up
// tiles summed in one pass
constexpr int kSwigluPer = 2;
__global__ void __launch_bounds__(256) batch_swiglu_kernel(const float* partials, int ksplit, int inter, int n_pad,
                                                           int batch, uint16_t* h) {
    __shared__ float tg[kSwigluPer * kEpiFloats + 128], tu[kSwigluPer * kEpiFloats + 128];
    pdl_launch_dependents();
    pdl_wait_on_producer();
    const int er = kSwigluPer * epi_rows(n_pad);
    const int j0 = blockIdx.x * er;
    const int nr = min(er, inter - j0);
    {
        const int r0[2] = {j0, inter + j0};
        float* const tt[2] = {tg, tu};
        sum_tiles<2, kSwigluPer>(partials, ksplit, 2 * inter, n_pad, r0, nr, tt);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < batch * er; e += blockDim.x) {
        const int b = e / er, i = e - b * er;
        if (i < nr) {
            const float g = round_bf16(tg[i * (n_pad + 1) + b]);
            const float u = round_bf16(tu[i * (n_pad + 1) + b]);
            const float act = round_bf16(g / (1.0F + expf(-g)));
            h[static_cast<int64_t>(b) * inter + j0 + i] = f32_to_bf16_bits(act * u);
        }
    }
}

// Per-sequence greedy argmax over bf16-rounded logits (lowest index on ties):
// stage 1 -- one (value, index) candidate per (CTA, sequence).  Lanes run over
// sequences (coalesced partial reads), warps over vocabulary rows.
constexpr int kArgCtas = 512;
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
    // rows r, r + stride, ... of this warp, four at a time (independent loads; the
    // candidates are merged in row order, so ties keep the lowest index)
    const int stride = kArgCtas * 8;
    for (int r = blockIdx.x * 8 + warp; r < vocab; r += 4 * stride) {
        float v[4][2];
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int rr = r + u * stride, b = lane + 32 * h;
                v[u][h] = (rr < vocab && b < batch) ? round_bf16(split_sum(partials, ksplit, vocab, n_pad, rr, b))
                                                    : -INFINITY;
            }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int h = 0; h < 2; ++h)
                if (r + u * stride < vocab && lane + 32 * h < batch) arg_better(bv[h], bi[h], v[u][h], r + u * stride);
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

// ---- tensor parallelism: the pieces around the NCCL collectives
// out[r][b] = sum over splits of partials[s][r][b] (split order), every column
// of the padded batch; the rank's row-parallel partial before the allreduce
__global__ void __launch_bounds__(256) batch_split_sum_kernel(const float* partials, int ksplit, int64_t n, float* out) {
    pdl_launch_dependents();
    pdl_wait_on_producer();
    for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < n;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float v = 0.F;
        for (int k = 0; k < ksplit; ++k) v += __ldg(partials + k * n + e);
        out[e] = v;
    }
}
// stage 2 of the argmax, vocabulary-parallel form: the rank's best (value, global
// index) per sequence as an int32 pair {float bits, index}
__global__ void __launch_bounds__(32) batch_argmax_pairs_stage2(const float* cand_v, const int* cand_i, int index_base,
                                                                int32_t* pairs) {
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
        pairs[2 * b] = __float_as_int(best);
        pairs[2 * b + 1] = bi + index_base;
    }
}
// per sequence: the lowest-index maximum over the ranks' pairs gathered as
// [world][batch][2]; then the state advance of batch_argmax_stage2
__global__ void batch_select_advance_kernel(const int32_t* gathered, int world, int batch, int32_t* state,
                                            int32_t* history, int history_len) {
    pdl_launch_dependents();
    pdl_wait_on_producer();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= batch) return;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int r = 0; r < world; ++r) {
        const int32_t* p = gathered + (static_cast<int64_t>(r) * batch + b) * 2;
        arg_better(best, bi, __int_as_float(p[0]), p[1]);
    }
    int32_t* st = state + 4 * b;
    const int pos = st[1] + 1;
    st[0] = bi;
    st[1] = pos;
    st[2] = pos + 1;
    if (history != nullptr && pos < history_len) history[static_cast<int64_t>(b) * history_len + pos] = bi;
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


}  // namespace

namespace {
// re-tile: record (t, kb) = codes of rows 128 t .. + 127, bytes 32 kb .. + 31,
// then their absmax of block kb; rows past the matrix are zero
__global__ void batch_retile_kernel(const uint8_t* packed, const float* absmax, int rows, int K, uint8_t* out) {
    const int nblk = K / kBlockK;
    const int tiles = (rows + kTcM - 1) / kTcM;
    const int64_t units = static_cast<int64_t>(tiles) * nblk * (kRetileRecord / 16);
    for (int64_t u = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; u < units;
         u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t recn = u / (kRetileRecord / 16);
        const int w = static_cast<int>(u - recn * (kRetileRecord / 16));  // 16-byte unit inside the record
        const int t = static_cast<int>(recn / nblk), kb = static_cast<int>(recn - static_cast<int64_t>(t) * nblk);
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (w < kTcM * 2) {  // codes: row w / 2, half w % 2
            const int row = t * kTcM + (w >> 1);
            if (row < rows)
                v = *reinterpret_cast<const uint4*>(packed + static_cast<int64_t>(row) * (K / 2) + kb * 32 + (w & 1) * 16);
        } else {  // absmax of four rows
            const int r0 = t * kTcM + (w - kTcM * 2) * 4;
            float f[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) f[i] = r0 + i < rows ? absmax[static_cast<int64_t>(r0 + i) * nblk + kb] : 0.F;
            v = make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
        }
        *reinterpret_cast<uint4*>(out + recn * kRetileRecord + w * 16) = v;
    }
}
}  // namespace

int64_t batch_retile_bytes(int rows, int K) {
    return static_cast<int64_t>((rows + kTcM - 1) / kTcM) * (K / kBlockK) * kRetileRecord;
}

cudaError_t batch_retile(const uint8_t* packed, const float* absmax, int rows, int K, uint8_t* out, cudaStream_t s) {
    if (rows < 1 || K < kBlockK || K % kBlockK != 0) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(packed) | reinterpret_cast<uintptr_t>(out)) & 15u) return cudaErrorMisalignedAddress;
    const int64_t units = batch_retile_bytes(rows, K) / 16;
    const int64_t g = (units + 255) / 256;
    const int grid = static_cast<int>(g < 4096 ? g : 4096);
    return launch_pdl(batch_retile_kernel, dim3(grid), dim3(256), 0, s, packed, absmax, rows, K, out);
}

int batch_gemm_ksplit(int rows, int K) {
    // A CTA's time is set by its K blocks (a per-block load -> dequant -> MMA
    // chain) plus a fixed start-up and drain, and two CTAs share an SM, so
    // what counts is how full the last wave of CTAs is.  The smallest split
    // whose last wave is at least 85% full wins, else the fullest; every CTA
    // keeps at least 4 K blocks, and a matrix with a wave of tiles already is
    // not split (its partials would grow for nothing).  Measured on B200
    // (n_pad 64, us per launch): gate|up 22016 x 2048 split 2 / 3 / 4: 31.7 /
    // 25.8 / 32.4; q|k|v 2560 x 2048 split 4 / 8: 9.4 / 7.7; down 2048 x
    // 11008 split 16 / 21 (a second wave of 40 CTAs): 13.2 / 20.0.
    const int mtiles = (rows + kTcM - 1) / kTcM;
    const int nblk = K / kBlockK;
    const int slots = 2 * device_sm_count();
    if (mtiles >= slots) return 1;
    int cap = nblk / 4;
    if (cap > 32) cap = 32;
    if (cap < 1) cap = 1;
    int best = 1;
    double best_fill = 0.0;
    for (int ks = 1; ks <= cap; ++ks) {
        const int ctas = mtiles * ks;
        const int waves = (ctas + slots - 1) / slots;
        const double fill = static_cast<double>(ctas) / (static_cast<double>(waves) * slots);
        if (fill >= 0.85) return ks;
        if (fill > best_fill + 1e-9) {
            best_fill = fill;
            best = ks;
        }
    }
    return best;
}

namespace {
template <int WT>
cudaError_t launch_gemm(const TcArgs& a, int ksplit, cudaStream_t s) {
    if (GemmSmem<WT>::raw_stages(a.n_pad) > kMaxRaw || GemmSmem<WT>::a_stages(a.n_pad) > kMaxA ||
        GemmSmem<WT>::a_stages(a.n_pad) > GemmSmem<WT>::raw_stages(a.n_pad))
        return cudaErrorInvalidConfiguration;  // barrier arrays, and the A-tile release rule needs R >= SA
    CUtensorMap mw, mx;
    cudaError_t st;
    if (WT == 2)
        st = cudaSuccess;  // the re-tiled records come by bulk copy; map_w is unused
    else if (WT == 0)
        st = encode_tmap_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.packed, a.K / 2, a.rows, a.K / 2, 32, kTcM,
                            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    else
        st = encode_tmap_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.packed, a.K, a.rows,
                            static_cast<uint64_t>(a.K) * 2, kBlockK, kTcM, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    if (st != cudaSuccess) return st;
    if (WT == 2) memset(&mw, 0, sizeof(mw));
    st = encode_tmap_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.x, a.K, a.n_pad, static_cast<uint64_t>(a.K) * 2,
                        kBlockK, a.n_pad, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
    if (st != cudaSuccess) return st;
    static thread_local int attr_dev[3] = {-1, -1, -1};
    int dev = 0;
    st = cudaGetDevice(&dev);
    if (st != cudaSuccess) return st;
    if (attr_dev[WT] != dev) {  // the largest footprint over n_pad once per device
        int mx_bytes = GemmSmem<WT>::bytes(16);
        if (GemmSmem<WT>::bytes(32) > mx_bytes) mx_bytes = GemmSmem<WT>::bytes(32);
        if (GemmSmem<WT>::bytes(64) > mx_bytes) mx_bytes = GemmSmem<WT>::bytes(64);
        st = cudaFuncSetAttribute(gemm_tc_kernel<WT>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx_bytes);
        if (st != cudaSuccess) return st;
        attr_dev[WT] = dev;
    }
    return launch_pdl(gemm_tc_kernel<WT>, dim3((a.rows + kTcM - 1) / kTcM, ksplit), dim3(kGThreads),
                      static_cast<size_t>(GemmSmem<WT>::bytes(a.n_pad)), s, mw, mx, a);
}
}  // namespace

cudaError_t batch_gemm(int weight_type, const void* weight, const float* absmax, int rows, int K, const uint16_t* x,
                       int n_pad, int ksplit, float* partials, int row_offset, int total_rows, int* err,
                       cudaStream_t s, const BatchEpilogue* epi) {
    if (rows < 1 || K < kBlockK || K % kBlockK != 0 || !(n_pad == 16 || n_pad == 32 || n_pad == 64) || ksplit < 1 ||
        ksplit > K / kBlockK || row_offset < 0 || row_offset + rows > total_rows ||
        weight_type < 0 || weight_type > 2 || (weight_type == 0 && absmax == nullptr))
        return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(x) |
         reinterpret_cast<uintptr_t>(partials) | reinterpret_cast<uintptr_t>(absmax)) & 15u)
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
    memset(&a.e, 0, sizeof(a.e));
    if (epi != nullptr && epi->mode != 0) {
        // fused epilogues: NF4 weights, the whole matrix in the partials, the tile shapes they need
        if (weight_type == 1 || epi->tickets == nullptr || epi->batch < 1 || epi->batch > n_pad || row_offset != 0 ||
            total_rows != rows || n_pad > 64 || epi->mode > 3 || (epi->mode == 1 && epi->resid == nullptr) ||
            (epi->mode == 2 && (epi->hout == nullptr || rows % kTcM != 0)) ||
            (epi->mode == 3 && (rows != (epi->q_heads + 2 * epi->kv_heads) * kTcM || epi->pos == nullptr ||
                                epi->q_out == nullptr || epi->kcache == nullptr || epi->vcache == nullptr ||
                                epi->rope_cos == nullptr || epi->rope_sin == nullptr)))
            return cudaErrorInvalidValue;
        a.e = *epi;
    }
    if (weight_type == 2) return launch_gemm<2>(a, ksplit, s);
    return weight_type == 0 ? launch_gemm<0>(a, ksplit, s) : launch_gemm<1>(a, ksplit, s);
}

cudaError_t batch_rmsnorm(const uint16_t* x, const uint16_t* w, uint16_t* out, int batch, int H, float eps,
                          cudaStream_t s) {
    if (H % 8 != 0 || H > 256 * 8 * kNormVec) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(out)) & 15u)
        return cudaErrorMisalignedAddress;
    return launch_pdl(batch_rmsnorm_kernel, dim3(batch), dim3(256), 0, s, x, w, out, H, eps);
}

cudaError_t batch_qkv_epilogue(const BatchQkv& q, cudaStream_t s) {
    if (q.n_pad > 64 || q.head_dim % (2 * kQkvPairs) != 0) return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(q.partials) & 15u) return cudaErrorMisalignedAddress;
    const int groups = q.head_dim / 2 / kQkvPairs;
    return launch_pdl(batch_qkv_epilogue_kernel, dim3((q.q_heads + 2 * q.kv_heads) * groups), dim3(256), 0, s, q);
}

cudaError_t batch_residual(const float* partials, int ksplit, int rows, int n_pad, int batch, uint16_t* x,
                           cudaStream_t s) {
    if (n_pad > 64) return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(partials) & 15u) return cudaErrorMisalignedAddress;
    const int er = epi_rows(n_pad);
    return launch_pdl(batch_residual_kernel, dim3((rows + er - 1) / er), dim3(256), 0, s, partials, ksplit,
                      rows, n_pad, batch, x);
}

cudaError_t batch_swiglu(const float* partials, int ksplit, int inter, int n_pad, int batch, uint16_t* h,
                         cudaStream_t s) {
    if (n_pad > 64) return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(partials) & 15u) return cudaErrorMisalignedAddress;
    const int er = kSwigluPer * epi_rows(n_pad);
    return launch_pdl(batch_swiglu_kernel, dim3((inter + er - 1) / er), dim3(256), 0, s, partials, ksplit,
                      inter, n_pad, batch, h);
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

cudaError_t batch_split_sum(const float* partials, int ksplit, int rows, int n_pad, float* out, cudaStream_t s) {
    const int64_t n = static_cast<int64_t>(rows) * n_pad;
    const int64_t g = (n + 255) / 256;
    return launch_pdl(batch_split_sum_kernel, dim3(static_cast<unsigned>(g < 2048 ? g : 2048)), dim3(256), 0, s,
                      partials, ksplit, n, out);
}

cudaError_t batch_argmax_pairs(const float* partials, int ksplit, int vocab, int n_pad, int batch, float* ws,
                               int index_base, int32_t* pairs, cudaStream_t s) {
    float* cv = ws;
    int* ci = reinterpret_cast<int*>(ws + batch * kArgCtas);
    cudaError_t st =
        launch_pdl(batch_argmax_stage1, dim3(kArgCtas), dim3(256), 0, s, partials, ksplit, vocab, n_pad, batch, cv, ci);
    if (st != cudaSuccess) return st;
    return launch_pdl(batch_argmax_pairs_stage2, dim3(batch), dim3(32), 0, s, static_cast<const float*>(cv),
                      static_cast<const int*>(ci), index_base, pairs);
}

cudaError_t batch_select_advance(const int32_t* gathered, int world, int batch, int32_t* state, int32_t* history,
                                 int history_len, cudaStream_t s) {
    return launch_pdl(batch_select_advance_kernel, dim3((batch + 63) / 64), dim3(64), 0, s, gathered, world, batch,
                      state, history, history_len);
}

cudaError_t batch_embedding(const uint16_t* emb, const int32_t* state, uint16_t* x, int batch, int H, int vocab,
                            int* err, cudaStream_t s) {
    return launch_pdl(batch_embedding_kernel, dim3(batch), dim3(256), 0, s, emb, state, x, H, vocab, err);
}

cudaError_t batch_state_views(const int32_t* state, int batch, int32_t* pos, int32_t* kv_len, cudaStream_t s) {
    return launch_pdl(batch_state_views_kernel, dim3((batch + 63) / 64), dim3(64), 0, s, state, batch, pos, kv_len);
}

}  // namespace kc
