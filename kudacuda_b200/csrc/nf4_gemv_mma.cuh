// nf4_gemv_mma.cuh -- the production NF4 GEMV for sm_100a: codebook-pair
// table lookups feed f16 tensor-core fragments (mma.m16n8k16, f32 accumulate).
//
// Why the tensor core for a batch-1 GEMV: the op is HBM-bound (0.5625 B per
// weight) only if dequantisation costs under ~2.5 instructions per weight at
// 148 SMs x 1.9 GHz.  One shared-memory lookup of a packed byte returns
// half2(level[hi], level[lo]) -- exactly one A-fragment register of an
// m16n8k16 f16 mma -- so a byte costs two integer ops (table offset) and one
// LDS, and the tensor core does the multiply-accumulate in fp32 with no
// f16->f32 conversions.  The B operand is the activation vector (column 0;
// columns 1..7 carry copies and are ignored at batch 1).
//
// Tiling.  A tile is 16 weight rows: rows 0-7 ("A" group) and 8-15 ("B"
// group) are chosen per epilogue so that lane (g, 0) ends with the pair the
// epilogue needs -- RoPE partners (i, i+64), SwiGLU partners (gate j, up j),
// K/V partners (k j, v j), or plain consecutive rows.  The CTA's 8 warps
// split K (64-element absmax blocks) and reduce their fragments through
// shared memory; CTAs loop over tiles so the 32 KB table is built once.
//
// K permutation inside a 64-element block (all rows of a tile agree, so the
// dot product is unchanged): thread (g, t) of the warp owns bytes
// [8t, 8t+8) of each of its two rows' 32-byte block; k-step s uses byte 2s
// for k-slots (2t, 2t+1) and byte 2s+1 for k-slots (2t+8, 2t+9), i.e.
// block elements 16t+4s+{0,1} and 16t+4s+{2,3}; the B fragment for the same
// slots is activation pair 8t+2s and 8t+2s+1 of the block.  The block's
// fp32 partial is scaled by the row's absmax and added to fp32 totals.
#pragma once

#include "nf4_gemv.cuh"

namespace kc {

constexpr int kMmaWarps = 8;
constexpr int kMmaThreads = kMmaWarps * 32;
constexpr int kMmaGroup = 2;  // 64-element blocks per prefetch step

// A pure function of its operands (no side effects), so the asm is not
// volatile: the compiler may interleave independent accumulator chains.
__device__ __forceinline__ void mma_f16_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Table offsets of byte j of a packed word (128-byte entry stride, lane slot).
__device__ __forceinline__ uint32_t lut_off_b0(uint32_t w, uint32_t lane_off) { return ((w << 7) & 0x7f80u) | lane_off; }
__device__ __forceinline__ uint32_t lut_off_b1(uint32_t w, uint32_t lane_off) { return ((w >> 1) & 0x7f80u) | lane_off; }
__device__ __forceinline__ uint32_t lut_off_b2(uint32_t w, uint32_t lane_off) { return ((w >> 9) & 0x7f80u) | lane_off; }
__device__ __forceinline__ uint32_t lut_off_b3(uint32_t w, uint32_t lane_off) { return ((w >> 17) & 0x7f80u) | lane_off; }

struct TileRows {
    const uint8_t* wA;  // packed base of row group A (8 rows, stride K/2)
    const uint8_t* wB;
    const float* sA;    // absmax base of row group A (stride K/64)
    const float* sB;
    int rA, rB;         // first row index of each group (epilogue bookkeeping)
    int nA, nB;         // valid rows in each group (tails)
    int mA, mB;         // matrix index of each group
    int kind;
};

template <int EPI>
__device__ __forceinline__ TileRows decode_tile(const Nf4GemvArgs& a, int t) {
    TileRows r;
    const int64_t rb = a.K / 2, ab = a.K / kBlocksize;
    auto set = [&](int mA, int rowA, int nA, int mB, int rowB, int nB) {
        r.wA = a.m[mA].packed + rb * rowA;
        r.sA = a.m[mA].absmax + ab * rowA;
        r.wB = a.m[mB].packed + rb * rowB;
        r.sB = a.m[mB].absmax + ab * rowB;
        r.rA = rowA;
        r.rB = rowB;
        r.nA = nA;
        r.nB = nB;
        r.mA = mA;
        r.mB = mB;
    };
    auto clamp8 = [](int rows, int start) { return max(0, min(8, rows - start)); };
    if constexpr (EPI == kEpiStore || EPI == kEpiResidHF) {
        const int r0 = 16 * t;
        const int rows = a.m[0].rows;
        set(0, r0, clamp8(rows, r0), 0, r0 + 8, clamp8(rows, r0 + 8));
        r.kind = 0;
    } else if constexpr (EPI == kEpiQkvRef) {
        const int qt = (a.m[0].rows + 15) / 16;
        if (t < qt) {
            const int r0 = 16 * t;
            set(0, r0, clamp8(a.m[0].rows, r0), 0, r0 + 8, clamp8(a.m[0].rows, r0 + 8));
            r.kind = 0;
        } else {
            const int j0 = 8 * (t - qt);
            set(1, j0, clamp8(a.m[1].rows, j0), 2, j0, clamp8(a.m[2].rows, j0));
            r.kind = 1;
        }
    } else if constexpr (EPI == kEpiQkvRopeHF) {
        const int half = a.head_dim / 2;  // 64: 8 tiles per head
        const int per_head = half / 8;
        const int qt = a.q_heads * per_head;
        const int kt = a.kv_heads * per_head;
        if (t < qt + kt) {
            const int s = t < qt ? 0 : 1;
            const int u = t < qt ? t : t - qt;
            const int head = u / per_head;
            const int i0 = 8 * (u - head * per_head);
            const int row = head * a.head_dim + i0;
            set(s, row, 8, s, row + half, 8);
            r.kind = s;
        } else {
            const int r0 = 16 * (t - qt - kt);
            const int rows = a.m[2].rows;
            set(2, r0, clamp8(rows, r0), 2, r0 + 8, clamp8(rows, r0 + 8));
            r.kind = 2;
        }
    } else {  // SwiGLU: gate rows in A, up rows in B
        const int j0 = 8 * t;
        set(0, j0, clamp8(a.m[0].rows, j0), 1, j0, clamp8(a.m[1].rows, j0));
        r.kind = 0;
    }
    return r;
}

template <int EPI>
__host__ __device__ inline int mma_tiles(const Nf4GemvArgs& a) {
    if constexpr (EPI == kEpiStore || EPI == kEpiResidHF) return (a.m[0].rows + 15) / 16;
    else if constexpr (EPI == kEpiQkvRef) return (a.m[0].rows + 15) / 16 + (a.m[1].rows + 7) / 8;
    else if constexpr (EPI == kEpiQkvRopeHF) return (a.q_heads + a.kv_heads) * (a.head_dim / 16) + (a.m[2].rows + 15) / 16;
    else return (a.m[0].rows + 7) / 8;
}

// Epilogue for one row pair (row A value vA, row B value vB) owned by lane g.
template <int EPI, int OT>
__device__ __forceinline__ void mma_epilogue(const Nf4GemvArgs& a, const TileRows& r, int g, float vA, float vB) {
    const bool okA = g < r.nA, okB = g < r.nB;
    if constexpr (EPI == kEpiStore || EPI == kEpiResidHF || EPI == kEpiQkvRef) {
        RowPair p;
        p.r0 = r.rA + g;
        p.r1 = r.rB + g;
        if constexpr (EPI == kEpiQkvRef) {
            if (r.kind == 1) {
                if (okA) store_elem<OT>(a.out[1], p.r0, vA + load_elem<OT>(a.bias[1], p.r0));
                if (okB) store_elem<OT>(a.out[2], p.r1, vB + load_elem<OT>(a.bias[2], p.r1));
                return;
            }
            if (okA) store_elem<OT>(a.out[0], p.r0, vA + load_elem<OT>(a.bias[0], p.r0));
            if (okB) store_elem<OT>(a.out[0], p.r1, vB + load_elem<OT>(a.bias[0], p.r1));
        } else if constexpr (EPI == kEpiStore) {
            if (okA) store_elem<OT>(a.out[0], p.r0, vA + (a.bias[0] ? load_elem<OT>(a.bias[0], p.r0) : 0.0F));
            if (okB) store_elem<OT>(a.out[0], p.r1, vB + (a.bias[0] ? load_elem<OT>(a.bias[0], p.r1) : 0.0F));
        } else {
            uint16_t* res = static_cast<uint16_t*>(a.resid);
            if (okA) res[p.r0] = f32_to_bf16_bits(bf16_bits_to_f32(res[p.r0]) + round_bf16(vA));
            if (okB) res[p.r1] = f32_to_bf16_bits(bf16_bits_to_f32(res[p.r1]) + round_bf16(vB));
        }
    } else if constexpr (EPI == kEpiQkvRopeHF) {
        RowPair p;
        p.r0 = r.rA + g;
        p.r1 = r.rB + g;
        if (r.kind == 2) {
            // V rows: no rotation; both groups are plain rows
            const int pos = *a.pos_dev;
            if (pos < 0 || pos >= a.kv_cap || pos >= a.max_pos) {
                if (a.err != nullptr) atomicOr(a.err, 2);
                return;
            }
            uint16_t* vc = static_cast<uint16_t*>(a.out[2]);
            float y[2] = {round_bf16(vA), round_bf16(vB)};
            const int rows[2] = {p.r0, p.r1};
            const bool ok[2] = {okA, okB};
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                if (!ok[i]) continue;
                float v = y[i];
                if (a.bias[2] != nullptr) v = round_bf16(v + load_elem<kBF16>(a.bias[2], rows[i]));
                const int h = rows[i] / a.head_dim, d = rows[i] - h * a.head_dim;
                vc[(static_cast<int64_t>(h) * a.kv_cap + pos) * a.head_dim + d] = f32_to_bf16_bits(v);
            }
            return;
        }
        p.kind = r.kind;
        epilogue<kEpiQkvRopeHF, OT>(a, p, vA, vB);
    } else if constexpr (EPI == kEpiSwiGluRef || EPI == kEpiSwiGluHF) {
        if (!okA) return;
        RowPair p;
        p.r0 = r.rA + g;
        p.r1 = p.r0;
        p.kind = 0;
        epilogue<EPI, OT>(a, p, vA, vB);
    }
}

// Consumer-group barrier: named barrier 1 over the first N threads (the
// producer warp of the TMA kernel never joins it); N == 0 is the whole CTA.
template <int N>
__device__ __forceinline__ void group_sync() {
    if constexpr (N == 0) __syncthreads();
    else asm volatile("bar.sync 1, %0;" ::"n"(N) : "memory");
}

// Stage the activation vector as plain (unswizzled) f16 pairs.

template <int IN, int XT, int GROUP = 0>
__device__ __forceinline__ void stage_x_plain(const Nf4GemvArgs& a, uint32_t* xp, float* red) {
    const int tid = threadIdx.x, K = a.K;
    const int nthreads = GROUP == 0 ? static_cast<int>(blockDim.x) : GROUP;
    float inv = 1.0F;
    if constexpr (IN != kInRaw) {
        float ss = 0.0F;
        for (int i = tid; i < K; i += nthreads) {
            const float v = load_elem<XT>(a.x, i);
            ss += v * v;
        }
        ss = warp_sum(ss);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        group_sync<GROUP>();
        if (tid < 32) {
            float v = tid < (nthreads >> 5) ? red[tid] : 0.0F;
            v = warp_sum(v);
            if (tid == 0) red[0] = 1.0F / sqrtf(v / static_cast<float>(K) + a.eps);
        }
        group_sync<GROUP>();
        inv = red[0];
    }
    bool overflow = false;
    for (int j = tid; j < K / 2; j += nthreads) {
        float v[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int i = 2 * j + h;
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
        xp[j] = static_cast<uint32_t>(f32_to_f16_bits(v[0])) | (static_cast<uint32_t>(f32_to_f16_bits(v[1])) << 16);
    }
    if (overflow && a.err != nullptr) atomicOr(a.err, 1);
    group_sync<GROUP>();
}

// Vector staging: the activation (and norm weight) vectors are read as
// octets of 8 elements (one 16-byte load for f16/bf16, two for fp32), up to
// kStageRound octets per thread issued back to back, so staging costs one
// global round trip per pass for K <= kStageRound * 8 * threads instead of a
// chain of dependent scalar loads.  Same arithmetic as stage_x_plain.
constexpr int kStageRound = 4;

template <int XT>
struct Octet {
    uint4 v[XT == kF32 ? 2 : 1];
};
template <int XT>
__device__ __forceinline__ void ld_octet(const void* base, int o, Octet<XT>& r) {
    const uint4* p = static_cast<const uint4*>(base) + (XT == kF32 ? 2 : 1) * o;
    r.v[0] = p[0];
    if constexpr (XT == kF32) r.v[1] = p[1];
}
template <int XT>
__device__ __forceinline__ float octet_at(const Octet<XT>& r, int i) {
    if constexpr (XT == kF32) {
        const uint4& w = r.v[i >> 2];
        const uint32_t u = (i & 3) == 0 ? w.x : (i & 3) == 1 ? w.y : (i & 3) == 2 ? w.z : w.w;
        return __uint_as_float(u);
    } else {
        const uint4& w = r.v[0];
        const int q = i >> 1;
        const uint32_t u = q == 0 ? w.x : q == 1 ? w.y : q == 2 ? w.z : w.w;
        const uint16_t h = static_cast<uint16_t>((i & 1) ? (u >> 16) : (u & 0xffffu));
        if constexpr (XT == kBF16) return bf16_bits_to_f32(h);
        else return f16_bits_to_f32(h);
    }
}

template <int IN, int XT, int GROUP = 0>
__device__ __forceinline__ void stage_x_vec(const Nf4GemvArgs& a, uint32_t* xp, float* red) {
    const int tid = threadIdx.x;
    const int nthreads = GROUP == 0 ? static_cast<int>(blockDim.x) : GROUP;
    const int noct = a.K >> 3;
    float inv = 1.0F;
    if constexpr (IN != kInRaw) {
        float ss = 0.0F;
        for (int base = tid; base < noct; base += kStageRound * nthreads) {
            Octet<XT> r[kStageRound];
#pragma unroll
            for (int u = 0; u < kStageRound; ++u)
                if (base + u * nthreads < noct) ld_octet<XT>(a.x, base + u * nthreads, r[u]);
#pragma unroll
            for (int u = 0; u < kStageRound; ++u) {
                if (base + u * nthreads < noct) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float v = octet_at<XT>(r[u], i);
                        ss += v * v;
                    }
                }
            }
        }
        ss = warp_sum(ss);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        group_sync<GROUP>();
        if (tid < 32) {
            float v = tid < (nthreads >> 5) ? red[tid] : 0.0F;
            v = warp_sum(v);
            if (tid == 0) red[0] = 1.0F / sqrtf(v / static_cast<float>(a.K) + a.eps);
        }
        group_sync<GROUP>();
        inv = red[0];
    }
    bool overflow = false;
    for (int base = tid; base < noct; base += kStageRound * nthreads) {
        Octet<XT> r[kStageRound];
        Octet<XT> nw[kStageRound];
#pragma unroll
        for (int u = 0; u < kStageRound; ++u) {
            const int o = base + u * nthreads;
            if (o < noct) {
                ld_octet<XT>(a.x, o, r[u]);
                if constexpr (IN != kInRaw) ld_octet<XT>(a.norm_w, o, nw[u]);
            }
        }
#pragma unroll
        for (int u = 0; u < kStageRound; ++u) {
            const int o = base + u * nthreads;
            if (o >= noct) continue;
            uint32_t w[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float v[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int i = 2 * q + h;
                    float x = octet_at<XT>(r[u], i);
                    if constexpr (IN == kInNormRef) {
                        x = x * inv * octet_at<XT>(nw[u], i);
                        if (a.norm_ws != nullptr && blockIdx.x == 0) a.norm_ws[8 * o + i] = x;
                    } else if constexpr (IN == kInNormHF) {
                        x = round_bf16(octet_at<XT>(nw[u], i) * round_bf16(x * inv));
                    }
                    overflow |= !(fabsf(x) <= 65504.0F);
                    v[h] = x;
                }
                w[q] = static_cast<uint32_t>(f32_to_f16_bits(v[0])) |
                       (static_cast<uint32_t>(f32_to_f16_bits(v[1])) << 16);
            }
            *reinterpret_cast<uint4*>(xp + 4 * o) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
    if (overflow && a.err != nullptr) atomicOr(a.err, 1);
    group_sync<GROUP>();
}

template <int IN, int XT, int GROUP = 0>
__device__ __forceinline__ void stage_x_pairs(const Nf4GemvArgs& a, uint32_t* xp, float* red) {
    if (a.xvec) stage_x_vec<IN, XT, GROUP>(a, xp, red);
    else stage_x_plain<IN, XT, GROUP>(a, xp, red);
}

struct MmaStepRegs {
    uint2 wA[kMmaGroup];
    uint2 wB[kMmaGroup];
    float sA[kMmaGroup];
    float sB[kMmaGroup];
};

__device__ __forceinline__ uint2 ld_stream_u2(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

// Load one prefetch step: kMmaGroup blocks starting at block b of the warp's
// rows g (group A) and g (group B); blocks at or past `bend` are skipped.
__device__ __forceinline__ void mma_load_step(MmaStepRegs& R, const TileRows& tr, int g, int t, int64_t rb, int64_t ab,
                                              int b, int bend) {
    const int gA = min(g, max(tr.nA - 1, 0));
    const int gB = min(g, max(tr.nB - 1, 0));
    const uint8_t* pA = tr.wA + rb * gA + 8 * t;
    const uint8_t* pB = tr.wB + rb * gB + 8 * t;
    const float* qA = tr.sA + ab * gA;
    const float* qB = tr.sB + ab * gB;
#pragma unroll
    for (int j = 0; j < kMmaGroup; ++j) {
        const int blk = b + j;
        if (blk < bend) {
            R.wA[j] = ld_stream_u2(pA + 32 * static_cast<int64_t>(blk));
            R.wB[j] = ld_stream_u2(pB + 32 * static_cast<int64_t>(blk));
            R.sA[j] = __ldg(qA + blk);
            R.sB[j] = __ldg(qB + blk);
        } else {
            R.wA[j] = make_uint2(0x77777777u, 0x77777777u);  // level 0.0 codes
            R.wB[j] = make_uint2(0x77777777u, 0x77777777u);
            R.sA[j] = 0.0F;
            R.sB[j] = 0.0F;
        }
    }
}

__device__ __forceinline__ void mma_compute_step(const MmaStepRegs& R, const uint32_t* lut, uint32_t lane_off,
                                                 const uint32_t* xp, int t, int b, int bend, float* tot) {
#pragma unroll
    for (int j = 0; j < kMmaGroup; ++j) {
        const int blk = b + j;
        if (blk >= bend) break;  // warp-uniform: the staged activations end at this warp's last block
        const uint4 x0 = *reinterpret_cast<const uint4*>(xp + 32 * blk + 8 * t);
        const uint4 x1 = *reinterpret_cast<const uint4*>(xp + 32 * blk + 8 * t + 4);
        float c[4] = {0.0F, 0.0F, 0.0F, 0.0F};
        const uint32_t wa0 = R.wA[j].x, wa1 = R.wA[j].y, wb0 = R.wB[j].x, wb1 = R.wB[j].y;
        // k-step 0: bytes 0,1   k-step 1: bytes 2,3   k-step 2: bytes 4,5   k-step 3: bytes 6,7
        mma_f16_16816(c, lut_at(lut, lut_off_b0(wa0, lane_off)), lut_at(lut, lut_off_b0(wb0, lane_off)),
                      lut_at(lut, lut_off_b1(wa0, lane_off)), lut_at(lut, lut_off_b1(wb0, lane_off)), x0.x, x0.y);
        mma_f16_16816(c, lut_at(lut, lut_off_b2(wa0, lane_off)), lut_at(lut, lut_off_b2(wb0, lane_off)),
                      lut_at(lut, lut_off_b3(wa0, lane_off)), lut_at(lut, lut_off_b3(wb0, lane_off)), x0.z, x0.w);
        mma_f16_16816(c, lut_at(lut, lut_off_b0(wa1, lane_off)), lut_at(lut, lut_off_b0(wb1, lane_off)),
                      lut_at(lut, lut_off_b1(wa1, lane_off)), lut_at(lut, lut_off_b1(wb1, lane_off)), x1.x, x1.y);
        mma_f16_16816(c, lut_at(lut, lut_off_b2(wa1, lane_off)), lut_at(lut, lut_off_b2(wb1, lane_off)),
                      lut_at(lut, lut_off_b3(wa1, lane_off)), lut_at(lut, lut_off_b3(wb1, lane_off)), x1.z, x1.w);
        tot[0] = fmaf(c[0], R.sA[j], tot[0]);
        tot[1] = fmaf(c[1], R.sA[j], tot[1]);
        tot[2] = fmaf(c[2], R.sB[j], tot[2]);
        tot[3] = fmaf(c[3], R.sB[j], tot[3]);
    }
}

template <int IN, int XT, int EPI, int OT>
__global__ void __launch_bounds__(kMmaThreads, 2) nf4_gemv_mma_kernel(const Nf4GemvArgs a) {
    __shared__ __align__(16) uint32_t lut[kLutWords];
    __shared__ float red[32];
    __shared__ __align__(16) float part[kMmaWarps][32][4];
    extern __shared__ __align__(16) uint32_t xp[];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const uint32_t lane_off = static_cast<uint32_t>(lane) << 2;
    const int nblk = a.K / kBlocksize;
    // this warp's slice of the K blocks (same step count for every warp)
    const int b_begin = (nblk * warp) / kMmaWarps;
    const int b_end = (nblk * (warp + 1)) / kMmaWarps;
    const int per_warp_max = (nblk + kMmaWarps - 1) / kMmaWarps;
    const int steps_per_tile = (per_warp_max + kMmaGroup - 1) / kMmaGroup;
    const int ntiles = mma_tiles<EPI>(a);
    const int64_t rb = a.K / 2, ab = nblk;

    build_pair_lut(lut, tid, blockDim.x);
    // weights are static: fetch this warp's first step before waiting on the producer
    MmaStepRegs R0, R1;
    int tile = blockIdx.x;
    TileRows tr = decode_tile<EPI>(a, tile < ntiles ? tile : 0);
    if (tile < ntiles) mma_load_step(R0, tr, g, t, rb, ab, b_begin, b_end);
    pdl_launch_dependents();
    pdl_wait_on_producer();
    stage_x_pairs<IN, XT>(a, xp, red);  // ends with __syncthreads (also covers the table)

    int step = 0;  // step index within the current tile
    while (tile < ntiles) {
        float tot[4] = {0.0F, 0.0F, 0.0F, 0.0F};
        for (step = 0; step < steps_per_tile; step += 2) {
            // R0 holds `step`; fetch step+1 (or the next tile's first step) into R1
            const bool has1 = step + 1 < steps_per_tile;
            TileRows nt = tr;
            int ntile = tile;
            if (has1) {
                mma_load_step(R1, tr, g, t, rb, ab, b_begin + (step + 1) * kMmaGroup, b_end);
            } else {
                ntile = tile + gridDim.x;
                if (ntile < ntiles) {
                    nt = decode_tile<EPI>(a, ntile);
                    mma_load_step(R1, nt, g, t, rb, ab, b_begin, b_end);
                }
            }
            mma_compute_step(R0, lut, lane_off, xp, t, b_begin + step * kMmaGroup, b_end, tot);
            if (has1) {
                // R1 holds step+1; fetch step+2 (or the next tile's first step) into R0
                const bool has2 = step + 2 < steps_per_tile;
                if (has2) {
                    mma_load_step(R0, tr, g, t, rb, ab, b_begin + (step + 2) * kMmaGroup, b_end);
                } else {
                    ntile = tile + gridDim.x;
                    if (ntile < ntiles) {
                        nt = decode_tile<EPI>(a, ntile);
                        mma_load_step(R0, nt, g, t, rb, ab, b_begin, b_end);
                    }
                }
                mma_compute_step(R1, lut, lane_off, xp, t, b_begin + (step + 1) * kMmaGroup, b_end, tot);
            } else {
                // next tile's first step sits in R1: move it to R0
                R0 = R1;
            }
        }
        // ---- cross-warp reduction of the fragments, then the epilogue
        *reinterpret_cast<float4*>(&part[warp][lane][0]) = make_float4(tot[0], tot[1], tot[2], tot[3]);
        __syncthreads();
        if (warp == 0 && t == 0) {
            float vA = 0.0F, vB = 0.0F;
#pragma unroll
            for (int w = 0; w < kMmaWarps; ++w) {
                vA += part[w][lane][0];  // column 0 (batch 0), row group A
                vB += part[w][lane][2];  // column 0, row group B
            }
            mma_epilogue<EPI, OT>(a, tr, g, vA, vB);
        }
        __syncthreads();
        tile += gridDim.x;
        if (tile < ntiles) tr = decode_tile<EPI>(a, tile);
    }
}

}  // namespace kc

namespace kc {

// ---------------------------------------------------------------------------
// Warp-specialised TMA variant (the production path when K % 256 == 0).
//
// One producer warp streams each 16-row tile through a shared-memory ring of
// `a.stages` stages with 2D bulk-tensor loads: per stage, a 1024-element K
// slice of both 8-row groups (8 boxes of 8 rows x 128 B with 128-byte
// swizzle) and their absmax (2 boxes of 8 rows x 16 fp32), completing on the
// stage's "full" mbarrier.  Eight consumer warps each take two consecutive
// 64-element blocks of the slice (the K split), read their A fragments
// conflict-free thanks to the swizzle, run the table->mma math, and release
// the stage on its "empty" mbarrier.  At the end of a tile the warps' column
// sums meet in shared memory (double-buffered by tile parity, one barrier per
// tile) and warp 0 adds them in warp order (bit-reproducible) and applies the
// epilogue.  The host sizes the ring from the shared-memory budget (up to 16
// stages = 144 KB in flight per CTA); the producer starts streaming before
// griddepcontrol.wait because weights are static.  No multicast is used
// anywhere.

struct GemvMaps {
    CUtensorMap w[3];  // packed nibbles, [rows][K/2] uint8, box 8 x 128 B, 128B swizzle
    CUtensorMap s[3];  // absmax, [rows][K/64] fp32, box 8 x 16
};

constexpr int kTmaCons = 8;
constexpr int kTmaThreads = (kTmaCons + 1) * 32;
constexpr int kSlice = 1024;                              // K elements per stage
constexpr int kSliceBlocks = kSlice / kBlocksize;         // 16: two per consumer warp
constexpr int kBoxBytes = 1024;                           // 8 rows x 128 B = 4 blocks of a row group
constexpr int kAbsBoxBytes = 8 * kSliceBlocks * 4;        // 8 rows x 16 fp32
constexpr int kTStageBytes = 8 * kBoxBytes + 2 * kAbsBoxBytes;  // 9 KB: every stage stays 1 KB aligned
constexpr uint32_t kTStageTx = kTStageBytes;
constexpr int kTMaxStages = 16;
constexpr int kTMinStages = 2;

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Table offset of byte 0 with one bit-field insert.
__device__ __forceinline__ uint32_t lut_off_b0_bfi(uint32_t w, uint32_t lane_off) {
    uint32_t d;
    asm("bfi.b32 %0, %1, %2, 7, 8;" : "=r"(d) : "r"(w), "r"(lane_off));
    return d;
}

// One 64-element block of both row groups: four mma k-steps; returns the
// batch-column sums (c0: row g, c2: row g + 8).
__device__ __forceinline__ float2 tma_block_dot(const uint32_t* lut, uint32_t lane_off, uint2 wa, uint2 wb, uint4 x0,
                                                uint4 x1) {
    float c[4] = {0.0F, 0.0F, 0.0F, 0.0F};
    mma_f16_16816(c, lut_at(lut, lut_off_b0_bfi(wa.x, lane_off)), lut_at(lut, lut_off_b0_bfi(wb.x, lane_off)),
                  lut_at(lut, lut_off_b1(wa.x, lane_off)), lut_at(lut, lut_off_b1(wb.x, lane_off)), x0.x, x0.y);
    mma_f16_16816(c, lut_at(lut, lut_off_b2(wa.x, lane_off)), lut_at(lut, lut_off_b2(wb.x, lane_off)),
                  lut_at(lut, lut_off_b3(wa.x, lane_off)), lut_at(lut, lut_off_b3(wb.x, lane_off)), x0.z, x0.w);
    mma_f16_16816(c, lut_at(lut, lut_off_b0_bfi(wa.y, lane_off)), lut_at(lut, lut_off_b0_bfi(wb.y, lane_off)),
                  lut_at(lut, lut_off_b1(wa.y, lane_off)), lut_at(lut, lut_off_b1(wb.y, lane_off)), x1.x, x1.y);
    mma_f16_16816(c, lut_at(lut, lut_off_b2(wa.y, lane_off)), lut_at(lut, lut_off_b2(wb.y, lane_off)),
                  lut_at(lut, lut_off_b3(wa.y, lane_off)), lut_at(lut, lut_off_b3(wb.y, lane_off)), x1.z, x1.w);
    return make_float2(c[0], c[2]);
}

template <int IN, int XT, int EPI, int OT>
__global__ void __launch_bounds__(kTmaThreads, 2) nf4_gemv_tma_kernel(const Nf4GemvArgs a,
                                                                     const __grid_constant__ GemvMaps maps) {
    __shared__ __align__(16) uint32_t lut[kLutWords];
    __shared__ float red[32];
    // column-0 fragment sums (rows g, g + 8) per warp, double-buffered by
    // tile parity so one consumer barrier per tile suffices
    __shared__ __align__(8) float2 part[2][kTmaCons][8];
    __shared__ __align__(8) uint64_t full_bar[kTMaxStages];
    __shared__ __align__(8) uint64_t empty_bar[kTMaxStages];
    extern __shared__ __align__(16) uint8_t dyn_raw[];
    const int nst = a.stages;
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_raw) + 1023) & ~uintptr_t(1023));
    uint32_t* xp = reinterpret_cast<uint32_t*>(ring + static_cast<size_t>(nst) * kTStageBytes);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nblk = a.K / kBlocksize;
    const int nslices = (a.K + kSlice - 1) / kSlice;
    const int ntiles = mma_tiles<EPI>(a);

    if (tid == 0) {
        for (int i = 0; i < nst; ++i) {
            mbar_init(&full_bar[i], 1);
            mbar_init(&empty_bar[i], kTmaCons);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kTmaCons) {
        // ---------------- producer: weights are static, no need to wait on the previous kernel
        if (lane == 0) {
            int slot = 0;
            uint32_t phase = 0;
            for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
                const TileRows tr = decode_tile<EPI>(a, tile);
                for (int sl = 0; sl < nslices; ++sl) {
                    if (!mbar_wait_bounded(&empty_bar[slot], phase ^ 1u)) {
                        if (a.err != nullptr) atomicOr(a.err, 16);
                        return;
                    }
                    uint8_t* st = ring + slot * kTStageBytes;
                    uint64_t* fb = &full_bar[slot];
                    mbar_arrive_expect_tx(fb, kTStageTx);
                    const int x0 = sl * (kSlice / 2);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        tma_load_2d(st + i * kBoxBytes, &maps.w[tr.mA], x0 + 128 * i, tr.rA, fb);
                        tma_load_2d(st + (4 + i) * kBoxBytes, &maps.w[tr.mB], x0 + 128 * i, tr.rB, fb);
                    }
                    tma_load_2d(st + 8 * kBoxBytes, &maps.s[tr.mA], sl * kSliceBlocks, tr.rA, fb);
                    tma_load_2d(st + 8 * kBoxBytes + kAbsBoxBytes, &maps.s[tr.mB], sl * kSliceBlocks, tr.rB, fb);
                    if (++slot == nst) {
                        slot = 0;
                        phase ^= 1u;
                    }
                }
            }
        }
        return;
    }

    // ---------------- consumers (warps 0..7)
    const int g = lane >> 2, t = lane & 3;
    const uint32_t lane_off = static_cast<uint32_t>(lane) << 2;
    build_pair_lut(lut, tid, kTmaCons * 32);
    pdl_wait_on_producer();
    stage_x_pairs<IN, XT, kTmaCons * 32>(a, xp, red);  // ends with the consumer barrier (covers the table)

    // Warp w takes blocks 2w and 2w+1 of each slice: both sit in 128-byte
    // box column w >> 1, at 16-byte chunks c0 and c0 + 2 of their rows
    // (128-byte swizzle: chunk c of box row r sits at chunk c ^ (r & 7)).
    const int boxcol = (warp >> 1) * kBoxBytes;
    const int c0 = 2 * ((2 * warp) & 3) + (t >> 1);
    const int f0 = boxcol + g * 128 + ((c0 ^ g) << 4) + 8 * (t & 1);
    const int f1 = boxcol + g * 128 + (((c0 + 2) ^ g) << 4) + 8 * (t & 1);
    const int abs_off = 8 * kBoxBytes + g * (kSliceBlocks * 4) + 2 * warp * 4;

    int slot = 0, buf = 0;
    uint32_t phase = 0;
    bool failed = false;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const TileRows tr = decode_tile<EPI>(a, tile);
        float totA = 0.0F, totB = 0.0F;
        for (int sl = 0; sl < nslices; ++sl) {
            if (!failed && !mbar_wait_bounded(&full_bar[slot], phase)) {
                failed = true;
                if (lane == 0 && a.err != nullptr) atomicOr(a.err, 16);
            }
            // nblk is a multiple of 4 (K % 256 == 0), so block 2w+1 is valid whenever block 2w is
            const int blk = sl * kSliceBlocks + 2 * warp;
            if (!failed && blk < nblk) {
                const uint8_t* st = ring + slot * kTStageBytes;
                const uint2 wa0 = *reinterpret_cast<const uint2*>(st + f0);
                const uint2 wb0 = *reinterpret_cast<const uint2*>(st + 4 * kBoxBytes + f0);
                const uint2 wa1 = *reinterpret_cast<const uint2*>(st + f1);
                const uint2 wb1 = *reinterpret_cast<const uint2*>(st + 4 * kBoxBytes + f1);
                const float2 sa = *reinterpret_cast<const float2*>(st + abs_off);
                const float2 sb = *reinterpret_cast<const float2*>(st + abs_off + kAbsBoxBytes);
                const uint4* xb = reinterpret_cast<const uint4*>(xp + 32 * blk + 8 * t);
                const uint4 x00 = xb[0], x01 = xb[1];
                const uint4 x10 = xb[8], x11 = xb[9];  // next block: 32 words further
                const float2 p0 = tma_block_dot(lut, lane_off, wa0, wb0, x00, x01);
                const float2 p1 = tma_block_dot(lut, lane_off, wa1, wb1, x10, x11);
                totA = fmaf(p0.x, sa.x, totA);
                totB = fmaf(p0.y, sb.x, totB);
                totA = fmaf(p1.x, sa.y, totA);
                totB = fmaf(p1.y, sb.y, totB);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[slot]);
            if (++slot == nst) {
                slot = 0;
                phase ^= 1u;
            }
        }
        // batch column 0 of the C fragment lives in lanes t == 0
        if (t == 0) part[buf][warp][g] = make_float2(totA, totB);
        group_sync<kTmaCons * 32>();
        if (warp == 0 && t == 0) {
            float vA = 0.0F, vB = 0.0F;
#pragma unroll
            for (int w = 0; w < kTmaCons; ++w) {
                const float2 pv = part[buf][w][g];
                vA += pv.x;
                vB += pv.y;
            }
            mma_epilogue<EPI, OT>(a, tr, g, vA, vB);
        }
        // the next tile writes the other buffer; warp 0 reaches that tile's
        // barrier only after this epilogue, which protects this buffer
        buf ^= 1;
    }
}

}  // namespace kc
