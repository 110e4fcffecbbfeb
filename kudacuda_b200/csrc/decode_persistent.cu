// decode_persistent.cu -- all decoder layers of one batch-1 decode step in a
// single persistent, cooperative launch on sm_100a.
//
// Replaces, for the static decode plan, the per-layer launch sequence
// (RMSNorm+QKV+RoPE+append, GQA decode, o_proj+residual, RMSNorm+SwiGLU,
// down+residual) that stands in for the reference's per-op kernels
// (kernels/common/nf4_tiled_gemv.cuh:61-278, nf4_swiglu_bf16.cuh:65-209,
// qwen2_gqa_decode.cuh:17-203) and the bitsandbytes o_proj/down matmuls
// (python/kudacuda_sidecar.py:947, :1746).  Arithmetic and rounding points are
// those of the per-op HF-semantics kernels in nf4_gemv.cuh / gqa_decode.cu.
//
// Why one launch: at batch 1 every op is a few MB of weights, so a launch per
// op pays its ramp (first DRAM round trip, activation staging, the cross-CTA
// reduction tail) five times per layer.  Here each of the 16 warps of a CTA
// owns a private ring of bulk-copy slots and streams its share of EVERY op's
// weights, layer after layer, without waiting for activations: the next op's
// weights are already in shared memory when its input vector is complete.
//
// Cross-CTA protocol (every dependency costs about three L2 round trips):
//   * producers never finish rows: after an op's GEMV each CTA reduces its
//     16 warps' partial sums in a fixed order and writes one 64-float slot per
//     row group it touched, then bumps the op's counter once (release);
//   * consumers wait for the counter to reach the number of CTAs (acquire),
//     sum each group's slots in slot order -- so the result is deterministic
//     -- and apply the epilogue themselves: the residual stream lives in every
//     CTA's shared memory (identical copies), h = SwiGLU(gate, up) is formed
//     where down needs it, and the attention CTAs build q and the new k/v row
//     (bias, RoPE) from the QKV slots;
//   * every wait is one thread's bounded spin; running out sets the step's
//     abort flag (all later waits return at once) and error bit 4.
//
// Weight stream format ("group tiles", produced once by nf4_retile_kernel
// from the bitsandbytes layout): an op's rows are taken 64 at a time
// (a group), its K in 64-element blocks.  Chunk (group G, block b) is 2304
// contiguous bytes: four 512-byte units (tiles ti = 0..3 of 16 rows), where
// lane l = 4g + t of a warp reads 16 bytes = bytes [32b + 8t, +8) of group
// rows 16ti + g and 16ti + 8 + g -- exactly its m16n8k16 A fragments -- then
// 256 bytes of absmax ordered [half][g][ti].  The row map inside a group puts
// epilogue partners 32 rows apart: RoPE pairs (i, i + head_dim/2) for q/k,
// (gate j, up j) for SwiGLU, consecutive rows otherwise.
#include <cuda_runtime.h>

#include <cstdint>

#include "kc_common.cuh"
#include "kc_launch.h"

// Phase timestamps for profiling builds only (-DKC_PERSIST_STAMPS; off in the
// library): thread 0 of every CTA records %globaltimer (comparable across
// SMs) and clock64 (this SM's cycle counter) at fixed points of one layer
// (KC_STAMP_LAYER) into g_persist_stamps[cta][64] (timer in [0, 32), cycles
// in [32, 64)), read back with kc_persist_read_stamps.  No work is skipped or
// added to the product build.
#ifdef KC_PERSIST_STAMPS
#ifndef KC_STAMP_LAYER
#define KC_STAMP_LAYER 18
#endif
__device__ unsigned long long g_persist_stamps[1024 * 64];
#define KC_STAMP(l, i)                                                          \
    do {                                                                        \
        if ((l) == KC_STAMP_LAYER && threadIdx.x == 0) {                        \
            unsigned long long t_;                                              \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_)::"memory");    \
            g_persist_stamps[blockIdx.x * 64 + (i)] = t_;                       \
            g_persist_stamps[blockIdx.x * 64 + 32 + (i)] = clock64();           \
        }                                                                       \
    } while (0)
extern "C" __attribute__((visibility("default"))) int kc_persist_read_stamps(unsigned long long* out, int n) {
    return static_cast<int>(cudaMemcpyFromSymbol(out, g_persist_stamps, sizeof(unsigned long long) * n));
}
#else
#define KC_STAMP(l, i) \
    do {               \
    } while (0)
#endif

namespace kc {
namespace {

constexpr int kPWarps = 16;
constexpr int kPThreads = kPWarps * 32;
#ifndef KC_PERSIST_RING_MAX
#define KC_PERSIST_RING_MAX 4
#endif
constexpr int kPMaxSlots = KC_PERSIST_RING_MAX;  // bulk-copy slots per warp (fewer when shared memory is short)
constexpr int kChunkCodes = 2048;
constexpr int kChunkAbs = 256;
constexpr int kChunkBytes = kChunkCodes + kChunkAbs;
constexpr int kPLutBytes = 65536;  // 256 entry rows x 256 B, lane replicas in the first 128 B of a row
constexpr int kPartGroups = 5;     // row groups one CTA may touch in one op (checked on the host)
constexpr int kAttTile = 64;       // tokens per attention tile (a split covers one or more tiles)
constexpr int kAttMaxSplits = 32;  // splits per KV head
constexpr int kMaxGroups = 512;    // row groups per op (checked on the host)
constexpr int kCounterStride = 8;  // per layer: 0 qkv, 1 attention, 2 o_proj, 3 gate/up, 4 down
constexpr uint32_t kSpinLimit = 1u << 21;

enum LayerSlot {
    kLQkvC = 0, kLQkvA, kLOC, kLOA, kLGuC, kLGuA, kLDnC, kLDnA,
    kLInNorm, kLPostNorm, kLQBias, kLKBias, kLVBias, kLKCache, kLVCache, kLPad, kLayerSlots
};
enum POp { kPQkv = 0, kPO = 1, kPGu = 2, kPDn = 3 };
enum PCounter { kCQkv = 0, kCAtt = 1, kCO = 2, kCGu = 3, kCDn = 4 };

struct PersistArgs {
    const uint64_t* layers;  // [nlayers][kLayerSlots] device pointers
    int nlayers, hidden, qh, kvh, hd, inter, cap, max_pos;
    float eps, scale_log2;
    const int32_t* state;  // {token, pos, kv_len, pad}
    uint16_t* x;           // bf16 [hidden]: the step's input (embedding row), then the last layer's output
    const uint16_t* rope_cos;
    const uint16_t* rope_sin;
    unsigned* counters;  // [nlayers * kCounterStride]
    unsigned* misc;      // [0] abort flag, [1] final ticket
    float* gslot[4];     // per op: [groups][gslots][64] partial sums
    float* apart;        // [kvh][kAttMaxSplits][gq][hd + 4] attention partials
    int* err;
    int gslots, ring_slots;
    int groups[4], nbpt[4];
    int work_bytes, xs_bytes, bias_rows;
    // debug / test hooks (all off in the production launch):
    uint16_t* taps;       // nullptr, or bf16 [nlayers][tap_stride] intermediates (layout in tap_offsets)
    int tap_stride;
    uint32_t spin_limit;  // polls of one dependency wait before it gives up
    int stall_counter;    // -1, or the counter (layer 0) whose wait target is made unreachable
};

// Offsets of the intermediates inside one layer's tap record (bf16 values):
// xn = RMSNorm(x) [hidden], q, k, v after bias + RoPE [q_heads*hd, 2 x kv_heads*hd],
// attention output [q_heads*hd], x1 = x + o_proj [hidden], xn2 [hidden],
// h = SwiGLU [inter], x2 = x1 + down [hidden].
struct TapOffsets {
    int xn, q, k, v, att, x1, xn2, h, x2, stride;
};
__host__ __device__ inline TapOffsets tap_offsets(int hidden, int qh, int kvh, int hd, int inter) {
    TapOffsets t;
    t.xn = 0;
    t.q = t.xn + hidden;
    t.k = t.q + qh * hd;
    t.v = t.k + kvh * hd;
    t.att = t.v + kvh * hd;
    t.x1 = t.att + qh * hd;
    t.xn2 = t.x1 + hidden;
    t.h = t.xn2 + hidden;
    t.x2 = t.h + inter;
    t.stride = t.x2 + hidden;
    return t;
}
__device__ __forceinline__ uint16_t* layer_taps(const PersistArgs& a, int layer) {
    return a.taps == nullptr ? nullptr : a.taps + static_cast<int64_t>(layer) * a.tap_stride;
}
__device__ __forceinline__ TapOffsets tap_offsets(const PersistArgs& a) {
    return tap_offsets(a.hidden, a.qh, a.kvh, a.hd, a.inter);
}

// ------------------------------------------------------------------ small helpers
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(s));
    return d;
}
__device__ __forceinline__ void mma16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Pair-table lookup of byte j of w (selector 0x55j4): entry row byte << 8, lane replica lane << 2.
__device__ __forceinline__ uint32_t lut_pair(const uint8_t* lut, uint32_t w, uint32_t sel, uint32_t lane4) {
    return *reinterpret_cast<const uint32_t*>(lut + prmt(w, lane4, sel));
}
// One 512-byte unit: rows g and g + 8 of a 16-row tile over one 64-element
// block.  w.x, w.y hold 8 bytes of row g; w.z, w.w 8 bytes of row g + 8.
// Returns the batch-column-0 sums (c0: row g, c2: row g + 8).
__device__ __forceinline__ float2 unit_dot(const uint8_t* lut, uint32_t lane4, uint4 w, uint4 x0, uint4 x1) {
    float c[4] = {0.F, 0.F, 0.F, 0.F};
    mma16816(c, lut_pair(lut, w.x, 0x5504u, lane4), lut_pair(lut, w.z, 0x5504u, lane4),
             lut_pair(lut, w.x, 0x5514u, lane4), lut_pair(lut, w.z, 0x5514u, lane4), x0.x, x0.y);
    mma16816(c, lut_pair(lut, w.x, 0x5524u, lane4), lut_pair(lut, w.z, 0x5524u, lane4),
             lut_pair(lut, w.x, 0x5534u, lane4), lut_pair(lut, w.z, 0x5534u, lane4), x0.z, x0.w);
    mma16816(c, lut_pair(lut, w.y, 0x5504u, lane4), lut_pair(lut, w.w, 0x5504u, lane4),
             lut_pair(lut, w.y, 0x5514u, lane4), lut_pair(lut, w.w, 0x5514u, lane4), x1.x, x1.y);
    mma16816(c, lut_pair(lut, w.y, 0x5524u, lane4), lut_pair(lut, w.w, 0x5524u, lane4),
             lut_pair(lut, w.y, 0x5534u, lane4), lut_pair(lut, w.w, 0x5534u, lane4), x1.z, x1.w);
    return make_float2(c[0], c[2]);
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
    asm volatile("fence.acq_rel.gpu;\n\tred.relaxed.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Thread 0 waits until *ctr >= target (or the step was aborted); then the
// whole CTA continues (the barrier orders every thread's later reads after
// the acquire).  A wait that runs out raises the abort flag and error bit 4.
__device__ void cta_wait(const PersistArgs& a, const unsigned* ctr, unsigned target) {
    if (threadIdx.x == 0) {
        if (a.stall_counter >= 0 && ctr == a.counters + a.stall_counter) ++target;  // test hook: never reached
        uint32_t n = 0;
        while (ld_acquire(ctr) < target) {
            if (ld_acquire(a.misc) != 0u) break;
            if (++n > a.spin_limit) {
                atomicExch(a.misc, 1u);
                atomicOr(a.err, 16);
                break;
            }
        }
    }
    __syncthreads();
}
// After every thread of the CTA wrote its part: one release increment.
__device__ __forceinline__ void cta_signal(unsigned* ctr) {
    __syncthreads();
    if (threadIdx.x == 0) red_release_add(ctr, 1u);
}

// ------------------------------------------------------------------ op geometry
struct OpRange {
    int c0, c1, w0, w1;  // this CTA's chunk range and this warp's part of it
    int nbpt, groups;
};

// Per-CTA table of every op's chunk ranges (all index math fits in 32 bits,
// checked on the host): [op][0] = c0, [op][1 + w] = warp w's first chunk,
// [op][17] = c1.  Filled once per launch.
constexpr int kRangeStride = kPWarps + 2;
__device__ __forceinline__ void fill_ranges(const PersistArgs& a, int* rng) {
    const int G = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
    for (int i = threadIdx.x; i < 4 * kRangeStride; i += kPThreads) {
        const int op = i / kRangeStride, k = i - op * kRangeStride;
        const int T = a.groups[op] * a.nbpt[op];
        const int c0 = cta * T / G, c1 = (cta + 1) * T / G;
        rng[i] = k == 0 ? c0 : k == kRangeStride - 1 ? c1 : c0 + (k - 1) * (c1 - c0) / kPWarps;
    }
}
__device__ __forceinline__ OpRange op_range(const PersistArgs& a, const int* rng, int op, int warp) {
    OpRange r;
    r.nbpt = a.nbpt[op];
    r.groups = a.groups[op];
    const int* q = rng + op * kRangeStride;
    r.c0 = q[0];
    r.c1 = q[kRangeStride - 1];
    r.w0 = q[1 + warp];
    r.w1 = warp + 1 < kPWarps ? q[2 + warp] : r.c1;
    return r;
}
// first CTA whose chunk range contains chunk q of an op with T chunks
__device__ __forceinline__ int chunk_owner(int q, int T) {
    return ((q + 1) * static_cast<int>(gridDim.x) - 1) / T;
}

// Sum of one group row's slots in slot order (= CTA order: deterministic).
// The loads are unrolled and predicated so they are all in flight at once.
template <int MAXN>
__device__ __forceinline__ float gather(const PersistArgs& a, const uint8_t* nsl, int op, int grp, int rr) {
    const float* p = a.gslot[op] + static_cast<size_t>(grp) * a.gslots * 64 + rr;
    const int n = nsl[op * kMaxGroups + grp];
    float v[MAXN];
#pragma unroll
    for (int j = 0; j < MAXN; ++j) v[j] = j < n ? __ldcg(p + j * 64) : 0.F;
    float s = 0.F;
#pragma unroll
    for (int j = 0; j < MAXN; ++j) s += v[j];
    return s;
}
// the same for four consecutive group rows rr .. rr + 3 (rr % 4 == 0)
template <int MAXN>
__device__ __forceinline__ float4 gather4(const PersistArgs& a, const uint8_t* nsl, int op, int grp, int rr) {
    const float4* p = reinterpret_cast<const float4*>(a.gslot[op] + static_cast<size_t>(grp) * a.gslots * 64 + rr);
    const int n = nsl[op * kMaxGroups + grp];
    float4 v[MAXN];
#pragma unroll
    for (int j = 0; j < MAXN; ++j) v[j] = j < n ? __ldcg(p + j * 16) : make_float4(0.F, 0.F, 0.F, 0.F);
    float4 s = make_float4(0.F, 0.F, 0.F, 0.F);
#pragma unroll
    for (int j = 0; j < MAXN; ++j) {
        s.x += v[j].x;
        s.y += v[j].y;
        s.z += v[j].z;
        s.w += v[j].w;
    }
    return s;
}
constexpr int kMaxSlotsGu = 3;   // gate/up groups span at most this many CTAs (checked on the host)
constexpr int kMaxSlots = 6;     // every other op

// The 64-element input blocks one CTA's chunk range of an op reads:
// (lo + i) % nbpt for i < n.
struct BlockSet {
    int lo, n, nbpt;
};
__device__ __forceinline__ BlockSet op_blocks(const PersistArgs& a, const int* rng, int op) {
    const OpRange r = op_range(a, rng, op, 0);
    BlockSet b;
    b.nbpt = r.nbpt;
    b.lo = r.c0 % r.nbpt;
    b.n = min(r.c1 - r.c0, r.nbpt);
    return b;
}

// ------------------------------------------------------------------ per-warp weight stream
struct Stream {  // producer cursor (lane 0)
    int layer, op;
    int c, end;
    bool done;
    const int* rng;
};

__device__ __forceinline__ void stream_normalise(const PersistArgs& a, Stream& s, int warp) {
    while (!s.done && s.c >= s.end) {
        if (++s.op == 4) {
            s.op = 0;
            if (++s.layer == a.nlayers) {
                s.done = true;
                break;
            }
        }
        const OpRange r = op_range(a, s.rng, s.op, warp);
        s.c = r.w0;
        s.end = r.w1;
    }
}

__device__ __forceinline__ void stream_issue(const PersistArgs& a, Stream& s, int warp, uint8_t* ring, uint64_t* bars,
                                             int slot) {
    stream_normalise(a, s, warp);
    if (s.done) return;
    const uint64_t* L = a.layers + static_cast<int64_t>(s.layer) * kLayerSlots;
    const uint8_t* codes = reinterpret_cast<const uint8_t*>(L[2 * s.op]) + static_cast<size_t>(s.c) * kChunkCodes;
    const uint8_t* absm = reinterpret_cast<const uint8_t*>(L[2 * s.op + 1]) + static_cast<size_t>(s.c) * kChunkAbs;
    uint8_t* dst = ring + slot * kChunkBytes;
    mbar_arrive_expect_tx(&bars[slot], kChunkBytes);
    bulk_g2s(dst, codes, kChunkCodes, &bars[slot]);
    bulk_g2s(dst + kChunkCodes, absm, kChunkAbs, &bars[slot]);
#ifdef KC_PERSIST_L2PF
    if (s.layer + 1 < a.nlayers) {  // the same chunk of the next layer into L2 (no data returns to the SM)
        const uint64_t* Ln = L + kLayerSlots;
        const uint8_t* cn = reinterpret_cast<const uint8_t*>(Ln[2 * s.op]) + static_cast<size_t>(s.c) * kChunkCodes;
        const uint8_t* an = reinterpret_cast<const uint8_t*>(Ln[2 * s.op + 1]) + static_cast<size_t>(s.c) * kChunkAbs;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(cn), "r"(kChunkCodes) : "memory");
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(an), "r"(kChunkAbs) : "memory");
    }
#endif
    ++s.c;
}

struct ConsumerState {
    int slot;
    uint32_t parity;
    bool failed;  // a ring wait ran out: no further waits or refills this step
};

// After a ring wait ran out: every slot of this warp's ring may still have a
// bulk copy in flight (one each, issued before the failure; none is issued
// after it).  Lane 0 waits for them, bounded, in ring order from the slot that
// failed, so no copy still writes into shared memory once the CTA has exited.
__device__ __noinline__ void ring_drain(uint64_t* bars, int ring_slots, int slot, uint32_t parity) {
    for (int i = 0; i < ring_slots; ++i) {
        for (int retry = 0; retry < 4 && !mbar_wait_bounded(&bars[slot], parity); ++retry) {
        }
        if (++slot == ring_slots) {
            slot = 0;
            parity ^= 1u;
        }
    }
}

// ------------------------------------------------------------------ one GEMV op of one layer
// xs holds the f16 input vector.  Every warp consumes its chunk range from its
// ring, refilling each slot from the producer cursor as soon as it is read;
// the CTA then publishes one partial slot per row group it touched.
template <int OP>
__device__ void gemv_op(const PersistArgs& a, int layer, const uint8_t* lut, uint8_t* ring, uint64_t* bars,
                        Stream& ps, ConsumerState& cs, const uint16_t* xs, float* part) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const OpRange r = op_range(a, ps.rng, OP, warp);
    const int nbpt = r.nbpt;
    const int first_grp = r.c0 / nbpt;
    const int nlg = r.c1 > r.c0 ? (r.c1 - 1) / nbpt - first_grp + 1 : 0;
    const uint32_t lane4 = static_cast<uint32_t>(lane) << 2;

    int cgrp = r.w0 / nbpt, cblk = r.w0 % nbpt;
    float acc[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = 0.F;
    uint4 x0 = make_uint4(0, 0, 0, 0), x1 = x0;
    for (int c = r.w0; c < r.w1; ++c) {
        if (!cs.failed && !mbar_wait_bounded(&bars[cs.slot], cs.parity)) {
            cs.failed = true;
            if (lane == 0) {
                atomicExch(a.misc, 1u);
                atomicOr(a.err, 16);
                ring_drain(bars, a.ring_slots, cs.slot, cs.parity);
            }
            __syncwarp();
        }
        const uint8_t* st = ring + cs.slot * kChunkBytes;
        if (g == 0) {  // only batch column 0 of B matters: lanes 0..3 carry x
            const uint4* xp = reinterpret_cast<const uint4*>(xs + cblk * 64 + 16 * t);
            x0 = xp[0];
            x1 = xp[1];
        }
        float4 aA = make_float4(0.F, 0.F, 0.F, 0.F), aB = aA;
        if (t == 0) {
            aA = reinterpret_cast<const float4*>(st + kChunkCodes)[g];
            aB = reinterpret_cast<const float4*>(st + kChunkCodes)[8 + g];
        }
        const float sA[4] = {aA.x, aA.y, aA.z, aA.w};
        const float sB[4] = {aB.x, aB.y, aB.z, aB.w};
#pragma unroll
        for (int ti = 0; ti < 4; ++ti) {
            const uint4 w = reinterpret_cast<const uint4*>(st + ti * 512)[lane];
            const float2 pr = unit_dot(lut, lane4, w, x0, x1);
            acc[ti][0] = fmaf(pr.x, sA[ti], acc[ti][0]);
            acc[ti][1] = fmaf(pr.y, sB[ti], acc[ti][1]);
        }
        __syncwarp();
        if (lane == 0 && !cs.failed) {
            fence_proxy_async_smem();  // this slot's generic reads before the async-proxy refill
            stream_issue(a, ps, warp, ring, bars, cs.slot);
        }
        if (++cs.slot == a.ring_slots) {
            cs.slot = 0;
            cs.parity ^= 1u;
        }
        if (++cblk == nbpt) {
            if (t == 0) {
                float* pp = part + ((cgrp - first_grp) * kPWarps + warp) * 64;
#pragma unroll
                for (int ti = 0; ti < 4; ++ti) {
                    pp[ti * 16 + g] = acc[ti][0];
                    pp[ti * 16 + 8 + g] = acc[ti][1];
                }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = 0.F;
            cblk = 0;
            ++cgrp;
        }
    }
    [[maybe_unused]] constexpr int kStampBase = OP == kPQkv ? 3 : OP == kPO ? 10 : OP == kPGu ? 15 : 20;
    KC_STAMP(layer, kStampBase);  // warp 0's chunks done
    if (r.w1 > r.w0 && cblk != 0 && t == 0) {
        float* pp = part + ((cgrp - first_grp) * kPWarps + warp) * 64;
#pragma unroll
        for (int ti = 0; ti < 4; ++ti) {
            pp[ti * 16 + g] = acc[ti][0];
            pp[ti * 16 + 8 + g] = acc[ti][1];
        }
    }
    __syncthreads();
    KC_STAMP(layer, kStampBase + 1);  // every warp's chunks done
    // fixed-order reduction over the 16 warps -> one slot per touched group
    const int T = r.groups * nbpt;
    for (int idx = tid; idx < nlg * 64; idx += kPThreads) {
        const int lg = idx >> 6, rr = idx & 63, grp = first_grp + lg;
        float v = 0.F;
#pragma unroll 4
        for (int w = 0; w < kPWarps; ++w) v += part[(lg * kPWarps + w) * 64 + rr];
        const int j = static_cast<int>(blockIdx.x) - chunk_owner(grp * nbpt, T);
        a.gslot[OP][(static_cast<size_t>(grp) * a.gslots + j) * 64 + rr] = v;
    }
    KC_STAMP(layer, 23 + OP);  // partial slots written
    cta_signal(a.counters + layer * kCounterStride + (OP == kPQkv ? kCQkv : OP == kPO ? kCO : OP == kPGu ? kCGu : kCDn));
    KC_STAMP(layer, kStampBase + 2);  // partials published
}

// ------------------------------------------------------------------ staging
// x (bf16, shared) += bf16(sum of the op's slots)  -- the HF residual add
__device__ void residual_from_slots(const PersistArgs& a, const uint8_t* nsl, int op, uint16_t* xres) {
#pragma unroll 2
    for (int q = threadIdx.x; q < a.hidden / 4; q += kPThreads) {
        const int r = 4 * q;
        const float4 v = gather4<kMaxSlots>(a, nsl, op, r >> 6, r & 63);
        const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; ++k)
            xres[r + k] = f32_to_bf16_bits(bf16_bits_to_f32(xres[r + k]) + round_bf16(vv[k]));
    }
}

// xs = f16(RMSNorm_HF(x) * w): x_norm = bf16(w * bf16(x * rsqrt(mean(x^2) + eps)));
// w was loaded into registers before the dependency wait.
constexpr int kNormPer = 4;  // hidden <= 8 * 512 * 4
__device__ __forceinline__ void norm_prefetch(const PersistArgs& a, const uint16_t* w, uint4* wv) {
#pragma unroll
    for (int i = 0; i < kNormPer; ++i) {
        const int o = threadIdx.x + i * kPThreads;
        if (o < a.hidden / 8) wv[i] = __ldg(reinterpret_cast<const uint4*>(w + 8 * o));
    }
}
__device__ void stage_norm(const PersistArgs& a, const uint16_t* xres, const uint4* wv, uint16_t* xs, float* red,
                           uint16_t* tap) {
    const int tid = threadIdx.x;
    const int n8 = a.hidden / 8;
    float ss = 0.F;
    for (int i = tid; i < a.hidden; i += kPThreads) {
        const float v = bf16_bits_to_f32(xres[i]);
        ss += v * v;
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.F;
#pragma unroll
    for (int i = 0; i < kPWarps; ++i) tot += red[i];
    const float inv = 1.0F / sqrtf(tot / static_cast<float>(a.hidden) + a.eps);
    bool overflow = false;
#pragma unroll
    for (int i = 0; i < kNormPer; ++i) {
        const int o = tid + i * kPThreads;
        if (o < n8) {
            const uint4 xv = reinterpret_cast<const uint4*>(xres)[o];
            const uint32_t xx[4] = {xv.x, xv.y, xv.z, xv.w};
            const uint32_t ww[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
            uint32_t out[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float v[2];
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const float xe = bf16_bits_to_f32(static_cast<uint16_t>(xx[j] >> (16 * hh)));
                    const float we = bf16_bits_to_f32(static_cast<uint16_t>(ww[j] >> (16 * hh)));
                    v[hh] = round_bf16(we * round_bf16(xe * inv));
                    overflow |= !(fabsf(v[hh]) <= 65504.F);
                    if (tap != nullptr) tap[8 * o + 2 * j + hh] = f32_to_bf16_bits(v[hh]);
                }
                out[j] = static_cast<uint32_t>(f32_to_f16_bits(v[0])) |
                         (static_cast<uint32_t>(f32_to_f16_bits(v[1])) << 16);
            }
            reinterpret_cast<uint4*>(xs)[o] = make_uint4(out[0], out[1], out[2], out[3]);
        }
    }
    if (overflow) atomicOr(a.err, 1);
}

// xs[j] = f16(h_j), h_j = bf16(bf16(silu(bf16 gate_j)) * bf16 up_j), from the
// gate/up slots, for the h blocks this CTA's share of down reads
__device__ void stage_swiglu(const PersistArgs& a, const int* rng, const uint8_t* nsl, uint16_t* xs, uint16_t* tap) {
    const BlockSet bs = op_blocks(a, rng, kPDn);
    bool overflow = false;
#pragma unroll 2
    for (int idx = threadIdx.x; idx < bs.n * 16; idx += kPThreads) {
        const int b = (bs.lo + (idx >> 4)) % bs.nbpt;
        const int j = 64 * b + 4 * (idx & 15);  // h index of four consecutive elements
        const int grp = j >> 5, rr = j & 31;
        const float4 gs = gather4<kMaxSlotsGu>(a, nsl, kPGu, grp, rr);
        const float4 us = gather4<kMaxSlotsGu>(a, nsl, kPGu, grp, rr + 32);
        const float gg[4] = {gs.x, gs.y, gs.z, gs.w}, uu[4] = {us.x, us.y, us.z, us.w};
        uint16_t hb[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float g = round_bf16(gg[k]);
            const float u = round_bf16(uu[k]);
            const float act = round_bf16(g / (1.0F + expf(-g)));
            const float hv = round_bf16(act * u);
            overflow |= !(fabsf(hv) <= 65504.F);
            hb[k] = f32_to_f16_bits(hv);
            if (tap != nullptr) tap[j + k] = f32_to_bf16_bits(hv);
        }
        *reinterpret_cast<uint2*>(xs + j) = make_uint2(hb[0] | (static_cast<uint32_t>(hb[1]) << 16),
                                                       hb[2] | (static_cast<uint32_t>(hb[3]) << 16));
    }
    if (overflow) atomicOr(a.err, 1);
}

// ------------------------------------------------------------------ attention
// A split of one KV head covers ts tokens (a multiple of kAttTile) in tiles of
// kAttTile tokens.  The tile's K and V rows land in padded shared rows by
// per-row bulk copies (the first tile's are issued before the split waits for
// q), then scores and P.V run on the tensor core, as in the cluster GQA
// kernel (gqa_decode.cu): mma.m16n8k16 bf16 with the group's query heads in
// A rows 0..gq-1 and 8 tokens per n-tile, q and K exact in bf16 with fp32
// accumulation; P split into bf16 hi + lo halves (P = hi + lo to ~16
// significant bits) against ldmatrix.trans V fragments.
struct AttPlan {
    int ns, ts;  // splits per KV head, tokens per split (a multiple of kAttTile)
};
__device__ __forceinline__ AttPlan att_plan(const PersistArgs& a, int kv_len) {
    AttPlan p;
    const int per_head = max(1, min(kAttMaxSplits, static_cast<int>(gridDim.x) / a.kvh));
    const int tiles = (kv_len + kAttTile - 1) / kAttTile;
    const int ns = min(per_head, tiles);
    p.ts = kAttTile * ((tiles + ns - 1) / ns);
    p.ns = (kv_len + p.ts - 1) / p.ts;
    return p;
}

constexpr int kKRow = 136;  // padded K/V/q row in shared memory (bf16): 272 bytes, conflict-free fragment loads

struct AttSmem {
    uint16_t* kt;  // [kAttTile][kKRow]
    uint16_t* vt;  // [kAttTile][kKRow]
    uint16_t* qb;  // [8][kKRow]: the group's q rows (bf16, unscaled), rows >= gq zero
    float* ss;     // [2][8][kAttTile]: score halves (dims 0-63, 64-127), then probabilities in [0]
    float* ml;     // [8][4]: running max, sum, correction
    float* knew;   // [hd]
    float* vnew;   // [hd]
};
constexpr int kAttSmemBytes = 2 * kAttTile * kKRow * 2 + 8 * kKRow * 2 + 2 * 8 * kAttTile * 4 + 8 * 4 * 4 + 2 * 128 * 4;
__device__ __forceinline__ AttSmem att_smem(uint8_t* work) {
    AttSmem s;
    s.kt = reinterpret_cast<uint16_t*>(work);
    s.vt = s.kt + kAttTile * kKRow;
    s.qb = s.vt + kAttTile * kKRow;
    s.ss = reinterpret_cast<float*>(s.qb + 8 * kKRow);
    s.ml = s.ss + 2 * 8 * kAttTile;
    s.knew = s.ml + 8 * 4;
    s.vnew = s.knew + 128;
    return s;
}

// Warp 0 (all lanes) issues the bulk copies of K and V rows [t0, t0 + nt) of
// one KV head into the padded tile rows, completing on `bar`.  The caller
// has ordered every earlier access to the tile rows before this (a CTA
// barrier after a proxy fence).
__device__ __forceinline__ void att_issue_tile(const uint16_t* kc, const uint16_t* vc, int t0, int nt,
                                               const AttSmem& sm, uint64_t* bar) {
    const int lane = threadIdx.x & 31;
    if (lane == 0) mbar_arrive_expect_tx(bar, static_cast<uint32_t>(nt) * 512u);
    __syncwarp();
    for (int r = lane; r < nt; r += 32) {
        bulk_g2s(sm.kt + r * kKRow, kc + static_cast<int64_t>(t0 + r) * 128, 256u, bar);
        bulk_g2s(sm.vt + r * kKRow, vc + static_cast<int64_t>(t0 + r) * 128, 256u, bar);
    }
}

__device__ __forceinline__ void mma_bf16_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x2_trans(uint32_t& r0, uint32_t& r1, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
// P pair -> bf16 hi pair and lo pair with p = hi + lo
__device__ __forceinline__ void split_bf16_pair(float p0, float p1, uint32_t& hi, uint32_t& lo) {
    const float h0 = round_bf16(p0), h1 = round_bf16(p1);
    hi = static_cast<uint32_t>(f32_to_bf16_bits(h0)) | (static_cast<uint32_t>(f32_to_bf16_bits(h1)) << 16);
    lo = static_cast<uint32_t>(f32_to_bf16_bits(p0 - h0)) | (static_cast<uint32_t>(f32_to_bf16_bits(p1 - h1)) << 16);
}

// QKV group row of q/k element (head, i) for i < hd/2; its RoPE partner is 32 rows on
__device__ __forceinline__ void rope_group_row(int hd, int head, int i, int base, int& grp, int& rr) {
    grp = base + head * (hd / 64) + i / 32;
    rr = i & 31;
}

// One split (KV head hk, tokens [tok0, tok1)) of one layer: q and the new k/v
// row from the QKV slots (bias, RoPE, Transformers' rounding), the tiles'
// scores, a chunk softmax per head (log2 domain, online across tiles) and
// P.V; then the partial (max, sum, acc) per query head.  The first tile's
// copies were issued by the caller on `bar` (parity `phase`).
__device__ void attention_split(const PersistArgs& a, int layer, const uint64_t* L, const uint8_t* nsl, int pos,
                                int kv_len, const AttPlan& ap, const uint16_t* bias_s, const float* rope_s,
                                const AttSmem& sm, uint64_t* bar, uint32_t& phase) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int gq = a.qh / a.kvh, hd = a.hd, half = hd / 2;
    const int hk = static_cast<int>(blockIdx.x) / ap.ns, s = static_cast<int>(blockIdx.x) - hk * ap.ns;
    const int tok0 = s * ap.ts, tok1 = min(kv_len, tok0 + ap.ts);
    const int qg = a.qh * (hd / 64), kg = a.kvh * (hd / 64);
    const bool bias = a.bias_rows > 0;
    uint16_t* tap = s == 0 ? layer_taps(a, layer) : nullptr;
    const TapOffsets to = tap_offsets(a);
    uint16_t* kc = reinterpret_cast<uint16_t*>(L[kLKCache]) + static_cast<int64_t>(hk) * a.cap * hd;
    uint16_t* vc = reinterpret_cast<uint16_t*>(L[kLVCache]) + static_cast<int64_t>(hk) * a.cap * hd;

    // q (gq heads, bf16 into qb) and k_new: four RoPE pairs (i .. i+3, i+half .. i+half+3) per thread;
    // v_new: four plain rows per thread
    const int nq4 = (gq + 1) * (half / 4), nv4 = hd / 4;
    for (int idx = tid; idx < nq4 + nv4; idx += kPThreads) {
        if (idx < nq4) {
            const bool isq = idx < gq * (half / 4);
            const int u = isq ? idx : idx - gq * (half / 4);
            const int head = isq ? hk * gq + u / (half / 4) : hk;
            const int i = 4 * (u % (half / 4));
            int grp, rr;
            rope_group_row(hd, head, i, isq ? 0 : qg, grp, rr);
            const float4 lo4 = gather4<kMaxSlots>(a, nsl, kPQkv, grp, rr);
            const float4 hi4 = gather4<kMaxSlots>(a, nsl, kPQkv, grp, rr + 32);
            const float y0s[4] = {lo4.x, lo4.y, lo4.z, lo4.w}, y1s[4] = {hi4.x, hi4.y, hi4.z, hi4.w};
            const int row0 = (isq ? 0 : a.qh * hd) + head * hd + i;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                float y0 = round_bf16(y0s[k]), y1 = round_bf16(y1s[k]);
                if (bias) {
                    y0 = round_bf16(y0 + bf16_bits_to_f32(bias_s[row0 + k]));
                    y1 = round_bf16(y1 + bf16_bits_to_f32(bias_s[row0 + k + half]));
                }
                const float c = rope_s[i + k], sn = rope_s[half + i + k];
                const float lo = round_bf16(round_bf16(y0 * c) + round_bf16(-y1 * sn));
                const float hi = round_bf16(round_bf16(y1 * c) + round_bf16(y0 * sn));
                if (isq) {
                    const int hq = head - hk * gq;
                    sm.qb[hq * kKRow + i + k] = f32_to_bf16_bits(lo);
                    sm.qb[hq * kKRow + i + k + half] = f32_to_bf16_bits(hi);
                } else {
                    sm.knew[i + k] = lo;
                    sm.knew[i + k + half] = hi;
                }
                if (tap != nullptr) {
                    uint16_t* tp = tap + (isq ? to.q : to.k) + head * hd + i + k;
                    tp[0] = f32_to_bf16_bits(lo);
                    tp[half] = f32_to_bf16_bits(hi);
                }
            }
        } else {
            const int d = 4 * (idx - nq4), v0 = hk * hd + d;  // row within the v matrix
            const float4 y4 = gather4<kMaxSlots>(a, nsl, kPQkv, qg + kg + (v0 >> 6), v0 & 63);
            const float ys[4] = {y4.x, y4.y, y4.z, y4.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                float y = round_bf16(ys[k]);
                if (bias) y = round_bf16(y + bf16_bits_to_f32(bias_s[(a.qh + a.kvh) * hd + v0 + k]));
                sm.vnew[d + k] = y;
                if (tap != nullptr) tap[to.v + v0 + k] = f32_to_bf16_bits(y);
            }
        }
    }
    for (int i = gq * hd + tid; i < 8 * hd; i += kPThreads) sm.qb[(i / hd) * kKRow + i % hd] = 0;  // A rows >= gq
    if (tid < 8) {
        sm.ml[tid * 4 + 0] = -INFINITY;
        sm.ml[tid * 4 + 1] = 0.F;
        sm.ml[tid * 4 + 2] = 1.F;
    }
    __syncthreads();
    // q A fragments (rows 8..15 of A are zero): k-step s8 covers dims 16*s8 .. 16*s8+15
    uint32_t qa[8][2];
    {
        const uint32_t* qw = reinterpret_cast<const uint32_t*>(sm.qb + g * kKRow);
#pragma unroll
        for (int s8 = 0; s8 < 8; ++s8) {
            qa[s8][0] = qw[8 * s8 + t];
            qa[s8][1] = qw[8 * s8 + t + 4];
        }
    }
    float o0[4] = {0.F, 0.F, 0.F, 0.F}, o1[4] = {0.F, 0.F, 0.F, 0.F};  // warp w: dims 8w .. 8w+7 of head g
    const uint32_t vbase = smem_u32(sm.vt) + static_cast<uint32_t>((lane & 15) * kKRow * 2 + 16 * warp);
    for (int t0 = tok0; t0 < tok1; t0 += kAttTile) {
        const int nt = min(kAttTile, tok1 - t0);
        if (t0 != tok0) {  // every thread is done with the previous tile's rows
            fence_proxy_async_smem();
            __syncthreads();
            if (warp == 0) att_issue_tile(kc, vc, t0, nt, sm, bar);
        }
        if (!mbar_wait_bounded(bar, phase)) {
            if (tid == 0) {
                atomicExch(a.misc, 1u);
                atomicOr(a.err, 16);
            }
            for (int retry = 0; retry < 8 && !mbar_wait_bounded(bar, phase); ++retry) {
            }
        }
        phase ^= 1u;
        const int n16 = (nt + 15) & ~15;
        if (pos >= t0 && pos < t0 + nt) {  // this step's row: computed above, also appended to the caches
            for (int d = tid; d < hd; d += kPThreads) {
                const uint16_t kb = f32_to_bf16_bits(sm.knew[d]), vb = f32_to_bf16_bits(sm.vnew[d]);
                sm.kt[(pos - t0) * kKRow + d] = kb;
                sm.vt[(pos - t0) * kKRow + d] = vb;
                kc[static_cast<int64_t>(pos) * hd + d] = kb;
                vc[static_cast<int64_t>(pos) * hd + d] = vb;
            }
        }
        // V rows nt .. n16-1 take part in the last P.V k-step with P = 0: make them finite
        for (int i = tid; i < (n16 - nt) * (hd / 2); i += kPThreads)
            reinterpret_cast<uint32_t*>(sm.vt + (nt + i / (hd / 2)) * kKRow)[i % (hd / 2)] = 0u;
        __syncthreads();
        // scores: unit (n-tile of 8 tokens, dim half) per warp, two accumulators over the half's four k-steps
        if (warp < (n16 >> 3) * 2) {
            const int ntl = warp >> 1, hf = warp & 1;
            float c0[4] = {0.F, 0.F, 0.F, 0.F}, c1[4] = {0.F, 0.F, 0.F, 0.F};
            const uint8_t* krow = reinterpret_cast<const uint8_t*>(sm.kt) + (ntl * 8 + g) * kKRow * 2 + 4 * t + 128 * hf;
#pragma unroll
            for (int s4 = 0; s4 < 4; s4 += 2) {
                const uint32_t qA0 = hf ? qa[4 + s4][0] : qa[s4][0], qA1 = hf ? qa[4 + s4][1] : qa[s4][1];
                const uint32_t qB0 = hf ? qa[5 + s4][0] : qa[s4 + 1][0], qB1 = hf ? qa[5 + s4][1] : qa[s4 + 1][1];
                mma_bf16_16816(c0, qA0, 0u, qA1, 0u, *reinterpret_cast<const uint32_t*>(krow + 32 * s4),
                               *reinterpret_cast<const uint32_t*>(krow + 32 * s4 + 16));
                mma_bf16_16816(c1, qB0, 0u, qB1, 0u, *reinterpret_cast<const uint32_t*>(krow + 32 * s4 + 32),
                               *reinterpret_cast<const uint32_t*>(krow + 32 * s4 + 48));
            }
            if (g < gq) {
                *reinterpret_cast<float2*>(sm.ss + (hf * 8 + g) * kAttTile + ntl * 8 + 2 * t) =
                    make_float2((c0[0] + c1[0]) * a.scale_log2, (c0[1] + c1[1]) * a.scale_log2);
            }
        }
        __syncthreads();
        // online softmax per head over the tile (log2 domain); probabilities zero past nt
        if (warp < gq) {
            float v[2];
            float mx = -INFINITY;
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int j = lane + 32 * k;
                v[k] = j < nt ? sm.ss[warp * kAttTile + j] + sm.ss[(8 + warp) * kAttTile + j] : -INFINITY;
                mx = fmaxf(mx, v[k]);
            }
            mx = warp_max(mx);
            const float m_old = sm.ml[warp * 4 + 0];
            const float m_new = fmaxf(m_old, mx);
            float ls = 0.F;
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int j = lane + 32 * k;
                const float p = j < nt ? exp2f(v[k] - m_new) : 0.F;
                if (j < n16) sm.ss[warp * kAttTile + j] = p;
                ls += p;
            }
            ls = warp_sum(ls);
            if (lane == 0) {
                const float corr = m_old == -INFINITY ? 0.F : exp2f(m_old - m_new);
                sm.ml[warp * 4 + 0] = m_new;
                sm.ml[warp * 4 + 1] = sm.ml[warp * 4 + 1] * corr + ls;
                sm.ml[warp * 4 + 2] = corr;
            }
        }
        __syncthreads();
        // P.V: warp w owns dims 8w .. 8w+7; k-steps of 16 tokens alternate between two accumulators
        if (warp < hd / 8) {
            const float corr = g < gq ? sm.ml[g * 4 + 2] : 1.F;
            o0[0] *= corr;
            o0[1] *= corr;
            o1[0] *= corr;
            o1[1] *= corr;
            const float* prow = sm.ss + (g < gq ? g : 0) * kAttTile + 2 * t;
            const int nk = n16 >> 4;
            for (int kk = 0; kk < nk; kk += 2) {
                const bool two = kk + 1 < nk;
                uint32_t b0, b1, b2 = 0u, b3 = 0u;
                ldsm_x2_trans(b0, b1, vbase + static_cast<uint32_t>(kk * 16 * kKRow * 2));
                if (two) ldsm_x2_trans(b2, b3, vbase + static_cast<uint32_t>((kk + 1) * 16 * kKRow * 2));
                float2 pa = make_float2(0.F, 0.F), pb = pa, pc = pa, pd = pa;
                if (g < gq) {
                    pa = *reinterpret_cast<const float2*>(prow + kk * 16);
                    pb = *reinterpret_cast<const float2*>(prow + kk * 16 + 8);
                    if (two) {
                        pc = *reinterpret_cast<const float2*>(prow + kk * 16 + 16);
                        pd = *reinterpret_cast<const float2*>(prow + kk * 16 + 24);
                    }
                }
                uint32_t ah0, al0, ah2, al2, ch0, cl0, ch2, cl2;
                split_bf16_pair(pa.x, pa.y, ah0, al0);
                split_bf16_pair(pb.x, pb.y, ah2, al2);
                split_bf16_pair(pc.x, pc.y, ch0, cl0);
                split_bf16_pair(pd.x, pd.y, ch2, cl2);
                mma_bf16_16816(o0, ah0, 0u, ah2, 0u, b0, b1);
                if (two) mma_bf16_16816(o1, ch0, 0u, ch2, 0u, b2, b3);
                mma_bf16_16816(o0, al0, 0u, al2, 0u, b0, b1);
                if (two) mma_bf16_16816(o1, cl0, 0u, cl2, 0u, b2, b3);
            }
        }
    }
    const int rec = hd + 4;
    float* mine = a.apart + ((static_cast<size_t>(hk) * kAttMaxSplits + s) * gq) * rec;
    if (warp < hd / 8 && g < gq)
        *reinterpret_cast<float2*>(mine + g * rec + 4 + 8 * warp + 2 * t) = make_float2(o0[0] + o1[0], o0[1] + o1[1]);
    if (tid < gq) {
        mine[tid * rec + 0] = sm.ml[tid * 4 + 0];
        mine[tid * rec + 1] = sm.ml[tid * 4 + 1];
    }
    cta_signal(a.counters + layer * kCounterStride + kCAtt);
}

// xs = f16(attention output) for the input blocks this CTA's share of o_proj
// reads.  First every (query head, split) pair's softmax weight w = 2^(m -
// M) / sum_s 2^(m_s - M) l_s is formed once (one warp per head, one lane per
// split, at most 32 splits) into shared memory; then four lanes per output
// quad sum w x acc over disjoint split subsets with float4 loads of the
// accumulators and a fixed shuffle order -- every CTA forms the same bits.
__device__ void stage_attention(const PersistArgs& a, const int* rng, const AttPlan& ap, uint16_t* xs, float* wn,
                                uint16_t* tap) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gq = a.qh / a.kvh, hd = a.hd, rec = hd + 4;
    for (int head = warp; head < a.qh; head += kPWarps) {
        const int hk = head / gq, hq = head - hk * gq;
        const float* p = a.apart + ((static_cast<size_t>(hk) * kAttMaxSplits + lane) * gq + hq) * rec;
        const bool live = lane < ap.ns;
        const float m = live ? __ldcg(p) : -INFINITY;
        const float l = live ? __ldcg(p + 1) : 0.F;
        const float M = warp_max(m);
        const float e = live && m != -INFINITY ? exp2f(m - M) : 0.F;
        const float den = warp_sum(e * l);
        wn[head * kAttMaxSplits + lane] = den > 0.F ? e / den : 0.F;
    }
    __syncthreads();
    const BlockSet bs = op_blocks(a, rng, kPO);
    bool overflow = false;
    const int nq = bs.n * 16;  // output quads
    // every lane of a warp runs the same trip count (the shuffles need all 32)
    for (int base = 0; base < nq * 4; base += kPThreads) {
        const int idx = base + tid;
        const bool live = idx < nq * 4;
        const int quad = live ? idx >> 2 : 0, part = idx & 3;
        const int b = (bs.lo + (quad >> 4)) % bs.nbpt;
        const int i = 64 * b + 4 * (quad & 15);  // four consecutive outputs of one head
        const int head = i / hd, d = i - head * hd, hk = head / gq, hq = head - hk * gq;
        const float* base_p = a.apart + (static_cast<size_t>(hk) * kAttMaxSplits * gq + hq) * rec + 4 + d;
        float4 acc = make_float4(0.F, 0.F, 0.F, 0.F);
#pragma unroll
        for (int k = 0; k < kAttMaxSplits / 4; ++k) {
            const int sidx = part + 4 * k;
            if (live && sidx < ap.ns) {
                const float w = wn[head * kAttMaxSplits + sidx];
                const float4 v = __ldcg(reinterpret_cast<const float4*>(base_p + static_cast<size_t>(sidx) * gq * rec));
                acc.x = fmaf(w, v.x, acc.x);
                acc.y = fmaf(w, v.y, acc.y);
                acc.z = fmaf(w, v.z, acc.z);
                acc.w = fmaf(w, v.w, acc.w);
            }
        }
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {  // (p0 + p1) + (p2 + p3), the same order on every lane
            acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
            acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
            acc.z += __shfl_xor_sync(0xffffffffu, acc.z, o);
            acc.w += __shfl_xor_sync(0xffffffffu, acc.w, o);
        }
        if (live && part == 0) {
            const float o4[4] = {round_bf16(acc.x), round_bf16(acc.y), round_bf16(acc.z), round_bf16(acc.w)};
            uint16_t hb[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                overflow |= !(fabsf(o4[k]) <= 65504.F);
                hb[k] = f32_to_f16_bits(o4[k]);
                if (tap != nullptr) tap[i + k] = f32_to_bf16_bits(o4[k]);
            }
            *reinterpret_cast<uint2*>(xs + i) = make_uint2(hb[0] | (static_cast<uint32_t>(hb[1]) << 16),
                                                           hb[2] | (static_cast<uint32_t>(hb[3]) << 16));
        }
    }
    if (overflow) atomicOr(a.err, 1);
}

__global__ void __launch_bounds__(kPThreads, 1) decode_layers_kernel(const PersistArgs a) {
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ __align__(8) uint64_t bars_all[kPWarps * kPMaxSlots];
    __shared__ __align__(8) uint64_t att_bar;  // attention tile copies
    __shared__ float red[kPWarps];
    __shared__ uint8_t nsl[4 * kMaxGroups];  // slots per row group, per op
    __shared__ int rng[4 * kRangeStride];    // chunk ranges of this CTA and its warps, per op

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint8_t* lut = dsm;
    uint8_t* rings = dsm + kPLutBytes;
    uint8_t* work = rings + kPWarps * a.ring_slots * kChunkBytes;
    uint16_t* xs = reinterpret_cast<uint16_t*>(work);
    float* part = reinterpret_cast<float*>(work + a.xs_bytes);
    uint16_t* xres = reinterpret_cast<uint16_t*>(work + a.work_bytes);
    uint16_t* bias_s = xres + ((a.hidden + 63) & ~63);
    float* rope_s = reinterpret_cast<float*>(bias_s + ((a.bias_rows + 63) & ~63));
    uint8_t* ring = rings + warp * a.ring_slots * kChunkBytes;
    uint64_t* bars = bars_all + warp * kPMaxSlots;

    // ---- per-warp stream: start every ring before anything else (weights are static)
    fill_ranges(a, rng);
    __syncthreads();
    Stream ps;
    ps.rng = rng;
    ps.layer = 0;
    ps.op = 0;
    {
        const OpRange r0 = op_range(a, rng, 0, warp);
        ps.c = r0.w0;
        ps.end = r0.w1;
    }
    ps.done = a.nlayers < 1;
    if (lane == 0) {
        for (int s = 0; s < a.ring_slots; ++s) mbar_init(&bars[s], 1);
        if (warp == 0) mbar_init(&att_bar, 1);
        fence_mbar_init();
        for (int s = 0; s < a.ring_slots; ++s) stream_issue(a, ps, warp, ring, bars, s);
    }
    // pair table: entry e -> half2(level[e >> 4], level[e & 15]) at row e, lane replica l
    for (int i = tid; i < 256 * 8; i += kPThreads) {
        const int e = i >> 3;
        const uint32_t v = static_cast<uint32_t>(f32_to_f16_bits(kNf4Levels[e >> 4])) |
                           (static_cast<uint32_t>(f32_to_f16_bits(kNf4Levels[e & 15])) << 16);
        reinterpret_cast<uint4*>(lut + e * 256)[i & 7] = make_uint4(v, v, v, v);
    }
    // slots per row group of every op
    for (int op = 0; op < 4; ++op) {
        const int T = a.groups[op] * a.nbpt[op];
        for (int gidx = tid; gidx < a.groups[op]; gidx += kPThreads) {
            const int ts = gidx * a.nbpt[op];
            nsl[op * kMaxGroups + gidx] =
                static_cast<uint8_t>(chunk_owner(ts + a.nbpt[op] - 1, T) - chunk_owner(ts, T) + 1);
        }
    }
    const int pos = __ldcg(a.state + 1);
    int kv_len = __ldcg(a.state + 2);
    if (kv_len < 1 || kv_len > a.cap || pos < 0 || pos >= a.cap || pos >= a.max_pos || pos != kv_len - 1) {
        if (tid == 0) atomicOr(a.err, 2);
        kv_len = max(1, min(kv_len, a.cap));
    }
    const int pos_c = max(0, min(pos, min(a.cap, a.max_pos) - 1));
    {   // the residual stream (the embedding row) and this step's RoPE row
        for (int i = tid; i < a.hidden; i += kPThreads) xres[i] = __ldcg(a.x + i);
        const int half = a.hd / 2;
        for (int i = tid; i < half; i += kPThreads) {
            rope_s[i] = bf16_bits_to_f32(a.rope_cos[static_cast<int64_t>(pos_c) * half + i]);
            rope_s[half + i] = bf16_bits_to_f32(a.rope_sin[static_cast<int64_t>(pos_c) * half + i]);
        }
    }
    __syncthreads();
    const AttPlan ap = att_plan(a, kv_len);
    const bool att_cta = static_cast<int>(blockIdx.x) < a.kvh * ap.ns;
    uint32_t att_phase = 0;

    ConsumerState cs;
    cs.slot = 0;
    cs.parity = 0;
    cs.failed = false;
    uint4 wv[kNormPer];
    for (int l = 0; l < a.nlayers; ++l) {
        const uint64_t* L = a.layers + static_cast<int64_t>(l) * kLayerSlots;
        unsigned* ctr = a.counters + l * kCounterStride;
        const unsigned G = gridDim.x;
        KC_STAMP(l, 0);
        // ---- RMSNorm + QKV
        norm_prefetch(a, reinterpret_cast<const uint16_t*>(L[kLInNorm]), wv);
        if (a.bias_rows > 0) {  // q, k, v biases of this layer, for the attention CTAs
            const int nq = a.qh * a.hd, nk = a.kvh * a.hd;
            for (int i = tid; i < a.bias_rows; i += kPThreads) {
                const uint16_t* b = reinterpret_cast<const uint16_t*>(
                    L[i < nq ? kLQBias : i < nq + nk ? kLKBias : kLVBias]);
                const int j = i < nq ? i : i < nq + nk ? i - nq : i - nq - nk;
                bias_s[i] = b != nullptr ? b[j] : static_cast<uint16_t>(0);
            }
        }
        for (int i = tid; i < kPartGroups * kPWarps * 64; i += kPThreads) part[i] = 0.F;
        uint16_t* tap = layer_taps(a, l);
        const TapOffsets to = tap_offsets(a);
        const bool tap0 = tap != nullptr && blockIdx.x == 0;
        if (l > 0) {
            cta_wait(a, a.counters + (l - 1) * kCounterStride + kCDn, G);
            residual_from_slots(a, nsl, kPDn, xres);
        }
        __syncthreads();
        KC_STAMP(l, 1);
        if (l > 0 && tap0)
            for (int i = tid; i < a.hidden; i += kPThreads) layer_taps(a, l - 1)[to.x2 + i] = xres[i];
        stage_norm(a, xres, wv, xs, red, tap0 ? tap + to.xn : nullptr);
        __syncthreads();
        KC_STAMP(l, 2);
        gemv_op<kPQkv>(a, l, lut, ring, bars, ps, cs, xs, part);
        // ---- attention
        if (att_cta) {
            // issue this split's first K/V tile before waiting for q (rows of earlier steps are final)
            const AttSmem att_sm = att_smem(work);
            const int hk = static_cast<int>(blockIdx.x) / ap.ns, sp = static_cast<int>(blockIdx.x) - hk * ap.ns;
            const int tok0 = sp * ap.ts;
            const uint16_t* kc = reinterpret_cast<const uint16_t*>(L[kLKCache]) + static_cast<int64_t>(hk) * a.cap * a.hd;
            const uint16_t* vc = reinterpret_cast<const uint16_t*>(L[kLVCache]) + static_cast<int64_t>(hk) * a.cap * a.hd;
            fence_proxy_async_smem();  // the tile rows' earlier generic accesses (xs, partials) before the copies
            __syncthreads();
            if (warp == 0) att_issue_tile(kc, vc, tok0, min(kAttTile, kv_len - tok0), att_sm, &att_bar);
            cta_wait(a, ctr + kCQkv, G);
            KC_STAMP(l, 6);
            attention_split(a, l, L, nsl, pos_c, kv_len, ap, bias_s, rope_s, att_sm, &att_bar, att_phase);
            KC_STAMP(l, 7);
        }
        // ---- o_proj (its input: every split of every head)
        norm_prefetch(a, reinterpret_cast<const uint16_t*>(L[kLPostNorm]), wv);
        cta_wait(a, ctr + kCAtt, static_cast<unsigned>(a.kvh * ap.ns));
        KC_STAMP(l, 8);
        stage_attention(a, rng, ap, xs, part, tap != nullptr ? tap + to.att : nullptr);
        __syncthreads();
        KC_STAMP(l, 9);
        for (int i = tid; i < kPartGroups * kPWarps * 64; i += kPThreads) part[i] = 0.F;
        __syncthreads();
        gemv_op<kPO>(a, l, lut, ring, bars, ps, cs, xs, part);
        // ---- residual + RMSNorm + gate/up
        for (int i = tid; i < kPartGroups * kPWarps * 64; i += kPThreads) part[i] = 0.F;
        cta_wait(a, ctr + kCO, G);
        KC_STAMP(l, 13);
        residual_from_slots(a, nsl, kPO, xres);
        __syncthreads();
        if (tap0)
            for (int i = tid; i < a.hidden; i += kPThreads) tap[to.x1 + i] = xres[i];
        stage_norm(a, xres, wv, xs, red, tap0 ? tap + to.xn2 : nullptr);
        __syncthreads();
        KC_STAMP(l, 14);
        gemv_op<kPGu>(a, l, lut, ring, bars, ps, cs, xs, part);
        // ---- SwiGLU + down
        for (int i = tid; i < kPartGroups * kPWarps * 64; i += kPThreads) part[i] = 0.F;
        cta_wait(a, ctr + kCGu, G);
        KC_STAMP(l, 18);
        stage_swiglu(a, rng, nsl, xs, tap != nullptr ? tap + to.h : nullptr);
        __syncthreads();
        KC_STAMP(l, 19);
        gemv_op<kPDn>(a, l, lut, ring, bars, ps, cs, xs, part);
    }
    // ---- the last residual add, written out by CTA 0; then the last CTA to
    // finish resets the counters for the next step (every issued copy has been
    // consumed: the stream and the consumers walk the same chunk sequence)
    if (blockIdx.x == 0) {
        cta_wait(a, a.counters + (a.nlayers - 1) * kCounterStride + kCDn, gridDim.x);
        residual_from_slots(a, nsl, kPDn, xres);
        __syncthreads();
        uint16_t* last = layer_taps(a, a.nlayers - 1);
        const int x2 = tap_offsets(a).x2;
        for (int i = tid; i < a.hidden; i += kPThreads) {
            a.x[i] = xres[i];
            if (last != nullptr) last[x2 + i] = xres[i];
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned old = atomicAdd(a.misc + 1, 1u);
        if (old == gridDim.x - 1) {
            for (int i = 0; i < a.nlayers * kCounterStride; ++i) a.counters[i] = 0u;
            a.misc[0] = 0u;
            a.misc[1] = 0u;
            __threadfence();
        }
    }
}

// ------------------------------------------------------------------ re-tiling
struct RetileArgs {
    const uint8_t* packed[3];
    const float* absmax[3];
    int rows[3];
    int mode, K, hd, groups;
    uint8_t* out_codes;
    float* out_absmax;
};

// (matrix, row) of group row rr in group grp
__device__ __forceinline__ void retile_row(const RetileArgs& r, int grp, int rr, int& m, int& row) {
    if (r.mode == kRetilePlain) {
        m = 0;
        row = 64 * grp + rr;
    } else if (r.mode == kRetileSwiGlu) {
        m = rr < 32 ? 0 : 1;
        row = 32 * grp + (rr & 31);
    } else {  // q/k heads with RoPE partners 32 rows apart, then plain v rows
        const int gph = r.hd / 64;
        const int qg = r.rows[0] / r.hd * gph, kg = r.rows[1] / r.hd * gph;
        if (grp < qg + kg) {
            m = grp < qg ? 0 : 1;
            const int u = grp < qg ? grp : grp - qg;
            const int head = u / gph, mm = u - head * gph;
            row = head * r.hd + 32 * mm + (rr & 31) + (rr >= 32 ? r.hd / 2 : 0);
        } else {
            m = 2;
            row = 64 * (grp - qg - kg) + rr;
        }
    }
}

__global__ void nf4_retile_kernel(const RetileArgs r) {
    const int nbpt = r.K / 64;
    const int64_t nchunks = static_cast<int64_t>(r.groups) * nbpt;
    const int64_t total = nchunks * 128;  // 4 units x 32 lanes, 16 B each
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t ch = i >> 7;
        const int ti = static_cast<int>((i >> 5) & 3), l = static_cast<int>(i & 31);
        const int grp = static_cast<int>(ch / nbpt), b = static_cast<int>(ch - static_cast<int64_t>(grp) * nbpt);
        const int g = l >> 2, t = l & 3;
        int mA, rowA, mB, rowB;
        retile_row(r, grp, 16 * ti + g, mA, rowA);
        retile_row(r, grp, 16 * ti + 8 + g, mB, rowB);
        const uint2 pa = *reinterpret_cast<const uint2*>(r.packed[mA] + static_cast<int64_t>(rowA) * (r.K / 2) + 32 * b + 8 * t);
        const uint2 pb = *reinterpret_cast<const uint2*>(r.packed[mB] + static_cast<int64_t>(rowB) * (r.K / 2) + 32 * b + 8 * t);
        reinterpret_cast<uint4*>(r.out_codes + ch * kChunkCodes)[ti * 32 + l] = make_uint4(pa.x, pa.y, pb.x, pb.y);
        // absmax: index j = (ti * 32 + l) covers 64 entries per chunk ([half][g][tile])
        const int j = ti * 32 + l;
        if (j < 64) {
            const int hh = j >> 5, gg = (j >> 2) & 7, tt = j & 3;
            int m, row;
            retile_row(r, grp, 16 * tt + 8 * hh + gg, m, row);
            r.out_absmax[ch * 64 + j] = r.absmax[m][static_cast<int64_t>(row) * nbpt + b];
        }
    }
}

}  // namespace

int retile_groups(int mode, int rows0, int rows1, int rows2, int head_dim) {
    if (mode == kRetilePlain) return rows0 % 64 == 0 && rows0 > 0 ? rows0 / 64 : -1;
    if (mode == kRetileSwiGlu) return rows0 == rows1 && rows0 % 32 == 0 && rows0 > 0 ? rows0 / 32 : -1;
    if (mode == kRetileQkvRope) {
        if (head_dim < 64 || head_dim % 64 != 0 || rows0 % head_dim != 0 || rows1 % head_dim != 0 || rows1 != rows2 ||
            rows0 <= 0 || rows1 <= 0 || rows2 % 64 != 0)
            return -1;
        return (rows0 + rows1 + rows2) / 64;
    }
    return -1;
}

cudaError_t nf4_retile(int mode, const uint8_t* const* packed, const float* const* absmax, const int* rows, int K,
                       int head_dim, uint8_t* out_codes, float* out_absmax, cudaStream_t stream) {
    RetileArgs r;
    for (int i = 0; i < 3; ++i) {
        r.packed[i] = packed[i];
        r.absmax[i] = absmax[i];
        r.rows[i] = rows[i];
    }
    r.mode = mode;
    r.K = K;
    r.hd = head_dim;
    r.groups = retile_groups(mode, rows[0], rows[1], rows[2], head_dim);
    if (r.groups < 1 || K < 64 || K % 64 != 0) return cudaErrorInvalidValue;
    r.out_codes = out_codes;
    r.out_absmax = out_absmax;
    const int64_t total = static_cast<int64_t>(r.groups) * (K / 64) * 128;
    const int threads = 256;
    const int64_t blocks = (total + threads - 1) / threads;
    nf4_retile_kernel<<<static_cast<unsigned>(blocks < 65535 * 16 ? blocks : 65535 * 16), threads, 0, stream>>>(r);
    return cudaGetLastError();
}

// ---------------------------------------------------------------- persistent launch
namespace {
struct PersistGeom {
    int groups[4], nbpt[4];
    int gslots, xs_bytes, work_bytes, bias_rows, ring_slots;
    int64_t off_misc, off_gslot[4], off_apart, total;
    int smem;
};

// slots (contributing CTAs) of the row group with the most of them
int max_group_slots(int groups, int nbpt, int sms) {
    const int64_t T = static_cast<int64_t>(groups) * nbpt;
    int worst = 0;
    for (int g = 0; g < groups; ++g) {
        const int64_t ts = static_cast<int64_t>(g) * nbpt, te = ts + nbpt;
        const int cf = static_cast<int>(((ts + 1) * sms - 1) / T), cl = static_cast<int>((te * sms - 1) / T);
        worst = cl - cf + 1 > worst ? cl - cf + 1 : worst;
    }
    return worst;
}

constexpr int kStaticSmemBudget = 3072;  // the kernel's static shared memory, rounded up

PersistGeom persist_geom(const PersistDims& d, int sms) {
    PersistGeom g;
    g.groups[0] = (d.q_heads + 2 * d.kv_heads) * d.head_dim / 64;
    g.nbpt[0] = d.hidden / 64;
    g.groups[1] = d.hidden / 64;
    g.nbpt[1] = d.q_heads * d.head_dim / 64;
    g.groups[2] = d.intermediate / 32;
    g.nbpt[2] = d.hidden / 64;
    g.groups[3] = d.hidden / 64;
    g.nbpt[3] = d.intermediate / 64;
    g.gslots = 0;
    for (int i = 0; i < 4; ++i) {
        const int s = max_group_slots(g.groups[i], g.nbpt[i], sms);
        g.gslots = s > g.gslots ? s : g.gslots;
    }
    int kmax = d.hidden > d.intermediate ? d.hidden : d.intermediate;
    kmax = kmax > d.q_heads * d.head_dim ? kmax : d.q_heads * d.head_dim;
    g.xs_bytes = (kmax * 2 + 127) & ~127;
    const int gq = d.kv_heads > 0 ? d.q_heads / d.kv_heads : 1;
    const int work = g.xs_bytes + kPartGroups * kPWarps * 64 * 4;
    const int att = kAttSmemBytes;
    g.work_bytes = ((work > att ? work : att) + 127) & ~127;
    g.bias_rows = (d.q_heads + 2 * d.kv_heads) * d.head_dim;
    const int tail = ((d.hidden + 63) & ~63) * 2 + ((g.bias_rows + 63) & ~63) * 2 + d.head_dim * 4;
    const int limit = 232448 - kStaticSmemBudget;
    g.ring_slots = kPMaxSlots;
    while (g.ring_slots > 1 && kPLutBytes + kPWarps * g.ring_slots * kChunkBytes + g.work_bytes + tail > limit)
        --g.ring_slots;
    g.smem = kPLutBytes + kPWarps * g.ring_slots * kChunkBytes + g.work_bytes + tail;
    auto up = [](int64_t v) { return (v + 255) & ~static_cast<int64_t>(255); };
    int64_t off = up(static_cast<int64_t>(d.layers) * kCounterStride * 4);
    g.off_misc = off;
    off = up(off + 64);
    for (int i = 0; i < 4; ++i) {
        g.off_gslot[i] = off;
        off = up(off + static_cast<int64_t>(g.groups[i]) * g.gslots * 64 * 4);
    }
    g.off_apart = off;
    off = up(off + static_cast<int64_t>(d.kv_heads) * kAttMaxSplits * gq * (d.head_dim + 4) * 4);
    g.total = off;
    return g;
}
}  // namespace

int64_t decode_persistent_scratch_bytes(const PersistDims& d, int sms) { return persist_geom(d, sms).total; }

int64_t decode_persistent_tap_stride(const PersistDims& d) {
    return tap_offsets(d.hidden, d.q_heads, d.kv_heads, d.head_dim, d.intermediate).stride;
}

const char* decode_persistent_check(const PersistDims& d, int sms) {
    if (d.layers < 1 || d.hidden < 64 || d.hidden % 64 != 0 || d.head_dim != 128 || d.q_heads < 1 || d.kv_heads < 1 ||
        d.q_heads % d.kv_heads != 0 || d.q_heads / d.kv_heads > 8 || d.intermediate % 64 != 0 ||
        d.hidden > 8 * kPThreads * kNormPer || d.kv_capacity < 1 || d.kv_heads > sms)
        return "persistent decode requires hidden % 64 == 0 (<= 16384), head_dim 128, q_heads/kv_heads <= 8, "
               "intermediate % 64 == 0";
    const PersistGeom g = persist_geom(d, sms);
    if (g.smem > 232448 - kStaticSmemBudget) return "persistent decode: shapes need more shared memory than one SM has";
    for (int i = 0; i < 4; ++i) {
        const int64_t T = static_cast<int64_t>(g.groups[i]) * g.nbpt[i];
        if (T < sms) return "persistent decode: an op has fewer 64x64 chunks than the GPU has SMs";
        if (T * static_cast<int64_t>(sms + 1) >= (int64_t{1} << 31)) return "persistent decode: an op is too large";
        if (g.groups[i] > kMaxGroups) return "persistent decode: an op has more than 512 row groups";
        if ((T / sms + 2) / g.nbpt[i] + 2 > kPartGroups) return "persistent decode: an op spans too many row groups per CTA";
        const int n = max_group_slots(g.groups[i], g.nbpt[i], sms);
        if (n > (i == 2 ? kMaxSlotsGu : kMaxSlots)) return "persistent decode: a row group spans too many CTAs";
    }
    return nullptr;
}

cudaError_t decode_layers_persistent(const PersistLaunch& p, cudaStream_t stream) {
    const int sms = device_sm_count();
    const PersistGeom g = persist_geom(p.dims, sms);
    PersistArgs a;
    a.layers = p.layer_table;
    a.nlayers = p.dims.layers;
    a.hidden = p.dims.hidden;
    a.qh = p.dims.q_heads;
    a.kvh = p.dims.kv_heads;
    a.hd = p.dims.head_dim;
    a.inter = p.dims.intermediate;
    a.cap = p.dims.kv_capacity;
    a.max_pos = p.max_pos;
    a.eps = p.eps;
    a.scale_log2 = p.scale * 1.4426950408889634F;
    a.state = p.state;
    a.x = p.x;
    a.rope_cos = p.rope_cos;
    a.rope_sin = p.rope_sin;
    char* s = static_cast<char*>(p.scratch);
    a.counters = reinterpret_cast<unsigned*>(s);
    a.misc = reinterpret_cast<unsigned*>(s + g.off_misc);
    for (int i = 0; i < 4; ++i) a.gslot[i] = reinterpret_cast<float*>(s + g.off_gslot[i]);
    a.apart = reinterpret_cast<float*>(s + g.off_apart);
    a.err = p.err;
    a.gslots = g.gslots;
    a.ring_slots = g.ring_slots;
    for (int i = 0; i < 4; ++i) {
        a.groups[i] = g.groups[i];
        a.nbpt[i] = g.nbpt[i];
    }
    a.work_bytes = g.work_bytes;
    a.xs_bytes = g.xs_bytes;
    a.bias_rows = g.bias_rows;
    a.taps = p.taps;
    a.tap_stride = tap_offsets(p.dims.hidden, p.dims.q_heads, p.dims.kv_heads, p.dims.head_dim, p.dims.intermediate).stride;
    a.spin_limit = p.spin_limit > 0 ? p.spin_limit : kSpinLimit;
    a.stall_counter = p.stall_counter;
    cudaError_t st = cudaFuncSetAttribute(decode_layers_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, g.smem);
    if (st != cudaSuccess) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(sms));
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(g.smem);
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: they wait on each other
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_layers_kernel, a);
}

}  // namespace kc
