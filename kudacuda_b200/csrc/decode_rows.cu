// decode_rows.cu -- all decoder layers of one batch-1 decode step in one
// persistent cooperative launch on sm_100a, with a row-complete work split.
//
// Replaces, for the static decode plan, the per-layer launch sequence
// (RMSNorm+QKV+RoPE+append, GQA decode, o_proj+residual, RMSNorm+SwiGLU,
// down+residual) that stands in for the reference's per-op kernels
// (kernels/common/nf4_tiled_gemv.cuh:61-278, nf4_swiglu_bf16.cuh:65-209,
// qwen2_gqa_decode.cuh:17-203) and the bitsandbytes o_proj/down matmuls
// (python/kudacuda_sidecar.py:947, :1746).  Arithmetic and rounding points are
// Transformers' (those of the per-op HF-semantics kernels in nf4_gemv.cuh).
//
// Work split: every op's output rows come in 16-row tiles, and each tile is
// owned by ONE CTA that streams all of its K -- so each output value is
// finished exactly once, by its owner, with the op's epilogue: q/k after bias
// and RoPE (k and v go straight into the cache row of this step), x + o_proj,
// SwiGLU, x + down.  Consumers then read the few KB of finished values they
// need (the residual stream, q, the attention output, h) instead of summing
// partial slots.  Each warp of a CTA streams a contiguous range of the CTA's
// (tile, K-block) units through its own ring of bulk copies, and the 16
// warps' per-tile sums meet in shared memory in a fixed order (the result is
// deterministic).
//
// Unit (tile, block b): 512 code bytes -- lane 4g + t holds bytes
// [32b + 8t, +8) of tile rows g and g + 8, exactly its m16n8k16 A fragments --
// then the 16 rows' fp32 absmax of block b as (row g, row g + 8) pairs, one
// 8-byte load per lane (576 bytes; nf4_retile16_kernel
// writes them tile-major from the bitsandbytes layout).  Tile rows: q/k heads
// in tiles of 8 RoPE pairs (row r and its partner r + 8), gate/up pairs, or
// 16 consecutive rows.
//
// Dependencies (each a counter per layer: release increments by the
// producers, one acquiring thread per consumer CTA, bounded spins that abort
// the step and set bit 4 of the error word): x ready -> q/k/v (all CTAs) ->
// attention splits (a ticket per KV head picks the split that merges them)
// -> o_proj owners -> x1 ready -> gate/up (all CTAs) -> down owners -> next
// layer.
#include <cuda_runtime.h>

#include <cstdint>

#include "kc_common.cuh"
#include "kc_launch.h"

// Phase timestamps for profiling builds only (-DKC_PERSIST_STAMPS; off in the
// library): thread 0 of every CTA records %globaltimer at up to 64 fixed
// points of one layer (KC_STAMP_LAYER) into g_rows_stamps[cta][64], read back
// with kc_rows_read_stamps.  No work is skipped or added to the product build.
#ifdef KC_PERSIST_STAMPS
#ifndef KC_STAMP_LAYER
#define KC_STAMP_LAYER 18
#endif
__device__ unsigned long long g_rows_stamps[1024 * 64];
#define KR_STAMP(l, i)                                                          \
    do {                                                                        \
        if ((l) == KC_STAMP_LAYER && threadIdx.x == 0) {                        \
            unsigned long long t_;                                              \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_)::"memory");    \
            g_rows_stamps[blockIdx.x * 64 + (i)] = t_;                          \
        }                                                                       \
    } while (0)
extern "C" __attribute__((visibility("default"))) int kc_rows_read_stamps(unsigned long long* out, int n) {
    return static_cast<int>(cudaMemcpyFromSymbol(out, g_rows_stamps, sizeof(unsigned long long) * n));
}
#else
#define KR_STAMP(l, i) \
    do {               \
    } while (0)
#endif

namespace kc {
namespace {

constexpr int kRW = 16;  // warps per CTA
constexpr int kRT = kRW * 32;
#ifndef KC_ROWS_RING_MAX
#define KC_ROWS_RING_MAX 3
#endif
constexpr int kRMaxSlots = KC_ROWS_RING_MAX;
constexpr int kUnitCodes = 512;
constexpr int kUnitBytes = 576;
#ifndef KC_ROWS_SLOT_UNITS
#define KC_ROWS_SLOT_UNITS 4
#endif
constexpr int kSlotUnits = KC_ROWS_SLOT_UNITS;  // units per bulk copy / ring slot
// per-tile partial sums of the warps, part[tile][row][warp] (a row's 16 warps
// contiguous: the reducing thread reads them as four 16-byte loads); a tile's
// block is padded by 16 floats
constexpr int kPartTile = 16 * 16 + 16;
constexpr int kPartFloats = 16 * kPartTile;  // kMaxCtaTiles tiles
constexpr int kSlotBytes = kSlotUnits * kUnitBytes;
constexpr int kRLutBytes = 65536;  // 256 entry rows x 256 B, lane replicas in the first 128 B of a row
constexpr int kMaxCtaTiles = 16;   // tiles of one op one CTA may own (checked on the host)
constexpr uint32_t kRSpinLimit = 1u << 21;
constexpr int kATile = 64;         // tokens per attention tile
constexpr int kSs = kATile + 8;    // score row stride (floats): P reads of the 8 heads fall in distinct bank pairs
constexpr int kAMaxSplits = 32;    // splits per KV head
constexpr int kKRow = 136;         // padded K/V/q row in shared memory (bf16): 272 bytes
constexpr int kRngStride = kRW + 3;  // per op: t0, t1, warp unit bounds 0..16

enum RowOp { kOQkv = 0, kOO = 1, kOGu = 2, kODn = 3 };
// stall_counter test hook: the op whose output a consumer never sees (0 q/k/v, 1 attention, 2 o_proj,
// 3 gate/up, 4 down, 5 the attention splits' partials)
enum RowCtr { kCQkv = 0, kCAtt = 1, kCO = 2, kCGu = 3, kCDn = 4, kCTicket = 5 };
// hops between ops, the low 4 bits of a tag (15: never written, the test hook's unreachable tag)
enum RowHop { kHX = 0, kHQ = 1, kHK = 2, kHV = 3, kHAtt = 4, kHX1 = 5, kHH = 6, kHPart = 7, kHTpO = 8, kHTpD = 9 };
__host__ __device__ constexpr int hop_counter(int hop) {  // the stall_counter index of a hop
    return hop == kHX                      ? kCDn
           : hop <= kHV                    ? kCQkv
           : hop == kHAtt || hop == kHTpO  ? kCAtt
           : hop == kHX1                   ? kCO
           : hop == kHH || hop == kHTpD    ? kCGu
                                           : kCTicket;
}
enum RowSlot { kTUnits0 = 0, kTInNorm = 4, kTPostNorm, kTQBias, kTKBias, kTVBias, kTKCache, kTVCache, kTSlots = 16 };

struct RowArgs {
    const uint64_t* layers;  // [nlayers][kTSlots] device pointers
    int nlayers, hidden, qh, kvh, hd, inter, cap, max_pos;
    float eps, scale_log2;
    const int32_t* state;  // {token, pos, kv_len, pad}
    uint16_t* x;           // bf16 [hidden]: the step's input, then every layer's x2 (the last is the output)
    const uint16_t* rope_cos;
    const uint16_t* rope_sin;
    unsigned* misc;      // [0] abort flag, [1] final ticket, [2] launch count (the tags' epoch)
    // Tagged words carry one op's output to the next: two 16-bit values
    // (element 2 i in the low half) and, in the high 32 bits, the tag of the
    // (launch, layer, hop) that wrote them.  A consumer polls the words it
    // needs until each carries the tag it expects, so the producer publishes
    // with plain relaxed 8-byte stores: no fence, no counter, one round trip.
    uint64_t* qw;   // [qh * hd / 2] q after bias and RoPE (bf16)
    uint64_t* kw;   // [kvh * hd / 2] this step's k row (bf16; also written to the cache)
    uint64_t* vw;   // [kvh * hd / 2] this step's v row (bf16; also written to the cache)
    uint64_t* aw;   // [qh * hd / 2] attention output (f16 of the bf16 value)
    uint64_t* x1w;  // [hidden / 2] x + o_proj (bf16)
    uint64_t* hw;   // [inter / 2] SwiGLU output (f16 of the bf16 value)
    uint64_t* xw;   // [hidden / 2] x2, the next layer's input (bf16)
    // tensor parallelism: rank `rank` of `world`; peers[p] = rank p's exchange
    // buffer (this process's mapping of its peer memory): o_proj partials
    // [world][hidden] then down partials [world][hidden], tagged f32 words
    int world, rank;
    const uint64_t* peers;
    uint64_t* pw;   // [kvh][kAMaxSplits][gq][2 + hd] attention partials: max, sum, accumulator (f32 bits)
    int* err;
    int ring_slots;
    int tiles[4], nbpt[4], ctas[4];
    int kvt_off, work_bytes, bias_rows;
    uint16_t* taps;  // test hooks, as decode_persistent.cu
    int tap_stride;
    uint32_t spin_limit;
    int stall_counter;
};

// tap record offsets (the same layout as the other persistent kernel)
struct RTaps {
    int xn, q, k, v, att, x1, xn2, h, x2, stride;
};
__host__ __device__ inline RTaps rtaps(int hidden, int qh, int kvh, int hd, int inter) {
    RTaps t;
    t.xn = 0;
    t.q = hidden;
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
__device__ __forceinline__ uint16_t* rtap(const RowArgs& a, int layer) {
    return a.taps == nullptr ? nullptr : a.taps + static_cast<int64_t>(layer) * a.tap_stride;
}

// ------------------------------------------------------------------ small helpers
__device__ __forceinline__ uint32_t prmt_r(uint32_t a, uint32_t b, uint32_t s) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(s));
    return d;
}
__device__ __forceinline__ void mma_f16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Pair-table lookup of byte j of w (selector 0x55j4): entry row byte << 8, lane replica lane << 2.
__device__ __forceinline__ uint32_t lut_pair_r(const uint8_t* lut, uint32_t w, uint32_t sel, uint32_t lane4) {
    return *reinterpret_cast<const uint32_t*>(lut + prmt_r(w, lane4, sel));
}
// One unit: rows g and g + 8 of a 16-row tile over one 64-element block
// (w.x, w.y: 8 bytes of row g; w.z, w.w: 8 bytes of row g + 8); returns the
// batch-column-0 sums (row g, row g + 8), valid in lanes with t == 0.
__device__ __forceinline__ float2 unit_dot_r(const uint8_t* lut, uint32_t lane4, uint4 w, uint4 x0, uint4 x1) {
    float c[4] = {0.F, 0.F, 0.F, 0.F};
    mma_f16(c, lut_pair_r(lut, w.x, 0x5504u, lane4), lut_pair_r(lut, w.z, 0x5504u, lane4),
            lut_pair_r(lut, w.x, 0x5514u, lane4), lut_pair_r(lut, w.z, 0x5514u, lane4), x0.x, x0.y);
    mma_f16(c, lut_pair_r(lut, w.x, 0x5524u, lane4), lut_pair_r(lut, w.z, 0x5524u, lane4),
            lut_pair_r(lut, w.x, 0x5534u, lane4), lut_pair_r(lut, w.z, 0x5534u, lane4), x0.z, x0.w);
    mma_f16(c, lut_pair_r(lut, w.y, 0x5504u, lane4), lut_pair_r(lut, w.w, 0x5504u, lane4),
            lut_pair_r(lut, w.y, 0x5514u, lane4), lut_pair_r(lut, w.w, 0x5514u, lane4), x1.x, x1.y);
    mma_f16(c, lut_pair_r(lut, w.y, 0x5524u, lane4), lut_pair_r(lut, w.w, 0x5524u, lane4),
            lut_pair_r(lut, w.y, 0x5534u, lane4), lut_pair_r(lut, w.w, 0x5534u, lane4), x1.z, x1.w);
    return make_float2(c[0], c[2]);
}
__device__ __forceinline__ unsigned ld_relaxed_r(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Error bit 0 (an activation outside the f16 range) from a whole-CTA point:
// one vote per warp and one atomic from a warp that saw it, so the common
// case costs no memory operation at all.
__device__ __forceinline__ void rflag_overflow(const RowArgs& a, bool overflow) {
    if (__any_sync(0xffffffffu, overflow) && (threadIdx.x & 31) == 0)
        asm volatile("red.relaxed.gpu.global.or.b32 [%0], %1;" ::"l"(a.err), "r"(1) : "memory");
}
// Tagged words (RowArgs): aligned 8-byte strong accesses are single-copy
// atomic, so a word read with the expected tag carries that write's payload.
__device__ __forceinline__ void st_tagged(uint64_t* p, uint32_t tag, uint32_t payload) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"((static_cast<uint64_t>(tag) << 32) | payload)
                 : "memory");
}
__device__ __forceinline__ uint64_t ld_tagged(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p));
    return v;
}
// the same across GPUs: a peer's store into this GPU's memory over NVLink
__device__ __forceinline__ void st_tagged_sys(uint64_t* p, uint32_t tag, uint32_t payload) {
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"((static_cast<uint64_t>(tag) << 32) | payload)
                 : "memory");
}
__device__ __forceinline__ uint64_t ld_tagged_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p));
    return v;
}
// Every thread polls words i = tid + k * kRT (k < KMAX, i < n) until each
// carries its tag, hands each payload to sink(slot, payload), then the CTA
// synchronises.  locate(i, tag, slot) gives word i's address, expected tag
// and sink slot (computed once per word).  All of a thread's outstanding
// words are read in one round; a poll that runs out raises the abort flag and
// error bit 4 of the error word.
template <int KMAX, bool SYS = false, class Locate, class Sink>
__device__ void rpoll(const RowArgs& a, int n, Locate locate, Sink sink) {
    const int tid = threadIdx.x;
    const uint64_t* src[KMAX];
    uint32_t tag[KMAX];
    int slot[KMAX];
    uint32_t pending = 0u;
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
        src[k] = nullptr;
        tag[k] = 0u;
        slot[k] = 0;
        if (tid + k * kRT < n) {
            src[k] = locate(tid + k * kRT, tag[k], slot[k]);
            pending |= 1u << k;
        }
    }
    uint32_t rounds = 0;
    while (pending != 0u) {
        uint64_t v[KMAX];
#pragma unroll
        for (int k = 0; k < KMAX; ++k)
            v[k] = (pending >> k & 1u) != 0u ? (SYS ? ld_tagged_sys(src[k]) : ld_tagged(src[k])) : 0ull;
#pragma unroll
        for (int k = 0; k < KMAX; ++k)
            if ((pending >> k & 1u) != 0u && static_cast<uint32_t>(v[k] >> 32) == tag[k]) {
                sink(slot[k], static_cast<uint32_t>(v[k]));
                pending &= ~(1u << k);
            }
        if (pending != 0u && (++rounds & 31u) == 0u) {
            if (ld_relaxed_r(a.misc) != 0u) break;
            if (rounds > a.spin_limit) {
                atomicExch(a.misc, 1u);
                atomicOr(a.err, 16);
                break;
            }
        }
    }
    __syncthreads();
}
// The common form: words base[0 .. n) with one tag, payloads to dst[i] (32-bit shared words).
template <int KMAX>
__device__ __forceinline__ void rpoll_vec(const RowArgs& a, const uint64_t* base, int n, uint32_t tg, uint32_t* dst) {
    rpoll<KMAX>(
        a, n,
        [&](int i, uint32_t& t, int& sl) {
            t = tg;
            sl = i;
            return base + i;
        },
        [&](int sl, uint32_t p) { dst[sl] = p; });
}
// Tensor-parallel row-parallel op (o_proj or down): every rank pushed its fp32
// partial of this CTA's tiles into every rank's exchange buffer `ex`
// ([world][hidden] tagged words; the tile owners are the same CTA index on
// every rank).  Poll the world partials of each owned row from this GPU's
// buffer, sum them in rank order (every rank gets the same value), and hand
// each row to fin(row, sum, lanes) with consecutive rows in consecutive lanes.
template <class Fin>
__device__ void rtp_finish(const RowArgs& a, const int* rr, const uint64_t* ex, uint32_t tag, float* buf, Fin fin) {
    const int t0 = rr[0], nrows = 16 * (rr[1] - rr[0]), world = a.world;
    const int lane = threadIdx.x & 31;
    rpoll<4, true>(
        a, nrows * world,
        [&](int i, uint32_t& tg, int& sl) {
            const int rl = i / world, src = i - rl * world;
            tg = tag;
            sl = i;
            return ex + static_cast<int64_t>(src) * a.hidden + 16 * t0 + rl;
        },
        [&](int sl, uint32_t p) { buf[sl] = __uint_as_float(p); });
    for (int idx = threadIdx.x; idx < nrows; idx += kRT) {
        const int left = nrows - (idx - lane);
        const unsigned lanes = left >= 32 ? 0xffffffffu : (1u << left) - 1u;
        float sum = 0.F;
        for (int src = 0; src < world; ++src) sum += buf[idx * world + src];
        fin(16 * t0 + idx, sum, lanes);
    }
    __syncthreads();
}
// This rank's partial of rows row and row + 8 into every rank's exchange buffer.
__device__ __forceinline__ void rtp_push(const RowArgs& a, int part_off, int row, float lo, float hi, uint32_t tag) {
    for (int p = 0; p < a.world; ++p) {
        uint64_t* dst = reinterpret_cast<uint64_t*>(a.peers[p]) + part_off + static_cast<int64_t>(a.rank) * a.hidden;
        st_tagged_sys(dst + row, tag, __float_as_uint(lo));
        st_tagged_sys(dst + row + 8, tag, __float_as_uint(hi));
    }
}
// Pairs of consecutive rows r, r + 1 sit in lanes r, r + 1 of an 8-lane group
// of the GEMV epilogue (`lanes`: the warp's lanes in that epilogue call): the
// even lane gets its partner's 16-bit value in the high half.
__device__ __forceinline__ uint32_t pair_up(uint32_t v, unsigned lanes) {
    return v | (__shfl_down_sync(lanes, v, 1, 8) << 16);
}

// ------------------------------------------------------------------ ownership
// rng[op * kRngStride]: [0] = first owned tile, [1] = one past the last,
// [2 + w] = warp w's first unit (relative to the CTA's first unit), [2 + 16] = unit count.
__device__ __forceinline__ void fill_rng(const RowArgs& a, int* rng) {
    const int G = static_cast<int>(gridDim.x), c = static_cast<int>(blockIdx.x);
    for (int i = threadIdx.x; i < 4 * kRngStride; i += kRT) {
        const int op = i / kRngStride, k = i - op * kRngStride;
        const int T = a.tiles[op];
        const int t0 = static_cast<int>(static_cast<int64_t>(c) * T / G);
        const int t1 = static_cast<int>(static_cast<int64_t>(c + 1) * T / G);
        const int U = (t1 - t0) * a.nbpt[op];
        rng[i] = k == 0 ? t0 : k == 1 ? t1 : (k - 2) * U / kRW;
    }
}

// ------------------------------------------------------------------ per-warp unit stream
struct RStream {  // producer cursor (lane 0)
    int layer, op, u, end;
    bool done;
};
__device__ __forceinline__ void rstream_normalise(const RowArgs& a, const int* rng, RStream& s, int warp) {
    while (!s.done && s.u >= s.end) {
        if (++s.op == 4) {
            s.op = 0;
            if (++s.layer == a.nlayers) {
                s.done = true;
                break;
            }
        }
        s.u = rng[s.op * kRngStride + 2 + warp];
        s.end = rng[s.op * kRngStride + 3 + warp];
    }
}
__device__ __forceinline__ void rstream_issue(const RowArgs& a, const int* rng, RStream& s, int warp, uint8_t* ring,
                                              uint64_t* bars, int slot) {
    rstream_normalise(a, rng, s, warp);
    if (s.done) return;
    const int n = min(kSlotUnits, s.end - s.u);
    const int64_t unit = static_cast<int64_t>(rng[s.op * kRngStride]) * a.nbpt[s.op] + s.u;
    const uint8_t* src = reinterpret_cast<const uint8_t*>(a.layers[static_cast<int64_t>(s.layer) * kTSlots + s.op]) +
                         unit * kUnitBytes;
    const uint32_t bytes = static_cast<uint32_t>(n) * kUnitBytes;
    mbar_arrive_expect_tx(&bars[slot], bytes);
    bulk_g2s(ring + slot * kSlotBytes, src, bytes, &bars[slot]);
    s.u += n;
}
struct RCons {
    int slot;
    uint32_t parity;
    bool failed;
};
// After a ring wait ran out: every slot may still have a copy in flight (one
// each, none issued after the failure); lane 0 waits for them, bounded, so no
// copy writes into shared memory after the CTA has exited.
__device__ __noinline__ void rring_drain(uint64_t* bars, int ring_slots, int slot, uint32_t parity) {
    for (int i = 0; i < ring_slots; ++i) {
        for (int retry = 0; retry < 4 && !mbar_wait_bounded(&bars[slot], parity); ++retry) {
        }
        if (++slot == ring_slots) {
            slot = 0;
            parity ^= 1u;
        }
    }
}

// ------------------------------------------------------------------ one GEMV op: this CTA's tiles
// xs holds the f16 input vector.  Each warp consumes its unit range slot by
// slot, refilling each slot from the stream as soon as it is read; per-tile
// sums of the warp go to part[tile][row][warp]; then the CTA sums the warps in
// fixed order and hands every (tile, row pair) to `epi` (rows r and r + 8).
template <int OP, class Epi>
__device__ void rgemv(const RowArgs& a, int layer, const int* rng, const uint8_t* lut, uint8_t* ring, uint64_t* bars,
                      RStream& ps, RCons& cs, const uint16_t* xs, float* part, Epi epi) {
    [[maybe_unused]] constexpr int kSt = 16 + 3 * OP;  // stamps: first slot ready, warp 0 done, all warps done
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int* rr = rng + OP * kRngStride;
    const int t0 = rr[0], ntiles = rr[1] - rr[0];
    const int nbpt = a.nbpt[OP];
    const int uw0 = rr[2 + warp], uw1 = rr[3 + warp];
    for (int i = tid; i < kPartFloats; i += kRT) part[i] = 0.F;
    __syncthreads();
    const uint32_t lane4 = static_cast<uint32_t>(lane) << 2;
#ifdef KC_PERSIST_STAMPS
    long long wcyc = 0;
    const long long tloop = clock64();
#endif
    int tile = uw0 / nbpt, blk = uw0 - (uw0 / nbpt) * nbpt;
    float acc_lo = 0.F, acc_hi = 0.F;
    uint4 x0 = make_uint4(0, 0, 0, 0), x1 = x0;
    for (int u = uw0; u < uw1;) {
#ifdef KC_PERSIST_STAMPS
        const long long tw0 = clock64();
#endif
        if (!cs.failed && !mbar_wait_bounded(&bars[cs.slot], cs.parity)) {
            cs.failed = true;
            if (lane == 0) {
                atomicExch(a.misc, 1u);
                atomicOr(a.err, 16);
                rring_drain(bars, a.ring_slots, cs.slot, cs.parity);
            }
            __syncwarp();
        }
#ifdef KC_PERSIST_STAMPS
        wcyc += clock64() - tw0;
#endif
        if (u == uw0) KR_STAMP(layer, kSt);
        const uint8_t* st = ring + cs.slot * kSlotBytes;
        const int n = min(kSlotUnits, uw1 - u);
#pragma unroll
        for (int k = 0; k < kSlotUnits; ++k) {  // unrolled: consecutive units' loads and mma chains overlap
            if (k >= n) break;
            if (g == 0) {  // only batch column 0 of B matters: lanes 0..3 carry x
                const uint4* xp = reinterpret_cast<const uint4*>(xs + blk * 64 + 16 * t);
                x0 = xp[0];
                x1 = xp[1];
            }
            float aA = 0.F, aB = 0.F;
            if (t == 0) {
                const float2 am = reinterpret_cast<const float2*>(st + k * kUnitBytes + kUnitCodes)[g];
                aA = am.x;  // row g
                aB = am.y;  // row g + 8
            }
            const uint4 w = reinterpret_cast<const uint4*>(st + k * kUnitBytes)[lane];
            const float2 pr = unit_dot_r(lut, lane4, w, x0, x1);
            acc_lo = fmaf(pr.x, aA, acc_lo);
            acc_hi = fmaf(pr.y, aB, acc_hi);
            if (++blk == nbpt) {  // tile done for this warp
                if (t == 0) {
                    float* pp = part + tile * kPartTile + warp;
                    pp[g * 16] = acc_lo;
                    pp[(8 + g) * 16] = acc_hi;
                }
                acc_lo = acc_hi = 0.F;
                blk = 0;
                ++tile;
            }
        }
        __syncwarp();
        if (lane == 0 && !cs.failed) {
            fence_proxy_async_smem();  // this slot's generic reads before the async-proxy refill
            rstream_issue(a, rng, ps, warp, ring, bars, cs.slot);
        }
        if (++cs.slot == a.ring_slots) {
            cs.slot = 0;
            cs.parity ^= 1u;
        }
        u += n;
    }
    if (uw1 > uw0 && blk != 0 && t == 0) {
        float* pp = part + tile * kPartTile + warp;
        pp[g * 16] = acc_lo;
        pp[(8 + g) * 16] = acc_hi;
    }
    KR_STAMP(layer, kSt + 1);
#ifdef KC_PERSIST_STAMPS
    if (layer == KC_STAMP_LAYER && lane == 0) {  // ring-wait and loop cycles of every warp
        g_rows_stamps[(256 + blockIdx.x) * 64 + OP * 16 + warp] = static_cast<unsigned long long>(wcyc);
        g_rows_stamps[(512 + blockIdx.x) * 64 + OP * 16 + warp] = static_cast<unsigned long long>(clock64() - tloop);
    }
#endif
    __syncthreads();
    KR_STAMP(layer, kSt + 2);
    // one thread per tile row sums the 16 warps in fixed order; the row r + 8
    // partner's sum comes over by shuffle and rows r < 8 run the epilogue
    for (int idx = tid; idx < ntiles * 16; idx += kRT) {
        const int tl = idx >> 4, rr = idx & 15;
        const int left = ntiles * 16 - (idx - lane);  // this warp's lanes in the loop: whole 16-lane tiles
        const unsigned active = left >= 32 ? 0xffffffffu : (1u << left) - 1u;
        const float4* pr = reinterpret_cast<const float4*>(part + tl * kPartTile + rr * 16);  // the row's 16 warps
        const float4 p0 = pr[0], p1 = pr[1], p2 = pr[2], p3 = pr[3];
        float sum = 0.F;  // warps in order 0 .. 15
        sum += p0.x; sum += p0.y; sum += p0.z; sum += p0.w;
        sum += p1.x; sum += p1.y; sum += p1.z; sum += p1.w;
        sum += p2.x; sum += p2.y; sum += p2.z; sum += p2.w;
        sum += p3.x; sum += p3.y; sum += p3.z; sum += p3.w;
        const float hi = __shfl_down_sync(active, sum, 8, 16);
        if (idx == 0) KR_STAMP(layer, 37 + 2 * OP);
        if (rr < 8) epi(t0 + tl, rr, sum, hi, active & 0x00ff00ffu);
    }
    KR_STAMP(layer, 38 + 2 * OP);
    __syncthreads();  // the epilogues' reads of shared memory (xres, part) before its next writers
    if (OP == kOGu) KR_STAMP(layer, 62);
}

// ------------------------------------------------------------------ staging
// xs = f16(RMSNorm_HF(x) * w): x_norm = bf16(w * bf16(x * rsqrt(mean(x^2) + eps)));
// w was loaded into registers before the dependency wait.
constexpr int kNormPer = 2;  // hidden <= 8 * 512 * 2
__device__ __forceinline__ void rnorm_prefetch(const RowArgs& a, const uint16_t* w, uint4* wv) {
#pragma unroll
    for (int i = 0; i < kNormPer; ++i) {
        const int o = threadIdx.x + i * kRT;
        if (o < a.hidden / 8) wv[i] = __ldg(reinterpret_cast<const uint4*>(w + 8 * o));
    }
}
__device__ void rstage_norm(const RowArgs& a, const uint16_t* xres, const uint4* wv, uint16_t* xs, float* red,
                            uint16_t* tap, [[maybe_unused]] int layer, [[maybe_unused]] int stamp) {
    const int tid = threadIdx.x;
    const int n8 = a.hidden / 8;
    float ss = 0.F;
#pragma unroll 4
    for (int i = tid; i < a.hidden; i += kRT) {
        const float v = bf16_bits_to_f32(xres[i]);
        ss += v * v;
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    KR_STAMP(layer, stamp);
    const float4* r4 = reinterpret_cast<const float4*>(red);  // the 16 warp sums, added in order
    const float4 q0 = r4[0], q1 = r4[1], q2 = r4[2], q3 = r4[3];
    float tot = 0.F;
    tot += q0.x; tot += q0.y; tot += q0.z; tot += q0.w;
    tot += q1.x; tot += q1.y; tot += q1.z; tot += q1.w;
    tot += q2.x; tot += q2.y; tot += q2.z; tot += q2.w;
    tot += q3.x; tot += q3.y; tot += q3.z; tot += q3.w;
    // the mean: a power-of-two hidden size divides exactly by multiplying with its reciprocal
    const float nh = static_cast<float>(a.hidden);
    const float mean = (a.hidden & (a.hidden - 1)) == 0 ? tot * (1.0F / nh) : tot / nh;
    const float inv = 1.0F / sqrtf(mean + a.eps);
    bool overflow = false;
#pragma unroll
    for (int i = 0; i < kNormPer; ++i) {
        const int o = tid + i * kRT;
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
    rflag_overflow(a, overflow);
    __syncthreads();
}
// dst (shared, n bf16) = src (global, written by other CTAs before the acquire)
__device__ __forceinline__ void rload_bf16(uint16_t* dst, const uint16_t* src, int n) {
    for (int i = threadIdx.x; i < n / 8; i += kRT)
        reinterpret_cast<uint4*>(dst)[i] = __ldcg(reinterpret_cast<const uint4*>(src) + i);
}

// ------------------------------------------------------------------ attention
// A split of one KV head covers ts tokens (a multiple of kATile) in tiles of
// kATile tokens.  The tile's K and V rows land in padded shared rows by
// per-row bulk copies (the first tile's are issued before the split waits for
// q); scores and P.V run on the tensor core as in the cluster GQA kernel
// (gqa_decode.cu): mma.m16n8k16 bf16 with the group's query heads in A rows
// 0..gq-1 and 8 tokens per n-tile, fp32 accumulation; P split into bf16 hi +
// lo halves against ldmatrix.trans V fragments.
struct RAttPlan {
    int ns, ts;
};
__device__ __forceinline__ RAttPlan ratt_plan(const RowArgs& a, int kv_len) {
    RAttPlan p;
    const int per_head = max(1, min(kAMaxSplits, static_cast<int>(gridDim.x) / a.kvh));
    const int tiles = (kv_len + kATile - 1) / kATile;
    const int ns = min(per_head, tiles);
    p.ts = kATile * ((tiles + ns - 1) / ns);
    p.ns = (kv_len + p.ts - 1) / p.ts;
    return p;
}
struct RAttSmem {
    uint16_t* kt;  // [kATile][kKRow]  (a region of its own: the first tile is fetched at layer start)
    uint16_t* vt;  // [kATile][kKRow]
    uint16_t* qb;  // [8][kKRow]: the group's q rows (bf16), rows >= gq zero   (in the work region)
    float* ss;     // [2][8][kSs]: score halves, then in row 8 + h head h's probabilities as bf16 hi/lo token pairs; the merge's weights and split max/sum
    float* ml;     // [8][4]: running max, sum, correction
    float* mb;     // [8][ns * nd <= 160]: the merge's slice of every split's accumulator, [hq][split][dim]
    uint16_t* kvpos;  // [2][128]: this step's k and v rows (bf16), from the q/k/v owners' tagged words
};
constexpr int kRKvTileBytes = 2 * kATile * kKRow * 2;
constexpr int kRAttWorkBytes = 8 * kKRow * 2 + 2 * 8 * kSs * 4 + 8 * 4 * 4 + 8 * 160 * 4 + 2 * 128 * 2;
__device__ __forceinline__ RAttSmem ratt_smem(uint8_t* work, uint8_t* kvt) {
    RAttSmem s;
    s.kt = reinterpret_cast<uint16_t*>(kvt);
    s.vt = s.kt + kATile * kKRow;
    s.qb = reinterpret_cast<uint16_t*>(work);
    s.ss = reinterpret_cast<float*>(s.qb + 8 * kKRow);
    s.ml = s.ss + 2 * 8 * kSs;
    s.mb = s.ml + 8 * 4;
    s.kvpos = reinterpret_cast<uint16_t*>(s.mb + 8 * 160);
    return s;
}
// Warp 0 (all lanes) issues the bulk copies of K and V rows [t0, t0 + nt) of
// one KV head into the padded tile rows, completing on `bar`.
// K and V rows t0 .. t0+nt-1 of one head into the padded tile rows: 16-byte
// cp.async by every thread of the CTA (thousands of small copies would queue
// behind the weight rings on the bulk-copy engine).  Row skip (this step's
// position, still being written by the q/k/v owners) is left out; the caller
// loads it with plain loads once it is final.  One commit group per call.
__device__ __forceinline__ void ratt_fetch(const uint16_t* kc, const uint16_t* vc, int t0, int nt, int skip,
                                           const RAttSmem& sm) {
    for (int i = threadIdx.x; i < nt * 16; i += kRT) {
        const int r = i >> 4, c = i & 15;
        if (t0 + r == skip) continue;
        const int64_t src = static_cast<int64_t>(t0 + r) * 128 + 8 * c;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(sm.kt + r * kKRow + 8 * c)),
                     "l"(kc + src)
                     : "memory");
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(sm.vt + r * kKRow + 8 * c)),
                     "l"(vc + src)
                     : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}
// This step's k and v rows (staged from the tagged words) into tile row pos - t0, if the tile holds it.
__device__ __forceinline__ void ratt_pos_row(int t0, int nt, int pos, const RAttSmem& sm) {
    if (pos < t0 || pos >= t0 + nt) return;
    for (int i = threadIdx.x; i < 2 * 16; i += kRT) {
        uint16_t* dst = (i < 16 ? sm.kt : sm.vt) + (pos - t0) * kKRow;
        reinterpret_cast<uint4*>(dst)[i & 15] = reinterpret_cast<const uint4*>(sm.kvpos + (i < 16 ? 0 : 128))[i & 15];
    }
}
__device__ __forceinline__ void rldsm_x2_trans(uint32_t& r0, uint32_t& r1, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void rsplit_pair(float p0, float p1, uint32_t& hi, uint32_t& lo) {
    const float h0 = round_bf16(p0), h1 = round_bf16(p1);
    hi = static_cast<uint32_t>(f32_to_bf16_bits(h0)) | (static_cast<uint32_t>(f32_to_bf16_bits(h1)) << 16);
    lo = static_cast<uint32_t>(f32_to_bf16_bits(p0 - h0)) | (static_cast<uint32_t>(f32_to_bf16_bits(p1 - h1)) << 16);
}

// One split (KV head hk, tokens [tok0, tok1)) of one layer; then, once every
// split of the head has published its partial, each split merges its slice of
// the head dims (all ns splits, all gq query heads) into the attention
// output, written once for all o_proj owners.
__device__ void rattention(const RowArgs& a, int layer, const uint64_t* L, int pos, int kv_len, const RAttPlan& ap,
                           const RAttSmem& sm, uint32_t tq, uint32_t tk, uint32_t tv, uint32_t tatt, uint32_t tpart,
                           uint32_t tpart_c) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int gq = a.qh / a.kvh, hd = a.hd;
    const int hk = static_cast<int>(blockIdx.x) / ap.ns, s = static_cast<int>(blockIdx.x) - hk * ap.ns;
    const int tok0 = s * ap.ts, tok1 = min(kv_len, tok0 + ap.ts);
    const uint16_t* kc = reinterpret_cast<const uint16_t*>(L[kTKCache]) + static_cast<int64_t>(hk) * a.cap * hd;
    const uint16_t* vc = reinterpret_cast<const uint16_t*>(L[kTVCache]) + static_cast<int64_t>(hk) * a.cap * hd;
    // the group's q rows (bf16 pairs, rows >= gq zero) and, for the split that
    // holds pos, this step's k and v rows: the q/k/v owners' tagged words
    const int hp = hd / 2, nq = gq * hp;
    const bool has_pos = pos >= tok0 && pos < tok1;
    for (int i = nq + tid; i < 8 * hp; i += kRT) reinterpret_cast<uint32_t*>(sm.qb + (i / hp) * kKRow)[i % hp] = 0u;
    uint32_t* qb32 = reinterpret_cast<uint32_t*>(sm.qb);
    uint32_t* kv32 = reinterpret_cast<uint32_t*>(sm.kvpos);
    rpoll<2>(
        a, nq + (has_pos ? 2 * hp : 0),
        [&](int i, uint32_t& tg, int& sl) -> const uint64_t* {
            if (i < nq) {  // q row i / 64 of the group, padded shared rows
                tg = tq;
                sl = (i >> 6) * (kKRow / 2) + (i & 63);
                return a.qw + hk * nq + i;
            }
            tg = i < nq + hp ? tk : tv;
            sl = -1 - (i - nq);  // k then v words of this step's row
            return i < nq + hp ? a.kw + hk * hp + (i - nq) : a.vw + hk * hp + (i - nq - hp);
        },
        [&](int sl, uint32_t p) {
            if (sl >= 0) qb32[sl] = p;
            else kv32[-1 - sl] = p;
        });
    ratt_pos_row(tok0, min(kATile, tok1 - tok0), pos, sm);  // the rest of the first tile was fetched at layer start
    if (tid < 8) {
        sm.ml[tid * 4 + 0] = -INFINITY;
        sm.ml[tid * 4 + 1] = 0.F;
        sm.ml[tid * 4 + 2] = 1.F;
    }
    __syncthreads();
    KR_STAMP(layer, 28);
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
    for (int t0 = tok0; t0 < tok1; t0 += kATile) {
        const int nt = min(kATile, tok1 - t0);
        if (t0 != tok0) {
            __syncthreads();  // every thread is done with the previous tile's rows
            ratt_fetch(kc, vc, t0, nt, pos, sm);
            ratt_pos_row(t0, nt, pos, sm);
        }
        const int n16 = (nt + 15) & ~15;
        // V rows nt .. n16-1 take part in the last P.V k-step with P = 0: make them finite
        for (int i = tid; i < (n16 - nt) * (hd / 2); i += kRT)
            reinterpret_cast<uint32_t*>(sm.vt + (nt + i / (hd / 2)) * kKRow)[i % (hd / 2)] = 0u;
        asm volatile("cp.async.wait_all;" ::: "memory");  // this thread's copies of the tile
        __syncthreads();
        if (t0 == tok0) KR_STAMP(layer, 29);
        if (warp < (n16 >> 3) * 2) {  // scores: unit (n-tile of 8 tokens, dim half) per warp
            const int ntl = warp >> 1, hf = warp & 1;
            float c0[4] = {0.F, 0.F, 0.F, 0.F}, c1[4] = {0.F, 0.F, 0.F, 0.F};
            const uint8_t* krow = reinterpret_cast<const uint8_t*>(sm.kt) + (ntl * 8 + g) * kKRow * 2 + 4 * t + 128 * hf;
#pragma unroll
            for (int s4 = 0; s4 < 4; s4 += 2) {
                const uint32_t qA0 = hf ? qa[4 + s4][0] : qa[s4][0], qA1 = hf ? qa[4 + s4][1] : qa[s4][1];
                const uint32_t qB0 = hf ? qa[5 + s4][0] : qa[s4 + 1][0], qB1 = hf ? qa[5 + s4][1] : qa[s4 + 1][1];
                mma_bf16(c0, qA0, 0u, qA1, 0u, *reinterpret_cast<const uint32_t*>(krow + 32 * s4),
                         *reinterpret_cast<const uint32_t*>(krow + 32 * s4 + 16));
                mma_bf16(c1, qB0, 0u, qB1, 0u, *reinterpret_cast<const uint32_t*>(krow + 32 * s4 + 32),
                         *reinterpret_cast<const uint32_t*>(krow + 32 * s4 + 48));
            }
            if (g < gq)
                *reinterpret_cast<float2*>(sm.ss + (hf * 8 + g) * kSs + ntl * 8 + 2 * t) =
                    make_float2((c0[0] + c1[0]) * a.scale_log2, (c0[1] + c1[1]) * a.scale_log2);
        }
        __syncthreads();
        if (t0 == tok0) KR_STAMP(layer, 32);
        if (warp < gq) {  // online softmax per head over the tile (log2 domain); probabilities zero past nt
            float v[2];
            float mx = -INFINITY;
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int j = lane + 32 * k;
                v[k] = j < nt ? sm.ss[warp * kSs + j] + sm.ss[(8 + warp) * kSs + j] : -INFINITY;
                mx = fmaxf(mx, v[k]);
            }
            mx = warp_max(mx);
            const float m_old = sm.ml[warp * 4 + 0];
            const float m_new = fmaxf(m_old, mx);
            // the probabilities as bf16 hi + lo pairs of consecutive tokens, split once here for every
            // P.V warp: row 8 + head of ss (its scores are consumed), hi pair i at word i, lo at 32 + i
            uint32_t* pk = reinterpret_cast<uint32_t*>(sm.ss + (8 + warp) * kSs);
            float ls = 0.F;
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int j = lane + 32 * k;
                const float p = j < nt ? exp2f(v[k] - m_new) : 0.F;
                const float pn = __shfl_down_sync(0xffffffffu, p, 1);
                if ((lane & 1) == 0 && j < n16) {
                    uint32_t hi, lo;
                    rsplit_pair(p, pn, hi, lo);
                    pk[j >> 1] = hi;
                    pk[32 + (j >> 1)] = lo;
                }
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
        if (t0 == tok0) KR_STAMP(layer, 33);
        if (warp < hd / 8) {  // P.V: warp w owns dims 8w .. 8w+7
            const float corr = g < gq ? sm.ml[g * 4 + 2] : 1.F;
            o0[0] *= corr;
            o0[1] *= corr;
            o1[0] *= corr;
            o1[1] *= corr;
            const uint32_t* prow = reinterpret_cast<const uint32_t*>(sm.ss + (8 + (g < gq ? g : 0)) * kSs) + t;
            const int nk = n16 >> 4;
            for (int kk = 0; kk < nk; kk += 2) {
                const bool two = kk + 1 < nk;
                uint32_t b0, b1, b2 = 0u, b3 = 0u;
                rldsm_x2_trans(b0, b1, vbase + static_cast<uint32_t>(kk * 16 * kKRow * 2));
                if (two) rldsm_x2_trans(b2, b3, vbase + static_cast<uint32_t>((kk + 1) * 16 * kKRow * 2));
                // tokens kk*16 + 2t (+1) are pair kk*8 + t; + 8 tokens is + 4 pairs (zero for rows >= gq)
                uint32_t ah0 = 0u, al0 = 0u, ah2 = 0u, al2 = 0u, ch0 = 0u, cl0 = 0u, ch2 = 0u, cl2 = 0u;
                if (g < gq) {
                    ah0 = prow[kk * 8];
                    al0 = prow[32 + kk * 8];
                    ah2 = prow[kk * 8 + 4];
                    al2 = prow[32 + kk * 8 + 4];
                    if (two) {
                        ch0 = prow[kk * 8 + 8];
                        cl0 = prow[32 + kk * 8 + 8];
                        ch2 = prow[kk * 8 + 12];
                        cl2 = prow[32 + kk * 8 + 12];
                    }
                }
                mma_bf16(o0, ah0, 0u, ah2, 0u, b0, b1);
                if (two) mma_bf16(o1, ch0, 0u, ch2, 0u, b2, b3);
                mma_bf16(o0, al0, 0u, al2, 0u, b0, b1);
                if (two) mma_bf16(o1, cl0, 0u, cl2, 0u, b2, b3);
            }
        }
    }
    KR_STAMP(layer, 34);
    // ---- this split's partial as tagged words: max, sum, then the accumulator of each head
    const int rec = hd + 2;
    uint64_t* mine = a.pw + (static_cast<size_t>(hk) * kAMaxSplits + s) * gq * rec;
    if (warp < hd / 8 && g < gq) {
        st_tagged(mine + g * rec + 2 + 8 * warp + 2 * t, tpart, __float_as_uint(o0[0] + o1[0]));
        st_tagged(mine + g * rec + 3 + 8 * warp + 2 * t, tpart, __float_as_uint(o0[1] + o1[1]));
    }
    if (tid < gq) {
        st_tagged(mine + tid * rec + 0, tpart, __float_as_uint(sm.ml[tid * 4 + 0]));
        st_tagged(mine + tid * rec + 1, tpart, __float_as_uint(sm.ml[tid * 4 + 1]));
    }
    KR_STAMP(layer, 35);
    // ---- each split merges dims [d0, d0 + nd) of the gq heads: the max, sum and
    // that slice of every split's accumulator, polled as tagged words
    // (ns x gq x (2 + nd) <= 2048 words, at most four per thread)
    float* wn = sm.ss;          // [gq][kAMaxSplits] normalised split weights
    float* mls = sm.ss + 256;   // [gq][kAMaxSplits][2] split max and sum
    const int d0 = 2 * (s * hp / ap.ns), nd = 2 * ((s + 1) * hp / ap.ns) - d0, per = ap.ns * nd;  // even slices
    const int nrec = 2 + nd;
    __syncthreads();  // every thread is past its reads of ss (P.V) before the sink writes it
    rpoll<4>(
        a, ap.ns * gq * nrec,
        [&](int i, uint32_t& tg, int& sl) -> const uint64_t* {
            const int sp = i / (gq * nrec), rem = i - sp * gq * nrec, hq = rem / nrec, j = rem - hq * nrec;
            tg = tpart_c;
            sl = j < 2 ? -1 - ((hq * kAMaxSplits + sp) * 2 + j) : hq * per + sp * nd + (j - 2);
            return a.pw + ((static_cast<size_t>(hk) * kAMaxSplits + sp) * gq + hq) * rec + (j < 2 ? j : d0 + j);
        },
        [&](int sl, uint32_t p) {
            if (sl < 0) mls[-1 - sl] = __uint_as_float(p);
            else sm.mb[sl] = __uint_as_float(p);
        });
    KR_STAMP(layer, 31);
    if (warp < gq) {
        const bool live = lane < ap.ns;
        const float m = live ? mls[(warp * kAMaxSplits + lane) * 2] : -INFINITY;
        const float l = live ? mls[(warp * kAMaxSplits + lane) * 2 + 1] : 0.F;
        const float M = warp_max(m);
        const float e = live && m != -INFINITY ? exp2f(m - M) : 0.F;
        const float den = warp_sum(e * l);
        wn[warp * kAMaxSplits + lane] = den > 0.F ? e / den : 0.F;
    }
    __syncthreads();
    KR_STAMP(layer, 36);
    uint16_t* tap = rtap(a, layer);
    const int att_off = tap != nullptr ? rtaps(a.hidden, a.qh, a.kvh, hd, a.inter).att : 0;
    bool overflow = false;
    const int np = nd / 2;
    for (int idx = tid; idx < gq * np; idx += kRT) {  // dims d, d + 1 of head hq: one tagged word
        const int hq = idx / np, dd = 2 * (idx - hq * np);
        const float* mrow = sm.mb + hq * per + dd;
        float acc0 = 0.F, acc1 = 0.F;
        for (int sp = 0; sp < ap.ns; ++sp) {
            const float w = wn[hq * kAMaxSplits + sp];
            acc0 = fmaf(w, mrow[sp * nd], acc0);
            acc1 = fmaf(w, mrow[sp * nd + 1], acc1);
        }
        const uint16_t b0 = f32_to_bf16_bits(acc0), b1 = f32_to_bf16_bits(acc1);
        const float f0 = bf16_bits_to_f32(b0), f1 = bf16_bits_to_f32(b1);
        overflow |= !(fabsf(f0) <= 65504.F) || !(fabsf(f1) <= 65504.F);
        const int o = (hk * gq + hq) * hd + d0 + dd;
        st_tagged(a.aw + o / 2, tatt,
                  static_cast<uint32_t>(f32_to_f16_bits(f0)) | (static_cast<uint32_t>(f32_to_f16_bits(f1)) << 16));
        if (tap != nullptr) {
            tap[att_off + o] = b0;
            tap[att_off + o + 1] = b1;
        }
    }
    rflag_overflow(a, overflow);
    __syncthreads();  // the merge's reads of wn / mb before the caller's next writes to the work area
}

// ------------------------------------------------------------------ the kernel
// kTP: the tensor-parallel form (world > 1: o_proj and down summed over the
// ranks' exchange buffers); the single-GPU form carries none of that code.
template <bool kTP>
__global__ void __launch_bounds__(kRT, 1) decode_rows_kernel(const RowArgs a) {
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ __align__(8) uint64_t bars_all[kRW * kRMaxSlots];
    __shared__ __align__(16) float red[kRW];
    __shared__ int rng[4 * kRngStride];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint8_t* lut = dsm;
    uint8_t* rings = dsm + kRLutBytes;
    // work: the GEMV input xs from 0; the attention's small arrays from 0 and
    // its K/V tile rows from kvt_off (above any QKV input, which the rows'
    // layer-start fetch overlaps; later inputs are staged after the attention)
    uint8_t* work = rings + kRW * a.ring_slots * kSlotBytes;
    uint16_t* xs = reinterpret_cast<uint16_t*>(work);
    uint8_t* kvt = work + a.kvt_off;  // attention K/V tile rows
    float* part = reinterpret_cast<float*>(work + a.work_bytes);
    uint16_t* xres = reinterpret_cast<uint16_t*>(work + a.work_bytes + kPartFloats * 4);
    uint16_t* bias_s = xres + ((a.hidden + 63) & ~63);
    float* rope_s = reinterpret_cast<float*>(bias_s + ((a.bias_rows + 63) & ~63));
    uint8_t* ring = rings + warp * a.ring_slots * kSlotBytes;
    uint64_t* bars = bars_all + warp * kRMaxSlots;

    // ---- per-warp stream: start every ring before anything else (weights are static)
    fill_rng(a, rng);
    __syncthreads();
    RStream ps;
    ps.layer = 0;
    ps.op = 0;
    ps.u = rng[2 + warp];
    ps.end = rng[3 + warp];
    ps.done = a.nlayers < 1;
    if (lane == 0) {
        for (int s = 0; s < a.ring_slots; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
        for (int s = 0; s < a.ring_slots; ++s) rstream_issue(a, rng, ps, warp, ring, bars, s);
    }
    // pair table: entry e -> half2(level[e >> 4], level[e & 15]) at row e, lane replica l
    for (int i = tid; i < 256 * 8; i += kRT) {
        const int e = i >> 3;
        const uint32_t v = static_cast<uint32_t>(f32_to_f16_bits(kNf4Levels[e >> 4])) |
                           (static_cast<uint32_t>(f32_to_f16_bits(kNf4Levels[e & 15])) << 16);
        reinterpret_cast<uint4*>(lut + e * 256)[i & 7] = make_uint4(v, v, v, v);
    }
    const int pos = __ldcg(a.state + 1);
    int kv_len = __ldcg(a.state + 2);
    if (kv_len < 1 || kv_len > a.cap || pos < 0 || pos >= a.cap || pos >= a.max_pos || pos != kv_len - 1) {
        if (tid == 0) atomicOr(a.err, 2);
        kv_len = max(1, min(kv_len, a.cap));
    }
    const int pos_c = max(0, min(pos, min(a.cap, a.max_pos) - 1));
    {
        const int half = a.hd / 2;
        for (int i = tid; i < half; i += kRT) {
            rope_s[i] = bf16_bits_to_f32(a.rope_cos[static_cast<int64_t>(pos_c) * half + i]);
            rope_s[half + i] = bf16_bits_to_f32(a.rope_sin[static_cast<int64_t>(pos_c) * half + i]);
        }
    }
    __syncthreads();
    const RAttPlan ap = ratt_plan(a, kv_len);
    const bool att_cta = static_cast<int>(blockIdx.x) < a.kvh * ap.ns;
    const bool own_o = rng[kOO * kRngStride + 1] > rng[kOO * kRngStride];
    const bool own_dn = rng[kODn * kRngStride + 1] > rng[kODn * kRngStride];
    const RTaps to = rtaps(a.hidden, a.qh, a.kvh, a.hd, a.inter);
    const int hd = a.hd, half = hd / 2;

    RCons cs;
    cs.slot = 0;
    cs.parity = 0;
    cs.failed = false;
    uint4 wv[kNormPer];
    // tags of this launch: epoch in [1, 65535], layer, hop
    const uint32_t e16 = 1u + (__ldcg(a.misc + 2) % 65535u);
    auto ptag = [&](int layer, int hop) {
        return (e16 << 16) | (static_cast<uint32_t>(layer) << 4) | static_cast<uint32_t>(hop);
    };
    auto ctag = [&](int layer, int hop) {  // test hook: stall_counter = layer * 16 + op makes that tag unreachable
        return a.stall_counter == layer * 16 + hop_counter(hop) ? (ptag(layer, hop) | 15u) : ptag(layer, hop);
    };
    for (int l = 0; l < a.nlayers; ++l) {
        const uint64_t* L = a.layers + static_cast<int64_t>(l) * kTSlots;
        uint16_t* tap = rtap(a, l);
        const bool tap0 = tap != nullptr && blockIdx.x == 0;
        KR_STAMP(l, 0);
        const RAttSmem att_sm = ratt_smem(work, kvt);
        // ---- x ready -> RMSNorm -> q/k/v owners (bias, RoPE, k/v into the cache row)
        rnorm_prefetch(a, reinterpret_cast<const uint16_t*>(L[kTInNorm]), wv);
        if (a.bias_rows > 0) {
            const int nq = a.qh * hd, nk = a.kvh * hd;
            for (int i = tid; i < a.bias_rows; i += kRT) {
                const uint16_t* b =
                    reinterpret_cast<const uint16_t*>(L[i < nq ? kTQBias : i < nq + nk ? kTKBias : kTVBias]);
                const int j = i < nq ? i : i < nq + nk ? i - nq : i - nq - nk;
                bias_s[i] = b != nullptr ? b[j] : static_cast<uint16_t>(0);
            }
        }
        if (l == 0) {
            rload_bf16(xres, a.x, a.hidden);
            __syncthreads();
        } else {  // the previous layer's x2
            rpoll_vec<8>(a, a.xw, a.hidden / 2, ctag(l, kHX), reinterpret_cast<uint32_t*>(xres));
        }
        // (every thread is now past the previous layer's reads of the K/V tile rows)
        KR_STAMP(l, 1);
        if (att_cta) {  // this layer's first K/V tile, after x (whose loads would queue behind these copies):
                        // rows before pos are final (row pos is loaded with q)
            const int hk = static_cast<int>(blockIdx.x) / ap.ns, sp = static_cast<int>(blockIdx.x) - hk * ap.ns;
            const int tok0 = sp * ap.ts;
            const uint16_t* kc = reinterpret_cast<const uint16_t*>(L[kTKCache]) + static_cast<int64_t>(hk) * a.cap * hd;
            const uint16_t* vc = reinterpret_cast<const uint16_t*>(L[kTVCache]) + static_cast<int64_t>(hk) * a.cap * hd;
            ratt_fetch(kc, vc, tok0, min(kATile, kv_len - tok0), pos_c, att_sm);
        }
        rstage_norm(a, xres, wv, xs, red, tap0 ? tap + to.xn : nullptr, l, 45);
        KR_STAMP(l, 2);
        {
            uint16_t* kcl = reinterpret_cast<uint16_t*>(L[kTKCache]);
            uint16_t* vcl = reinterpret_cast<uint16_t*>(L[kTVCache]);
            const int qt = a.qh * hd / 16, kt = a.kvh * hd / 16, per = hd / 16;
            const bool bias = a.bias_rows > 0;
            const uint32_t tq = ptag(l, kHQ), tk = ptag(l, kHK), tv = ptag(l, kHV);
            rgemv<kOQkv>(a, l, rng, lut, ring, bars, ps, cs, xs, part, [&](int T, int r, float ylo, float yhi, unsigned lanes) {
                // q/k: RoPE pair (dims i, i + half) of a head; v: rows d, d + 8 of a 16-row tile
                const bool qk = T < qt + kt, isq = T < qt;
                const int u = isq ? T : T - qt, head = u / per, i = 8 * (u - head * per) + r;
                const int d = 16 * (T - qt - kt) + r;
                uint16_t o0, o1;
                if (qk) {
                    const int row0 = (isq ? 0 : a.qh * hd) + head * hd + i;
                    float y0 = round_bf16(ylo), y1 = round_bf16(yhi);
                    if (bias) {
                        y0 = round_bf16(y0 + bf16_bits_to_f32(bias_s[row0]));
                        y1 = round_bf16(y1 + bf16_bits_to_f32(bias_s[row0 + half]));
                    }
                    const float c = rope_s[i], sn = rope_s[half + i];
                    o0 = f32_to_bf16_bits(round_bf16(round_bf16(y0 * c) + round_bf16(-y1 * sn)));
                    o1 = f32_to_bf16_bits(round_bf16(round_bf16(y1 * c) + round_bf16(y0 * sn)));
                } else {
                    float y0 = round_bf16(ylo), y1 = round_bf16(yhi);
                    if (bias) {
                        y0 = round_bf16(y0 + bf16_bits_to_f32(bias_s[(a.qh + a.kvh) * hd + d]));
                        y1 = round_bf16(y1 + bf16_bits_to_f32(bias_s[(a.qh + a.kvh) * hd + d + 8]));
                    }
                    o0 = f32_to_bf16_bits(y0);
                    o1 = f32_to_bf16_bits(y1);
                }
                const uint32_t p0 = pair_up(o0, lanes), p1 = pair_up(o1, lanes);  // every lane of the 8-lane group
                if (qk) {
                    if (!isq) {  // the cache row, read by later steps
                        kcl[(static_cast<int64_t>(head) * a.cap + pos_c) * hd + i] = o0;
                        kcl[(static_cast<int64_t>(head) * a.cap + pos_c) * hd + i + half] = o1;
                    }
                    if ((r & 1) == 0) {
                        uint64_t* w = (isq ? a.qw : a.kw) + (head * hd + i) / 2;
                        st_tagged(w, isq ? tq : tk, p0);
                        st_tagged(w + half / 2, isq ? tq : tk, p1);
                    }
                    if (tap != nullptr) {
                        uint16_t* tp = tap + (isq ? to.q : to.k) + head * hd + i;
                        tp[0] = o0;
                        tp[half] = o1;
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < 2; ++k) {
                        const int dd = d + 8 * k, hv = dd / hd;
                        vcl[(static_cast<int64_t>(hv) * a.cap + pos_c) * hd + (dd - hv * hd)] = k == 0 ? o0 : o1;
                        if (tap != nullptr) tap[to.v + dd] = k == 0 ? o0 : o1;
                    }
                    if ((r & 1) == 0) {
                        st_tagged(a.vw + d / 2, tv, p0);
                        st_tagged(a.vw + (d + 8) / 2, tv, p1);
                    }
                }
            });
        }
        KR_STAMP(l, 3);
        // ---- attention splits, merged once per KV head
        if (att_cta) {
            KR_STAMP(l, 4);
            rattention(a, l, L, pos_c, kv_len, ap, att_sm, ctag(l, kHQ), ctag(l, kHK), ctag(l, kHV), ptag(l, kHAtt),
                       ptag(l, kHPart), ctag(l, kHPart));
            KR_STAMP(l, 5);
        }
        // ---- o_proj owners: x1 = x + o_proj(attention)
        rnorm_prefetch(a, reinterpret_cast<const uint16_t*>(L[kTPostNorm]), wv);
        if (own_o) {
            KR_STAMP(l, 6);
            rpoll_vec<8>(a, a.aw, a.qh * hd / 2, ctag(l, kHAtt), reinterpret_cast<uint32_t*>(xs));
            KR_STAMP(l, 7);
            const uint32_t tx1 = ptag(l, kHX1);
            constexpr bool tp = kTP;
            const uint32_t tpo = ptag(l, kHTpO);
            rgemv<kOO>(a, l, rng, lut, ring, bars, ps, cs, xs, part, [&](int T, int r, float ylo, float yhi, unsigned lanes) {
                if constexpr (tp) {  // this rank's partial: the sum over ranks comes after every push
                    rtp_push(a, 0, 16 * T + r, ylo, yhi, tpo);
                } else {
                    uint16_t x1[2];
#pragma unroll
                    for (int k = 0; k < 2; ++k) {
                        const int row = 16 * T + r + 8 * k;
                        x1[k] = f32_to_bf16_bits(bf16_bits_to_f32(xres[row]) + round_bf16(k == 0 ? ylo : yhi));
                        if (tap != nullptr) tap[to.x1 + row] = x1[k];
                    }
                    const uint32_t p0 = pair_up(x1[0], lanes), p1 = pair_up(x1[1], lanes);
                    if ((r & 1) == 0) {
                        st_tagged(a.x1w + (16 * T + r) / 2, tx1, p0);
                        st_tagged(a.x1w + (16 * T + r + 8) / 2, tx1, p1);
                    }
                }
            });
            if constexpr (tp)
                rtp_finish(a, rng + kOO * kRngStride, reinterpret_cast<const uint64_t*>(a.peers[a.rank]),
                           ctag(l, kHTpO), part, [&](int row, float sum, unsigned lanes) {
                               const uint16_t x1 =
                                   f32_to_bf16_bits(bf16_bits_to_f32(xres[row]) + round_bf16(sum));
                               if (tap != nullptr) tap[to.x1 + row] = x1;
                               const uint32_t p = pair_up(x1, lanes);
                               if ((row & 1) == 0) st_tagged(a.x1w + row / 2, tx1, p);
                           });
            KR_STAMP(l, 8);
        }
        // ---- x1 ready -> RMSNorm -> gate/up owners (SwiGLU)
        rpoll_vec<8>(a, a.x1w, a.hidden / 2, ctag(l, kHX1), reinterpret_cast<uint32_t*>(xres));
        KR_STAMP(l, 9);
        rstage_norm(a, xres, wv, xs, red, tap0 ? tap + to.xn2 : nullptr, l, 46);
        KR_STAMP(l, 10);
        {
            bool overflow = false;
            const uint32_t th = ptag(l, kHH);
            rgemv<kOGu>(a, l, rng, lut, ring, bars, ps, cs, xs, part, [&](int T, int r, float ylo, float yhi, unsigned lanes) {
                const int j = 8 * T + r;
                const float gv = round_bf16(ylo), uv = round_bf16(yhi);
                const float act = round_bf16(gv / (1.0F + expf(-gv)));
                const uint16_t h = f32_to_bf16_bits(act * uv);
                const float hf = bf16_bits_to_f32(h);
                overflow |= !(fabsf(hf) <= 65504.F);
                if (tap != nullptr) tap[to.h + j] = h;
                const uint32_t p = pair_up(f32_to_f16_bits(hf), lanes);  // the down GEMV's f16 input
                if ((r & 1) == 0) st_tagged(a.hw + j / 2, th, p);
            });
            KR_STAMP(l, 63);
            rflag_overflow(a, overflow);
            KR_STAMP(l, 61);
        }
        KR_STAMP(l, 11);
        // ---- down owners: x2 = x1 + down(h), the next layer's input
        if (own_dn) {
            KR_STAMP(l, 12);
            rpoll_vec<16>(a, a.hw, a.inter / 2, ctag(l, kHH), reinterpret_cast<uint32_t*>(xs));
            KR_STAMP(l, 13);
            const uint32_t tx = ptag(l + 1, kHX);
            const bool last = l == a.nlayers - 1;
            constexpr bool tp = kTP;
            const uint32_t tpd = ptag(l, kHTpD);
            rgemv<kODn>(a, l, rng, lut, ring, bars, ps, cs, xs, part, [&](int T, int r, float ylo, float yhi, unsigned lanes) {
                if constexpr (tp) {
                    rtp_push(a, a.world * a.hidden, 16 * T + r, ylo, yhi, tpd);
                } else {
                    uint16_t x2[2];
#pragma unroll
                    for (int k = 0; k < 2; ++k) {
                        const int row = 16 * T + r + 8 * k;
                        x2[k] = f32_to_bf16_bits(bf16_bits_to_f32(xres[row]) + round_bf16(k == 0 ? ylo : yhi));
                        if (last) a.x[row] = x2[k];  // the step's output, read by the lm_head after the kernel
                        if (tap != nullptr) tap[to.x2 + row] = x2[k];
                    }
                    const uint32_t p0 = pair_up(x2[0], lanes), p1 = pair_up(x2[1], lanes);
                    if ((r & 1) == 0 && !last) {
                        st_tagged(a.xw + (16 * T + r) / 2, tx, p0);
                        st_tagged(a.xw + (16 * T + r + 8) / 2, tx, p1);
                    }
                }
            });
            if constexpr (tp)
                rtp_finish(a, rng + kODn * kRngStride,
                           reinterpret_cast<const uint64_t*>(a.peers[a.rank]) + static_cast<int64_t>(a.world) * a.hidden,
                           ctag(l, kHTpD), part, [&](int row, float sum, unsigned lanes) {
                               const uint16_t x2 =
                                   f32_to_bf16_bits(bf16_bits_to_f32(xres[row]) + round_bf16(sum));
                               if (last) a.x[row] = x2;
                               if (tap != nullptr) tap[to.x2 + row] = x2;
                               const uint32_t p = pair_up(x2, lanes);
                               if ((row & 1) == 0 && !last) st_tagged(a.xw + row / 2, tx, p);
                           });
            KR_STAMP(l, 14);
        }
    }
    // ---- the last CTA to finish resets the step flags and advances the epoch
    // (every issued copy has been consumed: the stream and the consumers walk
    // the same unit sequence); the kernel's end makes x final for the lm_head
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned old = atomicAdd(a.misc + 1, 1u);
        if (old == gridDim.x - 1) {
            a.misc[0] = 0u;
            a.misc[1] = 0u;
            a.misc[2] += 1u;  // the next launch's tags differ from every word written here
            __threadfence();
        }
    }
}

// ------------------------------------------------------------------ re-tiling into 16-row tiles
struct Retile16Args {
    const uint8_t* packed[3];
    const float* absmax[3];
    int rows[3];
    int mode, K, hd, tiles;
    uint8_t* out;
};
__device__ __forceinline__ void tile16_row(const Retile16Args& r, int tile, int rr, int& m, int& row) {
    if (r.mode == kRetilePlain) {
        m = 0;
        row = 16 * tile + rr;
    } else if (r.mode == kRetileSwiGlu) {
        m = rr < 8 ? 0 : 1;
        row = 8 * tile + (rr & 7);
    } else {  // q / k heads in tiles of 8 RoPE pairs, then 16-row v tiles
        const int per = r.hd / 16;
        const int qt = r.rows[0] / r.hd * per, kt = r.rows[1] / r.hd * per;
        if (tile < qt + kt) {
            m = tile < qt ? 0 : 1;
            const int u = tile < qt ? tile : tile - qt;
            const int head = u / per, mm = u - head * per;
            row = head * r.hd + 8 * mm + (rr & 7) + (rr >= 8 ? r.hd / 2 : 0);
        } else {
            m = 2;
            row = 16 * (tile - qt - kt) + rr;
        }
    }
}
__global__ void nf4_retile16_kernel(const Retile16Args r) {
    const int nbpt = r.K / 64;
    const int64_t total = static_cast<int64_t>(r.tiles) * nbpt * 32;  // 32 lanes x 16 code bytes per unit
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t unit = i >> 5;
        const int l = static_cast<int>(i & 31);
        const int tile = static_cast<int>(unit / nbpt), b = static_cast<int>(unit - static_cast<int64_t>(tile) * nbpt);
        const int g = l >> 2, t = l & 3;
        int mA, rowA, mB, rowB;
        tile16_row(r, tile, g, mA, rowA);
        tile16_row(r, tile, g + 8, mB, rowB);
        const uint2 pa = *reinterpret_cast<const uint2*>(r.packed[mA] + static_cast<int64_t>(rowA) * (r.K / 2) + 32 * b + 8 * t);
        const uint2 pb = *reinterpret_cast<const uint2*>(r.packed[mB] + static_cast<int64_t>(rowB) * (r.K / 2) + 32 * b + 8 * t);
        uint8_t* u = r.out + unit * kUnitBytes;
        reinterpret_cast<uint4*>(u)[l] = make_uint4(pa.x, pa.y, pb.x, pb.y);
        if (l < 16) {
            int m, row;
            tile16_row(r, tile, l, m, row);
            reinterpret_cast<float*>(u + kUnitCodes)[l < 8 ? 2 * l : 2 * (l - 8) + 1] =
                r.absmax[m][static_cast<int64_t>(row) * nbpt + b];
        }
    }
}

// ------------------------------------------------------------------ launch geometry
struct RowGeom {
    int tiles[4], nbpt[4], ctas[4];
    int kvt_off, work_bytes, bias_rows, ring_slots, smem;
    int64_t off_misc, off_qw, off_kw, off_vw, off_aw, off_x1w, off_hw, off_xw, off_pw, total;
};
constexpr int kRStaticSmemBudget = 3072;

RowGeom row_geom(const PersistDims& d, int sms) {
    RowGeom g;
    g.tiles[kOQkv] = (d.q_heads + 2 * d.kv_heads) * d.head_dim / 16;
    g.nbpt[kOQkv] = d.hidden / 64;
    g.tiles[kOO] = d.hidden / 16;
    g.nbpt[kOO] = d.q_heads * d.head_dim / 64;
    g.tiles[kOGu] = d.intermediate / 8;
    g.nbpt[kOGu] = d.hidden / 64;
    g.tiles[kODn] = d.hidden / 16;
    g.nbpt[kODn] = d.intermediate / 64;
    for (int i = 0; i < 4; ++i) g.ctas[i] = g.tiles[i] < sms ? g.tiles[i] : sms;
    int kmax = d.hidden > d.intermediate ? d.hidden : d.intermediate;
    kmax = kmax > d.q_heads * d.head_dim ? kmax : d.q_heads * d.head_dim;
    const int xs_bytes = (kmax * 2 + 127) & ~127;
    g.kvt_off = ((kRAttWorkBytes > d.hidden * 2 ? kRAttWorkBytes : d.hidden * 2) + 127) & ~127;
    g.work_bytes = ((xs_bytes > g.kvt_off + kRKvTileBytes ? xs_bytes : g.kvt_off + kRKvTileBytes) + 127) & ~127;
    g.bias_rows = (d.q_heads + 2 * d.kv_heads) * d.head_dim;
    const int tail = kPartFloats * 4 + ((d.hidden + 63) & ~63) * 2 + ((g.bias_rows + 63) & ~63) * 2 +
                     d.head_dim * 4;
    const int limit = 232448 - kRStaticSmemBudget;
    g.ring_slots = kRMaxSlots;
    while (g.ring_slots > 1 && kRLutBytes + kRW * g.ring_slots * kSlotBytes + g.work_bytes + tail > limit) --g.ring_slots;
    g.smem = kRLutBytes + kRW * g.ring_slots * kSlotBytes + g.work_bytes + tail;
    auto up = [](int64_t v) { return (v + 255) & ~static_cast<int64_t>(255); };
    const int gq = d.kv_heads > 0 ? d.q_heads / d.kv_heads : 1;
    int64_t off = 0;
    g.off_misc = off;
    off = up(off + 64);
    g.off_qw = off;  // tagged words: 8 bytes per two values
    off = up(off + static_cast<int64_t>(d.q_heads) * d.head_dim * 4);
    g.off_kw = off;
    off = up(off + static_cast<int64_t>(d.kv_heads) * d.head_dim * 4);
    g.off_vw = off;
    off = up(off + static_cast<int64_t>(d.kv_heads) * d.head_dim * 4);
    g.off_aw = off;
    off = up(off + static_cast<int64_t>(d.q_heads) * d.head_dim * 4);
    g.off_x1w = off;
    off = up(off + static_cast<int64_t>(d.hidden) * 4);
    g.off_hw = off;
    off = up(off + static_cast<int64_t>(d.intermediate) * 4);
    g.off_xw = off;
    off = up(off + static_cast<int64_t>(d.hidden) * 4);
    g.off_pw = off;
    off = up(off + static_cast<int64_t>(d.kv_heads) * kAMaxSplits * gq * (d.head_dim + 2) * 8);
    g.total = off;
    return g;
}
}  // namespace

int retile16_tiles(int mode, int rows0, int rows1, int rows2, int head_dim) {
    if (mode == kRetilePlain) return rows0 % 16 == 0 && rows0 > 0 ? rows0 / 16 : -1;
    if (mode == kRetileSwiGlu) return rows0 == rows1 && rows0 % 8 == 0 && rows0 > 0 ? rows0 / 8 : -1;
    if (mode == kRetileQkvRope) {
        if (head_dim < 16 || head_dim % 16 != 0 || rows0 % head_dim != 0 || rows1 % head_dim != 0 || rows1 != rows2 ||
            rows0 <= 0 || rows1 <= 0 || rows2 % 16 != 0)
            return -1;
        return rows0 / head_dim * (head_dim / 16) + rows1 / head_dim * (head_dim / 16) + rows2 / 16;
    }
    return -1;
}

cudaError_t nf4_retile16(int mode, const uint8_t* const* packed, const float* const* absmax, const int* rows, int K,
                         int head_dim, uint8_t* out, cudaStream_t stream) {
    Retile16Args r;
    for (int i = 0; i < 3; ++i) {
        r.packed[i] = packed[i];
        r.absmax[i] = absmax[i];
        r.rows[i] = rows[i];
    }
    r.mode = mode;
    r.K = K;
    r.hd = head_dim;
    r.tiles = retile16_tiles(mode, rows[0], rows[1], rows[2], head_dim);
    if (r.tiles < 1 || K < 64 || K % 64 != 0) return cudaErrorInvalidValue;
    r.out = out;
    const int64_t total = static_cast<int64_t>(r.tiles) * (K / 64) * 32;
    const int threads = 256;
    const int64_t blocks = (total + threads - 1) / threads;
    nf4_retile16_kernel<<<static_cast<unsigned>(blocks < 65535 * 16 ? blocks : 65535 * 16), threads, 0, stream>>>(r);
    return cudaGetLastError();
}

int64_t decode_rows_scratch_bytes(const PersistDims& d, int sms) { return row_geom(d, sms).total; }

const char* decode_rows_check(const PersistDims& d, int sms) {
    if (d.layers < 1 || d.hidden < 64 || d.hidden % 64 != 0 || d.head_dim != 128 || d.q_heads < 1 || d.kv_heads < 1 ||
        d.q_heads % d.kv_heads != 0 || d.q_heads / d.kv_heads > 8 || d.intermediate % 64 != 0 ||
        d.hidden > 8 * kRT * kNormPer || d.kv_capacity < 1 || d.kv_heads > sms ||
        d.hidden > 16 * kRT || d.q_heads * d.head_dim > 16 * kRT || d.intermediate > 32 * kRT || d.layers >= 4096)
        return "row-split persistent decode requires hidden % 64 == 0 (<= 8192), head_dim 128, q_heads/kv_heads <= 8, "
               "q_heads * head_dim <= 8192, kv_heads <= SM count, intermediate % 64 == 0 (<= 16384), layers < 4096";
    const RowGeom g = row_geom(d, sms);
    if (g.smem > 232448 - kRStaticSmemBudget) return "row-split persistent decode: shapes need more shared memory than one SM has";
    for (int i = 0; i < 4; ++i) {
        if ((g.tiles[i] + sms - 1) / sms > kMaxCtaTiles) return "row-split persistent decode: an op has more than 16 tiles per SM";
        if (static_cast<int64_t>(g.tiles[i]) * g.nbpt[i] >= (int64_t{1} << 30)) return "row-split persistent decode: an op is too large";
    }
    return nullptr;
}

int64_t decode_rows_tap_stride(const PersistDims& d) {
    return rtaps(d.hidden, d.q_heads, d.kv_heads, d.head_dim, d.intermediate).stride;
}

cudaError_t decode_layers_rows(const PersistLaunch& p, cudaStream_t stream) {
    const int sms = device_sm_count();
    const RowGeom g = row_geom(p.dims, sms);
    RowArgs a;
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
    a.misc = reinterpret_cast<unsigned*>(s + g.off_misc);
    a.qw = reinterpret_cast<uint64_t*>(s + g.off_qw);
    a.kw = reinterpret_cast<uint64_t*>(s + g.off_kw);
    a.vw = reinterpret_cast<uint64_t*>(s + g.off_vw);
    a.aw = reinterpret_cast<uint64_t*>(s + g.off_aw);
    a.x1w = reinterpret_cast<uint64_t*>(s + g.off_x1w);
    a.hw = reinterpret_cast<uint64_t*>(s + g.off_hw);
    a.xw = reinterpret_cast<uint64_t*>(s + g.off_xw);
    a.pw = reinterpret_cast<uint64_t*>(s + g.off_pw);
    a.err = p.err;
    a.ring_slots = g.ring_slots;
    for (int i = 0; i < 4; ++i) {
        a.tiles[i] = g.tiles[i];
        a.nbpt[i] = g.nbpt[i];
        a.ctas[i] = g.ctas[i];
    }
    a.kvt_off = g.kvt_off;
    a.work_bytes = g.work_bytes;
    a.bias_rows = g.bias_rows;
    a.taps = p.taps;
    a.tap_stride = rtaps(p.dims.hidden, p.dims.q_heads, p.dims.kv_heads, p.dims.head_dim, p.dims.intermediate).stride;
    a.spin_limit = p.spin_limit > 0 ? p.spin_limit : kRSpinLimit;
    a.stall_counter = p.stall_counter;
    a.world = p.world;
    a.rank = p.rank;
    a.peers = p.tp_peers;
    void (*kern)(RowArgs) = a.world > 1 ? decode_rows_kernel<true> : decode_rows_kernel<false>;
    cudaError_t st = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, g.smem);
    if (st != cudaSuccess) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(sms));
    cfg.blockDim = dim3(kRT);
    cfg.dynamicSmemBytes = static_cast<size_t>(g.smem);
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: they wait on each other
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace kc
