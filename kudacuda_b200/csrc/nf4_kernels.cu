// nf4_kernels.cu -- instantiations and launchers of the NF4 GEMV family, plus
// the bit-exact dequantiser and the on-device NF4 quantiser.
#include "kc_launch.h"
#include "nf4_gemv.cuh"
#include "kc_tma.h"
#include "nf4_gemv_mma.cuh"

#include <atomic>
#include <cstdlib>
#include <cstring>

namespace kc {

bool pdl_enabled() {
    static const bool enabled = std::getenv("KUDACUDA_DISABLE_PDL") == nullptr;
    return enabled;
}

int current_device_index() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    return dev;
}

int device_sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

namespace {
int device_attr_cached(int (&cache)[64], cudaDeviceAttr attr, int fallback) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fallback;
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, attr, dev) != cudaSuccess || n <= 0) n = fallback;
        cache[dev] = n;
    }
    return cache[dev];
}
}  // namespace

size_t device_smem_per_sm() {
    static int cached[64] = {0};
    return static_cast<size_t>(device_attr_cached(cached, cudaDevAttrMaxSharedMemoryPerMultiprocessor, 228 * 1024));
}
size_t device_smem_per_block_optin() {
    static int cached[64] = {0};
    return static_cast<size_t>(device_attr_cached(cached, cudaDevAttrMaxSharedMemoryPerBlockOptin, 227 * 1024));
}
size_t device_smem_reserved_per_block() {
    static int cached[64] = {0};
    return static_cast<size_t>(device_attr_cached(cached, cudaDevAttrReservedSharedMemoryPerBlock, 1024));
}

namespace {

inline Nf4Matrix to_mat(GemvMat g) { return Nf4Matrix{g.packed, g.absmax, g.rows}; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <int IN, int XT, int EPI, int OT>
cudaError_t run_gemv(Nf4GemvArgs& a, cudaStream_t s) {
    if (a.K <= 0 || (a.K % 64) != 0) return cudaErrorInvalidValue;
    for (int i = 0; i < 3; ++i) {
        if (a.m[i].packed != nullptr && (!aligned16(a.m[i].packed) || (reinterpret_cast<uintptr_t>(a.m[i].absmax) & 3u)))
            return cudaErrorMisalignedAddress;
    }
    a.ntasks = gemv_tasks(EPI, a);
    if (a.ntasks <= 0) return cudaSuccess;
    a.xvec = aligned16(a.x) && (a.norm_w == nullptr || aligned16(a.norm_w)) ? 1 : 0;
    const int dev = current_device_index();
    // Tensor-core kernel (table lookups -> mma fragments) unless the
    // measurement override asks for the CUDA-core variant.
    static const char* forced = std::getenv("KUDACUDA_NF4_GEMV_TACTIC");
    const bool use_mma = !(forced != nullptr && std::strcmp(forced, "fma") == 0);
    // TMA ring kernel when the tensor maps are legal: absmax rows must be
    // 16-byte strided (K % 256 == 0) and every base 16-byte aligned.
    bool tma_ok = use_mma && (a.K % 256) == 0 && !(forced != nullptr && std::strcmp(forced, "mma") == 0);
    GemvMaps maps;
    memset(&maps, 0, sizeof(maps));
    for (int i = 0; i < 3 && tma_ok; ++i) {
        if (a.m[i].packed == nullptr) continue;
        if (!aligned16(a.m[i].packed) || !aligned16(a.m[i].absmax)) {
            tma_ok = false;
            break;
        }
        const uint64_t rows = static_cast<uint64_t>(a.m[i].rows);
        if (encode_tmap_2d(&maps.w[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, a.m[i].packed, a.K / 2, rows, a.K / 2, 128, 8,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B) != cudaSuccess ||
            encode_tmap_2d(&maps.s[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.m[i].absmax, a.K / kBlocksize, rows,
                           a.K / kBlocksize * 4, kSliceBlocks, 8, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_128B) != cudaSuccess)
            tma_ok = false;
    }
    if (tma_ok) {
        auto kernel = nf4_gemv_tma_kernel<IN, XT, EPI, OT>;
        // per device: the kernel's static shared memory and the SM's budget
        static std::atomic<int> static_smem[64];
        int fixed = static_smem[dev].load(std::memory_order_acquire);
        if (fixed == 0) {
            cudaFuncAttributes fa;
            cudaError_t st = cudaFuncGetAttributes(&fa, kernel);
            if (st != cudaSuccess) return st;
            st = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(device_smem_per_block_optin() - fa.sharedSizeBytes));
            if (st != cudaSuccess) return st;
            fixed = static_cast<int>(fa.sharedSizeBytes);
            static_smem[dev].store(fixed, std::memory_order_release);
        }
        // Two resident CTAs per SM when there are more tiles than SMs, else
        // one CTA per SM with a deeper ring; the ring takes what is left
        // after the table, barriers, 1 KB alignment slack and the activations.
        const int tiles = mma_tiles<EPI>(a);
        const int sms = device_sm_count();
        const int per_sm = tiles > sms ? 2 : 1;
        const size_t xbytes = static_cast<size_t>(a.K) * 2;
        const size_t cta_budget = device_smem_per_sm() / per_sm - device_smem_reserved_per_block();
        const size_t dyn_cap = device_smem_per_block_optin() - fixed;
        size_t dyn_budget = cta_budget > static_cast<size_t>(fixed) ? cta_budget - fixed : 0;
        if (dyn_budget > dyn_cap) dyn_budget = dyn_cap;
        const size_t ring_budget = dyn_budget > 1024 + xbytes ? dyn_budget - 1024 - xbytes : 0;
        int stages = static_cast<int>(ring_budget / kTStageBytes);
        if (stages > kTMaxStages) stages = kTMaxStages;
        if (stages >= kTMinStages) {
            a.stages = stages;
            const size_t smem = 1024 + static_cast<size_t>(stages) * kTStageBytes + xbytes;
            const int blocks = tiles < sms * per_sm ? tiles : sms * per_sm;
            return launch_pdl(kernel, dim3(blocks), dim3(kTmaThreads), smem, s, a, maps);
        }
        // activations too large for a ring next to them: register-prefetch kernel below
    }
    if (use_mma) {
        const size_t smem = static_cast<size_t>(a.K) * 2;
        if (smem > 64 * 1024) return cudaErrorInvalidValue;
        auto kernel = nf4_gemv_mma_kernel<IN, XT, EPI, OT>;
        static std::atomic<bool> mma_attr[64];
        if (!mma_attr[dev].load(std::memory_order_acquire)) {
            const cudaError_t st = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
            if (st != cudaSuccess) return st;
            mma_attr[dev].store(true, std::memory_order_release);
        }
        const int tiles = mma_tiles<EPI>(a);
        int blocks = tiles < device_sm_count() * 2 ? tiles : device_sm_count() * 2;
        return launch_pdl(kernel, dim3(blocks), dim3(kMmaThreads), smem, s, a);
    }
    const size_t smem = static_cast<size_t>(a.K) * 2;
    auto kernel = nf4_gemv_kernel<IN, XT, EPI, OT>;
    // function attributes are per device: set once on each device used
    static std::atomic<bool> attr_set[64];
    if (!attr_set[dev].load(std::memory_order_acquire)) {
        const cudaError_t st = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
        if (st != cudaSuccess) return st;
        attr_set[dev].store(true, std::memory_order_release);
    }
    if (smem > 64 * 1024) return cudaErrorInvalidValue;
    const int warps = kGemvThreads / 32;
    const int max_blocks = device_sm_count() * 2;
    int blocks = (a.ntasks + warps - 1) / warps;
    if (blocks > max_blocks) blocks = max_blocks;
    return launch_pdl(kernel, dim3(blocks), dim3(kGemvThreads), smem, s, a);
}

Nf4GemvArgs blank_args() {
    Nf4GemvArgs a;
    memset(&a, 0, sizeof(a));
    return a;
}

}  // namespace

cudaError_t nf4_gemv(const void* x, int xt, GemvMat w, const void* bias, void* out, int ot, int K,
                     int* err, cudaStream_t s) {
    Nf4GemvArgs a = blank_args();
    a.m[0] = to_mat(w);
    a.K = K;
    a.x = x;
    a.bias[0] = bias;
    a.out[0] = out;
    a.err = err;
#define KC_GEMV_CASE(XT_, OT_) \
    if (xt == XT_ && ot == OT_) return run_gemv<kInRaw, XT_, kEpiStore, OT_>(a, s);
    KC_GEMV_CASE(kBF16, kBF16)
    KC_GEMV_CASE(kBF16, kF32)
    KC_GEMV_CASE(kF16, kF16)
    KC_GEMV_CASE(kF16, kF32)
    KC_GEMV_CASE(kF32, kF32)
    KC_GEMV_CASE(kF32, kBF16)
#undef KC_GEMV_CASE
    return cudaErrorInvalidValue;
}

cudaError_t nf4_rmsnorm_gemv_bf16(const void* x, const void* norm_w, float eps, GemvMat w, void* out, int ot, int K,
                                  int* err, cudaStream_t s) {
    Nf4GemvArgs a = blank_args();
    a.m[0] = to_mat(w);
    a.K = K;
    a.x = x;
    a.norm_w = norm_w;
    a.eps = eps;
    a.out[0] = out;
    a.err = err;
    if (ot == kF32) return run_gemv<kInNormHF, kBF16, kEpiStore, kF32>(a, s);
    if (ot == kBF16) return run_gemv<kInNormHF, kBF16, kEpiStore, kBF16>(a, s);
    return cudaErrorInvalidValue;
}

cudaError_t nf4_gemv_residual_bf16(const void* x, GemvMat w, void* resid, int K, int* err,
                                   cudaStream_t s) {
    Nf4GemvArgs a = blank_args();
    a.m[0] = to_mat(w);
    a.K = K;
    a.x = x;
    a.resid = resid;
    a.err = err;
    return run_gemv<kInRaw, kBF16, kEpiResidHF, kBF16>(a, s);
}

cudaError_t nf4_qkv_ref(const void* x, const void* norm_w, int dt, float eps, GemvMat q, GemvMat k,
                        GemvMat v, const void* qb, const void* kb, const void* vb, void* qo, void* ko,
                        void* vo, float* norm_ws, int K, int* err, cudaStream_t s) {
    if (k.rows != v.rows) return cudaErrorInvalidValue;
    Nf4GemvArgs a = blank_args();
    a.m[0] = to_mat(q);
    a.m[1] = to_mat(k);
    a.m[2] = to_mat(v);
    a.K = K;
    a.x = x;
    a.norm_w = norm_w;
    a.eps = eps;
    a.norm_ws = norm_ws;
    a.bias[0] = qb;
    a.bias[1] = kb;
    a.bias[2] = vb;
    a.out[0] = qo;
    a.out[1] = ko;
    a.out[2] = vo;
    a.err = err;
    if (dt == kF16) return run_gemv<kInNormRef, kF16, kEpiQkvRef, kF16>(a, s);
    if (dt == kBF16) return run_gemv<kInNormRef, kBF16, kEpiQkvRef, kBF16>(a, s);
    return cudaErrorInvalidValue;
}

cudaError_t nf4_swiglu_ref(const void* x, const void* norm_w, int dt, float eps, GemvMat g, GemvMat u,
                           void* out, int K, int* err, cudaStream_t s) {
    if (g.rows != u.rows) return cudaErrorInvalidValue;
    Nf4GemvArgs a = blank_args();
    a.m[0] = to_mat(g);
    a.m[1] = to_mat(u);
    a.K = K;
    a.x = x;
    a.norm_w = norm_w;
    a.eps = eps;
    a.out[0] = out;
    a.err = err;
    if (dt == kF16) return run_gemv<kInNormRef, kF16, kEpiSwiGluRef, kF16>(a, s);
    if (dt == kBF16) return run_gemv<kInNormRef, kBF16, kEpiSwiGluRef, kBF16>(a, s);
    return cudaErrorInvalidValue;
}

cudaError_t nf4_swiglu_hf_bf16(const void* x, const void* norm_w, float eps, GemvMat g, GemvMat u,
                               void* out, int K, int* err, cudaStream_t s) {
    if (g.rows != u.rows) return cudaErrorInvalidValue;
    Nf4GemvArgs a = blank_args();
    a.m[0] = to_mat(g);
    a.m[1] = to_mat(u);
    a.K = K;
    a.x = x;
    a.norm_w = norm_w;
    a.eps = eps;
    a.out[0] = out;
    a.err = err;
    return run_gemv<kInNormHF, kBF16, kEpiSwiGluHF, kBF16>(a, s);
}

cudaError_t nf4_qkv_rope_hf_bf16(const QkvRopeArgs& r, cudaStream_t s) {
    if (r.head_dim % 2 != 0 || r.q.rows != r.q_heads * r.head_dim || r.k.rows != r.kv_heads * r.head_dim ||
        r.v.rows != r.kv_heads * r.head_dim)
        return cudaErrorInvalidValue;
    Nf4GemvArgs a = blank_args();
    a.m[0] = to_mat(r.q);
    a.m[1] = to_mat(r.k);
    a.m[2] = to_mat(r.v);
    a.K = r.K;
    a.x = r.x;
    a.norm_w = r.norm_w;
    a.eps = r.eps;
    a.bias[0] = r.qb;
    a.bias[1] = r.kb;
    a.bias[2] = r.vb;
    a.out[0] = r.q_out;
    a.out[1] = r.key_cache;
    a.out[2] = r.value_cache;
    a.rope_cos = r.rope_cos;
    a.rope_sin = r.rope_sin;
    a.max_pos = r.max_pos;
    a.pos_dev = r.pos_dev;
    a.head_dim = r.head_dim;
    a.q_heads = r.q_heads;
    a.kv_heads = r.kv_heads;
    a.kv_cap = r.kv_cap;
    a.err = r.err;
    return run_gemv<kInNormHF, kBF16, kEpiQkvRopeHF, kBF16>(a, s);
}

// ---------------------------------------------------------------------------
// Bit-exact dequant: out[i] = level[code(i)] * absmax[i / blocksize], one fp32
// multiply (kernels/common/nf4_device.cuh:29-40).  Each thread expands one
// packed byte into two outputs.

template <int OT>
__global__ void nf4_dequant_kernel(const uint8_t* __restrict__ packed, const float* __restrict__ absmax,
                                   int64_t n, int blocksize, void* out) {
    pdl_launch_dependents();
    pdl_wait_on_producer();
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; 2 * b < n; b += stride) {
        const uint8_t byte = packed[b];
        const int64_t i0 = 2 * b;
        store_elem<OT>(out, i0, kNf4Levels[byte >> 4] * absmax[i0 / blocksize]);
        if (i0 + 1 < n) store_elem<OT>(out, i0 + 1, kNf4Levels[byte & 15] * absmax[(i0 + 1) / blocksize]);
    }
}

cudaError_t nf4_dequantize(const uint8_t* packed, const float* absmax, int64_t n, int blocksize,
                           void* out, int ot, cudaStream_t s) {
    if (n <= 0 || blocksize <= 0) return cudaErrorInvalidValue;
    const int64_t bytes = (n + 1) / 2;
    int64_t blocks = (bytes + 255) / 256;
    const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
    if (blocks > cap) blocks = cap;
    if (ot == kF32) return launch_pdl(nf4_dequant_kernel<kF32>, dim3(blocks), dim3(256), 0, s, packed, absmax, n, blocksize, out);
    if (ot == kBF16) return launch_pdl(nf4_dequant_kernel<kBF16>, dim3(blocks), dim3(256), 0, s, packed, absmax, n, blocksize, out);
    if (ot == kF16) return launch_pdl(nf4_dequant_kernel<kF16>, dim3(blocks), dim3(256), 0, s, packed, absmax, n, blocksize, out);
    return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------
// Blockwise NF4 quantiser (bitsandbytes' published algorithm): absmax =
// max|w| per block; n = w * (1/absmax) with IEEE reciprocal and multiply; code
// = number of level midpoints strictly below n; even element in the high
// nibble.  An all-zero block stores absmax 0 and the zero level (code 7).
// One warp per 64-element block; lane l owns elements 2l and 2l+1.

__constant__ float kNf4Midpoints[15];

template <int IT>
__global__ void nf4_quantize_kernel(const void* __restrict__ in, int64_t n, uint8_t* __restrict__ packed,
                                    float* __restrict__ absmax) {
    // No early launch_dependents: the GEMV kernels read weights before their
    // griddepcontrol.wait, so a kernel that writes weights releases its
    // dependents only by completing.
    pdl_wait_on_producer();
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    const int64_t nblocks = (n + 63) / 64;
    for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); b < nblocks; b += warps) {
        const int64_t i0 = b * 64 + 2 * lane;
        const float v0 = i0 < n ? load_elem<IT>(in, i0) : 0.0F;
        const float v1 = i0 + 1 < n ? load_elem<IT>(in, i0 + 1) : 0.0F;
        const float amax = warp_max(fmaxf(fabsf(v0), fabsf(v1)));
        if (lane == 0) absmax[b] = amax;
        if (i0 < n) {
            int c0 = 7, c1 = 7;
            if (amax > 0.0F) {
                const float inv = __frcp_rn(amax);
                const float n0 = __fmul_rn(v0, inv);
                const float n1 = __fmul_rn(v1, inv);
                c0 = 0;
                c1 = 0;
#pragma unroll
                for (int m = 0; m < 15; ++m) {
                    c0 += n0 > kNf4Midpoints[m] ? 1 : 0;
                    c1 += n1 > kNf4Midpoints[m] ? 1 : 0;
                }
                if (i0 + 1 >= n) c1 = 7;
            }
            packed[i0 >> 1] = static_cast<uint8_t>((c0 << 4) | c1);
        }
    }
}

cudaError_t nf4_quantize(const void* in, int it, int64_t n, int blocksize, uint8_t* packed,
                         float* absmax, cudaStream_t s) {
    if (blocksize != 64 || n <= 0) return cudaErrorInvalidValue;
    // __constant__ memory is per device: upload the midpoints once per device
    static std::atomic<bool> uploaded[64];
    const int dev = current_device_index();
    cudaError_t st = cudaSuccess;
    if (!uploaded[dev].load(std::memory_order_acquire)) {
        static const double levels[16] = {-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
                                          -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
                                          0.07958029955625534, 0.16093020141124725, 0.24611230194568634,
                                          0.33791524171829224, 0.44070982933044434, 0.5626170039176941,
                                          0.7229568362236023, 1.0};
        float mids[15];
        for (int i = 0; i < 15; ++i) {
            // levels are the fp32 codebook values widened exactly to double
            const double lo = static_cast<double>(static_cast<float>(levels[i]));
            const double hi = static_cast<double>(static_cast<float>(levels[i + 1]));
            mids[i] = static_cast<float>((lo + hi) * 0.5);
        }
        st = cudaMemcpyToSymbol(kNf4Midpoints, mids, sizeof(mids));
        if (st != cudaSuccess) return st;
        uploaded[dev].store(true, std::memory_order_release);
    }
    const int64_t nblocks = (n + 63) / 64;
    int64_t grid = (nblocks + 7) / 8;
    const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
    if (grid > cap) grid = cap;
    if (it == kF32) return launch_pdl(nf4_quantize_kernel<kF32>, dim3(grid), dim3(256), 0, s, in, n, packed, absmax);
    if (it == kBF16) return launch_pdl(nf4_quantize_kernel<kBF16>, dim3(grid), dim3(256), 0, s, in, n, packed, absmax);
    if (it == kF16) return launch_pdl(nf4_quantize_kernel<kF16>, dim3(grid), dim3(256), 0, s, in, n, packed, absmax);
    return cudaErrorInvalidValue;
}

}  // namespace kc
