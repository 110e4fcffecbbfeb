// kc_launch.h -- host-side launchers for the sm_100a kernels (internal; the
// public surface is the C ABI in include/kudacuda.h).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace kc {

// dtype codes shared by the C ABI and the kernels
enum DType : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

// Launch with programmatic stream serialization so the kernel's prologue
// (table build, weight prefetch) overlaps the tail of the previous kernel.
// KUDACUDA_DISABLE_PDL=1 launches with plain stream order (compatibility /
// debugging control; every kernel still executes in full).
bool pdl_enabled();

template <typename Kernel, typename... Args>
inline cudaError_t launch_pdl(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

int device_sm_count();
// shared-memory capacities of the current device (cached per device)
size_t device_smem_per_sm();
size_t device_smem_per_block_optin();
size_t device_smem_reserved_per_block();
int current_device_index();

// ---- NF4 GEMV family -------------------------------------------------------
// dtype codes: 0 = f32, 1 = f16, 2 = bf16
struct GemvMat {
    const uint8_t* packed;
    const float* absmax;
    int rows;
};

// generic y = x W^T (+bias); x dtype xt, out/bias dtype ot
cudaError_t nf4_gemv(const void* x, int xt, GemvMat w, const void* bias, void* out, int ot, int K,
                     int* err, cudaStream_t s);
// resid = bf16(resid + bf16(x W^T)), x bf16 (o_proj / down_proj, Transformers order)
cudaError_t nf4_gemv_residual_bf16(const void* x, GemvMat w, void* resid, int K, int* err,
                                   cudaStream_t s);
// reference-ABI fused RMSNorm + Q/K/V (fp32-normalised), io dtype dt (1 or 2)
cudaError_t nf4_qkv_ref(const void* x, const void* norm_w, int dt, float eps, GemvMat q, GemvMat k,
                        GemvMat v, const void* qb, const void* kb, const void* vb, void* qo, void* ko,
                        void* vo, float* norm_ws, int K, int* err, cudaStream_t s);
// reference-ABI fused RMSNorm + gate/up SwiGLU, io dtype dt
cudaError_t nf4_swiglu_ref(const void* x, const void* norm_w, int dt, float eps, GemvMat g, GemvMat u,
                           void* out, int K, int* err, cudaStream_t s);
// Transformers-order bf16 RMSNorm + gate/up SwiGLU
cudaError_t nf4_swiglu_hf_bf16(const void* x, const void* norm_w, float eps, GemvMat g, GemvMat u,
                               void* out, int K, int* err, cudaStream_t s);
// Transformers-order bf16 RMSNorm + Q/K/V + bias + RoPE + KV append at *pos
struct QkvRopeArgs {
    const void* x;
    const void* norm_w;
    float eps;
    GemvMat q, k, v;
    const void *qb, *kb, *vb;  // bf16, may be null
    const uint16_t* rope_cos;  // bf16 [max_pos][head_dim/2]
    const uint16_t* rope_sin;
    int max_pos;
    const int32_t* pos_dev;
    void* q_out;                // bf16 [q_heads*head_dim]
    void* key_cache;            // bf16 [kv_heads][kv_cap][head_dim]
    void* value_cache;
    int q_heads, kv_heads, head_dim, kv_cap, K;
    int* err;
};
cudaError_t nf4_qkv_rope_hf_bf16(const QkvRopeArgs& a, cudaStream_t s);

cudaError_t nf4_dequantize(const uint8_t* packed, const float* absmax, int64_t n, int blocksize,
                           void* out, int ot, cudaStream_t s);
cudaError_t nf4_quantize(const void* in, int it, int64_t n, int blocksize, uint8_t* packed,
                         float* absmax, cudaStream_t s);

// ---- attention ---------------------------------------------------------------
struct GqaArgs {
    const void* q;       // [B][q_heads][d]
    const void* kcache;  // [B][kv_heads][stride][d]
    const void* vcache;
    void* out;           // [B][q_heads][d]
    float* partials;     // [B][q_heads][nsplit][d + 2]
    int* counters;       // [B * kv_heads], zero between launches (null: separate combine)
    const int32_t* kv_len_dev;  // null: use kv_len
    int kv_len_per_batch;       // 1: kv_len_dev is an array [batch] (batched decode), 0: one shared length
    int kv_shared;              // 1: every batch entry reads cache 0 (the queries of one sequence's prompt)
    int kv_len;
    int stride;
    int batch, q_heads, kv_heads, head_dim;
    float scale;
    int chunk, nsplit;
    int* err;
    int split_only;  // 1: always the split-KV kernel with its global partials (never the cluster kernel)
};
// dt: 1 = f16, 2 = bf16.  Chooses split size from the capacity / length.
void gqa_plan_splits(int kv_extent, int batch, int kv_heads, int max_splits, int* chunk, int* nsplit);
cudaError_t gqa_decode(GqaArgs a, int dt, cudaStream_t s);
// Allocation-free split-KV decode: partials and tickets live in a fixed
// file-scope device array (see gqa_decode.cu); a.partials/a.counters are
// ignored.  Plans its own splits; fails with cudaErrorInvalidValue when the
// partials or tickets would not fit.
cudaError_t gqa_decode_static_scratch(GqaArgs a, int dt, cudaStream_t s);
// true when a static-scratch call of these sizes fits the fixed array
bool gqa_static_fits(int batch, int q_heads, int kv_heads, int extent);
size_t gqa_partials_floats(int batch, int q_heads, int nsplit, int head_dim);

// ---- tensor-parallel step ops (tp_ops.cu) ---------------------------------------
struct ArgPair {
    float value;
    int32_t index;
};
cudaError_t residual_add_f32_bf16(const float* partial, void* resid, int n, cudaStream_t s);
cudaError_t argmax_shard_f32(const float* logits, int n, int index_base, float* ws, int* ticket, ArgPair* out,
                             cudaStream_t s);
int argmax_shard_workspace_floats();
cudaError_t select_token(const ArgPair* pairs, int count, int32_t* next_token, cudaStream_t s);
// RMSNorm (Transformers' bf16 rounding points) fused into an NF4 GEMV; out f32 or bf16
cudaError_t nf4_rmsnorm_gemv_bf16(const void* x, const void* norm_w, float eps, GemvMat w, void* out, int ot, int K,
                                  int* err, cudaStream_t s);

// ---- lm_head / embedding ------------------------------------------------------
struct LmHeadArgs {
    const void* hidden;      // bf16 [H] residual stream
    const void* final_norm;  // bf16 [H]
    const void* emb;         // bf16 [V][H] (tied embedding)
    void* logits;            // bf16 [V] or null
    int32_t* token_out;      // argmax token
    float* partials;         // [2 * grid] scratch
    int* counter;            // zero between launches
    int vocab, H;
    float eps;
    int* err;
};
cudaError_t lm_head_argmax_bf16(const LmHeadArgs& a, cudaStream_t s);
int lm_head_grid();
cudaError_t decode_advance(int32_t* state, const int32_t* next_token, int32_t* history, int history_len,
                           cudaStream_t s);
cudaError_t embedding_gather_bf16(const void* emb, const int32_t* token_dev, void* out, int H, int vocab,
                                  int* err, cudaStream_t s);

// ---- small ABI-compatibility ops ---------------------------------------------
cudaError_t vector_add_f32(const float* a, const float* b, float* out, int64_t n, cudaStream_t s);
cudaError_t rmsnorm_f32(const float* x, const float* w, float* out, int64_t rows, int64_t hidden,
                        float eps, cudaStream_t s);
cudaError_t dense_rmsnorm_qkv_f16(const void* x, const void* norm_w, const void* w, const void* bias,
                                  void* out, int64_t rows, int64_t hidden, float eps, cudaStream_t s);

// ---- persistent decode of all layers (decode_persistent.cu) ----------------------
// Weight stream layout ("group tiles"), built once from the bitsandbytes layout.
enum RetileMode : int {
    kRetilePlain = 0,    // rows 64g .. 64g + 63                    (o_proj, down, generic)
    kRetileSwiGlu = 1,   // gate rows 32g .. +31, then up rows 32g .. +31
    kRetileQkvRope = 2,  // q / k heads with RoPE partners 32 rows apart, then plain v rows
};
int retile_groups(int mode, int rows0, int rows1, int rows2, int head_dim);
cudaError_t nf4_retile(int mode, const uint8_t* const* packed, const float* const* absmax, const int* rows, int K,
                       int head_dim, uint8_t* out_codes, float* out_absmax, cudaStream_t stream);

struct PersistDims {
    int layers, hidden, q_heads, kv_heads, head_dim, intermediate, kv_capacity;
};
struct PersistLaunch {
    const uint64_t* layer_table;  // device [layers][16]
    PersistDims dims;
    int max_pos;
    float eps, scale;
    const int32_t* state;  // {token, pos, kv_len, pad}
    uint16_t* x;  // bf16 [hidden]: the step's input, then the last layer's output
    const uint16_t* rope_cos;
    const uint16_t* rope_sin;
    void* scratch;
    int* err;
    // test hooks (off: nullptr / 0 / -1): per-layer bf16 intermediates, the
    // poll limit of a dependency wait, a counter whose wait never completes
    uint16_t* taps = nullptr;
    uint32_t spin_limit = 0;
    int stall_counter = -1;
    // tensor parallelism (row-split kernel only): this rank of `world`, and
    // the device array of every rank's exchange buffer address (peer memory)
    int world = 1, rank = 0;
    const uint64_t* tp_peers = nullptr;
};
// elements of one layer's tap record of the persistent kernel
int64_t decode_persistent_tap_stride(const PersistDims& d);
// ---- row-split persistent decode (decode_rows.cu): 16-row tiles, each owned by one CTA
int retile16_tiles(int mode, int rows0, int rows1, int rows2, int head_dim);
cudaError_t nf4_retile16(int mode, const uint8_t* const* packed, const float* const* absmax, const int* rows, int K,
                         int head_dim, uint8_t* out, cudaStream_t stream);
int64_t decode_rows_scratch_bytes(const PersistDims& d, int sms);
const char* decode_rows_check(const PersistDims& d, int sms);
int64_t decode_rows_tap_stride(const PersistDims& d);
cudaError_t decode_layers_rows(const PersistLaunch& p, cudaStream_t stream);
// ---- batched decode (batched.cu) ----------------------------------------------
// NF4 (weight_type 0), bf16 (1) or re-tiled NF4 (2) weights [rows][K] times bf16 activations
// [n_pad][K] (rows >= batch zero) on the tcgen05 tensor cores: fp32 split-K
// partials[(split * total_rows + row_offset + r) * n_pad + b].
int batch_gemm_ksplit(int rows, int K);
// Fused epilogue of the GEMM (NF4 forms), run by the last CTA of each 128-row
// tile's splits (per-tile int32 tickets, zero before the first launch, reset
// by the kernel): 1 residual (resid[b][r] = bf16(resid + bf16(sum))), 2 SwiGLU
// (each tile = 64 gate rows then the same 64 up rows; hout[b][j]), 3 q/k/v
// (each tile = one 128-dim head of q | k | v: bias, RoPE, K/V append).
struct BatchEpilogue {
    int mode;
    int batch;
    int* tickets;
    uint16_t* resid;
    uint16_t* hout;
    int q_heads, kv_heads, cap, max_pos, shared_cache;
    const uint16_t* q_bias;
    const uint16_t* k_bias;
    const uint16_t* v_bias;
    const uint16_t* rope_cos;
    const uint16_t* rope_sin;
    const int32_t* pos;
    uint16_t* q_out;
    uint16_t* kcache;
    uint16_t* vcache;
};
// NF4 re-tiled for the GEMM (weight_type 2): per 128-row tile and 64-element
// K block one 4,608-byte record (codes [128][32 B], absmax [128] fp32)
int64_t batch_retile_bytes(int rows, int K);
cudaError_t batch_retile(const uint8_t* packed, const float* absmax, int rows, int K, uint8_t* out, cudaStream_t s);
cudaError_t batch_gemm(int weight_type, const void* weight, const float* absmax, int rows, int K, const uint16_t* x,
                       int n_pad, int ksplit, float* partials, int row_offset, int total_rows, int* err,
                       cudaStream_t s, const BatchEpilogue* epi = nullptr);
cudaError_t batch_rmsnorm(const uint16_t* x, const uint16_t* w, uint16_t* out, int batch, int H, float eps,
                          cudaStream_t s);
struct BatchQkv {
    const float* partials;  // [ksplit][(qh + 2 kvh) * hd][n_pad]
    int ksplit, n_pad, batch;
    int q_heads, kv_heads, head_dim, cap, max_pos;
    const uint16_t* q_bias;
    const uint16_t* k_bias;
    const uint16_t* v_bias;
    const uint16_t* rope_cos;
    const uint16_t* rope_sin;
    const int32_t* pos;  // [batch]
    uint16_t* q_out;     // [batch][qh][hd]
    uint16_t* kcache;    // [batch][kvh][cap][hd], or one [kvh][cap][hd] cache when shared
    uint16_t* vcache;
    int shared_cache;    // 1: every batch entry appends to cache 0 (the tokens of one prompt)
    int* err;
};
cudaError_t batch_qkv_epilogue(const BatchQkv& q, cudaStream_t s);
cudaError_t batch_residual(const float* partials, int ksplit, int rows, int n_pad, int batch, uint16_t* x,
                           cudaStream_t s);
cudaError_t batch_swiglu(const float* partials, int ksplit, int inter, int n_pad, int batch, uint16_t* h,
                         cudaStream_t s);
int batch_argmax_workspace_floats(int batch);
cudaError_t batch_argmax_advance(const float* partials, int ksplit, int vocab, int n_pad, int batch, float* ws,
                                 int32_t* state, int32_t* history, int history_len, cudaStream_t s);
cudaError_t batch_embedding(const uint16_t* emb, const int32_t* state, uint16_t* x, int batch, int H, int vocab,
                            int* err, cudaStream_t s);
cudaError_t batch_state_views(const int32_t* state, int batch, int32_t* pos, int32_t* kv_len, cudaStream_t s);
// tensor parallelism around the NCCL collectives
cudaError_t batch_split_sum(const float* partials, int ksplit, int rows, int n_pad, float* out, cudaStream_t s);
cudaError_t batch_argmax_pairs(const float* partials, int ksplit, int vocab, int n_pad, int batch, float* ws,
                               int index_base, int32_t* pairs, cudaStream_t s);
cudaError_t batch_select_advance(const int32_t* gathered, int world, int batch, int32_t* state, int32_t* history,
                                 int history_len, cudaStream_t s);

int64_t decode_persistent_scratch_bytes(const PersistDims& d, int sms);
const char* decode_persistent_check(const PersistDims& d, int sms);
cudaError_t decode_layers_persistent(const PersistLaunch& p, cudaStream_t stream);

}  // namespace kc
