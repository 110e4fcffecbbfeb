/*
 * kudacuda.h -- stable C ABI of the B200 (sm_100a) KudaCuda decode library.
 *
 * Part 1 keeps every symbol of the reference ABI (include/kudacuda.h:19-267 of
 * lijeuki/KudaCuda) with identical names, argument order and types, so the
 * reference's ctypes bridge (python/kudacuda_sidecar.py:259-419) binds this
 * library unchanged.  Part 2 adds versioned sm100 entry points (new names,
 * never changed signatures -- the way the reference itself added
 * kudacuda_qwen2_swiglu_nf4_bf16).
 *
 * Conventions (reference runtime/kudacuda_runtime.cu):
 *   - device pointers and the stream are uint64_t (a cudaStream_t value);
 *   - sizes are int64_t; epsilon and scale are float;
 *   - return 0 on success and 1 on failure; the message is available from
 *     kudacuda_last_error(handle) and is cleared by the next success;
 *   - every op call before kudacuda_freeze fails;
 *   - launches are asynchronous on the caller's stream and never synchronise
 *     (the one exception, kudacuda_sm100_graph_step_host, says so);
 *   - the caller owns all tensors and workspaces; the handle owns only its
 *     graph and a small scratch area allocated once by kudacuda_freeze.
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#define KUDACUDA_API __attribute__((visibility("default")))

#ifdef __cplusplus
extern "C" {
#endif

/* ===================== Part 1: reference ABI ===================== */

/* runtime/kudacuda_runtime.cu:266 -- create a handle bound to device_id. */
KUDACUDA_API void* kudacuda_create(int device_id);

/* runtime/kudacuda_runtime.cu:282 -- finish set-up; ops are accepted after it. */
KUDACUDA_API int kudacuda_freeze(void* handle);

/* runtime/kudacuda_runtime.cu:298-327 -- 1 if the tactic exists in this
 * library's tactic table and accepts (batch_size, seq_len), else 0. */
KUDACUDA_API int kudacuda_can_dispatch(void* handle, const char* tactic_name, int64_t batch_size,
                                       int64_t seq_len);

/* kernels/vector_add.cu:11-20 -- fp32 output = a + b. */
KUDACUDA_API int kudacuda_vector_add(void* handle, uint64_t a, uint64_t b, uint64_t output, int64_t count,
                                     uint64_t stream);

/* kernels/common/rmsnorm.cuh:11-47 -- fp32 row-wise RMSNorm. */
KUDACUDA_API int kudacuda_rmsnorm(void* handle, uint64_t input, uint64_t weight, uint64_t output, int64_t rows,
                                  int64_t hidden, float epsilon, uint64_t stream);

/* kernels/common/rmsnorm_qkv_reference.cuh:12-66 -- dense fp16 RMSNorm + [3H,H] QKV. */
KUDACUDA_API int kudacuda_fused_rmsnorm_qkv(void* handle, uint64_t input, uint64_t norm_weight,
                                            uint64_t qkv_weight, uint64_t bias, uint64_t output, int64_t rows,
                                            int64_t hidden, float epsilon, uint64_t stream);

/* runtime/kudacuda_runtime.cu:465 (v1), :541 (v2), :619 (v3) -- fp16 RMSNorm +
 * NF4 Q/K/V + bias, Qwen2.5-3B contract rows=1, hidden=2048, q_out=2048,
 * kv_out=256, blocksize=64.  All three run the same sm_100a kernel; v2/v3
 * also write the fp32 normalised vector to normalized_workspace [rows, hidden]. */
KUDACUDA_API int kudacuda_qwen2_fused_rmsnorm_qkv_nf4(
    void* handle, uint64_t input, uint64_t norm_weight, uint64_t q_weight_packed, uint64_t q_absmax,
    uint64_t q_bias, uint64_t k_weight_packed, uint64_t k_absmax, uint64_t k_bias, uint64_t v_weight_packed,
    uint64_t v_absmax, uint64_t v_bias, uint64_t q_output, uint64_t k_output, uint64_t v_output, int64_t rows,
    int64_t hidden, int64_t q_out, int64_t kv_out, int64_t blocksize, float epsilon, uint64_t stream);

KUDACUDA_API int kudacuda_qwen2_fused_rmsnorm_qkv_nf4_v2(
    void* handle, uint64_t input, uint64_t norm_weight, uint64_t q_weight_packed, uint64_t q_absmax,
    uint64_t q_bias, uint64_t k_weight_packed, uint64_t k_absmax, uint64_t k_bias, uint64_t v_weight_packed,
    uint64_t v_absmax, uint64_t v_bias, uint64_t normalized_workspace, uint64_t q_output, uint64_t k_output,
    uint64_t v_output, int64_t rows, int64_t hidden, int64_t q_out, int64_t kv_out, int64_t blocksize,
    float epsilon, uint64_t stream);

KUDACUDA_API int kudacuda_qwen2_fused_rmsnorm_qkv_nf4_v3(
    void* handle, uint64_t input, uint64_t norm_weight, uint64_t q_weight_packed, uint64_t q_absmax,
    uint64_t q_bias, uint64_t k_weight_packed, uint64_t k_absmax, uint64_t k_bias, uint64_t v_weight_packed,
    uint64_t v_absmax, uint64_t v_bias, uint64_t normalized_workspace, uint64_t q_output, uint64_t k_output,
    uint64_t v_output, int64_t rows, int64_t hidden, int64_t q_out, int64_t kv_out, int64_t blocksize,
    float epsilon, uint64_t stream);

/* runtime/kudacuda_runtime.cu:697 (fp16), :753 (bf16) -- RMSNorm + NF4
 * gate/up + SwiGLU, contract rows=1, hidden=2048, intermediate=11008, blocksize=64. */
KUDACUDA_API int kudacuda_qwen2_swiglu_nf4(void* handle, uint64_t input, uint64_t norm_weight,
                                           uint64_t gate_weight_packed, uint64_t gate_absmax,
                                           uint64_t up_weight_packed, uint64_t up_absmax, uint64_t output,
                                           int64_t rows, int64_t hidden, int64_t intermediate, int64_t blocksize,
                                           float epsilon, uint64_t stream);

KUDACUDA_API int kudacuda_qwen2_swiglu_nf4_bf16(void* handle, uint64_t input, uint64_t norm_weight,
                                                uint64_t gate_weight_packed, uint64_t gate_absmax,
                                                uint64_t up_weight_packed, uint64_t up_absmax, uint64_t output,
                                                int64_t rows, int64_t hidden, int64_t intermediate,
                                                int64_t blocksize, float epsilon, uint64_t stream);

/* runtime/kudacuda_runtime.cu:808 -- fp16 GQA decode with a caller workspace
 * of query_heads*8*(2+head_dim) floats; kv_capacity=512, length on device. */
KUDACUDA_API int kudacuda_qwen2_gqa_decode_workspace_v3(void* handle, uint64_t query, uint64_t key_cache,
                                                        uint64_t value_cache, uint64_t output, uint64_t workspace,
                                                        uint64_t kv_len_device, int64_t batch_size,
                                                        int64_t query_len, int64_t kv_capacity,
                                                        int64_t query_heads, int64_t kv_heads, int64_t head_dim,
                                                        float scale, uint64_t stream);

/* runtime/kudacuda_runtime.cu:868 -- fp16 GQA decode, kv_len 1..2048. */
KUDACUDA_API int kudacuda_qwen2_gqa_decode(void* handle, uint64_t query, uint64_t key_cache, uint64_t value_cache,
                                           uint64_t output, int64_t batch_size, int64_t query_len, int64_t kv_len,
                                           int64_t query_heads, int64_t kv_heads, int64_t head_dim, float scale,
                                           uint64_t stream);

/* runtime/kudacuda_runtime.cu:927 -- graph variant: length read from
 * kv_len_device (int32) at run time, caches strided by kv_capacity. */
KUDACUDA_API int kudacuda_qwen2_gqa_decode_graph(void* handle, uint64_t query, uint64_t key_cache,
                                                 uint64_t value_cache, uint64_t output, int64_t batch_size,
                                                 int64_t query_len, int64_t kv_capacity, int64_t query_heads,
                                                 int64_t kv_heads, int64_t head_dim, float scale,
                                                 uint64_t kv_len_device, uint64_t stream);

/* runtime/kudacuda_runtime.cu:986, :1045 -- experimental variants, kv_len 1..512. */
KUDACUDA_API int kudacuda_qwen2_gqa_decode_group_tiled(void* handle, uint64_t query, uint64_t key_cache,
                                                       uint64_t value_cache, uint64_t output, int64_t batch_size,
                                                       int64_t query_len, int64_t kv_len, int64_t query_heads,
                                                       int64_t kv_heads, int64_t head_dim, float scale,
                                                       uint64_t stream);

KUDACUDA_API int kudacuda_qwen2_gqa_decode_vectorized(void* handle, uint64_t query, uint64_t key_cache,
                                                      uint64_t value_cache, uint64_t output, int64_t batch_size,
                                                      int64_t query_len, int64_t kv_len, int64_t query_heads,
                                                      int64_t kv_heads, int64_t head_dim, float scale,
                                                      uint64_t stream);

/* runtime/kudacuda_runtime.cu:1104-1212 -- CUDA graph lifecycle on one handle. */
KUDACUDA_API int kudacuda_begin_capture(void* handle, uint64_t stream);
KUDACUDA_API int kudacuda_end_capture(void* handle, uint64_t stream);
KUDACUDA_API int kudacuda_replay_graph(void* handle, uint64_t stream);
KUDACUDA_API int kudacuda_reset_graph(void* handle);

/* runtime/kudacuda_runtime.cu:1216-1222, :1224-1226. */
KUDACUDA_API const char* kudacuda_last_error(void* handle);
KUDACUDA_API void kudacuda_destroy(void* handle);

/* ===================== Part 2: sm100 additions ===================== */
/* dtype codes: 0 = float32, 1 = float16, 2 = bfloat16. */

/* Generic batch-1 NF4 GEMV: output[r] = sum_k x[k] * W[r,k] (+ bias[r]).
 * W is bitsandbytes NF4 (packed [rows*k/2] u8, 16-byte aligned; fp32 absmax
 * [rows*k/blocksize]); k % 64 == 0, blocksize == 64.  Supported (x, out)
 * dtypes: (2,2) (2,0) (1,1) (1,0) (0,0) (0,2); bias has the output dtype.
 * No reference counterpart: the reference runs this GEMV in bitsandbytes
 * (python/kudacuda_sidecar.py:947, :1746). */
KUDACUDA_API int kudacuda_sm100_nf4_gemv(void* handle, uint64_t x, int x_dtype, uint64_t weight_packed,
                                         uint64_t absmax, uint64_t bias, uint64_t output, int out_dtype,
                                         int64_t rows, int64_t k, int64_t blocksize, uint64_t stream);

/* o_proj / down_proj in Transformers order: residual[r] = bf16(residual[r] +
 * bf16(x . W[r])), x and residual bf16.  Replaces bnb o_proj/down_proj plus
 * the residual add (python/kudacuda_sidecar.py:947, :1746-1747). */
KUDACUDA_API int kudacuda_sm100_nf4_linear_residual_bf16(void* handle, uint64_t x, uint64_t weight_packed,
                                                         uint64_t absmax, uint64_t residual, int64_t rows,
                                                         int64_t k, int64_t blocksize, uint64_t stream);

/* Bit-exact NF4 dequant: out[i] = level[code(i)] * absmax[i/blocksize]
 * (kernels/common/nf4_device.cuh:29-40), out dtype 0 (exact) or 2/1 (rounded). */
KUDACUDA_API int kudacuda_sm100_nf4_dequantize(void* handle, uint64_t weight_packed, uint64_t absmax,
                                               uint64_t output, int out_dtype, int64_t n, int64_t blocksize,
                                               uint64_t stream);

/* Blockwise NF4 quantiser (bitsandbytes' algorithm; blocksize 64). */
KUDACUDA_API int kudacuda_sm100_nf4_quantize(void* handle, uint64_t input, int input_dtype,
                                             uint64_t weight_packed, uint64_t absmax, int64_t n, int64_t blocksize,
                                             uint64_t stream);

/* Qwen2/Llama attention input block, bf16, Transformers rounding order:
 * RMSNorm -> NF4 q/k/v (+ optional bf16 biases) -> RoPE (bf16 cos/sin tables
 * [max_position][head_dim/2]) -> q to q_output [q_heads*head_dim], k/v appended
 * to key/value_cache [kv_heads][kv_capacity][head_dim] at *position_device
 * (int32).  Replaces the sidecar path python/kudacuda_sidecar.py:824-855 and
 * GraphStaticCache.update (python/kudacuda_static_decode.py:147-153). */
KUDACUDA_API int kudacuda_sm100_rmsnorm_qkv_rope_nf4_bf16(
    void* handle, uint64_t input, uint64_t norm_weight, uint64_t q_weight_packed, uint64_t q_absmax,
    uint64_t q_bias, uint64_t k_weight_packed, uint64_t k_absmax, uint64_t k_bias, uint64_t v_weight_packed,
    uint64_t v_absmax, uint64_t v_bias, uint64_t rope_cos, uint64_t rope_sin, uint64_t position_device,
    uint64_t q_output, uint64_t key_cache, uint64_t value_cache, int64_t hidden, int64_t q_heads,
    int64_t kv_heads, int64_t head_dim, int64_t kv_capacity, int64_t max_position, int64_t blocksize,
    float epsilon, uint64_t stream);

/* MLP input block, bf16, Transformers rounding order: RMSNorm -> NF4 gate/up ->
 * bf16(bf16(silu(g)) * u).  Any hidden/intermediate (k % 64 == 0). */
KUDACUDA_API int kudacuda_sm100_swiglu_nf4_bf16(void* handle, uint64_t input, uint64_t norm_weight,
                                                uint64_t gate_weight_packed, uint64_t gate_absmax,
                                                uint64_t up_weight_packed, uint64_t up_absmax, uint64_t output,
                                                int64_t hidden, int64_t intermediate, int64_t blocksize,
                                                float epsilon, uint64_t stream);

/* Split-KV GQA flash-decode (dtype 1 or 2), head_dim 128, query_heads /
 * kv_heads in {1,2,4,8}, batch B independent sequences.  The length comes
 * from kv_len_device (int32, graph-safe) when it is non-zero, else kv_len.
 * Caches are [B][kv_heads][kv_stride][128].  workspace: at least
 * kudacuda_sm100_gqa_workspace_bytes(...) bytes; tickets: B*kv_heads int32
 * that are zero before the first call (the kernel leaves them zero). */
KUDACUDA_API int kudacuda_sm100_gqa_decode(void* handle, uint64_t query, uint64_t key_cache, uint64_t value_cache,
                                           uint64_t output, uint64_t workspace, int64_t workspace_bytes,
                                           uint64_t tickets, uint64_t kv_len_device, int dtype, int64_t batch_size,
                                           int64_t kv_len, int64_t kv_stride, int64_t query_heads,
                                           int64_t kv_heads, int64_t head_dim, float scale, uint64_t stream);
KUDACUDA_API int64_t kudacuda_sm100_gqa_workspace_bytes(int64_t batch_size, int64_t query_heads,
                                                        int64_t kv_heads, int64_t kv_extent, int64_t head_dim);

/* Final RMSNorm + tied bf16 lm_head [vocab, hidden] + greedy argmax on the
 * device (lowest index on ties), token written to token_out (int32); logits
 * (bf16 [vocab]) written when non-zero.  workspace >=
 * kudacuda_sm100_lm_head_workspace_bytes(); ticket: one int32, zero before
 * the first call.  Replaces lm_head + argmax in Transformers
 * (tools/benchmark/benchmark_gemma.py:324, :350). */
KUDACUDA_API int kudacuda_sm100_lm_head_argmax_bf16(void* handle, uint64_t hidden_state, uint64_t final_norm,
                                                    uint64_t embedding, uint64_t logits, uint64_t token_out,
                                                    uint64_t workspace, int64_t workspace_bytes, uint64_t ticket,
                                                    int64_t vocab, int64_t hidden, float epsilon, uint64_t stream);
KUDACUDA_API int64_t kudacuda_sm100_lm_head_workspace_bytes(void);

/* output[0:hidden] = embedding[*token_device] (bf16 rows). */
KUDACUDA_API int kudacuda_sm100_embedding_bf16(void* handle, uint64_t embedding, uint64_t token_device,
                                               uint64_t output, int64_t vocab, int64_t hidden, uint64_t stream);

/* Device-resident decode loop: step_state is int32 {token, position, kv_len, -};
 * sets token = *next_token, position += 1, kv_len = position + 1, and
 * history[position] = token when history is non-zero (history_len entries). */
KUDACUDA_API int kudacuda_sm100_decode_advance(void* handle, uint64_t step_state, uint64_t next_token,
                                               uint64_t history, int64_t history_len, uint64_t stream);

/* One end-to-end step of a captured graph with host buffers: copy in_bytes
 * from host_in to device_in, replay the handle's graph, copy out_bytes from
 * device_out to host_out, and wait for the stream (this call synchronises). */
KUDACUDA_API int kudacuda_sm100_graph_step_host(void* handle, const void* host_in, uint64_t device_in,
                                                int64_t in_bytes, void* host_out, uint64_t device_out,
                                                int64_t out_bytes, uint64_t stream);

/* Device-side error word written by the kernels (bit 0: activation outside
 * the f16 range, 1: position outside the cache, 2: kv length outside the
 * cache, 3: token id outside the vocabulary, 4: a bounded wait on a barrier
 * or an async copy ran out).  Reading synchronises the handle's device;
 * clear != 0 resets it. */
KUDACUDA_API int kudacuda_sm100_error_word(void* handle, int* out_word, int clear);

/* Tensor-parallel step ops (no reference counterpart; the reference runs one
 * GPU).  rmsnorm_nf4_gemv: Transformers-order RMSNorm of bf16 input fused into
 * an NF4 GEMV (output f32 or bf16), used for a vocab-parallel NF4 lm_head.
 * residual_add_f32: residual = bf16(residual + bf16(partial_sum)) after the
 * allreduce of a row-parallel GEMV's fp32 partials.  argmax_shard_f32: greedy
 * argmax over this rank's slice of fp32 logits (compared after rounding to
 * bf16, lowest index on ties), writing one {float value; int32 index} pair
 * with index = index_base + local index; the ticket is an int32 that starts
 * at zero and resets itself.  select_token: lowest-index maximum over count
 * gathered pairs -> int32 next token. */
KUDACUDA_API int kudacuda_sm100_rmsnorm_nf4_gemv(void* handle, uint64_t input, uint64_t norm_weight,
                                                 uint64_t weight_packed, uint64_t absmax, uint64_t output,
                                                 int output_dtype, int64_t rows, int64_t hidden, float epsilon,
                                                 uint64_t stream);
KUDACUDA_API int kudacuda_sm100_residual_add_f32(void* handle, uint64_t partial_sum, uint64_t residual, int64_t n,
                                                 uint64_t stream);
KUDACUDA_API int64_t kudacuda_sm100_argmax_workspace_bytes(void);
KUDACUDA_API int kudacuda_sm100_argmax_shard_f32(void* handle, uint64_t logits, int64_t n, int64_t index_base,
                                                 uint64_t workspace, int64_t workspace_bytes, uint64_t ticket,
                                                 uint64_t out_pair, uint64_t stream);
KUDACUDA_API int kudacuda_sm100_select_token(void* handle, uint64_t pairs, int64_t count, uint64_t next_token,
                                             uint64_t stream);

/* Allocation-free GQA decode.  No reference counterpart: it exists for
 * callers that cannot allocate device memory for a workspace (e.g. a host
 * runtime without a device allocator at hand, or code that may not allocate
 * after start-up).  Same arithmetic and arguments as kudacuda_sm100_gqa_decode
 * minus the workspace and tickets: it always runs the split-KV kernel, whose
 * partials and tickets live in a fixed 1 MiB file-scope device array
 * (limit: batch * query_heads * splits * 130 floats <= 262144 and
 * batch * kv_heads <= 1024; larger requests fail with a message).  The first
 * call on each device looks the array up and zeroes its tickets, so it must
 * come before any stream capture on that device.  Calls that overlap in time
 * share the array and race: serialise them.  An overlap can also leave the
 * shared tickets nonzero, and then every later call on that device combines
 * at the wrong time (wrong results) until the library is unloaded.  It
 * allocates nothing and does not synchronise. */
KUDACUDA_API int kudacuda_sm100_gqa_decode_static(void* handle, uint64_t query, uint64_t key_cache,
                                                  uint64_t value_cache, uint64_t output, uint64_t kv_len_device,
                                                  int dtype, int64_t batch_size, int64_t kv_len, int64_t kv_stride,
                                                  int64_t query_heads, int64_t kv_heads, int64_t head_dim, float scale,
                                                  uint64_t stream);

/* Persistent decode of all decoder layers (no reference counterpart: the
 * reference launches one kernel per op and leaves o_proj/down to bitsandbytes,
 * python/kudacuda_sidecar.py:947, :1746).
 *
 * nf4_retile copies bitsandbytes NF4 weights (packed uint8 [rows * k / 2],
 * fp32 absmax [rows * k / 64]) into the stream layout the persistent kernel
 * reads: groups of 64 rows x 64-element blocks, 2048 code bytes + 256 absmax
 * bytes per (group, block), rows within a group ordered for the epilogue.
 * mode 0: one matrix (rows % 64 == 0); mode 1: gate (matrix 0) and up
 * (matrix 1), equal rows % 32 == 0; mode 2: q, k, v with RoPE partners of
 * each q/k head (head_dim % 64 == 0) in one group.  Outputs hold
 * groups * 64 * k / 2 code bytes and groups * 64 * k / 64 floats;
 * nf4_retile_groups returns groups (or -1 for unsupported shapes).
 *
 * decode_layers_persistent runs every layer of one batch-1 Qwen2/Llama decode
 * step (RMSNorm, QKV + bias + RoPE + KV append at state[1], GQA attention
 * over state[2] tokens, o_proj + residual, RMSNorm, gate/up SwiGLU,
 * down + residual; Transformers' bf16 rounding points) in one cooperative
 * launch of one CTA per SM.  layer_table is a device int64 [layers][16] of
 * pointers: qkv codes, qkv absmax, o codes, o absmax, gate/up codes, gate/up
 * absmax, down codes, down absmax (all from nf4_retile), input norm, post
 * norm, q bias, k bias, v bias (0 when absent), this layer's K cache and
 * V cache ([kv_heads][kv_capacity][head_dim] bf16), 0.  x (bf16 [hidden]) is
 * read as the step's input and holds the last layer's output afterwards.
 * scratch (size from decode_persistent_scratch_bytes, zeroed once by the
 * caller) holds partial sums and counters that reset themselves at the end of
 * each step; the result is deterministic (fixed summation order).
 * Requires head_dim 128, q_heads/kv_heads <= 8, hidden and intermediate
 * multiples of 64.  Device waits are bounded: a wait that runs out sets bit 4
 * of the error word and ends the step early instead of hanging. */
KUDACUDA_API int64_t kudacuda_sm100_nf4_retile_groups(int mode, int64_t rows0, int64_t rows1, int64_t rows2,
                                                      int64_t head_dim);
KUDACUDA_API int kudacuda_sm100_nf4_retile(void* handle, int mode, uint64_t packed0, uint64_t absmax0, int64_t rows0,
                                           uint64_t packed1, uint64_t absmax1, int64_t rows1, uint64_t packed2,
                                           uint64_t absmax2, int64_t rows2, int64_t k, int64_t head_dim,
                                           uint64_t out_codes, uint64_t out_absmax, uint64_t stream);
KUDACUDA_API int64_t kudacuda_sm100_decode_persistent_scratch_bytes(void* handle, int64_t layers, int64_t hidden,
                                                                   int64_t q_heads, int64_t kv_heads,
                                                                   int64_t head_dim, int64_t intermediate,
                                                                   int64_t kv_capacity);
KUDACUDA_API int kudacuda_sm100_decode_layers_persistent(void* handle, uint64_t layer_table, int64_t layers,
                                                         uint64_t x, uint64_t state, uint64_t rope_cos,
                                                         uint64_t rope_sin, int64_t max_pos, uint64_t scratch,
                                                         int64_t scratch_bytes,
                                                         int64_t hidden, int64_t q_heads, int64_t kv_heads,
                                                         int64_t head_dim, int64_t intermediate,
                                                         int64_t kv_capacity, float eps, float scale,
                                                         uint64_t stream);
/* Test hooks of the same kernel (no reference counterpart).  taps (0: off) is
 * a device bf16 buffer of layers * decode_persistent_tap_elements(...) / layers
 * elements per layer, taps_bytes its size; each layer's record receives
 * xn = RMSNorm(x) [hidden], q, k, v after bias and RoPE [q_heads * head_dim,
 * 2 x kv_heads * head_dim], the attention output [q_heads * head_dim],
 * x1 = x + o_proj [hidden], RMSNorm(x1) [hidden], h = SwiGLU [intermediate]
 * and x2 = x1 + down [hidden], in that order.  spin_limit (0: default)
 * bounds the polls of every dependency wait; stall_counter (-1: off) makes
 * the wait on one counter of layer 0 (0 qkv, 1 attention, 2 o_proj,
 * 3 gate/up, 4 down) unreachable, so that wait runs out, sets bit 4 of the
 * error word and ends the step early -- the bounded-wait path, exercised
 * without a fault.  Everything else is decode_layers_persistent. */
KUDACUDA_API int64_t kudacuda_sm100_decode_persistent_tap_elements(int64_t layers, int64_t hidden, int64_t q_heads,
                                                                  int64_t kv_heads, int64_t head_dim,
                                                                  int64_t intermediate);
KUDACUDA_API int kudacuda_sm100_decode_layers_persistent_debug(void* handle, uint64_t layer_table, int64_t layers,
                                                               uint64_t x, uint64_t state, uint64_t rope_cos,
                                                               uint64_t rope_sin, int64_t max_pos, uint64_t scratch,
                                                               int64_t scratch_bytes, int64_t hidden, int64_t q_heads,
                                                               int64_t kv_heads, int64_t head_dim,
                                                               int64_t intermediate, int64_t kv_capacity, float eps,
                                                               float scale, uint64_t taps, int64_t taps_bytes,
                                                               int64_t spin_limit, int64_t stall_counter,
                                                               uint64_t stream);

/* Row-split persistent decode (no reference counterpart): the same step as
 * decode_layers_persistent with a different work split -- every op's output
 * rows come in 16-row tiles, each owned by one CTA that streams all of its K
 * and finishes the rows itself (q/k after bias and RoPE with k and v written
 * into the cache row, x + o_proj, SwiGLU, x + down), so consumers read
 * finished vectors instead of partial sums.  nf4_retile16 copies
 * bitsandbytes NF4 tensors into its units (tile, 64-element block): 512 code
 * bytes in m16n8k16 lane order then the tile rows' 16 fp32 absmax as
 * (row g, row g + 8) pairs, 576 bytes, tile-major; modes as nf4_retile (0 plain, rows % 16 == 0; 1 gate/up in
 * tiles of 8 pairs; 2 q/k/v with q/k heads in tiles of 8 RoPE pairs, then
 * 16-row v tiles); nf4_retile16_tiles returns the tile count (-1 when
 * unsupported).  layer_table is a device int64 [layers][16]: qkv units, o
 * units, gate/up units, down units, input norm, post norm, q bias, k bias,
 * v bias (0 when absent), K cache, V cache, then zeros.  taps / spin_limit /
 * stall_counter are the test hooks of decode_layers_persistent_debug (the
 * same tap layout; stall index = layer * 16 + {0 qkv, 1 attention,
 * 2 o_proj, 3 gate/up, 4 down, 5 attention partials}).  Ops hand their
 * outputs to the next op as tagged 8-byte words in the scratch (two 16-bit
 * values, or one f32, plus a launch/layer/hop tag) that consumers poll
 * directly, so the scratch starts zeroed and is kept across steps (it also
 * counts the launches).  Deterministic (fixed summation order); every
 * device wait is bounded and reports bit 4 of the error word. */
KUDACUDA_API int64_t kudacuda_sm100_nf4_retile16_tiles(int mode, int64_t rows0, int64_t rows1, int64_t rows2,
                                                       int64_t head_dim);
KUDACUDA_API int kudacuda_sm100_nf4_retile16(void* handle, int mode, uint64_t packed0, uint64_t absmax0, int64_t rows0,
                                             uint64_t packed1, uint64_t absmax1, int64_t rows1, uint64_t packed2,
                                             uint64_t absmax2, int64_t rows2, int64_t k, int64_t head_dim,
                                             uint64_t out_units, int64_t out_bytes, uint64_t stream);
KUDACUDA_API int64_t kudacuda_sm100_decode_rows_scratch_bytes(void* handle, int64_t layers, int64_t hidden,
                                                             int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                                             int64_t intermediate, int64_t kv_capacity);
KUDACUDA_API int kudacuda_sm100_decode_layers_rows(void* handle, uint64_t layer_table, int64_t layers, uint64_t x,
                                                   uint64_t state, uint64_t rope_cos, uint64_t rope_sin,
                                                   int64_t max_pos, uint64_t scratch, int64_t scratch_bytes,
                                                   int64_t hidden, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                                   int64_t intermediate, int64_t kv_capacity, float eps, float scale,
                                                   uint64_t taps, int64_t taps_bytes, int64_t spin_limit,
                                                   int64_t stall_counter, uint64_t stream);

/* Tensor-parallel row-split decode (no reference counterpart; the reference
 * runs one GPU): rank `rank` of `world` (<= 8) runs decode_layers_rows over
 * its shard -- column-parallel q/k/v (its kv_heads / world heads) and gate/up,
 * row-parallel o_proj and down (K split on 64-element blocks) -- with q_heads,
 * kv_heads and intermediate the per-rank values.  The owner CTA of each
 * o_proj / down tile pushes its fp32 partial rows as tagged words straight
 * into every rank's exchange buffer over NVLink (plain peer stores, no
 * multicast), then polls its own buffer for the world partials of its rows,
 * sums them in rank order and finishes the residual add: the allreduce is
 * fused into the GEMV tile by tile, no collective library call.  tp_peers is
 * a device array of `world` uint64 addresses: every rank's exchange buffer
 * (tp_exchange_bytes(world, hidden) bytes, zeroed once, kept across steps)
 * as mapped in this process (ipc_alloc on the owner, ipc_open on the
 * others).  Every rank must launch the same steps in the same order; a peer
 * that never arrives ends the wait with bit 4 of the error word. */
KUDACUDA_API int kudacuda_sm100_decode_layers_rows_tp(void* handle, uint64_t layer_table, int64_t layers, uint64_t x,
                                                      uint64_t state, uint64_t rope_cos, uint64_t rope_sin,
                                                      int64_t max_pos, uint64_t scratch, int64_t scratch_bytes,
                                                      int64_t hidden, int64_t q_heads, int64_t kv_heads,
                                                      int64_t head_dim, int64_t intermediate, int64_t kv_capacity,
                                                      float eps, float scale, int64_t world, int64_t rank,
                                                      uint64_t tp_peers, uint64_t stream);
KUDACUDA_API int64_t kudacuda_sm100_tp_exchange_bytes(int64_t world, int64_t hidden);
/* CUDA IPC for the exchange buffers: ipc_alloc makes a zeroed device
 * allocation of its own and writes its 64-byte IPC handle; ipc_open maps a
 * peer's handle into this process; ipc_close unmaps (owned 0) or frees
 * (owned 1). */
KUDACUDA_API int kudacuda_sm100_ipc_alloc(void* handle, int64_t bytes, uint64_t* out_ptr, void* out_handle,
                                          int64_t handle_bytes);
KUDACUDA_API int kudacuda_sm100_ipc_open(void* handle, const void* ipc_handle, int64_t handle_bytes,
                                         uint64_t* out_ptr);
KUDACUDA_API int kudacuda_sm100_ipc_close(void* handle, uint64_t ptr, int owned);

/* Batched decode: B independent sequences advance one token per step.  No
 * reference counterpart (the reference's projections and its GQA contract,
 * python/kudacuda_sidecar.py:145-153, are batch 1); the arithmetic is what
 * Transformers does with bitsandbytes NF4 weights on a batch: every weight is
 * dequantised to bf16 (level * absmax in fp32, rounded once), the matmul runs
 * in bf16 with fp32 accumulation, activations are rounded to bf16 at the
 * batch-1 points.  Activations are bf16 [n_pad][K] with zero rows from B up
 * (n_pad in {16, 32, 64}, B <= n_pad).
 *
 * batch_gemm: partials[(s * total_rows + row_offset + r) * n_pad + b] =
 *   sum over split s's share of K of W[r][k] * x[b][k] (fp32), on the tcgen05
 *   tensor cores (weight as the 128-row M operand, the batch as N, fp32
 *   accumulator in TMEM).  weight_type 0: NF4 packed [rows][k/2] + fp32 absmax
 *   [rows][k/64]; 1: bf16 [rows][k] (absmax unused); 2: NF4 re-tiled by
 *   batch_retile (absmax unused, the fastest NF4 form).  ksplit in [1, k/64];
 *   batch_gemm_ksplit suggests one (the smallest split whose last wave of CTAs,
 *   two per SM, is well filled; at least 4 K blocks per CTA).  Several
 *   matrices may share one partials
 *   buffer through row_offset.
 * The epilogues sum the splits in split order (deterministic); their
 * partials pointer is 16-byte aligned, as batch_gemm requires of its own:
 *   batch_qkv_rope: partials rows q | k | v; bias, RoPE at pos[b] (int32 [B]),
 *     q -> q_out [B][qh][hd], k/v appended to caches [B][kvh][kv_capacity][hd]
 *     at pos[b];
 *   batch_residual: x[b][r] = bf16(x[b][r] + bf16(sum));
 *   batch_swiglu: out[b][j] = bf16(bf16(silu(bf16 gate)) * bf16 up) over
 *     partials rows gate (intermediate) | up (intermediate);
 *   batch_argmax_advance: per sequence, the lowest-index maximum of the
 *     bf16-rounded logits; state is int32 [B][4] = {token, pos, kv_len, pad}
 *     and becomes {argmax, pos + 1, pos + 2, pad}; history [B][history_len]
 *     (optional) records the token at its new position.
 * batch_rmsnorm: per sequence, Transformers' RMSNorm in bf16 (hidden % 8 == 0,
 *   hidden <= 8192, x / weight / out 16-byte aligned).
 * batch_embedding: x[b] = embedding[state[b].token]; batch_state_views copies
 * state's pos and kv_len columns to pos[B] and kv_len[B] for the RoPE
 * epilogue and gqa_decode_batch (kudacuda_sm100_gqa_decode, bf16, with a
 * per-sequence int32 length array; workspace and tickets as for
 * kudacuda_sm100_gqa_decode with kv_len = kv_stride).
 * shared_cache = 1 (batch_qkv_rope, gqa_decode_batch): every batch entry
 * appends to and attends over ONE cache [kvh][kv_capacity][hd] -- the batch
 * is the tokens of one prompt at positions pos[b] with causal lengths
 * kv_len[b] = pos[b] + 1 (prefill through the batched path). */
KUDACUDA_API int64_t kudacuda_sm100_batch_gemm_ksplit(int64_t rows, int64_t k);
/* batch_retile: copy a bitsandbytes NF4 matrix into the GEMM's streaming form
 * (weight_type 2): per 128-row tile and 64-element K block one contiguous
 * 4,608-byte record (codes [128][32 B], then the block's absmax [128] fp32;
 * rows past the matrix zero), so each block arrives with one bulk copy.
 * Bit-exact: every code byte and absmax value is moved, none changed. */
KUDACUDA_API int64_t kudacuda_sm100_batch_retile_bytes(int64_t rows, int64_t k);
KUDACUDA_API int kudacuda_sm100_batch_retile(void* handle, uint64_t packed, uint64_t absmax, int64_t rows, int64_t k,
                                             uint64_t out, int64_t out_bytes, uint64_t stream);
KUDACUDA_API int kudacuda_sm100_batch_gemm(void* handle, int weight_type, uint64_t weight, uint64_t absmax,
                                           int64_t rows, int64_t k, uint64_t x, int64_t n_pad, int64_t ksplit,
                                           uint64_t partials, int64_t row_offset, int64_t total_rows,
                                           uint64_t stream);
/* The GEMM with its epilogue fused (NF4 weights, weight_type 0 or 2): every
 * split writes its fp32 partial tile, takes a per-tile ticket, and the last
 * split of each 128-row tile sums the tile's splits in split order (the same
 * bits as batch_gemm + the separate epilogue) and finishes the op.  tickets:
 * int32 [ceil(rows / 128)], zero before the first call (the kernel resets
 * them); partials: ksplit * rows * n_pad floats.
 *   batch_gemm_residual: resid[b][r] = bf16(resid[b][r] + bf16(sum));
 *   batch_gemm_swiglu: weights of 2 * intermediate rows in 64-row tiles, each
 *     tile = gate rows 64t..64t+63 then up rows 64t..64t+63; out[b][j] =
 *     bf16(bf16(silu(bf16 gate_j)) * bf16 up_j);
 *   batch_gemm_qkv_rope: weights q | k | v by 128-row heads; the
 *     batch_qkv_rope epilogue per head. */
KUDACUDA_API int kudacuda_sm100_batch_gemm_residual(void* handle, int weight_type, uint64_t weight, uint64_t absmax,
                                                    int64_t rows, int64_t k, uint64_t x, int64_t n_pad,
                                                    int64_t ksplit, int64_t batch, uint64_t partials,
                                                    int64_t partials_bytes, uint64_t tickets, uint64_t resid,
                                                    uint64_t stream);
KUDACUDA_API int kudacuda_sm100_batch_gemm_swiglu(void* handle, int weight_type, uint64_t weight, uint64_t absmax,
                                                  int64_t intermediate, int64_t k, uint64_t x, int64_t n_pad,
                                                  int64_t ksplit, int64_t batch, uint64_t partials,
                                                  int64_t partials_bytes, uint64_t tickets, uint64_t out,
                                                  uint64_t stream);
KUDACUDA_API int kudacuda_sm100_batch_gemm_qkv_rope(void* handle, int weight_type, uint64_t weight, uint64_t absmax,
                                                    int64_t k, uint64_t x, int64_t n_pad, int64_t ksplit,
                                                    int64_t batch, uint64_t partials, int64_t partials_bytes,
                                                    uint64_t tickets, int64_t q_heads, int64_t kv_heads,
                                                    int64_t head_dim, uint64_t q_bias, uint64_t k_bias,
                                                    uint64_t v_bias, uint64_t rope_cos, uint64_t rope_sin,
                                                    int64_t max_pos, uint64_t pos, uint64_t q_out, uint64_t key_cache,
                                                    uint64_t value_cache, int64_t kv_capacity, int shared_cache,
                                                    uint64_t stream);
KUDACUDA_API int kudacuda_sm100_batch_rmsnorm(void* handle, uint64_t x, uint64_t weight, uint64_t out,
                                              int64_t batch, int64_t hidden, float eps, uint64_t stream);
KUDACUDA_API int kudacuda_sm100_batch_qkv_rope(void* handle, uint64_t partials, int64_t ksplit, int64_t n_pad,
                                               int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                               uint64_t q_bias, uint64_t k_bias, uint64_t v_bias, uint64_t rope_cos,
                                               uint64_t rope_sin, int64_t max_pos, uint64_t pos, uint64_t q_out,
                                               uint64_t key_cache, uint64_t value_cache, int64_t kv_capacity,
                                               int shared_cache, uint64_t stream);
KUDACUDA_API int kudacuda_sm100_batch_residual(void* handle, uint64_t partials, int64_t ksplit, int64_t rows,
                                               int64_t n_pad, int64_t batch, uint64_t x, uint64_t stream);
KUDACUDA_API int kudacuda_sm100_batch_swiglu(void* handle, uint64_t partials, int64_t ksplit, int64_t intermediate,
                                             int64_t n_pad, int64_t batch, uint64_t out, uint64_t stream);
KUDACUDA_API int64_t kudacuda_sm100_batch_argmax_workspace_bytes(int64_t batch);
KUDACUDA_API int kudacuda_sm100_batch_argmax_advance(void* handle, uint64_t partials, int64_t ksplit, int64_t vocab,
                                                     int64_t n_pad, int64_t batch, uint64_t workspace,
                                                     int64_t workspace_bytes, uint64_t state, uint64_t history,
                                                     int64_t history_len, uint64_t stream);
KUDACUDA_API int kudacuda_sm100_batch_embedding(void* handle, uint64_t embedding, uint64_t state, uint64_t x,
                                                int64_t batch, int64_t hidden, int64_t vocab, uint64_t stream);
KUDACUDA_API int kudacuda_sm100_batch_state_views(void* handle, uint64_t state, int64_t batch, uint64_t pos,
                                                  uint64_t kv_len, uint64_t stream);
/* Tensor parallelism around the NCCL collectives of a batched step:
 * batch_split_sum: out[r][b] = sum of the splits of a row-parallel GEMM's
 *   partials (split order), fp32 [rows][n_pad] -- the rank's partial that the
 *   caller allreduces, then adds with batch_residual (ksplit 1);
 * batch_argmax_pairs: per sequence, this rank's lowest-index maximum of the
 *   bf16-rounded logits of its vocabulary slice, as int32 pairs
 *   {float bits, index_base + local index} [batch][2];
 * batch_select_advance: per sequence, the lowest-index maximum over the
 *   ranks' gathered pairs [world][batch][2], then the state advance of
 *   batch_argmax_advance. */
KUDACUDA_API int kudacuda_sm100_batch_split_sum(void* handle, uint64_t partials, int64_t ksplit, int64_t rows,
                                                int64_t n_pad, uint64_t out, uint64_t stream);
KUDACUDA_API int kudacuda_sm100_batch_argmax_pairs(void* handle, uint64_t partials, int64_t ksplit, int64_t vocab,
                                                   int64_t n_pad, int64_t batch, uint64_t workspace,
                                                   int64_t workspace_bytes, int64_t index_base, uint64_t pairs,
                                                   uint64_t stream);
KUDACUDA_API int kudacuda_sm100_batch_select_advance(void* handle, uint64_t gathered, int64_t world, int64_t batch,
                                                     uint64_t state, uint64_t history, int64_t history_len,
                                                     uint64_t stream);
KUDACUDA_API int64_t kudacuda_sm100_gqa_batch_workspace_bytes(int64_t batch_size, int64_t query_heads,
                                                              int64_t kv_heads, int64_t kv_stride);
KUDACUDA_API int kudacuda_sm100_gqa_decode_batch(void* handle, uint64_t query, uint64_t key_cache,
                                                 uint64_t value_cache, uint64_t output, uint64_t workspace,
                                                 int64_t workspace_bytes, uint64_t tickets, uint64_t kv_len_array,
                                                 int64_t batch_size, int64_t kv_stride, int64_t query_heads,
                                                 int64_t kv_heads, int64_t head_dim, float scale, int shared_cache,
                                                 uint64_t stream);

/* Library / build identification: "sm_100a". */
KUDACUDA_API const char* kudacuda_sm100_target_arch(void);

#ifdef __cplusplus
}
#endif
