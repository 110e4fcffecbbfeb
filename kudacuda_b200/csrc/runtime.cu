// runtime.cu -- the C ABI (include/kudacuda.h): handle, contract guards, graph
// lifecycle, and dispatch onto the sm_100a kernels.
//
// Mirrors runtime/kudacuda_runtime.cu of the reference: every entry point
// null-checks pointers, enforces the exact shape contract of its tactic,
// launches on the caller's stream, records failures in the per-handle
// last_error and returns 0/1.  Nothing here synchronises except
// kudacuda_sm100_graph_step_host and kudacuda_sm100_error_word, and nothing
// allocates per call: the small scratch area the reference-ABI attention
// entries need (they take no workspace argument) is allocated once by
// kudacuda_freeze.
#include "../../include/kudacuda.h"
#include "kc_launch.h"
#include "registry.h"

#include <cstring>
#include <new>
#include <string>

namespace kc {
namespace {

// scratch sizing for the reference-ABI GQA entries: batch 1, 16 query heads,
// at most 128 splits (chunks of 64..256 tokens cover up to 32768 tokens).
constexpr int kRefGqaMaxSplits = 128;
constexpr int kRefGqaHeads = 16;
// size bounds of the sm100 GQA entries, checked before any int arithmetic:
// batch * heads products stay far inside int
constexpr int64_t kMaxGqaBatch = 65536;
constexpr int64_t kMaxGqaHeads = 1024;

struct Handle {
    explicit Handle(int dev) : device_id(dev) {}
    ~Handle() {
        if (graph_exec != nullptr) cudaGraphExecDestroy(graph_exec);
        if (graph != nullptr) cudaGraphDestroy(graph);
        if (scratch != nullptr) cudaFree(scratch);
    }
    void set_error(const std::string& m) { last_error = m; }
    void set_cuda_error(const char* op, cudaError_t st) {
        last_error = std::string(op) + ": " + cudaGetErrorString(st);
    }

    int device_id;
    bool device_ready = false;
    bool frozen = false;
    bool capturing = false;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t graph_exec = nullptr;
    std::string last_error;
    // scratch: [err word (256 B)][gqa tickets (256 B)][lm ticket (256 B)][gqa partials][lm partials]
    char* scratch = nullptr;
    int* err_word = nullptr;
    int* gqa_tickets = nullptr;
    int* lm_ticket = nullptr;
    float* gqa_partials = nullptr;
    float* lm_partials = nullptr;
};

Handle* as_handle(void* h) { return reinterpret_cast<Handle*>(h); }

bool ready(Handle* h, const char* name) {
    if (h == nullptr) return false;
    if (!h->frozen) {
        h->set_error(std::string(name) + " called before kudacuda_freeze");
        return false;
    }
    return true;
}

int finish(Handle* h, const char* op, cudaError_t st) {
    if (st != cudaSuccess) {
        h->set_cuda_error(op, st);
        return 1;
    }
    h->last_error.clear();
    return 0;
}

template <typename T>
T* P(uint64_t v) {
    return reinterpret_cast<T*>(static_cast<uintptr_t>(v));
}
cudaStream_t S(uint64_t v) { return reinterpret_cast<cudaStream_t>(static_cast<uintptr_t>(v)); }

size_t ref_gqa_partial_bytes() {
    return gqa_partials_floats(1, kRefGqaHeads, kRefGqaMaxSplits, 128) * sizeof(float);
}

// Reference-ABI attention: fp16, batch 1, 16/2/128; stride = kv_len (direct)
// or capacity (graph / device length).
int run_ref_gqa(Handle* h, const char* op, uint64_t q, uint64_t k, uint64_t v, uint64_t out, int64_t kv_extent,
                const int32_t* kv_len_dev, float scale, uint64_t stream, float* partials, int max_splits,
                bool fused) {
    GqaArgs a;
    memset(&a, 0, sizeof(a));
    a.q = P<const void>(q);
    a.kcache = P<const void>(k);
    a.vcache = P<const void>(v);
    a.out = P<void>(out);
    a.partials = partials;
    a.counters = fused ? h->gqa_tickets : nullptr;
    a.kv_len_dev = kv_len_dev;
    a.kv_len = static_cast<int>(kv_extent);
    a.stride = static_cast<int>(kv_extent);
    a.batch = 1;
    a.q_heads = 16;
    a.kv_heads = 2;
    a.head_dim = 128;
    a.scale = scale;
    a.err = h->err_word;
    gqa_plan_splits(static_cast<int>(kv_extent), 1, 2, max_splits, &a.chunk, &a.nsplit);
    return finish(h, op, gqa_decode(a, kF16, S(stream)));
}

}  // namespace
}  // namespace kc

using kc::as_handle;
using kc::finish;
using kc::GemvMat;
using kc::Handle;
using kc::P;
using kc::ready;
using kc::S;

extern "C" {

void* kudacuda_create(int device_id) {
    auto* h = new (std::nothrow) Handle(device_id);
    if (h == nullptr) return nullptr;
    const cudaError_t st = cudaSetDevice(device_id);
    if (st != cudaSuccess) {
        h->set_cuda_error("cudaSetDevice", st);
        return h;
    }
    h->device_ready = true;
    return h;
}

int kudacuda_freeze(void* raw) {
    Handle* h = as_handle(raw);
    if (h == nullptr) return 1;
    if (!h->device_ready) {
        if (h->last_error.empty()) h->set_error("CUDA device is not ready");
        return 1;
    }
    if (h->scratch == nullptr) {
        const size_t lm_bytes = static_cast<size_t>(kc::lm_head_grid()) * 2 * sizeof(float);
        const size_t total = 768 + kc::ref_gqa_partial_bytes() + lm_bytes;
        cudaError_t st = cudaSetDevice(h->device_id);
        if (st == cudaSuccess) st = cudaMalloc(reinterpret_cast<void**>(&h->scratch), total);
        if (st == cudaSuccess) st = cudaMemset(h->scratch, 0, total);
        if (st == cudaSuccess) st = cudaDeviceSynchronize();
        if (st != cudaSuccess) {
            if (h->scratch != nullptr) cudaFree(h->scratch);
            h->scratch = nullptr;
            h->set_cuda_error("kudacuda_freeze scratch", st);
            return 1;
        }
        h->err_word = reinterpret_cast<int*>(h->scratch);
        h->gqa_tickets = reinterpret_cast<int*>(h->scratch + 256);
        h->lm_ticket = reinterpret_cast<int*>(h->scratch + 512);
        h->gqa_partials = reinterpret_cast<float*>(h->scratch + 768);
        h->lm_partials = reinterpret_cast<float*>(h->scratch + 768 + kc::ref_gqa_partial_bytes());
    }
    h->frozen = true;
    h->last_error.clear();
    return 0;
}

int kudacuda_can_dispatch(void* raw, const char* tactic_name, int64_t batch_size, int64_t seq_len) {
    const Handle* h = as_handle(raw);
    if (h == nullptr || !h->frozen || tactic_name == nullptr) return 0;
    if (batch_size <= 0 || seq_len <= 0) return 0;
    const kc::TacticEntry* t = kc::find_tactic(tactic_name);
    if (t == nullptr) return 0;
    if (t->max_batch > 0 && batch_size > t->max_batch) return 0;
    if (t->seq_len > 0 && seq_len != t->seq_len) return 0;
    return 1;
}

int kudacuda_vector_add(void* raw, uint64_t a, uint64_t b, uint64_t output, int64_t count, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_vector_add")) return 1;
    if (a == 0 || b == 0 || output == 0) {
        h->set_error("vector_add requires non-null device pointers");
        return 1;
    }
    if (count <= 0) {
        h->set_error("vector_add count must be positive");
        return 1;
    }
    return finish(h, "vector_add_kernel", kc::vector_add_f32(P<const float>(a), P<const float>(b), P<float>(output), count, S(stream)));
}

int kudacuda_rmsnorm(void* raw, uint64_t input, uint64_t weight, uint64_t output, int64_t rows, int64_t hidden,
                     float epsilon, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_rmsnorm")) return 1;
    if (input == 0 || weight == 0 || output == 0) {
        h->set_error("rmsnorm requires non-null device pointers");
        return 1;
    }
    if (rows <= 0 || hidden <= 0) {
        h->set_error("rmsnorm rows and hidden must be positive");
        return 1;
    }
    if (!(epsilon > 0.0F)) {
        h->set_error("rmsnorm epsilon must be positive");
        return 1;
    }
    return finish(h, "rmsnorm_kernel",
                  kc::rmsnorm_f32(P<const float>(input), P<const float>(weight), P<float>(output), rows, hidden, epsilon, S(stream)));
}

int kudacuda_fused_rmsnorm_qkv(void* raw, uint64_t input, uint64_t norm_weight, uint64_t qkv_weight, uint64_t bias,
                               uint64_t output, int64_t rows, int64_t hidden, float epsilon, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_fused_rmsnorm_qkv")) return 1;
    if (input == 0 || norm_weight == 0 || qkv_weight == 0 || output == 0) {
        h->set_error("fused_rmsnorm_qkv requires non-null input, weights, and output pointers");
        return 1;
    }
    if (rows <= 0 || hidden <= 0 || !(epsilon > 0.0F)) {
        h->set_error("fused_rmsnorm_qkv requires positive rows, hidden, and epsilon");
        return 1;
    }
    return finish(h, "fused_rmsnorm_qkv_kernel",
                  kc::dense_rmsnorm_qkv_f16(P<const void>(input), P<const void>(norm_weight), P<const void>(qkv_weight),
                                            P<const void>(bias), P<void>(output), rows, hidden, epsilon, S(stream)));
}

static int qkv_nf4_common(const char* name, const char* op, void* raw, uint64_t input, uint64_t norm_weight,
                          uint64_t qw, uint64_t qa, uint64_t qb, uint64_t kw, uint64_t ka, uint64_t kb, uint64_t vw,
                          uint64_t va, uint64_t vb, uint64_t ws, bool needs_ws, uint64_t qo, uint64_t ko, uint64_t vo,
                          int64_t rows, int64_t hidden, int64_t q_out, int64_t kv_out, int64_t blocksize,
                          float epsilon, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, name)) return 1;
    if (input == 0 || norm_weight == 0 || qw == 0 || qa == 0 || qb == 0 || kw == 0 || ka == 0 || kb == 0 ||
        vw == 0 || va == 0 || vb == 0 || qo == 0 || ko == 0 || vo == 0 || (needs_ws && ws == 0)) {
        h->set_error(std::string(op) + " requires non-null device pointers");
        return 1;
    }
    if (rows != 1 || hidden != 2048 || q_out != 2048 || kv_out != 256 || blocksize != 64 || !(epsilon > 0.0F)) {
        h->set_error(std::string(op) +
                     " requires rows=1, hidden=2048, q_out=2048, kv_out=256, blocksize=64, and positive epsilon");
        return 1;
    }
    return finish(h, op,
                  kc::nf4_qkv_ref(P<const void>(input), P<const void>(norm_weight), kc::kF16, epsilon,
                                  GemvMat{P<const uint8_t>(qw), P<const float>(qa), static_cast<int>(q_out)},
                                  GemvMat{P<const uint8_t>(kw), P<const float>(ka), static_cast<int>(kv_out)},
                                  GemvMat{P<const uint8_t>(vw), P<const float>(va), static_cast<int>(kv_out)},
                                  P<const void>(qb), P<const void>(kb), P<const void>(vb), P<void>(qo), P<void>(ko),
                                  P<void>(vo), needs_ws ? P<float>(ws) : nullptr, static_cast<int>(hidden),
                                  h->err_word, S(stream)));
}

int kudacuda_qwen2_fused_rmsnorm_qkv_nf4(void* raw, uint64_t input, uint64_t norm_weight, uint64_t qw, uint64_t qa,
                                         uint64_t qb, uint64_t kw, uint64_t ka, uint64_t kb, uint64_t vw, uint64_t va,
                                         uint64_t vb, uint64_t qo, uint64_t ko, uint64_t vo, int64_t rows,
                                         int64_t hidden, int64_t q_out, int64_t kv_out, int64_t blocksize,
                                         float epsilon, uint64_t stream) {
    return qkv_nf4_common("kudacuda_qwen2_fused_rmsnorm_qkv_nf4", "qwen2_fused_rmsnorm_qkv_nf4", raw, input,
                          norm_weight, qw, qa, qb, kw, ka, kb, vw, va, vb, 0, false, qo, ko, vo, rows, hidden, q_out,
                          kv_out, blocksize, epsilon, stream);
}

int kudacuda_qwen2_fused_rmsnorm_qkv_nf4_v2(void* raw, uint64_t input, uint64_t norm_weight, uint64_t qw,
                                            uint64_t qa, uint64_t qb, uint64_t kw, uint64_t ka, uint64_t kb,
                                            uint64_t vw, uint64_t va, uint64_t vb, uint64_t ws, uint64_t qo,
                                            uint64_t ko, uint64_t vo, int64_t rows, int64_t hidden, int64_t q_out,
                                            int64_t kv_out, int64_t blocksize, float epsilon, uint64_t stream) {
    return qkv_nf4_common("kudacuda_qwen2_fused_rmsnorm_qkv_nf4_v2", "qwen2_fused_rmsnorm_qkv_nf4_v2", raw, input,
                          norm_weight, qw, qa, qb, kw, ka, kb, vw, va, vb, ws, true, qo, ko, vo, rows, hidden, q_out,
                          kv_out, blocksize, epsilon, stream);
}

int kudacuda_qwen2_fused_rmsnorm_qkv_nf4_v3(void* raw, uint64_t input, uint64_t norm_weight, uint64_t qw,
                                            uint64_t qa, uint64_t qb, uint64_t kw, uint64_t ka, uint64_t kb,
                                            uint64_t vw, uint64_t va, uint64_t vb, uint64_t ws, uint64_t qo,
                                            uint64_t ko, uint64_t vo, int64_t rows, int64_t hidden, int64_t q_out,
                                            int64_t kv_out, int64_t blocksize, float epsilon, uint64_t stream) {
    return qkv_nf4_common("kudacuda_qwen2_fused_rmsnorm_qkv_nf4_v3", "qwen2_fused_rmsnorm_qkv_nf4_v3", raw, input,
                          norm_weight, qw, qa, qb, kw, ka, kb, vw, va, vb, ws, true, qo, ko, vo, rows, hidden, q_out,
                          kv_out, blocksize, epsilon, stream);
}

static int swiglu_common(const char* name, const char* op, int dt, bool clear_on_success, void* raw, uint64_t input,
                         uint64_t norm_weight, uint64_t gw, uint64_t ga, uint64_t uw, uint64_t ua, uint64_t out,
                         int64_t rows, int64_t hidden, int64_t inter, int64_t blocksize, float epsilon,
                         uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, name)) return 1;
    if (input == 0 || norm_weight == 0 || gw == 0 || ga == 0 || uw == 0 || ua == 0 || out == 0) {
        h->set_error(std::string(op) + " requires non-null device pointers");
        return 1;
    }
    if (rows != 1 || hidden != 2048 || inter != 11008 || blocksize != 64 || !(epsilon > 0.0F)) {
        h->set_error(std::string(op) +
                     " requires rows=1, hidden=2048, intermediate=11008, blocksize=64, and positive epsilon");
        return 1;
    }
    const cudaError_t st = kc::nf4_swiglu_ref(
        P<const void>(input), P<const void>(norm_weight), dt, epsilon,
        GemvMat{P<const uint8_t>(gw), P<const float>(ga), static_cast<int>(inter)},
        GemvMat{P<const uint8_t>(uw), P<const float>(ua), static_cast<int>(inter)}, P<void>(out),
        static_cast<int>(hidden), h->err_word, S(stream));
    if (st != cudaSuccess) {
        h->set_cuda_error(dt == kc::kF16 ? "nf4_swiglu" : "nf4_swiglu_bf16", st);
        return 1;
    }
    // runtime/kudacuda_runtime.cu:750 -- the fp16 entry leaves last_error as is on success
    if (clear_on_success) h->last_error.clear();
    return 0;
}

int kudacuda_qwen2_swiglu_nf4(void* raw, uint64_t input, uint64_t norm_weight, uint64_t gw, uint64_t ga,
                              uint64_t uw, uint64_t ua, uint64_t out, int64_t rows, int64_t hidden, int64_t inter,
                              int64_t blocksize, float epsilon, uint64_t stream) {
    return swiglu_common("kudacuda_qwen2_swiglu_nf4", "qwen2_swiglu_nf4", kc::kF16, false, raw, input, norm_weight, gw,
                         ga, uw, ua, out, rows, hidden, inter, blocksize, epsilon, stream);
}

int kudacuda_qwen2_swiglu_nf4_bf16(void* raw, uint64_t input, uint64_t norm_weight, uint64_t gw, uint64_t ga,
                                   uint64_t uw, uint64_t ua, uint64_t out, int64_t rows, int64_t hidden,
                                   int64_t inter, int64_t blocksize, float epsilon, uint64_t stream) {
    return swiglu_common("kudacuda_qwen2_swiglu_nf4_bf16", "qwen2_swiglu_nf4_bf16", kc::kBF16, true, raw, input,
                         norm_weight, gw, ga, uw, ua, out, rows, hidden, inter, blocksize, epsilon, stream);
}

int kudacuda_qwen2_gqa_decode_workspace_v3(void* raw, uint64_t query, uint64_t key_cache, uint64_t value_cache,
                                           uint64_t output, uint64_t workspace, uint64_t kv_len_device,
                                           int64_t batch_size, int64_t query_len, int64_t kv_capacity,
                                           int64_t query_heads, int64_t kv_heads, int64_t head_dim, float scale,
                                           uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_qwen2_gqa_decode_workspace_v3")) return 1;
    if (query == 0 || key_cache == 0 || value_cache == 0 || output == 0 || workspace == 0 || kv_len_device == 0) {
        h->set_error("qwen2_gqa_decode_workspace_v3 requires non-null device pointers");
        return 1;
    }
    if (batch_size != 1 || query_len != 1 || kv_capacity != 512 || query_heads != 16 || kv_heads != 2 ||
        head_dim != 128 || !(scale > 0.0F)) {
        h->set_error(
            "qwen2_gqa_decode_workspace_v3 requires 1x1, capacity=512, heads=16/2, head_dim=128, and positive scale");
        return 1;
    }
    // The caller's workspace holds query_heads * 8 * (2 + head_dim) floats
    // (python/kudacuda_sidecar.py:685): 8 splits of 64 tokens, combined by a
    // second kernel because there is no room for tickets.
    return kc::run_ref_gqa(h, "qwen2_gqa_decode_workspace_v3_kernel", query, key_cache, value_cache, output, 512,
                           P<const int32_t>(kv_len_device), scale, stream, P<float>(workspace), 8, false);
}

static int gqa_ref_direct(const char* name, const char* op, const char* guard_msg, int64_t max_len, void* raw,
                          uint64_t query, uint64_t key_cache, uint64_t value_cache, uint64_t output,
                          int64_t batch_size, int64_t query_len, int64_t kv_len, int64_t query_heads,
                          int64_t kv_heads, int64_t head_dim, float scale, uint64_t stream,
                          const int32_t* kv_len_dev) {
    Handle* h = as_handle(raw);
    if (!ready(h, name)) return 1;
    if (query == 0 || key_cache == 0 || value_cache == 0 || output == 0 ||
        (kv_len_dev == nullptr && std::strstr(op, "graph") != nullptr)) {
        h->set_error(std::string(op) + " requires non-null device pointers");
        return 1;
    }
    if (batch_size != 1 || query_len != 1 || kv_len < 1 || kv_len > max_len || query_heads != 16 || kv_heads != 2 ||
        head_dim != 128) {
        h->set_error(guard_msg);
        return 1;
    }
    if (!(scale > 0.0F)) {
        h->set_error(std::string(op) + " scale must be positive");
        return 1;
    }
    return kc::run_ref_gqa(h, (std::string(op) + "_kernel").c_str(), query, key_cache, value_cache, output, kv_len,
                           kv_len_dev, scale, stream, h->gqa_partials, kc::kRefGqaMaxSplits, true);
}

int kudacuda_qwen2_gqa_decode(void* raw, uint64_t query, uint64_t key_cache, uint64_t value_cache, uint64_t output,
                              int64_t batch_size, int64_t query_len, int64_t kv_len, int64_t query_heads,
                              int64_t kv_heads, int64_t head_dim, float scale, uint64_t stream) {
    return gqa_ref_direct("kudacuda_qwen2_gqa_decode", "qwen2_gqa_decode",
                          "qwen2_gqa_decode requires batch=1, query_len=1, kv_len=1..2048, q_heads=16, kv_heads=2, "
                          "head_dim=128",
                          2048, raw, query, key_cache, value_cache, output, batch_size, query_len, kv_len, query_heads,
                          kv_heads, head_dim, scale, stream, nullptr);
}

int kudacuda_qwen2_gqa_decode_graph(void* raw, uint64_t query, uint64_t key_cache, uint64_t value_cache,
                                    uint64_t output, int64_t batch_size, int64_t query_len, int64_t kv_capacity,
                                    int64_t query_heads, int64_t kv_heads, int64_t head_dim, float scale,
                                    uint64_t kv_len_device, uint64_t stream) {
    return gqa_ref_direct("kudacuda_qwen2_gqa_decode_graph", "qwen2_gqa_decode_graph",
                          "qwen2_gqa_decode_graph requires batch=1, query_len=1, kv_capacity=1..512, q_heads=16, "
                          "kv_heads=2, head_dim=128",
                          512, raw, query, key_cache, value_cache, output, batch_size, query_len, kv_capacity,
                          query_heads, kv_heads, head_dim, scale, stream, P<const int32_t>(kv_len_device));
}

int kudacuda_qwen2_gqa_decode_group_tiled(void* raw, uint64_t query, uint64_t key_cache, uint64_t value_cache,
                                          uint64_t output, int64_t batch_size, int64_t query_len, int64_t kv_len,
                                          int64_t query_heads, int64_t kv_heads, int64_t head_dim, float scale,
                                          uint64_t stream) {
    return gqa_ref_direct("kudacuda_qwen2_gqa_decode_group_tiled", "qwen2_gqa_decode_group_tiled",
                          "qwen2_gqa_decode_group_tiled requires batch=1, query_len=1, kv_len=1..512, q_heads=16, "
                          "kv_heads=2, head_dim=128",
                          512, raw, query, key_cache, value_cache, output, batch_size, query_len, kv_len, query_heads,
                          kv_heads, head_dim, scale, stream, nullptr);
}

int kudacuda_qwen2_gqa_decode_vectorized(void* raw, uint64_t query, uint64_t key_cache, uint64_t value_cache,
                                         uint64_t output, int64_t batch_size, int64_t query_len, int64_t kv_len,
                                         int64_t query_heads, int64_t kv_heads, int64_t head_dim, float scale,
                                         uint64_t stream) {
    return gqa_ref_direct("kudacuda_qwen2_gqa_decode_vectorized", "qwen2_gqa_decode_vectorized",
                          "qwen2_gqa_decode_vectorized requires batch=1, query_len=1, kv_len=1..512, q_heads=16, "
                          "kv_heads=2, head_dim=128",
                          512, raw, query, key_cache, value_cache, output, batch_size, query_len, kv_len, query_heads,
                          kv_heads, head_dim, scale, stream, nullptr);
}

int kudacuda_begin_capture(void* raw, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (h == nullptr || !h->frozen) {
        if (h != nullptr) h->set_error("kudacuda_begin_capture requires a frozen handle");
        return 1;
    }
    if (h->capturing) {
        h->set_error("CUDA graph capture is already active");
        return 1;
    }
    const cudaError_t st = cudaStreamBeginCapture(S(stream), cudaStreamCaptureModeGlobal);
    if (st != cudaSuccess) {
        h->set_cuda_error("cudaStreamBeginCapture", st);
        return 1;
    }
    h->capturing = true;
    h->last_error.clear();
    return 0;
}

int kudacuda_end_capture(void* raw, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (h == nullptr || !h->capturing) {
        if (h != nullptr) h->set_error("kudacuda_end_capture called without active capture");
        return 1;
    }
    const cudaError_t end_st = cudaStreamEndCapture(S(stream), &h->graph);
    h->capturing = false;
    if (end_st != cudaSuccess) {
        h->set_cuda_error("cudaStreamEndCapture", end_st);
        return 1;
    }
    if (h->graph_exec != nullptr) {
        cudaGraphExecDestroy(h->graph_exec);
        h->graph_exec = nullptr;
    }
    const cudaError_t inst = cudaGraphInstantiate(&h->graph_exec, h->graph, 0);
    cudaGraphDestroy(h->graph);
    h->graph = nullptr;
    if (inst != cudaSuccess) {
        h->graph_exec = nullptr;
        h->set_cuda_error("cudaGraphInstantiate", inst);
        return 1;
    }
    h->last_error.clear();
    return 0;
}

int kudacuda_replay_graph(void* raw, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (h == nullptr || h->graph_exec == nullptr) {
        if (h != nullptr) h->set_error("kudacuda_replay_graph called before graph instantiation");
        return 1;
    }
    return finish(h, "cudaGraphLaunch", cudaGraphLaunch(h->graph_exec, S(stream)));
}

int kudacuda_reset_graph(void* raw) {
    Handle* h = as_handle(raw);
    if (h == nullptr) return 1;
    if (h->capturing) {
        h->set_error("kudacuda_reset_graph called during active capture");
        return 1;
    }
    if (h->graph_exec != nullptr) {
        const cudaError_t st = cudaGraphExecDestroy(h->graph_exec);
        if (st != cudaSuccess) {
            h->set_cuda_error("cudaGraphExecDestroy", st);
            return 1;
        }
        h->graph_exec = nullptr;
    }
    if (h->graph != nullptr) {
        const cudaError_t st = cudaGraphDestroy(h->graph);
        if (st != cudaSuccess) {
            h->set_cuda_error("cudaGraphDestroy", st);
            return 1;
        }
        h->graph = nullptr;
    }
    h->last_error.clear();
    return 0;
}

const char* kudacuda_last_error(void* raw) {
    const Handle* h = as_handle(raw);
    if (h == nullptr) return "invalid KudaCuda handle";
    return h->last_error.c_str();
}

void kudacuda_destroy(void* raw) { delete as_handle(raw); }

// =========================== sm100 additions ===========================

int kudacuda_sm100_nf4_gemv(void* raw, uint64_t x, int x_dtype, uint64_t w, uint64_t absmax, uint64_t bias,
                            uint64_t output, int out_dtype, int64_t rows, int64_t k, int64_t blocksize,
                            uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_nf4_gemv")) return 1;
    if (x == 0 || w == 0 || absmax == 0 || output == 0) {
        h->set_error("sm100_nf4_gemv requires non-null device pointers");
        return 1;
    }
    if (rows < 1 || rows > (1 << 30) || k < 64 || k % 64 != 0 || k > 16384 || blocksize != 64) {
        h->set_error("sm100_nf4_gemv requires rows>=1, k a multiple of 64 in 64..16384, blocksize=64");
        return 1;
    }
    if ((w & 15u) != 0) {
        h->set_error("sm100_nf4_gemv requires a 16-byte aligned packed weight");
        return 1;
    }
    return finish(h, "nf4_gemv_kernel",
                  kc::nf4_gemv(P<const void>(x), x_dtype, GemvMat{P<const uint8_t>(w), P<const float>(absmax), static_cast<int>(rows)},
                               P<const void>(bias), P<void>(output), out_dtype, static_cast<int>(k), h->err_word, S(stream)));
}

int kudacuda_sm100_nf4_linear_residual_bf16(void* raw, uint64_t x, uint64_t w, uint64_t absmax, uint64_t residual,
                                            int64_t rows, int64_t k, int64_t blocksize, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_nf4_linear_residual_bf16")) return 1;
    if (x == 0 || w == 0 || absmax == 0 || residual == 0) {
        h->set_error("sm100_nf4_linear_residual_bf16 requires non-null device pointers");
        return 1;
    }
    if (rows < 1 || rows > (1 << 30) || k < 64 || k % 64 != 0 || k > 16384 || blocksize != 64 || (w & 15u) != 0) {
        h->set_error("sm100_nf4_linear_residual_bf16 requires rows>=1, k%64==0 (<=16384), blocksize=64, aligned weight");
        return 1;
    }
    return finish(h, "nf4_linear_residual_kernel",
                  kc::nf4_gemv_residual_bf16(P<const void>(x), GemvMat{P<const uint8_t>(w), P<const float>(absmax), static_cast<int>(rows)},
                                             P<void>(residual), static_cast<int>(k), h->err_word, S(stream)));
}

int kudacuda_sm100_nf4_dequantize(void* raw, uint64_t w, uint64_t absmax, uint64_t output, int out_dtype, int64_t n,
                                  int64_t blocksize, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_nf4_dequantize")) return 1;
    if (w == 0 || absmax == 0 || output == 0) {
        h->set_error("sm100_nf4_dequantize requires non-null device pointers");
        return 1;
    }
    if (n < 1 || blocksize < 1 || blocksize > (1 << 20) || out_dtype < 0 || out_dtype > 2) {
        h->set_error("sm100_nf4_dequantize requires n>=1, a positive blocksize and dtype 0..2");
        return 1;
    }
    return finish(h, "nf4_dequant_kernel",
                  kc::nf4_dequantize(P<const uint8_t>(w), P<const float>(absmax), n, static_cast<int>(blocksize),
                                     P<void>(output), out_dtype, S(stream)));
}

int kudacuda_sm100_nf4_quantize(void* raw, uint64_t input, int input_dtype, uint64_t w, uint64_t absmax, int64_t n,
                                int64_t blocksize, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_nf4_quantize")) return 1;
    if (input == 0 || w == 0 || absmax == 0) {
        h->set_error("sm100_nf4_quantize requires non-null device pointers");
        return 1;
    }
    if (n < 1 || blocksize != 64 || input_dtype < 0 || input_dtype > 2) {
        h->set_error("sm100_nf4_quantize requires n>=1, blocksize=64 and dtype 0..2");
        return 1;
    }
    return finish(h, "nf4_quantize_kernel",
                  kc::nf4_quantize(P<const void>(input), input_dtype, n, 64, P<uint8_t>(w), P<float>(absmax), S(stream)));
}

int kudacuda_sm100_rmsnorm_qkv_rope_nf4_bf16(void* raw, uint64_t input, uint64_t norm_weight, uint64_t qw,
                                             uint64_t qa, uint64_t qb, uint64_t kw, uint64_t ka, uint64_t kb,
                                             uint64_t vw, uint64_t va, uint64_t vb, uint64_t rope_cos,
                                             uint64_t rope_sin, uint64_t position_device, uint64_t q_output,
                                             uint64_t key_cache, uint64_t value_cache, int64_t hidden,
                                             int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                             int64_t kv_capacity, int64_t max_position, int64_t blocksize,
                                             float epsilon, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_rmsnorm_qkv_rope_nf4_bf16")) return 1;
    if (input == 0 || norm_weight == 0 || qw == 0 || qa == 0 || kw == 0 || ka == 0 || vw == 0 || va == 0 ||
        rope_cos == 0 || rope_sin == 0 || position_device == 0 || q_output == 0 || key_cache == 0 || value_cache == 0) {
        h->set_error("sm100_rmsnorm_qkv_rope_nf4_bf16 requires non-null device pointers (biases may be null)");
        return 1;
    }
    if (hidden < 64 || hidden % 64 != 0 || hidden > 16384 || q_heads < 1 || kv_heads < 1 || q_heads % kv_heads != 0 ||
        head_dim < 2 || head_dim % 2 != 0 || head_dim > 256 || kv_capacity < 1 || max_position < 1 ||
        blocksize != 64 || !(epsilon > 0.0F)) {
        h->set_error("sm100_rmsnorm_qkv_rope_nf4_bf16 requires hidden%64==0, q_heads%kv_heads==0, even head_dim, "
                     "positive capacity/max_position/epsilon, blocksize=64");
        return 1;
    }
    kc::QkvRopeArgs a;
    memset(&a, 0, sizeof(a));
    a.x = P<const void>(input);
    a.norm_w = P<const void>(norm_weight);
    a.eps = epsilon;
    a.q = GemvMat{P<const uint8_t>(qw), P<const float>(qa), static_cast<int>(q_heads * head_dim)};
    a.k = GemvMat{P<const uint8_t>(kw), P<const float>(ka), static_cast<int>(kv_heads * head_dim)};
    a.v = GemvMat{P<const uint8_t>(vw), P<const float>(va), static_cast<int>(kv_heads * head_dim)};
    a.qb = P<const void>(qb);
    a.kb = P<const void>(kb);
    a.vb = P<const void>(vb);
    a.rope_cos = P<const uint16_t>(rope_cos);
    a.rope_sin = P<const uint16_t>(rope_sin);
    a.max_pos = static_cast<int>(max_position);
    a.pos_dev = P<const int32_t>(position_device);
    a.q_out = P<void>(q_output);
    a.key_cache = P<void>(key_cache);
    a.value_cache = P<void>(value_cache);
    a.q_heads = static_cast<int>(q_heads);
    a.kv_heads = static_cast<int>(kv_heads);
    a.head_dim = static_cast<int>(head_dim);
    a.kv_cap = static_cast<int>(kv_capacity);
    a.K = static_cast<int>(hidden);
    a.err = h->err_word;
    return finish(h, "nf4_qkv_rope_kernel", kc::nf4_qkv_rope_hf_bf16(a, S(stream)));
}

int kudacuda_sm100_swiglu_nf4_bf16(void* raw, uint64_t input, uint64_t norm_weight, uint64_t gw, uint64_t ga,
                                   uint64_t uw, uint64_t ua, uint64_t output, int64_t hidden, int64_t inter,
                                   int64_t blocksize, float epsilon, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_swiglu_nf4_bf16")) return 1;
    if (input == 0 || norm_weight == 0 || gw == 0 || ga == 0 || uw == 0 || ua == 0 || output == 0) {
        h->set_error("sm100_swiglu_nf4_bf16 requires non-null device pointers");
        return 1;
    }
    if (hidden < 64 || hidden % 64 != 0 || hidden > 16384 || inter < 1 || inter > (1 << 26) || blocksize != 64 ||
        !(epsilon > 0.0F)) {
        h->set_error("sm100_swiglu_nf4_bf16 requires hidden%64==0 (<=16384), intermediate>=1, blocksize=64, positive epsilon");
        return 1;
    }
    return finish(h, "nf4_swiglu_hf_kernel",
                  kc::nf4_swiglu_hf_bf16(P<const void>(input), P<const void>(norm_weight), epsilon,
                                         GemvMat{P<const uint8_t>(gw), P<const float>(ga), static_cast<int>(inter)},
                                         GemvMat{P<const uint8_t>(uw), P<const float>(ua), static_cast<int>(inter)},
                                         P<void>(output), static_cast<int>(hidden), h->err_word, S(stream)));
}

int64_t kudacuda_sm100_gqa_workspace_bytes(int64_t batch_size, int64_t query_heads, int64_t kv_heads,
                                           int64_t kv_extent, int64_t head_dim) {
    if (batch_size < 1 || batch_size > kc::kMaxGqaBatch || query_heads < 1 || query_heads > kc::kMaxGqaHeads || kv_heads < 1 ||
        kv_heads > query_heads || kv_extent < 1 || kv_extent > (1 << 20) || head_dim < 1 || head_dim > 1024)
        return -1;
    int chunk = 0, nsplit = 0;
    kc::gqa_plan_splits(static_cast<int>(kv_extent), static_cast<int>(batch_size), static_cast<int>(kv_heads), 0,
                        &chunk, &nsplit);
    return static_cast<int64_t>(kc::gqa_partials_floats(static_cast<int>(batch_size), static_cast<int>(query_heads),
                                                        nsplit, static_cast<int>(head_dim)) * sizeof(float));
}

int kudacuda_sm100_gqa_decode(void* raw, uint64_t query, uint64_t key_cache, uint64_t value_cache, uint64_t output,
                              uint64_t workspace, int64_t workspace_bytes, uint64_t tickets, uint64_t kv_len_device,
                              int dtype, int64_t batch_size, int64_t kv_len, int64_t kv_stride, int64_t query_heads,
                              int64_t kv_heads, int64_t head_dim, float scale, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_gqa_decode")) return 1;
    if (query == 0 || key_cache == 0 || value_cache == 0 || output == 0 || workspace == 0 || tickets == 0) {
        h->set_error("sm100_gqa_decode requires non-null device pointers (kv_len_device may be null)");
        return 1;
    }
    const int64_t group = kv_heads > 0 ? query_heads / kv_heads : 0;
    if (batch_size < 1 || batch_size > kc::kMaxGqaBatch || kv_heads < 1 || query_heads > kc::kMaxGqaHeads ||
        query_heads % kv_heads != 0 ||
        !(group == 1 || group == 2 || group == 4 || group == 8) || head_dim != 128 || kv_stride < 1 ||
        kv_stride > (1 << 20) || (kv_len_device == 0 && (kv_len < 1 || kv_len > kv_stride)) || !(scale > 0.0F) ||
        (dtype != kc::kF16 && dtype != kc::kBF16)) {
        h->set_error("sm100_gqa_decode requires head_dim=128, query_heads/kv_heads in {1,2,4,8}, 1<=kv_len<=kv_stride, "
                     "positive scale, dtype f16 or bf16, batch_size<=65536, query_heads<=1024");
        return 1;
    }
    kc::GqaArgs a;
    memset(&a, 0, sizeof(a));
    a.q = P<const void>(query);
    a.kcache = P<const void>(key_cache);
    a.vcache = P<const void>(value_cache);
    a.out = P<void>(output);
    a.partials = P<float>(workspace);
    a.counters = P<int>(tickets);
    a.kv_len_dev = P<const int32_t>(kv_len_device);
    a.kv_len = static_cast<int>(kv_len_device != 0 ? kv_stride : kv_len);
    a.stride = static_cast<int>(kv_stride);
    a.batch = static_cast<int>(batch_size);
    a.q_heads = static_cast<int>(query_heads);
    a.kv_heads = static_cast<int>(kv_heads);
    a.head_dim = 128;
    a.scale = scale;
    a.err = h->err_word;
    const int extent = kv_len_device != 0 ? static_cast<int>(kv_stride) : static_cast<int>(kv_len);
    kc::gqa_plan_splits(extent, a.batch, a.kv_heads, 0, &a.chunk, &a.nsplit);
    const size_t need = kc::gqa_partials_floats(a.batch, a.q_heads, a.nsplit, 128) * sizeof(float);
    if (workspace_bytes < static_cast<int64_t>(need)) {
        h->set_error("sm100_gqa_decode workspace is smaller than kudacuda_sm100_gqa_workspace_bytes()");
        return 1;
    }
    return finish(h, "gqa_split_kernel", kc::gqa_decode(a, dtype, S(stream)));
}

int kudacuda_sm100_gqa_decode_static(void* raw, uint64_t query, uint64_t key_cache, uint64_t value_cache,
                                     uint64_t output, uint64_t kv_len_device, int dtype, int64_t batch_size,
                                     int64_t kv_len, int64_t kv_stride, int64_t query_heads, int64_t kv_heads,
                                     int64_t head_dim, float scale, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_gqa_decode_static")) return 1;
    if (query == 0 || key_cache == 0 || value_cache == 0 || output == 0) {
        h->set_error("sm100_gqa_decode_static requires non-null device pointers (kv_len_device may be null)");
        return 1;
    }
    const int64_t group = kv_heads > 0 ? query_heads / kv_heads : 0;
    if (batch_size < 1 || batch_size > kc::kMaxGqaBatch || kv_heads < 1 || query_heads > kc::kMaxGqaHeads ||
        query_heads % kv_heads != 0 ||
        !(group == 1 || group == 2 || group == 4 || group == 8) || head_dim != 128 || kv_stride < 1 ||
        kv_stride > (1 << 20) || (kv_len_device == 0 && (kv_len < 1 || kv_len > kv_stride)) || !(scale > 0.0F) ||
        (dtype != kc::kF16 && dtype != kc::kBF16)) {
        h->set_error("sm100_gqa_decode_static requires head_dim=128, query_heads/kv_heads in {1,2,4,8}, "
                     "1<=kv_len<=kv_stride, positive scale, dtype f16 or bf16, batch_size<=65536, query_heads<=1024");
        return 1;
    }
    kc::GqaArgs a;
    memset(&a, 0, sizeof(a));
    a.q = P<const void>(query);
    a.kcache = P<const void>(key_cache);
    a.vcache = P<const void>(value_cache);
    a.out = P<void>(output);
    a.kv_len_dev = P<const int32_t>(kv_len_device);
    a.kv_len = static_cast<int>(kv_len_device != 0 ? kv_stride : kv_len);
    a.stride = static_cast<int>(kv_stride);
    a.batch = static_cast<int>(batch_size);
    a.q_heads = static_cast<int>(query_heads);
    a.kv_heads = static_cast<int>(kv_heads);
    a.head_dim = 128;
    a.scale = scale;
    a.err = h->err_word;
    if (!kc::gqa_static_fits(a.batch, a.q_heads, a.kv_heads, a.kv_len_dev != nullptr ? a.stride : a.kv_len)) {
        h->set_error("sm100_gqa_decode_static: partials or tickets exceed the fixed scratch (1 MiB of partials, "
                     "1024 tickets); use kudacuda_sm100_gqa_decode with a caller workspace");
        return 1;
    }
    return finish(h, "gqa_split_kernel (static scratch)", kc::gqa_decode_static_scratch(a, dtype, S(stream)));
}

int kudacuda_sm100_rmsnorm_nf4_gemv(void* raw, uint64_t input, uint64_t norm_weight, uint64_t weight_packed,
                                    uint64_t absmax, uint64_t output, int output_dtype, int64_t rows, int64_t hidden,
                                    float epsilon, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_rmsnorm_nf4_gemv")) return 1;
    if (input == 0 || norm_weight == 0 || weight_packed == 0 || absmax == 0 || output == 0) {
        h->set_error("sm100_rmsnorm_nf4_gemv requires non-null device pointers");
        return 1;
    }
    if (rows < 1 || rows > (1 << 30) || hidden < 64 || hidden % 64 != 0 || hidden > 32768 || !(epsilon > 0.0F) ||
        (output_dtype != kc::kF32 && output_dtype != kc::kBF16)) {
        h->set_error("sm100_rmsnorm_nf4_gemv requires positive rows, hidden a multiple of 64 (<= 32768), "
                     "positive epsilon and an f32 or bf16 output");
        return 1;
    }
    return finish(h, "nf4_gemv (rmsnorm input)",
                  kc::nf4_rmsnorm_gemv_bf16(P<const void>(input), P<const void>(norm_weight), epsilon,
                                            GemvMat{P<const uint8_t>(weight_packed), P<const float>(absmax),
                                                    static_cast<int>(rows)},
                                            P<void>(output), output_dtype, static_cast<int>(hidden), h->err_word,
                                            S(stream)));
}

int kudacuda_sm100_residual_add_f32(void* raw, uint64_t partial_sum, uint64_t residual, int64_t n, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_residual_add_f32")) return 1;
    if (partial_sum == 0 || residual == 0 || n < 1 || n > (1 << 30)) {
        h->set_error("sm100_residual_add_f32 requires non-null pointers and a positive length");
        return 1;
    }
    return finish(h, "residual_add_f32_kernel",
                  kc::residual_add_f32_bf16(P<const float>(partial_sum), P<void>(residual), static_cast<int>(n),
                                            S(stream)));
}

int64_t kudacuda_sm100_argmax_workspace_bytes(void) {
    return static_cast<int64_t>(kc::argmax_shard_workspace_floats()) * static_cast<int64_t>(sizeof(float));
}

int kudacuda_sm100_argmax_shard_f32(void* raw, uint64_t logits, int64_t n, int64_t index_base, uint64_t workspace,
                                    int64_t workspace_bytes, uint64_t ticket, uint64_t out_pair, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_argmax_shard_f32")) return 1;
    if (logits == 0 || workspace == 0 || ticket == 0 || out_pair == 0 || n < 1 || n > (1 << 30) || index_base < 0 ||
        index_base > (1 << 30)) {
        h->set_error("sm100_argmax_shard_f32 requires non-null pointers, 1 <= n and a non-negative index base");
        return 1;
    }
    if (workspace_bytes < kudacuda_sm100_argmax_workspace_bytes()) {
        h->set_error("sm100_argmax_shard_f32 workspace is smaller than kudacuda_sm100_argmax_workspace_bytes()");
        return 1;
    }
    return finish(h, "argmax_shard_kernel",
                  kc::argmax_shard_f32(P<const float>(logits), static_cast<int>(n), static_cast<int>(index_base),
                                       P<float>(workspace), P<int>(ticket), P<kc::ArgPair>(out_pair), S(stream)));
}

int kudacuda_sm100_select_token(void* raw, uint64_t pairs, int64_t count, uint64_t next_token, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_select_token")) return 1;
    if (pairs == 0 || next_token == 0 || count < 1 || count > 4096) {
        h->set_error("sm100_select_token requires non-null pointers and 1 <= count <= 4096");
        return 1;
    }
    return finish(h, "select_token_kernel",
                  kc::select_token(P<const kc::ArgPair>(pairs), static_cast<int>(count), P<int32_t>(next_token),
                                   S(stream)));
}

int64_t kudacuda_sm100_lm_head_workspace_bytes(void) {
    return static_cast<int64_t>(kc::lm_head_grid()) * 2 * static_cast<int64_t>(sizeof(float));
}

int kudacuda_sm100_lm_head_argmax_bf16(void* raw, uint64_t hidden_state, uint64_t final_norm, uint64_t embedding,
                                       uint64_t logits, uint64_t token_out, uint64_t workspace, int64_t workspace_bytes,
                                       uint64_t ticket, int64_t vocab, int64_t hidden, float epsilon, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_lm_head_argmax_bf16")) return 1;
    if (hidden_state == 0 || final_norm == 0 || embedding == 0 || token_out == 0 || workspace == 0 || ticket == 0) {
        h->set_error("sm100_lm_head_argmax_bf16 requires non-null device pointers (logits may be null)");
        return 1;
    }
    if (vocab < 1 || vocab > (1 << 30) || hidden < 8 || hidden % 8 != 0 || hidden > 8192 || !(epsilon > 0.0F) ||
        (embedding & 15u) != 0) {
        h->set_error("sm100_lm_head_argmax_bf16 requires vocab>=1, hidden%8==0 (<=8192), positive epsilon, aligned embedding");
        return 1;
    }
    if (workspace_bytes < kudacuda_sm100_lm_head_workspace_bytes()) {
        h->set_error("sm100_lm_head_argmax_bf16 workspace is smaller than kudacuda_sm100_lm_head_workspace_bytes()");
        return 1;
    }
    kc::LmHeadArgs a;
    memset(&a, 0, sizeof(a));
    a.hidden = P<const void>(hidden_state);
    a.final_norm = P<const void>(final_norm);
    a.emb = P<const void>(embedding);
    a.logits = P<void>(logits);
    a.token_out = P<int32_t>(token_out);
    a.partials = P<float>(workspace);
    a.counter = P<int>(ticket);
    a.vocab = static_cast<int>(vocab);
    a.H = static_cast<int>(hidden);
    a.eps = epsilon;
    a.err = h->err_word;
    return finish(h, "lm_head_argmax_kernel", kc::lm_head_argmax_bf16(a, S(stream)));
}

int kudacuda_sm100_embedding_bf16(void* raw, uint64_t embedding, uint64_t token_device, uint64_t output, int64_t vocab,
                                  int64_t hidden, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_embedding_bf16")) return 1;
    if (embedding == 0 || token_device == 0 || output == 0) {
        h->set_error("sm100_embedding_bf16 requires non-null device pointers");
        return 1;
    }
    if (vocab < 1 || vocab > (1 << 30) || hidden < 1 || hidden > (1 << 20)) {
        h->set_error("sm100_embedding_bf16 requires positive vocab and hidden");
        return 1;
    }
    return finish(h, "embedding_gather_kernel",
                  kc::embedding_gather_bf16(P<const void>(embedding), P<const int32_t>(token_device), P<void>(output),
                                            static_cast<int>(hidden), static_cast<int>(vocab), h->err_word, S(stream)));
}

int kudacuda_sm100_decode_advance(void* raw, uint64_t step_state, uint64_t next_token, uint64_t history,
                                  int64_t history_len, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_decode_advance")) return 1;
    if (step_state == 0 || next_token == 0 || (history != 0 && history_len < 1)) {
        h->set_error("sm100_decode_advance requires step_state, next_token and a sized history");
        return 1;
    }
    return finish(h, "decode_advance_kernel",
                  kc::decode_advance(P<int32_t>(step_state), P<const int32_t>(next_token), P<int32_t>(history),
                                     static_cast<int>(history != 0 ? history_len : 0), S(stream)));
}

int kudacuda_sm100_graph_step_host(void* raw, const void* host_in, uint64_t device_in, int64_t in_bytes,
                                   void* host_out, uint64_t device_out, int64_t out_bytes, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (h == nullptr) return 1;
    if (h->graph_exec == nullptr) {
        h->set_error("kudacuda_sm100_graph_step_host called before graph instantiation");
        return 1;
    }
    if (in_bytes < 0 || out_bytes < 0 || (in_bytes > 0 && (host_in == nullptr || device_in == 0)) ||
        (out_bytes > 0 && (host_out == nullptr || device_out == 0))) {
        h->set_error("kudacuda_sm100_graph_step_host requires buffers for positive sizes");
        return 1;
    }
    cudaStream_t s = S(stream);
    cudaError_t st = cudaSuccess;
    if (in_bytes > 0) st = cudaMemcpyAsync(P<void>(device_in), host_in, static_cast<size_t>(in_bytes), cudaMemcpyHostToDevice, s);
    if (st != cudaSuccess) return finish(h, "cudaMemcpyAsync(H2D)", st);
    st = cudaGraphLaunch(h->graph_exec, s);
    if (st != cudaSuccess) return finish(h, "cudaGraphLaunch", st);
    if (out_bytes > 0) st = cudaMemcpyAsync(host_out, P<const void>(device_out), static_cast<size_t>(out_bytes), cudaMemcpyDeviceToHost, s);
    if (st != cudaSuccess) return finish(h, "cudaMemcpyAsync(D2H)", st);
    return finish(h, "cudaStreamSynchronize", cudaStreamSynchronize(s));
}

int kudacuda_sm100_error_word(void* raw, int* out_word, int clear) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_error_word")) return 1;
    if (out_word == nullptr) {
        h->set_error("sm100_error_word requires an output pointer");
        return 1;
    }
    cudaError_t st = cudaSetDevice(h->device_id);
    if (st == cudaSuccess) st = cudaMemcpy(out_word, h->err_word, sizeof(int), cudaMemcpyDeviceToHost);
    if (st == cudaSuccess && clear) st = cudaMemset(h->err_word, 0, sizeof(int));
    if (st == cudaSuccess && clear) st = cudaDeviceSynchronize();
    return finish(h, "sm100_error_word", st);
}

// ---------------------------------------------------------------- persistent decode of all layers
int64_t kudacuda_sm100_nf4_retile_groups(int mode, int64_t rows0, int64_t rows1, int64_t rows2, int64_t head_dim) {
    if (rows0 < 0 || rows1 < 0 || rows2 < 0 || rows0 > (1 << 24) || rows1 > (1 << 24) || rows2 > (1 << 24) ||
        head_dim < 0 || head_dim > 1024)
        return -1;
    return kc::retile_groups(mode, static_cast<int>(rows0), static_cast<int>(rows1), static_cast<int>(rows2),
                             static_cast<int>(head_dim));
}

int kudacuda_sm100_nf4_retile(void* raw, int mode, uint64_t packed0, uint64_t absmax0, int64_t rows0,
                              uint64_t packed1, uint64_t absmax1, int64_t rows1, uint64_t packed2, uint64_t absmax2,
                              int64_t rows2, int64_t k, int64_t head_dim, uint64_t out_codes, uint64_t out_absmax,
                              uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_nf4_retile")) return 1;
    const int64_t groups = kudacuda_sm100_nf4_retile_groups(mode, rows0, rows1, rows2, head_dim);
    const bool need1 = mode != kc::kRetilePlain, need2 = mode == kc::kRetileQkvRope;
    if (groups < 1 || k < 64 || k % 64 != 0 || k > (1 << 20) || packed0 == 0 || absmax0 == 0 || out_codes == 0 ||
        out_absmax == 0 || (need1 && (packed1 == 0 || absmax1 == 0)) || (need2 && (packed2 == 0 || absmax2 == 0))) {
        h->set_error("sm100_nf4_retile requires mode 0 (plain, rows % 64 == 0), 1 (SwiGLU, gate rows == up rows, "
                     "% 32 == 0) or 2 (q/k/v, head_dim % 64 == 0), K % 64 == 0 and non-null pointers");
        return 1;
    }
    const uint8_t* packed[3] = {P<const uint8_t>(packed0), P<const uint8_t>(packed1), P<const uint8_t>(packed2)};
    const float* absmax[3] = {P<const float>(absmax0), P<const float>(absmax1), P<const float>(absmax2)};
    const int rows[3] = {static_cast<int>(rows0), static_cast<int>(rows1), static_cast<int>(rows2)};
    return finish(h, "nf4_retile_kernel",
                  kc::nf4_retile(mode, packed, absmax, rows, static_cast<int>(k), static_cast<int>(head_dim),
                                 P<uint8_t>(out_codes), P<float>(out_absmax), S(stream)));
}

namespace {
bool persist_dims(int64_t layers, int64_t hidden, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                  int64_t intermediate, int64_t kv_capacity, kc::PersistDims& d) {
    const int64_t v[7] = {layers, hidden, q_heads, kv_heads, head_dim, intermediate, kv_capacity};
    for (int64_t x : v)
        if (x < 1 || x > (1 << 20)) return false;
    d.layers = static_cast<int>(layers);
    d.hidden = static_cast<int>(hidden);
    d.q_heads = static_cast<int>(q_heads);
    d.kv_heads = static_cast<int>(kv_heads);
    d.head_dim = static_cast<int>(head_dim);
    d.intermediate = static_cast<int>(intermediate);
    d.kv_capacity = static_cast<int>(kv_capacity);
    return true;
}
}  // namespace

int64_t kudacuda_sm100_decode_persistent_scratch_bytes(void* raw, int64_t layers, int64_t hidden, int64_t q_heads,
                                                      int64_t kv_heads, int64_t head_dim, int64_t intermediate,
                                                      int64_t kv_capacity) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_decode_persistent_scratch_bytes")) return -1;
    kc::PersistDims d;
    if (!persist_dims(layers, hidden, q_heads, kv_heads, head_dim, intermediate, kv_capacity, d)) return -1;
    const int sms = kc::device_sm_count();
    if (const char* why = kc::decode_persistent_check(d, sms)) {
        h->set_error(why);
        return -1;
    }
    return kc::decode_persistent_scratch_bytes(d, sms);
}

int kudacuda_sm100_decode_layers_persistent(void* raw, uint64_t layer_table, int64_t layers, uint64_t x,
                                            uint64_t state, uint64_t rope_cos, uint64_t rope_sin, int64_t max_pos,
                                            uint64_t scratch,
                                            int64_t scratch_bytes, int64_t hidden, int64_t q_heads, int64_t kv_heads,
                                            int64_t head_dim, int64_t intermediate, int64_t kv_capacity, float eps,
                                            float scale, uint64_t stream) {
    return kudacuda_sm100_decode_layers_persistent_debug(raw, layer_table, layers, x, state, rope_cos, rope_sin,
                                                         max_pos, scratch, scratch_bytes, hidden, q_heads, kv_heads,
                                                         head_dim, intermediate, kv_capacity, eps, scale, 0, 0, 0, -1,
                                                         stream);
}

int64_t kudacuda_sm100_decode_persistent_tap_elements(int64_t layers, int64_t hidden, int64_t q_heads,
                                                      int64_t kv_heads, int64_t head_dim, int64_t intermediate) {
    kc::PersistDims d;
    if (!persist_dims(layers, hidden, q_heads, kv_heads, head_dim, intermediate, 1, d)) return -1;
    return layers * kc::decode_persistent_tap_stride(d);
}

int kudacuda_sm100_decode_layers_persistent_debug(void* raw, uint64_t layer_table, int64_t layers, uint64_t x,
                                                  uint64_t state, uint64_t rope_cos, uint64_t rope_sin,
                                                  int64_t max_pos, uint64_t scratch, int64_t scratch_bytes,
                                                  int64_t hidden, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                                  int64_t intermediate, int64_t kv_capacity, float eps, float scale,
                                                  uint64_t taps, int64_t taps_bytes, int64_t spin_limit,
                                                  int64_t stall_counter, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_decode_layers_persistent")) return 1;
    kc::PersistDims d;
    if (!persist_dims(layers, hidden, q_heads, kv_heads, head_dim, intermediate, kv_capacity, d) || max_pos < 1 ||
        max_pos > (1 << 24) || !(eps > 0.0F) || !(scale > 0.0F)) {
        h->set_error("sm100_decode_layers_persistent requires positive shapes, max_pos, eps and scale");
        return 1;
    }
    if (layer_table == 0 || x == 0 || state == 0 || rope_cos == 0 || rope_sin == 0 || scratch == 0) {
        h->set_error("sm100_decode_layers_persistent requires non-null device pointers");
        return 1;
    }
    const int sms = kc::device_sm_count();
    if (const char* why = kc::decode_persistent_check(d, sms)) {
        h->set_error(why);
        return 1;
    }
    if (scratch_bytes < kc::decode_persistent_scratch_bytes(d, sms)) {
        h->set_error("sm100_decode_layers_persistent scratch is smaller than "
                     "kudacuda_sm100_decode_persistent_scratch_bytes()");
        return 1;
    }
    kc::PersistLaunch p;
    p.layer_table = P<const uint64_t>(layer_table);
    p.dims = d;
    p.max_pos = static_cast<int>(max_pos);
    p.eps = eps;
    p.scale = scale;
    p.state = P<const int32_t>(state);
    p.x = P<uint16_t>(x);
    p.rope_cos = P<const uint16_t>(rope_cos);
    p.rope_sin = P<const uint16_t>(rope_sin);
    p.scratch = P<void>(scratch);
    p.err = h->err_word;
    if (taps != 0 && taps_bytes < 2 * layers * kc::decode_persistent_tap_stride(d)) {
        h->set_error("sm100_decode_layers_persistent_debug: taps buffer is smaller than "
                     "2 * kudacuda_sm100_decode_persistent_tap_elements() bytes");
        return 1;
    }
    if (spin_limit < 0 || spin_limit > (int64_t{1} << 30) || stall_counter < -1 ||
        stall_counter >= static_cast<int64_t>(layers) * 8) {
        h->set_error("sm100_decode_layers_persistent_debug: spin_limit must be 0..2^30 (0: default) and "
                     "stall_counter -1 or a counter index below layers * 8");
        return 1;
    }
    p.taps = P<uint16_t>(taps);
    p.spin_limit = static_cast<uint32_t>(spin_limit);
    p.stall_counter = static_cast<int>(stall_counter);
    return finish(h, "decode_layers_kernel", kc::decode_layers_persistent(p, S(stream)));
}

// ---------------------------------------------------------------- row-split persistent decode
int64_t kudacuda_sm100_nf4_retile16_tiles(int mode, int64_t rows0, int64_t rows1, int64_t rows2, int64_t head_dim) {
    if (rows0 < 0 || rows1 < 0 || rows2 < 0 || head_dim < 0 || rows0 > (1 << 24) || rows1 > (1 << 24) ||
        rows2 > (1 << 24) || head_dim > 4096)
        return -1;
    return kc::retile16_tiles(mode, static_cast<int>(rows0), static_cast<int>(rows1), static_cast<int>(rows2),
                              static_cast<int>(head_dim));
}

int kudacuda_sm100_nf4_retile16(void* raw, int mode, uint64_t packed0, uint64_t absmax0, int64_t rows0,
                                uint64_t packed1, uint64_t absmax1, int64_t rows1, uint64_t packed2, uint64_t absmax2,
                                int64_t rows2, int64_t k, int64_t head_dim, uint64_t out_units, int64_t out_bytes,
                                uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_nf4_retile16")) return 1;
    const int64_t tiles = kudacuda_sm100_nf4_retile16_tiles(mode, rows0, rows1, rows2, head_dim);
    const bool need1 = mode != kc::kRetilePlain, need2 = mode == kc::kRetileQkvRope;
    if (tiles < 1 || k < 64 || k % 64 != 0 || k > (1 << 20) || packed0 == 0 || absmax0 == 0 || out_units == 0 ||
        (need1 && (packed1 == 0 || absmax1 == 0)) || (need2 && (packed2 == 0 || absmax2 == 0))) {
        h->set_error("sm100_nf4_retile16 requires mode 0 (plain, rows % 16 == 0), 1 (SwiGLU, gate rows == up rows, "
                     "% 8 == 0) or 2 (q/k/v, head_dim % 16 == 0), K % 64 == 0 and non-null pointers");
        return 1;
    }
    if (out_bytes < tiles * (k / 64) * 576) {
        h->set_error("sm100_nf4_retile16: output is smaller than tiles * (k / 64) * 576 bytes");
        return 1;
    }
    const uint8_t* packed[3] = {P<const uint8_t>(packed0), P<const uint8_t>(packed1), P<const uint8_t>(packed2)};
    const float* absmax[3] = {P<const float>(absmax0), P<const float>(absmax1), P<const float>(absmax2)};
    const int rows[3] = {static_cast<int>(rows0), static_cast<int>(rows1), static_cast<int>(rows2)};
    return finish(h, "nf4_retile16_kernel",
                  kc::nf4_retile16(mode, packed, absmax, rows, static_cast<int>(k), static_cast<int>(head_dim),
                                   P<uint8_t>(out_units), S(stream)));
}

int64_t kudacuda_sm100_decode_rows_scratch_bytes(void* raw, int64_t layers, int64_t hidden, int64_t q_heads,
                                                int64_t kv_heads, int64_t head_dim, int64_t intermediate,
                                                int64_t kv_capacity) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_decode_rows_scratch_bytes")) return -1;
    kc::PersistDims d;
    if (!persist_dims(layers, hidden, q_heads, kv_heads, head_dim, intermediate, kv_capacity, d)) return -1;
    const int sms = kc::device_sm_count();
    if (const char* why = kc::decode_rows_check(d, sms)) {
        h->set_error(why);
        return -1;
    }
    return kc::decode_rows_scratch_bytes(d, sms);
}

namespace {
int decode_rows_common(void* raw, uint64_t layer_table, int64_t layers, uint64_t x, uint64_t state, uint64_t rope_cos,
                       uint64_t rope_sin, int64_t max_pos, uint64_t scratch, int64_t scratch_bytes, int64_t hidden,
                       int64_t q_heads, int64_t kv_heads, int64_t head_dim, int64_t intermediate,
                       int64_t kv_capacity, float eps, float scale, uint64_t taps, int64_t taps_bytes,
                       int64_t spin_limit, int64_t stall_counter, int64_t world, int64_t rank, uint64_t tp_peers,
                       uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, world == 1 ? "kudacuda_sm100_decode_layers_rows" : "kudacuda_sm100_decode_layers_rows_tp")) return 1;
    if (world < 1 || world > 8 || rank < 0 || rank >= world || (world > 1 && tp_peers == 0)) {
        h->set_error("sm100_decode_layers_rows_tp requires 1 <= world <= 8, 0 <= rank < world and the peer table");
        return 1;
    }
    kc::PersistDims d;
    if (!persist_dims(layers, hidden, q_heads, kv_heads, head_dim, intermediate, kv_capacity, d) || max_pos < 1 ||
        max_pos > (1 << 24) || !(eps > 0.0F) || !(scale > 0.0F)) {
        h->set_error("sm100_decode_layers_rows requires positive shapes, max_pos, eps and scale");
        return 1;
    }
    if (layer_table == 0 || x == 0 || state == 0 || rope_cos == 0 || rope_sin == 0 || scratch == 0) {
        h->set_error("sm100_decode_layers_rows requires non-null device pointers");
        return 1;
    }
    const int sms = kc::device_sm_count();
    if (const char* why = kc::decode_rows_check(d, sms)) {
        h->set_error(why);
        return 1;
    }
    if (scratch_bytes < kc::decode_rows_scratch_bytes(d, sms)) {
        h->set_error("sm100_decode_layers_rows scratch is smaller than kudacuda_sm100_decode_rows_scratch_bytes()");
        return 1;
    }
    if (taps != 0 && taps_bytes < 2 * layers * kc::decode_rows_tap_stride(d)) {
        h->set_error("sm100_decode_layers_rows: taps buffer is smaller than 2 * kudacuda_sm100_decode_persistent_tap_elements() bytes");
        return 1;
    }
    if (spin_limit < 0 || spin_limit > (int64_t{1} << 30) || stall_counter < -1 || stall_counter >= layers * 16) {
        h->set_error("sm100_decode_layers_rows: spin_limit must be 0..2^30 (0: default) and stall_counter -1 or a "
                     "counter index below layers * 16");
        return 1;
    }
    kc::PersistLaunch p;
    p.layer_table = P<const uint64_t>(layer_table);
    p.dims = d;
    p.max_pos = static_cast<int>(max_pos);
    p.eps = eps;
    p.scale = scale;
    p.state = P<const int32_t>(state);
    p.x = P<uint16_t>(x);
    p.rope_cos = P<const uint16_t>(rope_cos);
    p.rope_sin = P<const uint16_t>(rope_sin);
    p.scratch = P<void>(scratch);
    p.err = h->err_word;
    p.taps = P<uint16_t>(taps);
    p.spin_limit = static_cast<uint32_t>(spin_limit);
    p.stall_counter = static_cast<int>(stall_counter);
    p.world = static_cast<int>(world);
    p.rank = static_cast<int>(rank);
    p.tp_peers = P<const uint64_t>(tp_peers);
    return finish(h, "decode_rows_kernel", kc::decode_layers_rows(p, S(stream)));
}
}  // namespace

int kudacuda_sm100_decode_layers_rows(void* raw, uint64_t layer_table, int64_t layers, uint64_t x, uint64_t state,
                                      uint64_t rope_cos, uint64_t rope_sin, int64_t max_pos, uint64_t scratch,
                                      int64_t scratch_bytes, int64_t hidden, int64_t q_heads, int64_t kv_heads,
                                      int64_t head_dim, int64_t intermediate, int64_t kv_capacity, float eps,
                                      float scale, uint64_t taps, int64_t taps_bytes, int64_t spin_limit,
                                      int64_t stall_counter, uint64_t stream) {
    return decode_rows_common(raw, layer_table, layers, x, state, rope_cos, rope_sin, max_pos, scratch, scratch_bytes,
                              hidden, q_heads, kv_heads, head_dim, intermediate, kv_capacity, eps, scale, taps,
                              taps_bytes, spin_limit, stall_counter, 1, 0, 0, stream);
}

int kudacuda_sm100_decode_layers_rows_tp(void* raw, uint64_t layer_table, int64_t layers, uint64_t x, uint64_t state,
                                         uint64_t rope_cos, uint64_t rope_sin, int64_t max_pos, uint64_t scratch,
                                         int64_t scratch_bytes, int64_t hidden, int64_t q_heads, int64_t kv_heads,
                                         int64_t head_dim, int64_t intermediate, int64_t kv_capacity, float eps,
                                         float scale, int64_t world, int64_t rank, uint64_t tp_peers,
                                         uint64_t stream) {
    return decode_rows_common(raw, layer_table, layers, x, state, rope_cos, rope_sin, max_pos, scratch, scratch_bytes,
                              hidden, q_heads, kv_heads, head_dim, intermediate, kv_capacity, eps, scale, 0, 0, 0, -1,
                              world, rank, tp_peers, stream);
}

int64_t kudacuda_sm100_tp_exchange_bytes(int64_t world, int64_t hidden) {
    if (world < 1 || world > 8 || hidden < 16 || hidden > (1 << 16)) return -1;
    return 2 * world * hidden * 8;
}

// Exchange buffers live in their own cudaMalloc allocations so that a CUDA IPC
// handle maps exactly the buffer into the peer processes.
int kudacuda_sm100_ipc_alloc(void* raw, int64_t bytes, uint64_t* out_ptr, void* out_handle, int64_t handle_bytes) {
    Handle* h = as_handle(raw);
    if (h == nullptr || out_ptr == nullptr || out_handle == nullptr || bytes < 1 || bytes > (int64_t{1} << 32) ||
        handle_bytes < static_cast<int64_t>(sizeof(cudaIpcMemHandle_t))) {
        if (h != nullptr) h->set_error("sm100_ipc_alloc requires 1 <= bytes <= 4 GiB and a 64-byte handle buffer");
        return 1;
    }
    void* p = nullptr;
    cudaError_t st = cudaSetDevice(h->device_id);
    if (st == cudaSuccess) st = cudaMalloc(&p, static_cast<size_t>(bytes));
    if (st == cudaSuccess) st = cudaMemset(p, 0, static_cast<size_t>(bytes));
    cudaIpcMemHandle_t ih;
    if (st == cudaSuccess) st = cudaIpcGetMemHandle(&ih, p);
    if (st != cudaSuccess) {
        if (p != nullptr) cudaFree(p);
        h->set_error(std::string("sm100_ipc_alloc: ") + cudaGetErrorString(st));
        return 1;
    }
    std::memcpy(out_handle, &ih, sizeof(ih));
    *out_ptr = reinterpret_cast<uint64_t>(p);
    h->last_error.clear();
    return 0;
}

int kudacuda_sm100_ipc_open(void* raw, const void* ipc_handle, int64_t handle_bytes, uint64_t* out_ptr) {
    Handle* h = as_handle(raw);
    if (h == nullptr || ipc_handle == nullptr || out_ptr == nullptr ||
        handle_bytes < static_cast<int64_t>(sizeof(cudaIpcMemHandle_t))) {
        if (h != nullptr) h->set_error("sm100_ipc_open requires a 64-byte handle and an output pointer");
        return 1;
    }
    cudaIpcMemHandle_t ih;
    std::memcpy(&ih, ipc_handle, sizeof(ih));
    void* p = nullptr;
    cudaError_t st = cudaSetDevice(h->device_id);
    if (st == cudaSuccess) st = cudaIpcOpenMemHandle(&p, ih, cudaIpcMemLazyEnablePeerAccess);
    if (st != cudaSuccess) {
        h->set_error(std::string("sm100_ipc_open: ") + cudaGetErrorString(st));
        return 1;
    }
    *out_ptr = reinterpret_cast<uint64_t>(p);
    h->last_error.clear();
    return 0;
}

int kudacuda_sm100_ipc_close(void* raw, uint64_t ptr, int owned) {
    Handle* h = as_handle(raw);
    if (h == nullptr || ptr == 0) return 1;
    cudaError_t st = cudaSetDevice(h->device_id);
    if (st == cudaSuccess)
        st = owned != 0 ? cudaFree(reinterpret_cast<void*>(ptr)) : cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr));
    if (st != cudaSuccess) {
        h->set_error(std::string("sm100_ipc_close: ") + cudaGetErrorString(st));
        return 1;
    }
    h->last_error.clear();
    return 0;
}

// ---------------------------------------------------------------- batched decode
namespace {
bool npad_ok(int64_t n_pad) { return n_pad == 16 || n_pad == 32 || n_pad == 64; }
}  // namespace

int64_t kudacuda_sm100_batch_gemm_ksplit(int64_t rows, int64_t k) {
    if (rows < 1 || k < 64 || k % 64 != 0 || rows > (1 << 24) || k > (1 << 20)) return -1;
    return kc::batch_gemm_ksplit(static_cast<int>(rows), static_cast<int>(k));
}

int kudacuda_sm100_batch_gemm(void* raw, int weight_type, uint64_t weight, uint64_t absmax, int64_t rows, int64_t k,
                              uint64_t x, int64_t n_pad, int64_t ksplit, uint64_t partials, int64_t row_offset,
                              int64_t total_rows, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_batch_gemm")) return 1;
    if (weight == 0 || x == 0 || partials == 0 || (weight_type == 0 && absmax == 0) || weight_type < 0 ||
        weight_type > 2 || rows < 1 || rows > (1 << 24) || k < 64 || k % 64 != 0 ||
        k > (1 << 20) || !npad_ok(n_pad) || ksplit < 1 || ksplit > k / 64 || row_offset < 0 ||
        total_rows > (1 << 24) || row_offset + rows > total_rows) {
        h->set_error("sm100_batch_gemm requires weight_type 0 (NF4 + absmax), 1 (bf16) or 2 (re-tiled NF4), K % 64 == 0, n_pad in "
                     "{16, 32, 64}, 1 <= ksplit <= K/64, row_offset + rows <= total_rows, non-null pointers");
        return 1;
    }
    return finish(h, "nf4_gemm_tc_kernel",
                  kc::batch_gemm(weight_type, P<const void>(weight), P<const float>(absmax), static_cast<int>(rows),
                                 static_cast<int>(k), P<const uint16_t>(x), static_cast<int>(n_pad),
                                 static_cast<int>(ksplit), P<float>(partials), static_cast<int>(row_offset),
                                 static_cast<int>(total_rows), h->err_word, S(stream)));
}

int64_t kudacuda_sm100_batch_retile_bytes(int64_t rows, int64_t k) {
    if (rows < 1 || k < 64 || k % 64 != 0 || rows > (1 << 24) || k > (1 << 20)) return -1;
    return kc::batch_retile_bytes(static_cast<int>(rows), static_cast<int>(k));
}

int kudacuda_sm100_batch_retile(void* raw, uint64_t packed, uint64_t absmax, int64_t rows, int64_t k, uint64_t out,
                                int64_t out_bytes, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_batch_retile")) return 1;
    const int64_t need = kudacuda_sm100_batch_retile_bytes(rows, k);
    if (packed == 0 || absmax == 0 || out == 0 || need < 0 || out_bytes < need) {
        h->set_error("sm100_batch_retile requires non-null pointers, K % 64 == 0 and out_bytes >= "
                     "kudacuda_sm100_batch_retile_bytes(rows, k)");
        return 1;
    }
    return finish(h, "batch_retile_kernel",
                  kc::batch_retile(P<const uint8_t>(packed), P<const float>(absmax), static_cast<int>(rows),
                                   static_cast<int>(k), P<uint8_t>(out), S(stream)));
}

namespace {
// shared checks of the fused-epilogue GEMM entries
bool fused_gemm_ok(Handle* h, const char* op, int weight_type, uint64_t weight, uint64_t absmax, int64_t rows,
                   int64_t k, uint64_t x, int64_t n_pad, int64_t ksplit, int64_t batch, uint64_t partials,
                   int64_t partials_bytes, uint64_t tickets) {
    if (weight == 0 || x == 0 || partials == 0 || tickets == 0 || (weight_type != 0 && weight_type != 2) ||
        (weight_type == 0 && absmax == 0) || rows < 1 || rows > (1 << 24) || k < 64 || k % 64 != 0 ||
        k > (1 << 20) || !npad_ok(n_pad) || ksplit < 1 || ksplit > k / 64 || batch < 1 || batch > n_pad ||
        partials_bytes < ksplit * rows * n_pad * 4) {
        std::string m(op);
        m += " requires NF4 weights (weight_type 0 with absmax, or 2 re-tiled), K % 64 == 0, n_pad in {16, 32, 64}, "
             "1 <= batch <= n_pad, 1 <= ksplit <= K/64, partials of ksplit * rows * n_pad floats, tickets";
        h->set_error(m.c_str());
        return false;
    }
    return true;
}
kc::BatchEpilogue fused_epi(int mode, int64_t batch, uint64_t tickets) {
    kc::BatchEpilogue e;
    memset(&e, 0, sizeof(e));
    e.mode = mode;
    e.batch = static_cast<int>(batch);
    e.tickets = P<int>(tickets);
    return e;
}
}  // namespace

int kudacuda_sm100_batch_gemm_residual(void* raw, int weight_type, uint64_t weight, uint64_t absmax, int64_t rows,
                                       int64_t k, uint64_t x, int64_t n_pad, int64_t ksplit, int64_t batch,
                                       uint64_t partials, int64_t partials_bytes, uint64_t tickets, uint64_t resid,
                                       uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_batch_gemm_residual")) return 1;
    if (!fused_gemm_ok(h, "sm100_batch_gemm_residual", weight_type, weight, absmax, rows, k, x, n_pad, ksplit, batch,
                       partials, partials_bytes, tickets))
        return 1;
    if (resid == 0) {
        h->set_error("sm100_batch_gemm_residual requires the residual stream [batch][rows] bf16");
        return 1;
    }
    kc::BatchEpilogue e = fused_epi(1, batch, tickets);
    e.resid = P<uint16_t>(resid);
    return finish(h, "gemm_tc_kernel (residual)",
                  kc::batch_gemm(weight_type, P<const void>(weight), P<const float>(absmax), static_cast<int>(rows),
                                 static_cast<int>(k), P<const uint16_t>(x), static_cast<int>(n_pad),
                                 static_cast<int>(ksplit), P<float>(partials), 0, static_cast<int>(rows), h->err_word,
                                 S(stream), &e));
}

int kudacuda_sm100_batch_gemm_swiglu(void* raw, int weight_type, uint64_t weight, uint64_t absmax,
                                     int64_t intermediate, int64_t k, uint64_t x, int64_t n_pad, int64_t ksplit,
                                     int64_t batch, uint64_t partials, int64_t partials_bytes, uint64_t tickets,
                                     uint64_t out, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_batch_gemm_swiglu")) return 1;
    if (!fused_gemm_ok(h, "sm100_batch_gemm_swiglu", weight_type, weight, absmax, 2 * intermediate, k, x, n_pad,
                       ksplit, batch, partials, partials_bytes, tickets))
        return 1;
    if (out == 0 || intermediate % 64 != 0) {
        h->set_error("sm100_batch_gemm_swiglu requires intermediate % 64 == 0 (weights in 64-row gate | up tiles) "
                     "and the output [batch][intermediate] bf16");
        return 1;
    }
    kc::BatchEpilogue e = fused_epi(2, batch, tickets);
    e.hout = P<uint16_t>(out);
    return finish(h, "gemm_tc_kernel (swiglu)",
                  kc::batch_gemm(weight_type, P<const void>(weight), P<const float>(absmax),
                                 static_cast<int>(2 * intermediate), static_cast<int>(k), P<const uint16_t>(x),
                                 static_cast<int>(n_pad), static_cast<int>(ksplit), P<float>(partials), 0,
                                 static_cast<int>(2 * intermediate), h->err_word, S(stream), &e));
}

int kudacuda_sm100_batch_gemm_qkv_rope(void* raw, int weight_type, uint64_t weight, uint64_t absmax, int64_t k,
                                       uint64_t x, int64_t n_pad, int64_t ksplit, int64_t batch, uint64_t partials,
                                       int64_t partials_bytes, uint64_t tickets, int64_t q_heads, int64_t kv_heads,
                                       int64_t head_dim, uint64_t q_bias, uint64_t k_bias, uint64_t v_bias,
                                       uint64_t rope_cos, uint64_t rope_sin, int64_t max_pos, uint64_t pos,
                                       uint64_t q_out, uint64_t key_cache, uint64_t value_cache, int64_t kv_capacity,
                                       int shared_cache, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_batch_gemm_qkv_rope")) return 1;
    const int64_t rows = (q_heads + 2 * kv_heads) * 128;
    if (head_dim != 128 || q_heads < 1 || kv_heads < 1 || q_heads > 256 || kv_heads > 256) {
        h->set_error("sm100_batch_gemm_qkv_rope requires head_dim 128 (one tile per head)");
        return 1;
    }
    if (!fused_gemm_ok(h, "sm100_batch_gemm_qkv_rope", weight_type, weight, absmax, rows, k, x, n_pad, ksplit, batch,
                       partials, partials_bytes, tickets))
        return 1;
    if (rope_cos == 0 || rope_sin == 0 || pos == 0 || q_out == 0 || key_cache == 0 || value_cache == 0 ||
        max_pos < 1 || kv_capacity < 1) {
        h->set_error("sm100_batch_gemm_qkv_rope requires rope tables, positions, q output and caches");
        return 1;
    }
    kc::BatchEpilogue e = fused_epi(3, batch, tickets);
    e.q_heads = static_cast<int>(q_heads);
    e.kv_heads = static_cast<int>(kv_heads);
    e.cap = static_cast<int>(kv_capacity);
    e.max_pos = static_cast<int>(max_pos);
    e.shared_cache = shared_cache != 0 ? 1 : 0;
    e.q_bias = P<const uint16_t>(q_bias);
    e.k_bias = P<const uint16_t>(k_bias);
    e.v_bias = P<const uint16_t>(v_bias);
    e.rope_cos = P<const uint16_t>(rope_cos);
    e.rope_sin = P<const uint16_t>(rope_sin);
    e.pos = P<const int32_t>(pos);
    e.q_out = P<uint16_t>(q_out);
    e.kcache = P<uint16_t>(key_cache);
    e.vcache = P<uint16_t>(value_cache);
    return finish(h, "gemm_tc_kernel (q/k/v + RoPE)",
                  kc::batch_gemm(weight_type, P<const void>(weight), P<const float>(absmax), static_cast<int>(rows),
                                 static_cast<int>(k), P<const uint16_t>(x), static_cast<int>(n_pad),
                                 static_cast<int>(ksplit), P<float>(partials), 0, static_cast<int>(rows), h->err_word,
                                 S(stream), &e));
}

int kudacuda_sm100_batch_rmsnorm(void* raw, uint64_t x, uint64_t weight, uint64_t out, int64_t batch, int64_t hidden,
                                 float eps, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_batch_rmsnorm")) return 1;
    if (x == 0 || weight == 0 || out == 0 || batch < 1 || batch > 64 || hidden < 8 || hidden % 8 != 0 ||
        hidden > 8192 || !(eps > 0.0F)) {
        h->set_error("sm100_batch_rmsnorm requires non-null pointers, 1 <= batch <= 64, hidden % 8 == 0, "
                     "hidden <= 8192, eps > 0");
        return 1;
    }
    return finish(h, "batch_rmsnorm_kernel",
                  kc::batch_rmsnorm(P<const uint16_t>(x), P<const uint16_t>(weight), P<uint16_t>(out),
                                    static_cast<int>(batch), static_cast<int>(hidden), eps, S(stream)));
}

int kudacuda_sm100_batch_qkv_rope(void* raw, uint64_t partials, int64_t ksplit, int64_t n_pad, int64_t batch,
                                  int64_t q_heads, int64_t kv_heads, int64_t head_dim, uint64_t q_bias, uint64_t k_bias,
                                  uint64_t v_bias, uint64_t rope_cos, uint64_t rope_sin, int64_t max_pos, uint64_t pos,
                                  uint64_t q_out, uint64_t key_cache, uint64_t value_cache, int64_t kv_capacity,
                                  int shared_cache, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_batch_qkv_rope")) return 1;
    if (partials == 0 || rope_cos == 0 || rope_sin == 0 || pos == 0 || q_out == 0 || key_cache == 0 ||
        value_cache == 0 || ksplit < 1 || ksplit > 64 || !npad_ok(n_pad) || batch < 1 || batch > n_pad ||
        q_heads < 1 || kv_heads < 1 || head_dim < 2 || head_dim % 2 != 0 || head_dim > 512 || max_pos < 1 ||
        kv_capacity < 1) {
        h->set_error("sm100_batch_qkv_rope requires non-null pointers (biases may be null), 1 <= batch <= n_pad, "
                     "n_pad in {16, 32, 64}, even head_dim");
        return 1;
    }
    kc::BatchQkv q;
    memset(&q, 0, sizeof(q));
    q.partials = P<const float>(partials);
    q.ksplit = static_cast<int>(ksplit);
    q.n_pad = static_cast<int>(n_pad);
    q.batch = static_cast<int>(batch);
    q.q_heads = static_cast<int>(q_heads);
    q.kv_heads = static_cast<int>(kv_heads);
    q.head_dim = static_cast<int>(head_dim);
    q.cap = static_cast<int>(kv_capacity);
    q.max_pos = static_cast<int>(max_pos);
    q.q_bias = P<const uint16_t>(q_bias);
    q.k_bias = P<const uint16_t>(k_bias);
    q.v_bias = P<const uint16_t>(v_bias);
    q.rope_cos = P<const uint16_t>(rope_cos);
    q.rope_sin = P<const uint16_t>(rope_sin);
    q.pos = P<const int32_t>(pos);
    q.q_out = P<uint16_t>(q_out);
    q.kcache = P<uint16_t>(key_cache);
    q.vcache = P<uint16_t>(value_cache);
    q.shared_cache = shared_cache != 0 ? 1 : 0;
    q.err = h->err_word;
    return finish(h, "batch_qkv_epilogue_kernel", kc::batch_qkv_epilogue(q, S(stream)));
}

int kudacuda_sm100_batch_residual(void* raw, uint64_t partials, int64_t ksplit, int64_t rows, int64_t n_pad,
                                  int64_t batch, uint64_t x, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_batch_residual")) return 1;
    if (partials == 0 || x == 0 || ksplit < 1 || ksplit > 64 || rows < 1 || rows > (1 << 24) || !npad_ok(n_pad) ||
        batch < 1 || batch > n_pad) {
        h->set_error("sm100_batch_residual requires non-null pointers, 1 <= batch <= n_pad, n_pad in {16, 32, 64}");
        return 1;
    }
    return finish(h, "batch_residual_kernel",
                  kc::batch_residual(P<const float>(partials), static_cast<int>(ksplit), static_cast<int>(rows),
                                     static_cast<int>(n_pad), static_cast<int>(batch), P<uint16_t>(x), S(stream)));
}

int kudacuda_sm100_batch_swiglu(void* raw, uint64_t partials, int64_t ksplit, int64_t intermediate, int64_t n_pad,
                                int64_t batch, uint64_t out, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_batch_swiglu")) return 1;
    if (partials == 0 || out == 0 || ksplit < 1 || ksplit > 64 || intermediate < 1 || intermediate > (1 << 23) ||
        !npad_ok(n_pad) || batch < 1 || batch > n_pad) {
        h->set_error("sm100_batch_swiglu requires non-null pointers, 1 <= batch <= n_pad, n_pad in {16, 32, 64}");
        return 1;
    }
    return finish(h, "batch_swiglu_kernel",
                  kc::batch_swiglu(P<const float>(partials), static_cast<int>(ksplit), static_cast<int>(intermediate),
                                   static_cast<int>(n_pad), static_cast<int>(batch), P<uint16_t>(out), S(stream)));
}

int64_t kudacuda_sm100_batch_argmax_workspace_bytes(int64_t batch) {
    if (batch < 1 || batch > 64) return -1;
    return static_cast<int64_t>(kc::batch_argmax_workspace_floats(static_cast<int>(batch))) * 4;
}

int kudacuda_sm100_batch_argmax_advance(void* raw, uint64_t partials, int64_t ksplit, int64_t vocab, int64_t n_pad,
                                        int64_t batch, uint64_t workspace, int64_t workspace_bytes, uint64_t state,
                                        uint64_t history, int64_t history_len, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_batch_argmax_advance")) return 1;
    if (partials == 0 || workspace == 0 || state == 0 || ksplit < 1 || ksplit > 64 || vocab < 1 ||
        vocab > (1 << 24) || !npad_ok(n_pad) || batch < 1 || batch > n_pad || history_len < 0 ||
        history_len > (1 << 24) || (history != 0 && history_len < 1)) {
        h->set_error("sm100_batch_argmax_advance requires non-null pointers (history may be null), "
                     "1 <= batch <= n_pad, n_pad in {16, 32, 64}");
        return 1;
    }
    if (workspace_bytes < kudacuda_sm100_batch_argmax_workspace_bytes(batch)) {
        h->set_error("sm100_batch_argmax_advance workspace is smaller than kudacuda_sm100_batch_argmax_workspace_bytes()");
        return 1;
    }
    return finish(h, "batch_argmax_stage1/2",
                  kc::batch_argmax_advance(P<const float>(partials), static_cast<int>(ksplit), static_cast<int>(vocab),
                                           static_cast<int>(n_pad), static_cast<int>(batch), P<float>(workspace),
                                           P<int32_t>(state), P<int32_t>(history), static_cast<int>(history_len),
                                           S(stream)));
}

int kudacuda_sm100_batch_split_sum(void* raw, uint64_t partials, int64_t ksplit, int64_t rows, int64_t n_pad,
                                   uint64_t out, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_batch_split_sum")) return 1;
    if (partials == 0 || out == 0 || ksplit < 1 || ksplit > 64 || rows < 1 || rows > (1 << 24) || !npad_ok(n_pad)) {
        h->set_error("sm100_batch_split_sum requires non-null pointers, 1 <= ksplit <= 64, n_pad in {16, 32, 64}");
        return 1;
    }
    return finish(h, "batch_split_sum_kernel",
                  kc::batch_split_sum(P<const float>(partials), static_cast<int>(ksplit), static_cast<int>(rows),
                                      static_cast<int>(n_pad), P<float>(out), S(stream)));
}

int kudacuda_sm100_batch_argmax_pairs(void* raw, uint64_t partials, int64_t ksplit, int64_t vocab, int64_t n_pad,
                                      int64_t batch, uint64_t workspace, int64_t workspace_bytes, int64_t index_base,
                                      uint64_t pairs, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_batch_argmax_pairs")) return 1;
    if (partials == 0 || workspace == 0 || pairs == 0 || ksplit < 1 || ksplit > 64 || vocab < 1 ||
        vocab > (1 << 24) || !npad_ok(n_pad) || batch < 1 || batch > n_pad || index_base < 0 ||
        index_base + vocab > (int64_t{1} << 30)) {
        h->set_error("sm100_batch_argmax_pairs requires non-null pointers, 1 <= batch <= n_pad, n_pad in {16, 32, 64}");
        return 1;
    }
    if (workspace_bytes < kudacuda_sm100_batch_argmax_workspace_bytes(batch)) {
        h->set_error("sm100_batch_argmax_pairs workspace is smaller than kudacuda_sm100_batch_argmax_workspace_bytes()");
        return 1;
    }
    return finish(h, "batch_argmax_stage1/pairs",
                  kc::batch_argmax_pairs(P<const float>(partials), static_cast<int>(ksplit), static_cast<int>(vocab),
                                         static_cast<int>(n_pad), static_cast<int>(batch), P<float>(workspace),
                                         static_cast<int>(index_base), P<int32_t>(pairs), S(stream)));
}

int kudacuda_sm100_batch_select_advance(void* raw, uint64_t gathered, int64_t world, int64_t batch, uint64_t state,
                                        uint64_t history, int64_t history_len, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_batch_select_advance")) return 1;
    if (gathered == 0 || state == 0 || world < 1 || world > 1024 || batch < 1 || batch > 64 || history_len < 0 ||
        history_len > (1 << 24) || (history != 0 && history_len < 1)) {
        h->set_error("sm100_batch_select_advance requires non-null pointers (history may be null), 1 <= batch <= 64");
        return 1;
    }
    return finish(h, "batch_select_advance_kernel",
                  kc::batch_select_advance(P<const int32_t>(gathered), static_cast<int>(world), static_cast<int>(batch),
                                           P<int32_t>(state), P<int32_t>(history), static_cast<int>(history_len),
                                           S(stream)));
}

int kudacuda_sm100_batch_embedding(void* raw, uint64_t embedding, uint64_t state, uint64_t x, int64_t batch,
                                   int64_t hidden, int64_t vocab, uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_batch_embedding")) return 1;
    if (embedding == 0 || state == 0 || x == 0 || batch < 1 || batch > 64 || hidden < 8 || hidden % 8 != 0 ||
        hidden > (1 << 20) || vocab < 1 || vocab > (1 << 24)) {
        h->set_error("sm100_batch_embedding requires non-null pointers, 1 <= batch <= 64, hidden % 8 == 0");
        return 1;
    }
    return finish(h, "batch_embedding_kernel",
                  kc::batch_embedding(P<const uint16_t>(embedding), P<const int32_t>(state), P<uint16_t>(x),
                                      static_cast<int>(batch), static_cast<int>(hidden), static_cast<int>(vocab),
                                      h->err_word, S(stream)));
}

int kudacuda_sm100_batch_state_views(void* raw, uint64_t state, int64_t batch, uint64_t pos, uint64_t kv_len,
                                     uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_batch_state_views")) return 1;
    if (state == 0 || pos == 0 || kv_len == 0 || batch < 1 || batch > 64) {
        h->set_error("sm100_batch_state_views requires non-null pointers and 1 <= batch <= 64");
        return 1;
    }
    return finish(h, "batch_state_views_kernel",
                  kc::batch_state_views(P<const int32_t>(state), static_cast<int>(batch), P<int32_t>(pos),
                                        P<int32_t>(kv_len), S(stream)));
}

namespace {
// Split plan of the per-sequence-length attention: the split-KV kernel with
// many (sequence, KV head) pairs, the cluster kernel (its own plan) with few;
// both on the default split plan (64-token chunks measured slower: 35.9 vs
// 24.6 us per launch at batch 64 with 2048-token caches).
bool batch_gqa_split(int64_t batch, int64_t kv_heads) { return batch * kv_heads >= 64; }
void batch_gqa_plan(int64_t batch, int64_t kv_heads, int64_t stride, int* chunk, int* nsplit) {
    kc::gqa_plan_splits(static_cast<int>(stride), static_cast<int>(batch), static_cast<int>(kv_heads), 0, chunk,
                        nsplit);
    // With 128 or more (sequence, kv head) pairs, 128-token chunks balance the
    // split-KV grid better (B200: batch 64 x 2 kv heads 3.6% faster per step);
    // at 64 pairs the default chunking is faster (batch 32: 5%).
    if (batch * kv_heads >= 128 && *chunk > 128) {
        *chunk = 128;
        *nsplit = static_cast<int>((stride + 127) / 128);
    }
}
}  // namespace

int64_t kudacuda_sm100_gqa_batch_workspace_bytes(int64_t batch_size, int64_t query_heads, int64_t kv_heads,
                                                 int64_t kv_stride) {
    if (batch_size < 1 || batch_size > 4096 || query_heads < 1 || query_heads > kc::kMaxGqaHeads || kv_heads < 1 ||
        kv_heads > query_heads || kv_stride < 1 || kv_stride > (1 << 20))
        return -1;
    int chunk = 0, nsplit = 0;
    batch_gqa_plan(batch_size, kv_heads, kv_stride, &chunk, &nsplit);
    return static_cast<int64_t>(kc::gqa_partials_floats(static_cast<int>(batch_size), static_cast<int>(query_heads),
                                                        nsplit, 128) * sizeof(float));
}

int kudacuda_sm100_gqa_decode_batch(void* raw, uint64_t query, uint64_t key_cache, uint64_t value_cache,
                                    uint64_t output, uint64_t workspace, int64_t workspace_bytes, uint64_t tickets,
                                    uint64_t kv_len_array, int64_t batch_size, int64_t kv_stride, int64_t query_heads,
                                    int64_t kv_heads, int64_t head_dim, float scale, int shared_cache,
                                    uint64_t stream) {
    Handle* h = as_handle(raw);
    if (!ready(h, "kudacuda_sm100_gqa_decode_batch")) return 1;
    if (query == 0 || key_cache == 0 || value_cache == 0 || output == 0 || workspace == 0 || tickets == 0 ||
        kv_len_array == 0) {
        h->set_error("sm100_gqa_decode_batch requires non-null device pointers");
        return 1;
    }
    const int64_t group = kv_heads > 0 ? query_heads / kv_heads : 0;
    if (batch_size < 1 || batch_size > 4096 || kv_heads < 1 || query_heads > kc::kMaxGqaHeads ||
        query_heads % kv_heads != 0 ||
        !(group == 1 || group == 2 || group == 4 || group == 8) || head_dim != 128 || kv_stride < 1 ||
        kv_stride > (1 << 20) || !(scale > 0.0F)) {
        h->set_error("sm100_gqa_decode_batch requires head_dim=128, query_heads/kv_heads in {1,2,4,8}, positive scale");
        return 1;
    }
    kc::GqaArgs a;
    memset(&a, 0, sizeof(a));
    a.q = P<const void>(query);
    a.kcache = P<const void>(key_cache);
    a.vcache = P<const void>(value_cache);
    a.out = P<void>(output);
    a.partials = P<float>(workspace);
    a.counters = P<int>(tickets);
    a.kv_len_dev = P<const int32_t>(kv_len_array);
    a.kv_len_per_batch = 1;
    a.kv_shared = shared_cache != 0 ? 1 : 0;
    // many (sequence, KV head) pairs: the split-KV kernel, whose splits past a
    // sequence's length exit at once, where the cluster kernel's CTAs would all
    // take part in its barriers (batch 64, 2048-token caches, lengths 63-510:
    // 5.55 vs 6.35 ms per step); few pairs: the cluster kernel (batch 16:
    // 3.90 vs 4.08 ms per step)
    a.split_only = batch_gqa_split(batch_size, kv_heads) ? 1 : 0;
    a.kv_len = static_cast<int>(kv_stride);
    a.stride = static_cast<int>(kv_stride);
    a.batch = static_cast<int>(batch_size);
    a.q_heads = static_cast<int>(query_heads);
    a.kv_heads = static_cast<int>(kv_heads);
    a.head_dim = 128;
    a.scale = scale;
    a.err = h->err_word;
    batch_gqa_plan(batch_size, kv_heads, kv_stride, &a.chunk, &a.nsplit);
    const size_t need = kc::gqa_partials_floats(a.batch, a.q_heads, a.nsplit, 128) * sizeof(float);
    if (workspace_bytes < static_cast<int64_t>(need)) {
        h->set_error("sm100_gqa_decode_batch workspace is smaller than kudacuda_sm100_gqa_batch_workspace_bytes()");
        return 1;
    }
    return finish(h, "gqa decode (per-sequence lengths)", kc::gqa_decode(a, kc::kBF16, S(stream)));
}

const char* kudacuda_sm100_target_arch(void) { return "sm_100a"; }

}  // extern "C"
