// registry.cu -- tactic table and Driver-API module registry.
//
// The reference hard-codes its tactic names inside kudacuda_can_dispatch
// (runtime/kudacuda_runtime.cu:298-327) and ships a module registry that
// nothing calls (runtime/kudacuda_registry.cu:33-115).  Here the table is data:
// kudacuda_can_dispatch, kudacuda_tactic_info and the manifest
// (kudacuda_b200/manifests/b200-sm100.json) all read it.  The reference's
// sm86/sm89 tactic names are kept as aliases so a bridge configured with the
// reference manifests dispatches onto the sm_100a kernels unchanged.
#include "../../include/kudacuda_registry.h"
#include "registry.h"

#include <cuda_runtime.h>

#include <cstring>

namespace kc {
namespace {

const TacticEntry kTactics[] = {
    // reference tactics (runtime/kudacuda_runtime.cu:311-326), served on sm_100a
    {"vector_add", "kudacuda_vector_add", 0, 0},
    {"rmsnorm", "kudacuda_rmsnorm", 0, 0},
    {"qwen2_gqa_decode_sm86_fp16", "kudacuda_qwen2_gqa_decode", 1, 1},
    {"qwen2_gqa_decode_sm89_fp16", "kudacuda_qwen2_gqa_decode", 1, 1},
    {"qwen2_gqa_decode_sm86_fp16_group_tiled_v2", "kudacuda_qwen2_gqa_decode_group_tiled", 1, 1},
    {"qwen2_gqa_decode_sm89_fp16_group_tiled_v2", "kudacuda_qwen2_gqa_decode_group_tiled", 1, 1},
    {"qwen2_gqa_decode_sm86_fp16_vectorized_v2", "kudacuda_qwen2_gqa_decode_vectorized", 1, 1},
    {"qwen2_gqa_decode_sm89_fp16_vectorized_v2", "kudacuda_qwen2_gqa_decode_vectorized", 1, 1},
    {"qwen2_gqa_decode_sm86_fp16_graph_v1", "kudacuda_qwen2_gqa_decode_graph", 1, 1},
    {"qwen2_gqa_decode_sm89_fp16_graph_v1", "kudacuda_qwen2_gqa_decode_graph", 1, 1},
    // the same tactics under sm100 names (manifests/b200-sm100.json)
    {"qwen2_gqa_decode_sm100_fp16", "kudacuda_qwen2_gqa_decode", 1, 1},
    {"qwen2_gqa_decode_sm100_fp16_group_tiled_v2", "kudacuda_qwen2_gqa_decode_group_tiled", 1, 1},
    {"qwen2_gqa_decode_sm100_fp16_vectorized_v2", "kudacuda_qwen2_gqa_decode_vectorized", 1, 1},
    {"qwen2_gqa_decode_sm100_fp16_graph_v1", "kudacuda_qwen2_gqa_decode_graph", 1, 1},
    {"qwen2_gqa_decode_sm100_fp16_workspace_v3", "kudacuda_qwen2_gqa_decode_workspace_v3", 1, 1},
    {"qwen2_fused_rmsnorm_qkv_sm100_nf4_v1", "kudacuda_qwen2_fused_rmsnorm_qkv_nf4", 1, 1},
    {"qwen2_fused_rmsnorm_qkv_sm100_nf4_v2", "kudacuda_qwen2_fused_rmsnorm_qkv_nf4_v2", 1, 1},
    {"qwen2_fused_rmsnorm_qkv_sm100_nf4_v3", "kudacuda_qwen2_fused_rmsnorm_qkv_nf4_v3", 1, 1},
    {"qwen2_swiglu_sm100_nf4_v1", "kudacuda_qwen2_swiglu_nf4", 1, 1},
    {"qwen2_swiglu_sm100_bf16_nf4_v1", "kudacuda_qwen2_swiglu_nf4_bf16", 1, 1},
    // sm100 additions
    {"nf4_gemv_sm100_v1", "kudacuda_sm100_nf4_gemv", 1, 1},
    {"nf4_linear_residual_sm100_bf16_v1", "kudacuda_sm100_nf4_linear_residual_bf16", 1, 1},
    {"nf4_dequantize_sm100_v1", "kudacuda_sm100_nf4_dequantize", 0, 0},
    {"qwen2_attention_input_sm100_bf16_nf4_v1", "kudacuda_sm100_rmsnorm_qkv_rope_nf4_bf16", 1, 1},
    {"qwen2_swiglu_sm100_bf16_nf4_hf_v1", "kudacuda_sm100_swiglu_nf4_bf16", 1, 1},
    {"qwen2_gqa_decode_sm100_bf16_splitkv_v1", "kudacuda_sm100_gqa_decode", 0, 1},
    {"lm_head_argmax_sm100_bf16_v1", "kudacuda_sm100_lm_head_argmax_bf16", 1, 1},
    {"qwen2_static_decode_graph_sm100_v1", "kudacuda_replay_graph", 1, 1},
    {"decode_advance_sm100_v1", "kudacuda_sm100_decode_advance", 1, 1},
};

constexpr int kTacticCount = static_cast<int>(sizeof(kTactics) / sizeof(kTactics[0]));

}  // namespace

const TacticEntry* find_tactic(const char* name) {
    if (name == nullptr) return nullptr;
    for (const TacticEntry& t : kTactics)
        if (std::strcmp(t.name, name) == 0) return &t;
    return nullptr;
}
int tactic_count() { return kTacticCount; }
const TacticEntry* tactic_at(int i) { return (i >= 0 && i < kTacticCount) ? &kTactics[i] : nullptr; }

}  // namespace kc

extern "C" int kudacuda_tactic_count(void) { return kc::tactic_count(); }

extern "C" int kudacuda_tactic_info(int index, const char** name, const char** symbol, int64_t* max_batch,
                                    int64_t* seq_len) {
    const kc::TacticEntry* t = kc::tactic_at(index);
    if (t == nullptr) return 1;
    if (name) *name = t->name;
    if (symbol) *symbol = t->symbol;
    if (max_batch) *max_batch = t->max_batch;
    if (seq_len) *seq_len = t->seq_len;
    return 0;
}

// ---------------------------------------------------------------------------
// KudaCudaModuleRegistry (runtime/kudacuda_registry.cu:33-115 of the
// reference): retain the device's primary context, load cubins by name,
// resolve module::symbol, refuse loads after freeze().

namespace kudacuda {
namespace {

using PFN_cuInit_t = CUresult (*)(unsigned int);
using PFN_cuDeviceGet_t = CUresult (*)(CUdevice*, int);
using PFN_cuDevicePrimaryCtxRetain_t = CUresult (*)(CUcontext*, CUdevice);
using PFN_cuDevicePrimaryCtxRelease_t = CUresult (*)(CUdevice);
using PFN_cuCtxSetCurrent_t = CUresult (*)(CUcontext);
using PFN_cuModuleLoad_t = CUresult (*)(CUmodule*, const char*);
using PFN_cuModuleUnload_t = CUresult (*)(CUmodule);
using PFN_cuModuleGetFunction_t = CUresult (*)(CUfunction*, CUmodule, const char*);

template <typename F>
bool driver_fn(const char* name, F* out) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess ||
        p == nullptr)
        return false;
    *out = reinterpret_cast<F>(p);
    return true;
}

std::string cu_message(const char* op, CUresult r) { return std::string(op) + " failed with CUresult " + std::to_string(static_cast<int>(r)); }

}  // namespace

KudaCudaModuleRegistry::KudaCudaModuleRegistry(int device_id) : device_id_(device_id) {
    PFN_cuInit_t cu_init = nullptr;
    PFN_cuDeviceGet_t cu_device_get = nullptr;
    PFN_cuDevicePrimaryCtxRetain_t retain = nullptr;
    if (!driver_fn("cuInit", &cu_init) || !driver_fn("cuDeviceGet", &cu_device_get) ||
        !driver_fn("cuDevicePrimaryCtxRetain", &retain))
        return;
    CUdevice dev = 0;
    if (cu_init(0) != CUDA_SUCCESS || cu_device_get(&dev, device_id) != CUDA_SUCCESS) return;
    CUcontext ctx = nullptr;
    if (retain(&ctx, dev) == CUDA_SUCCESS) context_ = ctx;
}

KudaCudaModuleRegistry::~KudaCudaModuleRegistry() {
    PFN_cuModuleUnload_t unload = nullptr;
    if (driver_fn("cuModuleUnload", &unload))
        for (auto& kv : modules_) unload(kv.second);
    PFN_cuDeviceGet_t cu_device_get = nullptr;
    PFN_cuDevicePrimaryCtxRelease_t release = nullptr;
    if (context_ != nullptr && driver_fn("cuDeviceGet", &cu_device_get) &&
        driver_fn("cuDevicePrimaryCtxRelease", &release)) {
        CUdevice dev = 0;
        if (cu_device_get(&dev, device_id_) == CUDA_SUCCESS) release(dev);
    }
}

int KudaCudaModuleRegistry::load(const std::string& name, const std::string& path, std::string* error) {
    if (frozen_) {
        if (error) *error = "module registry is frozen";
        return 1;
    }
    if (context_ == nullptr) {
        if (error) *error = "no CUDA primary context for device " + std::to_string(device_id_);
        return 1;
    }
    if (modules_.count(name) != 0) {
        if (error) *error = "module already loaded: " + name;
        return 1;
    }
    PFN_cuCtxSetCurrent_t set_current = nullptr;
    PFN_cuModuleLoad_t module_load = nullptr;
    if (!driver_fn("cuCtxSetCurrent", &set_current) || !driver_fn("cuModuleLoad", &module_load)) {
        if (error) *error = "CUDA driver entry points unavailable";
        return 1;
    }
    CUresult r = set_current(context_);
    CUmodule m = nullptr;
    if (r == CUDA_SUCCESS) r = module_load(&m, path.c_str());
    if (r != CUDA_SUCCESS) {
        if (error) *error = cu_message("cuModuleLoad", r);
        return 1;
    }
    modules_[name] = m;
    return 0;
}

int KudaCudaModuleRegistry::resolve(const std::string& module_name, const std::string& symbol, CUfunction* function,
                                    std::string* error) {
    if (function == nullptr) {
        if (error) *error = "null output function";
        return 1;
    }
    const std::string key = module_name + "::" + symbol;
    auto hit = functions_.find(key);
    if (hit != functions_.end()) {
        *function = hit->second;
        return 0;
    }
    auto mod = modules_.find(module_name);
    if (mod == modules_.end()) {
        if (error) *error = "unknown module: " + module_name;
        return 1;
    }
    PFN_cuModuleGetFunction_t get_fn = nullptr;
    if (!driver_fn("cuModuleGetFunction", &get_fn)) {
        if (error) *error = "CUDA driver entry points unavailable";
        return 1;
    }
    CUfunction f = nullptr;
    const CUresult r = get_fn(&f, mod->second, symbol.c_str());
    if (r != CUDA_SUCCESS) {
        if (error) *error = cu_message("cuModuleGetFunction", r);
        return 1;
    }
    functions_[key] = f;
    *function = f;
    return 0;
}

int KudaCudaModuleRegistry::freeze(std::string* error) {
    if (context_ == nullptr) {
        if (error) *error = "no CUDA primary context";
        return 1;
    }
    frozen_ = true;
    return 0;
}

}  // namespace kudacuda
