/*
 * kudacuda_registry.h -- tactic registry of the B200 KudaCuda library.
 *
 * Same class and descriptor as the reference (include/kudacuda_registry.h:10-41
 * of lijeuki/KudaCuda): a Driver-API module loader that maps name -> cubin
 * path and module::symbol -> CUfunction, and can be frozen against further
 * loads.  Differences: the driver functions are resolved at run time through
 * cudaGetDriverEntryPoint, so the library has no link-time dependency on
 * libcuda; and the built-in tactic table behind kudacuda_can_dispatch is
 * queryable through the C functions at the end of this header.
 */
#pragma once

#include <cuda.h>
#include <stdint.h>

#ifdef __cplusplus
#include <string>
#include <unordered_map>

namespace kudacuda {

struct KudaCudaKernelDescriptor {
    const char* name;
    const char* symbol;
    unsigned int grid_x;
    unsigned int grid_y;
    unsigned int grid_z;
    unsigned int block_x;
    unsigned int block_y;
    unsigned int block_z;
    unsigned int shared_memory_bytes;
};

class __attribute__((visibility("default"))) KudaCudaModuleRegistry {
public:
    explicit KudaCudaModuleRegistry(int device_id);
    ~KudaCudaModuleRegistry();

    KudaCudaModuleRegistry(const KudaCudaModuleRegistry&) = delete;
    KudaCudaModuleRegistry& operator=(const KudaCudaModuleRegistry&) = delete;

    int load(const std::string& name, const std::string& path, std::string* error);
    int resolve(const std::string& module_name, const std::string& symbol, CUfunction* function, std::string* error);
    int freeze(std::string* error);
    bool frozen() const { return frozen_; }

private:
    CUcontext context_ = nullptr;
    int device_id_ = 0;
    bool frozen_ = false;
    std::unordered_map<std::string, CUmodule> modules_;
    std::unordered_map<std::string, CUfunction> functions_;
};

}  // namespace kudacuda

extern "C" {
#endif

/* Number of entries in the built-in tactic table. */
__attribute__((visibility("default"))) int kudacuda_tactic_count(void);

/* Entry i of the table: name, the C-ABI symbol that serves it, the largest
 * accepted batch (0 = any) and the required seq_len (0 = any).  Returns 0 on
 * success, 1 when i is out of range. */
__attribute__((visibility("default"))) int kudacuda_tactic_info(int index, const char** name, const char** symbol,
                                                                int64_t* max_batch, int64_t* seq_len);

#ifdef __cplusplus
}
#endif
