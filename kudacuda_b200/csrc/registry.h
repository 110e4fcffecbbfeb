// registry.h -- internal view of the built-in tactic table.
#pragma once

#include <cstdint>

namespace kc {

struct TacticEntry {
    const char* name;
    const char* symbol;  // C-ABI entry point that serves the tactic
    int64_t max_batch;   // 0 = any
    int64_t seq_len;     // 0 = any
};

const TacticEntry* find_tactic(const char* name);
int tactic_count();
const TacticEntry* tactic_at(int i);

}  // namespace kc
