// Launcher of the fused rotary + KV append kernel (rope_append.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b200_paged_attn.h"

namespace b200 {

int launch_rope_append(const b200_cache_desc* c, const b200_rope_append_args* a, const void* query,
                       const void* key, const void* value, const void* cos, const void* sin,
                       const void* slots, void* query_out, uint32_t* error_word,
                       cudaStream_t stream);

}  // namespace b200
