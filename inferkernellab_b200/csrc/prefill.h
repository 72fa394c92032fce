// Launcher of the paged prefill kernel (prefill.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b200_paged_attn.h"

namespace b200 {

int launch_paged_prefill(const b200_cache_desc* c, const b200_prefill_args* a, const void* query,
                         const void* block_tables, const void* query_starts,
                         const void* context_lens, const int32_t* cu_seqlens_q, void* out,
                         uint32_t* error_word, cudaStream_t stream);

}  // namespace b200
