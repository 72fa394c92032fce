// Launcher of the KV append kernel (append.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b200_paged_attn.h"

namespace b200 {

int launch_append_kv(const b200_cache_desc* c, int32_t layer, const void* key, const void* value,
                     int64_t num_tokens, int64_t key_stride_token, int64_t key_stride_head,
                     int64_t value_stride_token, int64_t value_stride_head, const void* slots,
                     int32_t slots_dtype, uint32_t* error_word, cudaStream_t stream);

}  // namespace b200
