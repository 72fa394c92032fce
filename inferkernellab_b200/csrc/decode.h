// Launchers of the paged decode kernel (decode.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include "../../include/b200_paged_attn.h"

namespace b200 {

size_t decode_workspace_bytes(const b200_cache_desc* c, const b200_decode_args* a);

int launch_paged_decode(const b200_cache_desc* c, const b200_decode_args* a, const void* query,
                        const void* block_tables, const void* context_lens, void* out,
                        void* workspace, size_t workspace_bytes, cudaStream_t stream);

// Decode with the new token's K/V append (and rotary embedding) fused in.
int launch_paged_decode_append(const b200_cache_desc* c, const b200_decode_args* a,
                               const b200_decode_append_args* fa, const void* query,
                               const void* key, const void* value, const void* cos,
                               const void* sin, const void* slots, const void* block_tables,
                               const void* context_lens, void* out, void* workspace,
                               size_t workspace_bytes, cudaStream_t stream);

// Allocation-free variant: split scratch from a static device array (decode.cu).
size_t decode_noalloc_scratch_bytes();
int decode_noalloc_error_word(uint32_t** out);
int launch_paged_decode_noalloc(const b200_cache_desc* c, const b200_decode_args* a,
                                const void* query, const void* block_tables,
                                const void* context_lens, void* out, cudaStream_t stream);

}  // namespace b200
