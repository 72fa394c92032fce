// Launchers of the metadata builder and validation kernels (metadata.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

int launch_build_slot_mapping(const void* block_tables, int32_t table_dtype, int64_t table_stride,
                              int32_t table_width, const void* starts, const void* ends,
                              int32_t index_dtype, int32_t num_seqs, int32_t block_size,
                              int32_t num_blocks, void* slots_out, int32_t slots_dtype,
                              int64_t total_tokens, int32_t* cu_seqlens_out, uint32_t* error_word,
                              cudaStream_t stream);

int launch_validate_decode_metadata(const void* block_tables, int32_t table_dtype,
                                    int64_t table_stride, int32_t table_width,
                                    const void* context_lens, int32_t lens_dtype, int32_t num_seqs,
                                    int32_t block_size, int32_t num_blocks, int32_t* flags_out,
                                    cudaStream_t stream);

}  // namespace b200
