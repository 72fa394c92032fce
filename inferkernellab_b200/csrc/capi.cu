// extern "C" entry points of libb200_paged_attn.so (declared in
// include/b200_paged_attn.h).  Each one clears the thread's error message,
// forwards to its launcher and returns the launcher's status; nothing throws
// across this boundary.
#include <cuda_runtime.h>

#include <exception>

#include "../../include/b200_paged_attn.h"
#include "append.h"
#include "decode.h"
#include "host_common.h"
#include "layer_ops.h"
#include "metadata.h"
#include "prefill.h"
#include "rope_append.h"

namespace b200 {
const char* last_error_cstr();
int launch_tc_selftest(const void* a, const void* b, const void* v, float* c1, float* c2,
                       float* c3, int32_t dtype, uint32_t* err, cudaStream_t stream);
int launch_wait_selftest(int64_t limit_ns, int32_t arrive, uint32_t* result, uint32_t* err,
                         cudaStream_t stream);
}

namespace {
inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

template <typename F>
int guarded(F&& f) {
  b200::clear_error();
  try {
    return f();
  } catch (const std::exception& e) {
    return b200::set_error(B200_ERR_CUDA, std::string("internal error: ") + e.what());
  } catch (...) {
    return b200::set_error(B200_ERR_CUDA, "internal error");
  }
}
}  // namespace

extern "C" {

size_t b200_paged_decode_workspace_bytes(const b200_cache_desc* cache,
                                         const b200_decode_args* args) {
  try {
    return b200::decode_workspace_bytes(cache, args);
  } catch (...) {
    return 0;
  }
}

int b200_paged_decode(const b200_cache_desc* cache, const b200_decode_args* args, const void* query,
                      const void* block_tables, const void* context_lens, void* out,
                      void* workspace, size_t workspace_bytes, void* stream) {
  return guarded([&] {
    return b200::launch_paged_decode(cache, args, query, block_tables, context_lens, out,
                                     workspace, workspace_bytes, as_stream(stream));
  });
}

int b200_paged_decode_noalloc(const b200_cache_desc* cache, const b200_decode_args* args,
                              const void* query, const void* block_tables,
                              const void* context_lens, void* out, void* stream) {
  return guarded([&] {
    return b200::launch_paged_decode_noalloc(cache, args, query, block_tables, context_lens, out,
                                             as_stream(stream));
  });
}

size_t b200_paged_decode_noalloc_scratch_bytes(void) {
  return b200::decode_noalloc_scratch_bytes();
}

int b200_paged_decode_noalloc_error_word(uint32_t** error_word_out) {
  return guarded([&] { return b200::decode_noalloc_error_word(error_word_out); });
}

int b200_append_kv(const b200_cache_desc* cache, int32_t layer, const void* key, const void* value,
                   int64_t num_tokens, int64_t key_stride_token, int64_t key_stride_head,
                   int64_t value_stride_token, int64_t value_stride_head, const void* slots,
                   int32_t slots_dtype, uint32_t* error_word, void* stream) {
  return guarded([&] {
    return b200::launch_append_kv(cache, layer, key, value, num_tokens, key_stride_token,
                                  key_stride_head, value_stride_token, value_stride_head, slots,
                                  slots_dtype, error_word, as_stream(stream));
  });
}

int b200_paged_decode_append(const b200_cache_desc* cache, const b200_decode_args* args,
                             const b200_decode_append_args* append, const void* query,
                             const void* key, const void* value, const void* cos, const void* sin,
                             const void* slots, const void* block_tables, const void* context_lens,
                             void* out, void* workspace, size_t workspace_bytes, void* stream) {
  return guarded([&] {
    return b200::launch_paged_decode_append(cache, args, append, query, key, value, cos, sin,
                                            slots, block_tables, context_lens, out, workspace,
                                            workspace_bytes, as_stream(stream));
  });
}

int b200_rope_append_kv(const b200_cache_desc* cache, const b200_rope_append_args* args,
                        const void* query, const void* key, const void* value, const void* cos,
                        const void* sin, const void* slots, void* query_out,
                        uint32_t* error_word, void* stream) {
  return guarded([&] {
    return b200::launch_rope_append(cache, args, query, key, value, cos, sin, slots, query_out,
                                    error_word, as_stream(stream));
  });
}

int b200_tc_selftest(const void* a, const void* b, const void* v, float* c1, float* c2,
                     float* c3, int32_t dtype, uint32_t* error_word, void* stream) {
  return guarded([&] {
    return b200::launch_tc_selftest(a, b, v, c1, c2, c3, dtype, error_word, as_stream(stream));
  });
}

int b200_wait_selftest(int64_t limit_ns, int32_t arrive, uint32_t* result, uint32_t* error_word,
                       void* stream) {
  return guarded([&] {
    return b200::launch_wait_selftest(limit_ns, arrive, result, error_word, as_stream(stream));
  });
}

int b200_add_rmsnorm(const void* x, const void* residual, const void* weight, void* out,
                     void* residual_out, int64_t rows, int64_t cols, int64_t x_stride,
                     int64_t residual_stride, int64_t out_stride, int64_t residual_out_stride,
                     float eps, int32_t dtype, void* stream) {
  return guarded([&] {
    return b200::launch_add_rmsnorm(x, residual, weight, out, residual_out, rows, cols, x_stride,
                                    residual_stride, out_stride, residual_out_stride, eps, dtype,
                                    as_stream(stream));
  });
}

int b200_silu_mul(const void* gate_up, void* out, int64_t rows, int64_t cols, int64_t in_stride,
                  int64_t out_stride, int32_t dtype, void* stream) {
  return guarded([&] {
    return b200::launch_silu_mul(gate_up, out, rows, cols, in_stride, out_stride, dtype,
                                 as_stream(stream));
  });
}

int b200_paged_prefill(const b200_cache_desc* cache, const b200_prefill_args* args,
                       const void* query, const void* block_tables, const void* query_starts,
                       const void* context_lens, const int32_t* cu_seqlens_q, void* out,
                       uint32_t* error_word, void* stream) {
  return guarded([&] {
    return b200::launch_paged_prefill(cache, args, query, block_tables, query_starts,
                                      context_lens, cu_seqlens_q, out, error_word,
                                      as_stream(stream));
  });
}

int b200_build_slot_mapping(const void* block_tables, int32_t table_dtype, int64_t table_stride,
                            int32_t table_width, const void* starts, const void* ends,
                            int32_t index_dtype, int32_t num_seqs, int32_t block_size,
                            int32_t num_blocks, void* slots_out, int32_t slots_dtype,
                            int64_t total_tokens, int32_t* cu_seqlens_out, uint32_t* error_word,
                            void* stream) {
  return guarded([&] {
    return b200::launch_build_slot_mapping(block_tables, table_dtype, table_stride, table_width,
                                           starts, ends, index_dtype, num_seqs, block_size,
                                           num_blocks, slots_out, slots_dtype, total_tokens,
                                           cu_seqlens_out, error_word, as_stream(stream));
  });
}

int b200_validate_decode_metadata(const void* block_tables, int32_t table_dtype,
                                  int64_t table_stride, int32_t table_width,
                                  const void* context_lens, int32_t lens_dtype, int32_t num_seqs,
                                  int32_t block_size, int32_t num_blocks, int32_t* flags_out,
                                  void* stream) {
  return guarded([&] {
    return b200::launch_validate_decode_metadata(block_tables, table_dtype, table_stride,
                                                 table_width, context_lens, lens_dtype, num_seqs,
                                                 block_size, num_blocks, flags_out,
                                                 as_stream(stream));
  });
}

int b200_read_error_word(uint32_t* error_word, uint32_t* value, int32_t clear, void* stream) {
  return guarded([&] {
    if (error_word == nullptr || value == nullptr)
      return b200::set_error(B200_ERR_INVALID, "null pointer");
    cudaStream_t s = as_stream(stream);
    cudaError_t err = cudaMemcpyAsync(value, error_word, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
    if (err != cudaSuccess) return b200::cuda_status(err, "cudaMemcpyAsync(error word)");
    err = cudaStreamSynchronize(s);
    if (err != cudaSuccess) return b200::cuda_status(err, "cudaStreamSynchronize");
    if (clear) {
      err = cudaMemsetAsync(error_word, 0, sizeof(uint32_t), s);
      if (err != cudaSuccess) return b200::cuda_status(err, "cudaMemsetAsync(error word)");
    }
    return static_cast<int>(B200_OK);
  });
}

const char* b200_last_error(void) { return b200::last_error_cstr(); }

const char* b200_version(void) { return "b200_paged_attn 0.1.0 (sm_100a)"; }

}  // extern "C"
