/*
 * b200_paged_attn.h -- C ABI of the B200 (sm_100a) paged-KV attention library.
 *
 * Build:  nvcc -gencode arch=compute_100a,code=sm_100a -shared ... -> libb200_paged_attn.so
 *
 * Conventions
 *   - Plain device pointers and sizes only; no framework types cross this ABI.
 *   - Every entry point returns B200_OK (0) or a negative status code; no
 *     exception or abort crosses the ABI.  b200_last_error() returns the
 *     message of the calling thread's last failure.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *     All work is enqueued on it; no entry point synchronises the host except
 *     b200_read_error_word and the b200_validate_* helpers, which say so.
 *   - The KV cache layout is the reference's PagedKVCache storage
 *     (reference src/inferkernellab/cache.py:75-94): one contiguous tensor per K
 *     and V of shape [num_layers, num_blocks, block_size, num_kv_heads, head_dim].
 *   - Element types: float16 or bfloat16 (B200_F16 / B200_BF16).  Index arrays
 *     (block tables, lengths, slots) may be int32 or int64 (B200_I32 / B200_I64),
 *     like the reference wrappers accept (reference triton_ops.py:446-449).
 */
#ifndef B200_PAGED_ATTN_H
#define B200_PAGED_ATTN_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B200_API __attribute__((visibility("default")))
#else
#define B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum { B200_F16 = 0, B200_BF16 = 1 };
enum { B200_I32 = 0, B200_I64 = 1 };

enum {
  B200_OK = 0,
  B200_ERR_INVALID = -1,     /* bad shape / dtype / metadata  (Python: ValueError)   */
  B200_ERR_LAYER = -2,       /* layer index out of range       (Python: IndexError)   */
  B200_ERR_UNSUPPORTED = -3, /* shape this build does not cover (Python: ValueError)  */
  B200_ERR_WORKSPACE = -4,   /* workspace missing or too small (Python: RuntimeError) */
  B200_ERR_CUDA = -5,        /* CUDA runtime / driver failure  (Python: RuntimeError) */
  B200_ERR_DEVICE = -6       /* device error word was set      (Python: RuntimeError) */
};

/* Device error word bits (see b200_read_error_word). */
enum {
  B200_DEVERR_WAIT_FULL = 1,  /* a consumer gave up waiting for a TMA stage (bounded wait) */
  B200_DEVERR_WAIT_EMPTY = 2, /* a producer gave up waiting for a free stage               */
  B200_DEVERR_BAD_SLOT = 4,   /* append skipped a slot outside [0, num_blocks*block_size)  */
  B200_DEVERR_BAD_BLOCK = 8,  /* a block-table entry outside [0, num_blocks) was masked    */
  B200_DEVERR_DRAIN = 16      /* a producer gave up draining its copies after an abort     */
};

/* One paged KV cache (both K and V), reference layout, contiguous. */
typedef struct {
  void* k_cache;
  void* v_cache;
  int32_t num_layers;
  int32_t num_blocks; /* physical blocks per layer */
  int32_t block_size; /* tokens per block          */
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t dtype; /* B200_F16 or B200_BF16 */
} b200_cache_desc;

/* ------------------------------------------------------------------ decode
 * Paged decode attention: out[b, h, :] = softmax(q[b,h]·K_b^T·scale)·V_b over
 * the first context_lens[b] logical tokens of request b, K_b/V_b read through
 * block_tables[b, :] for kv head h / (num_q_heads / num_kv_heads).
 *
 * Replaces the reference's paged_decode_attention_triton /
 * paged_decode_attention_triton_grouped kernels and launch wrappers
 * (reference src/inferkernellab/triton_ops.py:80-167, 170-401, 404-610); the
 * math is the reference oracle paged_decode_attention (attention.py:134-175).
 * Same masking rules as the reference kernels: tokens past table_width *
 * block_size and tokens whose block id is outside [0, num_blocks) are skipped
 * (triton_ops.py:129-138).  A request with context_len <= 0 gets NaN output.
 *
 * Requirements: head_dim in {16, 32, 64, 128}; num_q_heads a multiple of
 * num_kv_heads with at most 64 query heads per KV head; block_size a power of
 * two <= 256 with block_size * head_dim * 2 a multiple of 128 bytes; q/out rows
 * contiguous in head_dim; num_seqs <= 8192.
 *
 * Workspace: `workspace` must hold b200_paged_decode_workspace_bytes() bytes
 * and be ZERO-FILLED before its first use; every launch that completes leaves
 * its split counters at zero again.  The counters sit after the split partials,
 * whose size depends only on (num_q_heads / num_kv_heads, num_kv_heads,
 * head_dim, block_size, dtype) -- the last four choose how many KV heads share
 * one tile -- so one workspace can serve any batch size without re-zeroing;
 * re-zero it when any of these changes, or after a device error.
 * Calls that share one workspace must be ordered (same stream, or synchronised).
 */
typedef struct {
  int32_t num_seqs;    /* B                                 */
  int32_t num_q_heads; /* Hq                                */
  int32_t table_width; /* W: columns of block_tables        */
  int32_t layer;       /* cache layer to read               */
  int64_t q_stride_seq, q_stride_head;     /* elements */
  int64_t out_stride_seq, out_stride_head; /* elements */
  int64_t table_stride;                    /* elements between block_tables rows */
  int32_t table_dtype;                     /* B200_I32 / B200_I64 */
  int32_t lens_dtype;                      /* B200_I32 / B200_I64 */
  float scale;                             /* softmax scale (reference default head_dim^-0.5) */
} b200_decode_args;

B200_API size_t b200_paged_decode_workspace_bytes(const b200_cache_desc* cache, const b200_decode_args* args);

B200_API int b200_paged_decode(const b200_cache_desc* cache, const b200_decode_args* args, const void* query,
                      const void* block_tables, const void* context_lens, void* out,
                      void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------- allocation-free decode
 * No counterpart in the reference: an addition of this library.
 *
 * Same computation and arguments as b200_paged_decode, minus the workspace.
 * It is for callers that cannot allocate device memory while attention runs --
 * a plugin or custom operator executing inside a host framework that owns all
 * buffers and forbids cudaMalloc at that point (it would also synchronise the
 * device), or code held to a fixed memory budget.  The caller still passes the
 * query, the metadata and the output buffer; the split-KV scratch comes from a
 * static device array of b200_paged_decode_noalloc_scratch_bytes() (8 MiB) that
 * every GPU loading the library holds until the process exits.
 *
 *  - Allocates nothing: no cudaMalloc / cudaFree, no allocating library call.
 *  - Shapes whose split scratch would exceed 8 MiB are rejected with
 *    B200_ERR_WORKSPACE and a message (for example 64 query heads per KV head
 *    at head_dim 128); use b200_paged_decode with a workspace for those.
 *  - The first call on a device, with that device current, resolves the
 *    array's device address (cudaGetSymbolAddress); make that first call
 *    before any stream capture.  The address is kept per device and per
 *    current context, so a new context on that device (after cudaDeviceReset)
 *    resolves it again.
 *  - All calls share the one array and it keeps the last call's contents:
 *    each call zeroes the error word and split counters (two cudaMemsetAsync
 *    on `stream`) before its launch.  Calls whose executions overlap on the
 *    GPU (different streams without ordering) race on the array.
 *  - Device-side conditions of a call (a masked out-of-pool block id, a
 *    bounded wait that gave up: the B200_DEVERR_* bits) land in the array's
 *    error word; read it after the call, before the next one clears it, with
 *    b200_read_error_word on the address from
 *    b200_paged_decode_noalloc_error_word.
 */
B200_API int b200_paged_decode_noalloc(const b200_cache_desc* cache, const b200_decode_args* args,
                                       const void* query, const void* block_tables,
                                       const void* context_lens, void* out, void* stream);

/* Size in bytes of the static scratch array used by b200_paged_decode_noalloc. */
B200_API size_t b200_paged_decode_noalloc_scratch_bytes(void);

/* Device address of the error word inside that static array, for the current
 * device (no counterpart in the reference).  Resolves the array's address like
 * the first b200_paged_decode_noalloc call does, and allocates nothing.  Pass
 * the address to b200_read_error_word after a b200_paged_decode_noalloc call
 * on the same device. */
B200_API int b200_paged_decode_noalloc_error_word(uint32_t** error_word_out);

/* ------------------------------------------------------------------ append
 * Reshape-and-cache: cache[layer, slot/BS, slot%BS, h, :] = key[t, h, :] (and V)
 * for every token t, bit-exact.  Replaces the reference's append_kv_triton and
 * _append_kv_kernel (reference src/inferkernellab/append.py:19-106) and the
 * torch scatter PagedKVCache.write_slots (cache.py:156-189).  Negative slots
 * are skipped (padding); slots >= num_blocks*block_size are skipped and set
 * B200_DEVERR_BAD_SLOT in *error_word when error_word is not NULL.
 */
B200_API int b200_append_kv(const b200_cache_desc* cache, int32_t layer, const void* key, const void* value,
                   int64_t num_tokens, int64_t key_stride_token, int64_t key_stride_head,
                   int64_t value_stride_token, int64_t value_stride_head, const void* slots,
                   int32_t slots_dtype, uint32_t* error_word, void* stream);

/* -------------------------------------------- decode with fused append
 * b200_paged_decode_append = b200_rope_append_kv (rope = 1) or b200_append_kv
 * (rope = 0) of every request's new token followed by b200_paged_decode, in one
 * launch (reference: hf_benchmark.py:69-85 rotary, append.py:69-106 append,
 * triton_ops.py:404-478 decode).  The new token of request b must be its last
 * context position, context_lens[b] - 1 (a decode step).  query is the
 * un-rotated query when rope = 1; key/value [B, Hkv, D] (strides below); cos/sin
 * [B, D] rows of the rotary table for each request's new position (rope = 1);
 * key/value/cos/sin rows 16-byte aligned, and with rope also query and out rows
 * (the rotated query is staged in out before the output overwrites it); slots
 * [B] (negative = skip the append).  The cache holds
 * exactly what the separate calls would write; the output matches
 * b200_paged_decode on the rotated query.  Workspace as b200_paged_decode.
 */
typedef struct {
  int32_t rope;        /* 1 = rotary embedding on query and the new key, 0 = plain append */
  int32_t slots_dtype; /* B200_I32 / B200_I64 */
  int64_t k_stride_seq, k_stride_head; /* elements */
  int64_t v_stride_seq, v_stride_head;
  int64_t cos_stride_seq, sin_stride_seq;
} b200_decode_append_args;

B200_API int b200_paged_decode_append(const b200_cache_desc* cache, const b200_decode_args* args,
                                      const b200_decode_append_args* append, const void* query,
                                      const void* key, const void* value, const void* cos,
                                      const void* sin, const void* slots, const void* block_tables,
                                      const void* context_lens, void* out, void* workspace,
                                      size_t workspace_bytes, void* stream);

/* ------------------------------------------------- fused rotary + append
 * For every token t and head h (rotate_half(x) = concat(-x[D/2:], x[:D/2])):
 *   query_out[t, h]            = query[t, h] * cos[t] + rotate_half(query[t, h]) * sin[t]
 *   cache.K[layer, slot[t], h] = key[t, h]   * cos[t] + rotate_half(key[t, h])   * sin[t]
 *   cache.V[layer, slot[t], h] = value[t, h]
 * rounded to the 16-bit type after each multiply and after the add, exactly like
 * the reference's torch elementwise rotary (reference hf_benchmark.py:69-85), so
 * results are bit-identical to rotating with torch and then calling
 * b200_append_kv.  One launch replaces the rotary ops, the layout copies and the
 * append of a layer (decode step or packed prefill batch).  cos/sin: [T, D] in
 * the cache dtype.  Slot rules as b200_append_kv.
 */
typedef struct {
  int64_t num_tokens;
  int32_t num_q_heads;
  int32_t layer;
  int64_t q_stride_token, q_stride_head; /* elements */
  int64_t k_stride_token, k_stride_head;
  int64_t v_stride_token, v_stride_head;
  int64_t q_out_stride_token, q_out_stride_head;
  int64_t cos_stride_token, sin_stride_token;
  int32_t slots_dtype; /* B200_I32 / B200_I64 */
} b200_rope_append_args;

B200_API int b200_rope_append_kv(const b200_cache_desc* cache, const b200_rope_append_args* args,
                                 const void* query, const void* key, const void* value,
                                 const void* cos, const void* sin, const void* slots,
                                 void* query_out, uint32_t* error_word, void* stream);

/* ------------------------------------------------------- diagnostics
 * b200_tc_selftest: one CTA checks the tcgen05 building blocks of the prefill
 * kernel (128-byte swizzled K-major / MN-major shared-memory descriptors,
 * kind::f16 MMAs into tensor memory, tcgen05.ld readback):
 *   c1[128, 64]  = a[128, 64] . b[64, 64]^T,   c2[128, 128] = a[128, 64] . v[64, 128],
 *   c3 = c2 with a read from tensor memory (the A-in-TMEM MMA form)
 * a, b, v row-major 16-bit (dtype), 16-byte aligned; c1, c2, c3 row-major float32.
 * No counterpart in the reference. */
B200_API int b200_tc_selftest(const void* a, const void* b, const void* v, float* c1, float* c2,
                              float* c3, int32_t dtype, uint32_t* error_word, void* stream);

/* b200_wait_selftest: runs the bounded mbarrier wait that every kernel of this
 * library uses (1 s limit there) with limit_ns instead, in a one-CTA kernel.
 * With arrive = 0 nobody arrives: the first waiter gives up after limit_ns,
 * sets B200_DEVERR_WAIT_FULL in *error_word and raises the CTA abort flag,
 * through which the other waiters leave; the kernel returns and the context
 * stays usable.  With arrive = 1 every wait completes and nothing is set.
 * result (device uint32[3]): waits completed in the first / second waiting
 * warp, and the ns the first waiter spent.  limit_ns in [1000, 2e9].
 * No counterpart in the reference. */
B200_API int b200_wait_selftest(int64_t limit_ns, int32_t arrive, uint32_t* result,
                                uint32_t* error_word, void* stream);

/* ------------------------------------------------- decoder-layer helpers
 * Kernels for the Llama layer around the attention call (the reference's
 * LlamaPagedDecodeRunner applies Transformers' LlamaRMSNorm and LlamaMLP
 * modules there, reference hf_benchmark.py:408-511; these have no kernel
 * counterpart in the reference).  dtype is B200_F16 or B200_BF16; strides are
 * row strides in elements; 16-byte aligned rows with cols % 8 == 0 take the
 * vectorised path.
 *
 * b200_add_rmsnorm: with x != NULL, residual_out = rnd(x + residual) (may alias
 * residual); then out = rnd(weight * rnd(s * rsqrt(mean(s^2) + eps))) where s is
 * the summed row (or residual itself when x == NULL) -- LlamaRMSNorm's
 * roundings, one launch (one CTA per row).
 * b200_silu_mul: gate_up rows hold [gate | up] (cols each);
 * out = rnd(rnd(silu(gate)) * up) -- LlamaMLP's act_fn(gate) * up.
 */
B200_API int b200_add_rmsnorm(const void* x, const void* residual, const void* weight, void* out,
                              void* residual_out, int64_t rows, int64_t cols, int64_t x_stride,
                              int64_t residual_stride, int64_t out_stride,
                              int64_t residual_out_stride, float eps, int32_t dtype, void* stream);

B200_API int b200_silu_mul(const void* gate_up, void* out, int64_t rows, int64_t cols,
                           int64_t in_stride, int64_t out_stride, int32_t dtype, void* stream);

/* ----------------------------------------------------------------- prefill
 * Ragged causal prefill attention over the paged cache.  Sequence b owns the
 * query tokens of logical positions query_starts[b] .. context_lens[b]-1; a
 * query at position p attends cache keys 0..p of sequence b (the cache must
 * already hold them -- append first).  Replaces the reference's
 * paged_prefill_attention_sdpa (reference src/inferkernellab/attention.py:230-321).
 *
 * query_layout 0 (padded, the reference signature): query/out [B, Hq, T, D]
 *   with T = max_query_len; padded rows t >= context_lens[b]-query_starts[b]
 *   attend key 0 only, exactly like the reference's mask (attention.py:313).
 * query_layout 1 (packed): query/out [total_query_tokens, Hq, D]; sequence b
 *   owns rows cu_seqlens_q[b] .. cu_seqlens_q[b+1]-1 (int32 [B+1]).
 * error_word (device uint32, may be NULL) collects B200_DEVERR_* bits.
 */
typedef struct {
  int32_t num_seqs;
  int32_t num_q_heads;
  int32_t table_width;
  int32_t layer;
  int32_t query_layout;       /* 0 = padded, 1 = packed          */
  int32_t max_query_len;      /* T (padded) / longest range      */
  int64_t total_query_tokens; /* rows of a packed query          */
  int64_t q_stride_seq, q_stride_head, q_stride_token; /* elements; stride_seq unused when packed */
  int64_t o_stride_seq, o_stride_head, o_stride_token;
  int64_t table_stride;
  int32_t table_dtype; /* B200_I32 / B200_I64 */
  int32_t index_dtype; /* dtype of query_starts / context_lens */
  float scale;
  int32_t kernel; /* B200_PREFILL_AUTO / _TCGEN05 / _MMA_SYNC */
} b200_prefill_args;

/* Prefill kernel choice.  AUTO takes the tcgen05 (TMEM) kernel for head_dim
 * 64 / 128 on 128-byte swizzled cache tiles (block_size >= 8) and the
 * mma.sync kernel otherwise; TCGEN05 fails with B200_ERR_UNSUPPORTED where it
 * cannot run. */
enum { B200_PREFILL_AUTO = 0, B200_PREFILL_TCGEN05 = 1, B200_PREFILL_MMA_SYNC = 2 };

B200_API int b200_paged_prefill(const b200_cache_desc* cache, const b200_prefill_args* args,
                       const void* query, const void* block_tables, const void* query_starts,
                       const void* context_lens, const int32_t* cu_seqlens_q, void* out,
                       uint32_t* error_word, void* stream);

/* --------------------------------------------------------------- metadata
 * GPU metadata builder for a scheduled batch (token-budget packing moved onto
 * the device).  For each sequence b the logical range starts[b] .. ends[b]-1 is
 * mapped through block_tables[b, :] to physical slots
 *     slot = table[b][p / block_size] * block_size + p % block_size
 * exactly like PagedKVCache.slot_mapping (reference cache.py:113-129), packed
 * in sequence order into slots_out (total_tokens entries), and cu_seqlens_out
 * (int32 [B+1], may be NULL) receives the prefix sums of ends - starts.
 * A position whose logical block is past table_width or whose block id is
 * outside [0, num_blocks) gets slot -1 and sets B200_DEVERR_BAD_BLOCK.
 */
B200_API int b200_build_slot_mapping(const void* block_tables, int32_t table_dtype, int64_t table_stride,
                            int32_t table_width, const void* starts, const void* ends,
                            int32_t index_dtype, int32_t num_seqs, int32_t block_size,
                            int32_t num_blocks, void* slots_out, int32_t slots_dtype,
                            int64_t total_tokens, int32_t* cu_seqlens_out, uint32_t* error_word,
                            void* stream);

/* ------------------------------------------------------------- validation
 * Device-side form of the reference wrappers' validate_inputs checks
 * (reference triton_ops.py:450-457).  Writes three int32 flags to flags_out
 * (device memory): [0] some context_len <= 0, [1] some context_len >
 * table_width*block_size, [2] some block-table entry outside [0, num_blocks).
 * Asynchronous; the caller reads flags_out.
 */
B200_API int b200_validate_decode_metadata(const void* block_tables, int32_t table_dtype,
                                  int64_t table_stride, int32_t table_width,
                                  const void* context_lens, int32_t lens_dtype, int32_t num_seqs,
                                  int32_t block_size, int32_t num_blocks, int32_t* flags_out,
                                  void* stream);

/* --------------------------------------------------------------- utilities */

/* Synchronises `stream`, reads the uint32 device error word at `error_word`
 * into *value, and (if clear != 0) zeroes it.  Host-blocking. */
B200_API int b200_read_error_word(uint32_t* error_word, uint32_t* value, int32_t clear, void* stream);

/* Message of this thread's last failure ("" if none). */
B200_API const char* b200_last_error(void);

/* Library version string. */
B200_API const char* b200_version(void);

#ifdef __cplusplus
}
#endif

#endif /* B200_PAGED_ATTN_H */
