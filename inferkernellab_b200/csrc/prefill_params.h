// Kernel parameters shared by the two paged prefill kernels (mma.sync in
// prefill.cu, tcgen05 in prefill_tc.cu) and the tcgen05 launcher.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "attn_core.cuh"

namespace b200 {

constexpr int kPreMaxSeqs = 8192;

struct PrefillParams {
  const void* q;
  void* out;
  const void* starts;
  const void* ends;
  const int* cu_seqlens;
  uint32_t* err;
  PagedSource src;
  long long q_stride_seq, q_stride_head, q_stride_token;
  long long o_stride_seq, o_stride_head, o_stride_token;
  int num_seqs, group, packed, max_query_len, index64;
  int num_kv_heads;
  int table_width;
  int sw_mask;
  float scale_log2;
};

// Rows of one tcgen05 query tile (one UMMA M tile).
constexpr int kTcRows = 128;

// Query tokens per CTA of the tcgen05 kernel for `group` query heads per kv
// head: the CTA's 256 rows are group heads x (256 / group) tokens.
int prefill_tc_query_block(int group);
// Query heads per 128-row tile of the tcgen05 kernel (the Q box's head extent).
int prefill_tc_query_heads_per_tile(int group);

// tcgen05 prefill: head_dim 64 or 128, cache tiles with 128-byte swizzle,
// 16-byte aligned query/output rows, a power-of-two number (<= 64) of query
// heads per kv head.  `qmap` is the query tensor's TMA map with box {64,
// heads per tile, 128 / heads per tile tokens (, 1)}: rank 3 {D, Hq, rows}
// when packed, rank 4 {D, Hq, T, B} when padded; `omap` the same over the
// output.  `grid_x` = query blocks x kv heads (packed: an upper bound on the
// blocks, excess CTAs exit); grid_y = 1.
int launch_prefill_tc(const CUtensorMap& kmap, const CUtensorMap& vmap, const CUtensorMap& qmap,
                      const CUtensorMap& omap, const PrefillParams& p, int head_dim, bool bf16,
                      unsigned grid_x, unsigned grid_y, cudaStream_t stream);

}  // namespace b200
