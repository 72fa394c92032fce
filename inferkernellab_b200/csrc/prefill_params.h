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
  int table_width;
  int sw_mask;
  float scale_log2;
};

// Query tokens per CTA of the tcgen05 kernel (one UMMA M tile).
constexpr int kTcRows = 128;

// tcgen05 prefill: head_dim 64 or 128, cache tiles with 128-byte swizzle,
// 16-byte aligned query/output rows.  `grid_x` counts 128-row query tiles
// (packed: an upper bound, excess CTAs exit).
int launch_prefill_tc(const CUtensorMap& kmap, const CUtensorMap& vmap, const PrefillParams& p,
                      int head_dim, bool bf16, unsigned grid_x, unsigned grid_y,
                      cudaStream_t stream);

}  // namespace b200
