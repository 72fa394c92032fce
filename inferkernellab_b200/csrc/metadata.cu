// GPU metadata builders: packed slot mapping + cu_seqlens for a scheduled
// batch, and the device-side form of the decode wrappers' input validation.
//
// slot mapping: the reference builds `slots` on the host once per request per
// step (PagedKVCache.slot_mapping, reference cache.py:113-129, called from
// decode.py:330-335,453-462 and hf_benchmark.py:363-368,397-402) and concatenates
// them with torch.cat.  Here one launch maps every scheduled token of every
// sequence straight from the device-resident block tables.
#include "../../include/b200_paged_attn.h"
#include "common.cuh"
#include "host_common.h"
#include "metadata.h"

namespace b200 {

constexpr int kMetaThreads = 256;
constexpr int kMetaMaxSeqs = 8192;

struct SlotParams {
  const void* tables;
  const void* starts;
  const void* ends;
  void* slots;
  int* cu;
  uint32_t* err;
  long long table_stride;
  long long total;
  int table64, index64, slots64;
  int table_width, num_seqs, block_size, num_blocks;
};

__global__ void __launch_bounds__(kMetaThreads) build_slot_mapping_kernel(const SlotParams p) {
  extern __shared__ long long prefix_s[];  // [num_seqs + 1]
  __shared__ long long scan_s[kMetaThreads];
  // Launched with programmatic stream serialization: no global access before
  // the previous kernel on the stream has completed.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int tid = threadIdx.x;
  const int B = p.num_seqs;
  const int chunk = (B + kMetaThreads - 1) / kMetaThreads;
  const int lo = tid * chunk;
  const int hi = min(B, lo + chunk);
  long long sum = 0;
  for (int i = lo; i < hi; ++i) {
    const long long n = load_index(p.ends, i, p.index64) - load_index(p.starts, i, p.index64);
    sum += n > 0 ? n : 0;
  }
  scan_s[tid] = sum;
  __syncthreads();
  if (tid == 0) {
    long long acc = 0;
    for (int i = 0; i < kMetaThreads; ++i) {
      const long long v = scan_s[i];
      scan_s[i] = acc;
      acc += v;
    }
    prefix_s[B] = acc;
  }
  __syncthreads();
  long long acc = scan_s[tid];
  for (int i = lo; i < hi; ++i) {
    prefix_s[i] = acc;
    const long long n = load_index(p.ends, i, p.index64) - load_index(p.starts, i, p.index64);
    acc += n > 0 ? n : 0;
  }
  __syncthreads();
  if (blockIdx.x == 0 && p.cu != nullptr)
    for (int i = tid; i <= B; i += kMetaThreads) p.cu[i] = static_cast<int>(prefix_s[i]);
  const long long total = prefix_s[B] < p.total ? prefix_s[B] : p.total;
  for (long long idx = blockIdx.x * static_cast<long long>(kMetaThreads) + tid; idx < total;
       idx += static_cast<long long>(gridDim.x) * kMetaThreads) {
    int l = 0, h = B;
    while (h - l > 1) {
      const int mid = (l + h) >> 1;
      if (prefix_s[mid] <= idx) l = mid; else h = mid;
    }
    const long long pos = load_index(p.starts, l, p.index64) + (idx - prefix_s[l]);
    const long long logical = pos / p.block_size;
    long long slot = -1;
    if (pos >= 0 && logical < p.table_width) {
      const long long blk =
          load_index(p.tables, static_cast<long long>(l) * p.table_stride + logical, p.table64);
      if (blk >= 0 && blk < p.num_blocks) slot = blk * p.block_size + (pos - logical * p.block_size);
    }
    if (slot < 0 && p.err) atomicOr(p.err, kErrBadBlock);
    if (p.slots64)
      reinterpret_cast<long long*>(p.slots)[idx] = slot;
    else
      reinterpret_cast<int*>(p.slots)[idx] = static_cast<int>(slot);
  }
}

int launch_build_slot_mapping(const void* block_tables, int32_t table_dtype, int64_t table_stride,
                              int32_t table_width, const void* starts, const void* ends,
                              int32_t index_dtype, int32_t num_seqs, int32_t block_size,
                              int32_t num_blocks, void* slots_out, int32_t slots_dtype,
                              int64_t total_tokens, int32_t* cu_seqlens_out, uint32_t* error_word,
                              cudaStream_t stream) {
  if (num_seqs <= 0 || num_seqs > kMetaMaxSeqs)
    return set_error(B200_ERR_INVALID, "num_seqs must be in [1, 8192]");
  if (block_size <= 0 || num_blocks <= 0 || table_width <= 0)
    return set_error(B200_ERR_INVALID, "block_size, num_blocks and table_width must be positive");
  if (total_tokens < 0) return set_error(B200_ERR_INVALID, "total_tokens must be non-negative");
  if (!block_tables || !starts || !ends || (total_tokens > 0 && !slots_out))
    return set_error(B200_ERR_INVALID, "null tensor pointer");
  SlotParams p;
  p.tables = block_tables;
  p.starts = starts;
  p.ends = ends;
  p.slots = slots_out;
  p.cu = cu_seqlens_out;
  p.err = error_word;
  p.table_stride = table_stride;
  p.total = total_tokens;
  p.table64 = table_dtype == B200_I64;
  p.index64 = index_dtype == B200_I64;
  p.slots64 = slots_dtype == B200_I64;
  p.table_width = table_width;
  p.num_seqs = num_seqs;
  p.block_size = block_size;
  p.num_blocks = num_blocks;
  long long blocks = (total_tokens + kMetaThreads - 1) / kMetaThreads;
  if (blocks < 1) blocks = 1;
  if (blocks > 148 * 4) blocks = 148 * 4;
  const size_t smem = (static_cast<size_t>(num_seqs) + 1) * sizeof(long long);
  if (smem > 48 * 1024) {
    cudaError_t err = cudaFuncSetAttribute(build_slot_mapping_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess) return cuda_status(err, "cudaFuncSetAttribute(slot mapping smem)");
  }
  return cuda_status(launch_dependent(build_slot_mapping_kernel, dim3(static_cast<unsigned>(blocks)),
                                      dim3(kMetaThreads), smem, stream, p),
                     "build_slot_mapping_kernel launch");
}

struct ValidateParams {
  const void* tables;
  const void* lens;
  int* flags;
  long long table_stride;
  long long capacity;
  int table64, lens64, table_width, num_seqs, num_blocks;
};

__global__ void __launch_bounds__(kMetaThreads) validate_decode_kernel(const ValidateParams p) {
  const long long n_table = static_cast<long long>(p.num_seqs) * p.table_width;
  bool bad_len = false, long_len = false, bad_blk = false;
  for (long long i = blockIdx.x * static_cast<long long>(kMetaThreads) + threadIdx.x;
       i < n_table + p.num_seqs; i += static_cast<long long>(gridDim.x) * kMetaThreads) {
    if (i < n_table) {
      const long long r = i / p.table_width;
      const long long c = i - r * p.table_width;
      const long long blk = load_index(p.tables, r * p.table_stride + c, p.table64);
      bad_blk |= blk < 0 || blk >= p.num_blocks;
    } else {
      const long long len = load_index(p.lens, i - n_table, p.lens64);
      bad_len |= len <= 0;
      long_len |= len > p.capacity;
    }
  }
  if (__any_sync(0xffffffffu, bad_len) && (threadIdx.x & 31) == 0) atomicOr(&p.flags[0], 1);
  if (__any_sync(0xffffffffu, long_len) && (threadIdx.x & 31) == 0) atomicOr(&p.flags[1], 1);
  if (__any_sync(0xffffffffu, bad_blk) && (threadIdx.x & 31) == 0) atomicOr(&p.flags[2], 1);
}

int launch_validate_decode_metadata(const void* block_tables, int32_t table_dtype,
                                    int64_t table_stride, int32_t table_width,
                                    const void* context_lens, int32_t lens_dtype, int32_t num_seqs,
                                    int32_t block_size, int32_t num_blocks, int32_t* flags_out,
                                    cudaStream_t stream) {
  if (num_seqs <= 0 || table_width <= 0 || block_size <= 0 || num_blocks <= 0)
    return set_error(B200_ERR_INVALID, "validation dimensions must be positive");
  if (!block_tables || !context_lens || !flags_out)
    return set_error(B200_ERR_INVALID, "null tensor pointer");
  cudaError_t err = cudaMemsetAsync(flags_out, 0, 3 * sizeof(int32_t), stream);
  if (err != cudaSuccess) return cuda_status(err, "cudaMemsetAsync(validation flags)");
  ValidateParams p;
  p.tables = block_tables;
  p.lens = context_lens;
  p.flags = flags_out;
  p.table_stride = table_stride;
  p.capacity = static_cast<long long>(table_width) * block_size;
  p.table64 = table_dtype == B200_I64;
  p.lens64 = lens_dtype == B200_I64;
  p.table_width = table_width;
  p.num_seqs = num_seqs;
  p.num_blocks = num_blocks;
  const long long n = static_cast<long long>(num_seqs) * table_width + num_seqs;
  long long blocks = (n + kMetaThreads - 1) / kMetaThreads;
  if (blocks > 148 * 4) blocks = 148 * 4;
  validate_decode_kernel<<<static_cast<unsigned>(blocks), kMetaThreads, 0, stream>>>(p);
  return cuda_status(cudaGetLastError(), "validate_decode_kernel launch");
}

}  // namespace b200
