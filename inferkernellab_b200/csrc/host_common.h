// Host-side helpers shared by the launchers: error reporting, device
// properties, TMA tensor-map encoding.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/b200_paged_attn.h"

namespace b200 {

// Records `msg` as this thread's last error and returns `code`.
int set_error(int code, const std::string& msg);
void clear_error();

// cudaError_t -> B200_ERR_CUDA with a message naming `what`.
int cuda_status(cudaError_t err, const char* what);

struct DeviceInfo {
  int device = -1;
  int num_sms = 0;
  int max_smem_optin = 0;
};
// Properties of the current device (cached per device).
int current_device_info(DeviceInfo* out);

// Geometry of the 3-D TMA view of one cache tensor:
//   dim0 = head_dim (contiguous), dim1 = kv heads, dim2 = every token slot of
//   every layer (num_layers * num_blocks * block_size).
struct CacheTmaGeometry {
  int chunk_elems;  // elements of head_dim per TMA box row (<= 128 bytes)
  int chunk_bytes;
  int num_chunks;   // head_dim / chunk_elems
  int box_rows;     // tokens per box
  int swizzle_bytes;  // 0, 32, 64 or 128
  // 1: the 3-D view above, one kv head and one chunk per box.  > 1: the 4-D
  // head-group view {chunk_elems, token slot, kv head, chunk} (strides row,
  // head, chunk bytes) whose box {chunk_elems, box_rows, heads_per_box,
  // num_chunks} lands in shared memory as num_chunks regions of
  // heads_per_box * box_rows rows, head-major (row = head * box_rows + token).
  int heads_per_box = 1;
};

// Chooses the box geometry for a cache and a token tile; returns false with a
// message if the layout cannot be expressed (see the header's requirements).
bool cache_tma_geometry(const b200_cache_desc* cache, int tile_tokens, CacheTmaGeometry* geo,
                        std::string* why);

// Head-group geometry: boxes of `heads` kv heads x (64 / heads) tokens, all
// chunks (one box per tile).  Only for heads in {2, 4} with 64 / heads <=
// block_size and head_dim 64 or 128; returns false otherwise.
bool cache_head_group_geometry(const b200_cache_desc* cache, int heads, CacheTmaGeometry* geo);

// Encodes (or returns a cached copy of) the tensor map of one cache tensor.
int encode_cache_tensor_map(const b200_cache_desc* cache, const void* base,
                            const CacheTmaGeometry& geo, CUtensorMap* out);

// Encodes (or returns a cached copy of) a tiled map of 16-bit elements with
// 128-byte swizzle: `rank` dims innermost first, byte strides of dims
// 1..rank-1 (multiples of 16), box sizes per dim.
int encode_tensor_map_16b(const void* base, int rank, const uint64_t* dims,
                          const uint64_t* strides_bytes, const uint32_t* box, int dtype,
                          CUtensorMap* out);

inline int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Launch with programmatic stream serialization: the grid may be scheduled while
// the previous kernel on the stream is finishing, so the kernel must execute
// griddepcontrol.wait before its first global memory access.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_dependent(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                    cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
}

}  // namespace b200
