// Host helpers: error strings, per-device properties, TMA tensor maps.
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "host_common.h"

namespace b200 {

namespace {
thread_local std::string g_last_error;

std::mutex g_mu;
std::vector<DeviceInfo> g_devices;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

struct MapKey {
  const void* base;
  int64_t slots;
  int heads, dim, dtype, chunk, rows, swz, box_heads;
  bool operator==(const MapKey& o) const {
    return base == o.base && slots == o.slots && heads == o.heads && dim == o.dim &&
           dtype == o.dtype && chunk == o.chunk && rows == o.rows && swz == o.swz &&
           box_heads == o.box_heads;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<const void*>()(k.base);
    h ^= std::hash<int64_t>()(k.slots) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
    h ^= static_cast<size_t>(k.heads * 131 + k.dim * 7 + k.dtype + k.chunk * 31 + k.rows * 17 +
                             k.swz * 3 + k.box_heads * 1009);
    return h;
  }
};
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

// Key of a general 16-bit tiled map (encode_tensor_map_16b).
struct GenKey {
  const void* base;
  int rank, dtype;
  uint64_t dims[5], strides[4];
  uint32_t box[5];
  bool operator==(const GenKey& o) const {
    return base == o.base && rank == o.rank && dtype == o.dtype &&
           std::memcmp(dims, o.dims, sizeof(dims)) == 0 &&
           std::memcmp(strides, o.strides, sizeof(strides)) == 0 &&
           std::memcmp(box, o.box, sizeof(box)) == 0;
  }
};
struct GenKeyHash {
  size_t operator()(const GenKey& k) const {
    size_t h = std::hash<const void*>()(k.base) ^ (static_cast<size_t>(k.rank) << 3);
    for (int i = 0; i < 5; ++i) h = h * 1000003u ^ std::hash<uint64_t>()(k.dims[i]);
    for (int i = 0; i < 4; ++i) h = h * 1000003u ^ std::hash<uint64_t>()(k.strides[i]);
    for (int i = 0; i < 5; ++i) h = h * 1000003u ^ k.box[i];
    return h ^ static_cast<size_t>(k.dtype);
  }
};
std::unordered_map<GenKey, CUtensorMap, GenKeyHash> g_gen_maps;

int load_encoder() {
  if (g_encode != nullptr) return B200_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (err != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
    return set_error(B200_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return B200_OK;
}
}  // namespace

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

void clear_error() { g_last_error.clear(); }

const char* last_error_cstr() { return g_last_error.c_str(); }

int cuda_status(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return B200_OK;
  return set_error(B200_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
}

int current_device_info(DeviceInfo* out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_status(err, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(g_mu);
  if (dev >= static_cast<int>(g_devices.size())) g_devices.resize(dev + 1);
  DeviceInfo& info = g_devices[dev];
  if (info.device < 0) {
    int sms = 0, smem = 0;
    err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (err != cudaSuccess) return cuda_status(err, "cudaDeviceGetAttribute(SM count)");
    err = cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (err != cudaSuccess) return cuda_status(err, "cudaDeviceGetAttribute(smem)");
    info.device = dev;
    info.num_sms = sms;
    info.max_smem_optin = smem;
  }
  *out = info;
  return B200_OK;
}

bool cache_tma_geometry(const b200_cache_desc* c, int tile_tokens, CacheTmaGeometry* geo,
                        std::string* why) {
  const int row_bytes = c->head_dim * 2;
  geo->chunk_bytes = row_bytes < 128 ? row_bytes : 128;
  geo->chunk_elems = geo->chunk_bytes / 2;
  geo->num_chunks = row_bytes / geo->chunk_bytes;
  geo->box_rows = c->block_size < tile_tokens ? c->block_size : tile_tokens;
  const int box_bytes = geo->box_rows * geo->chunk_bytes;
  if (box_bytes % 128 != 0) {
    *why = "block_size * head_dim * element_size must be a multiple of 128 bytes "
           "(TMA destination alignment)";
    return false;
  }
  // Swizzle only when every box starts on a swizzle-atom (1024-byte) boundary
  // so the pattern seen by the reader is the same however TMA anchors it.
  geo->swizzle_bytes = (box_bytes % 1024 == 0) ? geo->chunk_bytes : 0;
  geo->heads_per_box = 1;
  return true;
}

bool cache_head_group_geometry(const b200_cache_desc* c, int heads, CacheTmaGeometry* geo) {
  if (heads != 2 && heads != 4) return false;
  if (c->head_dim != 64 && c->head_dim != 128) return false;
  if (c->num_kv_heads % heads != 0) return false;
  const int tokens = 64 / heads;
  if (c->block_size < tokens) return false;  // one page must cover the tile
  geo->chunk_bytes = 128;
  geo->chunk_elems = 64;
  geo->num_chunks = c->head_dim / 64;
  geo->box_rows = tokens;
  geo->swizzle_bytes = 128;  // each region is 64 rows x 128 bytes, 1024-byte aligned
  geo->heads_per_box = heads;
  return true;
}

int encode_cache_tensor_map(const b200_cache_desc* c, const void* base,
                            const CacheTmaGeometry& geo, CUtensorMap* out) {
  const int64_t slots =
      static_cast<int64_t>(c->num_layers) * c->num_blocks * static_cast<int64_t>(c->block_size);
  MapKey key{base, slots, c->num_kv_heads, c->head_dim, c->dtype, geo.chunk_elems,
             geo.box_rows, geo.swizzle_bytes, geo.heads_per_box};
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_maps.find(key);
  if (it != g_maps.end()) {
    *out = it->second;
    return B200_OK;
  }
  const int enc = load_encoder();
  if (enc != B200_OK) return enc;
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return set_error(B200_ERR_INVALID, "cache tensor base must be 16-byte aligned");
  cuuint64_t gdim[3] = {static_cast<cuuint64_t>(c->head_dim),
                        static_cast<cuuint64_t>(c->num_kv_heads), static_cast<cuuint64_t>(slots)};
  cuuint64_t gstride[2] = {static_cast<cuuint64_t>(c->head_dim) * 2,
                           static_cast<cuuint64_t>(c->num_kv_heads) * c->head_dim * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(geo.chunk_elems), 1u,
                       static_cast<cuuint32_t>(geo.box_rows)};
  cuuint32_t estride[3] = {1u, 1u, 1u};
  CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_NONE;
  if (geo.swizzle_bytes == 32) swz = CU_TENSOR_MAP_SWIZZLE_32B;
  if (geo.swizzle_bytes == 64) swz = CU_TENSOR_MAP_SWIZZLE_64B;
  if (geo.swizzle_bytes == 128) swz = CU_TENSOR_MAP_SWIZZLE_128B;
  // Head-group view: dims {chunk elems, token slot, kv head, chunk}; the strides
  // are not in increasing order (row, then head, then chunk bytes), which is
  // what makes the box land head-major in shared memory.
  cuuint64_t gdim4[4] = {static_cast<cuuint64_t>(geo.chunk_elems), static_cast<cuuint64_t>(slots),
                         static_cast<cuuint64_t>(c->num_kv_heads),
                         static_cast<cuuint64_t>(geo.num_chunks)};
  cuuint64_t gstride4[3] = {static_cast<cuuint64_t>(c->num_kv_heads) * c->head_dim * 2,
                            static_cast<cuuint64_t>(c->head_dim) * 2,
                            static_cast<cuuint64_t>(geo.chunk_bytes)};
  cuuint32_t box4[4] = {static_cast<cuuint32_t>(geo.chunk_elems),
                        static_cast<cuuint32_t>(geo.box_rows),
                        static_cast<cuuint32_t>(geo.heads_per_box),
                        static_cast<cuuint32_t>(geo.num_chunks)};
  cuuint32_t estride4[4] = {1u, 1u, 1u, 1u};
  const bool grouped = geo.heads_per_box > 1;
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  CUresult r = g_encode(&map,
                        c->dtype == B200_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        grouped ? 4 : 3, const_cast<void*>(base), grouped ? gdim4 : gdim,
                        grouped ? gstride4 : gstride, grouped ? box4 : box,
                        grouped ? estride4 : estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(B200_ERR_CUDA,
                     "cuTensorMapEncodeTiled failed (code " + std::to_string(static_cast<int>(r)) +
                         ")");
  if (g_maps.size() > 4096) g_maps.clear();
  g_maps.emplace(key, map);
  *out = map;
  return B200_OK;
}

int encode_tensor_map_16b(const void* base, int rank, const uint64_t* dims,
                          const uint64_t* strides_bytes, const uint32_t* box, int dtype,
                          CUtensorMap* out) {
  if (rank < 2 || rank > 5) return set_error(B200_ERR_INVALID, "tensor map rank must be 2..5");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return set_error(B200_ERR_INVALID, "tensor base must be 16-byte aligned");
  GenKey key{};
  key.base = base;
  key.rank = rank;
  key.dtype = dtype;
  for (int i = 0; i < rank; ++i) {
    key.dims[i] = dims[i];
    key.box[i] = box[i];
    if (i + 1 < rank) {
      key.strides[i] = strides_bytes[i];
      if (strides_bytes[i] % 16 != 0)
        return set_error(B200_ERR_INVALID, "tensor strides must be multiples of 16 bytes");
    }
  }
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_gen_maps.find(key);
  if (it != g_gen_maps.end()) {
    *out = it->second;
    return B200_OK;
  }
  const int enc = load_encoder();
  if (enc != B200_OK) return enc;
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t gbox[5], estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = static_cast<cuuint64_t>(dims[i]);
    gbox[i] = static_cast<cuuint32_t>(box[i]);
    estride[i] = 1u;
    if (i + 1 < rank) gstride[i] = static_cast<cuuint64_t>(strides_bytes[i]);
  }
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  const CUresult r = g_encode(&map,
                              dtype == B200_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                              static_cast<cuuint32_t>(rank), const_cast<void*>(base), gdim, gstride,
                              gbox, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(B200_ERR_CUDA,
                     "cuTensorMapEncodeTiled failed (code " + std::to_string(static_cast<int>(r)) +
                         ")");
  if (g_gen_maps.size() > 4096) g_gen_maps.clear();
  g_gen_maps.emplace(key, map);
  *out = map;
  return B200_OK;
}

}  // namespace b200
