// KV append (reshape-and-cache) for sm_100a.
//
// cache[layer, slot / BS, slot % BS, h, :] = key[t, h, :]   (and the same for V)
//
// One thread moves one 16-byte vector of K *and* the matching vector of V, so a
// token row of head_dim*2 bytes is written by head_dim/8 consecutive threads
// with fully coalesced 128-bit loads and stores.  The copy is a raw byte move:
// bit-exact by construction (the reference's own test is torch.equal,
// tests/test_attention.py:196-207).  When a source row is not 16-byte aligned
// the kernel falls back to 2-byte elements (same result, slower).
#include <algorithm>

#include "../../include/b200_paged_attn.h"
#include "append.h"
#include "common.cuh"
#include "host_common.h"

namespace b200 {

struct AppendParams {
  const uint8_t* key;
  const uint8_t* value;
  uint8_t* k_cache;
  uint8_t* v_cache;
  const void* slots;
  uint32_t* err;
  long long num_tokens;
  long long key_stride_token, key_stride_head;  // bytes
  long long value_stride_token, value_stride_head;
  long long num_slots;        // num_blocks * block_size
  long long layer_slot_base;  // layer * num_slots
  int num_kv_heads;
  int row_bytes;  // head_dim * 2
  int slots64;
};

// One CTA per token: its threads walk the token's num_kv_heads x row vectors.
// The token's slot is read once per thread (one broadcast transaction) and the
// K/V loads are issued without waiting for it; index math is 32-bit.
template <typename V>
__global__ void __launch_bounds__(256) append_kv_kernel(const AppendParams p) {
  // Launched with programmatic stream serialization: no global access before
  // the previous kernel on the stream has completed.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int vec_per_row = p.row_bytes / static_cast<int>(sizeof(V));
  const int items = p.num_kv_heads * vec_per_row;
  const long long t = blockIdx.x;
  const long long slot = load_index(p.slots, t, p.slots64);
  if (slot >= p.num_slots && threadIdx.x == 0 && p.err) atomicOr(p.err, kErrBadSlot);
  const bool slot_ok = slot >= 0 && slot < p.num_slots;  // negative: padding, skipped
  const uint8_t* key = p.key + t * p.key_stride_token;
  const uint8_t* value = p.value + t * p.value_stride_token;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int h = it / vec_per_row;
    const int v = it - h * vec_per_row;
    const V kv = *reinterpret_cast<const V*>(key + h * p.key_stride_head + v * sizeof(V));
    const V vv = *reinterpret_cast<const V*>(value + h * p.value_stride_head + v * sizeof(V));
    if (!slot_ok) continue;
    const long long dst =
        ((p.layer_slot_base + slot) * p.num_kv_heads + h) * p.row_bytes + v * sizeof(V);
    *reinterpret_cast<V*>(p.k_cache + dst) = kv;
    *reinterpret_cast<V*>(p.v_cache + dst) = vv;
  }
}

int launch_append_kv(const b200_cache_desc* c, int32_t layer, const void* key, const void* value,
                     int64_t num_tokens, int64_t key_stride_token, int64_t key_stride_head,
                     int64_t value_stride_token, int64_t value_stride_head, const void* slots,
                     int32_t slots_dtype, uint32_t* error_word, cudaStream_t stream) {
  if (c == nullptr) return set_error(B200_ERR_INVALID, "null cache descriptor");
  if (c->num_layers <= 0 || c->num_blocks <= 0 || c->block_size <= 0 || c->num_kv_heads <= 0 ||
      c->head_dim <= 0)
    return set_error(B200_ERR_INVALID, "cache dimensions must be positive");
  if (c->dtype != B200_F16 && c->dtype != B200_BF16)
    return set_error(B200_ERR_UNSUPPORTED, "cache dtype must be float16 or bfloat16");
  if (layer < 0 || layer >= c->num_layers) return set_error(B200_ERR_LAYER, "layer is out of range");
  if (num_tokens < 0) return set_error(B200_ERR_INVALID, "num_tokens must be non-negative");
  if (num_tokens == 0) return B200_OK;
  if (!key || !value || !slots || !c->k_cache || !c->v_cache)
    return set_error(B200_ERR_INVALID, "null tensor pointer");
  AppendParams p;
  p.key = static_cast<const uint8_t*>(key);
  p.value = static_cast<const uint8_t*>(value);
  p.k_cache = static_cast<uint8_t*>(c->k_cache);
  p.v_cache = static_cast<uint8_t*>(c->v_cache);
  p.slots = slots;
  p.err = error_word;
  p.num_tokens = num_tokens;
  p.key_stride_token = key_stride_token * 2;
  p.key_stride_head = key_stride_head * 2;
  p.value_stride_token = value_stride_token * 2;
  p.value_stride_head = value_stride_head * 2;
  p.num_slots = static_cast<long long>(c->num_blocks) * c->block_size;
  p.layer_slot_base = static_cast<long long>(layer) * p.num_slots;
  p.num_kv_heads = c->num_kv_heads;
  p.row_bytes = c->head_dim * 2;
  p.slots64 = slots_dtype == B200_I64;
  const uintptr_t align = reinterpret_cast<uintptr_t>(key) | reinterpret_cast<uintptr_t>(value) |
                          reinterpret_cast<uintptr_t>(c->k_cache) |
                          reinterpret_cast<uintptr_t>(c->v_cache) |
                          static_cast<uintptr_t>(p.key_stride_token | p.key_stride_head |
                                                 p.value_stride_token | p.value_stride_head |
                                                 p.row_bytes);
  const bool vec16 = (align & 15) == 0;
  const long long vec_per_row = vec16 ? p.row_bytes / 16 : p.row_bytes / 2;
  // One CTA per token, as many threads as its vectors (a multiple of 32, <= 256).
  if (num_tokens > 0x7fffffffLL)
    return set_error(B200_ERR_UNSUPPORTED, "append is limited to 2^31 - 1 tokens");
  const long long items = c->num_kv_heads * vec_per_row;
  if (items > 0x7fffffffLL) return set_error(B200_ERR_UNSUPPORTED, "too many kv heads");
  const int threads = static_cast<int>(std::min<long long>(256, (items + 31) / 32 * 32));
  const dim3 grid(static_cast<unsigned>(num_tokens));
  const cudaError_t err =
      vec16 ? launch_dependent(append_kv_kernel<uint4>, grid, dim3(threads), 0, stream, p)
            : launch_dependent(append_kv_kernel<uint16_t>, grid, dim3(threads), 0, stream, p);
  return cuda_status(err, "append_kv_kernel launch");
}

}  // namespace b200
