// Fused rotary embedding + KV append for sm_100a.
//
// For every token t (a decode step's new tokens or a prefill batch's packed
// tokens) and head h:
//   q_out[t, h]                    = rope(q[t, h], cos[t], sin[t])
//   cache.K[layer, slot[t], h]     = rope(k[t, h], cos[t], sin[t])
//   cache.V[layer, slot[t], h]     = v[t, h]
// with rope(x)[i] = x[i] * cos[i] + rotate_half(x)[i] * sin[i],
// rotate_half(x) = concat(-x[D/2:], x[:D/2]) -- the rotation the reference
// applies with torch elementwise ops (hf_benchmark.py:69-85).  Each of those ops
// rounds to the 16-bit type, so the kernel rounds at the same three points
// (x*cos, rotate_half(x)*sin, their sum): its output is bit-identical to the
// reference's, and the appended K/V equal what append_kv would store.
// One launch replaces the rotary ops, the layout copies and the append.
#include <algorithm>

#include "../../include/b200_paged_attn.h"
#include "common.cuh"
#include "host_common.h"
#include "rope_append.h"

namespace b200 {

struct RopeParams {
  const uint8_t* q;
  const uint8_t* k;
  const uint8_t* v;
  const uint8_t* cos;
  const uint8_t* sin;
  uint8_t* q_out;
  uint8_t* k_cache;
  uint8_t* v_cache;
  const void* slots;
  uint32_t* err;
  long long num_tokens;
  long long q_st, q_sh, k_st, k_sh, v_st, v_sh;  // strides, elements
  long long qo_st, qo_sh;
  long long cos_st, sin_st;
  long long num_slots, layer_slot_base;
  int num_q_heads, num_kv_heads, head_dim, slots64;
};

// 8 x 16-bit elements = one 16-byte access.
struct alignas(16) Vec8 {
  uint16_t h[8];
};

template <typename E>
__device__ __forceinline__ float lane_f(const Vec8& v, int i) {
  typename E::T t;
  memcpy(&t, &v.h[i], 2);
  return to_float<E>(t);
}

template <typename E>
__device__ __forceinline__ void lane_set(Vec8& v, int i, float x) {
  typename E::T t = from_float<E>(x);
  memcpy(&v.h[i], &t, 2);
}

// One CTA per token; its threads walk the token's work items: W consecutive
// pair indices i..i+W-1 of one row (W = 8 with 16-byte vectors, else 1).  Rows:
// q heads, then k heads (rotated), then v heads (copied).  All index math is
// 32-bit within a token; the token's slot is read once per thread (one
// broadcast transaction) and every load of an item is issued before the slot
// is checked, so loads are not queued behind the slot's round trip.
template <typename E, int W>
__global__ void __launch_bounds__(1024) rope_append_kernel(const RopeParams p) {
  using T = typename E::T;
  const int half = p.head_dim / 2;
  const int items_per_row = half / W;
  const int rot_rows = p.num_q_heads + p.num_kv_heads;
  const int items = (rot_rows + p.num_kv_heads) * items_per_row;
  const long long t = blockIdx.x;
  const long long slot = load_index(p.slots, t, p.slots64);
  const bool slot_ok = slot >= 0 && slot < p.num_slots;
  if (slot >= p.num_slots && threadIdx.x == 0 && p.err) atomicOr(p.err, kErrBadSlot);
  const T* c = reinterpret_cast<const T*>(p.cos) + t * p.cos_st;
  const T* s = reinterpret_cast<const T*>(p.sin) + t * p.sin_st;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int row = it / items_per_row;
    const int i = (it - row * items_per_row) * W;
    const bool is_q = row < p.num_q_heads;
    const bool is_k = !is_q && row < rot_rows;
    if (!is_q && !slot_ok) continue;  // padding (negative) or out-of-pool slot: no append
    const T* src;
    T* dst;
    if (is_q) {
      src = reinterpret_cast<const T*>(p.q) + t * p.q_st + row * p.q_sh;
      dst = reinterpret_cast<T*>(p.q_out) + t * p.qo_st + row * p.qo_sh;
    } else if (is_k) {
      const int h = row - p.num_q_heads;
      src = reinterpret_cast<const T*>(p.k) + t * p.k_st + h * p.k_sh;
      dst = reinterpret_cast<T*>(p.k_cache) +
            ((p.layer_slot_base + slot) * p.num_kv_heads + h) * p.head_dim;
    } else {
      const int h = row - rot_rows;
      src = reinterpret_cast<const T*>(p.v) + t * p.v_st + h * p.v_sh;
      dst = reinterpret_cast<T*>(p.v_cache) +
            ((p.layer_slot_base + slot) * p.num_kv_heads + h) * p.head_dim;
    }
    if (W == 8) {
      const Vec8 x1 = *reinterpret_cast<const Vec8*>(src + i);
      const Vec8 x2 = *reinterpret_cast<const Vec8*>(src + i + half);
      if (!(is_q || is_k)) {
        *reinterpret_cast<Vec8*>(dst + i) = x1;
        *reinterpret_cast<Vec8*>(dst + i + half) = x2;
        continue;
      }
      const Vec8 c1 = *reinterpret_cast<const Vec8*>(c + i);
      const Vec8 c2 = *reinterpret_cast<const Vec8*>(c + i + half);
      const Vec8 s1 = *reinterpret_cast<const Vec8*>(s + i);
      const Vec8 s2 = *reinterpret_cast<const Vec8*>(s + i + half);
      Vec8 lo, hi;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float a = lane_f<E>(x1, j), b = lane_f<E>(x2, j);
        float l, h;
        rope_pair<E>(a, b, lane_f<E>(c1, j), lane_f<E>(s1, j), lane_f<E>(c2, j), lane_f<E>(s2, j),
                     l, h);
        lane_set<E>(lo, j, l);
        lane_set<E>(hi, j, h);
      }
      *reinterpret_cast<Vec8*>(dst + i) = lo;
      *reinterpret_cast<Vec8*>(dst + i + half) = hi;
    } else {
      if (!(is_q || is_k)) {
        dst[i] = src[i];
        dst[i + half] = src[i + half];
        continue;
      }
      float l, h;
      rope_pair<E>(to_float<E>(src[i]), to_float<E>(src[i + half]), to_float<E>(c[i]),
                   to_float<E>(s[i]), to_float<E>(c[i + half]), to_float<E>(s[i + half]), l, h);
      dst[i] = from_float<E>(l);
      dst[i + half] = from_float<E>(h);
    }
  }
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int launch_rope_append(const b200_cache_desc* c, const b200_rope_append_args* a, const void* query,
                       const void* key, const void* value, const void* cos, const void* sin,
                       const void* slots, void* query_out, uint32_t* error_word,
                       cudaStream_t stream) {
  if (c == nullptr || a == nullptr) return set_error(B200_ERR_INVALID, "null descriptor");
  if (c->num_layers <= 0 || c->num_blocks <= 0 || c->block_size <= 0 || c->num_kv_heads <= 0 ||
      c->head_dim <= 0)
    return set_error(B200_ERR_INVALID, "cache dimensions must be positive");
  if (c->dtype != B200_F16 && c->dtype != B200_BF16)
    return set_error(B200_ERR_UNSUPPORTED, "cache dtype must be float16 or bfloat16");
  if (c->head_dim % 2 != 0) return set_error(B200_ERR_INVALID, "head_dim must be even for rotary");
  if (a->layer < 0 || a->layer >= c->num_layers)
    return set_error(B200_ERR_LAYER, "layer is out of range");
  if (a->num_q_heads <= 0 || a->num_q_heads % c->num_kv_heads != 0)
    return set_error(B200_ERR_INVALID, "num_heads must be divisible by num_kv_heads");
  if (a->num_tokens < 0) return set_error(B200_ERR_INVALID, "num_tokens must be non-negative");
  if (a->num_tokens == 0) return B200_OK;
  if (!query || !key || !value || !cos || !sin || !slots || !query_out || !c->k_cache ||
      !c->v_cache)
    return set_error(B200_ERR_INVALID, "null tensor pointer");
  RopeParams p;
  p.q = static_cast<const uint8_t*>(query);
  p.k = static_cast<const uint8_t*>(key);
  p.v = static_cast<const uint8_t*>(value);
  p.cos = static_cast<const uint8_t*>(cos);
  p.sin = static_cast<const uint8_t*>(sin);
  p.q_out = static_cast<uint8_t*>(query_out);
  p.k_cache = static_cast<uint8_t*>(c->k_cache);
  p.v_cache = static_cast<uint8_t*>(c->v_cache);
  p.slots = slots;
  p.err = error_word;
  p.num_tokens = a->num_tokens;
  p.q_st = a->q_stride_token;
  p.q_sh = a->q_stride_head;
  p.k_st = a->k_stride_token;
  p.k_sh = a->k_stride_head;
  p.v_st = a->v_stride_token;
  p.v_sh = a->v_stride_head;
  p.qo_st = a->q_out_stride_token;
  p.qo_sh = a->q_out_stride_head;
  p.cos_st = a->cos_stride_token;
  p.sin_st = a->sin_stride_token;
  p.num_slots = static_cast<long long>(c->num_blocks) * c->block_size;
  p.layer_slot_base = static_cast<long long>(a->layer) * p.num_slots;
  p.num_q_heads = a->num_q_heads;
  p.num_kv_heads = c->num_kv_heads;
  p.head_dim = c->head_dim;
  p.slots64 = a->slots_dtype == B200_I64;
  // 16-byte vectors need every row start and both halves 16-byte aligned.
  const bool vec = c->head_dim % 16 == 0 && p.q_st % 8 == 0 && p.q_sh % 8 == 0 &&
                   p.k_st % 8 == 0 && p.k_sh % 8 == 0 && p.v_st % 8 == 0 && p.v_sh % 8 == 0 &&
                   p.qo_st % 8 == 0 && p.qo_sh % 8 == 0 && p.cos_st % 8 == 0 &&
                   p.sin_st % 8 == 0 && aligned16(query) && aligned16(key) && aligned16(value) &&
                   aligned16(cos) && aligned16(sin) && aligned16(query_out) &&
                   aligned16(c->k_cache) && aligned16(c->v_cache);
  const int width = vec ? 8 : 1;
  // One CTA per token: its (Hq + 2 Hkv) x head_dim / (2 width) items.
  if (a->num_tokens > 0x7fffffffLL)
    return set_error(B200_ERR_UNSUPPORTED, "rotary append is limited to 2^31 - 1 tokens");
  const long long items =
      (a->num_q_heads + 2LL * c->num_kv_heads) * (c->head_dim / 2 / width);
  if (items > 0x7fffffffLL) return set_error(B200_ERR_UNSUPPORTED, "too many heads per token");
  const unsigned b = static_cast<unsigned>(a->num_tokens);
  // A thread per item (up to 1024): every load of a token is in flight at once.
  const unsigned t = static_cast<unsigned>(std::min<long long>(1024, (items + 31) / 32 * 32));
  if (c->dtype == B200_BF16) {
    if (vec)
      rope_append_kernel<BF16, 8><<<b, t, 0, stream>>>(p);
    else
      rope_append_kernel<BF16, 1><<<b, t, 0, stream>>>(p);
  } else {
    if (vec)
      rope_append_kernel<Half, 8><<<b, t, 0, stream>>>(p);
    else
      rope_append_kernel<Half, 1><<<b, t, 0, stream>>>(p);
  }
  return cuda_status(cudaGetLastError(), "rope_append_kernel launch");
}

}  // namespace b200
