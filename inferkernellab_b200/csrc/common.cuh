// Shared device helpers for the sm_100a paged-attention kernels.
//
// Everything here is hand-written inline PTX for Blackwell (sm_100a):
//   * mbarrier init / arrive / expect-tx / bounded parity wait,
//   * TMA tiled loads (cp.async.bulk.tensor.3d, no multicast),
//   * ldmatrix (plain and transposed) and mma.sync m16n8k16 (f16/bf16 -> f32),
//   * ex2.approx and small conversion helpers.
//
// Bounded waits: every spin on an mbarrier gives up after kWaitLimitNs of
// %globaltimer time, records an error code in a device error word and raises
// an abort flag in shared memory so that every other waiter of the CTA leaves
// too.  No kernel here traps or spins forever.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

// Error codes written to the device error word (bit flags, OR-ed together).
enum DeviceError : uint32_t {
  kErrNone = 0u,
  kErrWaitFull = 1u,      // consumer gave up waiting for a TMA stage
  kErrWaitEmpty = 2u,     // producer gave up waiting for a free stage
  kErrBadSlot = 4u,       // append: slot outside [0, num_blocks*block_size)
  kErrBadBlock = 8u,      // a block-table entry outside [0, num_blocks) was masked
  kErrDrain = 16u,        // producer gave up draining its own copies at abort
};

constexpr unsigned long long kWaitLimitNs = 1000000000ull;  // 1 s per wait

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ----------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity.  Returns false (after setting the
// error word and the CTA abort flag) if it did not complete within the limit
// or if another warp of the CTA already aborted.
// Non-blocking probe of a phase (mbarrier.test_wait never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// `limit_ns` is kWaitLimitNs everywhere except the wait self-test, which gives
// it a short limit to drive the give-up path.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort_flag,
                                                  uint32_t* err_word, uint32_t err_code,
                                                  unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > limit_ns) {
      *abort_flag = 1;
      if (err_word) atomicOr(err_word, err_code);
      return false;
    }
  }
}

// -------------------------------------------------------------------- TMA
// Hint: bring the 128-byte line holding `ptr` into L2.  No value is read, so it
// is safe before griddepcontrol.wait (a later write by the previous kernel goes
// to L2 and is what the real load after the wait returns).  `ptr` must point at
// a byte of a live allocation.
__device__ __forceinline__ void prefetch_l2(const void* ptr) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}

// L2 prefetch of the lines holding bytes [base, base + bytes) -- only lines that
// contain at least one of those bytes -- by threads t, t + nthreads, ...
__device__ __forceinline__ void prefetch_l2_span(const void* base, long long bytes, int t,
                                                 int nthreads) {
  if (bytes <= 0) return;
  const uintptr_t first = reinterpret_cast<uintptr_t>(base) & ~static_cast<uintptr_t>(127);
  const uintptr_t last = (reinterpret_cast<uintptr_t>(base) + bytes - 1) & ~static_cast<uintptr_t>(127);
  for (uintptr_t a = first + static_cast<uintptr_t>(t) * 128; a <= last;
       a += static_cast<uintptr_t>(nthreads) * 128)
    prefetch_l2(reinterpret_cast<const void*>(a));
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 3-D tiled bulk-tensor load global -> shared, completion on an mbarrier.
// Coordinates are {x (innermost, elements), y, z}.  No multicast.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Tiled bulk-tensor stores shared -> global (bulk async-group completion):
// issue, then bulk_commit_group(), then bulk_wait_group_read0() before the
// shared memory is reused or the CTA exits.  Generic-proxy writes of the
// source must be fenced with fence.proxy.async.shared::cta first.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src,
                                             int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* smem_src,
                                             int32_t x, int32_t y, int32_t z, int32_t w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], "
      "[%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// 4-D tiled bulk-tensor load (coordinates {x, y, z, w}).  No multicast.
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y, int32_t z, int32_t w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// ------------------------------------------------------------ tensor cores
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Transpose an 8x8 matrix of 16-bit values held as one mma fragment register
// per thread (thread l holds row l/4, columns 2(l%4), 2(l%4)+1).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

// Element-type traits: 16-bit storage type and its mma.sync spelling.
struct Half {
  using T = __half;
  static constexpr bool kIsBf16 = false;
};
struct BF16 {
  using T = __nv_bfloat16;
  static constexpr bool kIsBf16 = true;
};

template <typename E>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1);

template <>
__device__ __forceinline__ void mma_16816<Half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <>
__device__ __forceinline__ void mma_16816<BF16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Pack two floats into one 32-bit register of 16-bit values (lo = first).
template <typename E>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);

template <>
__device__ __forceinline__ uint32_t pack2<Half>(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <>
__device__ __forceinline__ uint32_t pack2<BF16>(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Multiply both 16-bit values of a packed pair by `a` (rounded back to E).
template <typename E>
__device__ __forceinline__ uint32_t scale_pack2(uint32_t v, float a);

template <>
__device__ __forceinline__ uint32_t scale_pack2<Half>(uint32_t v, float a) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&v));
  return pack2<Half>(f.x * a, f.y * a);
}

template <>
__device__ __forceinline__ uint32_t scale_pack2<BF16>(uint32_t v, float a) {
  const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
  return pack2<BF16>(f.x * a, f.y * a);
}

template <typename E>
__device__ __forceinline__ typename E::T from_float(float x);
template <>
__device__ __forceinline__ __half from_float<Half>(float x) {
  return __float2half_rn(x);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<BF16>(float x) {
  return __float2bfloat16_rn(x);
}

template <typename E>
__device__ __forceinline__ float to_float(typename E::T x);
template <>
__device__ __forceinline__ float to_float<Half>(__half x) {
  return __half2float(x);
}
template <>
__device__ __forceinline__ float to_float<BF16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

// Round to the 16-bit type and widen back: what one torch elementwise op on
// 16-bit tensors stores.
template <typename E>
__device__ __forceinline__ float round_to(float x) {
  return to_float<E>(from_float<E>(x));
}

// Rotary embedding of one pair (a = x[i], b = x[i + D/2]) with the rounding of
// the reference's torch elementwise form x*cos + rotate_half(x)*sin
// (hf_benchmark.py:69-85): each product rounded, the sum rounded by the caller's
// final conversion.  c_lo/s_lo are cos/sin at i, c_hi/s_hi at i + D/2.
template <typename E>
__device__ __forceinline__ void rope_pair(float a, float b, float c_lo, float s_lo, float c_hi,
                                          float s_hi, float& lo, float& hi) {
  lo = round_to<E>(a * c_lo) + round_to<E>(-b * s_lo);
  hi = round_to<E>(b * c_hi) + round_to<E>(a * s_hi);
}

// Hardware base-2 exponential (PTX ex2.approx.ftz.f32); ex2(-inf) = +0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float quad_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
  return v;
}

__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  return v;
}

// Named barrier over `count` threads (ids 1..15 are free for the kernels).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Arrive on a named barrier without waiting (the other side uses bar.sync).
__device__ __forceinline__ void named_bar_arrive(uint32_t id, uint32_t count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Load an index from an int32 or int64 array.
__device__ __forceinline__ long long load_index(const void* base, long long i, bool is64) {
  return is64 ? reinterpret_cast<const long long*>(base)[i]
              : static_cast<long long>(reinterpret_cast<const int*>(base)[i]);
}

// Byte offset of (row, byte) inside a TMA-written region whose base is
// 1024-byte aligned, for swizzle span `sw_bytes` (0 = none, 32, 64, 128):
// the 16-byte chunk index (bits 4..6) is XOR-ed with bits 7..9 of the offset.
__device__ __forceinline__ uint32_t swizzle_offset(uint32_t off, uint32_t sw_mask) {
  return off ^ (((off >> 7) & sw_mask) << 4);
}

}  // namespace b200
