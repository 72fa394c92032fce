// Self-test of the tcgen05 building blocks the prefill kernel relies on: the
// SW128 K-major and MN-major shared-memory descriptors, kind::f16 MMAs into
// TMEM with K stepping, commit to an mbarrier, and tcgen05.ld readback.
//
//   C1[128, 64]  = A[128, 64] . B[64, 64]^T      (A, B K-major)
//   C2[128, 128] = A[128, 64] . V[64, 128]        (V row-major = MN-major B)
//   C3[128, 128] = same product with A read from tensor memory (the form the
//                  prefill kernel uses for P), A written there with tcgen05.st
//
// Shared-memory operands are written by threads with the 128-byte swizzle
// pattern TMA produces.  One CTA of 128 threads; TMEM columns: C1 [0,64),
// A [64,96), C2 [128,256), C3 [256,384).
#include "../../include/b200_paged_attn.h"
#include "common.cuh"
#include "host_common.h"
#include "tcgen05.cuh"

namespace b200 {

namespace {

template <typename E>
__global__ void __launch_bounds__(128) tc_selftest_kernel(const uint16_t* a, const uint16_t* b,
                                                          const uint16_t* v, float* c1, float* c2,
                                                          float* c3, uint32_t* err) {
  __shared__ __align__(1024) uint8_t sa[128 * 128];
  __shared__ __align__(1024) uint8_t sb[64 * 128];
  __shared__ __align__(1024) uint8_t sv[2 * 64 * 128];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;

  // Operands -> shared memory, swizzled.
  {
    const uint4* src = reinterpret_cast<const uint4*>(a + tid * 64);
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<uint4*>(sa + tc::sw128_offset(tid, c)) = src[c];
  }
  if (tid < 64) {
    const uint4* src = reinterpret_cast<const uint4*>(b + tid * 64);
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<uint4*>(sb + tc::sw128_offset(tid, c)) = src[c];
    const uint4* vs = reinterpret_cast<const uint4*>(v + tid * 128);  // K row `tid`
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      *reinterpret_cast<uint4*>(sv + tc::sw128_offset(tid, c)) = vs[c];
      *reinterpret_cast<uint4*>(sv + 8192 + tc::sw128_offset(tid, c)) = vs[8 + c];
    }
  }
  if (tid == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  tc::fence_proxy_async_smem();
  if (warp == 0) {
    tc::tmem_alloc(&tmem_base, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_base;
  const uint32_t lane_addr = tbase + (static_cast<uint32_t>(warp * 32) << 16);
  {  // A row `tid` -> TMEM columns [64, 96) of lane `tid`
    uint32_t r[32];
    const uint32_t* src = reinterpret_cast<const uint32_t*>(a + tid * 64);
#pragma unroll
    for (int j = 0; j < 32; ++j) r[j] = src[j];
    tc::st32(lane_addr + 64, r);
    tc::wait_st();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();

  if (tid == 0) {
    const bool bf16 = E::kIsBf16;
    const uint32_t a0 = smem_u32(sa), b0 = smem_u32(sb), v0 = smem_u32(sv);
    const uint32_t id1 = tc::idesc_f16(128, 64, bf16, false, false);
    const uint32_t id2 = tc::idesc_f16(128, 128, bf16, false, true);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      tc::mma_f16(tbase, tc::sdesc_sw128(a0 + 32 * k, 16, 1024),
                  tc::sdesc_sw128(b0 + 32 * k, 16, 1024), id1, k > 0);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      tc::mma_f16(tbase + 128, tc::sdesc_sw128(a0 + 32 * k, 16, 1024),
                  tc::sdesc_sw128(v0 + 2048 * k, 8192, 1024), id2, k > 0);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      tc::mma_f16_tmem_a(tbase + 256, tbase + 64 + 8 * k,
                         tc::sdesc_sw128(v0 + 2048 * k, 8192, 1024), id2, k > 0);
    tc::commit(&bar);
  }
  const bool ok = mbar_wait_bounded(&bar, 0, reinterpret_cast<volatile int*>(&abort_flag), err,
                                    kErrWaitFull);
  tc::fence_after_sync();
  if (ok) {
    const int row = warp * 32 + (tid & 31);
    uint32_t r[32];
#pragma unroll
    for (int cb = 0; cb < 2; ++cb) {
      tc::ld32(lane_addr + cb * 32, r);
      tc::wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) c1[row * 64 + cb * 32 + j] = __uint_as_float(r[j]);
    }
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
      tc::ld32(lane_addr + 128 + cb * 32, r);
      tc::wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) c2[row * 128 + cb * 32 + j] = __uint_as_float(r[j]);
    }
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
      tc::ld32(lane_addr + 256 + cb * 32, r);
      tc::wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) c3[row * 128 + cb * 32 + j] = __uint_as_float(r[j]);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, 512);
}

// Bounded-wait self-test: drives the give-up path of mbar_wait_bounded -- the
// wait every kernel of this library uses on its mbarriers -- with a short
// limit instead of the kernels' 1 s.  96 threads.  Warp 0 waits on an
// mbarrier that expects one arrival; warp 1's first thread arrives only when
// `arrive` is set; warp 2 waits with a limit four times longer, so when nobody
// arrives it must leave through the CTA abort flag that warp 0 raises when it
// gives up (the path every other waiter of an aborting kernel takes).  No copy
// or MMA is in flight, so the kernel simply returns.
//   result[0] = threads of warp 0 whose wait completed,
//   result[1] = threads of warp 2 whose wait completed,
//   result[2] = %globaltimer ns warp 0's first thread spent in its wait (capped).
__global__ void __launch_bounds__(96) wait_selftest_kernel(unsigned long long limit_ns,
                                                           int arrive, uint32_t* result,
                                                           uint32_t* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  __shared__ uint32_t done[2];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    abort_flag = 0;
    done[0] = done[1] = 0;
  }
  __syncthreads();
  volatile int* abort = reinterpret_cast<volatile int*>(&abort_flag);
  if (warp == 1) {
    if (arrive && tid == 32) mbar_arrive(&bar);
  } else {
    const unsigned long long t0 = global_timer_ns();
    const bool ok = mbar_wait_bounded(&bar, 0, abort, err, kErrWaitFull,
                                      warp == 0 ? limit_ns : 4 * limit_ns);
    const unsigned long long spent = global_timer_ns() - t0;
    if (ok) atomicAdd(&done[warp == 0 ? 0 : 1], 1u);
    if (tid == 0) result[2] = static_cast<uint32_t>(spent > 0xffffffffull ? 0xffffffffull : spent);
  }
  __syncthreads();
  if (tid == 0) {
    result[0] = done[0];
    result[1] = done[1];
  }
}

}  // namespace

int launch_wait_selftest(int64_t limit_ns, int32_t arrive, uint32_t* result, uint32_t* err,
                         cudaStream_t stream) {
  if (result == nullptr || err == nullptr)
    return set_error(B200_ERR_INVALID, "result and error_word must not be NULL");
  if (limit_ns < 1000 || limit_ns > 2000000000ll)
    return set_error(B200_ERR_INVALID, "limit_ns must be within [1 us, 2 s]");
  wait_selftest_kernel<<<1, 96, 0, stream>>>(static_cast<unsigned long long>(limit_ns),
                                             arrive ? 1 : 0, result, err);
  return cuda_status(cudaGetLastError(), "wait_selftest_kernel launch");
}

int launch_tc_selftest(const void* a, const void* b, const void* v, float* c1, float* c2,
                       float* c3, int32_t dtype, uint32_t* err, cudaStream_t stream) {
  if (!a || !b || !v || !c1 || !c2 || !c3) return set_error(B200_ERR_INVALID, "null pointer");
  if (((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
        reinterpret_cast<uintptr_t>(v)) & 15) != 0)
    return set_error(B200_ERR_INVALID, "operands must be 16-byte aligned");
  const uint16_t* pa = static_cast<const uint16_t*>(a);
  const uint16_t* pb = static_cast<const uint16_t*>(b);
  const uint16_t* pv = static_cast<const uint16_t*>(v);
  if (dtype == B200_BF16)
    tc_selftest_kernel<BF16><<<1, 128, 0, stream>>>(pa, pb, pv, c1, c2, c3, err);
  else if (dtype == B200_F16)
    tc_selftest_kernel<Half><<<1, 128, 0, stream>>>(pa, pb, pv, c1, c2, c3, err);
  else
    return set_error(B200_ERR_UNSUPPORTED, "dtype must be float16 or bfloat16");
  return cuda_status(cudaGetLastError(), "tc_selftest_kernel launch");
}

}  // namespace b200
