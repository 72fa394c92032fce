// Decoder-layer kernels around the paged attention call: residual add fused
// with RMSNorm, and the SiLU-gated product of the MLP.
//
// They replace the chains of small torch elementwise/reduction launches that
// a Transformers Llama layer issues around attention (LlamaRMSNorm: cast, pow,
// mean, add, rsqrt, mul, cast, mul; LlamaMLP: silu, mul; the residual adds)
// with one launch each, computing the same roundings:
//   add_rmsnorm: s   = rnd(x + residual)                (bf16/f16 add)
//                var = mean(float(s)^2)                  (float)
//                out = rnd(w * rnd(float(s) * rsqrt(var + eps)))
//   silu_mul:    out = rnd(rnd(g / (1 + exp(-g))) * u)   (g, u from one fused
//                                                          gate|up projection)
// rnd() rounds to the 16-bit type.  The only difference from the torch chain
// is the summation order inside the mean.
#include "../../include/b200_paged_attn.h"
#include "common.cuh"
#include "host_common.h"
#include "layer_ops.h"

namespace b200 {

namespace {

// 8 x 16-bit elements = one 16-byte access.
struct alignas(16) Vec8 {
  uint16_t h[8];
};

template <typename E>
__device__ __forceinline__ float lane(const Vec8& v, int i) {
  typename E::T t;
  memcpy(&t, &v.h[i], 2);
  return to_float<E>(t);
}

template <typename E>
__device__ __forceinline__ void set_lane(Vec8& v, int i, float x) {
  typename E::T t = from_float<E>(x);
  memcpy(&v.h[i], &t, 2);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lid = threadIdx.x & 31;
  if (lid == 0) red[warp] = v;
  __syncthreads();
  const int nwarps = blockDim.x >> 5;
  float t = lid < nwarps ? red[lid] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

struct NormParams {
  const uint8_t* x;         // may be null: no residual add
  const uint8_t* residual;  // [rows, cols]
  const uint8_t* weight;    // [cols]
  uint8_t* out;
  uint8_t* residual_out;    // may equal residual; null when x is null
  long long rows, cols, x_stride, r_stride, o_stride, ro_stride;
  float eps;
};

// One CTA per row.  VEC: 16-byte vectors (all row pointers and cols aligned to
// 8 elements) or scalar elements.
template <typename E, bool VEC>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(const NormParams p) {
  using T = typename E::T;
  __shared__ float red[32];
  const long long row = blockIdx.x;
  const T* r = reinterpret_cast<const T*>(p.residual) + row * p.r_stride;
  const T* x = p.x ? reinterpret_cast<const T*>(p.x) + row * p.x_stride : nullptr;
  T* ro = p.residual_out ? reinterpret_cast<T*>(p.residual_out) + row * p.ro_stride : nullptr;
  // The summed row is read back from residual_out (or residual when there is
  // no add) in the second pass; each thread reads only what it wrote itself.
  const T* s_src = ro ? ro : r;
  T* o = reinterpret_cast<T*>(p.out) + row * p.o_stride;
  const T* w = reinterpret_cast<const T*>(p.weight);
  float ss = 0.f;
  if (VEC) {
    const long long nv = p.cols / 8;
    for (long long c = threadIdx.x; c < nv; c += blockDim.x) {
      Vec8 rv = reinterpret_cast<const Vec8*>(r)[c];
      if (x) {
        const Vec8 xv = reinterpret_cast<const Vec8*>(x)[c];
#pragma unroll
        for (int i = 0; i < 8; ++i) set_lane<E>(rv, i, lane<E>(xv, i) + lane<E>(rv, i));
        reinterpret_cast<Vec8*>(ro)[c] = rv;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float s = lane<E>(rv, i);
        ss += s * s;
      }
    }
  } else {
    for (long long c = threadIdx.x; c < p.cols; c += blockDim.x) {
      float s = to_float<E>(r[c]);
      if (x) {
        s = round_to<E>(to_float<E>(x[c]) + s);
        ro[c] = from_float<E>(s);
      }
      ss += s * s;
    }
  }
  const float total = block_sum(ss, red);
  const float inv = rsqrtf(total * (1.0f / static_cast<float>(p.cols)) + p.eps);
  if (VEC) {
    const long long nv = p.cols / 8;
    for (long long c = threadIdx.x; c < nv; c += blockDim.x) {
      const Vec8 sv = reinterpret_cast<const Vec8*>(s_src)[c];
      const Vec8 wv = reinterpret_cast<const Vec8*>(w)[c];
      Vec8 ov;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        set_lane<E>(ov, i, lane<E>(wv, i) * round_to<E>(lane<E>(sv, i) * inv));
      reinterpret_cast<Vec8*>(o)[c] = ov;
    }
  } else {
    for (long long c = threadIdx.x; c < p.cols; c += blockDim.x) {
      const float s = to_float<E>(s_src[c]);
      o[c] = from_float<E>(to_float<E>(w[c]) * round_to<E>(s * inv));
    }
  }
}

struct SiluParams {
  const uint8_t* gate_up;  // [rows, 2*cols]: gate | up
  uint8_t* out;            // [rows, cols]
  long long rows, cols, in_stride, out_stride;
};

template <typename E>
__device__ __forceinline__ float silu_mul1(float g, float u) {
  return round_to<E>(g / (1.0f + expf(-g))) * u;
}

template <typename E, bool VEC>
__global__ void __launch_bounds__(256) silu_mul_kernel(const SiluParams p) {
  using T = typename E::T;
  const long long per_row = VEC ? p.cols / 8 : p.cols;
  const long long total = p.rows * per_row;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = idx / per_row;
    const long long c = idx - row * per_row;
    const T* g = reinterpret_cast<const T*>(p.gate_up) + row * p.in_stride;
    const T* u = g + p.cols;
    T* o = reinterpret_cast<T*>(p.out) + row * p.out_stride;
    if (VEC) {
      const Vec8 gv = reinterpret_cast<const Vec8*>(g)[c];
      const Vec8 uv = reinterpret_cast<const Vec8*>(u)[c];
      Vec8 ov;
#pragma unroll
      for (int i = 0; i < 8; ++i) set_lane<E>(ov, i, silu_mul1<E>(lane<E>(gv, i), lane<E>(uv, i)));
      reinterpret_cast<Vec8*>(o)[c] = ov;
    } else {
      o[c] = from_float<E>(silu_mul1<E>(to_float<E>(g[c]), to_float<E>(u[c])));
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int launch_add_rmsnorm(const void* x, const void* residual, const void* weight, void* out,
                       void* residual_out, int64_t rows, int64_t cols, int64_t x_stride,
                       int64_t residual_stride, int64_t out_stride, int64_t residual_out_stride,
                       float eps, int32_t dtype, cudaStream_t stream) {
  if (dtype != B200_F16 && dtype != B200_BF16)
    return set_error(B200_ERR_UNSUPPORTED, "dtype must be float16 or bfloat16");
  if (rows < 0 || cols <= 0) return set_error(B200_ERR_INVALID, "rows/cols out of range");
  if (!residual || !weight || !out || (x && !residual_out))
    return set_error(B200_ERR_INVALID, "null tensor pointer");
  if (rows > 0x7fffffffLL) return set_error(B200_ERR_INVALID, "too many rows");
  if (rows == 0) return B200_OK;
  NormParams p;
  p.x = static_cast<const uint8_t*>(x);
  p.residual = static_cast<const uint8_t*>(residual);
  p.weight = static_cast<const uint8_t*>(weight);
  p.out = static_cast<uint8_t*>(out);
  p.residual_out = x ? static_cast<uint8_t*>(residual_out) : nullptr;
  p.rows = rows;
  p.cols = cols;
  p.x_stride = x_stride;
  p.r_stride = residual_stride;
  p.o_stride = out_stride;
  p.ro_stride = residual_out_stride;
  p.eps = eps;
  bool vec = cols % 8 == 0 && residual_stride % 8 == 0 && out_stride % 8 == 0 &&
             aligned16(residual) && aligned16(weight) && aligned16(out);
  if (x) vec = vec && x_stride % 8 == 0 && residual_out_stride % 8 == 0 && aligned16(x) &&
               aligned16(residual_out);
  int threads = 256;
  const long long per_thread_units = vec ? cols / 8 : cols;
  if (per_thread_units < 256) threads = per_thread_units <= 32 ? 32 : ((per_thread_units + 31) / 32) * 32;
  const dim3 grid(static_cast<unsigned>(rows));
  if (dtype == B200_BF16) {
    if (vec)
      add_rmsnorm_kernel<BF16, true><<<grid, threads, 0, stream>>>(p);
    else
      add_rmsnorm_kernel<BF16, false><<<grid, threads, 0, stream>>>(p);
  } else {
    if (vec)
      add_rmsnorm_kernel<Half, true><<<grid, threads, 0, stream>>>(p);
    else
      add_rmsnorm_kernel<Half, false><<<grid, threads, 0, stream>>>(p);
  }
  return cuda_status(cudaGetLastError(), "add_rmsnorm_kernel launch");
}

int launch_silu_mul(const void* gate_up, void* out, int64_t rows, int64_t cols,
                    int64_t in_stride, int64_t out_stride, int32_t dtype, cudaStream_t stream) {
  if (dtype != B200_F16 && dtype != B200_BF16)
    return set_error(B200_ERR_UNSUPPORTED, "dtype must be float16 or bfloat16");
  if (rows < 0 || cols <= 0 || in_stride < 2 * cols)
    return set_error(B200_ERR_INVALID, "rows/cols/stride out of range");
  if (!gate_up || !out) return set_error(B200_ERR_INVALID, "null tensor pointer");
  if (rows == 0) return B200_OK;
  SiluParams p;
  p.gate_up = static_cast<const uint8_t*>(gate_up);
  p.out = static_cast<uint8_t*>(out);
  p.rows = rows;
  p.cols = cols;
  p.in_stride = in_stride;
  p.out_stride = out_stride;
  const bool vec = cols % 8 == 0 && in_stride % 8 == 0 && out_stride % 8 == 0 &&
                   aligned16(gate_up) && aligned16(out);
  const long long work = rows * (vec ? cols / 8 : cols);
  long long blocks = (work + 255) / 256;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  const unsigned b = static_cast<unsigned>(blocks);
  if (dtype == B200_BF16) {
    if (vec)
      silu_mul_kernel<BF16, true><<<b, 256, 0, stream>>>(p);
    else
      silu_mul_kernel<BF16, false><<<b, 256, 0, stream>>>(p);
  } else {
    if (vec)
      silu_mul_kernel<Half, true><<<b, 256, 0, stream>>>(p);
    else
      silu_mul_kernel<Half, false><<<b, 256, 0, stream>>>(p);
  }
  return cuda_status(cudaGetLastError(), "silu_mul_kernel launch");
}

}  // namespace b200
