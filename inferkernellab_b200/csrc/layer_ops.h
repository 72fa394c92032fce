// Launchers of the decoder-layer kernels (layer_ops.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

int launch_add_rmsnorm(const void* x, const void* residual, const void* weight, void* out,
                       void* residual_out, int64_t rows, int64_t cols, int64_t x_stride,
                       int64_t residual_stride, int64_t out_stride, int64_t residual_out_stride,
                       float eps, int32_t dtype, cudaStream_t stream);

int launch_silu_mul(const void* gate_up, void* out, int64_t rows, int64_t cols,
                    int64_t in_stride, int64_t out_stride, int32_t dtype, cudaStream_t stream);

}  // namespace b200
