// Shared between the generic row kernels (rowreduce.cu) and the 16-bit
// specialised ones (rowreduce16.cu).
#pragma once
#include <cstdint>

#include <cuda_runtime.h>

namespace b200k {

struct RowParams {
  int64_t rows, cols;
  const void* x;
  int64_t x_stride;
  const void* w;
  const void* b;
  void* out;
  int64_t out_stride;
  float* mean_out;
  float* rstd_out;
  float eps;
  int32_t x_dt, w_dt, b_dt, out_dt, flags, log_softmax;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Row kinds of the 16-bit kernels.
enum Row16Kind { R16_RMSNORM = 0, R16_LAYERNORM = 1, R16_SWIGLU = 2, R16_SOFTMAX = 3, R16_LOG_SOFTMAX = 4 };

// Launches the 16-bit specialised kernel for `kind` when the call qualifies
// (x, out, weight and bias all of one 16-bit type, rows 16-byte aligned,
// flags the kernel implements); returns -1 when it does not, so the caller
// runs the generic kernel, else a B200K_* status.
int launch_row16(Row16Kind kind, const RowParams& p, cudaStream_t st);

}  // namespace b200k
