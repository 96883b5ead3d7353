// Launch description shared by pointwise.cu (which merges dims and checks
// vector alignment) and pointwise_jit.cu (which generates, compiles, caches
// and launches a kernel per program).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "b200k.h"

namespace b200k {

struct PwJitLaunch {
  int rank;  // merged rank: 1 or 2
  int nin;
  int64_t units;        // 8-element units over the whole output
  int64_t inner_units;  // units per row of the inner dim (rank 2)
  int64_t stride0[B200K_MAX_INPUTS];  // rank 1: elements per unit; rank 2: elements per row
  int64_t stride1[B200K_MAX_INPUTS];  // rank 2: elements per unit of the inner dim
  int64_t inner_stride[B200K_MAX_INPUTS];  // element stride of the innermost dim (0 or 1)
};

// Launches the generated kernel of `a`'s program on `stream`.  Returns
// B200K_ERR_UNSUPPORTED, having launched nothing, when the launch is outside
// the generated kernels' scope or the kernel cannot be compiled or loaded.
int pointwise_jit_launch(const B200kPointwiseArgs* a, const PwJitLaunch& launch, cudaStream_t stream);

}  // namespace b200k
