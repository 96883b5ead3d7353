// Fused pointwise chains: out = program(inputs) over a broadcast N-d index space.
//
// Replaces the reference's generated elementwise Triton kernel
// (compiler/optimization/fusion_pointwise.py:155-192) and its launch closure
// (:224-230).  Where the reference unravels every element's flat index with a
// div/mod per dimension and gathers scalars, this kernel
//   * coalesces dimensions on the host (adjacent dims that are contiguous for
//     every operand merge), so most launches are rank 1 or 2;
//   * moves 8 elements per thread per step with 128-bit loads/stores whenever
//     the innermost dim allows it (unit or zero stride, 16-byte alignment),
//     unravelling the index once per 8 elements with multiply-shift division;
//   * runs the op chain through the register accumulator machine in
//     common.cuh, so one compiled kernel serves every chain (no codegen).
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "host_common.h"

namespace b200k {

struct PwParams {
  int32_t rank;
  int32_t n_in;
  uint32_t nunits;  // 32-bit index path
  int32_t out_dt;
  int64_t nunits64;  // 64-bit index path
  int64_t sizes[B200K_MAX_DIMS];  // per dim (innermost in units of VEC)
  FastDiv div[B200K_MAX_DIMS];
  int64_t strides[B200K_MAX_INPUTS][B200K_MAX_DIMS];  // elements; innermost pre-multiplied by VEC
  int64_t inner_stride[B200K_MAX_INPUTS];  // element stride of the innermost dim (0 or 1 on the vector path)
  const void* in[B200K_MAX_INPUTS];
  int32_t dt[B200K_MAX_INPUTS];
  void* out;
  B200kProgram prog;
};

template <int VEC, bool I64>
__global__ void __launch_bounds__(256) pointwise_kernel(const __grid_constant__ PwParams p) {
  const int64_t total = I64 ? p.nunits64 : static_cast<int64_t>(p.nunits);
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < total; u += step) {
    // Unravel the unit index (innermost dim last).
    int64_t idx[B200K_MAX_DIMS];
    if (I64) {
      int64_t rem = u;
#pragma unroll
      for (int d = B200K_MAX_DIMS - 1; d >= 1; --d) {
        if (d < p.rank) {
          idx[d] = rem % p.sizes[d];
          rem /= p.sizes[d];
        }
      }
      idx[0] = rem;
    } else {
      uint32_t rem = static_cast<uint32_t>(u);
#pragma unroll
      for (int d = B200K_MAX_DIMS - 1; d >= 1; --d) {
        if (d < p.rank) {
          const uint32_t q = fdiv(rem, p.div[d]);
          idx[d] = rem - q * p.div[d].d;
          rem = q;
        }
      }
      idx[0] = rem;
    }

    float r[kSlots][VEC];
    float acc[VEC];
#pragma unroll
    for (int i = 0; i < B200K_MAX_INPUTS; ++i) {
      if (i < p.n_in) {
        int64_t off = 0;
#pragma unroll
        for (int d = 0; d < B200K_MAX_DIMS; ++d)
          if (d < p.rank) off += idx[d] * p.strides[i][d];
        if (VEC == 8) {
          float v[8];
          if (p.inner_stride[i] == 1) {
            load_vec8(p.in[i], off, p.dt[i], v);
          } else {
            const float s = load_scalar(p.in[i], off, p.dt[i]);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = s;
          }
#pragma unroll
          for (int j = 0; j < VEC; ++j) r[i][j] = v[j];
        } else {
#pragma unroll
          for (int j = 0; j < VEC; ++j) r[i][j] = load_scalar(p.in[i], off, p.dt[i]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < VEC; ++j) acc[j] = r[0][j];

    run_program<VEC>(p.prog, r, acc);

    const int64_t out_off = u * VEC;
    if (VEC == 8) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = acc[j];
      store_vec8(p.out, out_off, p.out_dt, v);
    } else {
#pragma unroll
      for (int j = 0; j < VEC; ++j) store_scalar(p.out, out_off + j, p.out_dt, acc[j]);
    }
  }
}

namespace {

struct Dim {
  int64_t size;
  int64_t stride[B200K_MAX_INPUTS + 1];  // inputs..., output last
};

template <int VEC, bool I64>
int launch_grid_stride(const PwParams& p, int64_t units, cudaStream_t stream) {
  auto kernel = pointwise_kernel<VEC, I64>;
  const int sms = device_sm_count();
  if (sms <= 0) return B200K_ERR_DEVICE;
  static int per_sm = 0;  // resident CTAs per SM for this instantiation (device-independent here)
  if (per_sm == 0) {
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kernel, 256, 0) != cudaSuccess) return B200K_ERR_LAUNCH;
    per_sm = std::max(v, 1);
  }
  const int64_t want = (units + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sms) * per_sm;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min(want, cap)));
  kernel<<<grid, 256, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? B200K_OK : B200K_ERR_LAUNCH;
}

}  // namespace

}  // namespace b200k

using namespace b200k;

extern "C" int b200k_pointwise(const B200kPointwiseArgs* a, void* stream_) {
  if (!a) return B200K_ERR_ARG;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (a->rank < 0 || a->rank > B200K_MAX_DIMS) return B200K_ERR_SHAPE;
  if (a->n_inputs < 1 || a->n_inputs > B200K_MAX_INPUTS) return B200K_ERR_ARG;
  if (!valid_float_dtype(a->out_dtype)) return B200K_ERR_UNSUPPORTED;
  int rc = validate_program(a->program, a->n_inputs);
  if (rc != B200K_OK) return rc;
  for (int i = 0; i < a->n_inputs; ++i)
    if (!valid_dtype(a->inputs[i].dtype)) return B200K_ERR_UNSUPPORTED;
  int64_t numel = 1;
  for (int d = 0; d < a->rank; ++d) {
    if (a->sizes[d] < 0) return B200K_ERR_SHAPE;
    numel *= a->sizes[d];
  }
  if (numel == 0) return B200K_OK;  // empty tensors may carry null pointers
  if (!a->out) return B200K_ERR_ARG;
  for (int i = 0; i < a->n_inputs; ++i)
    if (!a->inputs[i].ptr) return B200K_ERR_ARG;

  // Collect non-trivial dims (outermost first); output is contiguous.
  const int nin = a->n_inputs;
  Dim dims[B200K_MAX_DIMS];
  int nd = 0;
  {
    int64_t out_stride = numel;
    for (int d = 0; d < a->rank; ++d) {
      out_stride /= a->sizes[d];
      if (a->sizes[d] == 1) continue;
      Dim& x = dims[nd++];
      x.size = a->sizes[d];
      for (int i = 0; i < nin; ++i) x.stride[i] = a->inputs[i].strides[d];
      x.stride[nin] = out_stride;
    }
  }
  if (nd == 0) {  // a single element
    nd = 1;
    dims[0].size = 1;
    for (int i = 0; i <= nin; ++i) dims[0].stride[i] = 1;
  }
  // Merge dim d into d+1 (the inner one) when every operand is contiguous across them.
  Dim merged[B200K_MAX_DIMS];
  int nm = 0;
  merged[nm++] = dims[nd - 1];
  for (int d = nd - 2; d >= 0; --d) {
    Dim& inner = merged[nm - 1];
    bool ok = true;
    for (int i = 0; i <= nin; ++i)
      if (dims[d].stride[i] != inner.stride[i] * inner.size) ok = false;
    if (ok) {
      inner.size *= dims[d].size;
    } else {
      merged[nm++] = dims[d];
    }
  }
  // merged[] is innermost-first; flip to outermost-first.
  std::reverse(merged, merged + nm);

  PwParams p;
  std::memset(&p, 0, sizeof(p));
  p.rank = nm;
  p.n_in = nin;
  p.out = a->out;
  p.out_dt = a->out_dtype;
  p.prog = a->program;
  for (int i = 0; i < nin; ++i) {
    p.in[i] = a->inputs[i].ptr;
    p.dt[i] = a->inputs[i].dtype;
  }

  // Vector path: innermost size % 8 == 0; each input's innermost stride is 0 or
  // 1; unit-stride inputs keep 8-element (and 16-byte) alignment at every
  // vector start; the output pointer is 16-byte aligned.
  const Dim& in_most = merged[nm - 1];
  bool vec = (in_most.size % 8 == 0) && aligned16(a->out);
  for (int i = 0; i < nin && vec; ++i) {
    const int64_t s = in_most.stride[i];
    if (s != 0 && s != 1) vec = false;
    if (s == 1) {
      if (!aligned16(p.in[i])) vec = false;
      for (int d = 0; d < nm - 1; ++d)
        if (merged[d].stride[i] % 8 != 0) vec = false;
    }
  }
  const int VEC = vec ? 8 : 1;
  for (int d = 0; d < nm; ++d) {
    const bool inner = (d == nm - 1);
    p.sizes[d] = inner ? merged[d].size / VEC : merged[d].size;
    for (int i = 0; i < nin; ++i) p.strides[i][d] = inner ? merged[d].stride[i] * VEC : merged[d].stride[i];
  }
  for (int i = 0; i < nin; ++i) p.inner_stride[i] = in_most.stride[i];
  const int64_t units = numel / VEC;
  const bool i64 = units >= (int64_t(1) << 31);
  if (i64) {
    p.nunits64 = units;
  } else {
    p.nunits = static_cast<uint32_t>(units);
    for (int d = 0; d < nm; ++d) p.div[d] = make_fastdiv(static_cast<uint32_t>(p.sizes[d]));
  }

  if (vec) return i64 ? launch_grid_stride<8, true>(p, units, stream) : launch_grid_stride<8, false>(p, units, stream);
  return i64 ? launch_grid_stride<1, true>(p, units, stream) : launch_grid_stride<1, false>(p, units, stream);
}
