// Fused pointwise chains: out = program(inputs) over a broadcast N-d index space.
//
// Replaces the reference's generated elementwise Triton kernel
// (compiler/optimization/fusion_pointwise.py:132-169) and its launch closure
// (:189-210).  Where the reference unravels every element's flat index with a
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
#include "pointwise_jit.h"

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

// Vector path for the common launches: merged rank 1 or 2, at most four
// inputs and four program slots, 32-bit unit indices, unit-stride inputs of
// bf16, f16 or f32.  The
// generic kernel above serves every launch with one thread-unit of work per
// loop step and index arithmetic over all six dims and eight input slots
// (~400 instructions per 8 elements, latency-bound at 2 warps per
// scheduler: a bf16 add moved ~1 TB/s).  Here the index arithmetic is only
// that of RANK dims and NIN inputs, and each thread issues the 16-byte loads
// of U units before it runs the program on the first, so U x NIN loads per
// thread are in flight.
constexpr int kFastSlots = 4;  // programs of at most four slots (the host checks)
// W: 16-byte words of one 8-element unit of every unit-stride input (1: all
// 16-bit, 2: all f32).
template <int RANK, int NIN, int U, int W>
__global__ void __launch_bounds__(256) pointwise_fast_kernel(const __grid_constant__ PwParams p) {
  const uint32_t total = p.nunits;
  const uint32_t step = gridDim.x * blockDim.x * U;
  for (uint32_t base = blockIdx.x * blockDim.x * U + threadIdx.x; base < total; base += step) {
    uint4 raw[U][NIN][W];
    // Element offset of input i at unit u (recomputed where needed rather
    // than kept per unit: registers go to the loads in flight).
    auto offset = [&](uint32_t u, int i) -> int64_t {
      uint32_t i0 = 0, i1 = u;
      if (RANK == 2) {
        i0 = fdiv(u, p.div[1]);
        i1 = u - i0 * p.div[1].d;
      }
      return RANK == 2 ? static_cast<int64_t>(i0) * p.strides[i][0] + static_cast<int64_t>(i1) * p.strides[i][1]
                       : static_cast<int64_t>(i1) * p.strides[i][0];
    };
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const uint32_t u = base + k * blockDim.x;
      if (u >= total) break;
#pragma unroll
      for (int i = 0; i < NIN; ++i) {
        if (p.inner_stride[i] == 1) {
          const uint4* q =
              reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(p.in[i]) + offset(u, i) * (2 * W));
#pragma unroll
          for (int w = 0; w < W; ++w) raw[k][i][w] = __ldg(q + w);
        }
      }
    }
    // One copy of the program loop (the interpreter is large): unit k's
    // operands are always in slot 0 of raw, shifted down after each unit.
#pragma unroll 1
    for (int k = 0; k < U; ++k) {
      const uint32_t u = base + k * blockDim.x;
      if (u >= total) break;
      float r[kFastSlots][8];
      float acc[8];
#pragma unroll
      for (int i = 0; i < NIN; ++i) {
        if (p.inner_stride[i] == 1) {
          if constexpr (W == 2) {
            const float* f = reinterpret_cast<const float*>(&raw[0][i][0]);
#pragma unroll
            for (int j = 0; j < 8; ++j) r[i][j] = f[j];
          } else {
            const uint32_t w[4] = {raw[0][i][0].x, raw[0][i][0].y, raw[0][i][0].z, raw[0][i][0].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f = p.dt[i] == B200K_BF16 ? __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]))
                                                     : __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
              r[i][2 * j] = f.x;
              r[i][2 * j + 1] = f.y;
            }
          }
        } else {
          const float sc = load_scalar(p.in[i], offset(u, i), p.dt[i]);
#pragma unroll
          for (int j = 0; j < 8; ++j) r[i][j] = sc;
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = r[0][j];
      run_program<8, kFastSlots>(p.prog, r, acc);
      store_vec8(p.out, static_cast<int64_t>(u) * 8, p.out_dt, acc);
#pragma unroll
      for (int kk = 0; kk + 1 < U; ++kk) {
#pragma unroll
        for (int i = 0; i < NIN; ++i) {
#pragma unroll
          for (int w = 0; w < W; ++w) raw[kk][i][w] = raw[kk + 1][i][w];
        }
      }
    }
  }
}

namespace {

template <int RANK, int NIN, int W>
int launch_fast(const PwParams& p, int64_t units, cudaStream_t stream) {
  constexpr int U = NIN * W <= 2 ? 4 : 2;  // units in flight per thread (more spill past ~128 registers)
  auto kernel = pointwise_fast_kernel<RANK, NIN, U, W>;
  const int sms = device_sm_count();
  if (sms <= 0) return B200K_ERR_DEVICE;
  static int per_sm = 0;  // resident CTAs per SM for this instantiation
  if (per_sm == 0) {
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kernel, 256, 0) != cudaSuccess) return B200K_ERR_LAUNCH;
    per_sm = std::max(v, 1);
  }
  const int64_t want = (units + 256 * U - 1) / (256 * U);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, static_cast<int64_t>(sms) * per_sm)));
  kernel<<<grid, 256, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? B200K_OK : B200K_ERR_LAUNCH;
}

template <int RANK, int W>
int launch_fast_nin(int nin, const PwParams& p, int64_t units, cudaStream_t stream) {
  switch (nin) {
    case 1: return launch_fast<RANK, 1, W>(p, units, stream);
    case 2: return launch_fast<RANK, 2, W>(p, units, stream);
    case 3: return launch_fast<RANK, 3, W>(p, units, stream);
    case 4: return launch_fast<RANK, 4, W>(p, units, stream);
    default: return B200K_ERR_UNSUPPORTED;
  }
}

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

  // Generated straight-line kernel of this program (pointwise_jit.cu) when
  // the launch is in its scope; the interpreter kernels below otherwise.
  if (vec && !i64 && nm <= 2) {
    PwJitLaunch L;
    std::memset(&L, 0, sizeof(L));
    L.rank = nm;
    L.nin = nin;
    L.units = units;
    L.inner_units = nm == 2 ? p.sizes[1] : 0;
    for (int i = 0; i < nin; ++i) {
      L.stride0[i] = p.strides[i][0];
      L.stride1[i] = nm == 2 ? p.strides[i][1] : 0;
      L.inner_stride[i] = p.inner_stride[i];
    }
    const int jrc = pointwise_jit_launch(a, L, stream);
    if (jrc != B200K_ERR_UNSUPPORTED) return jrc;
  }
  if (vec && !i64 && nm <= 2 && nin <= 4 && slots_used(a->program, nin) <= kFastSlots) {
    int w = 0;  // 16-byte words per unit, the same for every unit-stride input
    bool fast = true;
    for (int i = 0; i < nin; ++i) {
      if (p.inner_stride[i] != 1) continue;
      const int wi = p.dt[i] == B200K_F32 ? 2 : (p.dt[i] == B200K_BF16 || p.dt[i] == B200K_F16) ? 1 : 0;
      if (wi == 0 || (w != 0 && wi != w)) fast = false;
      w = wi;
    }
    if (fast && w == 1)
      return nm == 2 ? launch_fast_nin<2, 1>(nin, p, units, stream) : launch_fast_nin<1, 1>(nin, p, units, stream);
    if (fast && w == 2)
      return nm == 2 ? launch_fast_nin<2, 2>(nin, p, units, stream) : launch_fast_nin<1, 2>(nin, p, units, stream);
  }
  if (vec) return i64 ? launch_grid_stride<8, true>(p, units, stream) : launch_grid_stride<8, false>(p, units, stream);
  return i64 ? launch_grid_stride<1, true>(p, units, stream) : launch_grid_stride<1, false>(p, units, stream);
}
