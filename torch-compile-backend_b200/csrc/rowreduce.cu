// Row-reduction groups: RMSNorm, LayerNorm, RMSNorm->split->SiLU(gate)*up and
// softmax / log-softmax over the last dim.
//
// No reference counterpart: the reference backend has no reduction entries in
// POINTWISE_OPS (compiler/optimization/fusion_pointwise.py:12-30) and leaves
// pow/mean/native_layer_norm/_softmax to ATen, fusing only the pointwise
// fragments between them.  Each kernel here reads its row once from HBM into
// registers (128-bit loads), reduces with warp shuffles (+ shared memory across
// the warps of a row), and writes the result once: the algorithmic minimum of
// one read and one write.
//
// Layout: TPR threads per row, every thread holds up to VPT vectors of VEC
// elements of its row at vector indices lane + k*TPR.  A CTA holds
// max(1, 256/TPR) rows.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "host_common.h"
#include "rowreduce.cuh"

namespace b200k {

constexpr int kVPT = 4;  // vectors per thread


// Sum (IS_MAX=false) or max over the TPR threads of a row.  Every thread of the
// CTA must call it (it may synchronise the CTA).
template <int TPR, bool IS_MAX>
__device__ __forceinline__ float row_allreduce(float v, float* sm) {
  v = IS_MAX ? warp_max(v) : warp_sum(v);
  if constexpr (TPR > 32) {
    const int wid = threadIdx.x >> 5;
    const int first = (threadIdx.x / TPR) * (TPR / 32);
    if ((threadIdx.x & 31) == 0) sm[wid] = v;
    __syncthreads();
    float t = sm[first];
#pragma unroll
    for (int k = 1; k < TPR / 32; ++k) t = IS_MAX ? fmaxf(t, sm[first + k]) : t + sm[first + k];
    __syncthreads();
    v = t;
  }
  return v;
}

// A vector of VEC row elements as held in registers between the reduction
// and the output pass: 16-bit inputs stay packed (one 16-byte register
// quad per 8 elements), which halves the registers a row needs and doubles
// the resident rows per SM.
template <int VEC, bool X16>
struct RowFrag {
  float v[VEC];
  __device__ __forceinline__ void load(const void* base, int64_t off, int dt) {
    if constexpr (VEC == 8) {
      load_vec8(base, off, dt, v);
    } else {
#pragma unroll
      for (int j = 0; j < VEC; ++j) v[j] = load_scalar(base, off + j, dt);
    }
  }
  __device__ __forceinline__ float get(int j, int) const { return v[j]; }
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int j = 0; j < VEC; ++j) v[j] = 0.0f;
  }
};

template <>
struct RowFrag<8, true> {
  uint4 u;
  __device__ __forceinline__ void load(const void* base, int64_t off, int) {
    u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(base) + off));
  }
  __device__ __forceinline__ float get(int j, int dt) const {
    const uint32_t w = (j < 2) ? u.x : (j < 4) ? u.y : (j < 6) ? u.z : u.w;
    const uint32_t h = (j & 1) ? (w >> 16) : (w & 0xffffu);
    if (dt == B200K_BF16) return __uint_as_float(h << 16);
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
  }
  __device__ __forceinline__ void zero() { u = make_uint4(0, 0, 0, 0); }
};

template <int VEC>
__device__ __forceinline__ void load_row_vec(const void* base, int64_t off, int dt, float (&v)[VEC]) {
  if constexpr (VEC == 8) {
    load_vec8(base, off, dt, v);
  } else {
#pragma unroll
    for (int j = 0; j < VEC; ++j) v[j] = load_scalar(base, off + j, dt);
  }
}
template <int VEC>
__device__ __forceinline__ void store_row_vec(void* base, int64_t off, int dt, const float (&v)[VEC]) {
  if constexpr (VEC == 8) {
    store_vec8(base, off, dt, v);
  } else {
#pragma unroll
    for (int j = 0; j < VEC; ++j) store_scalar(base, off + j, dt, v[j]);
  }
}

__device__ __forceinline__ float round_to(float x, int dt) {
  if (dt == B200K_BF16) return round_bf16(x);
  if (dt == B200K_F16) return round_f16(x);
  return x;
}

__host__ __device__ constexpr int threads_for(int tpr) { return tpr >= 256 ? tpr : 256; }

// ---------------------------------------------------------------------------
// RMSNorm / LayerNorm:  y = affine(normalise(x))
// ---------------------------------------------------------------------------
template <int TPR, int VEC, bool LAYER, bool X16>
__global__ void __launch_bounds__(threads_for(TPR)) rownorm_kernel(const __grid_constant__ RowParams p) {
  constexpr int RPB = threads_for(TPR) / TPR;
  __shared__ float sm[threads_for(TPR) / 32];
  const int lane = threadIdx.x % TPR;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * RPB + threadIdx.x / TPR;
  const bool valid_row = row < p.rows;
  const int64_t nvec = p.cols / VEC;
  const int dt = p.x_dt;

  RowFrag<VEC, X16> f[kVPT];
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < kVPT; ++k) {
    const int64_t vi = lane + k * TPR;
    if (valid_row && vi < nvec) {
      f[k].load(p.x, row * p.x_stride + vi * VEC, dt);
    } else {
      f[k].zero();
    }
  }
#pragma unroll
  for (int k = 0; k < kVPT; ++k) {
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float x = f[k].get(j, dt);
      s += LAYER ? x : x * x;
    }
  }
  s = row_allreduce<TPR, false>(s, sm);
  const float inv_n = 1.0f / static_cast<float>(p.cols);
  float mean = 0.0f, rstd;
  if (LAYER) {
    mean = s * inv_n;
    float q = 0.0f;
#pragma unroll
    for (int k = 0; k < kVPT; ++k) {
      const int64_t vi = lane + k * TPR;
      if (valid_row && vi < nvec) {
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const float d = f[k].get(j, dt) - mean;
          q += d * d;
        }
      }
    }
    q = row_allreduce<TPR, false>(q, sm);
    rstd = rsqrtf(q * inv_n + p.eps);
  } else {
    rstd = rsqrtf(s * inv_n + p.eps);
  }
  if (!valid_row) return;
  if (lane == 0) {
    if (p.mean_out) p.mean_out[row] = mean;
    if (p.rstd_out) p.rstd_out[row] = rstd;
  }
  const bool round_normed = (p.flags & B200K_ROWF_ROUND_NORMED) != 0;
  const bool plus_one = (p.flags & B200K_ROWF_WEIGHT_PLUS_ONE) != 0;
#pragma unroll
  for (int k = 0; k < kVPT; ++k) {
    const int64_t vi = lane + k * TPR;
    if (vi < nvec) {
      float wv[VEC], bv[VEC], y[VEC];
      if (p.w) {
        load_row_vec<VEC>(p.w, vi * VEC, p.w_dt, wv);
      } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j) wv[j] = 1.0f;
      }
      if (LAYER && p.b) {
        load_row_vec<VEC>(p.b, vi * VEC, p.b_dt, bv);
      } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j) bv[j] = 0.0f;
      }
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        float n = (f[k].get(j, dt) - mean) * rstd;
        if (round_normed) n = round_to(n, dt);
        const float w = plus_one ? 1.0f + wv[j] : wv[j];
        y[j] = LAYER ? n * w + bv[j] : w * n;
      }
      store_row_vec<VEC>(p.out, row * p.out_stride + vi * VEC, p.out_dt, y);
    }
  }
}

// ---------------------------------------------------------------------------
// RMSNorm over the full row, then out[j] = silu(y[j]) * y[j + cols/2].
// ---------------------------------------------------------------------------
template <int TPR, int VEC, bool X16>
__global__ void __launch_bounds__(threads_for(TPR)) rmsnorm_swiglu_kernel(const __grid_constant__ RowParams p) {
  constexpr int RPB = threads_for(TPR) / TPR;
  __shared__ float sm[threads_for(TPR) / 32];
  const int lane = threadIdx.x % TPR;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * RPB + threadIdx.x / TPR;
  const bool valid_row = row < p.rows;
  const int64_t half = p.cols / 2;
  const int64_t nvec = half / VEC;
  const int dt = p.x_dt;

  RowFrag<VEC, X16> g[kVPT], u[kVPT];
#pragma unroll
  for (int k = 0; k < kVPT; ++k) {
    const int64_t vi = lane + k * TPR;
    if (valid_row && vi < nvec) {
      g[k].load(p.x, row * p.x_stride + vi * VEC, dt);
      u[k].load(p.x, row * p.x_stride + half + vi * VEC, dt);
    } else {
      g[k].zero();
      u[k].zero();
    }
  }
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < kVPT; ++k) {
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float a = g[k].get(j, dt), b = u[k].get(j, dt);
      s += a * a + b * b;
    }
  }
  s = row_allreduce<TPR, false>(s, sm);
  const float rstd = rsqrtf(s / static_cast<float>(p.cols) + p.eps);
  if (!valid_row) return;
  if (lane == 0 && p.rstd_out) p.rstd_out[row] = rstd;
  const bool round_normed = (p.flags & B200K_ROWF_ROUND_NORMED) != 0;
  const bool round_affine = (p.flags & B200K_ROWF_ROUND_AFFINE) != 0;
  const bool round_silu = (p.flags & B200K_ROWF_ROUND_SILU) != 0;
  const bool plus_one = (p.flags & B200K_ROWF_WEIGHT_PLUS_ONE) != 0;
#pragma unroll
  for (int k = 0; k < kVPT; ++k) {
    const int64_t vi = lane + k * TPR;
    if (vi < nvec) {
      float wg[VEC], wu[VEC], y[VEC];
      if (p.w) {
        load_row_vec<VEC>(p.w, vi * VEC, p.w_dt, wg);
        load_row_vec<VEC>(p.w, half + vi * VEC, p.w_dt, wu);
      } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j) wg[j] = wu[j] = 1.0f;
      }
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        float ng = g[k].get(j, dt) * rstd, nu = u[k].get(j, dt) * rstd;
        if (round_normed) {
          ng = round_to(ng, dt);
          nu = round_to(nu, dt);
        }
        float yg = (plus_one ? 1.0f + wg[j] : wg[j]) * ng;
        float yu = (plus_one ? 1.0f + wu[j] : wu[j]) * nu;
        if (round_affine) {
          yg = round_to(yg, p.out_dt);
          yu = round_to(yu, p.out_dt);
        }
        float sg = yg * op_sigmoid(yg);
        if (round_silu) sg = round_to(sg, p.out_dt);
        y[j] = sg * yu;
      }
      store_row_vec<VEC>(p.out, row * p.out_stride + vi * VEC, p.out_dt, y);
    }
  }
}

// ---------------------------------------------------------------------------
// Softmax / log-softmax over the row (fp32 math, like aten._softmax).
// ---------------------------------------------------------------------------
template <int TPR, int VEC, bool X16>
__global__ void __launch_bounds__(threads_for(TPR)) softmax_kernel(const __grid_constant__ RowParams p) {
  constexpr int RPB = threads_for(TPR) / TPR;
  __shared__ float sm[threads_for(TPR) / 32];
  const int lane = threadIdx.x % TPR;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * RPB + threadIdx.x / TPR;
  const bool valid_row = row < p.rows;
  const int64_t nvec = p.cols / VEC;
  const int dt = p.x_dt;

  RowFrag<VEC, X16> f[kVPT];
  float m = -INFINITY;
#pragma unroll
  for (int k = 0; k < kVPT; ++k) {
    const int64_t vi = lane + k * TPR;
    if (valid_row && vi < nvec) {
      f[k].load(p.x, row * p.x_stride + vi * VEC, dt);
#pragma unroll
      for (int j = 0; j < VEC; ++j) m = fmaxf(m, f[k].get(j, dt));
    }
  }
  m = row_allreduce<TPR, true>(m, sm);
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < kVPT; ++k) {
    const int64_t vi = lane + k * TPR;
    if (valid_row && vi < nvec) {
#pragma unroll
      for (int j = 0; j < VEC; ++j) s += __expf(f[k].get(j, dt) - m);
    }
  }
  s = row_allreduce<TPR, false>(s, sm);
  if (!valid_row) return;
  const float inv = 1.0f / s;
  const float ls = __logf(s);
#pragma unroll
  for (int k = 0; k < kVPT; ++k) {
    const int64_t vi = lane + k * TPR;
    if (vi < nvec) {
      float y[VEC];
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float d = f[k].get(j, dt) - m;
        y[j] = p.log_softmax ? d - ls : __expf(d) * inv;
      }
      store_row_vec<VEC>(p.out, row * p.out_stride + vi * VEC, p.out_dt, y);
    }
  }
}

namespace {

// Smallest power-of-two thread count per row (32..1024) whose kVPT vectors
// cover `nvec` vectors; 0 if the row does not fit in registers.
int pick_tpr(int64_t nvec) {
  for (int t = 32; t <= 1024; t *= 2)
    if (static_cast<int64_t>(t) * kVPT >= nvec) return t;
  return 0;
}

template <template <int, int, bool> class KSel>
int dispatch_tpr(int tpr, bool vec, bool x16, const RowParams& p, cudaStream_t st) {
  const int threads = std::max(tpr, 256);
  const int rpb = tpr >= 256 ? 1 : 256 / tpr;
  const int64_t grid64 = (p.rows + rpb - 1) / rpb;
  if (grid64 > 0x7fffffff) return B200K_ERR_SHAPE;
  const int grid = static_cast<int>(grid64);
#define B200K_LAUNCH_TPR(T)                                                          \
  case T:                                                                            \
    if (vec && x16) KSel<T, 8, true>::fn()<<<grid, threads, 0, st>>>(p);              \
    else if (vec) KSel<T, 8, false>::fn()<<<grid, threads, 0, st>>>(p);               \
    else KSel<T, 1, false>::fn()<<<grid, threads, 0, st>>>(p);                        \
    break;
  switch (tpr) {
    B200K_LAUNCH_TPR(32)
    B200K_LAUNCH_TPR(64)
    B200K_LAUNCH_TPR(128)
    B200K_LAUNCH_TPR(256)
    B200K_LAUNCH_TPR(512)
    B200K_LAUNCH_TPR(1024)
    default: return B200K_ERR_SHAPE;
  }
#undef B200K_LAUNCH_TPR
  return cudaGetLastError() == cudaSuccess ? B200K_OK : B200K_ERR_LAUNCH;
}

template <int T, int V, bool X> struct SelRms { static auto fn() { return rownorm_kernel<T, V, false, X>; } };
template <int T, int V, bool X> struct SelLayer { static auto fn() { return rownorm_kernel<T, V, true, X>; } };
template <int T, int V, bool X> struct SelSwiglu { static auto fn() { return rmsnorm_swiglu_kernel<T, V, X>; } };
template <int T, int V, bool X> struct SelSoftmax { static auto fn() { return softmax_kernel<T, V, X>; } };

bool row_vec_ok(const void* ptr, int64_t stride, int64_t len) {
  return ptr == nullptr || (aligned16(ptr) && stride % 8 == 0 && len % 8 == 0);
}

}  // namespace

}  // namespace b200k

using namespace b200k;

extern "C" int b200k_rownorm(const B200kRowNormArgs* a, void* stream_) {
  if (!a) return B200K_ERR_ARG;
  if (a->rows < 0 || a->cols <= 0) return B200K_ERR_SHAPE;
  if (a->rows > 0 && (!a->x || !a->out)) return B200K_ERR_ARG;
  if (a->kind < B200K_ROW_RMSNORM || a->kind > B200K_ROW_RMSNORM_SWIGLU) return B200K_ERR_ARG;
  const bool swiglu = a->kind == B200K_ROW_RMSNORM_SWIGLU;
  const bool layer = a->kind == B200K_ROW_LAYERNORM;
  for (int dt : {a->x_dtype, a->out_dtype})
    if (dt != B200K_F32 && dt != B200K_F16 && dt != B200K_BF16) return B200K_ERR_UNSUPPORTED;
  if (a->weight && a->w_dtype != B200K_F32 && a->w_dtype != B200K_F16 && a->w_dtype != B200K_BF16)
    return B200K_ERR_UNSUPPORTED;
  if (a->bias && (!layer || (a->b_dtype != B200K_F32 && a->b_dtype != B200K_F16 && a->b_dtype != B200K_BF16)))
    return B200K_ERR_UNSUPPORTED;
  if (swiglu && a->cols % 2 != 0) return B200K_ERR_SHAPE;
  if (a->rows == 0) return B200K_OK;

  RowParams p;
  std::memset(&p, 0, sizeof(p));
  p.rows = a->rows;
  p.cols = a->cols;
  p.x = a->x;
  p.x_stride = a->x_row_stride;
  p.w = a->weight;
  p.b = a->bias;
  p.out = a->out;
  p.out_stride = a->out_row_stride;
  p.mean_out = a->mean_out;
  p.rstd_out = a->rstd_out;
  p.eps = a->eps;
  p.x_dt = a->x_dtype;
  p.w_dt = a->w_dtype;
  p.b_dt = a->b_dtype;
  p.out_dt = a->out_dtype;
  p.flags = a->flags;

  const int64_t span = swiglu ? a->cols / 2 : a->cols;  // elements each thread group walks
  const int64_t out_len = swiglu ? a->cols / 2 : a->cols;
  const bool vec = row_vec_ok(a->x, a->x_row_stride, span) && row_vec_ok(a->out, a->out_row_stride, out_len) &&
                   row_vec_ok(a->weight, 8, span) && row_vec_ok(a->bias, 8, span);
  const int tpr = pick_tpr(vec ? span / 8 : span);
  if (tpr == 0) return B200K_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  const int rc16 = launch_row16(swiglu ? R16_SWIGLU : (layer ? R16_LAYERNORM : R16_RMSNORM), p, st);
  if (rc16 >= 0) return rc16;
  const bool x16 = a->x_dtype == B200K_BF16 || a->x_dtype == B200K_F16;
  if (swiglu) return dispatch_tpr<SelSwiglu>(tpr, vec, x16, p, st);
  if (layer) return dispatch_tpr<SelLayer>(tpr, vec, x16, p, st);
  return dispatch_tpr<SelRms>(tpr, vec, x16, p, st);
}

extern "C" int b200k_softmax(const B200kSoftmaxArgs* a, void* stream_) {
  if (!a) return B200K_ERR_ARG;
  if (a->rows < 0 || a->cols <= 0) return B200K_ERR_SHAPE;
  if (a->rows > 0 && (!a->x || !a->out)) return B200K_ERR_ARG;
  for (int dt : {a->x_dtype, a->out_dtype})
    if (dt != B200K_F32 && dt != B200K_F16 && dt != B200K_BF16) return B200K_ERR_UNSUPPORTED;
  if (a->rows == 0) return B200K_OK;
  RowParams p;
  std::memset(&p, 0, sizeof(p));
  p.rows = a->rows;
  p.cols = a->cols;
  p.x = a->x;
  p.x_stride = a->x_row_stride;
  p.out = a->out;
  p.out_stride = a->out_row_stride;
  p.x_dt = a->x_dtype;
  p.out_dt = a->out_dtype;
  p.log_softmax = a->log_softmax;
  const bool vec = row_vec_ok(a->x, a->x_row_stride, a->cols) && row_vec_ok(a->out, a->out_row_stride, a->cols);
  const int tpr = pick_tpr(vec ? a->cols / 8 : a->cols);
  if (tpr == 0) return B200K_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  const int rc16 = launch_row16(a->log_softmax ? R16_LOG_SOFTMAX : R16_SOFTMAX, p, st);
  if (rc16 >= 0) return rc16;
  const bool x16 = a->x_dtype == B200K_BF16 || a->x_dtype == B200K_F16;
  return dispatch_tpr<SelSoftmax>(tpr, vec, x16, p, st);
}
