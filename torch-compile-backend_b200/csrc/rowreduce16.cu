// Row-reduction kernels specialised for 16-bit rows: input, output, weight
// and bias of one type (bf16 or f16), rows and vectors 16-byte aligned -- the
// shape of every normalisation and softmax in a 16-bit model.
//
// What differs from the generic kernels in rowreduce.cu (same results up to
// the order of the row sums):
//   * the element type and the rounding steps are template parameters, so the
//     per-element code has no dtype or flag tests;
//   * the row stays packed (8 elements per 16-byte register quad) and is
//     unpacked on every pass, which keeps a 4096-element row of a warp in 64
//     registers;
//   * a row that fits one warp's registers (up to 4096 elements) is reduced
//     with shuffles only; longer rows span TPR = 64..256 threads and combine
//     their warps through shared memory behind a named barrier of those TPR
//     threads alone, never a CTA-wide barrier;
//   * each thread loads its whole share of the row (up to 16 x 16 bytes) with
//     no other work in between, and the launch bounds fix the registers so
//     that two (16 vectors per thread) to four (8 or fewer) CTAs of 256
//     threads fit an SM: 128 KB of reads in flight per SM, what HBM needs;
//   * where the decomposed graph rounds a product of two 16-bit values
//     (normalised x times a 16-bit weight, silu(g) times u), the product is
//     taken on packed bf16x2 / f16x2 pairs: the exact product of two 8- or
//     11-bit significands fits fp32, so one packed rounding equals fp32
//     multiply then rounding, bit for bit.
#include <algorithm>

#include "common.cuh"
#include "host_common.h"
#include "rowreduce.cuh"

namespace b200k {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

template <bool BF16>
struct P16;

template <>
struct P16<true> {
  static __device__ __forceinline__ float lo(uint32_t w) { return __uint_as_float(w << 16); }
  static __device__ __forceinline__ float hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
  // a -> low half (the lower-addressed element), b -> high half
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
    return r;
  }
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
};

template <>
struct P16<false> {
  static __device__ __forceinline__ float lo(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xffffu)));
  }
  static __device__ __forceinline__ float hi(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
  }
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
    return r;
  }
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
};

__device__ __forceinline__ uint32_t word(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Threads per CTA: RPB = 256 / TPR rows, one thread group of TPR per row.
constexpr int kRowThreads = 256;

// Sum or max over a row's TPR threads.  Rows of more than one warp exchange
// warp partials through `slots` (two sets per row group, alternated by the
// caller's `parity`, so back-to-back reductions need one barrier each).
template <int TPR, bool IS_MAX>
__device__ __forceinline__ float group_reduce(float v, float* slots, int grp, int parity) {
  v = IS_MAX ? warp_max(v) : warp_sum(v);
  if constexpr (TPR > 32) {
    constexpr int W = TPR / 32;
    float* s = slots + (grp * 2 + parity) * W;
    const int t = threadIdx.x % TPR;
    if ((t & 31) == 0) s[t >> 5] = v;
    asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "n"(TPR) : "memory");
    float r = s[0];
#pragma unroll
    for (int k = 1; k < W; ++k) r = IS_MAX ? fmaxf(r, s[k]) : r + s[k];
    v = r;
  }
  return v;
}

// FULL: the row fills all TPR x VPT slots (nvec == TPR * VPT), no tests at
// all.  Otherwise every slot is loaded (past the row end from a clamped, valid index) and
// then replaced by `fill` (two packed 16-bit values) when outside the row:
// unconditional loads issue back to back, where loads behind per-slot
// branches measured ~1.5x slower, and a neutral fill (0 for sums, -inf for
// a max and an exp-sum) keeps the reductions free of tests.
template <int TPR, int VPT, bool FULL>
__device__ __forceinline__ void load_row(const uint16_t* row, int t, int nvec, uint32_t fill, uint4 (&v)[VPT]) {
  const uint4* q = reinterpret_cast<const uint4*>(row);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int vi = t + k * TPR;
    if constexpr (FULL) {
      v[k] = __ldg(q + vi);
    } else {
      const bool ok = vi < nvec;
      const uint4 r = __ldg(q + (ok ? vi : 0));
      v[k] = ok ? r : make_uint4(fill, fill, fill, fill);
    }
  }
}

// CTAs per SM the launch bounds guarantee for VT vectors per thread (all
// segments): the registers of 16 vectors (64) plus working set fit 128 per
// thread, two CTAs; fewer vectors, more CTAs.
template <int VT>
constexpr int min_ctas() {
  return VT >= 16 ? 2 : (VT >= 8 ? 3 : 4);
}

#define B200K_ROW_BEGIN(TPR)                                        \
  constexpr int RPB = kRowThreads / (TPR);                          \
  __shared__ float slots[RPB * 2 * ((TPR) / 32)];                   \
  const int grp = threadIdx.x / (TPR);                              \
  const int t = threadIdx.x % (TPR);                                \
  const int64_t row = static_cast<int64_t>(blockIdx.x) * RPB + grp; \
  if (row >= p.rows) return; /* the whole row group leaves together */ \
  (void)slots;

// ---------------------------------------------------------------------------
// softmax / log-softmax: m = max x; s = sum 2^((x - m) log2 e);
// y = 2^((x - m) log2 e) / s, or (x - m) - ln s.
// ---------------------------------------------------------------------------
template <int TPR, int VPT, bool BF16, bool LOG, bool FULL>
__global__ void __launch_bounds__(kRowThreads, min_ctas<VPT>()) softmax16_kernel(const __grid_constant__ RowParams p) {
  using H = P16<BF16>;
  const int nvec = static_cast<int>(p.cols / 8);
  B200K_ROW_BEGIN(TPR)
  uint4 v[VPT];
  constexpr uint32_t kNegInf2 = BF16 ? 0xff80ff80u : 0xfc00fc00u;  // exp-sum adds 0 for them
  load_row<TPR, VPT, FULL>(reinterpret_cast<const uint16_t*>(p.x) + row * p.x_stride, t, nvec, kNegInf2, v);
  float m = -INFINITY;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
#pragma unroll
    for (int i = 0; i < 4; ++i) m = fmaxf(m, fmaxf(H::lo(word(v[k], i)), H::hi(word(v[k], i))));
  }
  m = group_reduce<TPR, true>(m, slots, grp, 0);
  const float ml = m * kLog2e;
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      s += exp2_approx(fmaf(H::lo(word(v[k], i)), kLog2e, -ml));
      s += exp2_approx(fmaf(H::hi(word(v[k], i)), kLog2e, -ml));
    }
  }
  s = group_reduce<TPR, false>(s, slots, grp, 1);
  const float inv = 1.0f / s;
  const float ls = __logf(s);
  uint4* out = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + row * p.out_stride);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int vi = t + k * TPR;
    const bool ok = FULL || vi < nvec;  // compute every slot, store the row's
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = H::lo(word(v[k], i)), b = H::hi(word(v[k], i));
      if constexpr (LOG) {
        o[i] = H::pack((a - m) - ls, (b - m) - ls);
      } else {
        o[i] = H::pack(exp2_approx(fmaf(a, kLog2e, -ml)) * inv, exp2_approx(fmaf(b, kLog2e, -ml)) * inv);
      }
    }
    if (ok) out[vi] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ---------------------------------------------------------------------------
// RMSNorm: n = x * rsqrt(mean(x^2) + eps); y = w * n, with n rounded to the
// 16-bit type first when RN (then the product is a packed multiply).
// ---------------------------------------------------------------------------
template <int TPR, int VPT, bool BF16, bool RN, bool FULL>
__global__ void __launch_bounds__(kRowThreads, min_ctas<VPT>()) rmsnorm16_kernel(const __grid_constant__ RowParams p) {
  using H = P16<BF16>;
  const int nvec = static_cast<int>(p.cols / 8);
  const uint4* w = reinterpret_cast<const uint4*>(p.w);
  B200K_ROW_BEGIN(TPR)
  uint4 v[VPT];
  load_row<TPR, VPT, FULL>(reinterpret_cast<const uint16_t*>(p.x) + row * p.x_stride, t, nvec, 0u, v);
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = H::lo(word(v[k], i)), b = H::hi(word(v[k], i));
      s = fmaf(a, a, s);
      s = fmaf(b, b, s);
    }
  }
  s = group_reduce<TPR, false>(s, slots, grp, 0);
  const float rstd = rsqrtf(s * (1.0f / static_cast<float>(p.cols)) + p.eps);
  if (t == 0 && p.rstd_out) p.rstd_out[row] = rstd;
  uint4* out = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + row * p.out_stride);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int vi = t + k * TPR;
    const bool ok = FULL || vi < nvec;
    const int vc = ok ? vi : 0;  // compute every slot (weights from a valid index), store the row's
    const uint4 wv = w ? __ldg(w + vc) : make_uint4(0u, 0u, 0u, 0u);
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float na = H::lo(word(v[k], i)) * rstd, nb = H::hi(word(v[k], i)) * rstd;
      const uint32_t ww = word(wv, i);
      if constexpr (RN) {
        const uint32_t n2 = H::pack(na, nb);
        o[i] = w ? H::mul(n2, ww) : n2;
      } else {
        o[i] = w ? H::pack(H::lo(ww) * na, H::hi(ww) * nb) : H::pack(na, nb);
      }
    }
    if (ok) out[vi] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ---------------------------------------------------------------------------
// LayerNorm (fp32 statistics, one rounding at the store, as ATen's):
// n = (x - mean) * rsqrt(var + eps); y = n * w + b.
// ---------------------------------------------------------------------------
template <int TPR, int VPT, bool BF16, bool FULL>
__global__ void __launch_bounds__(kRowThreads, min_ctas<VPT>()) layernorm16_kernel(const __grid_constant__ RowParams p) {
  using H = P16<BF16>;
  const int nvec = static_cast<int>(p.cols / 8);
  const float inv_n = 1.0f / static_cast<float>(p.cols);
  const uint4* w = reinterpret_cast<const uint4*>(p.w);
  const uint4* b = reinterpret_cast<const uint4*>(p.b);
  B200K_ROW_BEGIN(TPR)
  uint4 v[VPT];
  load_row<TPR, VPT, FULL>(reinterpret_cast<const uint16_t*>(p.x) + row * p.x_stride, t, nvec, 0u, v);
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
#pragma unroll
    for (int i = 0; i < 4; ++i) s += H::lo(word(v[k], i)) + H::hi(word(v[k], i));
  }
  s = group_reduce<TPR, false>(s, slots, grp, 0);
  const float mean = s * inv_n;
  float q = 0.0f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const float in = (FULL || t + k * TPR < nvec) ? 1.0f : 0.0f;  // slots past the row add nothing
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = (H::lo(word(v[k], i)) - mean) * in, c = (H::hi(word(v[k], i)) - mean) * in;
      q = fmaf(a, a, q);
      q = fmaf(c, c, q);
    }
  }
  q = group_reduce<TPR, false>(q, slots, grp, 1);
  const float rstd = rsqrtf(q * inv_n + p.eps);
  if (t == 0) {
    if (p.mean_out) p.mean_out[row] = mean;
    if (p.rstd_out) p.rstd_out[row] = rstd;
  }
  uint4* out = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + row * p.out_stride);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int vi = t + k * TPR;
    const bool ok = FULL || vi < nvec;
    const int vc = ok ? vi : 0;  // compute every slot (weights from a valid index), store the row's
    // absent weight / bias: 1.0 / 0.0 in the 16-bit type (bf16 0x3f80, f16 0x3c00)
    const uint32_t one2 = BF16 ? 0x3f803f80u : 0x3c003c00u;
    const uint4 wv = w ? __ldg(w + vc) : make_uint4(one2, one2, one2, one2);
    const uint4 bv = b ? __ldg(b + vc) : make_uint4(0u, 0u, 0u, 0u);
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float na = (H::lo(word(v[k], i)) - mean) * rstd, nb = (H::hi(word(v[k], i)) - mean) * rstd;
      const uint32_t ww = word(wv, i), bb = word(bv, i);
      o[i] = H::pack(fmaf(na, H::lo(ww), H::lo(bb)), fmaf(nb, H::hi(ww), H::hi(bb)));
    }
    if (ok) out[vi] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ---------------------------------------------------------------------------
// RMSNorm over the whole row, split into gate / up halves, silu(gate) * up,
// with the 16-bit model's roundings (normalised, affine and silu results):
// yg = w_g * round(g * r), yu = w_u * round(u * r)   (packed products)
// out = round(yg * sigmoid(yg)) * yu                   (packed product)
// ---------------------------------------------------------------------------
template <int TPR, int VPT, bool BF16, bool FULL>
__global__ void __launch_bounds__(kRowThreads, min_ctas<2 * VPT>()) swiglu16_kernel(const __grid_constant__ RowParams p) {
  using H = P16<BF16>;
  const int64_t half = p.cols / 2;
  const int nvec = static_cast<int>(half / 8);
  const uint4* w = reinterpret_cast<const uint4*>(p.w);
  const uint4* wu = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.w) + half);
  B200K_ROW_BEGIN(TPR)
  const uint16_t* xr = reinterpret_cast<const uint16_t*>(p.x) + row * p.x_stride;
  uint4 g[VPT], u[VPT];
  load_row<TPR, VPT, FULL>(xr, t, nvec, 0u, g);
  load_row<TPR, VPT, FULL>(xr + half, t, nvec, 0u, u);
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = H::lo(word(g[k], i)), b = H::hi(word(g[k], i));
      const float c = H::lo(word(u[k], i)), d = H::hi(word(u[k], i));
      s = fmaf(a, a, s);
      s = fmaf(b, b, s);
      s = fmaf(c, c, s);
      s = fmaf(d, d, s);
    }
  }
  s = group_reduce<TPR, false>(s, slots, grp, 0);
  const float rstd = rsqrtf(s / static_cast<float>(p.cols) + p.eps);
  if (t == 0 && p.rstd_out) p.rstd_out[row] = rstd;
  uint4* out = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + row * p.out_stride);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int vi = t + k * TPR;
    const bool ok = FULL || vi < nvec;
    const int vc = ok ? vi : 0;  // compute every slot (weights from a valid index), store the row's
    const uint4 wgv = __ldg(w + vc), wuv = __ldg(wu + vc);
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t gw = word(g[k], i), uw = word(u[k], i);
      const uint32_t yg = H::mul(H::pack(H::lo(gw) * rstd, H::hi(gw) * rstd), word(wgv, i));
      const uint32_t yu = H::mul(H::pack(H::lo(uw) * rstd, H::hi(uw) * rstd), word(wuv, i));
      const float ga = H::lo(yg), gb = H::hi(yg);
      const uint32_t sg = H::pack(__fmul_rn(ga, op_sigmoid(ga)), __fmul_rn(gb, op_sigmoid(gb)));
      o[i] = H::mul(sg, yu);
    }
    if (ok) out[vi] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

#undef B200K_ROW_BEGIN

// ---------------------------------------------------------------------------
// The same RMSNorm -> split -> silu(gate) * up as swiglu16_kernel, over rows
// that a row group walks in a grid-stride loop with its loads one row
// ahead: the gate / up vectors of row r + stride are in flight while row r
// is reduced, computed and stored, so the memory pipe is not idle while the
// row's math runs (the one-row-per-group kernel issues every load of a row
// before any work and nothing during the work; two such CTAs an SM left
// HBM at 57 % busy).  Two vectors a segment keep both rows' registers
// (4 x 2 x 4) small enough for three 256-thread CTAs an SM.
// ---------------------------------------------------------------------------
template <int TPR, int VPT, bool BF16, bool FULL>
__global__ void __launch_bounds__(kRowThreads, 3) swiglu16_rows_kernel(const __grid_constant__ RowParams p) {
  using H = P16<BF16>;
  constexpr int RPB = kRowThreads / TPR;
  __shared__ float slots[RPB * 2 * (TPR / 32 > 0 ? TPR / 32 : 1)];
  const int grp = threadIdx.x / TPR;
  const int t = threadIdx.x % TPR;
  const int64_t half = p.cols / 2;
  const int nvec = static_cast<int>(half / 8);
  const uint4* w = reinterpret_cast<const uint4*>(p.w);
  const uint4* wu = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.w) + half);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * RPB;
  int64_t row = static_cast<int64_t>(blockIdx.x) * RPB + grp;
  if (row >= p.rows) return;  // the whole row group leaves together
  auto load = [&](int64_t r, uint4 (&g)[VPT], uint4 (&u)[VPT]) {
    const uint16_t* xr = reinterpret_cast<const uint16_t*>(p.x) + r * p.x_stride;
    load_row<TPR, VPT, FULL>(xr, t, nvec, 0u, g);
    load_row<TPR, VPT, FULL>(xr + half, t, nvec, 0u, u);
  };
  auto process = [&](int64_t r, const uint4 (&g)[VPT], const uint4 (&u)[VPT], int parity) {
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float a = H::lo(word(g[k], i)), b = H::hi(word(g[k], i));
        const float c = H::lo(word(u[k], i)), d = H::hi(word(u[k], i));
        s = fmaf(a, a, s);
        s = fmaf(b, b, s);
        s = fmaf(c, c, s);
        s = fmaf(d, d, s);
      }
    }
    s = group_reduce<TPR, false>(s, slots, grp, parity);
    const float rstd = rsqrtf(s / static_cast<float>(p.cols) + p.eps);
    if (t == 0 && p.rstd_out) p.rstd_out[r] = rstd;
    uint4* out = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + r * p.out_stride);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int vi = t + k * TPR;
      const bool ok = FULL || vi < nvec;
      const int vc = ok ? vi : 0;
      const uint4 wgv = __ldg(w + vc), wuv = __ldg(wu + vc);
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t gw = word(g[k], i), uw = word(u[k], i);
        const uint32_t yg = H::mul(H::pack(H::lo(gw) * rstd, H::hi(gw) * rstd), word(wgv, i));
        const uint32_t yu = H::mul(H::pack(H::lo(uw) * rstd, H::hi(uw) * rstd), word(wuv, i));
        const float ga = H::lo(yg), gb = H::hi(yg);
        const uint32_t sg = H::pack(__fmul_rn(ga, op_sigmoid(ga)), __fmul_rn(gb, op_sigmoid(gb)));
        o[i] = H::mul(sg, yu);
      }
      if (ok) out[vi] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  };
  uint4 g0[VPT], u0[VPT], g1[VPT], u1[VPT];
  load(row, g0, u0);
  int parity = 0;
  for (;;) {
    const int64_t r1 = row + stride;
    if (r1 < p.rows) load(r1, g1, u1);
    process(row, g0, u0, parity);
    parity ^= 1;
    if (r1 >= p.rows) break;
    const int64_t r2 = r1 + stride;
    if (r2 < p.rows) load(r2, g0, u0);
    process(r1, g1, u1, parity);
    parity ^= 1;
    if (r2 >= p.rows) break;
    row = r2;
  }
}

// Launches swiglu16_rows_kernel when a segment of the row splits into
// TPR x 2 vectors with TPR in {64, 128, 256}; -1 otherwise.
int launch_swiglu_rows(bool bf16, const RowParams& p, int64_t nvec, cudaStream_t st) {
  int tpr = 0;
  const int vpt = 2;
  for (int tt : {64, 128, 256})
    if (static_cast<int64_t>(tt) * vpt == nvec) tpr = tt;
  if (!tpr) return -1;
  const int rpb = kRowThreads / tpr;
  const int sms = device_sm_count();
  if (sms <= 0) return B200K_ERR_DEVICE;
  const int64_t groups = (p.rows + rpb - 1) / rpb;
  const int grid = static_cast<int>(std::min<int64_t>(groups, 3 * static_cast<int64_t>(sms)));
#define B200K_SWR(T, V)                                                                                  \
  if (tpr == T && vpt == V) {                                                                            \
    if (bf16) swiglu16_rows_kernel<T, V, true, true><<<grid, kRowThreads, 0, st>>>(p);                   \
    else swiglu16_rows_kernel<T, V, false, true><<<grid, kRowThreads, 0, st>>>(p);                       \
    return cudaGetLastError() == cudaSuccess ? B200K_OK : B200K_ERR_LAUNCH;                              \
  }
  B200K_SWR(64, 2) B200K_SWR(128, 2) B200K_SWR(256, 2)
#undef B200K_SWR
  return -1;
}

// (TPR, VPT) for a row of nvec 16-byte vectors per segment: the fewest
// threads per row (a warp if it can), then the fewest vectors per thread,
// at most 16 vectors per thread over all segments; false past 256 threads
// (the generic kernels take such rows).
bool pick16(int64_t nvec, int nseg, int& tpr, int& vpt) {
  // A warp per row that the row fills exactly (FULL: no clamped lanes): rows
  // of 768, 1536 and 3072 16-bit values take 3, 6 and 12 vectors per lane.
  for (int vv : {3, 4, 6, 8, 12, 16})
    if (vv * nseg <= 16 && 32 * vv == nvec) {
      tpr = 32;
      vpt = vv;
      return true;
    }
  for (int tt : {32, 64, 128, 256})
    for (int vv : {4, 8, 16})
      if (vv * nseg <= 16 && static_cast<int64_t>(tt) * vv >= nvec) {
        tpr = tt;
        vpt = vv;
        return true;
      }
  return false;
}

template <template <int, int, bool, bool> class K>
int launch_tv(int tpr, int vpt, bool bf16, const RowParams& p, int64_t nvec, cudaStream_t st) {
  const int rpb = kRowThreads / tpr;
  const int64_t grid64 = (p.rows + rpb - 1) / rpb;
  if (grid64 > 0x7fffffff) return B200K_ERR_SHAPE;
  const int grid = static_cast<int>(grid64);
  const bool full = nvec == static_cast<int64_t>(tpr) * vpt;
#define B200K_TV(T, V)                                                                            \
  if (tpr == T && vpt == V) {                                                                     \
    if (full) {                                                                                   \
      if (bf16) K<T, V, true, true>::fn()<<<grid, kRowThreads, 0, st>>>(p);                      \
      else K<T, V, false, true>::fn()<<<grid, kRowThreads, 0, st>>>(p);                          \
    } else {                                                                                      \
      if (bf16) K<T, V, true, false>::fn()<<<grid, kRowThreads, 0, st>>>(p);                     \
      else K<T, V, false, false>::fn()<<<grid, kRowThreads, 0, st>>>(p);                         \
    }                                                                                             \
    return cudaGetLastError() == cudaSuccess ? B200K_OK : B200K_ERR_LAUNCH;                       \
  }
  B200K_TV(32, 3) B200K_TV(32, 4) B200K_TV(32, 6) B200K_TV(32, 8) B200K_TV(32, 12) B200K_TV(32, 16)
  B200K_TV(64, 4) B200K_TV(64, 8) B200K_TV(64, 16)
  B200K_TV(128, 4) B200K_TV(128, 8) B200K_TV(128, 16)
  B200K_TV(256, 4) B200K_TV(256, 8) B200K_TV(256, 16)
#undef B200K_TV
  return B200K_ERR_SHAPE;
}

template <int T, int V, bool B, bool F> struct KSoftmax { static auto fn() { return softmax16_kernel<T, V, B, false, F>; } };
template <int T, int V, bool B, bool F> struct KLogSoftmax { static auto fn() { return softmax16_kernel<T, V, B, true, F>; } };
template <int T, int V, bool B, bool F> struct KRms { static auto fn() { return rmsnorm16_kernel<T, V, B, false, F>; } };
template <int T, int V, bool B, bool F> struct KRmsRn { static auto fn() { return rmsnorm16_kernel<T, V, B, true, F>; } };
template <int T, int V, bool B, bool F> struct KLayer { static auto fn() { return layernorm16_kernel<T, V, B, F>; } };
// Gate and up halves: rows are capped at 8 vectors per half per thread
// (pick16), so the 16-vector instantiation is never launched.
template <int T, int V, bool B, bool F> struct KSwiglu {
  static auto fn() { return swiglu16_kernel<T, (V <= 8 ? V : 8), B, F>; }
};

bool aligned_rows(const void* ptr, int64_t stride) { return aligned16(ptr) && stride % 8 == 0; }

}  // namespace

int launch_row16(Row16Kind kind, const RowParams& p, cudaStream_t st) {
  const int dt = p.x_dt;
  if (dt != B200K_BF16 && dt != B200K_F16) return -1;
  if (p.out_dt != dt || (p.w && p.w_dt != dt) || (p.b && p.b_dt != dt)) return -1;
  const bool swiglu = kind == R16_SWIGLU;
  const int64_t span = swiglu ? p.cols / 2 : p.cols;
  if (span % 8 != 0 || !aligned_rows(p.x, p.x_stride) || !aligned_rows(p.out, p.out_stride)) return -1;
  if ((p.w && !aligned16(p.w)) || (p.b && !aligned16(p.b))) return -1;
  int tpr = 0, vpt = 0;
  if (!pick16(span / 8, swiglu ? 2 : 1, tpr, vpt)) return -1;
  const bool bf16 = dt == B200K_BF16;
  constexpr int kNormed = B200K_ROWF_ROUND_NORMED, kAffine = B200K_ROWF_ROUND_AFFINE, kSilu = B200K_ROWF_ROUND_SILU;
  switch (kind) {
    case R16_SOFTMAX: return launch_tv<KSoftmax>(tpr, vpt, bf16, p, span / 8, st);
    case R16_LOG_SOFTMAX: return launch_tv<KLogSoftmax>(tpr, vpt, bf16, p, span / 8, st);
    case R16_RMSNORM:
      if (p.flags == 0) return launch_tv<KRms>(tpr, vpt, bf16, p, span / 8, st);
      if (p.flags == kNormed) return launch_tv<KRmsRn>(tpr, vpt, bf16, p, span / 8, st);
      return -1;
    case R16_LAYERNORM:
      return p.flags == 0 ? launch_tv<KLayer>(tpr, vpt, bf16, p, span / 8, st) : -1;
    case R16_SWIGLU:
      if (p.flags == (kNormed | kAffine | kSilu) && p.w) {
        // rows long enough for the pipelined row loop take it
        if (p.rows >= 4 * static_cast<int64_t>(device_sm_count())) {
          const int rc = launch_swiglu_rows(bf16, p, span / 8, st);
          if (rc != -1) return rc;
        }
        return launch_tv<KSwiglu>(tpr, vpt, bf16, p, span / 8, st);
      }
      return -1;
  }
  return -1;
}

}  // namespace b200k
