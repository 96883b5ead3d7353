// Rotary position embedding in the rotate-half form (b200k_rope, include/b200k.h):
//   out = x * cos + rotate_half(x) * sin.
//
// No reference counterpart: the reference's pointwise fusion
// (compiler/optimization/fusion_pointwise.py:12-30) has no aten.cat, so
// rotate_half stays two ATen kernels (neg, cat) and the fused x*cos + r*sin
// reads the materialised rotation.  Here one thread takes 8 consecutive
// elements of one row of D: its own 16-byte chunk of x and the partner chunk
// D/2 away (the same 128-byte line for D <= 64, so the second read hits L1),
// the cos / sin chunks (L2-resident [S, D] tables), and stores one chunk.
// Each product and the sum are packed bf16x2 / f16x2 operations: products
// and sums of two 16-bit values are exact in fp32, so their single rounding
// equals eager's fp32-then-round.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "host_common.h"

namespace b200k {
namespace {

struct RopeParams {
  FastDiv div_c, div_s, div_h;  // unit -> (row, chunk), row -> (b, h, s)
  uint32_t rows;
  int32_t chunks;        // D / 8
  int32_t half_chunks;   // D / 16
  const uint16_t* x;
  const uint16_t* cs;
  const uint16_t* sn;
  uint16_t* out;
  int64_t xs[3], cst[3], snt[3], os[3];  // element strides of b, h, s
};

template <bool BF16>
__device__ __forceinline__ uint32_t pk_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  if (BF16) asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
template <bool BF16>
__device__ __forceinline__ uint32_t pk_add(uint32_t a, uint32_t b) {
  uint32_t d;
  if (BF16) asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

template <bool BF16>
__global__ void __launch_bounds__(256) rope_kernel(const __grid_constant__ RopeParams p) {
  const uint32_t total = p.rows * static_cast<uint32_t>(p.chunks);
  for (uint32_t u = blockIdx.x * blockDim.x + threadIdx.x; u < total; u += gridDim.x * blockDim.x) {
    const uint32_t row = fdiv(u, p.div_c);
    const int c = static_cast<int>(u - row * p.div_c.d);
    const uint32_t bh = fdiv(row, p.div_s);
    const uint32_t s = row - bh * p.div_s.d;
    const uint32_t b = fdiv(bh, p.div_h);
    const uint32_t h = bh - b * p.div_h.d;
    const int64_t xo = b * p.xs[0] + h * p.xs[1] + s * p.xs[2];
    const int64_t co = b * p.cst[0] + h * p.cst[1] + s * p.cst[2];
    const int64_t so = b * p.snt[0] + h * p.snt[1] + s * p.snt[2];
    const int64_t oo = b * p.os[0] + h * p.os[1] + s * p.os[2];
    const bool lower = c < p.half_chunks;
    const int partner = lower ? c + p.half_chunks : c - p.half_chunks;
    const uint4 xv = __ldg(reinterpret_cast<const uint4*>(p.x + xo) + c);
    uint4 rv = __ldg(reinterpret_cast<const uint4*>(p.x + xo) + partner);
    if (lower) {  // -x[j + D/2]: flip the sign bits (exact)
      rv.x ^= 0x80008000u;
      rv.y ^= 0x80008000u;
      rv.z ^= 0x80008000u;
      rv.w ^= 0x80008000u;
    }
    const uint4 cv = __ldg(reinterpret_cast<const uint4*>(p.cs + co) + c);
    const uint4 sv = __ldg(reinterpret_cast<const uint4*>(p.sn + so) + c);
    uint4 o;
    o.x = pk_add<BF16>(pk_mul<BF16>(xv.x, cv.x), pk_mul<BF16>(rv.x, sv.x));
    o.y = pk_add<BF16>(pk_mul<BF16>(xv.y, cv.y), pk_mul<BF16>(rv.y, sv.y));
    o.z = pk_add<BF16>(pk_mul<BF16>(xv.z, cv.z), pk_mul<BF16>(rv.z, sv.z));
    o.w = pk_add<BF16>(pk_mul<BF16>(xv.w, cv.w), pk_mul<BF16>(rv.w, sv.w));
    reinterpret_cast<uint4*>(p.out + oo)[c] = o;
  }
}

// Views that break the 16-byte layout (odd offsets or strides, a strided D):
// one element per thread, the same roundings on scalar 16-bit operations.
template <bool BF16>
__device__ __forceinline__ uint16_t sc_fma_rope(uint16_t x, uint16_t c, uint16_t r, uint16_t s) {
  uint16_t a, b, o;
  if (BF16) {
    asm("mul.rn.bf16 %0, %1, %2;" : "=h"(a) : "h"(x), "h"(c));
    asm("mul.rn.bf16 %0, %1, %2;" : "=h"(b) : "h"(r), "h"(s));
    asm("add.rn.bf16 %0, %1, %2;" : "=h"(o) : "h"(a), "h"(b));
  } else {
    asm("mul.rn.f16 %0, %1, %2;" : "=h"(a) : "h"(x), "h"(c));
    asm("mul.rn.f16 %0, %1, %2;" : "=h"(b) : "h"(r), "h"(s));
    asm("add.rn.f16 %0, %1, %2;" : "=h"(o) : "h"(a), "h"(b));
  }
  return o;
}

struct RopeScalarParams {
  FastDiv div_d, div_s, div_h;  // element -> (row, j), row -> (b, h, s)
  uint32_t total;
  int32_t half;
  const uint16_t* x;
  const uint16_t* cs;
  const uint16_t* sn;
  uint16_t* out;
  int64_t xs[4], cst[4], snt[4], os[4];
};

template <bool BF16>
__global__ void __launch_bounds__(256) rope_scalar_kernel(const __grid_constant__ RopeScalarParams p) {
  for (uint32_t u = blockIdx.x * blockDim.x + threadIdx.x; u < p.total; u += gridDim.x * blockDim.x) {
    const uint32_t row = fdiv(u, p.div_d);
    const int j = static_cast<int>(u - row * p.div_d.d);
    const uint32_t bh = fdiv(row, p.div_s);
    const uint32_t s = row - bh * p.div_s.d;
    const uint32_t b = fdiv(bh, p.div_h);
    const uint32_t h = bh - b * p.div_h.d;
    const int64_t xo = b * p.xs[0] + h * p.xs[1] + s * p.xs[2];
    const bool lower = j < p.half;
    const int jp = lower ? j + p.half : j - p.half;
    uint16_t r = p.x[xo + jp * p.xs[3]];
    if (lower) r ^= 0x8000u;
    const uint16_t c = p.cs[b * p.cst[0] + h * p.cst[1] + s * p.cst[2] + j * p.cst[3]];
    const uint16_t sn = p.sn[b * p.snt[0] + h * p.snt[1] + s * p.snt[2] + j * p.snt[3]];
    p.out[b * p.os[0] + h * p.os[1] + s * p.os[2] + j * p.os[3]] =
        sc_fma_rope<BF16>(p.x[xo + j * p.xs[3]], c, r, sn);
  }
}

bool strides_ok(const int64_t* st) { return st[0] % 8 == 0 && st[1] % 8 == 0 && st[2] % 8 == 0 && st[3] == 1; }

}  // namespace
}  // namespace b200k

using namespace b200k;

extern "C" int b200k_rope(const B200kRopeArgs* a, void* stream_) {
  if (!a) return B200K_ERR_ARG;
  for (int d = 0; d < 4; ++d)
    if (a->sizes[d] < 0) return B200K_ERR_SHAPE;
  const int64_t B = a->sizes[0], H = a->sizes[1], S = a->sizes[2], D = a->sizes[3];
  if (B * H * S * D == 0) return B200K_OK;
  if (!a->x || !a->cos || !a->sin || !a->out) return B200K_ERR_ARG;
  if (a->dtype != B200K_BF16 && a->dtype != B200K_F16) return B200K_ERR_UNSUPPORTED;
  if (D % 2 != 0) return B200K_ERR_SHAPE;
  if (B * H * S * D > 0x7fffffffLL) return B200K_ERR_SHAPE;
  const int sms = device_sm_count();
  if (sms <= 0) return B200K_ERR_DEVICE;
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  const bool vec = D % 16 == 0 && aligned16(a->x) && aligned16(a->cos) && aligned16(a->sin) && aligned16(a->out) &&
                   strides_ok(a->x_strides) && strides_ok(a->cos_strides) && strides_ok(a->sin_strides) &&
                   strides_ok(a->out_strides);
  if (!vec) {
    RopeScalarParams q;
    std::memset(&q, 0, sizeof(q));
    q.div_d = make_fastdiv(static_cast<uint32_t>(D));
    q.div_s = make_fastdiv(static_cast<uint32_t>(S));
    q.div_h = make_fastdiv(static_cast<uint32_t>(H));
    q.total = static_cast<uint32_t>(B * H * S * D);
    q.half = static_cast<int32_t>(D / 2);
    q.x = static_cast<const uint16_t*>(a->x);
    q.cs = static_cast<const uint16_t*>(a->cos);
    q.sn = static_cast<const uint16_t*>(a->sin);
    q.out = static_cast<uint16_t*>(a->out);
    for (int d = 0; d < 4; ++d) {
      q.xs[d] = a->x_strides[d];
      q.cst[d] = a->cos_strides[d];
      q.snt[d] = a->sin_strides[d];
      q.os[d] = a->out_strides[d];
    }
    const int grid = static_cast<int>(std::min<int64_t>((q.total + 255) / 256, static_cast<int64_t>(sms) * 8));
    if (a->dtype == B200K_BF16) rope_scalar_kernel<true><<<grid, 256, 0, st>>>(q);
    else rope_scalar_kernel<false><<<grid, 256, 0, st>>>(q);
    return cudaGetLastError() == cudaSuccess ? B200K_OK : B200K_ERR_LAUNCH;
  }
  RopeParams p;
  std::memset(&p, 0, sizeof(p));
  p.div_c = make_fastdiv(static_cast<uint32_t>(D / 8));
  p.div_s = make_fastdiv(static_cast<uint32_t>(S));
  p.div_h = make_fastdiv(static_cast<uint32_t>(H));
  p.rows = static_cast<uint32_t>(B * H * S);
  p.chunks = static_cast<int32_t>(D / 8);
  p.half_chunks = static_cast<int32_t>(D / 16);
  p.x = static_cast<const uint16_t*>(a->x);
  p.cs = static_cast<const uint16_t*>(a->cos);
  p.sn = static_cast<const uint16_t*>(a->sin);
  p.out = static_cast<uint16_t*>(a->out);
  for (int d = 0; d < 3; ++d) {
    p.xs[d] = a->x_strides[d];
    p.cst[d] = a->cos_strides[d];
    p.snt[d] = a->sin_strides[d];
    p.os[d] = a->out_strides[d];
  }
  const int64_t units = static_cast<int64_t>(p.rows) * p.chunks;
  const int grid = static_cast<int>(std::min<int64_t>((units + 255) / 256, static_cast<int64_t>(sms) * 8));
  if (a->dtype == B200K_BF16) rope_kernel<true><<<grid, 256, 0, st>>>(p);
  else rope_kernel<false><<<grid, 256, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? B200K_OK : B200K_ERR_LAUNCH;
}
