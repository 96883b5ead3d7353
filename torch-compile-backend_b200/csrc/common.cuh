// Shared device helpers for libb200k: dtype load/store, the accumulator-machine
// interpreter that evaluates fused pointwise chains, fast integer division and
// bounded waits.  sm_100a only.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "b200k.h"

namespace b200k {

// ---------------------------------------------------------------------------
// Scalar math with the reference's op semantics
// (compiler/optimization/fusion_pointwise.py:12-30): fp32 everywhere,
// sigmoid = 1/(1+exp(-x)), tanh = 2*sigmoid(2x)-1, relu/max/min keep the
// non-NaN operand (Triton's default maximum/minimum).
// ---------------------------------------------------------------------------
// exp, log: the hardware ex2/lg2 approximations (a few ulp), which is also
// what the reference's tl.exp / tl.log lower to; erf, sqrt and division stay
// IEEE-accurate.
__device__ __forceinline__ float op_exp(float x) { return __expf(x); }
__device__ __forceinline__ float op_log(float x) { return __logf(x); }
__device__ __forceinline__ float op_sigmoid(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
__device__ __forceinline__ float op_tanh(float x) { return 2.0f * op_sigmoid(2.0f * x) - 1.0f; }
__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float round_f16(float x) { return __half2float(__float2half_rn(x)); }

// ---------------------------------------------------------------------------
// Element loads / stores with conversion to/from fp32.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float load_scalar(const void* base, int64_t off, int dt) {
  switch (dt) {
    case B200K_F32: return __ldg(reinterpret_cast<const float*>(base) + off);
    case B200K_F16: return __half2float(__ldg(reinterpret_cast<const __half*>(base) + off));
    case B200K_BF16: return __bfloat162float(__ldg(reinterpret_cast<const __nv_bfloat16*>(base) + off));
    case B200K_F64: return static_cast<float>(__ldg(reinterpret_cast<const double*>(base) + off));
    case B200K_I32: return static_cast<float>(__ldg(reinterpret_cast<const int32_t*>(base) + off));
    case B200K_I64: return static_cast<float>(__ldg(reinterpret_cast<const long long*>(base) + off));
    case B200K_BOOL:
    case B200K_U8: return static_cast<float>(reinterpret_cast<const uint8_t*>(base)[off]);
    default: return 0.0f;
  }
}

// Loads 8 consecutive elements starting at element offset `off` (16-byte
// aligned for 2-byte types, 32-byte for fp32: the host guarantees it).
__device__ __forceinline__ void load_vec8(const void* base, int64_t off, int dt, float (&v)[8]) {
  switch (dt) {
    case B200K_BF16: {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(base) + off));
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
      }
      break;
    }
    case B200K_F16: {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(base) + off));
      const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
      }
      break;
    }
    case B200K_F32: {
      const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + off);
      const float4 a = __ldg(p), b = __ldg(p + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      break;
    }
    default: {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = load_scalar(base, off + j, dt);
      break;
    }
  }
}

__device__ __forceinline__ void store_scalar(void* base, int64_t off, int dt, float x) {
  switch (dt) {
    case B200K_F32: reinterpret_cast<float*>(base)[off] = x; break;
    case B200K_F16: reinterpret_cast<__half*>(base)[off] = __float2half_rn(x); break;
    case B200K_BF16: reinterpret_cast<__nv_bfloat16*>(base)[off] = __float2bfloat16_rn(x); break;
    case B200K_F64: reinterpret_cast<double*>(base)[off] = static_cast<double>(x); break;
    default: break;
  }
}

__device__ __forceinline__ uint4 pack_bf16x8(const float (&v)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
  return u;
}
__device__ __forceinline__ uint4 pack_f16x8(const float (&v)[8]) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
  return u;
}

__device__ __forceinline__ void store_vec8(void* base, int64_t off, int dt, const float (&v)[8]) {
  switch (dt) {
    case B200K_BF16:
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(base) + off) = pack_bf16x8(v);
      break;
    case B200K_F16:
      *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(base) + off) = pack_f16x8(v);
      break;
    case B200K_F32: {
      float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + off);
      p[0] = make_float4(v[0], v[1], v[2], v[3]);
      p[1] = make_float4(v[4], v[5], v[6], v[7]);
      break;
    }
    default:
#pragma unroll
      for (int j = 0; j < 8; ++j) store_scalar(base, off + j, dt, v[j]);
      break;
  }
}

// ---------------------------------------------------------------------------
// The accumulator machine.  Each dispatch is warp-uniform (the program lives
// in kernel parameter space), and every case names its slot at compile time,
// so slots and the accumulator stay in registers; the per-element cost is the
// arithmetic itself plus a dispatch amortised over VEC elements.
// ---------------------------------------------------------------------------
constexpr int kSlots = B200K_MAX_SLOTS;

#define B200K_BIN_CASES(OPC, EXPR)                                                  \
  case OPC * 10 + 0: { _Pragma("unroll") for (int j = 0; j < VEC; ++j) { float a = acc[j], x = r[0 % S][j]; acc[j] = (EXPR); } } break; \
  case OPC * 10 + 1: { _Pragma("unroll") for (int j = 0; j < VEC; ++j) { float a = acc[j], x = r[1 % S][j]; acc[j] = (EXPR); } } break; \
  case OPC * 10 + 2: { _Pragma("unroll") for (int j = 0; j < VEC; ++j) { float a = acc[j], x = r[2 % S][j]; acc[j] = (EXPR); } } break; \
  case OPC * 10 + 3: { _Pragma("unroll") for (int j = 0; j < VEC; ++j) { float a = acc[j], x = r[3 % S][j]; acc[j] = (EXPR); } } break; \
  case OPC * 10 + 4: { _Pragma("unroll") for (int j = 0; j < VEC; ++j) { float a = acc[j], x = r[4 % S][j]; acc[j] = (EXPR); } } break; \
  case OPC * 10 + 5: { _Pragma("unroll") for (int j = 0; j < VEC; ++j) { float a = acc[j], x = r[5 % S][j]; acc[j] = (EXPR); } } break; \
  case OPC * 10 + 6: { _Pragma("unroll") for (int j = 0; j < VEC; ++j) { float a = acc[j], x = r[6 % S][j]; acc[j] = (EXPR); } } break; \
  case OPC * 10 + 7: { _Pragma("unroll") for (int j = 0; j < VEC; ++j) { float a = acc[j], x = r[7 % S][j]; acc[j] = (EXPR); } } break; \
  case OPC * 10 + 8: { _Pragma("unroll") for (int j = 0; j < VEC; ++j) { float a = acc[j], x = imm; acc[j] = (EXPR); } } break;

#define B200K_UN_CASE(OPC, EXPR) \
  case OPC * 10 + B200K_OPERAND_NONE: { _Pragma("unroll") for (int j = 0; j < VEC; ++j) { float a = acc[j]; acc[j] = (EXPR); } } break;

#define B200K_SLOT_CASE(OPC, S, BODY) \
  case OPC * 10 + S: { _Pragma("unroll") for (int j = 0; j < VEC; ++j) { BODY; } } break;

// S < kSlots: a kernel that keeps only S slots in registers; programs it runs
// name no slot >= S (the host checks, slots_used()), so the cases that would
// (slot k maps to k % S) are never taken.
template <int VEC, int S = kSlots>
__device__ __forceinline__ void run_program(const B200kProgram& prog, float (&r)[S][VEC], float (&acc)[VEC]) {
  const int n = prog.n;
  for (int pc = 0; pc < n; ++pc) {
    const int code = prog.ins[pc].code;
    const float imm = prog.ins[pc].imm;
    switch (code) {
      // acc = slot / imm
      B200K_SLOT_CASE(B200K_OP_MOV, 0, acc[j] = r[0 % S][j])
      B200K_SLOT_CASE(B200K_OP_MOV, 1, acc[j] = r[1 % S][j])
      B200K_SLOT_CASE(B200K_OP_MOV, 2, acc[j] = r[2 % S][j])
      B200K_SLOT_CASE(B200K_OP_MOV, 3, acc[j] = r[3 % S][j])
      B200K_SLOT_CASE(B200K_OP_MOV, 4, acc[j] = r[4 % S][j])
      B200K_SLOT_CASE(B200K_OP_MOV, 5, acc[j] = r[5 % S][j])
      B200K_SLOT_CASE(B200K_OP_MOV, 6, acc[j] = r[6 % S][j])
      B200K_SLOT_CASE(B200K_OP_MOV, 7, acc[j] = r[7 % S][j])
      B200K_SLOT_CASE(B200K_OP_MOV, 8, acc[j] = imm)
      // slot = acc
      B200K_SLOT_CASE(B200K_OP_STORE, 0, r[0 % S][j] = acc[j])
      B200K_SLOT_CASE(B200K_OP_STORE, 1, r[1 % S][j] = acc[j])
      B200K_SLOT_CASE(B200K_OP_STORE, 2, r[2 % S][j] = acc[j])
      B200K_SLOT_CASE(B200K_OP_STORE, 3, r[3 % S][j] = acc[j])
      B200K_SLOT_CASE(B200K_OP_STORE, 4, r[4 % S][j] = acc[j])
      B200K_SLOT_CASE(B200K_OP_STORE, 5, r[5 % S][j] = acc[j])
      B200K_SLOT_CASE(B200K_OP_STORE, 6, r[6 % S][j] = acc[j])
      B200K_SLOT_CASE(B200K_OP_STORE, 7, r[7 % S][j] = acc[j])
      B200K_BIN_CASES(B200K_OP_ADD, a + x)
      B200K_BIN_CASES(B200K_OP_SUB, a - x)
      B200K_BIN_CASES(B200K_OP_RSUB, x - a)
      B200K_BIN_CASES(B200K_OP_MUL, a * x)
      B200K_BIN_CASES(B200K_OP_DIV, a / x)
      B200K_BIN_CASES(B200K_OP_RDIV, x / a)
      B200K_BIN_CASES(B200K_OP_MAX, fmaxf(a, x))
      B200K_BIN_CASES(B200K_OP_MIN, fminf(a, x))
      B200K_UN_CASE(B200K_OP_NEG, -a)
      B200K_UN_CASE(B200K_OP_ABS, fabsf(a))
      B200K_UN_CASE(B200K_OP_RELU, fmaxf(a, 0.0f))
      B200K_UN_CASE(B200K_OP_EXP, op_exp(a))
      B200K_UN_CASE(B200K_OP_LOG, op_log(a))
      B200K_UN_CASE(B200K_OP_SQRT, sqrtf(a))
      B200K_UN_CASE(B200K_OP_RSQRT, rsqrtf(a))
      B200K_UN_CASE(B200K_OP_ERF, erff(a))
      B200K_UN_CASE(B200K_OP_SIGMOID, op_sigmoid(a))
      B200K_UN_CASE(B200K_OP_TANH, op_tanh(a))
      B200K_UN_CASE(B200K_OP_ROUND_BF16, round_bf16(a))
      B200K_UN_CASE(B200K_OP_ROUND_F16, round_f16(a))
      default: break;
    }
  }
}

#undef B200K_BIN_CASES
#undef B200K_UN_CASE
#undef B200K_SLOT_CASE

// ---------------------------------------------------------------------------
// Unsigned 32-bit division by a run-time constant d >= 1 (round-up method:
// with s = ceil(log2 d) and m = floor(2^32 (2^s - d) / d) + 1,
// n / d == (umulhi(n, m) + n) >> s for every n < 2^31).
// ---------------------------------------------------------------------------
struct FastDiv {
  uint32_t d, m, s;
};

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
  return (__umulhi(n, f.m) + n) >> f.s;
}

// ---------------------------------------------------------------------------
// Timers and the error word.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

}  // namespace b200k
