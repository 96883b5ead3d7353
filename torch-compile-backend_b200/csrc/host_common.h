// Host-side helpers shared by the libb200k entry points.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>
#include <cstring>

#include "b200k.h"

namespace b200k {

inline bool valid_dtype(int dt) { return dt >= B200K_F32 && dt <= B200K_U8; }
inline bool valid_float_dtype(int dt) {
  return dt == B200K_F32 || dt == B200K_F16 || dt == B200K_BF16 || dt == B200K_F64;
}
inline int dtype_size(int dt) {
  switch (dt) {
    case B200K_F32: case B200K_I32: return 4;
    case B200K_F16: case B200K_BF16: return 2;
    case B200K_F64: case B200K_I64: return 8;
    default: return 1;
  }
}
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Slots a (validated) program touches: the loaded operands and every slot an
// instruction names.
inline int slots_used(const B200kProgram& prog, int n_loaded) {
  int n = n_loaded;
  for (int i = 0; i < prog.n; ++i) {
    const int op = prog.ins[i].code / 10, operand = prog.ins[i].code % 10;
    const bool names_slot = op == B200K_OP_STORE || op == B200K_OP_MOV || (op >= B200K_OP_ADD && op <= B200K_OP_MIN);
    if (names_slot && operand < B200K_MAX_SLOTS) n = operand + 1 > n ? operand + 1 : n;
  }
  return n;
}

// Checks every instruction of an accumulator-machine program: known opcode,
// operand kind allowed for that opcode.  `n_loaded` slots hold operands.
inline int validate_program(const B200kProgram& prog, int n_loaded) {
  if (prog.n < 0 || prog.n > B200K_MAX_INSTR) return B200K_ERR_PROGRAM;
  if (n_loaded > B200K_MAX_SLOTS) return B200K_ERR_PROGRAM;
  for (int i = 0; i < prog.n; ++i) {
    const int code = prog.ins[i].code;
    if (code < 0) return B200K_ERR_PROGRAM;
    const int op = code / 10, operand = code % 10;
    if (op >= B200K_OP_COUNT) return B200K_ERR_PROGRAM;
    if (op == B200K_OP_NOP) {
      if (operand != B200K_OPERAND_NONE) return B200K_ERR_PROGRAM;
    } else if (op == B200K_OP_MOV || (op >= B200K_OP_ADD && op <= B200K_OP_MIN)) {
      if (operand > B200K_OPERAND_IMM) return B200K_ERR_PROGRAM;
    } else if (op == B200K_OP_STORE) {
      if (operand >= B200K_MAX_SLOTS) return B200K_ERR_PROGRAM;
    } else {
      if (operand != B200K_OPERAND_NONE) return B200K_ERR_PROGRAM;
    }
  }
  return B200K_OK;
}

// Multiply-shift constants for FastDiv (see common.cuh).
template <typename FD>
inline FD make_fastdiv_t(uint32_t d) {
  FD f;
  f.d = d;
  uint32_t s = 0;
  while ((uint64_t(1) << s) < d) ++s;
  f.s = s;
  f.m = static_cast<uint32_t>(((uint64_t(1) << 32) * ((uint64_t(1) << s) - d)) / d + 1);
  return f;
}

// ------------------------------------------------------------------------
// Host emulation of the accumulator machine and of the canonical epilogue
// form, used to check that a caller's form describes its program.
// ------------------------------------------------------------------------
inline float h_sigmoid(float x) { return 1.0f / (1.0f + std::exp(-x)); }
inline float h_tanh(float x) { return 2.0f * h_sigmoid(2.0f * x) - 1.0f; }
inline float h_round_bf16(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) return x;
  u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}
inline float h_round_f16(float x) { return __half2float(__float2half_rn(x)); }

inline float host_run_program(const B200kProgram& prog, const float* init, int n_loaded) {
  float r[B200K_MAX_SLOTS] = {0};
  for (int i = 0; i < n_loaded && i < B200K_MAX_SLOTS; ++i) r[i] = init[i];
  float acc = r[0];
  for (int i = 0; i < prog.n; ++i) {
    const int op = prog.ins[i].code / 10, o = prog.ins[i].code % 10;
    const float x = o < B200K_MAX_SLOTS ? r[o] : prog.ins[i].imm;
    switch (op) {
      case B200K_OP_MOV: acc = x; break;
      case B200K_OP_STORE: r[o] = acc; break;
      case B200K_OP_ADD: acc = acc + x; break;
      case B200K_OP_SUB: acc = acc - x; break;
      case B200K_OP_RSUB: acc = x - acc; break;
      case B200K_OP_MUL: acc = acc * x; break;
      case B200K_OP_DIV: acc = acc / x; break;
      case B200K_OP_RDIV: acc = x / acc; break;
      case B200K_OP_MAX: acc = std::fmax(acc, x); break;
      case B200K_OP_MIN: acc = std::fmin(acc, x); break;
      case B200K_OP_NEG: acc = -acc; break;
      case B200K_OP_ABS: acc = std::fabs(acc); break;
      case B200K_OP_RELU: acc = std::fmax(acc, 0.0f); break;
      case B200K_OP_EXP: acc = std::exp(acc); break;
      case B200K_OP_LOG: acc = std::log(acc); break;
      case B200K_OP_SQRT: acc = std::sqrt(acc); break;
      case B200K_OP_RSQRT: acc = 1.0f / std::sqrt(acc); break;
      case B200K_OP_ERF: acc = std::erf(acc); break;
      case B200K_OP_SIGMOID: acc = h_sigmoid(acc); break;
      case B200K_OP_TANH: acc = h_tanh(acc); break;
      case B200K_OP_ROUND_BF16: acc = h_round_bf16(acc); break;
      case B200K_OP_ROUND_F16: acc = h_round_f16(acc); break;
      default: break;
    }
  }
  return acc;
}

inline float host_act(int act, float x) {
  switch (act) {
    case B200K_ACT_GELU_ERF: return (x * 0.5f) * (std::erf(x * 0.7071067811865476f) + 1.0f);
    case B200K_ACT_GELU_TANH: {
      const float t3 = x + ((x * x) * x) * 0.044715f;
      return (x * 0.5f) * (h_tanh(t3 * 0.7978845608028654f) + 1.0f);
    }
    case B200K_ACT_SILU: return x * h_sigmoid(x);
    case B200K_ACT_RELU: return std::fmax(x, 0.0f);
    case B200K_ACT_SIGMOID: return h_sigmoid(x);
    case B200K_ACT_TANH: return h_tanh(x);
    default: return x;
  }
}

// B200K_OK when `f` computes what `prog` computes on 16 probe points
// (slot 0 = accumulator, slot i+1 = extras[i]).
inline int check_form(const B200kEpilogueForm& f, const B200kProgram& prog, int n_extras) {
  if (f.kind != 1) return B200K_ERR_ARG;
  for (int idx : {f.bias, f.scale, f.residual})
    if (idx < -1 || idx >= n_extras) return B200K_ERR_ARG;
  if (f.act < 0 || f.act >= B200K_ACT_COUNT) return B200K_ERR_ARG;
  if (f.round != -1 && f.round != B200K_BF16 && f.round != B200K_F16) return B200K_ERR_ARG;
  int tight = 0;
  for (int k = 0; k < 16; ++k) {
    float init[B200K_MAX_SLOTS] = {0};
    init[0] = -4.0f + 0.53f * static_cast<float>(k);
    for (int i = 0; i < n_extras && i + 1 < B200K_MAX_SLOTS; ++i)
      init[i + 1] = 0.29f * static_cast<float>(i + 1) * (1.0f + 0.17f * static_cast<float>(k)) - 0.6f;
    const float want = host_run_program(prog, init, 1 + n_extras);
    float v = init[0];
    if (f.bias >= 0) v += init[f.bias + 1];
    v = host_act(f.act, v);
    if (f.round == B200K_BF16) v = h_round_bf16(v);
    if (f.round == B200K_F16) v = h_round_f16(v);
    if (f.scale >= 0) v *= init[f.scale + 1];
    if (f.residual >= 0) v += init[f.residual + 1];
    const float d = std::fabs(v - want), tol = 1.0f + std::fabs(want);
    if (!(d <= 2e-2f * tol)) return B200K_ERR_PROGRAM;
    if (d <= 1e-5f * tol) ++tight;
  }
  return tight >= 13 ? B200K_OK : B200K_ERR_PROGRAM;
}

int device_sm_count();

}  // namespace b200k

#define make_fastdiv(d) ::b200k::make_fastdiv_t<::b200k::FastDiv>(d)
