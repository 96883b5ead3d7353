// Host-side helpers shared by the libb200k entry points.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

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

int device_sm_count();

}  // namespace b200k

#define make_fastdiv(d) ::b200k::make_fastdiv_t<::b200k::FastDiv>(d)
