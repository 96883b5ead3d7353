// Compiled-epilogue GEMM kernels with 128x256 tiles (4 pipeline stages),
// one per (activation, B layout, output width) combination the library ships.
#include "gemm_kernel.cuh"

namespace b200k {
namespace gemm {

template <int ACT>
static int launch_act(bool bnm, int ob, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                      const Params& p, int grid, cudaStream_t st) {
  if (bnm) return launch_one<256, 4, true, 2, true, ACT>(ta, tb, to, p, grid, st);
  return ob == 2 ? launch_one<256, 4, false, 2, true, ACT>(ta, tb, to, p, grid, st)
                 : launch_one<256, 4, false, 4, true, ACT>(ta, tb, to, p, grid, st);
}

int launch_fast_bn256(int act, bool bnm, int ob, const CUtensorMap& ta, const CUtensorMap& tb,
                      const CUtensorMap& to, const Params& p, int grid, cudaStream_t st) {
  if (!fast_combo_exists(act, bnm, ob)) return B200K_ERR_UNSUPPORTED;
  if (bnm && ob == 4) return launch_one<256, 4, true, 4, true, B200K_ACT_NONE>(ta, tb, to, p, grid, st);
  switch (act) {
    case B200K_ACT_NONE: return launch_act<B200K_ACT_NONE>(bnm, ob, ta, tb, to, p, grid, st);
    case B200K_ACT_GELU_ERF: return launch_act<B200K_ACT_GELU_ERF>(bnm, ob, ta, tb, to, p, grid, st);
    case B200K_ACT_GELU_TANH: return launch_act<B200K_ACT_GELU_TANH>(bnm, ob, ta, tb, to, p, grid, st);
    case B200K_ACT_SILU: return launch_act<B200K_ACT_SILU>(bnm, ob, ta, tb, to, p, grid, st);
    case B200K_ACT_TANH: return launch_act<B200K_ACT_TANH>(bnm, ob, ta, tb, to, p, grid, st);
    case B200K_ACT_RELU: return launch_act<B200K_ACT_RELU>(bnm, ob, ta, tb, to, p, grid, st);
    default: return B200K_ERR_UNSUPPORTED;
  }
}

// Which combinations have a compiled kernel: every activation except sigmoid
// for K-major B with 16- or 32-bit output and N-major B with 16-bit output;
// N-major B with fp32 output only without an activation.
bool fast_combo_exists(int act, bool bnm, int ob) {
  if (act < 0 || act >= B200K_ACT_COUNT || act == B200K_ACT_SIGMOID) return false;
  if (bnm && ob == 4) return act == B200K_ACT_NONE;
  return true;
}

}  // namespace gemm
}  // namespace b200k
