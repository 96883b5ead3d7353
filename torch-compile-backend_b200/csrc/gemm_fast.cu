// Compiled-epilogue GEMM kernels for one (tile width, activation) pair.  The
// build compiles this file once per pair, defining B200K_FAST_BN (256, 192 or 128)
// and B200K_FAST_ACT (a B200K_ACT_* value), so the instantiations compile in
// parallel.  Each object defines launch_fast_<BN>_<ACT>, which covers K-major
// B with 16-bit output and every row role, N-major B with 16-bit output and
// every row role, and K-major B with fp32 output without a row operand.
#include "gemm_kernel.cuh"

#if !defined(B200K_FAST_BN) || !defined(B200K_FAST_ACT)
#error "compile with -DB200K_FAST_BN=<256|192|128|2|4> -DB200K_FAST_ACT=<activation> (2, 4: the CTA-pair kernels)"
#endif

namespace b200k {
namespace gemm {

#if B200K_FAST_BN == 2 || B200K_FAST_BN == 4
// CTA-pair kernels, 16-bit output: B200K_FAST_BN 2 builds the 256 x 256 tiles
// (config 3, launch_pair_<ACT>), 4 the 256 x 512 tiles (config 4,
// launch_pairw_<ACT>).
constexpr bool kWide = B200K_FAST_BN == 4;
constexpr int kPairCfg = kWide ? 4 : 3;
static_assert(kConfigs[kPairCfg].bm == 2 * BM && kConfigs[kPairCfg].bn == (kWide ? 2 : 1) * kPairMmaN,
              "pair tile configs");
constexpr int kStages = kConfigs[kPairCfg].stages;
#if B200K_FAST_BN == 4
#define B200K_PAIR_FN2(ACT) launch_pairw_##ACT
#else
#define B200K_PAIR_FN2(ACT) launch_pair_##ACT
#endif
#define B200K_PAIR_FN(ACT) B200K_PAIR_FN2(ACT)
int B200K_PAIR_FN(B200K_FAST_ACT)(int row, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                                  const Params& p, int grid, cudaStream_t st) {
  constexpr int kAct = B200K_FAST_ACT;
  switch (row) {
    case ROW_NONE: return launch_pair<kStages, 2, kAct, ROW_NONE, kWide>(ta, tb, to, p, grid, st);
    case ROW_SCALE: return launch_pair<kStages, 2, kAct, ROW_SCALE, kWide>(ta, tb, to, p, grid, st);
    case ROW_RES: return launch_pair<kStages, 2, kAct, ROW_RES, kWide>(ta, tb, to, p, grid, st);
    case ROW_SCALE_PK: return launch_pair<kStages, 2, kAct, ROW_SCALE_PK, kWide>(ta, tb, to, p, grid, st);
    case ROW_RES_PK: return launch_pair<kStages, 2, kAct, ROW_RES_PK, kWide>(ta, tb, to, p, grid, st);
#if B200K_FAST_ACT == 0 && B200K_FAST_BN == 2
    case ROW_ROPE: return launch_pair<kStages, 2, kAct, ROW_ROPE, false>(ta, tb, to, p, grid, st);
#endif
    default: return B200K_ERR_UNSUPPORTED;
  }
}
#else
namespace {

constexpr int config_of(int bn) {
  for (int c = 0; c < kNumConfigs; ++c)
    if (kConfigs[c].bn == bn) return c;
  return -1;
}
constexpr int kBN = B200K_FAST_BN;
static_assert(config_of(kBN) >= 0, "B200K_FAST_BN is one of the tile configs");
constexpr int kStages = kConfigs[config_of(kBN)].stages;
constexpr int kAct = B200K_FAST_ACT;

template <bool BNM>
int launch_row16(int row, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, const Params& p,
                 int grid, cudaStream_t st) {
  switch (row) {
    case ROW_NONE: return launch_one<kBN, kStages, BNM, 2, true, kAct, ROW_NONE>(ta, tb, to, p, grid, st);
    case ROW_SCALE: return launch_one<kBN, kStages, BNM, 2, true, kAct, ROW_SCALE>(ta, tb, to, p, grid, st);
    case ROW_RES: return launch_one<kBN, kStages, BNM, 2, true, kAct, ROW_RES>(ta, tb, to, p, grid, st);
    case ROW_SCALE_PK: return launch_one<kBN, kStages, BNM, 2, true, kAct, ROW_SCALE_PK>(ta, tb, to, p, grid, st);
    case ROW_RES_PK: return launch_one<kBN, kStages, BNM, 2, true, kAct, ROW_RES_PK>(ta, tb, to, p, grid, st);
#if B200K_FAST_ACT == 0 && B200K_FAST_BN != 192
    // the rotary-embedding epilogue (K-major B; eight epilogue warps)
    case ROW_ROPE:
      if (BNM) return B200K_ERR_UNSUPPORTED;
      return launch_one<kBN, kStages, false, 2, true, kAct, ROW_ROPE>(ta, tb, to, p, grid, st);
#endif
    default: return B200K_ERR_UNSUPPORTED;
  }
}

}  // namespace

#define B200K_FAST_FN2(BN, ACT) launch_fast_##BN##_##ACT
#define B200K_FAST_FN(BN, ACT) B200K_FAST_FN2(BN, ACT)

int B200K_FAST_FN(B200K_FAST_BN, B200K_FAST_ACT)(bool tf32, bool bnm, int ob, int row, const CUtensorMap& ta,
                                                 const CUtensorMap& tb, const CUtensorMap& to, const Params& p,
                                                 int grid, cudaStream_t st) {
  if (tf32) {
    // fp32 operands (TF32 tensor cores): K-major B, fp32 output, no row
    // operand -- the compiled forms of an fp32 model's bias + activation
#if B200K_FAST_BN != 192
    if (!bnm && ob == 4 && row == ROW_NONE)
      return launch_one<kBN, kStages, false, 4, true, kAct, ROW_NONE, true>(ta, tb, to, p, grid, st);
#endif
    return B200K_ERR_UNSUPPORTED;
  }
  if (ob == 2) return bnm ? launch_row16<true>(row, ta, tb, to, p, grid, st)
                          : launch_row16<false>(row, ta, tb, to, p, grid, st);
  if (ob == 4 && !bnm && row == ROW_NONE)
    return launch_one<kBN, kStages, false, 4, true, kAct, ROW_NONE>(ta, tb, to, p, grid, st);
  return B200K_ERR_UNSUPPORTED;
}
#endif

}  // namespace gemm
}  // namespace b200k
