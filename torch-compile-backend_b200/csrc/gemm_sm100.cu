// GEMM + fused epilogue on the sm_100a tensor cores: host side (tensor maps,
// tile table, argument checks, launch) and the C ABI.  Device code lives in
// gemm_kernel.cuh; the compiled-epilogue instantiations in gemm_fast_*.cu.
#include "gemm_kernel.cuh"

namespace b200k {
namespace gemm {

// ----------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

CUtensorMapDataType tma_dtype(int dt) {
  switch (dt) {
    case B200K_BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    case B200K_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    default: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  }
}

// 2-d tiled map over a row-major view: `inner` elements contiguous, `outer`
// rows `row_bytes` apart; box = box_inner x box_outer; 128-byte swizzle.
bool encode_map(CUtensorMap* map, int dt, const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, tma_dtype(dt), 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Host cost per launch: a model's compiled graph calls the same GEMMs on the
// same buffers (weights, the caching allocator's recycled activations) over
// and over, so the encoded tensor maps and the verified epilogue forms are
// kept in small direct-mapped caches keyed on everything they depend on
// (a map is a pure function of its arguments; it holds no device state).
struct MapKey {
  const void* ptr;
  uint64_t inner, outer, row_bytes;
  uint32_t box_inner, box_outer;
  int32_t dt;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && inner == o.inner && outer == o.outer && row_bytes == o.row_bytes &&
           box_inner == o.box_inner && box_outer == o.box_outer && dt == o.dt;
  }
};

inline uint64_t mix64(uint64_t h, uint64_t v) {
  h ^= v + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
  return h;
}

bool make_map(CUtensorMap* map, int dt, const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_bytes,
              uint32_t box_inner, uint32_t box_outer) {
  constexpr int kSlots = 512;
  struct Slot {
    MapKey key;
    CUtensorMap map;
    bool used;
  };
  static Slot slots[kSlots];
  static std::mutex mu;
  const MapKey key{ptr, inner, outer, row_bytes, box_inner, box_outer, dt};
  uint64_t h = reinterpret_cast<uint64_t>(ptr);
  for (uint64_t v : {inner, outer, row_bytes, static_cast<uint64_t>(box_inner) << 32 | box_outer,
                     static_cast<uint64_t>(dt)})
    h = mix64(h, v);
  Slot& slot = slots[h % kSlots];
  {
    std::lock_guard<std::mutex> lock(mu);
    if (slot.used && slot.key == key) {
      *map = slot.map;
      return true;
    }
  }
  if (!encode_map(map, dt, ptr, inner, outer, row_bytes, box_inner, box_outer)) return false;
  std::lock_guard<std::mutex> lock(mu);
  slot.key = key;
  slot.map = *map;
  slot.used = true;
  return true;
}

// check_form with a cache of the (program, form, operand count) triples that
// passed: the probe evaluation runs once per distinct epilogue.
int check_form_cached(const B200kEpilogueForm& f, const B200kProgram& prog, int n_extras) {
  constexpr int kSlots = 256;
  struct Slot {
    B200kEpilogueForm form;
    B200kProgram prog;
    int n_extras;
    bool used;
  };
  static Slot slots[kSlots];
  static std::mutex mu;
  const int n = std::max(0, std::min<int>(prog.n, B200K_MAX_INSTR));
  uint64_t h = mix64(static_cast<uint64_t>(n_extras), static_cast<uint64_t>(n));
  for (int i = 0; i < n; ++i) {
    uint32_t bits;
    std::memcpy(&bits, &prog.ins[i].imm, 4);
    h = mix64(h, static_cast<uint64_t>(static_cast<uint32_t>(prog.ins[i].code)) << 32 | bits);
  }
  for (int v : {f.kind, f.bias, f.act, f.round, f.scale, f.residual}) h = mix64(h, static_cast<uint64_t>(v + 2));
  Slot& slot = slots[h % kSlots];
  auto same = [&](const Slot& s) {
    if (!s.used || s.n_extras != n_extras || s.prog.n != prog.n) return false;
    if (std::memcmp(&s.form, &f, sizeof(f)) != 0) return false;
    return std::memcmp(s.prog.ins, prog.ins, sizeof(B200kInstr) * n) == 0;
  };
  {
    std::lock_guard<std::mutex> lock(mu);
    if (same(slot)) return B200K_OK;
  }
  const int rc = check_form(f, prog, n_extras);
  if (rc == B200K_OK) {
    std::lock_guard<std::mutex> lock(mu);
    slot.form = f;
    std::memset(&slot.prog, 0, sizeof(slot.prog));
    slot.prog.n = prog.n;
    std::memcpy(slot.prog.ins, prog.ins, sizeof(B200kInstr) * n);
    slot.n_extras = n_extras;
    slot.used = true;
  }
  return rc;
}

template <int BN, int STAGES>
int launch_interp(bool tf32, bool amm, bool bnm, int ob, const CUtensorMap& ta, const CUtensorMap& tb,
                  const CUtensorMap& to, const Params& p, int grid, cudaStream_t st) {
  if (amm) {  // M-major A (16-bit): interpreted epilogues only
    if (tf32) return B200K_ERR_UNSUPPORTED;
    if (bnm)
      return ob == 2 ? launch_one<BN, STAGES, true, 2, false, -1, ROW_NONE, false, true>(ta, tb, to, p, grid, st)
                     : launch_one<BN, STAGES, true, 4, false, -1, ROW_NONE, false, true>(ta, tb, to, p, grid, st);
    return ob == 2 ? launch_one<BN, STAGES, false, 2, false, -1, ROW_NONE, false, true>(ta, tb, to, p, grid, st)
                   : launch_one<BN, STAGES, false, 4, false, -1, ROW_NONE, false, true>(ta, tb, to, p, grid, st);
  }
  if (tf32) {  // fp32 operands on TF32 tensor cores, K-major B
    if (bnm) return B200K_ERR_UNSUPPORTED;
    return ob == 2 ? launch_one<BN, STAGES, false, 2, false, -1, ROW_NONE, true>(ta, tb, to, p, grid, st)
                   : launch_one<BN, STAGES, false, 4, false, -1, ROW_NONE, true>(ta, tb, to, p, grid, st);
  }
  if (bnm) {
    return ob == 2 ? launch_one<BN, STAGES, true, 2, false, -1, ROW_NONE>(ta, tb, to, p, grid, st)
                   : launch_one<BN, STAGES, true, 4, false, -1, ROW_NONE>(ta, tb, to, p, grid, st);
  }
  return ob == 2 ? launch_one<BN, STAGES, false, 2, false, -1, ROW_NONE>(ta, tb, to, p, grid, st)
                 : launch_one<BN, STAGES, false, 4, false, -1, ROW_NONE>(ta, tb, to, p, grid, st);
}

int launch_fast(int bn, int act, bool tf32, bool bnm, int ob, int row, const CUtensorMap& ta, const CUtensorMap& tb,
                const CUtensorMap& to, const Params& p, int grid, cudaStream_t st) {
#define B200K_FAST_CASE(BN, ACT) \
  if (bn == BN && act == ACT) return launch_fast_##BN##_##ACT(tf32, bnm, ob, row, ta, tb, to, p, grid, st);
  B200K_FAST_CASE(256, 0)
  B200K_FAST_CASE(256, 1)
  B200K_FAST_CASE(256, 2)
  B200K_FAST_CASE(256, 3)
  B200K_FAST_CASE(256, 4)
  B200K_FAST_CASE(128, 0)
  B200K_FAST_CASE(128, 1)
  B200K_FAST_CASE(128, 2)
  B200K_FAST_CASE(128, 3)
  B200K_FAST_CASE(128, 4)
  B200K_FAST_CASE(192, 0)
  B200K_FAST_CASE(192, 1)
  B200K_FAST_CASE(192, 2)
  B200K_FAST_CASE(192, 3)
  B200K_FAST_CASE(192, 4)
#undef B200K_FAST_CASE
  return B200K_ERR_UNSUPPORTED;
}

int pick(int64_t M, int64_t N, int64_t K, int sms, bool compiled, bool pair_ok) {
  // Per-SM time of a config ~ (tiles per SM, rounded up) x (tile width) x
  // (cost per column).  Measured on B200 (bias + residual epilogue, 4096^3):
  // 128x256 tiles, 4 waves: 0.134 ms; 128x128 tiles, 7 waves: 0.173 ms, i.e.
  // the narrow tile does ~1.5x less work per unit time (it re-reads A twice as
  // often, runs the MMA at N=128 and pays the epilogue per tile twice).  The
  // 192-wide tile (compiled epilogues only) spreads its epilogue over twelve
  // warps and loses little per column; it wins where 256-wide tiles leave a
  // mostly idle last wave (N = 768: 297 tiles on 148 SMs = 3 waves, against
  // 396 tiles of 3/4 the work = 3 shorter waves).  A CTA pair's 256 x 256
  // tile gives each SM the work of one 128 x 256 tile with a third less
  // operand traffic per FLOP (the pair shares B): measured 8-15 % faster
  // from K = 2048 up (4096^3 1148 -> 1321 TFLOP/s, 16384 x 4096 x 14336 with
  // GELU 1342 -> 1502), no faster at K = 768, where the epilogue bounds a tile
  // and the 192-wide tile's twelve epilogue warps win; pairs need K >= 1536.
  // From K = 1536 the 192-wide tile is costed at 1.25 per column: there the
  // main loop, not the epilogue, bounds a tile, and its 128 x 192 share moves
  // more operand bytes per FLOP than a pair's.  Measured on B200 at 12608 x
  // 768 x 3072 (bias + residual), both in 3 waves: 128 x 192 tiles 72.7 us
  // (62 % of the per-SM MMA rate), 256 x 256 pair tiles 67.6 us (88 %).
  // The 256 x 512 pair tile moves 3/4 of the operand bytes per FLOP of the
  // 256 x 256 one, but its single accumulator makes each tile's MMAs wait
  // for the previous tile's epilogue (~10-20 us): measured on B200, 16384 x
  // 4096 x 14336 with GELU 1410.6 -> 1295.0 us, 8192^3 754.0 -> 759.3 us,
  // 4096^3 106.0 -> 122.6 us, so it is taken only from K = 12288 up.
  pair_ok = pair_ok && K >= 1536;
  int best = 0;
  double best_cost = 1e300;
  for (int c = 0; c < kNumConfigs; ++c) {
    const int bm = kConfigs[c].bm, bn = kConfigs[c].bn;
    const bool pair = bm == 2 * BM;
    const bool wide = pair && bn == 2 * kPairMmaN;
    if ((bn == 192 && !compiled) || (pair && !pair_ok) || (wide && K < 12288)) continue;
    const int64_t tiles = ((M + bm - 1) / bm) * ((N + bn - 1) / bn);
    const int64_t slots = pair ? sms / 2 : sms;  // tiles that run at once
    const int64_t waves = (tiles + slots - 1) / slots;
    const double per_col = wide ? 0.82 : pair ? 0.9 : (bn == 256 ? 1.0 : (bn == 192 ? (K >= 1536 ? 1.25 : 1.05) : 1.5));
    const double cost = static_cast<double>(waves) * bn * per_col;
    if (cost < best_cost) {
      best_cost = cost;
      best = c;
    }
  }
  return best;
}

int launch_pair(bool wide, int act, int row, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                const Params& p, int grid, cudaStream_t st) {
#define B200K_PAIR_CASE(ACT) \
  case ACT: return wide ? launch_pairw_##ACT(row, ta, tb, to, p, grid, st) : launch_pair_##ACT(row, ta, tb, to, p, grid, st);
  switch (act) {
    B200K_PAIR_CASE(0)
    B200K_PAIR_CASE(1)
    B200K_PAIR_CASE(2)
    B200K_PAIR_CASE(3)
    B200K_PAIR_CASE(4)
    default: return B200K_ERR_UNSUPPORTED;
  }
#undef B200K_PAIR_CASE
}

}  // namespace gemm

int device_sm_count() {
  static int cache[64] = {0};  // per device ordinal; SM counts never change
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (dev >= 0 && dev < 64) cache[dev] = sms;
  return sms;
}

}  // namespace b200k

using namespace b200k;
using namespace b200k::gemm;

extern "C" int b200k_gemm_num_configs(void) { return kNumConfigs; }

extern "C" int b200k_gemm_config_info(int config, int* block_m, int* block_n, int* block_k, int* stages) {
  if (config < 0 || config >= kNumConfigs) return B200K_ERR_ARG;
  if (block_m) *block_m = kConfigs[config].bm;
  if (block_n) *block_n = kConfigs[config].bn;
  if (block_k) *block_k = BK;
  if (stages) *stages = kConfigs[config].stages;
  return B200K_OK;
}

extern "C" int b200k_gemm_pick_config(int64_t M, int64_t N, int64_t K) {
  int sms = device_sm_count();
  if (sms <= 0) sms = 148;
  return pick(M, N, K, sms, true, true);
}

namespace {
int gemm_run(const B200kGemmArgs* a, const B200kRopeTables* rope, void* stream_);
}  // namespace

extern "C" int b200k_gemm_epilogue(const B200kGemmArgs* a, void* stream_) { return gemm_run(a, nullptr, stream_); }

extern "C" int b200k_gemm_rope(const B200kGemmArgs* a, const B200kRopeTables* r, void* stream_) {
  if (!a || !r) return B200K_ERR_ARG;
  if (a->n_extras != 0 || a->program.n != 0) return B200K_ERR_ARG;
  if (r->head_dim != 64 || r->period <= 0 || r->period > 0x7fffffff || !r->cos || !r->sin) return B200K_ERR_ARG;
  if (a->ab_dtype != B200K_BF16 && a->ab_dtype != B200K_F16) return B200K_ERR_UNSUPPORTED;
  if (a->out_dtype != a->ab_dtype || r->dtype != a->out_dtype) return B200K_ERR_UNSUPPORTED;
  if (a->N % 64 != 0) return B200K_ERR_SHAPE;
  if (!aligned16(r->cos) || !aligned16(r->sin) || r->stride % 8 != 0) return B200K_ERR_ALIGN;
  if (a->b_stride_k != 1 || (a->a_stride_k != 1 && a->K > 1)) return B200K_ERR_UNSUPPORTED;
  return gemm_run(a, r, stream_);
}

namespace {
int gemm_run(const B200kGemmArgs* a, const B200kRopeTables* rope, void* stream_) {
  if (!a) return B200K_ERR_ARG;
  if (a->M < 0 || a->N < 0 || a->K < 0) return B200K_ERR_SHAPE;
  if (a->M == 0 || a->N == 0) return B200K_OK;  // empty output: nothing to launch
  if (!a->a || !a->b || !a->out) return B200K_ERR_ARG;
  if (a->K == 0) return B200K_ERR_SHAPE;
  if (a->M > 0x7fffffff || a->N > 0x7fffffff || a->K > 0x7fffffff) return B200K_ERR_SHAPE;
  // fp32 operands run on the TF32 tensor cores (the caller passes them only
  // where TF32 is allowed, as torch's allow_tf32 governs cuBLAS)
  if (a->ab_dtype != B200K_BF16 && a->ab_dtype != B200K_F16 && a->ab_dtype != B200K_F32)
    return B200K_ERR_UNSUPPORTED;
  const bool tf32 = a->ab_dtype == B200K_F32;
  const int eb = tf32 ? 4 : 2;  // operand element bytes
  if (a->out_dtype != B200K_BF16 && a->out_dtype != B200K_F16 && a->out_dtype != B200K_F32)
    return B200K_ERR_UNSUPPORTED;
  if (a->n_extras < 0 || a->n_extras > B200K_MAX_INPUTS - 1) return B200K_ERR_ARG;
  int rc = validate_program(a->program, 1 + a->n_extras);
  if (rc != B200K_OK) return rc;
  if (a->form.kind != 0) {
    rc = check_form_cached(a->form, a->program, a->n_extras);
    if (rc != B200K_OK) return rc;
  }

  // A: [M, K], K-major (unit K stride, rows 16-byte aligned) or M-major
  // (unit M stride, 16-bit only: the transposed operand of a weight-gradient
  // GEMM).
  bool amm;
  if (a->a_stride_k == 1 || a->K == 1) {
    amm = false;
    if (!aligned16(a->a) || (a->a_stride_m * eb) % 16 != 0) return B200K_ERR_ALIGN;
  } else if (a->a_stride_m == 1 && !tf32) {
    amm = true;
    if (!aligned16(a->a) || (a->a_stride_k * eb) % 16 != 0) return B200K_ERR_ALIGN;
  } else {
    return B200K_ERR_UNSUPPORTED;
  }
  // B: K-major (unit K stride) or N-major (unit N stride; 16-bit only).
  bool bnm;
  if (a->b_stride_k == 1) {
    bnm = false;
    if (!aligned16(a->b) || (a->b_stride_n * eb) % 16 != 0) return B200K_ERR_ALIGN;
  } else if (a->b_stride_n == 1 && !tf32) {
    bnm = true;
    if (!aligned16(a->b) || (a->b_stride_k * eb) % 16 != 0) return B200K_ERR_ALIGN;
  } else {
    return B200K_ERR_UNSUPPORTED;
  }
  if (a->out_stride_n != 1 && a->N > 1) return B200K_ERR_UNSUPPORTED;
  for (int i = 0; i < a->n_extras; ++i) {
    if (!a->extras[i].ptr) return B200K_ERR_ARG;
    if (!valid_dtype(a->extras[i].dtype)) return B200K_ERR_UNSUPPORTED;
  }

  const int ob = a->out_dtype == B200K_F32 ? 4 : 2;
  auto mode_of = [&](int idx, bool allow_row) -> int32_t {
    if (idx < 0) return XM_NONE;
    const B200kEpiOperand& e = a->extras[idx];
    const bool f_or_16 = e.dtype == B200K_F32 || e.dtype == B200K_BF16 || e.dtype == B200K_F16;
    if (e.stride_m == 0) return f_or_16 ? XM_BCAST : XM_GENERIC;
    if (allow_row && e.stride_n == 1 && (e.dtype == B200K_BF16 || e.dtype == B200K_F16) && aligned16(e.ptr) &&
        e.stride_m % 8 == 0)
      return XM_ROW16;
    return XM_GENERIC;
  };
  // Compiled path: canonical form, output storable by TMA, a row-broadcast
  // bias (or none), at most one of scale and residual as a full 16-bit
  // matrix of the output's type, and an activation with compiled kernels.
  const bool tma_out = aligned16(a->out) && (a->out_stride_m * ob) % 16 == 0;
  const int role_idx = a->form.residual >= 0 ? a->form.residual : a->form.scale;
  const bool both = a->form.residual >= 0 && a->form.scale >= 0;
  bool act_ok = false;
  for (int fa : kFastActs) act_ok = act_ok || fa == a->form.act;
  const bool row_ok = role_idx < 0 || (ob == 2 && mode_of(role_idx, true) == XM_ROW16 &&
                                       a->extras[role_idx].dtype == a->out_dtype);
  const int bias_mode = mode_of(a->form.bias, false);
  const bool fast = rope ? tma_out
                         : a->form.kind == 1 && tma_out && act_ok && !both && row_ok && !(bnm && ob == 4) && !amm &&
                               (bias_mode == XM_NONE || bias_mode == XM_BCAST);
  if (rope && !fast) return B200K_ERR_ALIGN;  // the rotary epilogue stores with TMA only

  const bool pair_ok = fast && !bnm && ob == 2 && !tf32;  // the CTA-pair kernels' domain

  const int sms = device_sm_count();
  if (sms <= 0) return B200K_ERR_DEVICE;
  int cfg = a->tile_config;
  if (cfg < 0) cfg = pick(a->M, a->N, a->K, sms, fast, pair_ok);
  if (cfg >= kNumConfigs) return B200K_ERR_ARG;
  if (kConfigs[cfg].bn == 192 && (!fast || tf32)) cfg = 0;  // 192-wide tiles: compiled 16-bit epilogues only
  if (kConfigs[cfg].bm == 2 * BM && !pair_ok) cfg = 0;
  if (rope && kConfigs[cfg].bn == 192) cfg = 0;  // the rotary epilogue runs on eight-warp tiles
  if (rope && kConfigs[cfg].bn == 2 * kPairMmaN) cfg = 3;  // and on narrow pair tiles
  const int bn = kConfigs[cfg].bn;
  const int bm = kConfigs[cfg].bm;
  const bool pair = bm == 2 * BM;
  const bool wide = pair && bn == 2 * kPairMmaN;
  const int mma_n = pair ? kPairMmaN : bn;  // N of one tcgen05.mma

  Params p;
  std::memset(&p, 0, sizeof(p));
  p.M = static_cast<int32_t>(a->M);
  p.N = static_cast<int32_t>(a->N);
  p.K = static_cast<int32_t>(a->K);
  p.tiles_m = static_cast<int32_t>((a->M + bm - 1) / bm);
  p.tiles_n = static_cast<int32_t>((a->N + bn - 1) / bn);
  const int64_t tiles = static_cast<int64_t>(p.tiles_m) * p.tiles_n;
  if (tiles > 0x7fffffff) return B200K_ERR_SHAPE;
  p.num_tiles = static_cast<int32_t>(tiles);
  const int kb_elems = tf32 ? BK / 2 : BK;  // a K block is 128 bytes of each operand row
  p.k_blocks = static_cast<int32_t>((a->K + kb_elems - 1) / kb_elems);
  p.n_extras = a->n_extras;
  p.out_dt = a->out_dtype;
  p.out = a->out;
  p.out_sm = a->out_stride_m;
  p.status = a->status;
  p.timeout_ns = a->timeout_ns > 0 ? a->timeout_ns : 2000000000ll;
  p.test_flags = a->test_flags;
  // operand format of the instruction descriptor: f16 0 / bf16 1 (kind::f16), tf32 2 (kind::tf32)
  const uint32_t fmt = tf32 ? 2u : (a->ab_dtype == B200K_BF16 ? 1u : 0u);
  p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((amm ? 1u : 0u) << 15) | ((bnm ? 1u : 0u) << 16) |
            (static_cast<uint32_t>(mma_n >> 3) << 17) | (static_cast<uint32_t>(bm >> 4) << 24);
  p.group_m = pair ? kGroupMPair : kGroupM;
  for (int i = 0; i < a->n_extras; ++i) {
    const B200kEpiOperand& e = a->extras[i];
    EpiOperand& q = p.ex[i];
    q.ptr = e.ptr;
    q.sm = e.stride_m;
    q.sn = e.stride_n;
    q.dt = e.dtype;
    const int dt = e.dtype;
    q.vec = (e.stride_n == 1 && aligned16(e.ptr) && e.stride_m % 8 == 0 &&
             (dt == B200K_BF16 || dt == B200K_F16 || dt == B200K_F32))
                ? 1
                : 0;
  }
  p.prog = a->program;
  p.f_bias = a->form.bias;
  p.f_act = a->form.act;
  p.f_round = a->form.round;
  p.f_scale = a->form.scale;
  p.f_res = a->form.residual;
  p.xm_bias = bias_mode;
  if (a->form.bias >= 0) {
    const B200kEpiOperand& e = a->extras[a->form.bias];
    p.bias_ptr = e.ptr;
    p.bias_sn = e.stride_n;
    p.bias_dt = e.dtype;
  }
  p.xm_scale = mode_of(a->form.scale, true);
  p.xm_res = mode_of(a->form.residual, true);
  p.trace = nullptr;

  CUtensorMap ta, tb, to;
  std::memset(&to, 0, sizeof(to));
  if (amm) {
    if (!make_map(&ta, a->ab_dtype, a->a, a->M, a->K, a->a_stride_k * eb, 64, BK)) return B200K_ERR_LAUNCH;
  } else {
    if (!make_map(&ta, a->ab_dtype, a->a, a->K, a->M, a->a_stride_m * eb, kb_elems, BM)) return B200K_ERR_LAUNCH;
  }
  if (bnm) {
    if (!make_map(&tb, a->ab_dtype, a->b, a->N, a->K, a->b_stride_k * eb, 64, BK)) return B200K_ERR_LAUNCH;
  } else {
    // a CTA of a pair loads its half of each MMA's B rows
    if (!make_map(&tb, a->ab_dtype, a->b, a->K, a->N, a->b_stride_n * eb, kb_elems, pair ? kPairMmaN / 2 : bn))
      return B200K_ERR_LAUNCH;
  }
  p.direct_store = tma_out ? 0 : 1;
  if (tma_out) {
    if (!make_map(&to, a->out_dtype, a->out, a->N, a->M, a->out_stride_m * ob, 128 / ob, 32)) return B200K_ERR_LAUNCH;
  }
  const int grid = pair ? 2 * static_cast<int>(std::min<int64_t>(tiles, sms / 2))
                        : static_cast<int>(std::min<int64_t>(tiles, sms));
  if (a->trace && a->trace_words >= static_cast<int64_t>(grid) * B200K_GEMM_TRACE_WORDS)
    p.trace = reinterpret_cast<unsigned long long*>(a->trace);
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  if (rope) {
    p.f_bias = -1;
    p.rope_cos = rope->cos;
    p.rope_sin = rope->sin;
    p.rope_stride = rope->stride;
    p.rope_period = static_cast<int32_t>(rope->period);
    if (pair) return launch_pair(false, B200K_ACT_NONE, ROW_ROPE, ta, tb, to, p, grid, st);
    return launch_fast(bn, B200K_ACT_NONE, false, false, ob, ROW_ROPE, ta, tb, to, p, grid, st);
  }
  if (fast) {
    int row = ROW_NONE;
    if (role_idx >= 0) {
      const bool packed = a->form.round == a->out_dtype;  // round to the output type, then the 16-bit op
      const bool res = a->form.residual >= 0;
      row = res ? (packed ? ROW_RES_PK : ROW_RES) : (packed ? ROW_SCALE_PK : ROW_SCALE);
      p.row_idx = role_idx;
      p.row_ptr = a->extras[role_idx].ptr;
      p.row_sm = a->extras[role_idx].stride_m;
    } else if (a->form.round == a->out_dtype) {
      p.f_round = -1;  // the store's own rounding is the same one
    }
    if (pair) return launch_pair(wide, a->form.act, row, ta, tb, to, p, grid, st);
    const int rc = launch_fast(bn, a->form.act, tf32, bnm, ob, row, ta, tb, to, p, grid, st);
    if (rc != B200K_ERR_UNSUPPORTED || !tf32) return rc;
    // TF32 forms without a compiled kernel (a row operand, 16-bit output) interpret the program
  }
  if (cfg == 0 || bn == 192) return launch_interp<256, 4>(tf32, amm, bnm, ob, ta, tb, to, p, grid, st);
  return launch_interp<128, 6>(tf32, amm, bnm, ob, ta, tb, to, p, grid, st);
}
}  // namespace

// ---------------------------------------------------------------------------
// Allocation-free entry (see b200k.h): the status word lives in this
// file-scope array instead of caller memory.  In host code the name below is
// only a host-side stand-in; the device address comes from
// cudaGetSymbolAddress, looked up once per device with that device current.
// ---------------------------------------------------------------------------
static __device__ __align__(256) int32_t g_noalloc_scratch[B200K_NOALLOC_SCRATCH_BYTES / sizeof(int32_t)];

namespace {
// Device address of this device's copy of g_noalloc_scratch, looked up on the
// first use per device with that device current.  The lookup may load the
// library's module into the context, which is not a stream operation, so it
// is refused while `st` is capturing (B200K_ERR_LAUNCH, nothing enqueued).
// The cache lives for the process: cudaDeviceReset invalidates it.
int noalloc_scratch(cudaStream_t st, void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return B200K_ERR_DEVICE;
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return B200K_ERR_LAUNCH;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return B200K_ERR_LAUNCH;
    addr[dev] = p;
  }
  *out = addr[dev];
  return B200K_OK;
}
}  // namespace

extern "C" int b200k_gemm_epilogue_noalloc(const B200kGemmArgs* args, void* stream_) {
  if (!args) return B200K_ERR_ARG;
  const size_t need = B200K_NOALLOC_STATUS_BYTES;  // one status word per call
  if (need > sizeof(g_noalloc_scratch)) return B200K_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  void* scratch = nullptr;
  const int rc = noalloc_scratch(st, &scratch);
  if (rc != B200K_OK) return rc;
  if (cudaMemsetAsync(scratch, 0, need, st) != cudaSuccess) return B200K_ERR_LAUNCH;
  B200kGemmArgs a = *args;
  a.status = static_cast<int32_t*>(scratch);
  return b200k_gemm_epilogue(&a, stream_);
}

extern "C" int b200k_gemm_noalloc_status(int32_t* host_out, void* stream_) {
  if (!host_out) return B200K_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  void* scratch = nullptr;
  const int rc = noalloc_scratch(st, &scratch);
  if (rc != B200K_OK) return rc;
  if (cudaMemcpyAsync(host_out, scratch, sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return B200K_ERR_LAUNCH;
  return cudaStreamSynchronize(st) == cudaSuccess ? B200K_OK : B200K_ERR_LAUNCH;
}
