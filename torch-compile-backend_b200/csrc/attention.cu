// Fused attention forward on the sm_100a tensor cores (b200k_attention).
//
//   out[b, h, i, :] = sum_j softmax_j(scale * q_i . k_j) v_j,  k, v of kv head h / G
//
// The reference leaves attention to ATen (compiler/optimization/
// fusion_pointwise.py:12-30 has no attention op; the graph keeps
// aten._scaled_dot_product_*_attention, i.e. cuDNN / flash kernels).  This
// kernel replaces that node for head_dim 64, bf16 / f16, with or without the
// causal mask, for multi-head and grouped-query attention.
//
// One CTA per (batch, head, 256 query rows), 384 threads:
//   warp 0      TMA producer: the CTA's two 128-row query tiles once, then
//               128-row key and value blocks into a kStages-deep ring;
//   warps 1, 3  MMA issuers (one thread each, for query tile 0 and 1):
//               S_t = Q_t K^T into tensor memory (tcgen05.mma M=128, N=128,
//               K=64) and O_t += P_t V (M=128, N=64, K=128, V read N-major
//               from its TMA tile);
//   warp 2      owns the tensor-memory allocation (S of both tiles, O of
//               both tiles: 384 of 512 columns);
//   warps 4-7   softmax of query tile 0, warps 8-11 of tile 1: one thread per
//               query row reads its 128 scores from tensor memory, applies
//               the mask, keeps the running max and sum, writes the
//               probabilities as 16-bit values into a swizzled shared-memory
//               tile (the A operand of the second MMA) and, when the running
//               max moved by more than 2^8, rescales its row of O in tensor
//               memory.  At the end it divides O by the sum and stores it.
// The MMA thread issues the next block's S_t as soon as the softmax has
// loaded the current one, so the scores of block j+1 are computed while the
// exponentials of block j run; the two query tiles share every K/V load.
// Every wait is bounded, as in the GEMM kernel: on timeout the kernel sets
// B200K_ERR_TIMEOUT in the status word, drains and returns.
#include "gemm_kernel.cuh"

namespace b200k {
namespace gemm {
// Host helpers defined with the GEMM's host code (gemm_sm100.cu).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn();
CUtensorMapDataType tma_dtype(int dt);
}  // namespace gemm

namespace attn {

using gemm::Ctl;
using gemm::smem_u32;

constexpr int kD = 64;       // head dim: one 128-byte swizzle row of 16-bit values
constexpr int kBQ = 128;     // query rows per tile (MMA M)
constexpr int kBKV = 128;    // key / value rows per block
constexpr int kStages = 2;   // K/V ring depth
constexpr int kThreads = 384;
constexpr uint32_t kTileBytes = kBQ * kD * 2;  // 16 KB: a Q tile, a K block or a V block
constexpr uint32_t kPBytes = kBQ * kBKV * 2;   // 32 KB: one tile's probabilities (two swizzle columns)
constexpr uint32_t kOffQ = 0;                        // 2 items x 2 query tiles
constexpr uint32_t kOffK = kOffQ + 4 * kTileBytes;
constexpr uint32_t kOffV = kOffK + kStages * kTileBytes;
constexpr uint32_t kOffP = kOffV + kStages * kTileBytes;
constexpr uint32_t kOffBar = kOffP + 2 * kPBytes;
constexpr uint32_t kSmem = 1024 + kOffBar + 256;
static_assert(kSmem <= 232448, "shared memory budget");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemO = 256;            // O of tile t at column 256 + 64 t
constexpr float kRescaleLog2 = 8.0f;        // lazy rescale threshold (a factor of 256)
// Register split (setmaxnreg): the kernel is compiled for kLaunchRegs per
// thread (384 threads: 64512 registers); the control warpgroup (warps 0-3)
// drops to kCtlRegs and each softmax warpgroup rises to kSoftmaxRegs (a
// softmax thread holds its row's 128 scores), which needs
// 2 x 128 x (200 - 168) = 8192 of the 128 x (168 - 104) = 8192 the control
// warpgroup returns.  The host launches only when the compiled register
// count is kLaunchRegs (cudaFuncGetAttributes).
constexpr int kLaunchRegs = 168;
constexpr int kCtlRegs = 104;
constexpr int kSoftmaxRegs = 200;
static_assert(128 * kCtlRegs + 256 * kSoftmaxRegs <= kThreads * kLaunchRegs, "register split exceeds the launch");
constexpr float kLog2e = 1.4426950408889634f;

struct Params {
  int32_t B, H, group, Sq, Skv;
  int32_t n_ctiles;  // ceil(Sq / 256)
  int32_t causal;
  int32_t half;      // 1: f16, 0: bf16
  float scale_log2;
  int32_t test_flags;
  void* out;
  int64_t os_b, os_h, os_s;
  uint32_t idesc_s, idesc_pv;
  int32_t* status;
  int64_t timeout_ns;
};

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// 32 lanes x 32 bit, 32 consecutive columns, register -> tensor memory.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ uint32_t pack2(float a, float b, bool half) {
  uint32_t u;
  if (half) {
    __half2 h = __floats2half2_rn(a, b);
    u = *reinterpret_cast<uint32_t*>(&h);
  } else {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    u = *reinterpret_cast<uint32_t*>(&h);
  }
  return u;
}

// A bounded wait whose outcome is the same for the whole warp, so that no
// lane leaves for the timeout path while the others go on to the
// warp-collective tensor-memory instructions.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, const Ctl& c) {
  const bool ok = gemm::wait_bar(bar, parity, c);
  return __all_sync(0xffffffffu, ok);
}

// Query rows [q0, q0 + 128) need key blocks [0, n): every block with a
// column <= the tile's last row under the causal mask, all blocks without.
__device__ __forceinline__ int blocks_for(int q0, const Params& p) {
  if (q0 >= p.Sq) return 0;
  const int nkv = (p.Skv + kBKV - 1) / kBKV;
  if (!p.causal) return nkv;
  const int last_row = min(q0 + kBQ - 1, p.Sq - 1);
  return min(nkv, last_row / kBKV + 1);
}

// One work item: a (batch, head) and 256 query rows (two tiles).  Items are
// numbered heaviest first under the causal mask (the last query rows of
// every head), and CTA c takes items c, c + grid, c + 2 grid, ...
struct Item {
  int b, h, hk;
  int q0[2];
  int n[2];   // key blocks per tile
  int n_all;  // key blocks loaded for the item
};

__device__ __forceinline__ Item item_at(int w, const Params& p) {
  Item it;
  const int bh_count = p.B * p.H;
  const int bh = w % bh_count;
  const int ci = p.n_ctiles - 1 - w / bh_count;
  it.b = bh / p.H;
  it.h = bh - it.b * p.H;
  it.hk = it.h / p.group;
  it.q0[0] = ci * 2 * kBQ;
  it.q0[1] = it.q0[0] + kBQ;
  it.n[0] = blocks_for(it.q0[0], p);
  it.n[1] = blocks_for(it.q0[1], p);
  it.n_all = max(it.n[0], it.n[1]);
  return it;
}

__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* sbase = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sQ = sbase + kOffQ;  // two items' query tiles (by item parity)
  uint8_t* sK = sbase + kOffK;
  uint8_t* sV = sbase + kOffV;
  uint8_t* sP = sbase + kOffP;
  uint64_t* q_full = reinterpret_cast<uint64_t*>(sbase + kOffBar);  // [2] by item parity
  uint64_t* q_empty = q_full + 2;                                    // [2]
  uint64_t* kv_full = q_empty + 2;
  uint64_t* kv_empty = kv_full + kStages;
  uint64_t* s_full = kv_empty + kStages;  // [2] by query tile
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* o_done = p_full + 2;
  uint64_t* o_free = o_done + 2;
  uint64_t* drain = o_free + 2;  // [2] by MMA thread
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_items = p.n_ctiles * p.B * p.H;
  const int first = static_cast<int>(blockIdx.x);
  const int step = static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      gemm::mbar_init(&q_full[i], 1);
      gemm::mbar_init(&q_empty[i], 2);  // both tiles' MMA threads
    }
    for (int s = 0; s < kStages; ++s) {
      gemm::mbar_init(&kv_full[s], 1);
      gemm::mbar_init(&kv_empty[s], 2);
    }
    for (int t = 0; t < 2; ++t) {
      gemm::mbar_init(&s_full[t], 1);
      gemm::mbar_init(&s_free[t], 4);
      gemm::mbar_init(&p_full[t], 4);
      gemm::mbar_init(&o_done[t], 1);
      gemm::mbar_init(&o_free[t], 4);
    }
    gemm::mbar_init(&drain[0], 1);
    gemm::mbar_init(&drain[1], 1);
    *abort_flag = 0;
    gemm::fence_mbar_init();
  }
  if (warp == 2) {
    gemm::tmem_alloc(tmem_slot, kTmemCols);
    gemm::tmem_relinquish();
  }
  gemm::tc_fence_before();
  __syncthreads();
  gemm::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const Ctl ctl{abort_flag, p.status, static_cast<uint64_t>(p.timeout_ns)};
  if (warp < 4) {
  regs_dec<kCtlRegs>();
  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      gemm::prefetch_map(&tmQ);
      gemm::prefetch_map(&tmK);
      gemm::prefetch_map(&tmV);
      int kvc = 0;  // K/V blocks issued, over all items
      int li = 0;   // this CTA's item count
      bool ok = true;
      for (int w = first; w < n_items && ok; w += step, ++li) {
        const Item it = item_at(w, p);
        const int qb = li & 1;
        if (li >= 2 && !gemm::wait_bar(&q_empty[qb], static_cast<uint32_t>(li / 2 - 1) & 1u, ctl)) break;
        gemm::mbar_arrive_expect_tx(&q_full[qb], 2 * kTileBytes);
        tma_load_4d(sQ + qb * 2 * kTileBytes, &tmQ, &q_full[qb], 0, it.q0[0], it.h, it.b);
        tma_load_4d(sQ + qb * 2 * kTileBytes + kTileBytes, &tmQ, &q_full[qb], 0, it.q0[1], it.h, it.b);
        for (int j = 0; j < it.n_all; ++j, ++kvc) {
          const int s = kvc % kStages;
          if (!gemm::wait_bar(&kv_empty[s], (static_cast<uint32_t>(kvc / kStages) & 1u) ^ 1u, ctl)) {
            ok = false;
            break;
          }
          gemm::mbar_arrive_expect_tx(&kv_full[s], 2 * kTileBytes);
          tma_load_4d(sK + s * kTileBytes, &tmK, &kv_full[s], 0, j * kBKV, it.hk, it.b);
          tma_load_4d(sV + s * kTileBytes, &tmV, &kv_full[s], 0, j * kBKV, it.hk, it.b);
        }
        if (!ok) {
          ++li;
          break;
        }
      }
      // Every load lands before the CTA can exit (after a timeout elsewhere
      // the consumers may not have waited for them; otherwise these phases
      // are complete already).
      for (int i = max(0, li - 2); i < li; ++i)
        gemm::wait_bar_drain(&q_full[i & 1], static_cast<uint32_t>(i / 2) & 1u, 100000000ull);
      for (int k = max(0, kvc - kStages); k < kvc; ++k)
        gemm::wait_bar_drain(&kv_full[k % kStages], static_cast<uint32_t>(k / kStages) & 1u, 100000000ull);
    }
    __syncwarp();
  } else if (warp == 1 || warp == 3) {
    // ---------------------------------------------------------------- MMA issuers
    // One thread per query tile (warp 1: tile 0, warp 3: tile 1), so each
    // tile's products follow its own softmax and neither waits for the
    // other's.  Each thread's tcgen05.commit tracks only its own MMAs; the
    // K/V and Q buffers are released when both tiles' threads have arrived.
    if (lane == 0) {
      const int t = warp == 1 ? 0 : 1;
      bool ok = true;
      int kv_ready = -1;  // highest K/V block (over all items) waited for
      int q_ready = -1;   // highest item whose query tiles were waited for
      int gs = 0;         // score blocks issued for this tile, over all items
      int gp = 0;         // P V products issued
      int items_done = 0; // items whose last product was issued
      bool s0_ready = false;  // block 0 of the current item's scores issued
      auto ensure_kv = [&](int g) -> bool {
        while (kv_ready < g) {
          ++kv_ready;
          if (!gemm::wait_bar(&kv_full[kv_ready % kStages], static_cast<uint32_t>(kv_ready / kStages) & 1u, ctl))
            return false;
        }
        return true;
      };
      auto ensure_q = [&](int li) -> bool {
        while (q_ready < li) {
          ++q_ready;
          if (!gemm::wait_bar(&q_full[q_ready & 1], static_cast<uint32_t>(q_ready / 2) & 1u, ctl)) return false;
        }
        return true;
      };
      // Scores of this tile of item li against K/V block g (over all items).
      auto issue_s = [&](int li, int g) -> bool {
        if (!ensure_q(li) || !ensure_kv(g)) return false;
        if (gs > 0 && !gemm::wait_bar(&s_free[t], static_cast<uint32_t>(gs - 1) & 1u, ctl)) return false;
        gemm::tc_fence_after();
        const uint32_t a0 = smem_u32(sQ + (li & 1) * 2 * kTileBytes + t * kTileBytes);
        const uint32_t b0 = smem_u32(sK + (g % kStages) * kTileBytes);
#pragma unroll
        for (int k = 0; k < kD / gemm::UMMA_K; ++k)
          gemm::umma_f16(tmem_base + static_cast<uint32_t>(t * kBKV), gemm::sw128_desc(a0 + k * 32, 16, 1024),
                         gemm::sw128_desc(b0 + k * 32, 16, 1024), p.idesc_s, k != 0 ? 1u : 0u);
        if (!(t == 0 && gs == 0 && (p.test_flags & B200K_ATTN_TEST_WITHHOLD_SCORES))) gemm::umma_commit(&s_full[t]);
        ++gs;
        return true;
      };
      int kvbase = 0;  // index of the current item's block 0 among all K/V blocks
      int li = 0;
      for (int w = first; w < n_items && ok; w += step, ++li) {
        const Item it = item_at(w, p);
        const int n = t ? it.n[1] : it.n[0];
        const bool has_next = w + step < n_items;
        int n_next = 0;
        if (has_next) {
          const Item nx = item_at(w + step, p);
          n_next = t ? nx.n[1] : nx.n[0];
        }
        const int kvnext = kvbase + it.n_all;
        bool s0_next = false;
        if (n > 0 && !s0_ready) ok = issue_s(li, kvbase);
        for (int j = 0; j < it.n_all && ok; ++j) {
          if (j < n) {
            // the next scores: block j + 1, or the next item's block 0 while
            // this item finishes (once that block's ring slot is free)
            if (j + 1 < n) {
              ok = issue_s(li, kvbase + j + 1);
            } else if (has_next && n_next > 0 && kvnext - kStages <= kvbase + j - 1) {
              ok = issue_s(li + 1, kvnext);
              s0_next = ok;
            }
            if (!ok) break;
            // O of the previous item has been read out before the first
            // product of this one overwrites it
            if (j == 0 && items_done > 0 &&
                !gemm::wait_bar(&o_free[t], static_cast<uint32_t>(items_done - 1) & 1u, ctl)) {
              ok = false;
              break;
            }
            if (!gemm::wait_bar(&p_full[t], static_cast<uint32_t>(gp) & 1u, ctl)) {
              ok = false;
              break;
            }
            gemm::tc_fence_after();
            const uint32_t a0 = smem_u32(sP + t * kPBytes);
            const uint32_t b0 = smem_u32(sV + ((kvbase + j) % kStages) * kTileBytes);
#pragma unroll
            for (int k = 0; k < kBKV / gemm::UMMA_K; ++k)
              gemm::umma_f16(tmem_base + kTmemO + static_cast<uint32_t>(t * kD),
                             gemm::sw128_desc(a0 + (k >> 2) * (kBQ * 128) + (k & 3) * 32, 16, 1024),
                             gemm::sw128_desc(b0 + k * (gemm::UMMA_K * 128), kTileBytes, 1024), p.idesc_pv,
                             (j | k) != 0 ? 1u : 0u);
            gemm::umma_commit(&o_done[t]);
            ++gp;
            if (j + 1 == n) ++items_done;
            gemm::umma_commit(&kv_empty[(kvbase + j) % kStages]);  // this tile's reads of block j
          } else {
            // This tile does not read block j.  Its arrival waits for the
            // block's load, so that it can never complete a later phase of
            // the slot's barrier while the other tile still reads this one.
            ok = ensure_kv(kvbase + j);
            if (!ok) break;
            gemm::mbar_arrive(&kv_empty[(kvbase + j) % kStages]);
          }
        }
        if (!ok) break;
        if (n > 0) {
          gemm::umma_commit(&q_empty[li & 1]);  // this tile's score products of item li
        } else {
          if (!ensure_q(li)) break;  // (as above: never ahead of the buffer's current phase)
          gemm::mbar_arrive(&q_empty[li & 1]);
        }
        s0_ready = s0_next;
        kvbase = kvnext;
      }
      // Every MMA this thread issued completes before tensor memory is freed.
      gemm::umma_commit(&drain[t]);
      gemm::wait_bar_drain(&drain[t], 0, 100000000ull);
    }
    __syncwarp();
  }
  } else {
    regs_inc<kSoftmaxRegs>();
    // ---------------------------------------------------------------- softmax
    const int t = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    uint8_t* pt = sP + t * kPBytes;
    const bool half = p.half != 0;
    int g = 0;  // score blocks consumed by this tile, over all items
    bool ok = true;
    for (int w = first; w < n_items && ok; w += step) {
      const Item it = item_at(w, p);
      const int n = t ? it.n[1] : it.n[0];
      if (n == 0) continue;
      const int q0t = t ? it.q0[1] : it.q0[0];
      const int row = q0t + r;
      float m = 0.0f, l = 0.0f;  // running max (log2 domain, scaled) and sum
      for (int j = 0; j < n; ++j, ++g) {
        if (!warp_wait(&s_full[t], static_cast<uint32_t>(g) & 1u, ctl)) {
          ok = false;
          break;
        }
        gemm::tc_fence_after();
        float s[kBKV];
        {
          uint32_t raw[4][32];
#pragma unroll
          for (int c = 0; c < 4; ++c) gemm::tmem_ld32(t_lane + static_cast<uint32_t>(t * kBKV + c * 32), raw[c]);
          gemm::tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(raw[c][i]);
        }
        gemm::tc_fence_before();
        __syncwarp();
        if (lane == 0) gemm::mbar_arrive(&s_free[t]);
        const int col0 = j * kBKV;
        if (col0 + kBKV > p.Skv || (p.causal && col0 + kBKV - 1 > q0t)) {  // warp-uniform
          const int lim = (p.causal ? min(p.Skv - 1, row) : p.Skv - 1) - col0;
#pragma unroll
          for (int c = 0; c < kBKV; ++c)
            if (c > lim) s[c] = -INFINITY;
        }
        float mx[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
        for (int c = 4; c < kBKV; c += 4)
#pragma unroll
          for (int i = 0; i < 4; ++i) mx[i] = fmaxf(mx[i], s[c + i]);
        const float mrow = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * p.scale_log2;
        float alpha = 1.0f;
        bool resc = false;
        if (j == 0) {
          m = mrow == -INFINITY ? 0.0f : mrow;
        } else if (mrow > m + kRescaleLog2) {
          alpha = gemm::approx_exp2(m - mrow);
          m = mrow;
          resc = true;
        }
        float2 sum2[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
        const float2 sc2 = make_float2(p.scale_log2, p.scale_log2), nm2 = make_float2(-m, -m);
#pragma unroll
        for (int c = 0; c < kBKV; c += 4)
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const float2 x = __ffma2_rn(make_float2(s[c + 2 * i], s[c + 2 * i + 1]), sc2, nm2);
            const float2 e = make_float2(gemm::approx_exp2(x.x), gemm::approx_exp2(x.y));
            s[c + 2 * i] = e.x;
            s[c + 2 * i + 1] = e.y;
            sum2[i] = __fadd2_rn(sum2[i], e);
          }
        l = fmaf(l, alpha, (sum2[0].x + sum2[0].y) + (sum2[1].x + sum2[1].y));
        // The previous product P V has read P (and, within the item, written O).
        if (g > 0) {
          if (!warp_wait(&o_done[t], static_cast<uint32_t>(g - 1) & 1u, ctl)) {
            ok = false;
            break;
          }
          gemm::tc_fence_after();
        }
        if (j > 0 && __any_sync(0xffffffffu, resc)) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t o[32];
            const uint32_t ta = t_lane + kTmemO + static_cast<uint32_t>(t * kD + c * 32);
            gemm::tmem_ld32(ta, o);
            gemm::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(ta, o);
          }
          tmem_wait_st();
        }
        // P row r: 16 chunks of 8 values into two 128-row x 128-byte swizzled columns
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          uint4 u;
          u.x = pack2(s[c * 8 + 0], s[c * 8 + 1], half);
          u.y = pack2(s[c * 8 + 2], s[c * 8 + 3], half);
          u.z = pack2(s[c * 8 + 4], s[c * 8 + 5], half);
          u.w = pack2(s[c * 8 + 6], s[c * 8 + 7], half);
          const int cc = c & 7;
          *reinterpret_cast<uint4*>(pt + (c >> 3) * (kBQ * 128) + r * 128 + ((cc ^ (r & 7)) << 4)) = u;
        }
        gemm::fence_async_smem();
        gemm::tc_fence_before();
        __syncwarp();
        if (lane == 0) gemm::mbar_arrive(&p_full[t]);
      }
      if (!ok || !warp_wait(&o_done[t], static_cast<uint32_t>(g - 1) & 1u, ctl)) {
        ok = false;
        break;
      }
      gemm::tc_fence_after();
      uint32_t o[2][32];
#pragma unroll
      for (int c = 0; c < 2; ++c) gemm::tmem_ld32(t_lane + kTmemO + static_cast<uint32_t>(t * kD + c * 32), o[c]);
      gemm::tmem_wait_ld();
      gemm::tc_fence_before();
      __syncwarp();
      if (lane == 0) gemm::mbar_arrive(&o_free[t]);
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      if (row < p.Sq) {
        uint8_t* dst = reinterpret_cast<uint8_t*>(p.out) +
                       2 * (static_cast<int64_t>(it.b) * p.os_b + static_cast<int64_t>(it.h) * p.os_h +
                            static_cast<int64_t>(row) * p.os_s);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t* wv = &o[c >> 2][(c & 3) * 8];
          uint4 u;
          u.x = pack2(__uint_as_float(wv[0]) * inv, __uint_as_float(wv[1]) * inv, half);
          u.y = pack2(__uint_as_float(wv[2]) * inv, __uint_as_float(wv[3]) * inv, half);
          u.z = pack2(__uint_as_float(wv[4]) * inv, __uint_as_float(wv[5]) * inv, half);
          u.w = pack2(__uint_as_float(wv[6]) * inv, __uint_as_float(wv[7]) * inv, half);
          *reinterpret_cast<uint4*>(dst + c * 16) = u;
        }
      }
    }
  }

  gemm::tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    gemm::tc_fence_after();
    gemm::tmem_dealloc(tmem_base, kTmemCols);
  }
}

// 4-d tiled map over a [B, H, S, D] view (D contiguous): box 64 x 128 x 1 x 1,
// 128-byte swizzle, rows past S read as zeros.
bool make_map_4d(CUtensorMap* map, int dt, const void* ptr, const int64_t* sizes, const int64_t* strides) {
  auto fn = gemm::encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(sizes[3]), static_cast<cuuint64_t>(sizes[2]),
                              static_cast<cuuint64_t>(sizes[1]), static_cast<cuuint64_t>(sizes[0])};
  // A size-1 dim's stride is never stepped; give it a legal value.
  cuuint64_t gstr[3];
  uint64_t natural = static_cast<uint64_t>(sizes[3]) * 2;
  for (int i = 0; i < 3; ++i) {
    const int d = 2 - i;  // s, h, b
    const uint64_t st = static_cast<uint64_t>(strides[d]) * 2;
    gstr[i] = sizes[d] == 1 ? ((natural + 15) / 16) * 16 : st;
    natural = static_cast<uint64_t>(gstr[i]) * static_cast<uint64_t>(sizes[d]);
  }
  const cuuint32_t box[4] = {kD, kBKV, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, gemm::tma_dtype(dt), 4, const_cast<void*>(ptr), dims, gstr, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace attn
}  // namespace b200k

using namespace b200k::attn;

extern "C" int b200k_attention(const B200kAttentionArgs* a, void* stream_) {
  if (!a) return B200K_ERR_ARG;
  if (a->batch < 0 || a->heads < 0 || a->kv_heads < 0 || a->q_len < 0 || a->kv_len < 0) return B200K_ERR_SHAPE;
  if (a->batch == 0 || a->heads == 0 || a->q_len == 0) return B200K_OK;  // empty output
  if (!a->q || !a->k || !a->v || !a->out) return B200K_ERR_ARG;
  if (a->kv_len == 0 || a->kv_heads == 0) return B200K_ERR_SHAPE;
  if (a->head_dim != kD) return B200K_ERR_UNSUPPORTED;
  if (a->dtype != B200K_BF16 && a->dtype != B200K_F16) return B200K_ERR_UNSUPPORTED;
  if (a->heads % a->kv_heads != 0) return B200K_ERR_SHAPE;
  if (a->q_len > 0x7fffff00ll || a->kv_len > 0x7fffff00ll || a->batch * a->heads > 0x7fffffffll ||
      a->batch > 0x7fffffffll)
    return B200K_ERR_SHAPE;
  const int64_t* strides[4] = {a->q_strides, a->k_strides, a->v_strides, a->out_strides};
  const void* ptrs[4] = {a->q, a->k, a->v, a->out};
  for (int i = 0; i < 4; ++i) {
    if (strides[i][3] != 1) return B200K_ERR_UNSUPPORTED;
    if (!b200k::aligned16(ptrs[i])) return B200K_ERR_ALIGN;
    for (int d = 0; d < 3; ++d)
      if (strides[i][d] < 0 || strides[i][d] % 8 != 0) return B200K_ERR_ALIGN;
  }
  const int64_t n_ctiles = (a->q_len + 2 * kBQ - 1) / (2 * kBQ);
  const int64_t items = n_ctiles * a->batch * a->heads;
  if (items > 0x7fffffffll) return B200K_ERR_SHAPE;

  const int64_t qs[4] = {a->batch, a->heads, a->q_len, a->head_dim};
  const int64_t ks[4] = {a->batch, a->kv_heads, a->kv_len, a->head_dim};
  CUtensorMap tq, tk, tv;
  if (!make_map_4d(&tq, a->dtype, a->q, qs, a->q_strides) || !make_map_4d(&tk, a->dtype, a->k, ks, a->k_strides) ||
      !make_map_4d(&tv, a->dtype, a->v, ks, a->v_strides))
    return B200K_ERR_LAUNCH;

  Params p;
  std::memset(&p, 0, sizeof(p));
  p.B = static_cast<int32_t>(a->batch);
  p.H = static_cast<int32_t>(a->heads);
  p.group = static_cast<int32_t>(a->heads / a->kv_heads);
  p.Sq = static_cast<int32_t>(a->q_len);
  p.Skv = static_cast<int32_t>(a->kv_len);
  p.n_ctiles = static_cast<int32_t>(n_ctiles);
  p.causal = a->causal ? 1 : 0;
  p.half = a->dtype == B200K_F16 ? 1 : 0;
  const float scale = a->scale > 0.0f ? a->scale : 1.0f / sqrtf(static_cast<float>(a->head_dim));
  p.scale_log2 = scale * kLog2e;
  p.test_flags = a->test_flags;
  p.out = a->out;
  p.os_b = a->out_strides[0];
  p.os_h = a->out_strides[1];
  p.os_s = a->out_strides[2];
  const uint32_t fmt = a->dtype == B200K_BF16 ? 1u : 0u;
  // kind::f16 instruction descriptors: fp32 accumulate, A/B format, K-major A;
  // B K-major for Q K^T (K rows are head_dim-contiguous), N-major for P V.
  p.idesc_s = (1u << 4) | (fmt << 7) | (fmt << 10) | (static_cast<uint32_t>(kBKV >> 3) << 17) |
              (static_cast<uint32_t>(kBQ >> 4) << 24);
  p.idesc_pv = (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 16) | (static_cast<uint32_t>(kD >> 3) << 17) |
               (static_cast<uint32_t>(kBQ >> 4) << 24);
  p.status = a->status;
  p.timeout_ns = a->timeout_ns > 0 ? a->timeout_ns : 2000000000ll;

  static bool attr_set = false;
  if (!attr_set) {
    // The register split inside the kernel is sized for kLaunchRegs
    // registers per thread at launch; with any other count setmaxnreg.inc
    // could wait for registers that do not exist, so do not launch.
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, attention_kernel) != cudaSuccess || fa.numRegs != kLaunchRegs)
      return B200K_ERR_UNSUPPORTED;
    if (cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
      return B200K_ERR_LAUNCH;
    attr_set = true;
  }
  const int sms = b200k::device_sm_count();
  if (sms <= 0) return B200K_ERR_DEVICE;
  const int64_t ctas = std::min<int64_t>(items, sms);  // persistent: one CTA per SM
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  attention_kernel<<<static_cast<unsigned>(ctas), kThreads, kSmem, st>>>(tq, tk, tv, p);
  return cudaGetLastError() == cudaSuccess ? B200K_OK : B200K_ERR_LAUNCH;
}
