// GEMM + fused epilogue on the sm_100a tensor cores: device code and launch
// templates shared by gemm_sm100.cu and the gemm_fast_*.cu instantiation files.
//
//   out[m, n] = program(acc[m, n], extras...[m, n]),  acc = sum_k a[m, k] * b[k, n]
//
// Replaces the reference's generated, autotuned Triton kernel
// (compiler/optimization/fusion_epilogue.py:72-151, launched by :164-177, tile
// candidates :31-38) and the standalone demos hand_written/gemm_kernel.py and
// hand_written/gemm_swizzled_kernel.py.
//
// Design (one CTA per SM, persistent, warp-specialised, 384 threads):
//   warp 0      TMA producer: one thread streams 128xBK tiles of A and BNxBK
//               tiles of B into a STAGES-deep shared-memory ring (128-byte
//               swizzle), completing `full[s]` mbarriers by transaction count.
//   warp 1      MMA issuer: one thread issues tcgen05.mma (kind::f16, fp32
//               accumulate, M=128, N=BN, K=16) from smem descriptors into one
//               of two TMEM accumulators, releases ring slots with
//               tcgen05.commit -> empty[s], and hands a finished accumulator to
//               the epilogue with tcgen05.commit -> tmem_full[acc].
//   warp 2      owns the TMEM allocation (2*BN columns).
//   warps 4..   epilogue, NG warps per SM sub-partition (NG = 2 column
//               groups for 256- and 128-wide tiles, 3 for 192-wide ones):
//               warp w reads TMEM lane quarter (w % 4) and one column group
//               of the tile with tcgen05.ld (one output row per thread), runs the epilogue
//               program in registers (bias, activation, residual, scale,
//               casts) while the next 8 columns' operands are in flight, packs
//               to the output dtype into a swizzled smem tile and stores it
//               with a TMA bulk-tensor store.  It frees the accumulator with
//               tmem_empty[acc] so the MMA warp can start tile i+2 while tile
//               i+1 accumulates into the other buffer.
// Tiles are visited in grouped order (GROUP_M tiles down M per column band)
// so that co-resident CTAs share A and B panels in L2.
//
// Every mbarrier wait is bounded (global timer): on timeout the kernel records
// B200K_ERR_TIMEOUT in the caller's status word, raises a CTA abort flag so the
// other roles leave their loops, drains what it has in flight, frees TMEM and
// returns.
#pragma once
#include <cuda.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "host_common.h"

namespace b200k {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // one 128-byte swizzle atom of 16-bit elements
constexpr int UMMA_K = 16;
// Tile rows per raster group (Params::group_m): a wave of persistent CTAs
// walks group_m tile rows down before moving right, so the A rows and B
// columns it reads at once stay in L2.  The per-wave working set
// group_m * (A bytes of a tile row) + (slots / group_m) * (B bytes of a tile
// column) is smallest near group_m = sqrt(slots * B / A): 16 for 128 x 256
// tiles on 148 SMs, 8 for the 74 CTA pairs of 256-row tiles.
constexpr int kGroupM = 16;
constexpr int kGroupMPair = 8;
// The MMA thread signals tsoon[acc] this many K blocks before a tile's last
// one (~5 us at B200 MMA rates), and the epilogue warps then warm L2 with the
// tile's full-matrix operand rows (residual / scale).  Warmed one whole tile
// earlier, as first done, those rows were evicted again by the operand
// streams of large GEMMs before the epilogue read them.
constexpr int kSoonBlocks = 12;

// Epilogue warp layout of a BN-wide tile: NG column groups of CW columns,
// one warp per (TMEM lane quarter, column group); warps 0-3 are control.
template <int BN>
struct Epi {
  static constexpr int NG = BN == 192 ? 3 : 2;
  static constexpr int CW = BN / NG;  // a multiple of 64: whole 128-byte staging rows of 16-bit output
  static constexpr int kWarps = 4 * NG;
  static constexpr int kThreads = 128 + 32 * kWarps;
  static_assert(CW % 64 == 0, "column groups are whole staging rows");
};
constexpr uint32_t kStgBytes = 32 * 128;  // one epilogue warp's 32 rows x 128 bytes

struct EpiOperand {
  const void* ptr;
  int64_t sm, sn;
  int32_t dt;
  int32_t vec;  // 8-wide loads along n are legal
};

struct Params {
  int32_t M, N, K;
  int32_t tiles_m, tiles_n, num_tiles, k_blocks;
  int32_t n_extras;
  int32_t out_dt;
  int32_t direct_store;  // 1: write with st.global (output not TMA-storable)
  void* out;
  int64_t out_sm;
  int32_t* status;
  int64_t timeout_ns;
  uint32_t idesc;
  int32_t f_bias, f_act, f_round, f_scale, f_res;  // canonical epilogue form (fast path)
  int32_t xm_bias, xm_scale, xm_res;               // how the fast path stages each operand (XM_*)
  int32_t row_idx;                                 // extras index of the fast path's full-matrix operand
  int32_t test_flags;                              // B200K_GEMM_TEST_* hooks (0 in production)
  int32_t group_m;                                 // tile rows per raster group (tile_coords)
  // Fast path: the bias (ex[f_bias]) and the full-matrix operand (ex[row_idx])
  // copied out of `ex`, so the epilogue's hot loop reads fixed parameter slots.
  const void* bias_ptr;
  int64_t bias_sn;
  int32_t bias_dt;
  const void* row_ptr;
  int64_t row_sm;
  // ROW_ROPE: rotary tables [period, 64] of the output type, row stride in
  // elements; output row m takes table row m % period
  const void* rope_cos;
  const void* rope_sin;
  int64_t rope_stride;
  int32_t rope_period;
  unsigned long long* trace;                       // diagnostic timeline, null = off
  EpiOperand ex[B200K_MAX_INPUTS - 1];
  B200kProgram prog;
};

// ----------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// The waiting thread is suspended until the phase completes or, at the
// latest, after kSuspendNs; the hint keeps waiting warps from spinning and
// taking issue slots from the epilogue warps on the same scheduler.
constexpr uint32_t kSuspendNs = 1000000;
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "n"(kSuspendNs)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void prefetch_map(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(m) : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// fp32 operands on the tensor cores in TF32 (each operand's significand
// rounded to 10 bits), fp32 accumulate: the same 32-byte K step as the
// 16-bit form (8 elements instead of 16).
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05 format): start address, leading and
// stride byte offsets (16-byte units), descriptor version 1, 128-byte swizzle.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// ------------------------------------------------ CTA-pair (cta_group::2) forms
// A cluster of two CTAs on two SMs computes one 256-row tile: each CTA holds
// its own 128 rows of A and one half of the tile's B columns in its shared
// memory (same offsets in both), and the even CTA issues M = 256 MMAs that
// read both CTAs' halves and write each CTA's 128 accumulator rows into that
// CTA's TMEM.  None of these forms multicasts a load.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the barrier at shared::cluster address `bar` (this CTA's or the
// peer's) when every pair MMA this thread issued so far has completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// Tile load into this CTA's shared memory whose byte count completes on the
// barrier at shared::cluster address `bar` (the even CTA's).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

// ------------------------------------------------------------- bounded waits
struct Ctl {
  volatile int* abort;
  int32_t* status;
  uint64_t timeout_ns;
};

// Waits for the phase of `bar` with parity `parity`.  Returns false when the
// CTA is aborting or this wait ran out of time (then it raises the abort).
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, const Ctl& c) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*c.abort) return false;
    if (global_timer_ns() - t0 > c.timeout_ns) {
      *c.abort = 1;
      if (c.status) atomicCAS(c.status, 0, B200K_ERR_TIMEOUT);
      return false;
    }
  }
}

// Same, ignoring the abort flag: used only to drain in-flight async work.
__device__ __forceinline__ bool wait_bar_drain(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
  return true;
}

__device__ __forceinline__ void stamp(const Params& p, int field) {
  if (p.trace) p.trace[static_cast<int64_t>(blockIdx.x) * B200K_GEMM_TRACE_WORDS + field] = global_timer_ns();
}
__device__ __forceinline__ void stamp_tile(const Params& p, int i, int field) {
  if (p.trace && i < 40) stamp(p, 8 + 6 * i + field);
}

__device__ __forceinline__ void tile_coords(int t, const Params& p, int& tm, int& tn) {
  const int per_group = p.group_m * p.tiles_n;
  const int g = t / per_group;
  const int first_m = g * p.group_m;
  const int gsize = min(p.tiles_m - first_m, p.group_m);
  const int r = t - g * per_group;
  tm = first_m + r % gsize;
  tn = r / gsize;
}

// Epilogue operand values at (m, n..n+7), zero outside [M, N).
__device__ __forceinline__ void load_extra8(const EpiOperand& e, int m, int n, int M, int N, float (&v)[8]) {
  if (m < M && n + 8 <= N && e.vec) {
    load_vec8(e.ptr, static_cast<int64_t>(m) * e.sm + n, e.dt, v);
  } else if (e.sn == 0) {
    const float s = (m < M) ? load_scalar(e.ptr, static_cast<int64_t>(m) * e.sm, e.dt) : 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = s;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      v[j] = (m < M && n + j < N)
                 ? load_scalar(e.ptr, static_cast<int64_t>(m) * e.sm + static_cast<int64_t>(n + j) * e.sn, e.dt)
                 : 0.0f;
  }
}

// Epilogue operand values at (m, n..n+3), zero outside [M, N).
__device__ __forceinline__ void load_extra4(const EpiOperand& e, int m, int n, int M, int N, float (&v)[4]) {
  if (m < M && n + 4 <= N && e.vec) {
    const int64_t off = static_cast<int64_t>(m) * e.sm + n;
    if (e.dt == B200K_F32) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(e.ptr) + off));
      v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
    } else {
      const uint2 u = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(e.ptr) + off));
      if (e.dt == B200K_BF16) {
        const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
        const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
        v[0] = lo.x; v[1] = lo.y; v[2] = hi.x; v[3] = hi.y;
      } else {
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
        v[0] = lo.x; v[1] = lo.y; v[2] = hi.x; v[3] = hi.y;
      }
    }
  } else if (e.sn == 0) {
    const float s = (m < M) ? load_scalar(e.ptr, static_cast<int64_t>(m) * e.sm, e.dt) : 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = s;
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      v[j] = (m < M && n + j < N)
                 ? load_scalar(e.ptr, static_cast<int64_t>(m) * e.sm + static_cast<int64_t>(n + j) * e.sn, e.dt)
                 : 0.0f;
  }
}

// 32 lanes x 32 bit, 8 consecutive columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

// 32 lanes x 32 bit, 4 consecutive columns.
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}

constexpr int kEV = 4;  // epilogue group width (columns per interpreter pass)
using ExtraRegs = float[B200K_MAX_INPUTS - 1][kEV];

__device__ __forceinline__ void load_extras(const Params& p, int m, int n, ExtraRegs& x) {
#pragma unroll
  for (int i = 0; i < B200K_MAX_INPUTS - 1; ++i)
    if (i < p.n_extras) load_extra4(p.ex[i], m, n, p.M, p.N, x[i]);
}

// One 4-column group of one output row: TMEM -> registers, issue the next
// group's operand loads (`nxt`), run the program, pack into the swizzled
// staging row (or store directly when the output is not TMA-storable).
template <int OUT_BYTES>
__device__ __forceinline__ void epilogue_group(const Params& p, uint32_t taddr, int m, int n, int g, int lane,
                                               uint8_t* sb, const ExtraRegs& cur, ExtraRegs& nxt, bool prefetch) {
  uint32_t raw[kEV];
  tmem_ld4(taddr, raw);
  if (prefetch) load_extras(p, m, n + kEV, nxt);
  tmem_wait_ld();
  float r[kSlots][kEV];
  float accv[kEV];
#pragma unroll
  for (int j = 0; j < kEV; ++j) {
    r[0][j] = __uint_as_float(raw[j]);
    accv[j] = r[0][j];
  }
#pragma unroll
  for (int i = 0; i < B200K_MAX_INPUTS - 1; ++i)
    if (i < p.n_extras) {
#pragma unroll
      for (int j = 0; j < kEV; ++j) r[i + 1][j] = cur[i][j];
    }
  run_program<kEV>(p.prog, r, accv);
  if (p.direct_store) {
    if (m < p.M) {
      const int64_t off = static_cast<int64_t>(m) * p.out_sm + n;
#pragma unroll
      for (int j = 0; j < kEV; ++j)
        if (n + j < p.N) store_scalar(p.out, off + j, p.out_dt, accv[j]);
    }
  } else if (OUT_BYTES == 2) {
    uint2 u;
    if (p.out_dt == B200K_BF16) {
      *reinterpret_cast<__nv_bfloat162*>(&u.x) = __floats2bfloat162_rn(accv[0], accv[1]);
      *reinterpret_cast<__nv_bfloat162*>(&u.y) = __floats2bfloat162_rn(accv[2], accv[3]);
    } else {
      *reinterpret_cast<__half2*>(&u.x) = __floats2half2_rn(accv[0], accv[1]);
      *reinterpret_cast<__half2*>(&u.y) = __floats2half2_rn(accv[2], accv[3]);
    }
    const int chunk = g >> 1;
    *reinterpret_cast<uint2*>(sb + lane * 128 + ((chunk ^ (lane & 7)) << 4) + ((g & 1) << 3)) = u;
  } else {
    *reinterpret_cast<float4*>(sb + lane * 128 + ((g ^ (lane & 7)) << 4)) =
        make_float4(accv[0], accv[1], accv[2], accv[3]);
  }
}

// ------------------------------------------------------- canonical fast path
// v = acc; v += E[bias]; v = act(v); v = round(v); v *= E[scale]; v += E[res]
// with the same fp32 operation order as the decomposed ATen graph it replaces.
__device__ __forceinline__ float approx_rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float approx_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// GELU(x) = x/2 (1 + erf(x / sqrt 2)) through the complementary error
// function of Abramowitz & Stegun, Handbook of Mathematical Functions,
// eq. 7.1.26: for y >= 0, erfc(y) = t (a1 + t (a2 + t (a3 + t (a4 + t a5))))
// exp(-y^2) + e(y), t = 1 / (1 + p y), |e(y)| <= 1.5e-7.  With y = |x|/sqrt 2
// and r = 1/2 - erfc(y)/2, GELU = x/2 + |x| r for either sign of x.  The
// coefficients below are a1..a5 halved and p / sqrt 2; exp(-y^2) =
// 2^(-x^2 log2(e) / 2).  Absolute error of the result is below
// 1e-7 (1 + |x|) plus the hardware rcp/ex2 rounding; +inf maps to +inf and
// NaN / -inf to NaN as in the erf formula.  Written stage by stage over the
// eight values so the independent chains interleave, two values per
// instruction with the sm_100 packed fp32 ops (__ffma2_rn, __fmul2_rn: each
// lane rounds exactly as fmaf / __fmul_rn does).  The polynomial runs on the
// negated coefficients, which gives -q and then -(q t) bit for bit (round to
// nearest is symmetric in sign), so r = fma(-(q t), e, 1/2) needs no
// separate negation.
__device__ __forceinline__ float2 splat2(float a) { return make_float2(a, a); }

__device__ __forceinline__ void gelu_erf_as8(float (&v)[8]) {
  float2 x[4], ax[4], t[4], e[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[i] = make_float2(v[2 * i], v[2 * i + 1]);
    ax[i] = make_float2(fabsf(v[2 * i]), fabsf(v[2 * i + 1]));
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 a = __ffma2_rn(splat2(0.2316418882663604f), ax[i], splat2(1.0f));
    t[i] = make_float2(approx_rcp(a.x), approx_rcp(a.y));
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 b = __fmul2_rn(__fmul2_rn(x[i], splat2(-0.72134752044448170f)), x[i]);
    e[i] = make_float2(approx_exp2(b.x), approx_exp2(b.y));
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 nq = __ffma2_rn(splat2(-0.5307027145f), t[i], splat2(0.7265760135f));
    nq = __ffma2_rn(nq, t[i], splat2(-0.7107068705f));
    nq = __ffma2_rn(nq, t[i], splat2(0.142248368f));
    nq = __ffma2_rn(nq, t[i], splat2(-0.127414796f));
    const float2 r = __ffma2_rn(__fmul2_rn(nq, t[i]), e[i], splat2(0.5f));
    const float2 o = __ffma2_rn(ax[i], r, __fmul2_rn(splat2(0.5f), x[i]));
    v[2 * i] = o.x;
    v[2 * i + 1] = o.y;
  }
}

// v[j] = v[j] + b[j] (or * b[j]) for j < 2 N, each rounded once, two per
// instruction.
template <int N2, bool MUL>
__device__ __forceinline__ void op2_rn(float* v, const float* b) {
#pragma unroll
  for (int j = 0; j < N2; ++j) {
    const float2 a = make_float2(v[2 * j], v[2 * j + 1]), c = make_float2(b[2 * j], b[2 * j + 1]);
    const float2 d = MUL ? __fmul2_rn(a, c) : __fadd2_rn(a, c);
    v[2 * j] = d.x;
    v[2 * j + 1] = d.y;
  }
}

// Separate ops of the decomposed graph (bias add, the activation's final
// multiply, the scale / residual op) use __fadd_rn / __fmul_rn or their packed
// forms (op2_rn) so the compiler never contracts two of them into one
// rounding, as eager execution would not.
template <int ACT>
__device__ __forceinline__ void apply_act8(float (&v)[8]) {
  if constexpr (ACT == B200K_ACT_GELU_ERF) {
    gelu_erf_as8(v);
  } else {
  float x0[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) x0[j] = v[j];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float x = v[j];
    if constexpr (ACT == B200K_ACT_GELU_TANH) {
      const float t3 = x + ((x * x) * x) * 0.044715f;
      v[j] = (x * 0.5f) * (op_tanh(t3 * 0.7978845608028654f) + 1.0f);
    } else if constexpr (ACT == B200K_ACT_SILU) {
      v[j] = op_sigmoid(x);  // times x below, two per instruction
    } else if constexpr (ACT == B200K_ACT_RELU) {
      v[j] = fmaxf(x, 0.0f);
    } else if constexpr (ACT == B200K_ACT_SIGMOID) {
      v[j] = op_sigmoid(x);
    } else if constexpr (ACT == B200K_ACT_TANH) {
      v[j] = op_tanh(x);
    }
  }
  if constexpr (ACT == B200K_ACT_SILU) op2_rn<4, true>(v, x0);
  }
}

// ------------------------------------------- fast path, latency-hiding loop
// Operand staging modes, chosen on the host per operand:
//   XM_BCAST   row-broadcast f32/bf16/f16 vector (stride_m == 0, e.g. a
//              bias): each lane loads one column's value a sub-chunk ahead
//              and the warp exchanges them through a 128-byte shared slot
//              (a shuffle per value costs more than the whole rest of a
//              bias-only epilogue; warp-uniform vector loads at the point of
//              use, an earlier design, missed L1 and waited on L2 for
//              600-1400 cycles a sub-chunk);
//   XM_ROW16   full 16-bit matrix with unit column stride (a residual, or the
//              `up` operand of SwiGLU): each lane loads its own row's 32
//              values (64 bytes) into registers;
//   XM_GENERIC anything else -- such programs run on the interpreter kernel.
// The compiled path takes a bias in XM_BCAST and at most one of scale and
// residual, in XM_ROW16 (its role is the kernel's ROW parameter, below).
// The full-matrix operand is loaded one 32-column sub-chunk ahead, across
// tile boundaries, into a second register set that becomes the current one
// when the sub-chunk is done.  The sub-chunk body exists once in the code and
// edge-of-matrix loads are out of line, which keeps the epilogue warps' hot
// loop small enough for the instruction cache.
enum { XM_NONE = 0, XM_BCAST = 1, XM_ROW16 = 2, XM_GENERIC = 3 };

// Role of the full-matrix operand in a compiled epilogue:
//   ROW_NONE     no scale, no residual;
//   ROW_SCALE    v * s and ROW_RES  v + r in fp32, rounded once by the store;
//   ROW_SCALE_PK / ROW_RES_PK: the form rounds the activation to the output
//                type and s / r has that type, so the multiply / add runs on
//                packed bf16x2 / f16x2 pairs.  A product or sum of two values
//                of an 8- or 11-bit-significand type is exact in fp32, so the
//                packed op's single rounding equals fp32-then-round, the
//                decomposed graph's order.
enum { ROW_NONE = 0, ROW_SCALE = 1, ROW_RES = 2, ROW_SCALE_PK = 3, ROW_RES_PK = 4, ROW_ROPE = 5 };

struct FastOps {
  uint4 row_r[4];  // the full-matrix operand's 32 values of this lane's row
  float bias;      // the bias of column n + lane (0 beyond N)
};

// 32 lanes x 32 bit, 32 consecutive columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// tcgen05.wait::ld that also names the destination registers of the load it
// waits for, so that no use of them can be scheduled before it.
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// The bias of one column as fp32 (0 at and beyond N), any stride and
// 16/32-bit dtype.  The compiled epilogue loads one column per lane a
// sub-chunk ahead and adds it rounded on its own (__fadd_rn), as the
// decomposed graph's bias add is.
__device__ __forceinline__ float bias_at(const Params& p, int col) {
  if (col >= p.N) return 0.0f;
  const int64_t off = static_cast<int64_t>(col) * p.bias_sn;
  if (p.bias_dt == B200K_F32) return __ldg(reinterpret_cast<const float*>(p.bias_ptr) + off);
  const unsigned short u = __ldg(reinterpret_cast<const unsigned short*>(p.bias_ptr) + off);
  return p.bias_dt == B200K_BF16 ? __uint_as_float(static_cast<uint32_t>(u) << 16) : __half2float(__ushort_as_half(u));
}

// Eight 16-bit values of one row from column n, zero at and beyond column N.
static __device__ __noinline__ uint4 load_row16_edge8(const uint16_t* row, int n, int N) {
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t lo = n + 2 * j < N ? row[n + 2 * j] : 0u;
    const uint32_t hi = n + 2 * j + 1 < N ? row[n + 2 * j + 1] : 0u;
    w[j] = lo | (hi << 16);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ void load_row16(const void* ptr, int64_t sm, int m, int n, int M, int N, uint4 (&b)[4]) {
  const uint16_t* row = reinterpret_cast<const uint16_t*>(ptr) + static_cast<int64_t>(m) * sm;
  if (m < M && n + 32 <= N) {
    const uint4* q = reinterpret_cast<const uint4*>(row + n);
#pragma unroll
    for (int i = 0; i < 4; ++i) b[i] = __ldg(q + i);
  } else if (m < M) {
#pragma unroll
    for (int i = 0; i < 4; ++i) b[i] = load_row16_edge8(row, n + 8 * i, N);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) b[i] = make_uint4(0u, 0u, 0u, 0u);
  }
}

__device__ __forceinline__ void prefetch_l2(const void* ptr) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}

// Warms L2 with this lane's row of the full-matrix operand (residual or
// scale) for the tile at (m, n): the warp's CW columns, which the
// sub-chunks later read straight into registers.  Issued when the MMA
// thread signals that the tile is kSoonBlocks K blocks from done, so those
// reads wait on L2 rather than DRAM.
template <int CW, int ROW>
__device__ __forceinline__ void prefetch_row16_l2(const Params& p, int m, int n) {
  if (ROW == ROW_NONE || m >= p.M || n >= p.N) return;
  const int bytes = min(CW, p.N - n) * 2;
  const char* row = reinterpret_cast<const char*>(p.row_ptr) + (static_cast<int64_t>(m) * p.row_sm + n) * 2;
  for (int off = 0; off < bytes; off += 128) prefetch_l2(row + off);
  prefetch_l2(row + bytes - 1);  // the line of the last byte when the row is not 128-byte aligned
}

// Issues the loads of the next sub-chunk's operands: this lane's row of the
// full-matrix operand and the bias of column n + lane.  Their latency (an
// L2 round trip: the 28 KB of L1 beside 227 KB of shared memory does not
// keep a bias) then overlaps the current sub-chunk instead of stalling the
// next.
template <int ROW>
__device__ __forceinline__ void fast_prefetch(const Params& p, int m, int n, int lane, FastOps& f) {
  if constexpr (ROW != ROW_NONE) load_row16(p.row_ptr, p.row_sm, m, n, p.M, p.N, f.row_r);
  if (p.f_bias >= 0) f.bias = bias_at(p, n + lane);
}

__device__ __forceinline__ uint32_t pk_op(uint32_t a, uint32_t b, bool bf16, bool mul) {
  uint32_t d;
  if (bf16) {
    if (mul) asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    else asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  } else {
    if (mul) asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    else asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  }
  return d;
}

__device__ __forceinline__ void unpack16x8(uint4 u, int dt, float (&x)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  if (dt == B200K_BF16) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      x[2 * j] = __uint_as_float(w[j] << 16);
      x[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      x[2 * j] = f.x;
      x[2 * j + 1] = f.y;
    }
  }
}

// One 32-column sub-chunk of one output row per lane (columns n..n+31 of
// row m, TMEM columns t_col..t_col+31): read the accumulator, apply the
// canonical epilogue with the full-matrix operand in `use`, stage, and store
// every 128-byte staging row with one TMA store per warp.  Each step runs
// over all 32 values before the next (bias, activation, rounding, operand,
// packing), so independent values interleave; the dtype choices are
// warp-uniform branches around whole steps.
// The sub-chunk's accumulator values arrive in `raw` (loaded from tensor
// memory by the caller).
template <int BN, int OUT_BYTES, int ACT, int ROW>
__device__ __forceinline__ void fast_sub_chunk(const Params& p, const CUtensorMap* tmO, const uint32_t (&raw)[32],
                                               int row0, int n, int s, int lane, uint8_t* sb, float* bslot,
                                               const FastOps& use) {
  constexpr int kEC = 128 / OUT_BYTES;
  constexpr int NSUB = Epi<BN>::CW / 32;
  constexpr int SUB_PER_STG = kEC / 32;
  constexpr bool kPacked = ROW == ROW_SCALE_PK || ROW == ROW_RES_PK;
  constexpr bool kMul = ROW == ROW_SCALE || ROW == ROW_SCALE_PK;
  static_assert(OUT_BYTES == 2 || ROW == ROW_NONE, "full-matrix operands are 16-bit, as is the output");
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(raw[j]);
  const int sub = s % SUB_PER_STG;
  if (p.f_bias >= 0) {
    // Each lane holds the bias of one column (loaded a sub-chunk ahead); the
    // warp's 128-byte slot hands every lane all 32 (broadcast reads).
    __syncwarp();  // every lane has read the previous sub-chunk's values
    bslot[lane] = use.bias;
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 b4 = reinterpret_cast<const float4*>(bslot)[i];
      const float b[4] = {b4.x, b4.y, b4.z, b4.w};
      op2_rn<2, false>(&v[4 * i], b);
    }
  }
#pragma unroll
  for (int g = 0; g < 4; ++g) apply_act8<ACT>(*reinterpret_cast<float(*)[8]>(&v[8 * g]));
  const bool out_bf16 = p.out_dt == B200K_BF16;
  uint4 u[4];
  if constexpr (kPacked) {
    if (out_bf16) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        u[g] = pack_bf16x8(*reinterpret_cast<float(*)[8]>(&v[8 * g]));
        const uint4 r = use.row_r[g];
        u[g] = make_uint4(pk_op(u[g].x, r.x, true, kMul), pk_op(u[g].y, r.y, true, kMul),
                          pk_op(u[g].z, r.z, true, kMul), pk_op(u[g].w, r.w, true, kMul));
      }
    } else {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        u[g] = pack_f16x8(*reinterpret_cast<float(*)[8]>(&v[8 * g]));
        const uint4 r = use.row_r[g];
        u[g] = make_uint4(pk_op(u[g].x, r.x, false, kMul), pk_op(u[g].y, r.y, false, kMul),
                          pk_op(u[g].z, r.z, false, kMul), pk_op(u[g].w, r.w, false, kMul));
      }
    }
  } else {
    if (p.f_round == B200K_BF16) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = round_bf16(v[j]);
    } else if (p.f_round == B200K_F16) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = round_f16(v[j]);
    }
    if constexpr (ROW != ROW_NONE) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        float x[8];
        unpack16x8(use.row_r[g], out_bf16 ? B200K_BF16 : B200K_F16, x);
        op2_rn<4, kMul>(&v[8 * g], x);
      }
    }
    if constexpr (OUT_BYTES == 2) {
      if (out_bf16) {
#pragma unroll
        for (int g = 0; g < 4; ++g) u[g] = pack_bf16x8(*reinterpret_cast<float(*)[8]>(&v[8 * g]));
      } else {
#pragma unroll
        for (int g = 0; g < 4; ++g) u[g] = pack_f16x8(*reinterpret_cast<float(*)[8]>(&v[8 * g]));
      }
    }
  }
  // The staging row is rewritten only once the previous TMA store has read
  // it; waiting here rather than before the math lets that read overlap it.
  if (sub == 0) {
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();
  }
  if constexpr (OUT_BYTES == 2) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int chunk = sub * 4 + g;
      *reinterpret_cast<uint4*>(sb + lane * 128 + ((chunk ^ (lane & 7)) << 4)) = u[g];
    }
  } else {
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<float4*>(sb + lane * 128 + ((c ^ (lane & 7)) << 4)) =
          make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
  }
  if (sub == SUB_PER_STG - 1 || s + 1 == NSUB || n + 32 >= p.N) {
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmO, sb, n - sub * 32, row0);
      bulk_commit();
    }
  }
}

// ------------------------------------------------- rotary-embedding epilogue
// ROW_ROPE: the output is the projection q = round(acc) (16-bit) rotated as
//   out[d]      = round(round(q[d] cos[d])           - round(q[d + 32] sin[d]))
//   out[d + 32] = round(round(q[d + 32] cos[d + 32]) + round(q[d] sin[d + 32]))
// for each 64-column head (d < 32), with cos / sin the row's table entries:
// x cos + rotate_half(x) sin with every product and the sum rounded to the
// 16-bit type, as eager PyTorch computes it (a product or sum of two 16-bit
// values is exact in fp32, so the packed bf16x2 / f16x2 ops round exactly
// once, as the fp32-then-round of eager does).  A warp's step covers one head
// of its 32 rows: two 32-column accumulator loads, one 128-byte staging row,
// one TMA store.  The row's 64 cos and 64 sin values are loaded once per tile,
// before the accumulator wait.
__device__ __forceinline__ uint32_t pk_sub(uint32_t a, uint32_t b, bool bf16) {
  uint32_t d;
  if (bf16) asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ void load_rope_row(const Params& p, int m, uint4 (&cs)[16]) {
  const int64_t off = static_cast<int64_t>(m % p.rope_period) * p.rope_stride;
  const uint4* c = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.rope_cos) + off);
  const uint4* sn = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.rope_sin) + off);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    cs[i] = __ldg(c + i);
    cs[8 + i] = __ldg(sn + i);
  }
}

__device__ __forceinline__ void tmem_wait_ld_regs2(uint32_t (&a)[32], uint32_t (&b)[32]) {
  tmem_wait_ld_regs(a);
  // orders every use of b after the wait as well (volatile asm statements keep their order)
  asm volatile(""
               : "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]),
                 "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]), "+r"(b[12]), "+r"(b[13]), "+r"(b[14]),
                 "+r"(b[15]), "+r"(b[16]), "+r"(b[17]), "+r"(b[18]), "+r"(b[19]), "+r"(b[20]), "+r"(b[21]),
                 "+r"(b[22]), "+r"(b[23]), "+r"(b[24]), "+r"(b[25]), "+r"(b[26]), "+r"(b[27]), "+r"(b[28]),
                 "+r"(b[29]), "+r"(b[30]), "+r"(b[31])
               :
               : "memory");
}

// 32 accumulator values of a row rounded to the 16-bit output type, packed in pairs.
__device__ __forceinline__ void round_pack32(const uint32_t (&raw)[32], bool bf16, uint32_t (&q)[16]) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(raw[8 * g + j]);
    const uint4 u = bf16 ? pack_bf16x8(v) : pack_f16x8(v);
    q[4 * g] = u.x;
    q[4 * g + 1] = u.y;
    q[4 * g + 2] = u.z;
    q[4 * g + 3] = u.w;
  }
}

template <int BN, bool PAIR>
__device__ __forceinline__ void epilogue_rope_loop(const Params& p, const CUtensorMap* tmO, uint32_t tmem_base,
                                                   uint64_t* tfull, uint64_t* tempty, uint8_t* sb, int quarter,
                                                   int cg, int lane, const Ctl& ctl, uint32_t rank) {
  constexpr int CW = Epi<BN>::CW;
  static_assert(CW % 64 == 0, "whole heads per warp");
  constexpr int TM = PAIR ? 2 * BM : BM;
  const int t0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int step = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const int rank_rows = static_cast<int>(rank) * BM;
  const bool bf16 = p.out_dt == B200K_BF16;
  int acc = 0;
  uint32_t aph = 0;
  for (int t = t0; t < p.num_tiles; t += step) {
    int tm, tn;
    tile_coords(t, p, tm, tn);
    const int row0 = tm * TM + rank_rows + quarter * 32;
    uint4 cs[16];  // cos[0:64] in cs[0..7], sin[0:64] in cs[8..15]
    load_rope_row(p, row0 + lane, cs);
    if (!wait_bar(&tfull[acc], aph, ctl)) break;
    tc_fence_after();
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                           static_cast<uint32_t>(acc * BN + cg * CW);
#pragma unroll 1
    for (int h = 0; h < CW / 64; ++h) {
      const int n = tn * BN + cg * CW + h * 64;
      if (n >= p.N) break;  // warp-uniform; N is a multiple of 64
      uint32_t a0[32], a1[32];
      tmem_ld32(t_row + h * 64, a0);
      tmem_ld32(t_row + h * 64 + 32, a1);
      tmem_wait_ld_regs2(a0, a1);
      uint32_t q0[16], q1[16];
      round_pack32(a0, bf16, q0);
      round_pack32(a1, bf16, q1);
      const uint32_t* c = reinterpret_cast<const uint32_t*>(cs);  // c[0..31] cos, c[32..63] sin (bf16x2)
      uint32_t o[32];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        o[k] = pk_sub(pk_op(q0[k], c[k], bf16, true), pk_op(q1[k], c[32 + k], bf16, true), bf16);
        o[16 + k] = pk_op(pk_op(q1[k], c[16 + k], bf16, true), pk_op(q0[k], c[48 + k], bf16, true), bf16, false);
      }
      // the previous store has read the staging row
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
#pragma unroll
      for (int g = 0; g < 8; ++g)
        *reinterpret_cast<uint4*>(sb + lane * 128 + ((g ^ (lane & 7)) << 4)) =
            make_uint4(o[4 * g], o[4 * g + 1], o[4 * g + 2], o[4 * g + 3]);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(tmO, sb, n, row0);
        bulk_commit();
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      if (PAIR && rank != 0) mbar_arrive_cluster(cluster_addr(&tempty[acc], 0));
      else mbar_arrive(&tempty[acc]);
    }
    if (++acc == 2) {
      acc = 0;
      aph ^= 1u;
    }
  }
  if (lane == 0) bulk_wait_all();
  __syncwarp();
}

// PAIR: the tiles are 256 rows high, one per CTA pair (the grid's cluster
// index walks them), and this CTA's 128 rows start at `rank` x 128; the
// accumulator is released on the even CTA's barrier.
// WIDE (pairs only): the tile is 256 x 2*BN and its accumulator is the whole
// 512-column TMEM allocation in two BN-column halves.  tfull[0] signals the
// tile; half h is released on tempty[h] as soon as it has been read, so the
// next tile's MMAs into half 0 start while half 1 is still being drained.
template <int BN, int OUT_BYTES, int ACT, int ROW, bool PAIR = false, bool WIDE = false>
__device__ __forceinline__ void epilogue_fast_loop(const Params& p, const CUtensorMap* tmO, uint32_t tmem_base,
                                                   uint64_t* tfull, uint64_t* tempty, uint64_t* tsoon, uint8_t* sb,
                                                   float* bslot,
                                                   int quarter, int cg, int lane, const Ctl& ctl,
                                                   uint32_t rank = 0) {
  static_assert(PAIR || !WIDE, "wide tiles run on CTA pairs");
  if constexpr (ROW == ROW_ROPE) {
    static_assert(!WIDE && OUT_BYTES == 2 && ACT == B200K_ACT_NONE, "rotary epilogue: narrow tiles, 16-bit output");
    epilogue_rope_loop<BN, PAIR>(p, tmO, tmem_base, tfull, tempty, sb, quarter, cg, lane, ctl, rank);
    return;
  }
  constexpr int CW = Epi<BN>::CW;
  constexpr int NSUB = CW / 32;  // 32-column sub-chunks per warp and accumulator half
  constexpr int TM = PAIR ? 2 * BM : BM;  // rows per tile
  constexpr int H = WIDE ? 2 : 1;         // accumulator halves per tile
  constexpr int TN = H * BN;              // columns per tile
  const int t0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int step = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const int rank_rows = static_cast<int>(rank) * BM;
  FastOps cur{}, nxt{};
  if (t0 < p.num_tiles) {
    int tm, tn;
    tile_coords(t0, p, tm, tn);
    fast_prefetch<ROW>(p, tm * TM + rank_rows + quarter * 32 + lane, tn * TN + cg * CW, lane, cur);
  }
  int acc = 0;
  uint32_t aph = 0;
  const bool stamper = quarter == 0 && cg == 0 && lane == 0;
  int ti = 0;
  for (int t = t0; t < p.num_tiles; t += step, ++ti) {
    int tm, tn;
    tile_coords(t, p, tm, tn);
    const bool more = t + step < p.num_tiles;
    int m2 = 0, n2 = 0;
    if (more) {
      int tm2, tn2;
      tile_coords(t + step, p, tm2, tn2);
      m2 = tm2 * TM + rank_rows + quarter * 32 + lane;
      n2 = tn2 * TN + cg * CW;
    }
    if constexpr (ROW != ROW_NONE) {
      // a few K blocks before the accumulator is ready: warm L2 with this
      // lane's row of the operand for the whole tile (in a pair, the even
      // CTA's warps warm both CTAs' rows; the odd CTA has no signal)
      if (!PAIR || rank == 0) {
        if (!wait_bar(&tsoon[acc], aph, ctl)) break;
#pragma unroll
        for (int h = 0; h < H; ++h)
#pragma unroll
          for (int r = 0; r < (PAIR ? 2 : 1); ++r)
            prefetch_row16_l2<CW, ROW>(p, tm * TM + r * BM + quarter * 32 + lane, tn * TN + h * BN + cg * CW);
      }
    }
    if (!wait_bar(&tfull[acc], aph, ctl)) break;
    tc_fence_after();
    if (stamper) stamp_tile(p, ti, 4);
    const int row0 = tm * TM + rank_rows + quarter * 32;
    const int m = row0 + lane;
#pragma unroll 1
    for (int h = 0; h < H; ++h) {
      const int n0 = tn * TN + h * BN + cg * CW;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>((WIDE ? h : acc) * BN + cg * CW);
      // Each sub-chunk's accumulator columns are loaded when due: loading
      // them one sub-chunk ahead (a second 32-register set) measured no
      // faster (16384 x 4096 x 14336 + GELU + residual 1244-1249 us against
      // 1239-1245 us loaded when due, same boxes).
#pragma unroll 1
      for (int s = 0; s < NSUB; ++s) {
        const int n = n0 + s * 32;
        if (stamper && ti == 0 && h == 0 && s < 4) stamp(p, 248 + 2 * s);
        if (s + 1 < NSUB) fast_prefetch<ROW>(p, m, n + 32, lane, nxt);
        else if (h + 1 < H) fast_prefetch<ROW>(p, m, n0 + BN, lane, nxt);
        else if (more) fast_prefetch<ROW>(p, m2, n2, lane, nxt);
        if (n < p.N) {  // warp-uniform
          uint32_t now[32];
          tmem_ld32(t_row + s * 32, now);
          tmem_wait_ld_regs(now);
          fast_sub_chunk<BN, OUT_BYTES, ACT, ROW>(p, tmO, now, row0, n, s, lane, sb, bslot, cur);
        }
        if (stamper && ti == 0 && h == 0 && s < 4) stamp(p, 249 + 2 * s);
        cur = nxt;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        uint64_t* rel = &tempty[WIDE ? h : acc];
        if (PAIR && rank != 0) mbar_arrive_cluster(cluster_addr(rel, 0));
        else mbar_arrive(rel);
      }
    }
    if (stamper) stamp_tile(p, ti, 5);
    if (WIDE) {
      aph ^= 1u;
    } else if (++acc == 2) {
      acc = 0;
      aph ^= 1u;
    }
  }
  if (lane == 0) bulk_wait_all();
  __syncwarp();
}

template <int BN, int STAGES, bool B_NMAJOR, int OUT_BYTES>
struct Cfg {
  static constexpr uint32_t kABytes = BM * BK * 2;
  static constexpr uint32_t kBBytes = BN * BK * 2;
  static constexpr uint32_t kTmemCols = BN == 128 ? 256 : 512;  // two accumulators, power-of-two allocation
  static constexpr int kEC = 128 / OUT_BYTES;  // output columns per 128-byte staging row
  static constexpr uint32_t kBarOff = STAGES * (kABytes + kBBytes) + Epi<BN>::kWarps * kStgBytes;
  static constexpr uint32_t kBiasOff = kBarOff + 256;  // one 32-float bias slot per epilogue warp
  static constexpr uint32_t kSmem = 1024 + kBiasOff + Epi<BN>::kWarps * 128;
  static_assert(kSmem <= 232448, "shared memory budget");
  static_assert(kSmem > 232448 / 2, "one CTA per SM keeps the TMEM allocation uncontended");
  static_assert(2 * BN <= kTmemCols, "two accumulators fit the allocation");
};

// TF32: fp32 A and B (K-major B only); a K block is then 32 elements, the
// same 128 bytes a row as 64 16-bit ones, so the shared-memory layout,
// descriptors and stage sizes are those of the 16-bit kernel.
// A_MMAJOR: A is stored M-major (unit M stride, e.g. the transposed gradient
// of a weight-gradient GEMM), loaded as two 64-row by BK-column boxes whose
// 128-byte rows run along M, the mirror of N-major B; the instruction
// descriptor's A-major bit tells the MMA (16-bit operands only).
template <int BN, int STAGES, bool B_NMAJOR, int OUT_BYTES, bool FAST, int ACT, int ROW, bool TF32 = false,
          bool A_MMAJOR = false>
__global__ void __launch_bounds__(Epi<BN>::kThreads, 1)
    gemm_epilogue_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmO, const __grid_constant__ Params p) {
  using C = Cfg<BN, STAGES, B_NMAJOR, OUT_BYTES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* sbase = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sA = sbase;
  uint8_t* sB = sA + STAGES * C::kABytes;
  uint8_t* sStg = sB + STAGES * C::kBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sbase + C::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* tsoon = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tsoon + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) stamp(p, 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], Epi<BN>::kWarps);
    }
    mbar_init(drain, 1);
    for (int a = 0; a < 2; ++a) mbar_init(&tsoon[a], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_map(&tmA);
    prefetch_map(&tmB);
    if (!p.direct_store) prefetch_map(&tmO);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const Ctl ctl{abort_flag, p.status, static_cast<uint64_t>(p.timeout_ns)};
  if (threadIdx.x == 0) stamp(p, 1);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int64_t issued = 0;
      bool ok = true;
      int ti = 0;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++ti) {
        int tm, tn;
        tile_coords(t, p, tm, tn);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!wait_bar(&empty[s], ph ^ 1u, ctl)) {
            ok = false;
            break;
          }
          if (kb == 0) stamp_tile(p, ti, 0);
          if (kb == p.k_blocks - 1) stamp_tile(p, ti, 1);
          mbar_arrive_expect_tx(&full[s], C::kABytes + C::kBBytes);
          constexpr int kKb = TF32 ? BK / 2 : BK;  // elements of a K block
          static_assert(!(TF32 && B_NMAJOR), "TF32 runs K-major B only");
          static_assert(!(TF32 && A_MMAJOR), "TF32 runs K-major A only");
          if (A_MMAJOR) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_2d(sA + s * C::kABytes + j * (64 * BK * 2), &tmA, &full[s], tm * BM + j * 64, kb * BK);
          } else {
            tma_load_2d(sA + s * C::kABytes, &tmA, &full[s], kb * kKb, tm * BM);
          }
          if (B_NMAJOR) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sB + s * C::kBBytes + j * (64 * BK * 2), &tmB, &full[s], tn * BN + j * 64, kb * BK);
          } else {
            tma_load_2d(sB + s * C::kBBytes, &tmB, &full[s], kb * kKb, tn * BN);
          }
          ++issued;
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // Every load lands before the CTA can exit: after a timeout the MMA
      // thread may not have waited for the last ones (otherwise these phases
      // are complete already and the waits return at once).
      for (int x = 0; x < STAGES; ++x) {
        if (issued > x) {
          const uint32_t par = (x < s) ? ph : (ph ^ 1u);
          wait_bar_drain(&full[x], par, 100000000ull);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int s = 0, acc = 0;
      uint32_t ph = 0, aph = 0;
      bool ok = true;
      int ti = 0;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++ti) {
        if (!wait_bar(&tempty[acc], aph ^ 1u, ctl)) break;
        tc_fence_after();
        stamp_tile(p, ti, 2);
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!wait_bar(&full[s], ph, ctl)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * C::kABytes);
          const uint32_t b0 = smem_u32(sB + s * C::kBBytes);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            const uint64_t ad = A_MMAJOR ? sw128_desc(a0 + k * (UMMA_K * 128), 64 * BK * 2, 1024)
                                         : sw128_desc(a0 + k * (UMMA_K * 2), 16, 1024);
            const uint64_t bd = B_NMAJOR ? sw128_desc(b0 + k * (UMMA_K * 128), 64 * BK * 2, 1024)
                                         : sw128_desc(b0 + k * (UMMA_K * 2), 16, 1024);
            if constexpr (TF32) umma_tf32(d_tmem, ad, bd, p.idesc, (kb | k) != 0 ? 1u : 0u);
            else umma_f16(d_tmem, ad, bd, p.idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[s]);
          if (kb == max(0, p.k_blocks - kSoonBlocks)) mbar_arrive(&tsoon[acc]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        if (!(ti == 0 && (p.test_flags & B200K_GEMM_TEST_WITHHOLD_READY))) umma_commit(&tfull[acc]);
        stamp_tile(p, ti, 3);
        if (++acc == 2) {
          acc = 0;
          aph ^= 1u;
        }
      }
      // Every MMA this thread issued completes before TMEM can be released.
      umma_commit(drain);
      wait_bar_drain(drain, 0, 100000000ull);
    }
    __syncwarp();
  } else if (warp >= 4) {
    if constexpr (FAST) {
    // ------------------------------------------------------------ epilogue (compiled form)
    const int ew = warp - 4;
    epilogue_fast_loop<BN, OUT_BYTES, ACT, ROW>(p, &tmO, tmem_base, tfull, tempty, tsoon, sStg + ew * kStgBytes,
                                                reinterpret_cast<float*>(sbase + C::kBiasOff) + 32 * ew,
                                                warp & 3, ew >> 2, lane, ctl);
    } else {
    // ------------------------------------------------------------ epilogue (interpreted program)
    // Warp w reads TMEM lane quarter (w % 4) and one half of the tile's columns.
    static_assert(Epi<BN>::NG == 2, "the interpreted epilogue runs on 256- and 128-wide tiles");
    const int ew = warp - 4;
    const int quarter = warp & 3;
    const int half = ew >> 2;
    uint8_t* sb = sStg + ew * kStgBytes;
    int acc = 0;
    uint32_t aph = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
      int tm, tn;
      tile_coords(t, p, tm, tn);
      if (!wait_bar(&tfull[acc], aph, ctl)) break;
      tc_fence_after();
      const int m = tm * BM + quarter * 32 + lane;
      const int ncol0 = tn * BN + half * (BN / 2);
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc * BN + half * (BN / 2));
#pragma unroll 1
      for (int c = 0; c < (BN / 2) / C::kEC; ++c) {
        const int n0 = ncol0 + c * C::kEC;
        if (n0 >= p.N) break;
        if (!p.direct_store) {
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
        }
        {
          ExtraRegs xa, xb;
          load_extras(p, m, n0, xa);
#pragma unroll 1
          for (int g = 0; g < C::kEC / kEV; g += 2) {
            epilogue_group<OUT_BYTES>(p, t_row + c * C::kEC + g * kEV, m, n0 + g * kEV, g, lane, sb, xa, xb, true);
            epilogue_group<OUT_BYTES>(p, t_row + c * C::kEC + (g + 1) * kEV, m, n0 + (g + 1) * kEV, g + 1, lane, sb,
                                      xb, xa, g + 2 < C::kEC / kEV);
          }
        }
        if (!p.direct_store) {
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmO, sb, n0, tm * BM + quarter * 32);
            bulk_commit();
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        aph ^= 1u;
      }
    }
    if (!p.direct_store && lane == 0) bulk_wait_all();
    __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) stamp(p, 2);
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ------------------------------------------------------------ CTA-pair kernel
// 256-row tiles on a cluster of two CTAs (compiled epilogues, K-major B),
// the MMAs tcgen05 cta_group::2 with M = 256 and N = 256, each CTA supplying
// its own 128 A rows and half (128 rows) of each MMA's B rows.
//   narrow (WIDE = false): 256 x 256 tiles, a 32 KB stage per CTA (its A rows
//     and B half: a third less operand traffic per FLOP than one CTA's
//     128 x 256 tile), two 256-column accumulators, so a tile's epilogue
//     overlaps the next tile's MMAs;
//   wide (WIDE = true): 256 x 512 tiles, two MMAs per K step, one into each
//     256-column half of a single 512-column accumulator; a 48 KB stage per
//     CTA (its A rows and a B half for each MMA) carries 4/3 the FLOPs per
//     byte of the narrow tile.  The B200 tensor pipe outruns the operand
//     loads of the narrow tile (measured ~2030 TFLOP/s with the loads
//     removed, ~1450-1500 with them), so the wider tile's lower traffic per
//     FLOP is the one that pays; the price is that the next tile's MMAs
//     wait for the epilogue to release each half.
// Barriers: full[s] and tempty[a] live in the even CTA (the odd CTA's loads
// and epilogue complete and arrive there); empty[s] and tfull[a] in both
// CTAs (the even CTA's MMA thread commits to each copy).  Every wait is
// bounded as in the one-CTA kernel; cluster barriers open and close the
// kernel so that no CTA leaves while the other may still signal one of its
// barriers.
constexpr int kPairMmaN = 256;
template <int STAGES, int OUT_BYTES, bool WIDE>
struct PairCfg {
  static constexpr int kHalves = WIDE ? 2 : 1;  // MMAs (and B halves) per K step
  static constexpr uint32_t kABytes = BM * BK * 2;
  static constexpr uint32_t kBHalfBytes = (kPairMmaN / 2) * BK * 2;
  static constexpr uint32_t kBBytes = kHalves * kBHalfBytes;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kBarOff = STAGES * (kABytes + kBBytes) + Epi<kPairMmaN>::kWarps * kStgBytes;
  static constexpr uint32_t kBiasOff = kBarOff + 256;  // one 32-float bias slot per epilogue warp
  static constexpr uint32_t kSmem = 1024 + kBiasOff + Epi<kPairMmaN>::kWarps * 128;
  static_assert(kSmem <= 232448, "shared memory budget");
  static_assert(kSmem > 232448 / 2, "one CTA per SM keeps the TMEM allocation uncontended");
};

template <int STAGES, int OUT_BYTES, int ACT, int ROW, bool WIDE>
__global__ void __launch_bounds__(Epi<kPairMmaN>::kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmO, const __grid_constant__ Params p) {
  using C = PairCfg<STAGES, OUT_BYTES, WIDE>;
  constexpr int TN = C::kHalves * kPairMmaN;  // tile columns
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* sbase = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sA = sbase;
  uint8_t* sB = sA + STAGES * C::kABytes;
  uint8_t* sStg = sB + STAGES * C::kBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sbase + C::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* tsoon = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tsoon + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t rank = cluster_rank();
  const bool even = rank == 0;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) stamp(p, 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * Epi<kPairMmaN>::kWarps);
    }
    mbar_init(drain, 1);
    for (int a = 0; a < 2; ++a) mbar_init(&tsoon[a], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_map(&tmA);
    prefetch_map(&tmB);
    prefetch_map(&tmO);
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, C::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs: barriers initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const Ctl ctl{abort_flag, p.status, static_cast<uint64_t>(p.timeout_ns)};
  const int cid = static_cast<int>(blockIdx.x >> 1);
  const int ncl = static_cast<int>(gridDim.x >> 1);
  if (threadIdx.x == 0) stamp(p, 1);

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int64_t issued = 0;
      bool ok = true;
      int ti = 0;
      constexpr uint32_t kTx = 2 * (C::kABytes + C::kBBytes);  // both CTAs' loads of a stage
      for (int t = cid; t < p.num_tiles && ok; t += ncl, ++ti) {
        int tm, tn;
        tile_coords(t, p, tm, tn);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!wait_bar(&empty[s], ph ^ 1u, ctl)) {
            ok = false;
            break;
          }
          if (kb == 0) stamp_tile(p, ti, 0);
          if (kb == p.k_blocks - 1) stamp_tile(p, ti, 1);
          const uint32_t fb = cluster_addr(&full[s], 0);
          if (even) mbar_arrive_expect_tx(&full[s], kTx);
          tma_load_2d_pair(sA + s * C::kABytes, &tmA, fb, kb * BK, tm * (2 * BM) + static_cast<int>(rank) * BM);
#pragma unroll
          for (int h = 0; h < C::kHalves; ++h)
            tma_load_2d_pair(sB + s * C::kBBytes + h * C::kBHalfBytes, &tmB, fb, kb * BK,
                             tn * TN + h * kPairMmaN + static_cast<int>(rank) * (kPairMmaN / 2));
          ++issued;
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // Tail: wait until the MMA has released every stage this CTA filled, so
      // that no commit of the even CTA targets this CTA's barriers after the
      // closing cluster barrier.
      for (int x = 0; x < STAGES; ++x)
        if (issued > x) wait_bar_drain(&empty[x], x < s ? ph : (ph ^ 1u), 100000000ull);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (even && lane == 0) {
      int s = 0, acc = 0;
      uint32_t ph = 0, aph = 0;
      bool ok = true;
      int ti = 0;
      for (int t = cid; t < p.num_tiles && ok; t += ncl, ++ti) {
        if (!WIDE) {
          if (!wait_bar(&tempty[acc], aph ^ 1u, ctl)) break;
          tc_fence_after();
        }
        stamp_tile(p, ti, 2);
        for (int kb = 0; kb < p.k_blocks && ok; ++kb) {
          if (!wait_bar(&full[s], ph, ctl)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * C::kABytes);
#pragma unroll
          for (int h = 0; h < C::kHalves; ++h) {
            if (WIDE && kb == 0) {
              // the previous tile's epilogue has read this half
              if (!wait_bar(&tempty[h], (static_cast<uint32_t>(ti) & 1u) ^ 1u, ctl)) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>((WIDE ? h : acc) * kPairMmaN);
            const uint32_t b0 = smem_u32(sB + s * C::kBBytes + h * C::kBHalfBytes);
#pragma unroll
            for (int k = 0; k < BK / UMMA_K; ++k)
              umma_f16_pair(d_tmem, sw128_desc(a0 + k * (UMMA_K * 2), 16, 1024),
                            sw128_desc(b0 + k * (UMMA_K * 2), 16, 1024), p.idesc, (kb | k) != 0 ? 1u : 0u);
          }
          if (!ok) break;
          umma_commit_pair(smem_u32(&empty[s]));
          umma_commit_pair(cluster_addr(&empty[s], 1));
          // Local only: the even CTA's epilogue warms L2 for both CTAs' rows.
          // Signalling the odd CTA as well cost MMA issue time (measured on
          // 8192^3: a remote mbarrier arrive from this thread 701 -> 967 us,
          // two extra commits 722 -> 777 us).
          if (kb == max(0, p.k_blocks - kSoonBlocks)) mbar_arrive(&tsoon[acc]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        if (!(ti == 0 && (p.test_flags & B200K_GEMM_TEST_WITHHOLD_READY))) {
          umma_commit_pair(smem_u32(&tfull[acc]));
          umma_commit_pair(cluster_addr(&tfull[acc], 1));
        }
        stamp_tile(p, ti, 3);
        if (!WIDE && ++acc == 2) {
          acc = 0;
          aph ^= 1u;
        }
      }
      // Every MMA this thread issued completes before TMEM can be released.
      umma_commit_pair(smem_u32(drain));
      wait_bar_drain(drain, 0, 100000000ull);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int ew = warp - 4;
    epilogue_fast_loop<kPairMmaN, OUT_BYTES, ACT, ROW, true, WIDE>(p, &tmO, tmem_base, tfull, tempty, tsoon,
                                                                   sStg + ew * kStgBytes,
                                                                   reinterpret_cast<float*>(sbase + C::kBiasOff) +
                                                                       32 * ew,
                                                                   warp & 3, ew >> 2, lane,
                                                                   ctl, rank);
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the other can still signal its barriers
  if (threadIdx.x == 0) stamp(p, 2);
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::kTmemCols);
  }
}

template <int STAGES, int OB, int ACT, int ROW, bool WIDE>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, const Params& p, int grid,
                cudaStream_t st) {
  using C = PairCfg<STAGES, OB, WIDE>;
  auto kern = gemm_pair_kernel<STAGES, OB, ACT, ROW, WIDE>;
  static bool attr_set = false;  // per instantiation; idempotent
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) != cudaSuccess)
      return B200K_ERR_LAUNCH;
    attr_set = true;
  }
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(Epi<kPairMmaN>::kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, ta, tb, to, p) != cudaSuccess) return B200K_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? B200K_OK : B200K_ERR_LAUNCH;
}

struct TileConfig {
  int bm, bn, stages;  // bm 256: a CTA pair per tile
};
// Config 2 (192-wide tiles, twelve epilogue warps) and configs 3 and 4
// (256 x 256 and 256 x 512 tiles on CTA pairs) exist for compiled epilogues
// only; the pair configs also need K-major B and 16-bit output.
constexpr TileConfig kConfigs[] = {{128, 256, 4}, {128, 128, 6}, {128, 192, 4}, {256, 256, 6}, {256, 512, 4}};
constexpr int kNumConfigs = sizeof(kConfigs) / sizeof(kConfigs[0]);

template <int BN, int STAGES, bool BNM, int OB, bool FAST, int ACT, int ROW, bool TF32 = false, bool AMM = false>
int launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, const Params& p, int grid,
               cudaStream_t st) {
  using C = Cfg<BN, STAGES, BNM, OB>;
  auto kern = gemm_epilogue_kernel<BN, STAGES, BNM, OB, FAST, ACT, ROW, TF32, AMM>;
  static bool attr_set = false;  // per instantiation; idempotent
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) != cudaSuccess)
      return B200K_ERR_LAUNCH;
    attr_set = true;
  }
  kern<<<grid, Epi<BN>::kThreads, C::kSmem, st>>>(ta, tb, to, p);
  return cudaGetLastError() == cudaSuccess ? B200K_OK : B200K_ERR_LAUNCH;
}

// Compiled-epilogue kernels exist for these activations (others interpret).
constexpr int kFastActs[] = {B200K_ACT_NONE, B200K_ACT_GELU_ERF, B200K_ACT_GELU_TANH, B200K_ACT_SILU, B200K_ACT_RELU};

// Launchers of the compiled-epilogue kernels, one translation unit per
// (tile width, activation) so they compile in parallel (gemm_fast_*.cu).
// Each covers K-major B with 16-bit output and every row role, N-major B
// with 16-bit output and every row role, and K-major B with fp32 output
// without a row operand; B200K_ERR_UNSUPPORTED for anything else.
#define B200K_DECLARE_FAST(BN, ACT)                                                                          \
  int launch_fast_##BN##_##ACT(bool tf32, bool bnm, int ob, int row, const CUtensorMap& ta, const CUtensorMap& tb, \
                               const CUtensorMap& to, const Params& p, int grid, cudaStream_t st);
B200K_DECLARE_FAST(256, 0)
B200K_DECLARE_FAST(256, 1)
B200K_DECLARE_FAST(256, 2)
B200K_DECLARE_FAST(256, 3)
B200K_DECLARE_FAST(256, 4)
B200K_DECLARE_FAST(128, 0)
B200K_DECLARE_FAST(128, 1)
B200K_DECLARE_FAST(128, 2)
B200K_DECLARE_FAST(128, 3)
B200K_DECLARE_FAST(128, 4)
B200K_DECLARE_FAST(192, 0)
B200K_DECLARE_FAST(192, 1)
B200K_DECLARE_FAST(192, 2)
B200K_DECLARE_FAST(192, 3)
B200K_DECLARE_FAST(192, 4)
#undef B200K_DECLARE_FAST
// CTA-pair kernels (K-major B, 16-bit output, every row role): launch_pair_*
// runs the 256 x 256 tiles (config 3), launch_pairw_* the 256 x 512 tiles
// (config 4).
#define B200K_DECLARE_PAIR(ACT)                                                                                   \
  int launch_pair_##ACT(int row, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, const Params& p, \
                        int grid, cudaStream_t st);                                                               \
  int launch_pairw_##ACT(int row, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,            \
                         const Params& p, int grid, cudaStream_t st);
B200K_DECLARE_PAIR(0)
B200K_DECLARE_PAIR(1)
B200K_DECLARE_PAIR(2)
B200K_DECLARE_PAIR(3)
B200K_DECLARE_PAIR(4)
#undef B200K_DECLARE_PAIR

}  // namespace gemm
}  // namespace b200k
