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
//   warps 4..11 epilogue, two warps per SM sub-partition: warp w reads TMEM
//               lane quarter (w % 4) and one half of the tile's columns with
//               tcgen05.ld (one output row per thread), runs the epilogue
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
constexpr int kEpiWarps = 8;               // two per SM sub-partition
constexpr int kThreads = 128 + 32 * kEpiWarps;  // warps 0-3 control, 4.. epilogue
constexpr int kGroupM = 16;
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
  int32_t pad2;
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
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
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
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 15u) == 0) {
      if (*c.abort) return false;
      if (global_timer_ns() - t0 > c.timeout_ns) {
        *c.abort = 1;
        if (c.status) atomicCAS(c.status, 0, B200K_ERR_TIMEOUT);
        return false;
      }
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
  const int per_group = kGroupM * p.tiles_n;
  const int g = t / per_group;
  const int first_m = g * kGroupM;
  const int gsize = min(p.tiles_m - first_m, kGroupM);
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
template <int ACT>
__device__ __forceinline__ void apply_act8(float (&v)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float x = v[j];
    if constexpr (ACT == B200K_ACT_GELU_ERF) {
      v[j] = (x * 0.5f) * (erff(x * 0.7071067811865476f) + 1.0f);
    } else if constexpr (ACT == B200K_ACT_GELU_TANH) {
      const float t3 = x + ((x * x) * x) * 0.044715f;
      v[j] = (x * 0.5f) * (op_tanh(t3 * 0.7978845608028654f) + 1.0f);
    } else if constexpr (ACT == B200K_ACT_SILU) {
      v[j] = x * op_sigmoid(x);
    } else if constexpr (ACT == B200K_ACT_RELU) {
      v[j] = fmaxf(x, 0.0f);
    } else if constexpr (ACT == B200K_ACT_SIGMOID) {
      v[j] = op_sigmoid(x);
    } else if constexpr (ACT == B200K_ACT_TANH) {
      v[j] = op_tanh(x);
    }
  }
}

// ------------------------------------------- fast path, latency-hiding loop
// Operand staging modes, chosen on the host per operand:
//   XM_BCAST   row-broadcast vector (stride_m == 0, e.g. a bias): each lane
//              loads one column of the 32-column sub-chunk (one coalesced
//              load per warp) and the values reach every row by __shfl_sync;
//   XM_ROW16   full 16-bit matrix with unit column stride (a residual, or the
//              `up` operand of SwiGLU): each lane loads its own row's 32
//              values (64 bytes) into registers;
//   XM_GENERIC anything else -- such programs run on the interpreter kernel.
// At most one operand is XM_ROW16.  Operands are prefetched one 32-column
// sub-chunk ahead, across tile boundaries, into one of two register sets
// that alternate between statically named copies.
enum { XM_NONE = 0, XM_BCAST = 1, XM_ROW16 = 2, XM_GENERIC = 3 };

struct FastOps {
  float bias_b, scale_b, res_b;
  uint4 row_r[4];  // the XM_ROW16 operand (scale or residual)
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

__device__ __forceinline__ float load_bcast(const EpiOperand& e, int n, int lane, int N) {
  const int col = n + lane;
  return col < N ? load_scalar(e.ptr, static_cast<int64_t>(col) * e.sn, e.dt) : 0.0f;
}

__device__ __forceinline__ void load_row16(const EpiOperand& e, int m, int n, int M, int N, uint4 (&b)[4]) {
  const uint16_t* base = reinterpret_cast<const uint16_t*>(e.ptr);
  if (m < M && n + 32 <= N) {
    const uint4* q = reinterpret_cast<const uint4*>(base + static_cast<int64_t>(m) * e.sm + n);
#pragma unroll
    for (int i = 0; i < 4; ++i) b[i] = __ldg(q + i);
  } else {
    uint32_t w[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t lo = (m < M && n + 2 * j < N) ? base[static_cast<int64_t>(m) * e.sm + n + 2 * j] : 0u;
      const uint32_t hi = (m < M && n + 2 * j + 1 < N) ? base[static_cast<int64_t>(m) * e.sm + n + 2 * j + 1] : 0u;
      w[j] = lo | (hi << 16);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) b[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
  }
}

__device__ __forceinline__ void fast_prefetch(const Params& p, int m, int n, int lane, FastOps& f) {
  if (p.xm_bias == XM_BCAST) f.bias_b = load_bcast(p.ex[p.f_bias], n, lane, p.N);
  if (p.xm_scale == XM_BCAST) f.scale_b = load_bcast(p.ex[p.f_scale], n, lane, p.N);
  else if (p.xm_scale == XM_ROW16) load_row16(p.ex[p.f_scale], m, n, p.M, p.N, f.row_r);
  if (p.xm_res == XM_BCAST) f.res_b = load_bcast(p.ex[p.f_res], n, lane, p.N);
  else if (p.xm_res == XM_ROW16) load_row16(p.ex[p.f_res], m, n, p.M, p.N, f.row_r);
}

__device__ __forceinline__ void unpack16x8(uint4 u, int dt, float (&x)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 f;
    if (dt == B200K_BF16) f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
    else f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
    x[2 * j] = f.x;
    x[2 * j + 1] = f.y;
  }
}

// The operand of one role for columns [n_g, n_g + 8) of the current sub-chunk (group g).
__device__ __forceinline__ void operand8(const Params& p, int mode, int idx, float bval, const uint4 (&r)[4], int g,
                                         float (&x)[8]) {
  if (mode == XM_BCAST) {
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = __shfl_sync(0xffffffffu, bval, g * 8 + j);
  } else {
    unpack16x8(r[g], p.ex[idx].dt, x);
  }
}

// One 32-column sub-chunk of one output row per lane: prefetch the operands
// of the next sub-chunk into `fill`, read the accumulator from TMEM, apply
// the canonical epilogue with the operands already in `use`, stage, store.
// `use` and `fill` are distinct named register sets at every call site, so
// reading `use` never waits on the loads just issued into `fill`.
template <int BN, int OUT_BYTES, int ACT>
__device__ __forceinline__ void fast_sub_chunk(const Params& p, const CUtensorMap* tmO, uint32_t t_row, int t,
                                               int tm, int tn, int s, int quarter, int half, int lane, uint8_t* sb,
                                               const FastOps& use, FastOps& fill, bool stamp_subs) {
  constexpr int kEC = 128 / OUT_BYTES;
  constexpr int NSUB = (BN / 2) / 32;
  constexpr int SUB_PER_STG = kEC / 32;
  const int m = tm * BM + quarter * 32 + lane;
  const int n = tn * BN + half * (BN / 2) + s * 32;
  if (s + 1 < NSUB) {
    fast_prefetch(p, m, n + 32, lane, fill);
  } else if (t + static_cast<int>(gridDim.x) < p.num_tiles) {
    int tm2, tn2;
    tile_coords(t + gridDim.x, p, tm2, tn2);
    fast_prefetch(p, tm2 * BM + quarter * 32 + lane, tn2 * BN + half * (BN / 2), lane, fill);
  }
  if (n >= p.N) return;  // warp-uniform
  uint32_t raw[32];
  tmem_ld32(t_row + s * 32, raw);
  tmem_wait_ld();
  // first tile of the trace: per sub-chunk, TMEM data in hand / staging free
  if (stamp_subs && s < 4) stamp(p, 248 + 2 * s);
  const int sub = s % SUB_PER_STG;
  if (sub == 0 && !p.direct_store) {
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();
  }
  if (stamp_subs && s < 4) stamp(p, 249 + 2 * s);
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int ng = n + g * 8;
    float v[8], x[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(raw[g * 8 + j]);
    if (p.f_bias >= 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] += __shfl_sync(0xffffffffu, use.bias_b, g * 8 + j);
    }
    apply_act8<ACT>(v);
    if (p.f_round == B200K_BF16) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = round_bf16(v[j]);
    } else if (p.f_round == B200K_F16) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = round_f16(v[j]);
    }
    if (p.f_scale >= 0) {
      operand8(p, p.xm_scale, p.f_scale, use.scale_b, use.row_r, g, x);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] *= x[j];
    }
    if (p.f_res >= 0) {
      operand8(p, p.xm_res, p.f_res, use.res_b, use.row_r, g, x);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] += x[j];
    }
    if (p.direct_store) {
      if (m < p.M) {
        const int64_t off = static_cast<int64_t>(m) * p.out_sm + ng;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (ng + j < p.N) store_scalar(p.out, off + j, p.out_dt, v[j]);
      }
    } else if (OUT_BYTES == 2) {
      const uint4 u = (p.out_dt == B200K_BF16) ? pack_bf16x8(v) : pack_f16x8(v);
      const int chunk = sub * 4 + g;
      *reinterpret_cast<uint4*>(sb + lane * 128 + ((chunk ^ (lane & 7)) << 4)) = u;
    } else {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int chunk = 2 * g + h;
        *reinterpret_cast<float4*>(sb + lane * 128 + ((chunk ^ (lane & 7)) << 4)) =
            make_float4(v[4 * h], v[4 * h + 1], v[4 * h + 2], v[4 * h + 3]);
      }
    }
  }
  if (!p.direct_store && (sub == SUB_PER_STG - 1 || s + 1 == NSUB || n + 32 >= p.N)) {
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmO, sb, n - sub * 32, tm * BM + quarter * 32);
      bulk_commit();
    }
  }
}

template <int BN, int OUT_BYTES, int ACT>
__device__ __forceinline__ void epilogue_fast_loop(const Params& p, const CUtensorMap* tmO, uint32_t tmem_base,
                                                   uint64_t* tfull, uint64_t* tempty, uint8_t* sb, int quarter,
                                                   int half, int lane, const Ctl& ctl) {
  constexpr int NSUB = (BN / 2) / 32;  // 32-column sub-chunks per warp and tile (even)
  static_assert(NSUB % 2 == 0, "sub-chunks alternate between two named register sets");
  FastOps opa, opb;
  if (static_cast<int>(blockIdx.x) < p.num_tiles) {
    int tm, tn;
    tile_coords(blockIdx.x, p, tm, tn);
    fast_prefetch(p, tm * BM + quarter * 32 + lane, tn * BN + half * (BN / 2), lane, opa);
  }
  int acc = 0;
  uint32_t aph = 0;
  const bool stamper = quarter == 0 && half == 0 && lane == 0;
  int ti = 0;
  for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++ti) {
    int tm, tn;
    tile_coords(t, p, tm, tn);
    if (!wait_bar(&tfull[acc], aph, ctl)) break;
    tc_fence_after();
    if (stamper) stamp_tile(p, ti, 4);
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                           static_cast<uint32_t>(acc * BN + half * (BN / 2));
#pragma unroll 1
    for (int s = 0; s < NSUB; s += 2) {
      fast_sub_chunk<BN, OUT_BYTES, ACT>(p, tmO, t_row, t, tm, tn, s, quarter, half, lane, sb, opa, opb,
                                         stamper && ti == 0);
      fast_sub_chunk<BN, OUT_BYTES, ACT>(p, tmO, t_row, t, tm, tn, s + 1, quarter, half, lane, sb, opb, opa,
                                         stamper && ti == 0);
    }
    if (stamper) stamp_tile(p, ti, 5);
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

template <int BN, int STAGES, bool B_NMAJOR, int OUT_BYTES>
struct Cfg {
  static constexpr uint32_t kABytes = BM * BK * 2;
  static constexpr uint32_t kBBytes = BN * BK * 2;
  static constexpr uint32_t kTmemCols = 2 * BN;
  static constexpr int kEC = 128 / OUT_BYTES;  // output columns per 128-byte staging row
  static constexpr uint32_t kBarOff = STAGES * (kABytes + kBBytes) + kEpiWarps * kStgBytes;
  static constexpr uint32_t kSmem = 1024 + kBarOff + 256;
  static_assert(kSmem <= 232448, "shared memory budget");
  static_assert(kSmem > 232448 / 2, "one CTA per SM keeps the TMEM allocation uncontended");
  static_assert(kTmemCols == 256 || kTmemCols == 512, "TMEM columns must be a power of two");
};

template <int BN, int STAGES, bool B_NMAJOR, int OUT_BYTES, bool FAST, int ACT>
__global__ void __launch_bounds__(kThreads, 1)
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
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
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
      mbar_init(&tempty[a], kEpiWarps);
    }
    mbar_init(drain, 1);
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
          tma_load_2d(sA + s * C::kABytes, &tmA, &full[s], kb * BK, tm * BM);
          if (B_NMAJOR) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sB + s * C::kBBytes + j * (64 * BK * 2), &tmB, &full[s], tn * BN + j * 64, kb * BK);
          } else {
            tma_load_2d(sB + s * C::kBBytes, &tmB, &full[s], kb * BK, tn * BN);
          }
          ++issued;
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let every load still in flight land before the CTA can exit.
        for (int x = 0; x < STAGES; ++x) {
          if (issued > x) {
            const uint32_t par = (x < s) ? ph : (ph ^ 1u);
            wait_bar_drain(&full[x], par, 100000000ull);
          }
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
            const uint64_t ad = sw128_desc(a0 + k * (UMMA_K * 2), 16, 1024);
            const uint64_t bd = B_NMAJOR ? sw128_desc(b0 + k * (UMMA_K * 128), 64 * BK * 2, 1024)
                                         : sw128_desc(b0 + k * (UMMA_K * 2), 16, 1024);
            umma_f16(d_tmem, ad, bd, p.idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[s]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
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
    epilogue_fast_loop<BN, OUT_BYTES, ACT>(p, &tmO, tmem_base, tfull, tempty, sStg + ew * kStgBytes, warp & 3,
                                           ew >> 2, lane, ctl);
    } else {
    // ------------------------------------------------------------ epilogue (interpreted program)
    // Warp w reads TMEM lane quarter (w % 4) and one half of the tile's columns.
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

struct TileConfig {
  int bn, stages;
};
constexpr TileConfig kConfigs[] = {{256, 4}, {128, 6}};
constexpr int kNumConfigs = sizeof(kConfigs) / sizeof(kConfigs[0]);

template <int BN, int STAGES, bool BNM, int OB, bool FAST, int ACT>
int launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, const Params& p, int grid,
               cudaStream_t st) {
  using C = Cfg<BN, STAGES, BNM, OB>;
  auto kern = gemm_epilogue_kernel<BN, STAGES, BNM, OB, FAST, ACT>;
  static bool attr_set = false;  // per instantiation; idempotent
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) != cudaSuccess)
      return B200K_ERR_LAUNCH;
    attr_set = true;
  }
  kern<<<grid, kThreads, C::kSmem, st>>>(ta, tb, to, p);
  return cudaGetLastError() == cudaSuccess ? B200K_OK : B200K_ERR_LAUNCH;
}

// Launchers of the compiled-epilogue kernels (one translation unit per tile
// width so they compile in parallel); B200K_ERR_UNSUPPORTED for a combination
// that has no compiled kernel (the caller then interprets the program).
int launch_fast_bn256(int act, bool bnm, int ob, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                      const Params& p, int grid, cudaStream_t st);
int launch_fast_bn128(int act, bool bnm, int ob, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                      const Params& p, int grid, cudaStream_t st);
bool fast_combo_exists(int act, bool bnm, int ob);

}  // namespace gemm
}  // namespace b200k
