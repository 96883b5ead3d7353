// Runtime-generated kernels for fused pointwise chains.
//
// The reference emits one Triton kernel per fused group
// (compiler/optimization/fusion_pointwise.py:132-169) and compiles it on first
// use (load_kernel, :178-186).  This file does the same for sm_100a with
// NVRTC: the group's accumulator-machine program (include/b200k.h) becomes
// straight-line CUDA C, one kernel per (program, input dtypes, broadcast
// kinds, output dtype, merged rank), compiled once per process and device
// and cached.  Compared with the interpreter kernels in pointwise.cu, the
// generated kernel has no per-instruction dispatch (the interpreter's switch
// costs ~10 branches per instruction per 8 elements), keeps only the slots the
// program names, and sizes its loads in flight to the registers that frees.
//
// Scope: merged rank 1 or 2, 32-bit unit indices, every input bf16, f16 or
// f32 with innermost stride 1 (16-byte vectors) or 0 (a broadcast scalar per
// unit), output bf16, f16 or f32.  Everything else, and any failure to
// compile or load (no NVRTC library, a stream in capture on first use), takes
// the interpreter kernels: those are the same op semantics on the GPU.
//
// Op semantics follow common.cuh: fp32 arithmetic, one IEEE rounding per op
// (the __f*_rn intrinsics are never contracted into FMAs), exp/log/sigmoid on
// the hardware ex2/lg2 approximations, tanh = 2*sigmoid(2x)-1, erf IEEE.
#include <cuda.h>
#include <dlfcn.h>
#include <nvrtc.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "host_common.h"
#include "pointwise_jit.h"

#define B200K_STR_(...) #__VA_ARGS__
#define B200K_STR(...) B200K_STR_(__VA_ARGS__)

namespace b200k {

// Kernel parameters: defined once, compiled here and pasted into every
// generated source.
#define B200K_PW_JIT_PARAMS                                                               \
  struct PwJitParams {                                                                  \
    const void* in[4];                                                                   \
    void* out;                                                                           \
    long long stride0[4]; /* elements per step of dim 0 (rank 2) or per unit (rank 1) */ \
    long long stride1[4]; /* elements per unit of the inner dim (rank 2)              */ \
    unsigned int nunits;                                                                 \
    unsigned int div_d, div_m, div_s; /* units per row (rank 2), multiply-shift form  */ \
  };
B200K_PW_JIT_PARAMS

namespace {

constexpr int kJitMaxInputs = 4;

// Device helpers of every generated kernel.  Conversions are single PTX cvt
// instructions (round to nearest even), so no CUDA header is needed.
const char* kPrelude = R"(
typedef unsigned int u32;
typedef unsigned long long u64;
typedef long long i64;
)" B200K_STR(B200K_PW_JIT_PARAMS) R"(
__device__ __forceinline__ uint4 ldg16(const void* p) {
  uint4 r;
  asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ float bf_lo(u32 w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(u32 w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ float h_to_f(unsigned short h) { float f; asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h)); return f; }
__device__ __forceinline__ float h_lo(u32 w) { return h_to_f((unsigned short)(w & 0xffffu)); }
__device__ __forceinline__ float h_hi(u32 w) { return h_to_f((unsigned short)(w >> 16)); }
__device__ __forceinline__ u32 pack_bf(float lo, float hi) {
  u32 d; asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo)); return d;
}
__device__ __forceinline__ u32 pack_h(float lo, float hi) {
  u32 d; asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo)); return d;
}
__device__ __forceinline__ float rnd_bf(float x) { return __uint_as_float(pack_bf(x, 0.0f) << 16); }
__device__ __forceinline__ float rnd_h(float x) {
  float y; asm("{ .reg .b16 h; cvt.rn.f16.f32 h, %1; cvt.f32.f16 %0, h; }" : "=f"(y) : "f"(x)); return y;
}
__device__ __forceinline__ float op_sigmoid(float x) { return __fdividef(1.0f, __fadd_rn(1.0f, __expf(-x))); }
__device__ __forceinline__ float op_tanh(float x) {
  return __fsub_rn(__fmul_rn(2.0f, op_sigmoid(__fmul_rn(2.0f, x))), 1.0f);
}
)";

int elem_bytes(int dt) { return dt == B200K_F32 ? 4 : 2; }

// One fp32 literal, bit-exact.
std::string lit(float v) {
  uint32_t u;
  std::memcpy(&u, &v, 4);
  char b[32];
  std::snprintf(b, sizeof b, "__uint_as_float(0x%08xu)", u);
  return b;
}

// CUDA C for one instruction on the per-element state (acc, s0..s7).
std::string emit_instr(const B200kInstr& in) {
  const int op = in.code / 10, operand = in.code % 10;
  const std::string x = operand == B200K_OPERAND_IMM ? lit(in.imm) : "s" + std::to_string(operand);
  switch (op) {
    case B200K_OP_NOP: return "";
    case B200K_OP_MOV: return "acc = " + x + ";";
    case B200K_OP_STORE: return "s" + std::to_string(operand) + " = acc;";
    case B200K_OP_ADD: return "acc = __fadd_rn(acc, " + x + ");";
    case B200K_OP_SUB: return "acc = __fsub_rn(acc, " + x + ");";
    case B200K_OP_RSUB: return "acc = __fsub_rn(" + x + ", acc);";
    case B200K_OP_MUL: return "acc = __fmul_rn(acc, " + x + ");";
    case B200K_OP_DIV: return "acc = __fdiv_rn(acc, " + x + ");";
    case B200K_OP_RDIV: return "acc = __fdiv_rn(" + x + ", acc);";
    case B200K_OP_MAX: return "acc = fmaxf(acc, " + x + ");";
    case B200K_OP_MIN: return "acc = fminf(acc, " + x + ");";
    case B200K_OP_NEG: return "acc = -acc;";
    case B200K_OP_ABS: return "acc = fabsf(acc);";
    case B200K_OP_RELU: return "acc = fmaxf(acc, 0.0f);";
    case B200K_OP_EXP: return "acc = __expf(acc);";
    case B200K_OP_LOG: return "acc = __logf(acc);";
    case B200K_OP_SQRT: return "acc = __fsqrt_rn(acc);";
    case B200K_OP_RSQRT: return "acc = rsqrtf(acc);";
    case B200K_OP_ERF: return "acc = erff(acc);";
    case B200K_OP_SIGMOID: return "acc = op_sigmoid(acc);";
    case B200K_OP_TANH: return "acc = op_tanh(acc);";
    case B200K_OP_ROUND_BF16: return "acc = rnd_bf(acc);";
    case B200K_OP_ROUND_F16: return "acc = rnd_h(acc);";
    default: return "";
  }
}

struct JitKey {
  int rank, nin, out_dt, units_per_thread;
  int dt[kJitMaxInputs];
  bool unit[kJitMaxInputs];  // innermost stride 1 (else 0: one scalar per unit)
};

std::string key_string(const JitKey& k, const B200kProgram& prog, int device) {
  std::string s(reinterpret_cast<const char*>(&k), sizeof(k));
  s.append(reinterpret_cast<const char*>(&device), sizeof(device));
  s.append(reinterpret_cast<const char*>(&prog.n), sizeof(prog.n));
  s.append(reinterpret_cast<const char*>(prog.ins), sizeof(B200kInstr) * prog.n);
  return s;
}

// Loads per thread in flight: units of 8 elements per loop step, chosen by
// the 16-byte words one unit reads over all unit-stride inputs.
int units_per_thread(const JitKey& k) {
  int words = 0;
  for (int i = 0; i < k.nin; ++i)
    if (k.unit[i]) words += elem_bytes(k.dt[i]) / 2;
  return words <= 2 ? 4 : words <= 4 ? 2 : 1;
}

std::string generate(const JitKey& k, const B200kProgram& prog) {
  std::string s = kPrelude;
  const int U = k.units_per_thread;
  s += "extern \"C\" __global__ void __launch_bounds__(256) b200k_pw_jit(const __grid_constant__ PwJitParams p) {\n";
  s += "  const u32 total = p.nunits;\n";
  s += "  const u32 step = gridDim.x * blockDim.x * " + std::to_string(U) + "u;\n";
  s += "  for (u32 base = blockIdx.x * blockDim.x * " + std::to_string(U) +
       "u + threadIdx.x; base < total; base += step) {\n";
  // Declarations of the raw inputs of every unit.
  for (int i = 0; i < k.nin; ++i) {
    const std::string I = std::to_string(i);
    if (!k.unit[i]) {
      s += "    float c" + I + "[" + std::to_string(U) + "];\n";
    } else {
      const int words = elem_bytes(k.dt[i]) / 2;
      s += "    uint4 w" + I + "[" + std::to_string(U) + "][" + std::to_string(words) + "];\n";
    }
  }
  // Phase 1: issue every load of the U units.
  s += "#pragma unroll\n    for (int k = 0; k < " + std::to_string(U) + "; ++k) {\n";
  s += "      const u32 u = base + k * blockDim.x;\n      if (u >= total) break;\n";
  if (k.rank == 2)
    s += "      const u32 i0 = (__umulhi(u, p.div_m) + u) >> p.div_s;\n      const u32 i1 = u - i0 * p.div_d;\n";
  for (int i = 0; i < k.nin; ++i) {
    const std::string I = std::to_string(i);
    const std::string off = k.rank == 2 ? "(i64)i0 * p.stride0[" + I + "] + (i64)i1 * p.stride1[" + I + "]"
                                        : "(i64)u * p.stride0[" + I + "]";
    const std::string addr = "(const char*)p.in[" + I + "] + (" + off + ") * " + std::to_string(elem_bytes(k.dt[i]));
    if (k.unit[i]) {
      const int words = elem_bytes(k.dt[i]) / 2;
      s += "      { const uint4* q = (const uint4*)(" + addr + ");\n";
      for (int w = 0; w < words; ++w)
        s += "        w" + I + "[k][" + std::to_string(w) + "] = ldg16(q + " + std::to_string(w) + ");\n";
      s += "      }\n";
    } else {
      switch (k.dt[i]) {
        case B200K_F32: s += "      c" + I + "[k] = __ldg((const float*)(" + addr + "));\n"; break;
        case B200K_BF16:
          s += "      c" + I + "[k] = __uint_as_float((u32)__ldg((const unsigned short*)(" + addr + ")) << 16);\n";
          break;
        default: s += "      c" + I + "[k] = h_to_f(__ldg((const unsigned short*)(" + addr + ")));\n"; break;
      }
    }
  }
  s += "    }\n";
  // Phase 2: per unit, unpack, run the program per element, pack, store.
  s += "#pragma unroll\n    for (int k = 0; k < " + std::to_string(U) + "; ++k) {\n";
  s += "      const u32 u = base + k * blockDim.x;\n      if (u >= total) break;\n";
  for (int i = 0; i < k.nin; ++i) {
    if (!k.unit[i]) continue;
    const std::string I = std::to_string(i);
    s += "      float v" + I + "[8];\n";
    if (k.dt[i] == B200K_F32) {
      s += "      { const float* f = (const float*)&w" + I + "[k][0];\n";
      s += "#pragma unroll\n        for (int j = 0; j < 8; ++j) v" + I + "[j] = f[j]; }\n";
    } else {
      const char* lo = k.dt[i] == B200K_BF16 ? "bf_lo" : "h_lo";
      const char* hi = k.dt[i] == B200K_BF16 ? "bf_hi" : "h_hi";
      s += "      { const u32 q[4] = {w" + I + "[k][0].x, w" + I + "[k][0].y, w" + I + "[k][0].z, w" + I + "[k][0].w};\n";
      s += "#pragma unroll\n        for (int j = 0; j < 4; ++j) { v" + I + "[2 * j] = " + lo + "(q[j]); v" + I +
           "[2 * j + 1] = " + hi + "(q[j]); } }\n";
    }
  }
  s += "      float o[8];\n#pragma unroll\n      for (int j = 0; j < 8; ++j) {\n";
  const int nslots = slots_used(prog, k.nin);
  for (int t = 0; t < nslots; ++t) {
    const std::string T = std::to_string(t);
    if (t < k.nin)
      s += "        float s" + T + " = " + (k.unit[t] ? "v" + T + "[j]" : "c" + T + "[k]") + ";\n";
    else
      s += "        float s" + T + " = 0.0f;\n";
  }
  s += "        float acc = s0;\n";
  for (int pc = 0; pc < prog.n; ++pc) {
    const std::string line = emit_instr(prog.ins[pc]);
    if (!line.empty()) s += "        " + line + "\n";
  }
  for (int t = 0; t < nslots; ++t) s += "        (void)s" + std::to_string(t) + ";\n";
  s += "        o[j] = acc;\n      }\n";
  s += "      char* dst = (char*)p.out + (i64)u * " + std::to_string(8 * elem_bytes(k.out_dt)) + ";\n";
  if (k.out_dt == B200K_F32) {
    s += "      ((float4*)dst)[0] = make_float4(o[0], o[1], o[2], o[3]);\n";
    s += "      ((float4*)dst)[1] = make_float4(o[4], o[5], o[6], o[7]);\n";
  } else {
    const char* pk = k.out_dt == B200K_BF16 ? "pack_bf" : "pack_h";
    s += std::string("      *(uint4*)dst = make_uint4(") + pk + "(o[0], o[1]), " + pk + "(o[2], o[3]), " + pk +
         "(o[4], o[5]), " + pk + "(o[6], o[7]));\n";
  }
  s += "    }\n  }\n}\n";
  return s;
}

// ---- NVRTC, loaded on first use -------------------------------------------
struct Nvrtc {
  decltype(&nvrtcCreateProgram) create = nullptr;
  decltype(&nvrtcCompileProgram) compile = nullptr;
  decltype(&nvrtcGetProgramLogSize) log_size = nullptr;
  decltype(&nvrtcGetProgramLog) log = nullptr;
  decltype(&nvrtcGetCUBINSize) cubin_size = nullptr;
  decltype(&nvrtcGetCUBIN) cubin = nullptr;
  decltype(&nvrtcDestroyProgram) destroy = nullptr;
  bool ok = false;
};

const Nvrtc& nvrtc() {
  static Nvrtc n;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* names[] = {"libnvrtc.so.12", "libnvrtc.so", "/usr/local/cuda/lib64/libnvrtc.so.12"};
    void* h = nullptr;
    for (const char* nm : names)
      if ((h = dlopen(nm, RTLD_NOW | RTLD_LOCAL)) != nullptr) break;
    if (!h) return;
    n.create = reinterpret_cast<decltype(n.create)>(dlsym(h, "nvrtcCreateProgram"));
    n.compile = reinterpret_cast<decltype(n.compile)>(dlsym(h, "nvrtcCompileProgram"));
    n.log_size = reinterpret_cast<decltype(n.log_size)>(dlsym(h, "nvrtcGetProgramLogSize"));
    n.log = reinterpret_cast<decltype(n.log)>(dlsym(h, "nvrtcGetProgramLog"));
    n.cubin_size = reinterpret_cast<decltype(n.cubin_size)>(dlsym(h, "nvrtcGetCUBINSize"));
    n.cubin = reinterpret_cast<decltype(n.cubin)>(dlsym(h, "nvrtcGetCUBIN"));
    n.destroy = reinterpret_cast<decltype(n.destroy)>(dlsym(h, "nvrtcDestroyProgram"));
    n.ok = n.create && n.compile && n.log_size && n.log && n.cubin_size && n.cubin && n.destroy;
  });
  return n;
}

// Compiles `src` for sm_100a; returns the cubin or an empty vector (log in `err`).
std::vector<char> compile_cubin(const std::string& src, std::string* err) {
  const Nvrtc& n = nvrtc();
  if (!n.ok) {
    if (err) *err = "NVRTC library not found";
    return {};
  }
  nvrtcProgram prog;
  if (n.create(&prog, src.c_str(), "b200k_pw_jit.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS) {
    if (err) *err = "nvrtcCreateProgram failed";
    return {};
  }
  const char* opts[] = {"-arch=sm_100a", "-std=c++17"};
  const nvrtcResult rc = n.compile(prog, 2, opts);
  std::vector<char> out;
  if (rc != NVRTC_SUCCESS) {
    size_t ls = 0;
    n.log_size(prog, &ls);
    std::string log(ls, '\0');
    if (ls) n.log(prog, &log[0]);
    if (err) *err = log;
  } else {
    size_t cs = 0;
    n.cubin_size(prog, &cs);
    out.resize(cs);
    n.cubin(prog, out.data());
  }
  n.destroy(&prog);
  return out;
}

// ---- Driver entry points (module load and launch) -------------------------
struct Driver {
  CUresult (*load)(CUmodule*, const void*) = nullptr;
  CUresult (*get)(CUfunction*, CUmodule, const char*) = nullptr;
  CUresult (*launch)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, CUstream,
                     void**, void**) = nullptr;
  CUresult (*occupancy)(int*, CUfunction, int, size_t) = nullptr;
  bool ok = false;
};

template <typename F>
void entry(const char* name, F* fn) {
  void* f = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &f, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
    *fn = reinterpret_cast<F>(f);
}

const Driver& driver() {
  static Driver d;
  static std::once_flag once;
  std::call_once(once, [] {
    entry("cuModuleLoadData", &d.load);
    entry("cuModuleGetFunction", &d.get);
    entry("cuLaunchKernel", &d.launch);
    entry("cuOccupancyMaxActiveBlocksPerMultiprocessor", &d.occupancy);
    d.ok = d.load && d.get && d.launch && d.occupancy;
  });
  return d;
}

struct JitKernel {
  CUfunction fn = nullptr;  // null: compiling or loading failed (the interpreter serves the key)
  int per_sm = 1;
};

struct JitCache {
  std::mutex mu;
  std::unordered_map<std::string, JitKernel> map;
  int64_t compiled = 0, failed = 0, launches = 0;
};

JitCache& cache() {
  static JitCache* c = new JitCache();  // never destroyed: modules live for the process
  return *c;
}

// Read at every launch, so a host can switch per call.
bool jit_enabled() {
  const char* e = std::getenv("B200K_POINTWISE_JIT");
  return !(e && e[0] == '0');
}

// Fills `k` for a launch, or returns false when the launch is outside the
// generated kernels' scope.
bool make_key(const B200kPointwiseArgs* a, const PwJitLaunch& L, JitKey* k) {
  if (L.rank < 1 || L.rank > 2 || L.nin > kJitMaxInputs) return false;
  if (a->out_dtype != B200K_F32 && a->out_dtype != B200K_BF16 && a->out_dtype != B200K_F16) return false;
  std::memset(k, 0, sizeof(*k));
  k->rank = L.rank;
  k->nin = L.nin;
  k->out_dt = a->out_dtype;
  for (int i = 0; i < L.nin; ++i) {
    const int dt = a->inputs[i].dtype;
    if (dt != B200K_F32 && dt != B200K_BF16 && dt != B200K_F16) return false;
    if (L.inner_stride[i] != 0 && L.inner_stride[i] != 1) return false;
    k->dt[i] = dt;
    k->unit[i] = L.inner_stride[i] == 1;
  }
  k->units_per_thread = units_per_thread(*k);
  return true;
}

}  // namespace

int pointwise_jit_launch(const B200kPointwiseArgs* a, const PwJitLaunch& L, cudaStream_t stream) {
  if (!jit_enabled()) return B200K_ERR_UNSUPPORTED;
  JitKey k;
  if (!make_key(a, L, &k)) return B200K_ERR_UNSUPPORTED;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return B200K_ERR_DEVICE;
  const std::string key = key_string(k, a->program, device);
  JitCache& c = cache();
  JitKernel kern;
  {
    std::lock_guard<std::mutex> lock(c.mu);
    auto it = c.map.find(key);
    if (it != c.map.end()) {
      kern = it->second;
    } else {
      // Loading a module is not a stream operation: never the first use of a
      // program inside a stream capture (the interpreter serves that launch).
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone)
        return B200K_ERR_UNSUPPORTED;
      const Driver& d = driver();
      std::vector<char> bin = d.ok ? compile_cubin(generate(k, a->program), nullptr) : std::vector<char>();
      CUmodule mod = nullptr;
      if (!bin.empty() && d.load(&mod, bin.data()) == CUDA_SUCCESS &&
          d.get(&kern.fn, mod, "b200k_pw_jit") == CUDA_SUCCESS) {
        int v = 0;
        if (d.occupancy(&v, kern.fn, 256, 0) == CUDA_SUCCESS && v > 0) kern.per_sm = v;
        ++c.compiled;
      } else {
        kern.fn = nullptr;
        ++c.failed;
      }
      c.map.emplace(key, kern);
    }
  }
  if (!kern.fn) return B200K_ERR_UNSUPPORTED;

  PwJitParams p;
  std::memset(&p, 0, sizeof(p));
  for (int i = 0; i < L.nin; ++i) {
    p.in[i] = a->inputs[i].ptr;
    p.stride0[i] = L.stride0[i];
    p.stride1[i] = L.stride1[i];
  }
  p.out = a->out;
  p.nunits = static_cast<uint32_t>(L.units);
  if (L.rank == 2) {
    const auto f = make_fastdiv(static_cast<uint32_t>(L.inner_units));
    p.div_d = f.d;
    p.div_m = f.m;
    p.div_s = f.s;
  }
  const int sms = device_sm_count();
  if (sms <= 0) return B200K_ERR_DEVICE;
  const int64_t per_cta = 256 * static_cast<int64_t>(k.units_per_thread);
  const int64_t want = (L.units + per_cta - 1) / per_cta;
  const unsigned grid =
      static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(want, static_cast<int64_t>(sms) * kern.per_sm)));
  void* params[] = {&p};
  if (driver().launch(kern.fn, grid, 1, 1, 256, 1, 1, 0, reinterpret_cast<CUstream>(stream), params, nullptr) !=
      CUDA_SUCCESS)
    return B200K_ERR_LAUNCH;
  {
    std::lock_guard<std::mutex> lock(c.mu);
    ++c.launches;
  }
  return B200K_OK;
}

}  // namespace b200k

using namespace b200k;

extern "C" int b200k_pointwise_jit_stats(int64_t* compiled, int64_t* failed, int64_t* launches) {
  JitCache& c = cache();
  std::lock_guard<std::mutex> lock(c.mu);
  if (compiled) *compiled = c.compiled;
  if (failed) *failed = c.failed;
  if (launches) *launches = c.launches;
  return B200K_OK;
}

extern "C" int b200k_pointwise_jit_compile(int rank, int n_inputs, const int32_t* dtypes, const int32_t* unit_stride,
                                           int32_t out_dtype, const B200kProgram* program, char* log,
                                           int64_t log_len) {
  if (!program || !dtypes || !unit_stride) return B200K_ERR_ARG;
  if (n_inputs < 1 || n_inputs > kJitMaxInputs || rank < 1 || rank > 2) return B200K_ERR_UNSUPPORTED;
  int rc = validate_program(*program, n_inputs);
  if (rc != B200K_OK) return rc;
  JitKey k;
  std::memset(&k, 0, sizeof(k));
  k.rank = rank;
  k.nin = n_inputs;
  k.out_dt = out_dtype;
  if (out_dtype != B200K_F32 && out_dtype != B200K_BF16 && out_dtype != B200K_F16) return B200K_ERR_UNSUPPORTED;
  for (int i = 0; i < n_inputs; ++i) {
    if (dtypes[i] != B200K_F32 && dtypes[i] != B200K_BF16 && dtypes[i] != B200K_F16) return B200K_ERR_UNSUPPORTED;
    k.dt[i] = dtypes[i];
    k.unit[i] = unit_stride[i] != 0;
  }
  k.units_per_thread = units_per_thread(k);
  std::string err;
  const std::vector<char> bin = compile_cubin(generate(k, *program), &err);
  if (log && log_len > 0) {
    const size_t n = std::min<size_t>(err.size(), static_cast<size_t>(log_len - 1));
    std::memcpy(log, err.data(), n);
    log[n] = '\0';
  }
  return bin.empty() ? B200K_ERR_LAUNCH : B200K_OK;
}
