/*
 * b200k.h — C ABI of libb200k.so, the sm_100a (B200) kernel library behind the
 * torch.compile backend in torch-compile-backend_b200/compiler.
 *
 * Plain C: device pointers, int64 sizes/strides (in ELEMENTS, not bytes), dtype
 * enums and a small epilogue program.  No torch or CUDA types appear in the
 * signatures; `stream` is a cudaStream_t passed as void* (NULL = legacy default
 * stream).  The library never allocates or frees device memory: outputs are
 * allocated by the caller.  Every entry point returns B200K_OK (0) or an error
 * code; b200k_status_string() turns it into text.  Errors detected on the host
 * (shapes, alignment, unsupported dtypes, launch failure) are returned
 * immediately; a device-side wait that runs out of time is reported through the
 * optional `status` word of the GEMM arguments (read it after synchronising).
 *
 * Reference interfaces replaced (aashrith-madasu/torch-compile-backend):
 *   b200k_pointwise      <- the generated `fused_<n>` Triton kernel and its launch
 *                           closure `fused_op(*tensors)`
 *                           compiler/optimization/fusion_pointwise.py:132-169,189-210
 *   b200k_gemm_epilogue  <- the generated autotuned `gemm_epilogue_<n>` Triton kernel
 *                           and its closure `epilogue_op(a, b, *tensors)`
 *                           compiler/optimization/fusion_epilogue.py:72-180; also the
 *                           standalone demos hand_written/gemm_kernel.py:6-71 and
 *                           hand_written/gemm_swizzled_kernel.py:5-89
 *   b200k_pointwise (ADD program) <- hand_written/matrix_add_kernel.py:6-46
 *   b200k_rownorm, b200k_softmax  <- no Triton counterpart: the reference leaves
 *                           pow/mean/native_layer_norm/_softmax to ATen
 *                           (compiler/optimization/fusion_pointwise.py:12-30 has no
 *                           reduction entries); these fuse the whole row group.
 */
#ifndef B200K_H
#define B200K_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200K_MAX_DIMS 6
#define B200K_MAX_INPUTS 8
#define B200K_MAX_SLOTS 8
#define B200K_MAX_INSTR 64

/* Element types. */
enum {
  B200K_F32 = 0,
  B200K_F16 = 1,
  B200K_BF16 = 2,
  B200K_F64 = 3,
  B200K_I32 = 4,
  B200K_I64 = 5,
  B200K_BOOL = 6,
  B200K_U8 = 7
};

/* Return codes. */
enum {
  B200K_OK = 0,
  B200K_ERR_ARG = 1,         /* null pointer, negative size, bad enum */
  B200K_ERR_ALIGN = 2,       /* pointer/stride alignment the kernel needs is not met */
  B200K_ERR_SHAPE = 3,       /* inconsistent or too large shape */
  B200K_ERR_UNSUPPORTED = 4, /* dtype/layout combination not implemented */
  B200K_ERR_LAUNCH = 5,      /* CUDA launch or attribute error */
  B200K_ERR_TIMEOUT = 6,     /* a device-side wait ran out of time (status word) */
  B200K_ERR_PROGRAM = 7,     /* malformed epilogue program */
  B200K_ERR_DEVICE = 8       /* no sm_100 device current */
};

/*
 * Epilogue / pointwise program: an accumulator machine evaluated per element in
 * fp32.  State: one accumulator `acc` and B200K_MAX_SLOTS value slots.  Before
 * the first instruction the slots hold the operands:
 *   b200k_pointwise:     slot i = inputs[i]             (i < n_inputs)
 *   b200k_gemm_epilogue: slot 0 = A·B accumulator, slot i = extras[i-1]
 * Instruction word: code = op * 10 + operand, operand 0..7 = slot, 8 = imm,
 * 9 = none.  Binary ops compute acc = acc (op) x; R* ops swap the operands.
 * After the last instruction `acc` is rounded to the output dtype and stored.
 * Op semantics follow compiler/optimization/fusion_pointwise.py:12-30 (fp32
 * math; tanh is 2*sigmoid(2x)-1; sigmoid is 1/(1+exp(-x)); relu/max/min return
 * the non-NaN operand).  ROUND_* are for fusions that cross a sub-fp32 cast.
 */
enum {
  B200K_OP_NOP = 0,
  B200K_OP_MOV = 1,    /* acc = x                    */
  B200K_OP_STORE = 2,  /* slot[operand] = acc        */
  B200K_OP_ADD = 3,
  B200K_OP_SUB = 4,    /* acc = acc - x              */
  B200K_OP_RSUB = 5,   /* acc = x - acc              */
  B200K_OP_MUL = 6,
  B200K_OP_DIV = 7,    /* acc = acc / x              */
  B200K_OP_RDIV = 8,   /* acc = x / acc              */
  B200K_OP_MAX = 9,
  B200K_OP_MIN = 10,
  B200K_OP_NEG = 11,
  B200K_OP_ABS = 12,
  B200K_OP_RELU = 13,
  B200K_OP_EXP = 14,
  B200K_OP_LOG = 15,
  B200K_OP_SQRT = 16,
  B200K_OP_RSQRT = 17,
  B200K_OP_ERF = 18,
  B200K_OP_SIGMOID = 19,
  B200K_OP_TANH = 20,
  B200K_OP_ROUND_BF16 = 21,
  B200K_OP_ROUND_F16 = 22,
  B200K_OP_COUNT = 23
};
#define B200K_OPERAND_IMM 8
#define B200K_OPERAND_NONE 9

typedef struct {
  int32_t code; /* op * 10 + operand */
  float imm;    /* used when operand == B200K_OPERAND_IMM */
} B200kInstr;

typedef struct {
  int32_t n;
  int32_t pad;
  B200kInstr ins[B200K_MAX_INSTR];
} B200kProgram;

/* A strided view broadcast to the output shape (stride 0 on broadcast dims). */
typedef struct {
  const void* ptr;
  int32_t dtype;
  int32_t pad;
  int64_t strides[B200K_MAX_DIMS];
} B200kTensorRef;

/*
 * out[i0..i_{r-1}] = program(inputs at the same index), out contiguous.
 * Replaces fusion_pointwise.py:132-169 (generated kernel) + :201-207 (launch).
 */
typedef struct {
  int32_t rank; /* 0..B200K_MAX_DIMS */
  int32_t n_inputs;
  int64_t sizes[B200K_MAX_DIMS];
  B200kTensorRef inputs[B200K_MAX_INPUTS];
  void* out;
  int32_t out_dtype;
  int32_t pad;
  B200kProgram program;
} B200kPointwiseArgs;

int b200k_pointwise(const B200kPointwiseArgs* args, void* stream);

/* b200k_pointwise runs a kernel generated for its program (compiled for
 * sm_100a by NVRTC on first use, cached per process and device) when the
 * launch merges to rank <= 2 with 32-bit unit indices and every operand is
 * bf16, f16 or f32 with innermost stride 0 or 1; the reference likewise
 * compiles one Triton kernel per fused group on first use
 * (compiler/optimization/fusion_pointwise.py:178-186).  Other launches, and
 * programs whose kernel could not be compiled or loaded, run the interpreter
 * kernels.  Setting B200K_POINTWISE_JIT=0 in the environment disables the
 * generated kernels.
 *
 * Counters of this process: kernels compiled and loaded, compile or load
 * failures, launches of generated kernels.  Any pointer may be null. */
int b200k_pointwise_jit_stats(int64_t* compiled, int64_t* failed, int64_t* launches);

/* Generates and compiles (no device needed, nothing loaded) the kernel for a
 * program over `n_inputs` (<= 4) operands of the given dtypes, each with
 * innermost stride 1 (unit_stride[i] != 0) or 0, at merged rank 1 or 2.
 * Writes NVRTC's log (truncated, NUL-terminated) to `log` when log_len > 0.
 * Returns B200K_OK, B200K_ERR_UNSUPPORTED (out of scope) or B200K_ERR_LAUNCH
 * (NVRTC missing or the compile failed). */
int b200k_pointwise_jit_compile(int rank, int n_inputs, const int32_t* dtypes, const int32_t* unit_stride,
                                int32_t out_dtype, const B200kProgram* program, char* log, int64_t log_len);

/* An epilogue operand indexed by the output coordinate (m, n). */
typedef struct {
  const void* ptr;
  int32_t dtype;
  int32_t pad;
  int64_t stride_m;
  int64_t stride_n;
} B200kEpiOperand;

/*
 * Canonical epilogue form.  When a program computes
 *     v = acc;  v += E[bias];  v = act(v);  v = round(v);  v *= E[scale];  v += E[residual]
 * (each step optional; E[i] = extras[i]) the GEMM kernel runs a compiled
 * path instead of interpreting the program.  The library checks the form
 * against the program (host-side evaluation on probe values) and rejects a
 * mismatch with B200K_ERR_PROGRAM.  kind = 0 always interprets.
 */
enum {
  B200K_ACT_NONE = 0,
  B200K_ACT_GELU_ERF = 1,   /* x*0.5 * (1 + erf(x*0.70710678)) */
  B200K_ACT_GELU_TANH = 2,  /* x*0.5 * (1 + tanh(0.79788456*(x + 0.044715*x^3))) */
  B200K_ACT_SILU = 3,       /* x * sigmoid(x) */
  B200K_ACT_RELU = 4,
  B200K_ACT_SIGMOID = 5,
  B200K_ACT_TANH = 6,
  B200K_ACT_COUNT = 7
};

typedef struct {
  int32_t kind;     /* 0 = interpret the program, 1 = canonical form */
  int32_t bias;     /* extras index or -1 */
  int32_t act;      /* B200K_ACT_* */
  int32_t round;    /* -1 none, else B200K_BF16 / B200K_F16: round after act */
  int32_t scale;    /* extras index or -1 */
  int32_t residual; /* extras index or -1 */
} B200kEpilogueForm;

/*
 * out[m,n] = program(acc[m,n], extras[..][m,n]) with acc = sum_k a[m,k]*b[k,n]
 * accumulated in fp32 on the tcgen05 tensor cores.  a is [M,K] with unit K
 * stride, or (16-bit, interpreted epilogues) unit M stride -- the transposed
 * gradient of a backward graph's weight-gradient mm; b is the reference's
 * mat2 [K,N] (usually t(W) with unit K stride, "K-major"; unit N stride,
 * "N-major", is also accepted).  a/b dtype: f16 or bf16, or f32 on the TF32
 * tensor cores (K-major a and b).  out: f16, bf16 or f32 with unit N
 * stride.
 * Replaces fusion_epilogue.py:72-151 (kernel), :164-177 (launch) and the
 * AUTOTUNE_CONFIGS table (:31-38) with a fixed B200 tile table.
 */
typedef struct {
  int64_t M, N, K;
  const void* a;
  int64_t a_stride_m, a_stride_k;
  const void* b;
  int64_t b_stride_k, b_stride_n;
  int32_t ab_dtype;
  int32_t out_dtype;
  void* out;
  int64_t out_stride_m, out_stride_n;
  int32_t n_extras;
  int32_t tile_config; /* -1 = pick from the built-in table */
  B200kEpiOperand extras[B200K_MAX_INPUTS - 1];
  B200kProgram program;
  int32_t* status;     /* optional device word: set to B200K_ERR_TIMEOUT by a stuck wait */
  int64_t timeout_ns;  /* 0 = default (2 s) */
  B200kEpilogueForm form;
  int32_t test_flags;  /* 0, or B200K_GEMM_TEST_* hooks for failure-detection tests */
  /* Optional diagnostic timeline (NULL = off): per CTA, B200K_GEMM_TRACE_WORDS
   * global-timer stamps (ns) -- [0] entry, [1] set-up done, [2] exit, then per
   * tile i < 40 at 8 + 6*i: first and last TMA issue, MMA start, last MMA
   * commit, epilogue start, epilogue end; for the first tile, words 248..255
   * hold per 32-column sub-chunk (s < 4) the time the accumulator was read
   * and the time the staging buffer was free.  Ignored unless trace_words covers
   * every CTA (148 x B200K_GEMM_TRACE_WORDS on a B200). */
  uint64_t* trace;
  int64_t trace_words;
} B200kGemmArgs;
#define B200K_GEMM_TRACE_WORDS 256
/* Test hook (test_flags bit): the MMA thread does not signal the first tile's
 * accumulator as ready, so the epilogue's wait on it runs out after
 * timeout_ns.  The kernel then takes its timeout path -- status word set to
 * B200K_ERR_TIMEOUT, every role leaves its loop, in-flight copies and MMAs
 * drain, TMEM is freed -- and returns; no fault, the context stays usable.
 * Never set outside failure-detection tests. */
#define B200K_GEMM_TEST_WITHHOLD_READY 1

int b200k_gemm_epilogue(const B200kGemmArgs* args, void* stream);

/*
 * Projection with the rotary position embedding as its epilogue:
 *   out[m, :] = rope(round(a[m, :] @ b)) per 64-column head, with
 *   rope(q)[d]      = round(round(q[d] cos[p][d]) - round(q[d + 32] sin[p][d]))
 *   rope(q)[d + 32] = round(round(q[d + 32] cos[p][d + 32]) + round(q[d] sin[p][d + 32]))
 * for d < 32 and p = m % period: x * cos + rotate_half(x) * sin with each
 * product and the sum rounded to the 16-bit output type, as eager PyTorch
 * computes it on the projection's 16-bit output.  Replaces the reference's
 * plain mm (left to ATen, compiler/optimization/fusion_epilogue.py:45-69
 * finds no pointwise anchor behind the view / transpose) followed by the
 * rotation's separate kernels; not in the reference.
 * args: as for b200k_gemm_epilogue with no extras and an empty program; a
 * K-major in a, K-major b (t(W)), out of a/b's 16-bit type, N a multiple of
 * 64, 16-byte aligned rows.  rope->cos / sin: [period, 64] tables of the
 * output type, unit column stride, row stride `stride` elements (a multiple
 * of 8), 16-byte aligned.  Runs the compiled epilogue on the 128 x 256,
 * 128 x 128 or 256 x 256 (CTA pair) tiles.
 */
typedef struct {
  const void* cos;
  const void* sin;
  int64_t stride;   /* elements between table rows */
  int64_t period;   /* table rows; output row m uses row m % period */
  int32_t head_dim; /* 64 */
  int32_t dtype;    /* the tables' (= the output's) */
} B200kRopeTables;
int b200k_gemm_rope(const B200kGemmArgs* args, const B200kRopeTables* rope, void* stream);

/*
 * b200k_gemm_epilogue for callers that cannot allocate device memory.
 * No reference counterpart: the reference has no allocation-free entry.
 * Hosts that run inside a graph-capture-only runtime, a plugin sandbox or a
 * custom memory manager may be unable to call cudaMalloc; the regular entry
 * needs them to supply the device status word (args->status).  This variant
 * ignores args->status and uses the library's own scratch instead: a
 * file-scope __device__ array of B200K_NOALLOC_SCRATCH_BYTES (256 bytes) that
 * every GPU which loads the library keeps until exit.  A call needs
 * B200K_NOALLOC_STATUS_BYTES of it (the status word, cleared on the stream
 * before the launch); a larger need is rejected with B200K_ERR_SHAPE.
 * The first call on a device looks up that device's copy of the array
 * (cudaGetSymbolAddress, with the device current); make that first call
 * before any stream capture: a first call on a capturing stream returns
 * B200K_ERR_LAUNCH and enqueues nothing.  The looked-up address is kept for
 * the life of the process; cudaDeviceReset invalidates it.  All calls share
 * the array: calls whose kernels overlap on the GPU race on the status word.
 * Inputs and outputs are passed as for b200k_gemm_epilogue; nothing is
 * allocated or freed.
 */
#define B200K_NOALLOC_SCRATCH_BYTES 256
#define B200K_NOALLOC_STATUS_BYTES 4
int b200k_gemm_epilogue_noalloc(const B200kGemmArgs* args, void* stream);
/* Reads the status word of the last b200k_gemm_epilogue_noalloc call on this
 * device into *host_out (B200K_OK, or B200K_ERR_TIMEOUT when one of its
 * device-side waits ran out): copies it on `stream` and synchronises with
 * that stream, so call it after the GEMM's launch on the same stream.  No
 * reference counterpart; allocates nothing (host_out is caller memory). */
int b200k_gemm_noalloc_status(int32_t* host_out, void* stream);

/* Number of GEMM tile configurations in the built-in table and their shapes
 * (block_m x block_n).  Config 2 (128 x 192 tiles) runs compiled epilogues
 * only; configs 3 and 4 (256 x 256 and 256 x 512 tiles, each computed by a
 * cluster of two CTAs on two SMs) run compiled epilogues with K-major B and
 * 16-bit output only.  A call forcing one outside its domain runs config 0
 * instead. */
int b200k_gemm_num_configs(void);
int b200k_gemm_config_info(int config, int* block_m, int* block_n, int* block_k, int* stages);
/* The configuration b200k_gemm_epilogue picks for a problem with a compiled
 * epilogue when tile_config is -1 (interpreted epilogues choose among 0, 1). */
int b200k_gemm_pick_config(int64_t M, int64_t N, int64_t K);

/*
 * Row normalisation over the last dim of a [rows, cols] view (unit column
 * stride), fp32 statistics.  No reference counterpart (the reference leaves
 * pow/mean/rsqrt partly to ATen and native_layer_norm wholly to ATen).
 *   RMSNORM:        n = x * rsqrt(mean(x^2) + eps)
 *   LAYERNORM:      n = (x - mean) * rsqrt(var + eps)          (biased var)
 *   RMSNORM_SWIGLU: n as RMSNORM over the full row, then
 *                   out[:, j] = silu(g_j) * u_j, g = y[:, :cols/2], u = y[:, cols/2:]
 * with y = affine(n) and the rounding points given by `flags`, so that the
 * kernel reproduces eager PyTorch's bf16/f16 rounding of the decomposed graph.
 */
enum {
  B200K_ROW_RMSNORM = 0,
  B200K_ROW_LAYERNORM = 1,
  B200K_ROW_RMSNORM_SWIGLU = 2
};
enum {
  B200K_ROWF_ROUND_NORMED = 1,  /* round n to x's dtype before the weight multiply */
  B200K_ROWF_ROUND_AFFINE = 2,  /* round y = n*w (+b) to the output dtype (affine done in low precision) */
  B200K_ROWF_ROUND_SILU = 4,    /* round silu(g) to the output dtype before multiplying by u */
  B200K_ROWF_WEIGHT_PLUS_ONE = 8 /* use (1 + w) as the scale (Gemma-style) */
};

typedef struct {
  int64_t rows, cols;
  const void* x;
  int64_t x_row_stride;
  int32_t x_dtype;
  int32_t kind;
  const void* weight; /* [cols] or NULL */
  int32_t w_dtype;
  int32_t flags;
  const void* bias;   /* [cols] or NULL (LAYERNORM only) */
  int32_t b_dtype;
  float eps;
  void* out;
  int64_t out_row_stride;
  int32_t out_dtype;
  int32_t pad;
  float* mean_out;    /* [rows] fp32 or NULL (LAYERNORM) */
  float* rstd_out;    /* [rows] fp32 or NULL (RMSNORM, LAYERNORM) */
} B200kRowNormArgs;

int b200k_rownorm(const B200kRowNormArgs* args, void* stream);

/* Row softmax (or log-softmax) over the last dim, fp32 math, like aten._softmax. */
typedef struct {
  int64_t rows, cols;
  const void* x;
  int64_t x_row_stride;
  int32_t x_dtype;
  int32_t log_softmax;
  void* out;
  int64_t out_row_stride;
  int32_t out_dtype;
  int32_t pad;
} B200kSoftmaxArgs;

int b200k_softmax(const B200kSoftmaxArgs* args, void* stream);

/* Rotary position embedding, rotate-half form (an extension: the reference
 * has no counterpart; its pointwise pass leaves the aten.cat of rotate_half
 * in ATen and fuses only x*cos + r*sin):
 *   out = x * cos + rotate_half(x) * sin,
 *   rotate_half(x)[..., j] = -x[..., j + D/2] for j < D/2, x[..., j - D/2] after,
 * over a rank-4 index space [B, H, S, D] (lower ranks padded with size-1
 * dims).  x, cos, sin and out are all bf16 or all f16, with any element
 * strides (0 broadcasts cos / sin).  Each product
 * and the sum round to that type, as the decomposed graph does, so the
 * result equals eager PyTorch bit for bit.  D even.  With D a multiple of 16,
 * unit stride in D and 16-byte aligned pointers and outer strides, each
 * thread moves 8 elements; any other layout runs an element-wise kernel. */
typedef struct {
  int64_t sizes[4];
  const void* x;
  int64_t x_strides[4];
  const void* cos;
  int64_t cos_strides[4];
  const void* sin;
  int64_t sin_strides[4];
  void* out;
  int64_t out_strides[4];
  int32_t dtype;
  int32_t pad;
} B200kRopeArgs;

int b200k_rope(const B200kRopeArgs* args, void* stream);

/*
 * Fused attention forward (an extension: the reference leaves
 * aten._scaled_dot_product_{flash,cudnn,efficient}_attention to ATen --
 * compiler/optimization/fusion_pointwise.py:12-30 has no attention op):
 *   out[b, h, i, :] = softmax_j(scale * q[b, h, i, :] . k[b, h / G, j, :]) v[b, h / G, j, :]
 * with G = heads / kv_heads (grouped-query attention; G = 1 for plain
 * multi-head attention) and, when `causal` is set, j restricted to j <= i
 * (the top-left aligned mask of torch SDPA's is_causal).  q, k, v, out are
 * bf16 or f16 (all the same), head_dim 64, element strides per [b, h, s, d]
 * with unit d stride, other strides multiples of 8 elements and 16-byte
 * aligned pointers (tensor-memory-access tiles).  Scores and the softmax run
 * in fp32; the probabilities are rounded to the input type for the second
 * product, as the flash kernels do.  `status`, when not NULL, receives
 * B200K_ERR_TIMEOUT if a device-side wait runs out (timeout_ns, 0 = 2 s).
 */
typedef struct {
  int64_t batch, heads, kv_heads, q_len, kv_len, head_dim;
  const void* q;
  int64_t q_strides[4];
  const void* k;
  int64_t k_strides[4];
  const void* v;
  int64_t v_strides[4];
  void* out;
  int64_t out_strides[4];
  int32_t dtype;  /* B200K_BF16 or B200K_F16 */
  int32_t causal;
  float scale;    /* <= 0: 1 / sqrt(head_dim) */
  int32_t test_flags; /* B200K_ATTN_TEST_* hooks (0 in production) */
  int32_t* status;
  int64_t timeout_ns;
} B200kAttentionArgs;
/* Test hook (test_flags bit): the MMA thread does not signal the first
 * score block of the first query tile as ready, so the softmax's wait on it
 * runs out after timeout_ns; the kernel reports B200K_ERR_TIMEOUT in the
 * status word, drains, frees its tensor memory and returns (no fault).
 * Failure-detection tests only. */
#define B200K_ATTN_TEST_WITHHOLD_SCORES 1

int b200k_attention(const B200kAttentionArgs* args, void* stream);

const char* b200k_status_string(int code);
/* Library version, for the loader's sanity check. */
int b200k_version(void);

#ifdef __cplusplus
}
#endif

#endif /* B200K_H */
