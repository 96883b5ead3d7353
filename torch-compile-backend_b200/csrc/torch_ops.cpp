// Thin PyTorch binding: registers torch.ops.b200.* (CUDA dispatch key) and
// forwards each call to the C ABI of libb200k.so (include/b200k.h).
//
// These ops are what the rewritten FX graph calls in place of the reference's
// Python closures `fused_op(*tensors)` (compiler/optimization/
// fusion_pointwise.py:201-207) and `epilogue_op(a, b, *tensors)`
// (compiler/optimization/fusion_epilogue.py:164-177).  Like those closures they
// allocate the output with the caching allocator (torch.empty) and launch on
// the current stream; unlike them they never fall back to anything: a
// library error becomes a RuntimeError.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <vector>

#include "b200k.h"

namespace {

int to_dt(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return B200K_F32;
    case at::kHalf: return B200K_F16;
    case at::kBFloat16: return B200K_BF16;
    case at::kDouble: return B200K_F64;
    case at::kInt: return B200K_I32;
    case at::kLong: return B200K_I64;
    case at::kBool: return B200K_BOOL;
    case at::kByte: return B200K_U8;
    default: TORCH_CHECK(false, "b200: unsupported dtype ", t);
  }
  return -1;
}

void check(int rc, const char* what) {
  TORCH_CHECK(rc == B200K_OK, "b200::", what, " failed: ", b200k_status_string(rc), " (code ", rc, ")");
}

B200kProgram make_program(at::IntArrayRef code, at::ArrayRef<double> imm) {
  TORCH_CHECK(code.size() == imm.size(), "b200: program code/imm length mismatch");
  TORCH_CHECK(static_cast<int64_t>(code.size()) <= B200K_MAX_INSTR, "b200: program too long (", code.size(), ")");
  B200kProgram p;
  std::memset(&p, 0, sizeof(p));
  p.n = static_cast<int32_t>(code.size());
  for (size_t i = 0; i < code.size(); ++i) {
    p.ins[i].code = static_cast<int32_t>(code[i]);
    p.ins[i].imm = static_cast<float>(imm[i]);
  }
  return p;
}

void* stream_of(const at::Tensor& t) {
  return static_cast<void*>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

std::atomic<int64_t> g_test_stall_ns{0};

// Per-device status word the GEMM kernel writes when a wait times out.
at::Tensor& status_word(int dev) {
  static std::mutex mu;
  static std::vector<at::Tensor> words;
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(words.size()) <= dev) words.resize(dev + 1);
  if (!words[dev].defined())
    words[dev] = at::zeros({1}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, dev));
  return words[dev];
}

// out_stride (optional) gives the output the layout the replaced ATen op would
// have produced (elementwise ops keep their inputs' memory order); it must be
// a dense permutation of a contiguous layout.  The kernel then iterates the
// dims in output-stride order, so it still writes the output densely.
at::Tensor pointwise(at::TensorList inputs, at::IntArrayRef code, at::ArrayRef<double> imm,
                     at::IntArrayRef out_shape, at::ScalarType out_dtype, at::IntArrayRef out_stride) {
  TORCH_CHECK(!inputs.empty() && inputs.size() <= B200K_MAX_INPUTS, "b200::pointwise: 1..8 inputs, got ",
              inputs.size());
  const int rank = static_cast<int>(out_shape.size());
  TORCH_CHECK(rank <= B200K_MAX_DIMS, "b200::pointwise: rank > 6");
  TORCH_CHECK(out_stride.empty() || static_cast<int>(out_stride.size()) == rank,
              "b200::pointwise: out_stride rank mismatch");
  const at::Tensor& first = inputs[0];
  TORCH_CHECK(first.is_cuda(), "b200::pointwise: inputs must be CUDA tensors");
  c10::cuda::CUDAGuard guard(first.device());
  at::Tensor out = out_stride.empty() ? at::empty(out_shape, first.options().dtype(out_dtype))
                                      : at::empty_strided(out_shape, out_stride, first.options().dtype(out_dtype));
  // Iteration order: dims sorted by output stride, largest first (identity when contiguous).
  std::vector<int> perm(rank);
  for (int d = 0; d < rank; ++d) perm[d] = d;
  if (!out_stride.empty()) {
    std::stable_sort(perm.begin(), perm.end(), [&](int x, int y) {
      return out.stride(x) > out.stride(y) || (out.stride(x) == out.stride(y) && out.size(x) > out.size(y));
    });
    int64_t expect = 1;
    for (int k = rank - 1; k >= 0; --k) {
      const int d = perm[k];
      TORCH_CHECK(out.size(d) == 1 || out.stride(d) == expect, "b200::pointwise: out_stride is not dense");
      expect *= out.size(d);
    }
  }
  B200kPointwiseArgs a;
  std::memset(&a, 0, sizeof(a));
  a.rank = rank;
  a.n_inputs = static_cast<int32_t>(inputs.size());
  for (int k = 0; k < rank; ++k) a.sizes[k] = out_shape[perm[k]];
  for (size_t i = 0; i < inputs.size(); ++i) {
    const at::Tensor& t = inputs[i];
    TORCH_CHECK(t.is_cuda() && t.device() == first.device(), "b200::pointwise: inputs on different devices");
    const at::Tensor e = t.expand(out_shape);
    a.inputs[i].ptr = e.data_ptr();
    a.inputs[i].dtype = to_dt(e.scalar_type());
    for (int k = 0; k < rank; ++k) a.inputs[i].strides[k] = e.stride(perm[k]);
  }
  a.out = out.data_ptr();
  a.out_dtype = to_dt(out_dtype);
  a.program = make_program(code, imm);
  check(b200k_pointwise(&a, stream_of(first)), "pointwise");
  return out;
}

// (m, n) strides of an epilogue operand broadcast to out_shape, whose leading
// dims flatten into m.
void mn_strides(const at::Tensor& t, at::IntArrayRef out_shape, int64_t& sm, int64_t& sn) {
  const at::Tensor e = t.expand(out_shape);
  const int r = static_cast<int>(out_shape.size());
  TORCH_CHECK(r >= 1, "b200::gemm_epilogue: output rank 0");
  sn = e.stride(r - 1);
  if (r == 1) {
    sm = 0;
    return;
  }
  sm = e.stride(r - 2);
  // Leading dims must merge into one index m with stride sm.
  int64_t expect = sm * out_shape[r - 2];
  for (int d = r - 3; d >= 0; --d) {
    if (out_shape[d] != 1) {
      TORCH_CHECK(e.stride(d) == expect, "b200::gemm_epilogue: epilogue operand leading dims do not flatten");
    }
    expect *= out_shape[d];
  }
}

at::Tensor gemm_epilogue(const at::Tensor& a, const at::Tensor& b, at::TensorList extras, at::IntArrayRef code,
                         at::ArrayRef<double> imm, at::IntArrayRef out_shape, at::ScalarType out_dtype,
                         at::IntArrayRef form) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda(), "b200::gemm_epilogue: a and b must be CUDA tensors");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2, "b200::gemm_epilogue: a [M,K] and b [K,N] must be 2-d");
  TORCH_CHECK(a.size(1) == b.size(0), "b200::gemm_epilogue: incompatible shapes ", a.sizes(), " and ", b.sizes());
  TORCH_CHECK(a.scalar_type() == b.scalar_type(), "b200::gemm_epilogue: a and b dtypes differ");
  TORCH_CHECK(static_cast<int64_t>(extras.size()) <= B200K_MAX_INPUTS - 1, "b200::gemm_epilogue: too many extras");
  const int64_t M = a.size(0), K = a.size(1), N = b.size(1);
  int64_t numel = 1;
  for (auto s : out_shape) numel *= s;
  TORCH_CHECK(numel == M * N && !out_shape.empty() && out_shape.back() == N,
              "b200::gemm_epilogue: out_shape ", out_shape, " does not hold [", M, ", ", N, "]");
  c10::cuda::CUDAGuard guard(a.device());
  at::Tensor out = at::empty(out_shape, a.options().dtype(out_dtype));
  B200kGemmArgs g;
  std::memset(&g, 0, sizeof(g));
  g.M = M;
  g.N = N;
  g.K = K;
  g.a = a.data_ptr();
  g.a_stride_m = a.stride(0);
  g.a_stride_k = a.stride(1);
  g.b = b.data_ptr();
  g.b_stride_k = b.stride(0);
  g.b_stride_n = b.stride(1);
  g.ab_dtype = to_dt(a.scalar_type());
  g.out_dtype = to_dt(out_dtype);
  g.out = out.data_ptr();
  g.out_stride_m = N;
  g.out_stride_n = 1;
  g.n_extras = static_cast<int32_t>(extras.size());
  g.tile_config = -1;
  for (size_t i = 0; i < extras.size(); ++i) {
    const at::Tensor& t = extras[i];
    TORCH_CHECK(t.is_cuda() && t.device() == a.device(), "b200::gemm_epilogue: extras must be on a's device");
    int64_t sm, sn;
    mn_strides(t, out_shape, sm, sn);
    g.extras[i].ptr = t.data_ptr();
    g.extras[i].dtype = to_dt(t.scalar_type());
    g.extras[i].stride_m = sm;
    g.extras[i].stride_n = sn;
  }
  g.program = make_program(code, imm);
  TORCH_CHECK(form.empty() || form.size() == 6, "b200::gemm_epilogue: form needs 6 ints");
  if (form.size() == 6) {
    g.form.kind = static_cast<int32_t>(form[0]);
    g.form.bias = static_cast<int32_t>(form[1]);
    g.form.act = static_cast<int32_t>(form[2]);
    g.form.round = static_cast<int32_t>(form[3]);
    g.form.scale = static_cast<int32_t>(form[4]);
    g.form.residual = static_cast<int32_t>(form[5]);
  }
  g.status = status_word(a.device().index()).data_ptr<int32_t>();
  const int64_t stall = g_test_stall_ns.exchange(0);
  if (stall > 0) {  // failure-detection test hook, armed by gemm_test_stall_next
    g.test_flags = B200K_GEMM_TEST_WITHHOLD_READY;
    g.timeout_ns = stall;
  }
  check(b200k_gemm_epilogue(&g, stream_of(a)), "gemm_epilogue");
  return out;
}

// out [M, N] = rope(round(a @ b)) per 64-column head with the rotary tables
// cos / sin [period, 64] (b200k_gemm_rope); out_shape as for gemm_epilogue.
at::Tensor gemm_rope(const at::Tensor& a, const at::Tensor& b, const at::Tensor& cos, const at::Tensor& sin,
                     int64_t period, at::IntArrayRef out_shape) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && cos.is_cuda() && sin.is_cuda(), "b200::gemm_rope: CUDA tensors only");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(0), "b200::gemm_rope: a [M,K], b [K,N]");
  TORCH_CHECK(cos.dim() == 2 && sin.dim() == 2 && cos.size(0) == period && sin.size(0) == period &&
                  cos.size(1) == 64 && sin.size(1) == 64 && cos.stride(1) == 1 && sin.stride(1) == 1 &&
                  cos.stride(0) == sin.stride(0),
              "b200::gemm_rope: cos / sin must be [period, 64] tables with unit column stride");
  TORCH_CHECK(a.scalar_type() == b.scalar_type() && cos.scalar_type() == a.scalar_type() &&
                  sin.scalar_type() == a.scalar_type(),
              "b200::gemm_rope: a, b, cos, sin must share one 16-bit dtype");
  const int64_t M = a.size(0), K = a.size(1), N = b.size(1);
  int64_t numel = 1;
  for (auto s : out_shape) numel *= s;
  TORCH_CHECK(numel == M * N && !out_shape.empty(), "b200::gemm_rope: out_shape ", out_shape, " does not hold [", M,
              ", ", N, "]");
  c10::cuda::CUDAGuard guard(a.device());
  at::Tensor out = at::empty(out_shape, a.options());
  B200kGemmArgs g;
  std::memset(&g, 0, sizeof(g));
  g.M = M;
  g.N = N;
  g.K = K;
  g.a = a.data_ptr();
  g.a_stride_m = a.stride(0);
  g.a_stride_k = a.stride(1);
  g.b = b.data_ptr();
  g.b_stride_k = b.stride(0);
  g.b_stride_n = b.stride(1);
  g.ab_dtype = to_dt(a.scalar_type());
  g.out_dtype = g.ab_dtype;
  g.out = out.data_ptr();
  g.out_stride_m = N;
  g.out_stride_n = 1;
  g.tile_config = -1;
  g.status = status_word(a.device().index()).data_ptr<int32_t>();
  B200kRopeTables r;
  std::memset(&r, 0, sizeof(r));
  r.cos = cos.data_ptr();
  r.sin = sin.data_ptr();
  r.stride = cos.stride(0);
  r.period = period;
  r.head_dim = 64;
  r.dtype = g.ab_dtype;
  check(b200k_gemm_rope(&g, &r, stream_of(a)), "gemm_rope");
  return out;
}

int64_t gemm_status(int64_t device, bool reset) {
  at::Tensor& w = status_word(static_cast<int>(device));
  const int64_t v = w.item<int32_t>();
  if (reset) w.zero_();
  return v;
}

// Asynchronous watch of the status word for the compiled graphs.  After a
// graph has queued its GEMMs, `status_check(dev, arm=true)` queues a copy of
// the word into pinned host memory and an event behind them on the current
// stream; every check first looks at the last copy whose event has
// completed and raises when a wait timed out (then the word and the copy are
// cleared, so each timeout is reported once).  Nothing here synchronises;
// inside a stream capture the copy is not queued.
struct StatusWatch {
  int32_t* host = nullptr;
  cudaEvent_t ev = nullptr;
  bool armed = false;
};

int64_t status_check(int64_t device, bool arm) {
  static std::mutex mu;
  static std::vector<StatusWatch> watches;
  const int dev = static_cast<int>(device);
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(dev));
  at::Tensor& word = status_word(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev).stream();
  int32_t seen = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (static_cast<int>(watches.size()) <= dev) watches.resize(dev + 1);
    StatusWatch& w = watches[dev];
    if (w.host == nullptr) {
      TORCH_CHECK(cudaHostAlloc(reinterpret_cast<void**>(&w.host), sizeof(int32_t), cudaHostAllocDefault) ==
                      cudaSuccess, "b200::status_check: pinned allocation failed");
      *w.host = 0;
      TORCH_CHECK(cudaEventCreateWithFlags(&w.ev, cudaEventDisableTiming) == cudaSuccess,
                  "b200::status_check: event creation failed");
    }
    if (w.armed && cudaEventQuery(w.ev) == cudaSuccess) {
      seen = *reinterpret_cast<volatile int32_t*>(w.host);
      if (seen != 0) {
        *w.host = 0;
        w.armed = false;
      }
    }
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    const bool capturing = cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone;
    if (seen == 0 && arm && !capturing) {
      TORCH_CHECK(cudaMemcpyAsync(w.host, word.data_ptr<int32_t>(), sizeof(int32_t), cudaMemcpyDeviceToHost, st) ==
                      cudaSuccess, "b200::status_check: copy failed");
      TORCH_CHECK(cudaEventRecord(w.ev, st) == cudaSuccess, "b200::status_check: event record failed");
      w.armed = true;
    }
  }
  if (seen != 0) {
    word.zero_();
    TORCH_CHECK(false, "b200::gemm_epilogue on cuda:", dev, " reported ", b200k_status_string(static_cast<int>(seen)),
                " (code ", seen, "): an earlier GEMM's output is incomplete");
  }
  return 0;
}

// Test hook: the next gemm_epilogue launch through this binding withholds
// its first tile's accumulator-ready signal (B200K_GEMM_TEST_WITHHOLD_READY),
// so the epilogue's wait runs out after `timeout_ns`.  Failure-detection
// tests only.
void gemm_test_stall_next(int64_t timeout_ns) {
  TORCH_CHECK(timeout_ns > 0, "b200::gemm_test_stall_next: timeout_ns must be positive");
  g_test_stall_ns.store(timeout_ns);
}

void rows_of(const at::Tensor& x, int64_t& rows, int64_t& cols, int64_t& row_stride) {
  TORCH_CHECK(x.dim() >= 1, "b200: row op on a 0-d tensor");
  cols = x.size(-1);
  rows = cols == 0 ? 0 : x.numel() / cols;
  TORCH_CHECK(x.stride(-1) == 1 || cols == 1, "b200: row op needs a unit last-dim stride");
  row_stride = x.dim() >= 2 ? x.stride(-2) : cols;
  int64_t expect = row_stride * (x.dim() >= 2 ? x.size(-2) : 1);
  for (int d = static_cast<int>(x.dim()) - 3; d >= 0; --d) {
    if (x.size(d) != 1) TORCH_CHECK(x.stride(d) == expect, "b200: row op needs leading dims that flatten");
    expect *= x.size(d);
  }
  if (x.dim() < 2) row_stride = cols;
}

at::Tensor rms_norm_impl(const at::Tensor& x_in, const c10::optional<at::Tensor>& weight, double eps, int64_t flags,
                         at::ScalarType out_dtype, bool swiglu) {
  TORCH_CHECK(x_in.is_cuda(), "b200::rms_norm: x must be a CUDA tensor");
  c10::cuda::CUDAGuard guard(x_in.device());
  const at::Tensor x = x_in.stride(-1) == 1 ? x_in : x_in.contiguous();
  int64_t rows, cols, rs;
  rows_of(x, rows, cols, rs);
  std::vector<int64_t> oshape(x.sizes().begin(), x.sizes().end());
  if (swiglu) {
    TORCH_CHECK(cols % 2 == 0, "b200::rms_norm_swiglu: odd last dim");
    oshape.back() = cols / 2;
  }
  at::Tensor out = at::empty(oshape, x.options().dtype(out_dtype));
  B200kRowNormArgs a;
  std::memset(&a, 0, sizeof(a));
  a.rows = rows;
  a.cols = cols;
  a.x = x.data_ptr();
  a.x_row_stride = rs;
  a.x_dtype = to_dt(x.scalar_type());
  a.kind = swiglu ? B200K_ROW_RMSNORM_SWIGLU : B200K_ROW_RMSNORM;
  at::Tensor w;
  if (weight.has_value() && weight->defined()) {
    w = weight->contiguous();
    TORCH_CHECK(w.numel() == cols, "b200::rms_norm: weight has ", w.numel(), " elements, expected ", cols);
    a.weight = w.data_ptr();
    a.w_dtype = to_dt(w.scalar_type());
  }
  a.flags = static_cast<int32_t>(flags);
  a.eps = static_cast<float>(eps);
  a.out = out.data_ptr();
  a.out_row_stride = oshape.back();
  a.out_dtype = to_dt(out_dtype);
  check(b200k_rownorm(&a, stream_of(x)), swiglu ? "rms_norm_swiglu" : "rms_norm");
  return out;
}

at::Tensor rms_norm(const at::Tensor& x, const c10::optional<at::Tensor>& weight, double eps, int64_t flags,
                    at::ScalarType out_dtype) {
  return rms_norm_impl(x, weight, eps, flags, out_dtype, false);
}
at::Tensor rms_norm_swiglu(const at::Tensor& x, const c10::optional<at::Tensor>& weight, double eps, int64_t flags,
                           at::ScalarType out_dtype) {
  return rms_norm_impl(x, weight, eps, flags, out_dtype, true);
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> layer_norm(const at::Tensor& x_in, at::IntArrayRef normalized_shape,
                                                          const c10::optional<at::Tensor>& weight,
                                                          const c10::optional<at::Tensor>& bias, double eps) {
  TORCH_CHECK(x_in.is_cuda(), "b200::layer_norm: x must be a CUDA tensor");
  TORCH_CHECK(normalized_shape.size() == 1, "b200::layer_norm: only last-dim normalisation is supported");
  c10::cuda::CUDAGuard guard(x_in.device());
  const at::Tensor x = x_in.contiguous();
  int64_t rows, cols, rs;
  rows_of(x, rows, cols, rs);
  TORCH_CHECK(cols == normalized_shape[0], "b200::layer_norm: normalized_shape mismatch");
  at::Tensor out = at::empty(x.sizes(), x.options());
  std::vector<int64_t> stat_shape(x.sizes().begin(), x.sizes().end());
  stat_shape.back() = 1;
  // native_layer_norm on CUDA keeps mean/rstd in fp32 for reduced-precision input.
  const auto stat_dt = (x.scalar_type() == at::kDouble) ? at::kDouble : at::kFloat;
  TORCH_CHECK(stat_dt == at::kFloat, "b200::layer_norm: fp64 input unsupported");
  at::Tensor mean = at::empty(stat_shape, x.options().dtype(stat_dt));
  at::Tensor rstd = at::empty(stat_shape, x.options().dtype(stat_dt));
  B200kRowNormArgs a;
  std::memset(&a, 0, sizeof(a));
  a.rows = rows;
  a.cols = cols;
  a.x = x.data_ptr();
  a.x_row_stride = rs;
  a.x_dtype = to_dt(x.scalar_type());
  a.kind = B200K_ROW_LAYERNORM;
  at::Tensor w, b;
  if (weight.has_value() && weight->defined()) {
    w = weight->contiguous();
    a.weight = w.data_ptr();
    a.w_dtype = to_dt(w.scalar_type());
  }
  if (bias.has_value() && bias->defined()) {
    b = bias->contiguous();
    a.bias = b.data_ptr();
    a.b_dtype = to_dt(b.scalar_type());
  }
  a.eps = static_cast<float>(eps);
  a.out = out.data_ptr();
  a.out_row_stride = cols;
  a.out_dtype = a.x_dtype;
  a.mean_out = mean.data_ptr<float>();
  a.rstd_out = rstd.data_ptr<float>();
  check(b200k_rownorm(&a, stream_of(x)), "layer_norm");
  return {out, mean, rstd};
}

at::Tensor softmax_impl(const at::Tensor& x_in, int64_t dim, bool half_to_float, bool log) {
  TORCH_CHECK(x_in.is_cuda(), "b200::softmax: x must be a CUDA tensor");
  const int64_t nd = x_in.dim();
  TORCH_CHECK(nd >= 1 && (dim == -1 || dim == nd - 1), "b200::softmax: only the last dim is supported");
  c10::cuda::CUDAGuard guard(x_in.device());
  const at::Tensor x = x_in.stride(-1) == 1 ? x_in : x_in.contiguous();
  int64_t rows, cols, rs;
  rows_of(x, rows, cols, rs);
  const at::ScalarType odt = half_to_float ? at::kFloat : x.scalar_type();
  at::Tensor out = at::empty(x.sizes(), x.options().dtype(odt));
  B200kSoftmaxArgs a;
  std::memset(&a, 0, sizeof(a));
  a.rows = rows;
  a.cols = cols;
  a.x = x.data_ptr();
  a.x_row_stride = rs;
  a.x_dtype = to_dt(x.scalar_type());
  a.log_softmax = log ? 1 : 0;
  a.out = out.data_ptr();
  a.out_row_stride = cols;
  a.out_dtype = to_dt(odt);
  check(b200k_softmax(&a, stream_of(x)), log ? "log_softmax" : "softmax");
  return out;
}

at::Tensor softmax(const at::Tensor& x, int64_t dim, bool half_to_float) {
  return softmax_impl(x, dim, half_to_float, false);
}
at::Tensor log_softmax(const at::Tensor& x, int64_t dim, bool half_to_float) {
  return softmax_impl(x, dim, half_to_float, true);
}

// out = x * cos + rotate_half(x) * sin with cos / sin broadcast to x's shape;
// out has x's shape, `out_stride` (the decomposed graph's layout) or dense.
at::Tensor rope(const at::Tensor& x, const at::Tensor& cos, const at::Tensor& sin, at::IntArrayRef out_stride) {
  TORCH_CHECK(x.is_cuda() && cos.is_cuda() && sin.is_cuda(), "b200::rope: CUDA tensors expected");
  TORCH_CHECK(x.dim() >= 1 && x.dim() <= 4, "b200::rope: rank 1..4");
  TORCH_CHECK(cos.scalar_type() == x.scalar_type() && sin.scalar_type() == x.scalar_type(),
              "b200::rope: x, cos and sin of one dtype");
  c10::cuda::CUDAGuard guard(x.device());
  const at::Tensor c = cos.expand(x.sizes());
  const at::Tensor s = sin.expand(x.sizes());
  at::Tensor out = out_stride.empty() ? at::empty(x.sizes(), x.options())
                                      : at::empty_strided(x.sizes(), out_stride, x.options());
  B200kRopeArgs a;
  std::memset(&a, 0, sizeof(a));
  const int pad = 4 - static_cast<int>(x.dim());
  for (int d = 0; d < 4; ++d) {
    const bool real = d >= pad;
    a.sizes[d] = real ? x.size(d - pad) : 1;
    a.x_strides[d] = real ? x.stride(d - pad) : 0;
    a.cos_strides[d] = real ? c.stride(d - pad) : 0;
    a.sin_strides[d] = real ? s.stride(d - pad) : 0;
    a.out_strides[d] = real ? out.stride(d - pad) : 0;
  }
  a.x = x.data_ptr();
  a.cos = c.data_ptr();
  a.sin = s.data_ptr();
  a.out = out.data_ptr();
  a.dtype = to_dt(x.scalar_type());
  check(b200k_rope(&a, stream_of(x)), "rope");
  return out;
}

// Fused attention over [B, H, S, D] views; the output gets `out_stride`
// (the replaced SDPA node's layout) or is contiguous.
at::Tensor attention(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, bool causal, double scale,
                     at::IntArrayRef out_stride) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(), "b200::attention: q, k, v must be CUDA tensors");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "b200::attention: q, k, v must be [B, H, S, D]");
  TORCH_CHECK(q.scalar_type() == k.scalar_type() && q.scalar_type() == v.scalar_type(),
              "b200::attention: q, k, v dtypes differ");
  TORCH_CHECK(k.sizes() == v.sizes(), "b200::attention: k and v shapes differ");
  TORCH_CHECK(q.size(0) == k.size(0) && q.size(3) == k.size(3), "b200::attention: q ", q.sizes(), " and k ",
              k.sizes(), " do not match");
  TORCH_CHECK(out_stride.empty() || out_stride.size() == 4, "b200::attention: out_stride needs 4 entries");
  c10::cuda::CUDAGuard guard(q.device());
  at::Tensor out = out_stride.empty() ? at::empty(q.sizes(), q.options())
                                      : at::empty_strided(q.sizes(), out_stride, q.options());
  B200kAttentionArgs a;
  std::memset(&a, 0, sizeof(a));
  a.batch = q.size(0);
  a.heads = q.size(1);
  a.kv_heads = k.size(1);
  a.q_len = q.size(2);
  a.kv_len = k.size(2);
  a.head_dim = q.size(3);
  const at::Tensor* ts[4] = {&q, &k, &v, &out};
  int64_t* st[4] = {a.q_strides, a.k_strides, a.v_strides, a.out_strides};
  for (int i = 0; i < 4; ++i)
    for (int d = 0; d < 4; ++d) st[i][d] = ts[i]->stride(d);
  a.q = q.data_ptr();
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.out = out.data_ptr();
  a.dtype = to_dt(q.scalar_type());
  a.causal = causal ? 1 : 0;
  a.scale = static_cast<float>(scale);
  a.status = status_word(q.device().index()).data_ptr<int32_t>();
  check(b200k_attention(&a, stream_of(q)), "attention");
  return out;
}

}  // namespace

TORCH_LIBRARY(b200, m) {
  m.def(
      "pointwise(Tensor[] inputs, int[] code, float[] imm, int[] out_shape, ScalarType out_dtype, "
      "int[] out_stride=[]) -> Tensor");
  m.def(
      "gemm_epilogue(Tensor a, Tensor b, Tensor[] extras, int[] code, float[] imm, int[] out_shape, "
      "ScalarType out_dtype, int[] form=[]) -> Tensor");
  m.def("rms_norm(Tensor x, Tensor? weight, float eps, int flags, ScalarType out_dtype) -> Tensor");
  m.def("rms_norm_swiglu(Tensor x, Tensor? weight, float eps, int flags, ScalarType out_dtype) -> Tensor");
  m.def(
      "layer_norm(Tensor x, int[] normalized_shape, Tensor? weight, Tensor? bias, float eps) -> "
      "(Tensor, Tensor, Tensor)");
  m.def("softmax(Tensor x, int dim, bool half_to_float) -> Tensor");
  m.def("log_softmax(Tensor x, int dim, bool half_to_float) -> Tensor");
  m.def("rope(Tensor x, Tensor cos, Tensor sin, int[] out_stride=[]) -> Tensor");
  m.def("gemm_rope(Tensor a, Tensor b, Tensor cos, Tensor sin, int period, int[] out_shape) -> Tensor");
  m.def("attention(Tensor q, Tensor k, Tensor v, bool causal, float scale, int[] out_stride=[]) -> Tensor");
  m.def("gemm_status(int device, bool reset) -> int", &gemm_status);
  m.def("status_check(int device, bool arm) -> int", &status_check);
  m.def("gemm_test_stall_next(int timeout_ns) -> ()", &gemm_test_stall_next);
}

TORCH_LIBRARY_IMPL(b200, CUDA, m) {
  m.impl("pointwise", &pointwise);
  m.impl("gemm_epilogue", &gemm_epilogue);
  m.impl("rms_norm", &rms_norm);
  m.impl("rms_norm_swiglu", &rms_norm_swiglu);
  m.impl("layer_norm", &layer_norm);
  m.impl("softmax", &softmax);
  m.impl("log_softmax", &log_softmax);
  m.impl("rope", &rope);
  m.impl("gemm_rope", &gemm_rope);
  m.impl("attention", &attention);
}

