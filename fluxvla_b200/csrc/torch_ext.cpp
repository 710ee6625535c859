// fluxvla_b200._C: the thin torch C++ extension over the C ABI
// (include/fluxvla_b200.h) for the operator-level entry points that callers
// reach once per op outside a CUDA graph (the reference's atomic_ops /
// Triton call sites): tensors in, the C entry point on the current torch
// CUDA stream, arguments checked on entry (a Python ValueError for a bad
// argument, RuntimeError for an error the library reports), as the
// reference's own pybind extension checks its inputs
// (fluxvla/ops/cuda/matmul_bias/src/matmul_bias_forward.cpp:21-60).
// Nothing here allocates; every output is caller-allocated.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include <sstream>
#include <stdexcept>
#include <string>

#include "../../include/fluxvla_b200.h"

namespace {

using OptT = c10::optional<at::Tensor>;

void* stream_ptr() {
  return reinterpret_cast<void*>(at::cuda::getCurrentCUDAStream().stream());
}

// Argument check: std::invalid_argument, which pybind11 raises as
// ValueError.  (Plain C++ exceptions rather than TORCH_CHECK: a c10::Error
// thrown from this module crashed the process on the error path.)
template <typename... Ts>
void require(bool ok, const Ts&... parts) {
  if (ok) return;
  std::ostringstream os;
  (os << ... << parts);
  throw std::invalid_argument(os.str());
}

void check(int rc, const char* what) {
  if (rc == FVB_OK) return;
  std::string msg = std::string("fluxvla_b200 ") + what + " error " + std::to_string(rc) +
                    ": " + fvb_last_error();
  throw std::runtime_error(msg);
}

template <typename T = void>
T* ptr(const OptT& t) {
  return t.has_value() && t->defined() ? static_cast<T*>(t->data_ptr()) : nullptr;
}

int64_t rowmajor(const at::Tensor& t, at::ScalarType dt, const char* name) {
  require(t.scalar_type() == dt, name, ": expected ", dt, ", got ", t.scalar_type());
  require(t.is_cuda(), name, ": must be a CUDA tensor");
  require(t.dim() == 2 && t.stride(1) == 1, name, ": expected a 2-D row-major view");
  return t.stride(0);
}

void check_vec_f32(const OptT& t, const char* name) {
  if (!t.has_value() || !t->defined()) return;
  require(t->scalar_type() == at::kFloat && t->is_contiguous() && t->is_cuda(), name,
              ": expected a contiguous float32 CUDA tensor");
}

// C[M,N] = A[M,K] @ B[N,K]^T with the fused epilogue of fvb_gemm.
void gemm(const at::Tensor& a, const at::Tensor& b, const at::Tensor& out,
          int64_t epilogue, bool swap, int64_t act, const OptT& bias, const OptT& gate,
          double alpha, int64_t split_k, int64_t block_n, const OptT& row_add,
          int64_t row_add_mod, const OptT& k_out, const OptT& v_out, int64_t n_heads,
          int64_t head_dim, const OptT& rope_cs, const OptT& positions,
          const OptT& workspace, bool pair, const OptT& res, const OptT& gate_tok,
          bool rope_interleaved, int64_t norm_mode, const OptT& norm_out,
          const OptT& norm_w, const OptT& norm_b, double norm_eps,
          const OptT& norm_sync) {
  fvb_gemm_args g;
  memset(&g, 0, sizeof(g));
  g.lda = rowmajor(a, at::kBFloat16, "a");
  g.ldb = rowmajor(b, at::kBFloat16, "b");
  require(a.size(1) == b.size(1), "K mismatch ", a.sizes(), " ", b.sizes());
  const bool f32 = epilogue == FVB_EPI_F32_STORE || epilogue == FVB_EPI_F32_ACC;
  g.ldo = rowmajor(out, f32 ? at::kFloat : at::kBFloat16, "out");
  check_vec_f32(bias, "bias");
  check_vec_f32(gate, "gate");
  g.a = a.data_ptr(); g.b = b.data_ptr();
  g.m = (int32_t)a.size(0); g.n = (int32_t)b.size(0); g.k = (int32_t)a.size(1);
  g.swap = swap; g.epilogue = (int32_t)epilogue; g.act = (int32_t)act;
  g.split_k = (int32_t)split_k; g.block_n = (int32_t)block_n;
  g.out = out.data_ptr();
  g.bias = ptr<const float>(bias); g.gate = ptr<const float>(gate);
  g.alpha = (float)alpha;
  g.row_add = ptr(row_add); g.row_add_mod = (int32_t)row_add_mod;
  g.k_out = ptr(k_out); g.v_out = ptr(v_out);
  g.ld_kv = k_out.has_value() ? k_out->stride(0) : 0;
  g.n_heads = (int32_t)n_heads; g.head_dim = (int32_t)head_dim;
  g.rope_cs = ptr<const float>(rope_cs); g.positions = ptr<const int32_t>(positions);
  g.workspace = ptr(workspace);
  g.workspace_bytes = workspace.has_value() ? workspace->numel() * workspace->element_size() : 0;
  g.pair = pair;
  g.res = ptr(res);
  g.ld_res = res.has_value() ? rowmajor(*res, at::kBFloat16, "res") : 0;
  g.gate_tok = ptr(gate_tok);
  g.ld_gate_tok = gate_tok.has_value() ? rowmajor(*gate_tok, at::kBFloat16, "gate_tok") : 0;
  g.rope_interleaved = rope_interleaved;
  if (norm_out.has_value()) {
    g.norm_mode = (int32_t)norm_mode;
    g.norm_out = norm_out->data_ptr();
    g.ld_norm_out = rowmajor(*norm_out, at::kBFloat16, "norm_out");
    g.norm_w = ptr(norm_w); g.norm_b = ptr(norm_b);
    g.norm_eps = (float)norm_eps;
    g.norm_sync = ptr(norm_sync);
  }
  check(fvb_gemm(&g, stream_ptr()), "fvb_gemm");
}

// Row norms of f32 rows (fvb_norm), output bf16 or f32.
void norm(int64_t mode, const at::Tensor& x, const at::Tensor& out, const OptT& w,
          const OptT& b, const OptT& mod, double eps) {
  const int64_t ld_in = rowmajor(x, at::kFloat, "x");
  const bool out_f32 = out.scalar_type() == at::kFloat;
  const int64_t ld_out = rowmajor(out, out_f32 ? at::kFloat : at::kBFloat16, "out");
  check(fvb_norm((int32_t)mode, x.data_ptr<float>(), ld_in, out.data_ptr(), ld_out,
                 out_f32, (int32_t)x.size(0), (int32_t)x.size(1), ptr(w), ptr(b),
                 ptr<const float>(mod), (float)eps, stream_ptr()),
        "fvb_norm");
}

// Row norms of bf16 rows (fvb_norm_bf16).
void norm_bf16(int64_t mode, const at::Tensor& x, const at::Tensor& out, const OptT& w,
               const OptT& b, const OptT& style, const OptT& gate_out, double eps) {
  const int64_t ld_in = rowmajor(x, at::kBFloat16, "x");
  const int64_t ld_out = rowmajor(out, at::kBFloat16, "out");
  const int64_t ld_gate = gate_out.has_value() ? rowmajor(*gate_out, at::kBFloat16, "gate_out") : 0;
  check(fvb_norm_bf16((int32_t)mode, x.data_ptr(), ld_in, out.data_ptr(), ld_out,
                      (int32_t)x.size(0), (int32_t)x.size(1), ptr(w), ptr(b), ptr(style),
                      ptr(gate_out), ld_gate, (float)eps, stream_ptr()),
        "fvb_norm_bf16");
}

// bf16 softmax over the attended keys of f32 logits rows (fvb_softmax_rows).
void softmax_rows(const at::Tensor& logits, const at::Tensor& out, int64_t n_prefix,
                  const at::Tensor& valid_prefix) {
  require(valid_prefix.scalar_type() == at::kInt && valid_prefix.is_cuda(),
              "valid_prefix: expected an int32 CUDA tensor");
  const int64_t ld_in = rowmajor(logits, at::kFloat, "logits");
  const int64_t ld_out = rowmajor(out, at::kBFloat16, "out");
  check(fvb_softmax_rows(logits.data_ptr<float>(), ld_in, (int32_t)logits.size(0),
                         (int32_t)logits.size(1), (int32_t)n_prefix,
                         valid_prefix.data_ptr<int32_t>(), out.data_ptr(), ld_out,
                         stream_ptr()),
        "fvb_softmax_rows");
}

// y = act(x @ w[:, :k]^T + bias), f32 x, bf16 w (fvb_small_linear).
void small_linear(const at::Tensor& x, const at::Tensor& w, const at::Tensor& out,
                  const OptT& bias, int64_t act, int64_t mode, double alpha, int64_t k) {
  const int64_t ldx = rowmajor(x, at::kFloat, "x");
  const int64_t ldw = rowmajor(w, at::kBFloat16, "w");
  const int64_t ldo = rowmajor(out, mode == 1 ? at::kBFloat16 : at::kFloat, "out");
  check_vec_f32(bias, "bias");
  check(fvb_small_linear(x.data_ptr<float>(), ldx, (int32_t)x.size(0),
                         (int32_t)(k > 0 ? k : x.size(1)), w.data_ptr(), ldw,
                         (int32_t)w.size(0), ptr<const float>(bias), (int32_t)act,
                         (int32_t)mode, (float)alpha, out.data_ptr(), ldo, stream_ptr()),
        "fvb_small_linear");
}

// A C-ABI error surfaced as a Python exception without touching the GPU
// (fvb_get_device_status rejects a NULL pointer): used by the tests.
void error_path_probe() { check(fvb_get_device_status(nullptr, 0), "fvb_get_device_status"); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "fluxvla_b200 torch extension over the C ABI (include/fluxvla_b200.h)";
  m.def("gemm", &gemm);
  m.def("norm", &norm);
  m.def("norm_bf16", &norm_bf16);
  m.def("softmax_rows", &softmax_rows);
  m.def("small_linear", &small_linear);
  m.def("error_path_probe", &error_path_probe);
}
