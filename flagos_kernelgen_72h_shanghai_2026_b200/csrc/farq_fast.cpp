// farq_fast.cpp — C++ launch path of the two Python operators.
//
// The Python wrappers (task01.py, task02.py) check tensors and fill the C
// argument structs in Python, which costs about 10 us per call — more than
// the kernel itself for a few rows (the reference's small-M regime,
// reports/task01_fused_add_rmsnorm_group_quant.md:57). This extension does the
// same checks and the struct fill in C++ for the common case (contiguous
// tensors on one CUDA device) and calls the same plain-C entry points
// (farq_launch, dsa_topk_launch) on the current stream. Anything else — an
// unusual layout, a bad argument — returns -1 without launching, and the
// Python path handles the call (and raises its precise error).
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "dsa_topk.h"
#include "farq.h"

namespace {

constexpr int kNotHandled = -1;

int float_code(at::ScalarType t) {
  switch (t) {
    case at::kBFloat16: return FARQ_DTYPE_BF16;
    case at::kHalf: return FARQ_DTYPE_FP16;
    case at::kFloat: return FARQ_DTYPE_FP32;
    default: return -1;
  }
}

bool same_cuda(const at::Tensor& t, const at::Device& dev) {
  return t.defined() && t.device() == dev && t.is_contiguous();
}

bool is_2d(const at::Tensor& t, int64_t rows, int64_t cols) {
  return t.dim() == 2 && t.size(0) == rows && t.size(1) == cols;
}

// fused_add_rmsnorm_group_quant (task01.py); returns farq_launch's status or
// kNotHandled.
int64_t task01(const at::Tensor& x, const at::Tensor& residual, const at::Tensor& gamma,
               const at::Tensor& residual_out, const c10::optional<at::Tensor>& norm_out,
               const at::Tensor& x_q, const at::Tensor& x_scale, double eps, int64_t group_size,
               bool ue8m0) {
  if (!x.defined() || !x.is_cuda() || x.dim() != 2) return kNotHandled;
  const at::Device dev = x.device();
  const int64_t M = x.size(0), D = x.size(1);
  if (!same_cuda(x, dev) || !same_cuda(residual, dev) || !same_cuda(gamma, dev) ||
      !same_cuda(residual_out, dev) || !same_cuda(x_q, dev) || !same_cuda(x_scale, dev))
    return kNotHandled;
  const bool write_norm = norm_out.has_value() && norm_out->defined() && norm_out->numel() > 0;
  if (write_norm && (!same_cuda(*norm_out, dev) || !is_2d(*norm_out, M, D))) return kNotHandled;
  const at::ScalarType xt = x.scalar_type();
  if ((xt != at::kBFloat16 && xt != at::kHalf) || residual.scalar_type() != xt) return kNotHandled;
  const int g_dt = float_code(gamma.scalar_type());
  const int ro_dt = float_code(residual_out.scalar_type());
  const int no_dt = write_norm ? float_code(norm_out->scalar_type()) : 0;
  const at::ScalarType qt = x_q.scalar_type();
  if (g_dt < 0 || ro_dt < 0 || no_dt < 0) return kNotHandled;
  if (qt != at::kChar && qt != at::kFloat8_e4m3fn) return kNotHandled;
  if (x_scale.scalar_type() != at::kFloat) return kNotHandled;
  if (group_size <= 0 || D % group_size != 0) return kNotHandled;
  if (gamma.dim() != 1 || gamma.size(0) != D || !is_2d(residual, M, D) ||
      !is_2d(residual_out, M, D) || !is_2d(x_q, M, D) || !is_2d(x_scale, M, D / group_size))
    return kNotHandled;
  if (M == 0) return FARQ_OK;

  farq_args_t a = {};
  a.struct_size = sizeof(farq_args_t);
  a.x_dtype = xt == at::kBFloat16 ? FARQ_DTYPE_BF16 : FARQ_DTYPE_FP16;
  a.gamma_dtype = g_dt;
  a.residual_out_dtype = ro_dt;
  a.norm_out_dtype = no_dt;
  a.q_dtype = qt == at::kChar ? FARQ_DTYPE_INT8 : FARQ_DTYPE_E4M3;
  a.flags = ue8m0 ? FARQ_FLAG_UE8M0 : 0;
  a.group_size = (int32_t)group_size;
  a.M = M;
  a.D = D;
  a.eps = (float)eps;
  a.x = x.data_ptr();
  a.residual = residual.data_ptr();
  a.gamma = gamma.data_ptr();
  a.residual_out = residual_out.data_ptr();
  a.norm_out = write_norm ? norm_out->data_ptr() : nullptr;
  a.x_q = x_q.data_ptr();
  a.x_scale = x_scale.data_ptr<float>();
  const c10::cuda::CUDAGuard guard(dev);
  return farq_launch(&a, c10::cuda::getCurrentCUDAStream(dev.index()).stream());
}

int index_code(at::ScalarType t) {
  return t == at::kInt ? DSA_DTYPE_INT32 : t == at::kLong ? DSA_DTYPE_INT64 : -1;
}

// dsa_topk_page_table_transform (task02.py); returns dsa_topk_launch's
// status or kNotHandled.
int64_t task02(const at::Tensor& scores, const at::Tensor& page_table, const at::Tensor& q_pos,
               const at::Tensor& kv_lens, const at::Tensor& out_blocks,
               const at::Tensor& out_pages, int64_t block_size, int64_t top_k) {
  if (!scores.defined() || !scores.is_cuda() || scores.dim() != 4) return kNotHandled;
  const at::Device dev = scores.device();
  if (!same_cuda(scores, dev) || !same_cuda(page_table, dev) || !same_cuda(q_pos, dev) ||
      !same_cuda(kv_lens, dev) || !same_cuda(out_blocks, dev) || !same_cuda(out_pages, dev))
    return kNotHandled;
  const int64_t B = scores.size(0), H = scores.size(1), Q = scores.size(2), NB = scores.size(3);
  int s_dt;
  switch (scores.scalar_type()) {
    case at::kFloat: s_dt = DSA_DTYPE_FP32; break;
    case at::kBFloat16: s_dt = DSA_DTYPE_BF16; break;
    case at::kHalf: s_dt = DSA_DTYPE_FP16; break;
    default: return kNotHandled;
  }
  const int i_dt = index_code(q_pos.scalar_type());
  const int p_dt = index_code(page_table.scalar_type());
  const int b_dt = index_code(out_blocks.scalar_type());
  if (i_dt < 0 || p_dt < 0 || b_dt < 0 || kv_lens.scalar_type() != q_pos.scalar_type() ||
      out_pages.scalar_type() != page_table.scalar_type())
    return kNotHandled;
  const std::vector<int64_t> out_shape = {B, H, Q, top_k};
  if (!is_2d(page_table, B, NB) || !is_2d(q_pos, B, Q) || kv_lens.dim() != 1 ||
      kv_lens.size(0) != B || out_blocks.sizes() != at::IntArrayRef(out_shape) ||
      out_pages.sizes() != at::IntArrayRef(out_shape))
    return kNotHandled;
  dsa_topk_args_t a = {};
  a.struct_size = sizeof(dsa_topk_args_t);
  a.scores_dtype = s_dt;
  a.index_dtype = i_dt;
  a.page_dtype = p_dt;
  a.blocks_dtype = b_dt;
  a.block_size = (int32_t)block_size;
  a.top_k = (int32_t)top_k;
  if ((int64_t)a.block_size != block_size || (int64_t)a.top_k != top_k) return kNotHandled;
  a.B = B;
  a.H = H;
  a.Q = Q;
  a.NB = NB;
  a.scores = scores.data_ptr();
  a.page_table = page_table.data_ptr();
  a.q_pos = q_pos.data_ptr();
  a.kv_lens = kv_lens.data_ptr();
  a.out_blocks = out_blocks.data_ptr();
  a.out_pages = out_pages.data_ptr();
  const c10::cuda::CUDAGuard guard(dev);
  return dsa_topk_launch(&a, c10::cuda::getCurrentCUDAStream(dev.index()).stream());
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "C++ launch path of fused_add_rmsnorm_group_quant and dsa_topk_page_table_transform";
  m.def("task01", &task01, "checks + farq_launch; status, or -1 when not handled");
  m.def("task02", &task02, "checks + dsa_topk_launch; status, or -1 when not handled");
}
