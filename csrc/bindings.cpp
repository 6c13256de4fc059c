// PyTorch bindings for the minispeed_b200 CUDA library (module
// minispeed_b200._C).  Only this file includes ATen; it validates tensors
// (device, dtype, contiguity) and forwards raw pointers plus the current CUDA
// stream to the kernels, which are declared in kernels_api.h.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "kernels_api.h"

namespace {

int dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return msb::kF32;
    case at::kHalf: return msb::kF16;
    case at::kBFloat16: return msb::kBF16;
    default: TORCH_CHECK(false, "unsupported dtype ", t.scalar_type());
  }
  return -1;
}

void check_cuda_contig(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

cudaStream_t stream_of(const at::Tensor& t) {
  return at::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

int64_t grad_stats(const at::Tensor& x, double mul, const at::Tensor& partials,
                   const at::Tensor& flags, int64_t slot, int64_t max_blocks) {
  check_cuda_contig(x, "x");
  check_cuda_contig(partials, "partials");
  check_cuda_contig(flags, "flags");
  TORCH_CHECK(partials.scalar_type() == at::kFloat && flags.scalar_type() == at::kInt);
  TORCH_CHECK(slot >= 0 && slot + max_blocks <= partials.numel() &&
              slot + max_blocks <= flags.numel(), "stats scratch overflow");
  c10::cuda::CUDAGuard g(x.device());
  return msb::grad_stats(x.data_ptr(), dtype_code(x), x.numel(), (float)mul,
                         partials.data_ptr<float>() + slot,
                         reinterpret_cast<unsigned*>(flags.data_ptr<int>()) + slot,
                         (int)max_blocks, stream_of(x));
}

void stats_finalize(const at::Tensor& partials, const at::Tensor& flags, int64_t n,
                    const at::Tensor& out, double max_norm, bool epilogue) {
  check_cuda_contig(partials, "partials");
  check_cuda_contig(out, "out");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.numel() >= 4);
  TORCH_CHECK(n <= partials.numel());
  c10::cuda::CUDAGuard g(out.device());
  msb::stats_finalize(partials.data_ptr<float>(),
                      reinterpret_cast<const unsigned*>(flags.data_ptr<int>()), (int)n,
                      out.data_ptr<float>(), max_norm, epilogue, stream_of(out));
}

void stats_epilogue(const at::Tensor& out, double max_norm) {
  check_cuda_contig(out, "out");
  c10::cuda::CUDAGuard g(out.device());
  msb::stats_epilogue(out.data_ptr<float>(), max_norm, stream_of(out));
}

void adamw(const at::Tensor& master, const at::Tensor& m, const at::Tensor& v,
           const at::Tensor& grad, const c10::optional<at::Tensor>& param_out,
           const c10::optional<at::Tensor>& stats, double lr, double beta1, double beta2,
           double eps, double wd, double bc1, double bc2, double grad_mul) {
  check_cuda_contig(master, "master");
  check_cuda_contig(m, "exp_avg");
  check_cuda_contig(v, "exp_avg_sq");
  check_cuda_contig(grad, "grad");
  TORCH_CHECK(master.scalar_type() == at::kFloat && m.scalar_type() == at::kFloat &&
              v.scalar_type() == at::kFloat, "master and moments must be fp32");
  const int64_t n = master.numel();
  TORCH_CHECK(m.numel() == n && v.numel() == n && grad.numel() == n, "size mismatch");
  void* pout = nullptr;
  int pdt = 0;
  if (param_out.has_value() && param_out->defined()) {
    check_cuda_contig(*param_out, "param_out");
    TORCH_CHECK(param_out->numel() == n, "param_out size mismatch");
    pout = param_out->data_ptr();
    pdt = dtype_code(*param_out);
  }
  const float* st = nullptr;
  if (stats.has_value() && stats->defined()) {
    check_cuda_contig(*stats, "stats");
    st = stats->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(master.device());
  msb::adamw(master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
             grad.data_ptr(), dtype_code(grad), pout, pdt, n, st, lr, beta1, beta2, eps, wd,
             bc1, bc2, grad_mul, stream_of(master));
}

void cast_scale(const at::Tensor& src, const at::Tensor& dst, double mul) {
  check_cuda_contig(src, "src");
  check_cuda_contig(dst, "dst");
  TORCH_CHECK(src.numel() == dst.numel(), "size mismatch");
  c10::cuda::CUDAGuard g(src.device());
  msb::cast_scale(src.data_ptr(), dtype_code(src), dst.data_ptr(), dtype_code(dst), src.numel(),
                  (float)mul, stream_of(src));
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, mod) {
  mod.doc() = "minispeed_b200 sm_100a kernels";
  mod.def("grad_stats", &grad_stats);
  mod.def("stats_finalize", &stats_finalize);
  mod.def("stats_epilogue", &stats_epilogue);
  mod.def("adamw", &adamw);
  mod.def("cast_scale", &cast_scale);
  mod.def("launch_count", &msb::launch_count);
}
