// PyTorch bindings for the minispeed_b200 CUDA library (module
// minispeed_b200._C).  Only this file includes ATen; it validates tensors
// (device, dtype, contiguity) and forwards raw pointers plus the current CUDA
// stream to the kernels, which are declared in kernels_api.h.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

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

using OptT = c10::optional<at::Tensor>;

const void* optr(const OptT& t) {
  return (t.has_value() && t->defined()) ? t->data_ptr() : nullptr;
}
void* optr_mut(const OptT& t) {
  return (t.has_value() && t->defined()) ? t->data_ptr() : nullptr;
}
float* optr_f(const OptT& t) {
  if (!(t.has_value() && t->defined())) return nullptr;
  TORCH_CHECK(t->scalar_type() == at::kFloat);
  return t->data_ptr<float>();
}

void add_norm_fwd(const at::Tensor& x, const OptT& delta, const at::Tensor& w, const OptT& b,
                  const OptT& s_out, const at::Tensor& y, const OptT& mean,
                  const at::Tensor& rstd, double eps, bool rms) {
  check_cuda_contig(x, "x");
  check_cuda_contig(y, "y");
  const int64_t C = x.size(-1), M = x.numel() / C;
  TORCH_CHECK(C % 8 == 0, "hidden size must be a multiple of 8");
  TORCH_CHECK(w.numel() == C && y.numel() == x.numel() && rstd.numel() >= M);
  c10::cuda::CUDAGuard g(x.device());
  msb::add_norm_fwd(x.data_ptr(), optr(delta), w.data_ptr(), optr(b), optr_mut(s_out),
                    y.data_ptr(), optr_f(mean), rstd.data_ptr<float>(), (int)M, (int)C,
                    (float)eps, rms, dtype_code(x), stream_of(x));
}

int64_t norm_bwd(const at::Tensor& dy, const at::Tensor& s, const at::Tensor& w,
                 const OptT& mean, const at::Tensor& rstd, const OptT& dres,
                 const at::Tensor& dx, const at::Tensor& dw_part, const OptT& db_part, bool rms,
                 int64_t max_blocks) {
  check_cuda_contig(dy, "dy");
  check_cuda_contig(s, "s");
  const int64_t C = s.size(-1), M = s.numel() / C;
  TORCH_CHECK(dw_part.numel() >= max_blocks * C, "dw partial buffer too small");
  c10::cuda::CUDAGuard g(s.device());
  return msb::norm_bwd(dy.data_ptr(), s.data_ptr(), w.data_ptr(), optr_f(mean),
                       rstd.data_ptr<float>(), optr(dres), dx.data_ptr(),
                       dw_part.data_ptr<float>(), optr_f(db_part), (int)M, (int)C, rms,
                       dtype_code(s), (int)max_blocks, stream_of(s));
}

void check_rows(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1 && t.stride(0) >= t.size(1),
              name, " must be a row-major matrix (unit column stride)");
}

int64_t colsum_partial(const at::Tensor& a, const at::Tensor& part, int64_t max_chunks) {
  check_rows(a, "a");
  const int64_t N = a.size(1), M = a.size(0);
  TORCH_CHECK(part.numel() >= max_chunks * N, "partial buffer too small");
  c10::cuda::CUDAGuard g(a.device());
  return msb::colsum_partial(a.data_ptr(), part.data_ptr<float>(), (int)M, (int)N, a.stride(0),
                             dtype_code(a), (int)max_chunks, stream_of(a));
}

void colsum_finish(const at::Tensor& part, int64_t nparts, const at::Tensor& out,
                   bool accumulate) {
  check_cuda_contig(out, "out");
  c10::cuda::CUDAGuard g(out.device());
  msb::colsum_finish(part.data_ptr<float>(), (int)nparts, (int)out.numel(), out.data_ptr(),
                     dtype_code(out), accumulate ? 1 : 0, stream_of(out));
}

// Several column-sum finishes in as few launches as possible (one per
// kMaxColsumJobs); every output has the same dtype and device.
void colsum_finish_many(const std::vector<at::Tensor>& parts, const std::vector<int64_t>& nparts,
                        const std::vector<at::Tensor>& outs, const std::vector<bool>& accumulate) {
  const size_t n = outs.size();
  TORCH_CHECK(parts.size() == n && nparts.size() == n && accumulate.size() == n,
              "colsum_finish_many: list lengths differ");
  if (n == 0) return;
  std::vector<msb::ColsumJob> jobs(n);
  for (size_t i = 0; i < n; ++i) {
    check_cuda_contig(outs[i], "out");
    TORCH_CHECK(outs[i].scalar_type() == outs[0].scalar_type() &&
                    outs[i].device() == outs[0].device(),
                "colsum_finish_many: outputs differ in dtype or device");
    TORCH_CHECK(parts[i].scalar_type() == at::kFloat && parts[i].is_contiguous() &&
                    parts[i].device() == outs[0].device(),
                "colsum_finish_many: partials must be contiguous fp32 on the outputs' device");
    TORCH_CHECK(parts[i].numel() >= nparts[i] * outs[i].numel(), "partial buffer too small");
    jobs[i] = {parts[i].data_ptr<float>(), outs[i].data_ptr(), (int)nparts[i],
               (int)outs[i].numel(), accumulate[i] ? 1 : 0};
  }
  c10::cuda::CUDAGuard g(outs[0].device());
  msb::colsum_finish_many(jobs.data(), (int)n, dtype_code(outs[0]), stream_of(outs[0]));
}

void accum_cast(const at::Tensor& src, const at::Tensor& dst, bool accumulate) {
  check_cuda_contig(src, "src");
  check_cuda_contig(dst, "dst");
  TORCH_CHECK(src.scalar_type() == at::kFloat && src.numel() == dst.numel());
  c10::cuda::CUDAGuard g(dst.device());
  msb::accum_cast(src.data_ptr<float>(), dst.data_ptr(), dst.numel(), dtype_code(dst),
                  accumulate ? 1 : 0, stream_of(dst));
}

void bias_gelu_fwd(const at::Tensor& u, const OptT& bias, const at::Tensor& h) {
  check_cuda_contig(u, "u");
  check_cuda_contig(h, "h");
  TORCH_CHECK(u.size(-1) % 8 == 0);
  c10::cuda::CUDAGuard g(u.device());
  msb::bias_gelu_fwd(u.data_ptr(), optr(bias), h.data_ptr(), u.numel(), (int)u.size(-1),
                     dtype_code(u), stream_of(u));
}

void gelu_bwd(const at::Tensor& dh, const at::Tensor& u, const at::Tensor& du) {
  check_cuda_contig(dh, "dh");
  check_cuda_contig(u, "u");
  TORCH_CHECK(u.numel() % 8 == 0);
  c10::cuda::CUDAGuard g(u.device());
  msb::gelu_bwd(dh.data_ptr(), u.data_ptr(), du.data_ptr(), u.numel(), dtype_code(u),
                stream_of(u));
}

void swiglu_fwd(const at::Tensor& gu, const at::Tensor& h) {
  check_cuda_contig(gu, "gu");
  const int64_t F = h.size(-1);
  TORCH_CHECK(gu.size(-1) == 2 * F && F % 8 == 0);
  c10::cuda::CUDAGuard g(gu.device());
  msb::swiglu_fwd(gu.data_ptr(), h.data_ptr(), h.numel() / F, (int)F, dtype_code(gu),
                  stream_of(gu));
}

void swiglu_bwd(const at::Tensor& dh, const at::Tensor& gu, const at::Tensor& dgu) {
  const int64_t F = dh.size(-1);
  c10::cuda::CUDAGuard g(gu.device());
  msb::swiglu_bwd(dh.data_ptr(), gu.data_ptr(), dgu.data_ptr(), dh.numel() / F, (int)F,
                  dtype_code(gu), stream_of(gu));
}

void cross_entropy_fwd(const at::Tensor& logits, const at::Tensor& tgt, const at::Tensor& lse,
                       const at::Tensor& loss_rows, const at::Tensor& loss,
                       const at::Tensor& inv_count, int64_t ignore_index) {
  check_rows(logits, "logits");
  check_cuda_contig(tgt, "targets");
  TORCH_CHECK(tgt.scalar_type() == at::kLong, "targets must be int64");
  const int64_t V = logits.size(1), M = logits.size(0);
  TORCH_CHECK(tgt.numel() == M && lse.numel() >= M && loss_rows.numel() >= M);
  c10::cuda::CUDAGuard g(logits.device());
  msb::cross_entropy_fwd(logits.data_ptr(), reinterpret_cast<const long long*>(tgt.data_ptr<int64_t>()),
                         lse.data_ptr<float>(), loss_rows.data_ptr<float>(), loss.data_ptr<float>(),
                         inv_count.data_ptr<float>(), M, (int)V, logits.stride(0), ignore_index,
                         dtype_code(logits), stream_of(logits));
}

void cross_entropy_fwd_grad(const at::Tensor& logits, const at::Tensor& tgt,
                            const at::Tensor& lse, const at::Tensor& loss_rows,
                            const at::Tensor& loss, const at::Tensor& inv_count,
                            const at::Tensor& g_hint, int64_t ignore_index) {
  check_rows(logits, "logits");
  check_cuda_contig(tgt, "targets");
  TORCH_CHECK(tgt.scalar_type() == at::kLong, "targets must be int64");
  TORCH_CHECK(g_hint.is_cuda() && g_hint.scalar_type() == at::kFloat && g_hint.numel() >= 1,
              "g_hint: fp32 CUDA scalar");
  const int64_t V = logits.size(1), M = logits.size(0);
  TORCH_CHECK(tgt.numel() == M && lse.numel() >= M && loss_rows.numel() >= M);
  c10::cuda::CUDAGuard g(logits.device());
  msb::cross_entropy_fwd_grad(logits.data_ptr(),
                              reinterpret_cast<const long long*>(tgt.data_ptr<int64_t>()),
                              lse.data_ptr<float>(), loss_rows.data_ptr<float>(),
                              loss.data_ptr<float>(), inv_count.data_ptr<float>(),
                              g_hint.data_ptr<float>(), M, (int)V, logits.stride(0),
                              ignore_index, dtype_code(logits), stream_of(logits));
}

void cross_entropy_grad_rescale(const at::Tensor& dlogits, const at::Tensor& grad_out,
                                const at::Tensor& g_hint) {
  check_rows(dlogits, "dlogits");
  TORCH_CHECK(grad_out.scalar_type() == at::kFloat && grad_out.is_cuda());
  TORCH_CHECK(g_hint.scalar_type() == at::kFloat && g_hint.is_cuda());
  c10::cuda::CUDAGuard g(dlogits.device());
  msb::cross_entropy_grad_rescale(dlogits.data_ptr(), dlogits.size(0), (int)dlogits.size(1),
                                  dlogits.stride(0), grad_out.data_ptr<float>(),
                                  g_hint.data_ptr<float>(), dtype_code(dlogits),
                                  stream_of(dlogits));
}

void cross_entropy_bwd(const at::Tensor& logits, const at::Tensor& tgt, const at::Tensor& lse,
                       const at::Tensor& grad_out, const at::Tensor& inv_count,
                       int64_t ignore_index) {
  check_rows(logits, "logits");
  TORCH_CHECK(grad_out.scalar_type() == at::kFloat && grad_out.is_cuda());
  const int64_t V = logits.size(1), M = logits.size(0);
  c10::cuda::CUDAGuard g(logits.device());
  msb::cross_entropy_bwd(logits.data_ptr(), reinterpret_cast<const long long*>(tgt.data_ptr<int64_t>()),
                         lse.data_ptr<float>(), grad_out.data_ptr<float>(),
                         inv_count.data_ptr<float>(), M, (int)V, logits.stride(0), ignore_index,
                         dtype_code(logits), stream_of(logits));
}

void embedding_fwd(const at::Tensor& idx, const at::Tensor& wte, const OptT& wpe,
                   const at::Tensor& out, int64_t T) {
  check_cuda_contig(idx, "idx");
  TORCH_CHECK(idx.scalar_type() == at::kLong);
  const int64_t C = wte.size(-1);
  TORCH_CHECK(C % 8 == 0);
  c10::cuda::CUDAGuard g(wte.device());
  msb::embedding_fwd(reinterpret_cast<const long long*>(idx.data_ptr<int64_t>()), wte.data_ptr(), optr(wpe), out.data_ptr(),
                     idx.numel(), (int)T, (int)C, wte.size(0), dtype_code(wte), stream_of(wte));
}

void embedding_bwd(const at::Tensor& dout, const at::Tensor& idx, const at::Tensor& acc,
                   const at::Tensor& touched, const at::Tensor& dwte, bool acc_wte,
                   const OptT& dwpe, bool acc_wpe, int64_t T) {
  check_cuda_contig(dout, "dout");
  check_cuda_contig(idx, "idx");
  check_cuda_contig(acc, "acc");
  check_cuda_contig(dwte, "dwte");
  TORCH_CHECK(idx.scalar_type() == at::kLong);
  const int64_t C = dout.size(-1);
  const int64_t V = dwte.size(0);
  TORCH_CHECK(C % 8 == 0 && dwte.size(-1) == C && dwte.scalar_type() == dout.scalar_type());
  TORCH_CHECK(acc.scalar_type() == at::kFloat && acc.numel() >= V * C, "acc: fp32 [V, C]");
  TORCH_CHECK(touched.scalar_type() == at::kByte && touched.numel() >= V, "touched: uint8 [V]");
  TORCH_CHECK(idx.numel() % T == 0, "tokens must be a whole number of sequences");
  if (dwpe) {
    check_cuda_contig(*dwpe, "dwpe");
    TORCH_CHECK(dwpe->size(-1) == C && dwpe->size(0) >= T &&
                dwpe->scalar_type() == dout.scalar_type());
  }
  c10::cuda::CUDAGuard g(dout.device());
  msb::embedding_bwd(dout.data_ptr(), reinterpret_cast<const long long*>(idx.data_ptr<int64_t>()),
                     acc.data_ptr<float>(), touched.data_ptr<uint8_t>(), dwte.data_ptr(),
                     acc_wte ? 1 : 0, dwpe ? dwpe->data_ptr() : nullptr, acc_wpe ? 1 : 0,
                     idx.numel(), (int)T, (int)C, V, dtype_code(dout), stream_of(dout));
}

void rope(const at::Tensor& x, const at::Tensor& cos_t, const at::Tensor& sin_t, int64_t BT,
          int64_t T, int64_t H, int64_t D, int64_t row_stride, bool inverse) {
  TORCH_CHECK(x.is_cuda() && cos_t.scalar_type() == at::kFloat);
  c10::cuda::CUDAGuard g(x.device());
  msb::rope(x.data_ptr(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), BT, (int)T, (int)H,
            (int)D, row_stride, inverse, dtype_code(x), stream_of(x));
}

void cuda_ok(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e));
}

// ---- GEMM tile/split selection by measurement.  The first call of each
// (shape, operand majorness, dtype, epilogue kind) times every candidate
// configuration into a scratch output (no accumulate, so the real output is
// untouched) and caches the fastest; later calls use the cache.
struct PlanKey {
  int64_t M, N, K;
  int a_mn, b_mn, dtype, fused;
  bool operator<(const PlanKey& o) const {
    return std::tie(M, N, K, a_mn, b_mn, dtype, fused) <
           std::tie(o.M, o.N, o.K, o.a_mn, o.b_mn, o.dtype, o.fused);
  }
};
std::map<PlanKey, std::pair<int, int>> g_plans;
std::mutex g_plan_mutex;
bool g_autotune = std::getenv("MSB_GEMM_AUTOTUNE") == nullptr ||
                  std::string(std::getenv("MSB_GEMM_AUTOTUNE")) != "0";

// MSB_GEMM_TUNE_LOG=1: print every candidate's time to stderr
bool g_tune_log = std::getenv("MSB_GEMM_TUNE_LOG") != nullptr &&
                  std::string(std::getenv("MSB_GEMM_TUNE_LOG")) == "1";
bool g_stream_k = std::getenv("MSB_GEMM_STREAMK") == nullptr ||
                 std::string(std::getenv("MSB_GEMM_STREAMK")) != "0";

// fp32 partial-tile slots of a stream-K launch: one per resident CTA pair
long long stream_k_ws_floats() { return 74LL * msb::kStreamKSlotFloats; }

// split-K workspace: [splits][M][N] for the reduce kernel, or (pair kernel,
// in-kernel fixup) one 256 x 256 slot per tile of every split but the last
long long split_ws_floats(int64_t M, int64_t N, int splits, int bn) {
  long long need = (long long)splits * M * N;
  if (bn == 512)
    need = std::max<long long>(need, (long long)(splits - 1) * ((M + 255) / 256) *
                                         ((N + 255) / 256) * msb::kStreamKSlotFloats);
  return need;
}

// Per-device zeroed tile counters of the stream-K GEMM (persistent: each
// launch leaves them zero again).
int* stream_k_counters(const at::Device& dev) {
  static std::map<int, at::Tensor> bufs;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  auto it = bufs.find(dev.index());
  if (it == bufs.end())
    it = bufs.emplace(dev.index(), at::zeros({msb::kStreamKCounters},
                                             at::TensorOptions().dtype(at::kInt).device(dev)))
             .first;
  return it->second.data_ptr<int>();
}

void gemm_reset_stream_k(const at::Tensor& like) {
  c10::cuda::CUDAGuard g(like.device());
  cuda_ok(cudaMemsetAsync(stream_k_counters(like.device()), 0,
                          msb::kStreamKCounters * sizeof(int), stream_of(like)),
          "stream-K counter reset");
}

std::pair<int, int> tune_gemm(const at::Tensor& a, const at::Tensor& b, int a_mn, int b_mn,
                              int64_t M, int64_t N, int64_t K, bool fused, const at::Tensor& err,
                              double timeout_s, cudaStream_t st) {
  std::vector<std::pair<int, int>> cands;
  const int kb = (int)((K + 63) / 64);
  const char* force = std::getenv("MSB_GEMM_VARIANT");
  const std::string fv = force ? force : "";
  for (int bn : {512, 256, 128}) {
    if (fv == "1cta" && bn == 512) continue;
    if (fv == "2cta" && bn != 512) continue;
    if (bn == 256 && N <= 128) continue;
    for (int s : {1, 2, 4, 8}) {
      if (fused && s > 1) continue;
      if (s > 1 && kb / s < 4) continue;
      if (s > 1 && (long long)s * M * N > (1LL << 31)) continue;
      cands.push_back({bn, s});
    }
    // stream-K: the pair kernel over an even cut of all K slices
    if (bn == 512 && g_stream_k && (M + 255) / 256 * ((N + 255) / 256) <= msb::kStreamKCounters)
      cands.push_back({bn, -1});
  }
  if (cands.size() <= 1) return cands.empty() ? std::make_pair(0, 0) : cands[0];
  const int64_t ldn = (N + 7) / 8 * 8;  // aligned rows, as the real outputs use
  at::Tensor scratch = at::empty({M, ldn}, a.options());
  long long ws_need = 0;
  for (auto& c : cands)
    ws_need = std::max<long long>(ws_need, c.second > 1 ? split_ws_floats(M, N, c.second, c.first)
                                           : (c.second == -1 ? stream_k_ws_floats() : 0));
  int* ctr = stream_k_counters(a.device());
  at::Tensor ws;
  if (ws_need > 0) ws = at::empty({ws_need}, a.options().dtype(at::kFloat));
  cudaEvent_t e0, e1;
  cuda_ok(cudaEventCreate(&e0), "event");
  cuda_ok(cudaEventCreate(&e1), "event");
  float best = 1e30f;
  std::pair<int, int> pick = cands[0];
  for (auto& c : cands) {
    float t = 1e30f;
    for (int rep = 0; rep < 3; ++rep) {
      cuda_ok(cudaEventRecord(e0, st), "event");
      msb::gemm_tcgen05(a.data_ptr(), a.stride(0), a_mn, b.data_ptr(), b.stride(0), b_mn,
                        scratch.data_ptr(), ldn, nullptr, (int)M, (int)N, (int)K, dtype_code(a), 0,
                        0, nullptr, 0, ws_need > 0 ? ws.data_ptr<float>() : nullptr, ws_need,
                        reinterpret_cast<unsigned*>(err.data_ptr<int>()), timeout_s, st, c.first,
                        c.second, ctr, msb::kStreamKCounters);
      cuda_ok(cudaEventRecord(e1, st), "event");
      cuda_ok(cudaEventSynchronize(e1), "event");
      float ms = 0.f;
      cuda_ok(cudaEventElapsedTime(&ms, e0, e1), "event");
      if (rep > 0) t = std::min(t, ms);
    }
    if (g_tune_log)
      std::fprintf(stderr, "gemm tune M=%lld N=%lld K=%lld a_mn=%d b_mn=%d bn=%d splits=%d: %.4f ms\n",
                   (long long)M, (long long)N, (long long)K, a_mn, b_mn, c.first, c.second, t);
    if (t < best) {
      best = t;
      pick = c;
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  return pick;
}

// ------------------------------------------------------------- attention
// qkv2d: [B*T, (H + 2*Hkv)*D] rows of the fused projection (q, k, v heads);
// out2d: [B*T, H*D]; lse: fp32 [B*H, T].
void attention_fwd_py(const at::Tensor& qkv2d, int64_t q_col, int64_t k_col, int64_t v_col,
                      const at::Tensor& out2d, const at::Tensor& lse, int64_t B, int64_t T,
                      int64_t H, int64_t Hkv, int64_t D, double scale, const at::Tensor& err,
                      double timeout_s) {
  check_rows(qkv2d, "qkv");
  check_rows(out2d, "attention output");
  TORCH_CHECK(qkv2d.scalar_type() == out2d.scalar_type(), "attention dtype mismatch");
  TORCH_CHECK(qkv2d.size(0) == B * T && out2d.size(0) == B * T && out2d.size(1) == H * D);
  TORCH_CHECK(lse.is_cuda() && lse.scalar_type() == at::kFloat && lse.is_contiguous() &&
              lse.numel() == B * H * T, "lse must be fp32 [B*H, T]");
  c10::cuda::CUDAGuard g(qkv2d.device());
  msb::attention_fwd(qkv2d.data_ptr(), qkv2d.stride(0), qkv2d.size(1), (int)q_col, (int)k_col,
                     (int)v_col, out2d.data_ptr(), out2d.stride(0), lse.data_ptr<float>(), (int)B,
                     (int)T, (int)H, (int)Hkv, (int)D, dtype_code(qkv2d), (float)scale,
                     reinterpret_cast<unsigned*>(err.data_ptr<int>()), timeout_s, stream_of(qkv2d));
}

void attention_bwd_py(const at::Tensor& qkv2d, int64_t q_col, int64_t k_col, int64_t v_col,
                      const at::Tensor& out2d, const at::Tensor& dout2d, const at::Tensor& lse,
                      const at::Tensor& delta, const at::Tensor& dq_acc, const at::Tensor& dqkv2d,
                      int64_t B, int64_t T, int64_t H, int64_t Hkv, int64_t D, double scale,
                      const at::Tensor& err, double timeout_s) {
  check_rows(qkv2d, "qkv");
  check_rows(out2d, "attention output");
  check_rows(dout2d, "attention output gradient");
  check_rows(dqkv2d, "qkv gradient");
  TORCH_CHECK(dqkv2d.sizes() == qkv2d.sizes() && dout2d.sizes() == out2d.sizes());
  TORCH_CHECK(delta.scalar_type() == at::kFloat && delta.is_contiguous() &&
              delta.numel() == B * H * T, "delta must be fp32 [B*H, T]");
  TORCH_CHECK(dq_acc.scalar_type() == at::kFloat && dq_acc.is_contiguous() &&
              dq_acc.numel() == B * T * H * D, "dq accumulator must be fp32 [B*T, H*D]");
  c10::cuda::CUDAGuard g(qkv2d.device());
  msb::attention_bwd(qkv2d.data_ptr(), qkv2d.stride(0), qkv2d.size(1), (int)q_col, (int)k_col,
                     (int)v_col, out2d.data_ptr(), out2d.stride(0), dout2d.data_ptr(),
                     dout2d.stride(0), lse.data_ptr<float>(), delta.data_ptr<float>(),
                     dq_acc.data_ptr<float>(), dqkv2d.data_ptr(), dqkv2d.stride(0), (int)B, (int)T,
                     (int)H, (int)Hkv, (int)D, dtype_code(qkv2d), (float)scale,
                     reinterpret_cast<unsigned*>(err.data_ptr<int>()), timeout_s, stream_of(qkv2d));
}

// C[M,N] (+)= A * B^T with A given as [M,K] (a_kmajor) or [K,M], B as [N,K]
// (b_kmajor) or [K,N]; every matrix row-major with unit column stride.
// force_bn > 0 picks the plan (bn 512 = 2-CTA pair, 256/128 = 1-CTA; splits
// 1-8 split-K, -1 stream-K) instead of the tuned one (tests, benchmarks).
void gemm(const at::Tensor& a, const at::Tensor& b, bool a_kmajor, bool b_kmajor,
          const OptT& bias, const at::Tensor& out, bool accumulate, const at::Tensor& err,
          double timeout_s, int64_t mode, const OptT& aux, int64_t force_bn,
          int64_t force_splits, const OptT& colsum_part) {
  check_rows(a, "A");
  check_rows(b, "B");
  check_rows(out, "C");
  TORCH_CHECK(a.scalar_type() == b.scalar_type() && a.scalar_type() == out.scalar_type(),
              "gemm operands and output must share one 16-bit dtype");
  TORCH_CHECK(a.scalar_type() == at::kHalf || a.scalar_type() == at::kBFloat16,
              "tcgen05 gemm takes fp16 or bf16");
  const int64_t M = a_kmajor ? a.size(0) : a.size(1);
  const int64_t K = a_kmajor ? a.size(1) : a.size(0);
  const int64_t N = b_kmajor ? b.size(0) : b.size(1);
  const int64_t Kb = b_kmajor ? b.size(1) : b.size(0);
  TORCH_CHECK(K == Kb, "gemm K mismatch: ", K, " vs ", Kb);
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm output shape mismatch");
  TORCH_CHECK(err.is_cuda() && err.scalar_type() == at::kInt && err.numel() >= 1);
  if (bias.has_value() && bias->defined()) {
    TORCH_CHECK(bias->numel() == N && bias->scalar_type() == a.scalar_type(), "bias mismatch");
  }
  TORCH_CHECK(mode >= 0 && mode <= 2, "gemm epilogue mode must be 0, 1 or 2");
  void* auxp = nullptr;
  int64_t ld_aux = 0;
  if (mode != 0) {
    TORCH_CHECK(aux.has_value() && aux->defined(), "gemm epilogue mode needs aux");
    check_rows(*aux, "aux");
    TORCH_CHECK(aux->size(0) == M && aux->size(1) == N && aux->scalar_type() == a.scalar_type());
    auxp = aux->data_ptr();
    ld_aux = aux->stride(0);
    TORCH_CHECK(!accumulate, "gemm epilogue modes do not accumulate");
  }
  float* csp = nullptr;
  if (colsum_part.has_value() && colsum_part->defined()) {
    TORCH_CHECK(mode == 2, "gemm column sums come with the dGELU epilogue (mode 2)");
    TORCH_CHECK(colsum_part->is_cuda() && colsum_part->scalar_type() == at::kFloat &&
                    colsum_part->is_contiguous() && colsum_part->numel() >= (M + 31) / 32 * N,
                "gemm column-sum partials: fp32 [ceil(M/32), N]");
    csp = colsum_part->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(a.device());
  cudaStream_t st = stream_of(a);
  const int a_mn = a_kmajor ? 0 : 1, b_mn = b_kmajor ? 0 : 1;
  int bn = 0, splits = 0;
  if (force_bn > 0) {
    bn = (int)force_bn;
    splits = (int)force_splits;
  } else if (g_autotune) {
    const PlanKey key{M, N, K, a_mn, b_mn, dtype_code(a), mode != 0 ? 1 : 0};
    std::lock_guard<std::mutex> lock(g_plan_mutex);
    auto it = g_plans.find(key);
    if (it == g_plans.end()) {
      // timing candidates synchronizes: never inside a CUDA-graph capture
      // (a shape first seen there runs the heuristic plan, untuned)
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      cuda_ok(cudaStreamIsCapturing(st, &cs), "cudaStreamIsCapturing");
      if (cs == cudaStreamCaptureStatusNone)
        it = g_plans.emplace(key, tune_gemm(a, b, a_mn, b_mn, M, N, K, mode != 0, err, timeout_s,
                                            st)).first;
    }
    if (it != g_plans.end()) {
      bn = it->second.first;
      splits = it->second.second;
    }
  }
  long long need = 0;
  if (bn > 0) {
    need = splits > 1 ? split_ws_floats(M, N, splits, bn)
                      : (splits == -1 ? stream_k_ws_floats() : 0);
  } else {
    int pbn = 0, ps = 1;
    need = msb::gemm_plan((int)M, (int)N, (int)K, 148, &pbn, &ps);
  }
  if (mode != 0 && splits != -1) need = 0;
  at::Tensor ws;
  if (need > 0) ws = at::empty({need}, a.options().dtype(at::kFloat));
  msb::gemm_tcgen05(a.data_ptr(), a.stride(0), a_mn, b.data_ptr(), b.stride(0), b_mn,
                    out.data_ptr(), out.stride(0), optr(bias), (int)M, (int)N, (int)K,
                    dtype_code(a), accumulate ? 1 : 0, (int)mode, auxp, ld_aux,
                    need > 0 ? ws.data_ptr<float>() : nullptr, need,
                    reinterpret_cast<unsigned*>(err.data_ptr<int>()), timeout_s, st, bn, splits,
                    (splits == -1 || splits > 1) ? stream_k_counters(a.device()) : nullptr,
                    msb::kStreamKCounters, csp);
}

std::vector<int64_t> gemm_cached_plan(int64_t M, int64_t N, int64_t K, int64_t a_mn,
                                      int64_t b_mn, int64_t dtype, int64_t fused) {
  std::lock_guard<std::mutex> lock(g_plan_mutex);
  auto it = g_plans.find(PlanKey{M, N, K, (int)a_mn, (int)b_mn, (int)dtype, (int)fused});
  if (it == g_plans.end()) return {};
  return {it->second.first, it->second.second};
}

std::vector<int64_t> gemm_plan_py(int64_t M, int64_t N, int64_t K) {
  int bn = 0, splits = 1;
  const long long need = msb::gemm_plan((int)M, (int)N, (int)K, 148, &bn, &splits);
  return {bn, splits, need};
}

// ------------------------------------------------- peer heap / collectives
char* const* heap_table(const at::Tensor& heaps) {
  TORCH_CHECK(heaps.is_cuda() && heaps.scalar_type() == at::kLong && heaps.is_contiguous(),
              "heap table must be a CUDA int64 tensor");
  return reinterpret_cast<char* const*>(heaps.data_ptr<int64_t>());
}

int64_t peer_alloc_py(int64_t bytes) { return reinterpret_cast<int64_t>(msb::peer_alloc(bytes)); }
void peer_free_py(int64_t p) { msb::peer_free(reinterpret_cast<void*>(p)); }
py::bytes peer_handle_py(int64_t p) {
  char h[64];
  msb::peer_handle(reinterpret_cast<void*>(p), h);
  return py::bytes(h, 64);
}
int64_t peer_open_py(const std::string& h) {
  TORCH_CHECK(h.size() == 64, "IPC handle must be 64 bytes");
  return reinterpret_cast<int64_t>(msb::peer_open(h.data()));
}
void peer_close_py(int64_t p) { msb::peer_close(reinterpret_cast<void*>(p)); }

// Non-owning tensor over device memory at `ptr` (the heap object owns it).
at::Tensor tensor_from_ptr(int64_t ptr, int64_t numel, int64_t dtype, int64_t device) {
  static const at::ScalarType types[3] = {at::kFloat, at::kHalf, at::kBFloat16};
  TORCH_CHECK(dtype >= 0 && dtype < 3);
  auto opts = at::TensorOptions().dtype(types[dtype]).device(at::kCUDA, (int)device);
  return at::from_blob(reinterpret_cast<void*>(ptr), {numel}, opts);
}

// Device-to-device copies on the current stream of `like`'s device, one
// cudaMemcpyAsync each (peer pointers mapped into this process included:
// the copy engines move those over NVLink without using SMs).
void copy_many(const at::Tensor& like, const std::vector<int64_t>& dst,
               const std::vector<int64_t>& src, const std::vector<int64_t>& nbytes) {
  TORCH_CHECK(dst.size() == src.size() && src.size() == nbytes.size(), "copy lists differ");
  c10::cuda::CUDAGuard g(like.device());
  cudaStream_t st = stream_of(like);
  for (size_t k = 0; k < dst.size(); ++k) {
    if (nbytes[k] <= 0) continue;
    cuda_ok(cudaMemcpyAsync(reinterpret_cast<void*>(dst[k]), reinterpret_cast<const void*>(src[k]),
                            static_cast<size_t>(nbytes[k]), cudaMemcpyDeviceToDevice, st),
            "peer copy");
  }
}

unsigned* epoch_counter(const at::Tensor& ctr) {
  TORCH_CHECK(ctr.is_cuda() && ctr.scalar_type() == at::kInt && ctr.numel() >= 1,
              "epoch counter must be a CUDA int32 tensor");
  return reinterpret_cast<unsigned*>(ctr.data_ptr<int>());
}

void peer_barrier_py(const at::Tensor& heaps, int64_t sync_off, int64_t rank, int64_t world,
                     const at::Tensor& ctr, double timeout_s, const at::Tensor& status) {
  c10::cuda::CUDAGuard g(heaps.device());
  msb::peer_barrier(heap_table(heaps), sync_off, (int)rank, (int)world, epoch_counter(ctr),
                    timeout_s, reinterpret_cast<unsigned*>(status.data_ptr<int>()),
                    stream_of(heaps));
}

int64_t rs_stats_py(const at::Tensor& heaps, int64_t grad_off, int64_t dtype, int64_t s0,
                    const at::Tensor& out, int64_t world, double mul, const OptT& mul_dev,
                    int64_t fanout_off, const at::Tensor& partials, const at::Tensor& flags,
                    int64_t slot, int64_t max_blocks, bool aligned16, int64_t threads) {
  check_cuda_contig(out, "out");
  TORCH_CHECK(out.scalar_type() == at::kFloat);
  TORCH_CHECK(slot >= 0 && slot + max_blocks <= partials.numel(), "stats scratch overflow");
  const float* md = nullptr;
  if (mul_dev.has_value() && mul_dev->defined()) {
    TORCH_CHECK(mul_dev->is_cuda() && mul_dev->scalar_type() == at::kFloat, "mul_dev: fp32 CUDA");
    md = mul_dev->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(heaps.device());
  return msb::rs_stats(heap_table(heaps), grad_off, (int)dtype, s0, out.numel(), (int)world,
                       (float)mul, md, out.data_ptr<float>(), fanout_off,
                       partials.data_ptr<float>() + slot,
                       reinterpret_cast<unsigned*>(flags.data_ptr<int>()) + slot, (int)max_blocks,
                       aligned16, stream_of(heaps), (int)threads);
}

void stats_exchange_py(const at::Tensor& heaps, int64_t sync_off, int64_t rank, int64_t world,
                       const at::Tensor& ctr, const at::Tensor& out, double max_norm,
                       double timeout_s, const at::Tensor& status) {
  c10::cuda::CUDAGuard g(heaps.device());
  msb::stats_exchange(heap_table(heaps), sync_off, (int)rank, (int)world, epoch_counter(ctr),
                      out.data_ptr<float>(), max_norm, timeout_s,
                      reinterpret_cast<unsigned*>(status.data_ptr<int>()), stream_of(heaps));
}

void adamw_fanout_py(const at::Tensor& master, const at::Tensor& m, const at::Tensor& v,
                     const at::Tensor& grad, const at::Tensor& heaps, int64_t param_off,
                     int64_t pdtype, int64_t s0, int64_t world, const at::Tensor& stats,
                     double lr, double beta1, double beta2, double eps, double wd, double bc1,
                     double bc2, double grad_mul) {
  check_cuda_contig(master, "master");
  TORCH_CHECK(grad.scalar_type() == at::kFloat && grad.numel() == master.numel());
  c10::cuda::CUDAGuard g(master.device());
  msb::adamw_fanout(master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
                    grad.data_ptr<float>(), heap_table(heaps), param_off, (int)pdtype, s0,
                    master.numel(), (int)world, stats.data_ptr<float>(), lr, beta1, beta2, eps,
                    wd, bc1, bc2, grad_mul, stream_of(master));
}

bool base_aligned(const at::Tensor& heaps, int64_t shard_off, const at::Tensor& dst) {
  // heap bases are cudaMalloc'd (256-byte aligned); the region offset and the
  // destination decide the 16-byte path
  return (shard_off % 16) == 0 && (reinterpret_cast<uintptr_t>(dst.data_ptr()) & 15) == 0;
}

void gather_pull_py(const at::Tensor& heaps, int64_t shard_off, int64_t shard, int64_t world,
                    const at::Tensor& dst) {
  check_cuda_contig(dst, "dst");
  TORCH_CHECK(dst.numel() >= shard * world);
  c10::cuda::CUDAGuard g(dst.device());
  msb::gather_pull(heap_table(heaps), shard_off, shard, (int)world, dst.data_ptr(),
                   dtype_code(dst), base_aligned(heaps, shard_off, dst), stream_of(dst));
}

// dst (the full flat arena) [lo, hi) <- the owners' shards
void gather_range_py(const at::Tensor& heaps, int64_t shard_off, int64_t shard, int64_t lo,
                     int64_t hi, const at::Tensor& dst) {
  check_cuda_contig(dst, "dst");
  TORCH_CHECK(0 <= lo && lo <= hi && hi <= dst.numel(), "gather range out of bounds");
  c10::cuda::CUDAGuard g(dst.device());
  msb::gather_range(heap_table(heaps), shard_off, shard, lo, hi, dst.data_ptr(), dtype_code(dst),
                    base_aligned(heaps, shard_off, dst), stream_of(dst));
}

}  // namespace

// Records of the bounds-checked debug build, one per translation unit with
// checks: (unit, failed checks, site of the first failure, its index, its
// limit).  All zero in the release build.
std::vector<std::tuple<std::string, int64_t, int64_t, int64_t, int64_t>> bounds_status(
    bool reset) {
  using Reader = void (*)(msb::BoundsRecord*, bool);
  const std::pair<const char*, Reader> units[] = {{"nn", &msb::bounds_read_nn},
                                                  {"gemm", &msb::bounds_read_gemm},
                                                  {"attention", &msb::bounds_read_attention}};
  std::vector<std::tuple<std::string, int64_t, int64_t, int64_t, int64_t>> out;
  for (const auto& u : units) {
    msb::BoundsRecord r{};
    u.second(&r, reset);
    out.emplace_back(u.first, (int64_t)r.count, (int64_t)r.site, (int64_t)r.index,
                     (int64_t)r.limit);
  }
  return out;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, mod) {
  mod.doc() = "minispeed_b200 sm_100a kernels";
  mod.def("grad_stats", &grad_stats);
  mod.def("stats_finalize", &stats_finalize);
  mod.def("stats_epilogue", &stats_epilogue);
  mod.def("adamw", &adamw);
  mod.def("cast_scale", &cast_scale);
  mod.def("launch_count", &msb::launch_count);
  mod.def("bounds_check_build", &msb::bounds_check_build);
  mod.def("bounds_status", &bounds_status);
  mod.def("count_launches", [](int64_t n) { msb::count_launch((int)n); },
          "add n to the launch counter (kernels replayed from a captured CUDA graph)");
  mod.def("add_norm_fwd", &add_norm_fwd);
  mod.def("norm_bwd", &norm_bwd);
  mod.def("colsum_partial", &colsum_partial);
  mod.def("colsum_finish", &colsum_finish);
  mod.def("colsum_finish_many", &colsum_finish_many);
  mod.def("accum_cast", &accum_cast);
  mod.def("bias_gelu_fwd", &bias_gelu_fwd);
  mod.def("gelu_bwd", &gelu_bwd);
  mod.def("swiglu_fwd", &swiglu_fwd);
  mod.def("swiglu_bwd", &swiglu_bwd);
  mod.def("cross_entropy_fwd", &cross_entropy_fwd);
  mod.def("cross_entropy_bwd", &cross_entropy_bwd);
  mod.def("cross_entropy_fwd_grad", &cross_entropy_fwd_grad);
  mod.def("cross_entropy_grad_rescale", &cross_entropy_grad_rescale);
  mod.def("embedding_fwd", &embedding_fwd);
  mod.def("embedding_bwd", &embedding_bwd);
  mod.def("rope", &rope);
  mod.def("gemm", &gemm);
  mod.def("attention_fwd", &attention_fwd_py);
  mod.def("attention_bwd", &attention_bwd_py);
  mod.def("gemm_plan", &gemm_plan_py);
  mod.def("gemm_cached_plan", &gemm_cached_plan);
  mod.def("gemm_reset_stream_k", &gemm_reset_stream_k);
  mod.def("peer_alloc", &peer_alloc_py);
  mod.def("peer_free", &peer_free_py);
  mod.def("peer_handle", &peer_handle_py);
  mod.def("peer_open", &peer_open_py);
  mod.def("peer_close", &peer_close_py);
  mod.def("tensor_from_ptr", &tensor_from_ptr);
  mod.def("copy_many", &copy_many);
  mod.def("peer_barrier", &peer_barrier_py);
  mod.def("rs_stats", &rs_stats_py);
  mod.def("stats_exchange", &stats_exchange_py);
  mod.def("adamw_fanout", &adamw_fanout_py);
  mod.def("gather_pull", &gather_pull_py);
  mod.def("gather_range", &gather_range_py);
}
