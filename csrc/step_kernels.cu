// Step-pipeline kernels: gradient statistics, AdamW(+cast), cast/scale.
//
// These replace the per-step chain of the reference optimizer step
// (minispeed/engine.py:268-322): flatten copies, isfinite().all() with a host
// sync, unscale, sum of squares with a second host sync, ~10 elementwise
// AdamW kernels and the per-parameter fp32->fp16 copies.  Here:
//
//   grad_stats     one read of the gradient -> per-block (sum of squares of
//                  g*mul, inf/nan flag) partials, written to a scratch array
//   stats_finalize one block folds the partials in a fixed order (the result
//                  is bitwise reproducible run to run) into
//                  out = [flag, sumsq, norm, clip_coef]
//   adamw          one pass: reads master/m/v/grad, skips on the device when
//                  out[0] flags an overflow, applies grad*mul*clip_coef,
//                  writes master/m/v and the model-dtype cast of the master
//                  into the parameter arena.
//
// Everything is memory bound; 16-byte vector accesses are used whenever all
// operands are aligned for them, scalar accesses otherwise.
#include "common.cuh"

namespace msb {

namespace {

constexpr int kStatThreads = 256;

template <typename T, int VEC>
struct alignas(sizeof(T) * VEC) Vec {
  T v[VEC];
};

template <typename T>
__device__ __forceinline__ void stat_accum(T x, float mul, float& ss, unsigned& bad) {
  float f = to_f32(x);
  bad |= finite_f32(f) ? 0u : 1u;
  float s = f * mul;
  ss = fmaf(s, s, ss);
}

template <typename T, int VEC>
__global__ void __launch_bounds__(kStatThreads)
grad_stats_kernel(const T* __restrict__ x, long long n, float mul,
                  float* __restrict__ partials, unsigned* __restrict__ flags) {
  ::msb::pdl_begin();
  float ss = 0.f;
  unsigned bad = 0u;
  const long long nvec = n / VEC;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const Vec<T, VEC>* xv = reinterpret_cast<const Vec<T, VEC>*>(x);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    Vec<T, VEC> r = xv[i];
#pragma unroll
    for (int k = 0; k < VEC; ++k) stat_accum(r.v[k], mul, ss, bad);
  }
  for (long long i = nvec * VEC + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += stride)
    stat_accum(x[i], mul, ss, bad);

  __shared__ float s_ss[kStatThreads / 32];
  __shared__ unsigned s_bad[kStatThreads / 32];
  ss = warp_sum(ss);
  bad = warp_or(bad);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    s_ss[warp] = ss;
    s_bad[warp] = bad;
  }
  __syncthreads();
  if (warp == 0) {
    ss = lane < kStatThreads / 32 ? s_ss[lane] : 0.f;
    bad = lane < kStatThreads / 32 ? s_bad[lane] : 0u;
    ss = warp_sum(ss);
    bad = warp_or(bad);
    if (lane == 0) {
      partials[blockIdx.x] = ss;
      flags[blockIdx.x] = bad;
    }
  }
}

constexpr int kFinThreads = 512;

__device__ void compute_norm_coef(float* out, double max_norm) {
  float norm = sqrtf(out[1]);
  out[2] = norm;
  float coef = 1.f;
  if (max_norm > 0.0 && (double)norm > max_norm) coef = (float)(max_norm / ((double)norm + 1e-6));
  out[3] = coef;
}

__global__ void __launch_bounds__(kFinThreads)
stats_finalize_kernel(const float* __restrict__ partials, const unsigned* __restrict__ flags,
                      int n, float* __restrict__ out, double max_norm, int epilogue) {
  ::msb::pdl_begin();
  // fixed assignment of partials to threads + fixed tree => deterministic
  double acc = 0.0;
  unsigned bad = 0u;
  for (int i = threadIdx.x; i < n; i += kFinThreads) {
    acc += (double)partials[i];
    bad |= flags[i];
  }
  __shared__ double s_acc[kFinThreads];
  __shared__ unsigned s_bad[kFinThreads];
  s_acc[threadIdx.x] = acc;
  s_bad[threadIdx.x] = bad;
  __syncthreads();
  for (int w = kFinThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) {
      s_acc[threadIdx.x] += s_acc[threadIdx.x + w];
      s_bad[threadIdx.x] |= s_bad[threadIdx.x + w];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    out[0] = s_bad[0] ? 1.f : 0.f;
    out[1] = (float)s_acc[0];
    if (epilogue) compute_norm_coef(out, max_norm);
  }
}

__global__ void stats_epilogue_kernel(float* out, double max_norm) {
  ::msb::pdl_begin();
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    out[0] = out[0] > 0.f ? 1.f : 0.f;
    compute_norm_coef(out, max_norm);
  }
}

struct AdamArgs {
  float lr_neg;       // -lr
  float wd_term;      // -lr*wd
  float b1, omb1;     // beta1, 1-beta1
  float b2, omb2;     // beta2, 1-beta2
  float bc1, bc2;     // bias corrections
  float eps;
  float grad_mul;     // unscale / averaging factor (exact power of two in practice)
};

template <typename G, typename P>
__device__ __forceinline__ void adam_elem(float& p, float& m, float& v, G graw, float coef,
                                          const AdamArgs& a) {
  float g = to_f32(graw) * a.grad_mul;
  g = g * coef;
  if (a.wd_term != 0.f) p = p + a.wd_term * p;
  m = m * a.b1 + a.omb1 * g;
  v = v * a.b2 + a.omb2 * g * g;
  float denom = sqrtf(v / a.bc2) + a.eps;
  p = p + a.lr_neg * ((m / a.bc1) / denom);
}

template <typename G, typename P, int VEC, bool WRITE_P>
__global__ void __launch_bounds__(256)
adamw_kernel(float* __restrict__ master, float* __restrict__ exp_avg,
             float* __restrict__ exp_avg_sq, const G* __restrict__ grad,
             P* __restrict__ param_out, long long n, const float* __restrict__ stats,
             AdamArgs a) {
  ::msb::pdl_begin();
  float coef = 1.f;
  if (stats != nullptr) {
    if (stats[0] != 0.f) return;  // overflow: the whole step is skipped
    coef = stats[3];
  }
  const long long nvec = n / VEC;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    Vec<float, VEC> p = reinterpret_cast<Vec<float, VEC>*>(master)[i];
    Vec<float, VEC> m = reinterpret_cast<Vec<float, VEC>*>(exp_avg)[i];
    Vec<float, VEC> v = reinterpret_cast<Vec<float, VEC>*>(exp_avg_sq)[i];
    Vec<G, VEC> g = reinterpret_cast<const Vec<G, VEC>*>(grad)[i];
#pragma unroll
    for (int k = 0; k < VEC; ++k) adam_elem<G, P>(p.v[k], m.v[k], v.v[k], g.v[k], coef, a);
    reinterpret_cast<Vec<float, VEC>*>(master)[i] = p;
    reinterpret_cast<Vec<float, VEC>*>(exp_avg)[i] = m;
    reinterpret_cast<Vec<float, VEC>*>(exp_avg_sq)[i] = v;
    if (WRITE_P) {
      Vec<P, VEC> o;
#pragma unroll
      for (int k = 0; k < VEC; ++k) o.v[k] = from_f32<P>(p.v[k]);
      reinterpret_cast<Vec<P, VEC>*>(param_out)[i] = o;
    }
  }
  for (long long i = nvec * VEC + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    float p = master[i], m = exp_avg[i], v = exp_avg_sq[i];
    adam_elem<G, P>(p, m, v, grad[i], coef, a);
    master[i] = p;
    exp_avg[i] = m;
    exp_avg_sq[i] = v;
    if (WRITE_P) param_out[i] = from_f32<P>(p);
  }
}

template <typename S, typename D, int VEC>
__global__ void __launch_bounds__(256)
cast_scale_kernel(const S* __restrict__ src, D* __restrict__ dst, long long n, float mul) {
  ::msb::pdl_begin();
  const long long nvec = n / VEC;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    Vec<S, VEC> s = reinterpret_cast<const Vec<S, VEC>*>(src)[i];
    Vec<D, VEC> d;
#pragma unroll
    for (int k = 0; k < VEC; ++k) d.v[k] = from_f32<D>(to_f32(s.v[k]) * mul);
    reinterpret_cast<Vec<D, VEC>*>(dst)[i] = d;
  }
  for (long long i = nvec * VEC + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += stride)
    dst[i] = from_f32<D>(to_f32(src[i]) * mul);
}

inline bool aligned(const void* p, int bytes) {
  return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

}  // namespace

int grad_stats(const void* x, int dtype, long long n, float mul, float* partials,
               unsigned* flags, int max_blocks, cudaStream_t stream) {
  int blocks = 1;
  MSB_DISPATCH_FLOAT(dtype, T, {
    constexpr int V = 16 / sizeof(T);
    const bool vec = aligned(x, 16);
    const long long items = vec ? n / V : n;
    blocks = grid_for(items, kStatThreads, max_blocks < 1 ? 1 : max_blocks);
    if (vec)
      ::msb::launch(grad_stats_kernel<T, V>, blocks, kStatThreads, 0, stream, 
          static_cast<const T*>(x), n, mul, partials, flags);
    else
      ::msb::launch(grad_stats_kernel<T, 1>, blocks, kStatThreads, 0, stream, 
          static_cast<const T*>(x), n, mul, partials, flags);
  });
  MSB_CHECK_LAUNCH("grad_stats");
  return blocks;
}

void stats_finalize(const float* partials, const unsigned* flags, int n, float* out,
                    double max_norm, bool epilogue, cudaStream_t stream) {
  ::msb::launch(stats_finalize_kernel, 1, kFinThreads, 0, stream, partials, flags, n, out, max_norm,
                                                       epilogue ? 1 : 0);
  MSB_CHECK_LAUNCH("stats_finalize");
}

void stats_epilogue(float* out, double max_norm, cudaStream_t stream) {
  ::msb::launch(stats_epilogue_kernel, 1, 32, 0, stream, out, max_norm);
  MSB_CHECK_LAUNCH("stats_epilogue");
}

void adamw(float* master, float* m, float* v, const void* grad, int gdtype, void* param_out,
           int pdtype, long long n, const float* stats, double lr, double beta1, double beta2,
           double eps, double wd, double bc1, double bc2, double grad_mul,
           cudaStream_t stream) {
  AdamArgs a;
  a.lr_neg = (float)(-lr);
  a.wd_term = (float)(-lr * wd);
  a.b1 = (float)beta1;
  a.omb1 = (float)(1.0 - beta1);
  a.b2 = (float)beta2;
  a.omb2 = (float)(1.0 - beta2);
  a.bc1 = (float)bc1;
  a.bc2 = (float)bc2;
  a.eps = (float)eps;
  a.grad_mul = (float)grad_mul;
  const int threads = 256;
  const bool vec = aligned(master, 16) && aligned(m, 16) && aligned(v, 16) &&
                   aligned(grad, gdtype == kF32 ? 16 : 8) &&
                   (param_out == nullptr || aligned(param_out, pdtype == kF32 ? 16 : 8));
  const long long items = vec ? n / 4 : n;
  const int blocks = grid_for(items, threads, kNumSMs * 16);
  MSB_DISPATCH_FLOAT(gdtype, G, {
    if (param_out == nullptr) {
      if (vec)
        ::msb::launch(adamw_kernel<G, float, 4, false>, blocks, threads, 0, stream, 
            master, m, v, static_cast<const G*>(grad), nullptr, n, stats, a);
      else
        ::msb::launch(adamw_kernel<G, float, 1, false>, blocks, threads, 0, stream, 
            master, m, v, static_cast<const G*>(grad), nullptr, n, stats, a);
    } else {
      MSB_DISPATCH_FLOAT(pdtype, P, {
        if (vec)
          ::msb::launch(adamw_kernel<G, P, 4, true>, blocks, threads, 0, stream, 
              master, m, v, static_cast<const G*>(grad), static_cast<P*>(param_out), n, stats,
              a);
        else
          ::msb::launch(adamw_kernel<G, P, 1, true>, blocks, threads, 0, stream, 
              master, m, v, static_cast<const G*>(grad), static_cast<P*>(param_out), n, stats,
              a);
      });
    }
  });
  MSB_CHECK_LAUNCH("adamw");
}

void cast_scale(const void* src, int sdtype, void* dst, int ddtype, long long n, float mul,
                cudaStream_t stream) {
  const int threads = 256;
  const bool vec = aligned(src, 16) && aligned(dst, 16);
  const long long items = vec ? n / 4 : n;
  const int blocks = grid_for(items, threads, kNumSMs * 16);
  MSB_DISPATCH_FLOAT(sdtype, S, {
    MSB_DISPATCH_FLOAT(ddtype, D, {
      if (vec)
        ::msb::launch(cast_scale_kernel<S, D, 4>, blocks, threads, 0, stream, 
            static_cast<const S*>(src), static_cast<D*>(dst), n, mul);
      else
        ::msb::launch(cast_scale_kernel<S, D, 1>, blocks, threads, 0, stream, 
            static_cast<const S*>(src), static_cast<D*>(dst), n, mul);
    });
  });
  MSB_CHECK_LAUNCH("cast_scale");
}

}  // namespace msb
