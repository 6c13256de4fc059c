// Shared helpers for the sm_100a kernels of minispeed_b200.
//
// The .cu translation units include only CUDA headers and this file; the
// PyTorch binding layer (bindings.cpp) passes raw device pointers, sizes and
// the current stream.  Keeping ATen out of the .cu files keeps each nvcc
// invocation to a few seconds.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <stdexcept>
#include <string>

#include "kernels_api.h"

namespace msb {

// Host-side count of kernel launches issued by this library (bench evidence).
void count_launch(int n = 1);

inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
  }
}

// Launch errors; the launches themselves are counted by launch() below.
#define MSB_CHECK_LAUNCH(name)                                  \
  do {                                                          \
    ::msb::check_cuda(cudaGetLastError(), name);                \
  } while (0)

// Programmatic dependent launch (opt-in: MSB_PDL=1).  Every kernel of this
// library is then launched with programmatic stream serialization allowed,
// so the GPU may start it while the previous kernel of the stream is still
// finishing; its launch latency and the set-up before pdl_begin() overlap
// that tail.  Off by default: inside the replayed CUDA graph of a GPT-2 step
// the kernels already run back to back, and the A/B runs measured no gain.  Every kernel calls pdl_begin() before its first access to
// global memory: griddepcontrol.wait returns once the previous kernel has
// completed and its writes are visible (at once when there is none or it was
// launched without the attribute), and launch_dependents then lets the next
// kernel start early in turn.  Inside a CUDA-graph capture the attribute
// becomes a programmatic edge of the graph.
bool pdl_enabled();

__device__ __forceinline__ void pdl_begin() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline void launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                   cudaStream_t st, Args... args) {
  static_assert(sizeof...(KArgs) == sizeof...(Args), "kernel argument count");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  check_cuda(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...), "kernel launch");
  count_launch();
}

constexpr int kNumSMs = 148;

// Bounds checks (see BoundsRecord).  MSB_INB(i, n, site): i in [0, n);
// MSB_CHECK(cond, site, i, n): an invariant.  Both are `true` in the release
// build.  MSB_OK(cond, site, i, n): a condition the release build tests as
// well (an out-of-range token id reads as a zero row there); the debug build
// also records its failure.  MSB_BOUNDS_TU(name) defines the translation
// unit's bounds_read_<name>.
#ifdef MSB_BOUNDS_CHECK
static __device__ BoundsRecord g_bounds;
static __device__ __noinline__ bool bounds_fail(int site, long long index, long long limit) {
  if (atomicAdd(&g_bounds.count, 1ull) == 0ull) {
    g_bounds.site = site;
    g_bounds.index = index;
    g_bounds.limit = limit;
  }
  return false;
}
#define MSB_INB(i, n, site)                                                  \
  (((long long)(i) >= 0 && (long long)(i) < (long long)(n)) ||               \
   ::msb::bounds_fail((site), (long long)(i), (long long)(n)))
#define MSB_CHECK(cond, site, i, n) \
  ((cond) || ::msb::bounds_fail((site), (long long)(i), (long long)(n)))
#define MSB_OK(cond, site, i, n) MSB_CHECK(cond, site, i, n)
#define MSB_BOUNDS_TU(NAME)                                                          \
  void bounds_read_##NAME(BoundsRecord* out, bool reset) {                           \
    check_cuda(cudaMemcpyFromSymbol(out, g_bounds, sizeof(BoundsRecord)), "bounds"); \
    if (reset) {                                                                     \
      const BoundsRecord z = {0ull, 0, 0, 0};                                        \
      check_cuda(cudaMemcpyToSymbol(g_bounds, &z, sizeof z), "bounds reset");        \
    }                                                                                \
  }
#else
#define MSB_INB(i, n, site) true
#define MSB_CHECK(cond, site, i, n) true
#define MSB_OK(cond, site, i, n) (cond)
#define MSB_BOUNDS_TU(NAME) \
  void bounds_read_##NAME(BoundsRecord* out, bool) { *out = BoundsRecord{0ull, 0, 0, 0}; }
#endif

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

__device__ __forceinline__ bool finite_f32(float x) {
  // exponent all ones <=> inf or nan
  return (__float_as_uint(x) & 0x7f800000u) != 0x7f800000u;
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ unsigned warp_or(unsigned v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v |= __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// exact (erf) GELU and its derivative, as torch.nn.GELU()
__device__ __forceinline__ float gelu_f(float u) {
  return 0.5f * u * (1.f + erff(u * 0.70710678118654752f));
}
__device__ __forceinline__ float gelu_grad_f(float u) {
  const float cdf = 0.5f * (1.f + erff(u * 0.70710678118654752f));
  const float pdf = expf(-0.5f * u * u) * 0.39894228040143268f;
  return cdf + u * pdf;
}

// 2^x on the FMA and integer pipes (the special-function unit that ex2 uses
// is the softmax's bottleneck).  Range reduction x = n + f, n = rint(x),
// f in [-1/2, 1/2]: adding 1.5 * 2^23 leaves rint(x) in the low mantissa
// bits.  2^f is a degree-3 polynomial whose coefficients minimise the maximum
// relative error on [-1/2, 1/2] (a linear program over 4001 points):
// 7.5e-5, below half an fp16 ulp.  n is added to the exponent field; x is
// clamped at -125 so the result stays a normal number.
__device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -125.f);
  const float t = x + 12582912.f;
  const float f = x - (t - 12582912.f);
  float q = fmaf(0.05517222f, f, 0.24261115f);
  q = fmaf(q, f, 0.69326085f);
  q = fmaf(q, f, 0.99992806f);
  return __int_as_float(__float_as_int(q) + (__float_as_int(t) << 23));
}

// Dispatch a functor over the three float dtypes.
#define MSB_DISPATCH_FLOAT(code, T, ...)                                      \
  switch (code) {                                                             \
    case ::msb::kF32: { using T = float; __VA_ARGS__; break; }                \
    case ::msb::kF16: { using T = __half; __VA_ARGS__; break; }               \
    case ::msb::kBF16: { using T = __nv_bfloat16; __VA_ARGS__; break; }       \
    default: throw std::runtime_error("unsupported dtype code");             \
  }

inline int grid_for(long long work_items, int threads, int max_blocks) {
  long long b = (work_items + threads - 1) / threads;
  if (b < 1) b = 1;
  if (b > max_blocks) b = max_blocks;
  return static_cast<int>(b);
}

}  // namespace msb
