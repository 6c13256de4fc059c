// Column sums without device allocation.
//
// This entry point has no counterpart in the reference (minispeed has no
// native code); it is an addition of this library.
//
// What it computes: out[c] (+)= sum over rows r of a[r, c] for a row-major
// [M, N] matrix of fp32/fp16/bf16 with row stride `ld` elements (a bias
// gradient is the column sum of the layer's output gradient).  It is the same
// two-pass reduction as the library's column-sum path (per-chunk partial rows,
// then a fixed-order sum of the partials), but the partial rows live in a
// buffer that is part of the library image instead of being allocated per
// call.
//
// Who needs it: callers that cannot call cudaMalloc (or any allocator) when
// they run this operation.  Examples: an inference or training runtime that
// plans all device memory once at start-up and forbids allocation afterwards,
// so that memory use stays fixed and no allocator latency or fragmentation
// appears mid-run; code linked into a process whose device memory is owned by
// another framework's allocator, where a direct cudaMalloc would escape that
// allocator's accounting and limits; and callers that reach this library only
// through a C ABI, passing device pointers they already own, with no CUDA
// allocator of their own at hand.
//
// Contract:
//   * The scratch is the file-scope array g_noalloc_colsum_scratch of
//     kScratchFloats floats (4 MiB).  Every GPU that loads the library holds
//     it until the process exits.
//   * The caller passes the input matrix and the output vector; nothing is
//     allocated or freed (no cudaMalloc, no cudaFree, no allocating library
//     call) on any call.
//   * N must be at most kScratchFloats; a larger N is rejected with
//     kNoallocTooWide before anything is launched.
//   * Set-up: the first call on a device (with that device current) looks up
//     the array's device address with cudaGetSymbolAddress and caches it for
//     that device.  Make that first call before capturing any stream.
//   * All calls share the one array and it keeps the last call's contents.
//     Nothing in it must start at zero: every partial a call reads is written
//     by the same call first.  Calls that overlap on the GPU (different
//     streams, or different host threads) race on the array; serialize them.
#include <mutex>

#include "colsum_noalloc.h"
#include "common.cuh"

namespace {

constexpr long long kScratchFloats = MSB_COLSUM_NOALLOC_MAX_N;
constexpr int kMaxChunks = 256;
constexpr int kMaxDevices = 64;

// return codes of msb_colsum_noalloc (declared in colsum_noalloc.h)
constexpr int kNoallocOk = MSB_NOALLOC_OK;
constexpr int kNoallocBadArgs = MSB_NOALLOC_BAD_ARGS;
constexpr int kNoallocTooWide = MSB_NOALLOC_TOO_WIDE;
constexpr int kNoallocCudaError = MSB_NOALLOC_CUDA_ERROR;

static __device__ __align__(256) float g_noalloc_colsum_scratch[kScratchFloats];

float* g_scratch_addr[kMaxDevices] = {nullptr};
std::mutex g_setup_mutex;

template <typename T>
__device__ __forceinline__ float ld_f(const T* p) {
  return msb::to_f32(*p);
}

// block (256-column slab, row chunk): partial[chunk][c] = sum of its rows
template <typename T>
__global__ void __launch_bounds__(256)
noalloc_colsum_partial(const T* __restrict__ a, long long M, long long N, long long ld,
                       long long rows_per_chunk, float* __restrict__ partial) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long c = blockIdx.x * 256LL + threadIdx.x;
  const long long r0 = blockIdx.y * rows_per_chunk;
  const long long r1 = r0 + rows_per_chunk < M ? r0 + rows_per_chunk : M;
  __shared__ float red[8][256];
  // each warp walks every 8th row of the chunk; each thread one column per
  // 32-column group of the slab (coalesced row reads)
  float acc[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) acc[g] = 0.f;
  for (long long r = r0 + warp; r < r1; r += 8) {
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const long long col = blockIdx.x * 256LL + g * 32 + lane;
      if (col < N) acc[g] += ld_f(a + r * ld + col);
    }
  }
#pragma unroll
  for (int g = 0; g < 8; ++g) red[warp][g * 32 + lane] = acc[g];
  __syncthreads();
  if (c < N) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w][threadIdx.x];
    partial[blockIdx.y * N + c] = t;
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
noalloc_colsum_finish(const float* __restrict__ partial, int chunks, long long N,
                      T* __restrict__ out, int accumulate) {
  const long long c = blockIdx.x * 256LL + threadIdx.x;
  if (c >= N) return;
  float t = 0.f;
  for (int q = 0; q < chunks; ++q) t += partial[q * N + c];
  if (accumulate) t += msb::to_f32(out[c]);
  out[c] = msb::from_f32<T>(t);
}

// Device address of the scratch array for the current device (set-up once).
float* scratch_for_current_device(int* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err = kNoallocCudaError;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_colsum_scratch);
    if (e != cudaSuccess || p == nullptr) {
      std::fprintf(stderr, "msb_colsum_noalloc: cudaGetSymbolAddress failed: %s\n",
                   cudaGetErrorString(e));
      *err = kNoallocCudaError;
      return nullptr;
    }
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  return g_scratch_addr[dev];
}

template <typename T>
int run(const void* a, long long M, long long N, long long ld, void* out, int accumulate,
        float* scratch, cudaStream_t stream) {
  long long chunks = kScratchFloats / N;
  if (chunks > kMaxChunks) chunks = kMaxChunks;
  const long long need = (M + 63) / 64;
  if (chunks > need) chunks = need < 1 ? 1 : need;
  const long long rows = (M + chunks - 1) / chunks;
  chunks = (M + rows - 1) / rows;
  dim3 grid(static_cast<unsigned>((N + 255) / 256), static_cast<unsigned>(chunks));
  noalloc_colsum_partial<T><<<grid, 256, 0, stream>>>(static_cast<const T*>(a), M, N, ld, rows,
                                                      scratch);
  noalloc_colsum_finish<T><<<static_cast<unsigned>((N + 255) / 256), 256, 0, stream>>>(
      scratch, static_cast<int>(chunks), N, static_cast<T*>(out), accumulate);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    std::fprintf(stderr, "msb_colsum_noalloc: launch failed: %s\n", cudaGetErrorString(e));
    return kNoallocCudaError;
  }
  return kNoallocOk;
}

}  // namespace

// out[N] (+)= column sums of a[M, N] (row stride ld elements), on `stream`.
// dtype: 0 fp32, 1 fp16, 2 bf16 (input and output share it).  Returns 0 on
// success, -1 for invalid arguments, -2 when N exceeds the 1,048,576-column
// scratch capacity (nothing is launched), -3 for a CUDA error.
extern "C" int msb_colsum_noalloc(const void* a, int dtype, long long M, long long N,
                                  long long ld, void* out, int accumulate, void* stream) {
  if (a == nullptr || out == nullptr || M < 1 || N < 1 || ld < N || dtype < 0 || dtype > 2) {
    std::fprintf(stderr, "msb_colsum_noalloc: invalid arguments\n");
    return kNoallocBadArgs;
  }
  if (N > kScratchFloats) {
    std::fprintf(stderr,
                 "msb_colsum_noalloc: N=%lld exceeds the scratch capacity of %lld columns\n", N,
                 kScratchFloats);
    return kNoallocTooWide;
  }
  int err = kNoallocOk;
  float* scratch = scratch_for_current_device(&err);
  if (scratch == nullptr) return err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case 0: return run<float>(a, M, N, ld, out, accumulate, scratch, st);
    case 1: return run<__half>(a, M, N, ld, out, accumulate, scratch, st);
    default: return run<__nv_bfloat16>(a, M, N, ld, out, accumulate, scratch, st);
  }
}
