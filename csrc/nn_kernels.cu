// Memory-bound model kernels of the GPT / Llama blocks.
//
//   add_layernorm_fwd  s = x (+ delta); y = LN(s) * w + b  (or RMSNorm: no
//                      mean, no bias); saves mean/rstd per row.  Fusing the
//                      residual add into the norm removes one read+write of
//                      the residual stream per add.
//   layernorm_bwd      dx = LN'(dy) (+ dresidual), per-block fp32 partial
//                      column sums for dw/db (deterministic second pass)
//   colsum_*           column sums of [M,N] (bias grads) via partials
//   bias_gelu_fwd      u += b; h = gelu(u)  (exact erf GELU, as nn.GELU())
//   gelu_bwd           du = dh * gelu'(u)
//   swiglu_fwd/bwd     h = silu(g) * u and its gradient
//   cross_entropy_*    fused softmax cross-entropy over model-dtype logits:
//                      forward = one online-softmax pass per row (loss, lse),
//                      backward = one pass writing dlogits in place; the fp32
//                      logits the reference materializes never exist.
//   embedding_*        token (+ position) gather-add; backward: scatter-add into a
//                      persistent fp32 accumulator, then only the touched rows are
//                      added into the gradient and cleared
//   rope_*             rotary position embedding on q/k in place
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>

#include "common.cuh"

namespace msb {
namespace {

template <typename T>
struct alignas(16) Pack8 {
  T v[8];
};

// 2^x on the special-function unit; e^x = 2^(x * log2(e))
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 8-element accesses: one 16-byte transaction when the address allows it,
// element-wise otherwise.  Parameters are views into a flat arena at
// arbitrary element offsets, so weights and biases need not be aligned.
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&f)[8]) {
  if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
    Pack8<T> r = *reinterpret_cast<const Pack8<T>*>(p);
#pragma unroll
    for (int k = 0; k < 8; ++k) f[k] = to_f32(r.v[k]);
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) f[k] = to_f32(p[k]);
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&f)[8]) {
  if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
    Pack8<T> r;
#pragma unroll
    for (int k = 0; k < 8; ++k) r.v[k] = from_f32<T>(f[k]);
    *reinterpret_cast<Pack8<T>*>(p) = r;
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) p[k] = from_f32<T>(f[k]);
  }
}

// 8 16-bit values as one 16-byte quad of registers, unpacked and packed two
// at a time (a bf16 is the upper half of an fp32; element 0 is the low half
// of the first word), so packed rows take 4 registers per 8 values.
template <typename T>
__device__ __forceinline__ void unpack_u4(const uint4& r, float (&f)[8]) {
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      f[2 * q] = __uint_as_float(w[q] << 16);
      f[2 * q + 1] = __uint_as_float(w[q] & 0xffff0000u);
    } else {
      const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w[q]));
      f[2 * q] = v.x;
      f[2 * q + 1] = v.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack_u4(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * q], f[2 * q + 1]);
      w[q] = *reinterpret_cast<const uint32_t*>(&h);
    } else {
      const __half2 h = __floats2half2_rn(f[2 * q], f[2 * q + 1]);
      w[q] = *reinterpret_cast<const uint32_t*>(&h);
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// ------------------------------------------------------------ layernorm
// One warp per row; the row stays in registers (NV vectors of 8 per lane).
template <typename T, int NV, bool RMS>
__global__ void __launch_bounds__(256)
add_norm_fwd_kernel(const T* __restrict__ x, const T* __restrict__ delta,
                    const T* __restrict__ w, const T* __restrict__ b, T* __restrict__ s_out,
                    T* __restrict__ y, float* __restrict__ mean_out,
                    float* __restrict__ rstd_out, int M, int C, float eps) {
  ::msb::pdl_begin();
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const int nvec = C >> 3;
  const size_t base = (size_t)row * C;
  float v[NV][8];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (lane + i * 32) << 3;
    if ((lane + i * 32) < nvec) {
      load8(x + base + c, v[i]);
      if (delta != nullptr) {
        float d[8];
        load8(delta + base + c, d);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[i][k] += d[k];
        // the residual stream is stored in the model dtype: normalise the
        // rounded value so that forward and backward see the same input
#pragma unroll
        for (int k = 0; k < 8; ++k) v[i][k] = to_f32(from_f32<T>(v[i][k]));
        if (s_out != nullptr) store8(s_out + base + c, v[i]);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) sum += v[i][k];
    }
  }
  float mean = 0.f;
  if (!RMS) mean = warp_sum(sum) / (float)C;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i)
    if ((lane + i * 32) < nvec) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float d = v[i][k] - mean;
        sq += d * d;
      }
    }
  const float var = warp_sum(sq) / (float)C;
  const float rstd = rsqrtf(var + eps);
  if (lane == 0) {
    if (mean_out != nullptr) mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (lane + i * 32) << 3;
    if ((lane + i * 32) < nvec) {
      float wf[8], o[8];
      load8(w + c, wf);
      if (RMS) {
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = (v[i][k] * rstd) * wf[k];
      } else {
        float bf[8] = {0, 0, 0, 0, 0, 0, 0, 0};   // a LayerNorm without bias: b == nullptr
        if (b != nullptr) load8(b + c, bf);
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = ((v[i][k] - mean) * rstd) * wf[k] + bf[k];
      }
      store8(y + base + c, o);
    }
  }
}

// Forward for 16-byte aligned rows (every row pointer aligned, C % 8 == 0):
// each warp issues all of its row's loads before it uses any, so a row costs
// one memory round trip rather than one per vector (the per-vector loads
// above sit behind a bounds branch and a store, and are not hoisted); the
// rounded residual sum stays packed in the model dtype (4 registers per 8
// values), and the weight and bias are read from shared memory, staged once
// per block as fp32.  Blocks loop over groups of 8 rows.
template <typename T, int NV, bool RMS>
__global__ void __launch_bounds__(256, 2)
add_norm_fwd_rows_kernel(const T* __restrict__ x, const T* __restrict__ delta,
                         const T* __restrict__ w, const T* __restrict__ b, T* __restrict__ s_out,
                         T* __restrict__ y, float* __restrict__ mean_out,
                         float* __restrict__ rstd_out, int M, int C, float eps) {
  extern __shared__ float4 norm_smem4[];
  float* sw = reinterpret_cast<float*>(norm_smem4);
  float* sb = sw + C;
  ::msb::pdl_begin();
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    sw[c] = to_f32(w[c]);
    if (!RMS) sb[c] = b != nullptr ? to_f32(b[c]) : 0.f;   // LayerNorm without bias
  }
  __syncthreads();
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int nvec = C >> 3;
  const uint4* x4 = reinterpret_cast<const uint4*>(x);
  const uint4* d4 = reinterpret_cast<const uint4*>(delta);
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
    const size_t base = (size_t)row * nvec;   // in 8-value vectors
    uint4 xr[NV], dr[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = lane + i * 32;
      if (j < nvec) {
        xr[i] = x4[base + j];
        if (delta != nullptr) dr[i] = d4[base + j];
      }
    }
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = lane + i * 32;
      if (j < nvec) {
        float v[8];
        unpack_u4<T>(xr[i], v);
        if (delta != nullptr) {
          // the residual stream is stored in the model dtype: normalise the
          // rounded value so that forward and backward see the same input
          float d[8];
          unpack_u4<T>(dr[i], d);
#pragma unroll
          for (int k = 0; k < 8; ++k) v[k] += d[k];
          xr[i] = pack_u4<T>(v);
          unpack_u4<T>(xr[i], v);
          if (s_out != nullptr) reinterpret_cast<uint4*>(s_out)[base + j] = xr[i];
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) sum += v[k];
      }
    }
    const float mean = RMS ? 0.f : warp_sum(sum) / (float)C;
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i)
      if (lane + i * 32 < nvec) {
        float v[8];
        unpack_u4<T>(xr[i], v);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float d = v[k] - mean;
          sq += d * d;
        }
      }
    const float rstd = rsqrtf(warp_sum(sq) / (float)C + eps);
    if (lane == 0) {
      if (mean_out != nullptr) mean_out[row] = mean;
      rstd_out[row] = rstd;
    }
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = lane + i * 32;
      if (j < nvec) {
        float v[8], o[8];
        unpack_u4<T>(xr[i], v);
        const float4* w4 = reinterpret_cast<const float4*>(sw + j * 8);
        const float4 wa = w4[0], wb = w4[1];
        const float wf[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        if (RMS) {
#pragma unroll
          for (int k = 0; k < 8; ++k) o[k] = (v[k] * rstd) * wf[k];
        } else {
          const float4* b4 = reinterpret_cast<const float4*>(sb + j * 8);
          const float4 ba = b4[0], bb = b4[1];
          const float bf[8] = {ba.x, ba.y, ba.z, ba.w, bb.x, bb.y, bb.z, bb.w};
#pragma unroll
          for (int k = 0; k < 8; ++k) o[k] = ((v[k] - mean) * rstd) * wf[k] + bf[k];
        }
        reinterpret_cast<uint4*>(y)[base + j] = pack_u4<T>(o);
      }
    }
  }
}

// Row-parallel norm backward: one warp per row, no column accumulators, so
// many rows are in flight per SM (the column sums are a separate tiled pass).
template <typename T, int NV, bool RMS>
__global__ void __launch_bounds__(256)
norm_dx_kernel(const T* __restrict__ dy, const T* __restrict__ s, const T* __restrict__ w,
               const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
               const T* __restrict__ dres, T* __restrict__ dx, int M, int C) {
  ::msb::pdl_begin();
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nvec = C >> 3;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
    const size_t base = (size_t)row * C;
    const float mean = RMS ? 0.f : mean_in[row];
    const float rstd = rstd_in[row];
    float xh[NV][8], g[NV][8];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (lane + i * 32) << 3;
      if ((lane + i * 32) < nvec) {
        float sv[8], dyv[8], wv[8];
        load8(s + base + c, sv);
        load8(dy + base + c, dyv);
        load8(w + c, wv);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          xh[i][k] = (sv[k] - mean) * rstd;
          g[i][k] = dyv[k] * wv[k];
          s1 += g[i][k];
          s2 += g[i][k] * xh[i][k];
        }
      }
    }
    s1 = warp_sum(s1) / (float)C;
    s2 = warp_sum(s2) / (float)C;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (lane + i * 32) << 3;
      if ((lane + i * 32) < nvec) {
        float o[8];
#pragma unroll
        for (int k = 0; k < 8; ++k)
          o[k] = RMS ? rstd * (g[i][k] - xh[i][k] * s2) : rstd * (g[i][k] - s1 - xh[i][k] * s2);
        if (dres != nullptr) {
          float r[8];
          load8(dres + base + c, r);
#pragma unroll
          for (int k = 0; k < 8; ++k) o[k] += r[k];
        }
        store8(dx + base + c, o);
      }
    }
  }
}

// Same computation with every load of a row issued before the row
// reductions: the raw 16-byte packs of s, dy and the residual gradient stay in
// registers (4 registers per 8 values) and x-hat / g are recomputed in the
// second pass.  Used for 16-bit activations whose rows are 16-byte aligned
// and at most 2048 wide (NV <= 8); blocks of 4 warps loop over rows.
template <typename T>
__device__ __forceinline__ void unpack8(const Pack8<T>& r, float (&f)[8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) f[k] = to_f32(r.v[k]);
}

template <typename T, int NV, bool RMS>
__global__ void __launch_bounds__(128, 3)
norm_dx_prefetch_kernel(const T* __restrict__ dy, const T* __restrict__ s,
                        const T* __restrict__ w, const float* __restrict__ mean_in,
                        const float* __restrict__ rstd_in, const T* __restrict__ dres,
                        T* __restrict__ dx, int M, int C) {
  // the weight, staged once per block as fp32 (it was re-read from L2 per
  // vector in both passes, one round trip each)
  extern __shared__ float4 norm_smem4[];
  float* sw = reinterpret_cast<float*>(norm_smem4);
  ::msb::pdl_begin();
  for (int c = threadIdx.x; c < C; c += blockDim.x) sw[c] = to_f32(w[c]);
  __syncthreads();
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nvec = C >> 3;
  auto wvec = [&](int j, float (&wv)[8]) {
    const float4* w4 = reinterpret_cast<const float4*>(sw + j * 8);
    const float4 a = w4[0], b = w4[1];
    wv[0] = a.x; wv[1] = a.y; wv[2] = a.z; wv[3] = a.w;
    wv[4] = b.x; wv[5] = b.y; wv[6] = b.z; wv[7] = b.w;
  };
  const uint4* s4 = reinterpret_cast<const uint4*>(s);
  const uint4* dy4 = reinterpret_cast<const uint4*>(dy);
  const uint4* r4 = reinterpret_cast<const uint4*>(dres);
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
    const size_t base = (size_t)row * nvec;   // in 8-value vectors
    uint4 sp[NV], dp[NV], rp[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = lane + i * 32;
      if (j < nvec) {
        sp[i] = s4[base + j];
        dp[i] = dy4[base + j];
        if (dres != nullptr) rp[i] = r4[base + j];
      }
    }
    const float mean = RMS ? 0.f : mean_in[row];
    const float rstd = rstd_in[row];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = lane + i * 32;
      if (j < nvec) {
        float sv[8], dyv[8], wv[8];
        unpack_u4<T>(sp[i], sv);
        unpack_u4<T>(dp[i], dyv);
        wvec(j, wv);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float xh = (sv[k] - mean) * rstd;
          const float g = dyv[k] * wv[k];
          s1 += g;
          s2 += g * xh;
        }
      }
    }
    s1 = warp_sum(s1) / (float)C;
    s2 = warp_sum(s2) / (float)C;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = lane + i * 32;
      if (j < nvec) {
        float sv[8], dyv[8], wv[8], o[8];
        unpack_u4<T>(sp[i], sv);
        unpack_u4<T>(dp[i], dyv);
        wvec(j, wv);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float xh = (sv[k] - mean) * rstd;
          const float g = dyv[k] * wv[k];
          o[k] = RMS ? rstd * (g - xh * s2) : rstd * (g - s1 - xh * s2);
        }
        if (dres != nullptr) {
          float r[8];
          unpack_u4<T>(rp[i], r);
#pragma unroll
          for (int k = 0; k < 8; ++k) o[k] += r[k];
        }
        reinterpret_cast<uint4*>(dx)[base + j] = pack_u4<T>(o);
      }
    }
  }
}

// The prefetch pass above plus the weight and bias gradients' column
// partials in the same sweep: while a warp has a row's dy and s in
// registers it also adds dy * xhat and dy into per-lane accumulators for its
// 8-column groups.  Each block then reduces its 8 warps in shared memory (a
// fixed order, 256 columns at a time) and writes one partial row of dw and
// one of db; colsum_finish sums the gridDim.x partial rows.  The separate
// partial kernel, which read dy and s a second time, is not launched.
template <typename T, int NV, bool RMS>
__global__ void __launch_bounds__(256)
norm_bwd_fused_kernel(const T* __restrict__ dy, const T* __restrict__ s,
                      const T* __restrict__ w, const float* __restrict__ mean_in,
                      const float* __restrict__ rstd_in, const T* __restrict__ dres,
                      T* __restrict__ dx, float* __restrict__ dw_part,
                      float* __restrict__ db_part, int M, int C) {
  ::msb::pdl_begin();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nvec = C >> 3;
  float aw[NV][8], ab[NV][8];
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      aw[i][k] = 0.f;
      ab[i][k] = 0.f;
    }
  for (int row = blockIdx.x * 8 + warp; row < M; row += gridDim.x * 8) {
    const size_t base = (size_t)row * C;
    Pack8<T> sp[NV], dp[NV], rp[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (lane + i * 32) << 3;
      if ((lane + i * 32) < nvec) {
        sp[i] = *reinterpret_cast<const Pack8<T>*>(s + base + c);
        dp[i] = *reinterpret_cast<const Pack8<T>*>(dy + base + c);
        if (dres != nullptr) rp[i] = *reinterpret_cast<const Pack8<T>*>(dres + base + c);
      }
    }
    const float mean = RMS ? 0.f : mean_in[row];
    const float rstd = rstd_in[row];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (lane + i * 32) << 3;
      if ((lane + i * 32) < nvec) {
        float sv[8], dyv[8], wv[8];
        unpack8(sp[i], sv);
        unpack8(dp[i], dyv);
        load8(w + c, wv);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float xh = (sv[k] - mean) * rstd;
          const float g = dyv[k] * wv[k];
          s1 += g;
          s2 += g * xh;
          aw[i][k] += dyv[k] * xh;
          ab[i][k] += dyv[k];
        }
      }
    }
    s1 = warp_sum(s1) / (float)C;
    s2 = warp_sum(s2) / (float)C;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (lane + i * 32) << 3;
      if ((lane + i * 32) < nvec) {
        float sv[8], dyv[8], wv[8], o[8];
        unpack8(sp[i], sv);
        unpack8(dp[i], dyv);
        load8(w + c, wv);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float xh = (sv[k] - mean) * rstd;
          const float g = dyv[k] * wv[k];
          o[k] = RMS ? rstd * (g - xh * s2) : rstd * (g - s1 - xh * s2);
        }
        if (dres != nullptr) {
          float r[8];
          unpack8(rp[i], r);
#pragma unroll
          for (int k = 0; k < 8; ++k) o[k] += r[k];
        }
        store8(dx + base + c, o);
      }
    }
  }
  // per-block column partials: lane l of vector group i owns columns
  // (l + 32 i) * 8 .. +7; reduce the 8 warps 256 columns (32 groups) at a time
  __shared__ float red[8][256 + 8];
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1 && (RMS || db_part == nullptr)) break;
    float* out = pass == 0 ? dw_part : db_part;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
#pragma unroll
      for (int k = 0; k < 8; ++k) red[warp][lane * 8 + k] = pass == 0 ? aw[i][k] : ab[i][k];
      __syncthreads();
      const int c = i * 256 + threadIdx.x;
      if (c < C) {
        float t = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) t += red[q][threadIdx.x];
        out[(size_t)blockIdx.x * C + c] = t;
      }
      __syncthreads();
    }
  }
}

// Column partials of dw = sum_rows dy * xhat and db = sum_rows dy, tiled like
// colsum_partial_kernel: block (256-column slab, row chunk).
template <typename T, bool RMS>
__global__ void __launch_bounds__(256)
norm_dwdb_partial_kernel(const T* __restrict__ dy, const T* __restrict__ s,
                         const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
                         float* __restrict__ dw_part, float* __restrict__ db_part, int M, int C,
                         int rows_per_block) {
  ::msb::pdl_begin();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = blockIdx.x * 256 + lane * 8;
  const int r0 = blockIdx.y * rows_per_block;
  const int r1 = min(M, r0 + rows_per_block);
  float aw[8] = {0, 0, 0, 0, 0, 0, 0, 0}, ab[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  auto row = [&](const float (&d)[8], const float (&x)[8], int r) {
    const float mean = RMS ? 0.f : mean_in[r];
    const float rstd = rstd_in[r];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      aw[k] += d[k] * ((x[k] - mean) * rstd);
      ab[k] += d[k];
    }
  };
  if (c0 < C) {
    int r = r0 + warp;
    // two rows per step: four 16-byte loads in flight per lane
    for (; r + 8 < r1; r += 16) {
      float d0[8], x0[8], d1[8], x1[8];
      load8(dy + (size_t)r * C + c0, d0);
      load8(s + (size_t)r * C + c0, x0);
      load8(dy + (size_t)(r + 8) * C + c0, d1);
      load8(s + (size_t)(r + 8) * C + c0, x1);
      row(d0, x0, r);
      row(d1, x1, r + 8);
    }
    for (; r < r1; r += 8) {
      float d[8], x[8];
      load8(dy + (size_t)r * C + c0, d);
      load8(s + (size_t)r * C + c0, x);
      row(d, x, r);
    }
  }
  __shared__ float red[8][256 + 8];
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1 && (RMS || db_part == nullptr)) break;
#pragma unroll
    for (int k = 0; k < 8; ++k) red[warp][lane * 8 + k] = pass == 0 ? aw[k] : ab[k];
    __syncthreads();
    const int c = blockIdx.x * 256 + threadIdx.x;
    if (c < C) {
      float t = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q) t += red[q][threadIdx.x];
      (pass == 0 ? dw_part : db_part)[(size_t)blockIdx.y * C + c] = t;
    }
    __syncthreads();
  }
}

// Column sums of a [M, N] matrix (row stride ld) into partials
// [gridDim.y, N]: block (x, y) sums rows [y*rpb, (y+1)*rpb) of a 256-column
// slab; each thread owns 8 adjacent columns (16-byte loads), each warp a row.
template <typename T>
__global__ void __launch_bounds__(256)
colsum_partial_kernel(const T* __restrict__ a, float* __restrict__ part, int M, int N,
                      long long ld, int rows_per_block) {
  ::msb::pdl_begin();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = blockIdx.x * 256 + lane * 8;
  const int r0 = blockIdx.y * rows_per_block;
  const int r1 = min(M, r0 + rows_per_block);
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const bool vec = c0 + 8 <= N &&
                   ((reinterpret_cast<uintptr_t>(a) | (uintptr_t)(ld * (long long)sizeof(T))) & 15) == 0;
  if (vec) {
    // four rows per step: four independent 16-byte loads in flight per lane
    int r = r0 + warp;
    for (; r + 24 < r1; r += 32) {
      Pack8<T> v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        v[u] = *reinterpret_cast<const Pack8<T>*>(a + (long long)(r + 8 * u) * ld + c0);
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] += to_f32(v[u].v[k]);
    }
    for (; r < r1; r += 8) {
      const Pack8<T> v = *reinterpret_cast<const Pack8<T>*>(a + (long long)r * ld + c0);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] += to_f32(v.v[k]);
    }
  } else if (c0 < N) {
    for (int r = r0 + warp; r < r1; r += 8) {
      float f[8];
      const T* p = a + (long long)r * ld + c0;
      if (c0 + 8 <= N) {
        load8(p, f);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) f[k] = (c0 + k < N) ? to_f32(p[k]) : 0.f;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] += f[k];
    }
  }
  __shared__ float red[8][256 + 8];
#pragma unroll
  for (int k = 0; k < 8; ++k) red[warp][lane * 8 + k] = acc[k];
  __syncthreads();
  const int c = blockIdx.x * 256 + threadIdx.x;
  if (c < N) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w][threadIdx.x];
    part[(size_t)blockIdx.y * N + c] = t;
  }
}

// out[c] (+)= sum_p part[p][c] for the 32 columns of column block `cb`:
// 8 warps over the parts, then one warp adds the 8 sums in warp order.
template <typename T>
__device__ __forceinline__ void colsum_finish_block(const float* __restrict__ part, int nparts,
                                                    int N, T* __restrict__ out, int accumulate,
                                                    int cb) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = cb * 32 + lane;
  float t = 0.f;
  if (c < N)
    for (int q = warp; q < nparts; q += 8) t += part[(size_t)q * N + c];
  __shared__ float red[8][33];
  red[warp][lane] = t;
  __syncthreads();
  if (warp == 0 && c < N) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) acc += red[w][lane];
    if (accumulate) acc += to_f32(out[c]);
    out[c] = from_f32<T>(acc);
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
colsum_finish_kernel(const float* __restrict__ part, int nparts, int N, T* __restrict__ out,
                     int accumulate) {
  ::msb::pdl_begin();
  colsum_finish_block<T>(part, nparts, N, out, accumulate, blockIdx.x);
}

// Several finishes in one launch: job j owns the blocks first[j] ..
// first[j + 1] - 1 (ceil(N_j / 32) of them); the same sums in the same order
// as one colsum_finish_kernel launch per job.
struct ColsumBatch {
  ColsumJob job[kMaxColsumJobs];
  int first[kMaxColsumJobs + 1];
  int njobs;
};

template <typename T>
__global__ void __launch_bounds__(256)
colsum_finish_many_kernel(const __grid_constant__ ColsumBatch b) {
  ::msb::pdl_begin();
  int j = 0;
  while (j + 1 < b.njobs && (int)blockIdx.x >= b.first[j + 1]) ++j;
  const ColsumJob& jb = b.job[j];
  colsum_finish_block<T>(jb.part, jb.nparts, jb.N, static_cast<T*>(jb.out), jb.accumulate,
                         (int)blockIdx.x - b.first[j]);
}

// dst (+)= float(src) for a float32 source (accumulating gradients in place)
template <typename T>
__global__ void __launch_bounds__(256)
accum_cast_kernel(const float* __restrict__ src, T* __restrict__ dst, long long n, int accumulate) {
  ::msb::pdl_begin();
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float v = src[i];
    if (accumulate) v += to_f32(dst[i]);
    dst[i] = from_f32<T>(v);
  }
}

// ---------------------------------------------------------------- GELU
template <typename T>
__global__ void __launch_bounds__(256)
bias_gelu_fwd_kernel(T* __restrict__ u, const T* __restrict__ bias, T* __restrict__ h,
                     long long total, int N) {
  ::msb::pdl_begin();
  const long long nvec = total >> 3;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec;
       i += (long long)gridDim.x * blockDim.x) {
    const long long e = i << 3;
    const int c = (int)(e % N);
    float f[8], bf[8], o[8];
    load8(u + e, f);
    if (bias != nullptr) {
      load8(bias + c, bf);
#pragma unroll
      for (int k = 0; k < 8; ++k) f[k] += bf[k];
      store8(u + e, f);
#pragma unroll
      for (int k = 0; k < 8; ++k) f[k] = to_f32(from_f32<T>(f[k]));
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = gelu_f(f[k]);
    store8(h + e, o);
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
gelu_bwd_kernel(const T* __restrict__ dh, const T* __restrict__ u, T* __restrict__ du,
                long long total) {
  ::msb::pdl_begin();
  const long long nvec = total >> 3;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec;
       i += (long long)gridDim.x * blockDim.x) {
    float a[8], b[8], o[8];
    load8(dh + (i << 3), a);
    load8(u + (i << 3), b);
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = a[k] * gelu_grad_f(b[k]);
    store8(du + (i << 3), o);
  }
}

// -------------------------------------------------------------- SwiGLU
// gu = [.., 2F] with gate in [0,F) and up in [F,2F) of each row; h = silu(gate)*up
template <typename T>
__global__ void __launch_bounds__(256)
swiglu_fwd_kernel(const T* __restrict__ gu, T* __restrict__ h, long long rows, int F) {
  ::msb::pdl_begin();
  const long long nvec = rows * (F >> 3);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / (F >> 3);
    const int c = (int)(i % (F >> 3)) << 3;
    float g[8], u[8], o[8];
    load8(gu + r * 2 * F + c, g);
    load8(gu + r * 2 * F + F + c, u);
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = (g[k] / (1.f + expf(-g[k]))) * u[k];
    store8(h + r * F + c, o);
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
swiglu_bwd_kernel(const T* __restrict__ dh, const T* __restrict__ gu, T* __restrict__ dgu,
                  long long rows, int F) {
  ::msb::pdl_begin();
  const long long nvec = rows * (F >> 3);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / (F >> 3);
    const int c = (int)(i % (F >> 3)) << 3;
    float d[8], g[8], u[8], dg[8], du[8];
    load8(dh + r * F + c, d);
    load8(gu + r * 2 * F + c, g);
    load8(gu + r * 2 * F + F + c, u);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float sg = 1.f / (1.f + expf(-g[k]));
      const float silu = g[k] * sg;
      du[k] = d[k] * silu;
      dg[k] = d[k] * u[k] * (sg * (1.f + g[k] * (1.f - sg)));
    }
    store8(dgu + r * 2 * F + c, dg);
    store8(dgu + r * 2 * F + F + c, du);
  }
}

// -------------------------------------------------------- cross entropy
// Walk one row of V elements starting at an arbitrary 2-byte address with
// 16-byte loads in the aligned middle.
template <typename T, typename F>
__device__ __forceinline__ void for_row(const T* row, int V, F&& f) {
  const int head = (int)(((16 - (reinterpret_cast<uintptr_t>(row) & 15)) & 15) / sizeof(T));
  const int h = min(head, V);
  for (int i = threadIdx.x; i < h; i += blockDim.x) f(i, to_f32(row[i]));
  const int nvec = (V - h) / 8;
  const T* mid = row + h;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float v[8];
    load8(mid + i * 8, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) f(h + i * 8 + k, v[k]);
  }
  for (int i = h + nvec * 8 + threadIdx.x; i < V; i += blockDim.x) f(i, to_f32(row[i]));
}

// running (max, sum) pairs in base-2 units: value y = x * log2(e)
__device__ __forceinline__ void softmax_merge(float& m, float& s, float m2, float s2) {
  const float mx = fmaxf(m, m2);
  if (mx == -INFINITY) return;
  s = s * ex2_approx(m - mx) + s2 * ex2_approx(m2 - mx);
  m = mx;
}

template <typename T>
__global__ void __launch_bounds__(512)
ce_fwd_kernel(const T* __restrict__ logits, const long long* __restrict__ tgt,
              float* __restrict__ lse_out, float* __restrict__ loss_rows, int V, long long ld,
              long long ignore_index) {
  ::msb::pdl_begin();
  const long long r = blockIdx.x;
  const T* row = logits + r * ld;
  float m = -INFINITY, s = 0.f;
  for_row(row, V, [&](int, float v) {
    const float y = v * kLog2e;
    if (y > m) {
      s = s * ex2_approx(m - y) + 1.f;
      m = y;
    } else {
      s += ex2_approx(y - m);
    }
  });
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    softmax_merge(m, s, m2, s2);
  }
  __shared__ float sm[32], ss[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    m = lane < nw ? sm[lane] : -INFINITY;
    s = lane < nw ? ss[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      softmax_merge(m, s, m2, s2);
    }
    if (lane == 0) {
      const float lse = m * kLn2 + logf(s);
      lse_out[r] = lse;
      const long long t = tgt[r];
      // ignored (or out-of-range) targets contribute nothing
      const bool valid = t != ignore_index && MSB_OK(t >= 0 && t < V, kSiteTarget, t, V);
      loss_rows[r] = valid ? lse - to_f32(row[t]) : 0.f;
    }
  }
}

// loss = sum(loss_rows) / count(valid); deterministic single block
__global__ void __launch_bounds__(1024)
ce_reduce_kernel(const float* __restrict__ loss_rows, const long long* __restrict__ tgt,
                 long long M, int V, long long ignore_index, float* __restrict__ out_loss,
                 float* __restrict__ out_inv_count) {
  ::msb::pdl_begin();
  double acc = 0.0;
  long long cnt = 0;
  for (long long i = threadIdx.x; i < M; i += blockDim.x) {
    acc += loss_rows[i];
    cnt += tgt[i] != ignore_index && tgt[i] >= 0 && tgt[i] < V;
  }
  __shared__ double sa[1024];
  __shared__ long long sc[1024];
  sa[threadIdx.x] = acc;
  sc[threadIdx.x] = cnt;
  __syncthreads();
  for (int w = 512; w > 0; w >>= 1) {
    if (threadIdx.x < w) {
      sa[threadIdx.x] += sa[threadIdx.x + w];
      sc[threadIdx.x] += sc[threadIdx.x + w];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const double c = sc[0] > 0 ? (double)sc[0] : 0.0;
    out_loss[0] = c > 0 ? (float)(sa[0] / c) : NAN;
    out_inv_count[0] = c > 0 ? (float)(1.0 / c) : 0.f;
  }
}

template <typename T>
__global__ void __launch_bounds__(512)
ce_bwd_kernel(T* __restrict__ logits, const long long* __restrict__ tgt,
              const float* __restrict__ lse, const float* __restrict__ grad_out,
              const float* __restrict__ inv_count, int V, long long ld, long long ignore_index) {
  ::msb::pdl_begin();
  const long long r = blockIdx.x;
  T* row = logits + r * ld;
  const long long t = tgt[r];
  const float scale =
      (t == ignore_index || t < 0 || t >= V) ? 0.f : grad_out[0] * inv_count[0];
  const float l = lse[r];
  const int head = (int)(((16 - (reinterpret_cast<uintptr_t>(row) & 15)) & 15) / sizeof(T));
  const int h = min(head, V);
  auto g = [&](int i, float v) {
    return (ex2_approx((v - l) * kLog2e) - (i == t ? 1.f : 0.f)) * scale;
  };
  for (int i = threadIdx.x; i < h; i += blockDim.x) row[i] = from_f32<T>(g(i, to_f32(row[i])));
  const int nvec = (V - h) / 8;
  T* mid = row + h;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float v[8];
    load8(mid + i * 8, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = g(h + i * 8 + k, v[k]);
    store8(mid + i * 8, v);
  }
  for (int i = h + nvec * 8 + threadIdx.x; i < V; i += blockDim.x)
    row[i] = from_f32<T>(g(i, to_f32(row[i])));
}

// inv_count[0] = 1 / (number of valid targets) (0 when there is none),
// before the fused forward that scales its gradient with it
__global__ void __launch_bounds__(1024)
ce_count_kernel(const long long* __restrict__ tgt, long long M, int V, long long ignore_index,
                float* __restrict__ out_inv_count) {
  ::msb::pdl_begin();
  long long cnt = 0;
  for (long long i = threadIdx.x; i < M; i += blockDim.x)
    cnt += tgt[i] != ignore_index && tgt[i] >= 0 && tgt[i] < V;
  __shared__ long long sc[1024];
  sc[threadIdx.x] = cnt;
  __syncthreads();
  for (int w = 512; w > 0; w >>= 1) {
    if (threadIdx.x < w) sc[threadIdx.x] += sc[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) out_inv_count[0] = sc[0] > 0 ? (float)(1.0 / (double)sc[0]) : 0.f;
}

// Forward and gradient of one row in one kernel: pass 1 is the online
// softmax of ce_fwd_kernel (lse, the row's loss); pass 2 overwrites the
// logits with their gradient for an expected upstream gradient g_hint (the
// loss-scale seed of backward):
//   dlogits[i] = (softmax[i] - [i == target]) * g_hint * inv_count.
// The row was just read, so pass 2 mostly hits L2: the logits cross DRAM
// once for reading and once for writing, against twice for reading when the
// gradient waits for backward.  Backward checks the real upstream gradient
// against g_hint (ce_grad_rescale_kernel).
template <typename T>
__global__ void __launch_bounds__(512)
ce_fwd_grad_kernel(T* __restrict__ logits, const long long* __restrict__ tgt,
                   float* __restrict__ lse_out, float* __restrict__ loss_rows, int V, long long ld,
                   long long ignore_index, const float* __restrict__ g_hint,
                   const float* __restrict__ inv_count) {
  ::msb::pdl_begin();
  const long long r = blockIdx.x;
  T* row = logits + r * ld;
  const int head = (int)(((16 - (reinterpret_cast<uintptr_t>(row) & 15)) & 15) / sizeof(T));
  const int h = min(head, V);
  const int nvec = (V - h) / 8;
  T* mid = row + h;
  // Pass 1: running (max, sum) in base-2 units.  The kernel is bound by
  // instruction issue, not by DRAM, so the middle of the row goes 8 values
  // at a time: one max and one rescale per vector, then one fma + ex2 + add
  // per value, without a data-dependent branch.
  float m = -INFINITY, s = 0.f;
  auto add1 = [&](float v) {
    const float y = v * kLog2e;
    const float mn = fmaxf(m, y);
    s = s * ex2_approx(m - mn) + ex2_approx(y - mn);
    m = mn;
  };
  for (int i = threadIdx.x; i < h; i += blockDim.x) add1(to_f32(row[i]));
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float v[8];
    load8(mid + i * 8, v);
    float mx = v[0];
#pragma unroll
    for (int k = 1; k < 8; ++k) mx = fmaxf(mx, v[k]);
    const float mn = fmaxf(m, mx * kLog2e);
    s *= ex2_approx(m - mn);   // m = -inf: 0 (s is 0 then)
    m = mn;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += ex2_approx(fmaf(v[k], kLog2e, -mn));
  }
  for (int i = h + nvec * 8 + threadIdx.x; i < V; i += blockDim.x) add1(to_f32(row[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    softmax_merge(m, s, m2, s2);
  }
  __shared__ float sm[32], ss[32];
  __shared__ float s_lse;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  const long long t = tgt[r];
  const bool valid = t != ignore_index && t >= 0 && t < V;
  if (threadIdx.x == 0 && t != ignore_index) (void)MSB_OK(t >= 0 && t < V, kSiteTarget, t, V);
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    m = lane < nw ? sm[lane] : -INFINITY;
    s = lane < nw ? ss[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      softmax_merge(m, s, m2, s2);
    }
    if (lane == 0) {
      const float lse = m * kLn2 + logf(s);
      lse_out[r] = lse;
      loss_rows[r] = valid ? lse - to_f32(row[t]) : 0.f;
      s_lse = lse;
    }
  }
  __syncthreads();   // every thread has read the row before it is overwritten
  // Pass 2: dlogits[i] = softmax[i] * scale (- scale at the target), with the
  // scale folded into the exponent: 2^(v log2 e - lse log2 e + log2 scale).
  // scale = 0 (an ignored target) gives -inf there and zeros.
  const float scale = valid ? g_hint[0] * inv_count[0] : 0.f;
  const float base = (scale > 0.f ? log2f(scale) : -INFINITY) - s_lse * kLog2e;
  auto g1 = [&](int i, float v) {
    return ex2_approx(fmaf(v, kLog2e, base)) - (i == t ? scale : 0.f);
  };
  for (int i = threadIdx.x; i < h; i += blockDim.x) row[i] = from_f32<T>(g1(i, to_f32(row[i])));
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float v[8];
    load8(mid + i * 8, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = ex2_approx(fmaf(v[k], kLog2e, base));
    const long long kt = t - (h + (long long)i * 8);   // the target inside this vector?
    if (kt >= 0 && kt < 8) {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k == kt) v[k] -= scale;
    }
    store8(mid + i * 8, v);
  }
  for (int i = h + nvec * 8 + threadIdx.x; i < V; i += blockDim.x)
    row[i] = from_f32<T>(g1(i, to_f32(row[i])));
}

// Backward of the fused forward: the stored gradient assumed the upstream
// gradient g_hint; when the real one differs (a loss that was rescaled
// before backward), multiply by grad_out / g_hint.  Otherwise every block
// returns after reading two scalars.
template <typename T>
__global__ void __launch_bounds__(256)
ce_grad_rescale_kernel(T* __restrict__ dlogits, long long M, int V, long long ld,
                       const float* __restrict__ grad_out, const float* __restrict__ g_hint) {
  ::msb::pdl_begin();
  const float go = grad_out[0], gh = g_hint[0];
  if (go == gh) return;
  const float f = gh != 0.f ? go / gh : 0.f;
  for (long long r = blockIdx.x; r < M; r += gridDim.x) {
    T* row = dlogits + r * ld;
    for (int i = threadIdx.x; i < V; i += blockDim.x) row[i] = from_f32<T>(to_f32(row[i]) * f);
  }
}

// ------------------------------------------------------------ embedding
template <typename T>
__global__ void __launch_bounds__(256)
embedding_fwd_kernel(const long long* __restrict__ idx, const T* __restrict__ wte,
                     const T* __restrict__ wpe, T* __restrict__ out, long long M, int T_len,
                     int C, long long V) {
  ::msb::pdl_begin();
  const int nvec = C >> 3;
  const long long total = M * nvec;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / nvec;
    const int c = (int)(i % nvec) << 3;
    const long long tok = idx[m];
    float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (c == 0) (void)MSB_OK(tok >= 0 && tok < V, kSiteEmbeddingToken, tok, V);
    if (tok >= 0 && tok < V) load8(wte + tok * C + c, a);
    if (wpe != nullptr) {
      float b[8];
      load8(wpe + (long long)(m % T_len) * C + c, b);
#pragma unroll
      for (int k = 0; k < 8; ++k) a[k] += b[k];
    }
    store8(out + m * C + c, a);
  }
}

// Token-embedding gradient, pass 1: scatter-add every row of dout into the
// fp32 accumulator row of its token (atomics) and mark the row as touched.
// The accumulator and the flags persist between steps and are all zero on
// entry: pass 2 returns every row it reads to zero.
template <typename T>
__global__ void __launch_bounds__(256)
embedding_bwd_tok_kernel(const T* __restrict__ dout, const long long* __restrict__ idx,
                         float* __restrict__ acc, unsigned char* __restrict__ touched,
                         long long M, int C, long long V) {
  ::msb::pdl_begin();
  const int nvec = C >> 3;
  const long long total = M * nvec;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / nvec;
    const int c = (int)(i % nvec) << 3;
    const long long tok = idx[m];
    if (tok < 0 || tok >= V) {
      if (c == 0) (void)MSB_OK(false, kSiteEmbeddingToken, tok, V);
      continue;
    }
    float a[8];
    load8(dout + m * C + c, a);
    float* te = acc + tok * C + c;
#pragma unroll
    for (int k = 0; k < 8; ++k) atomicAdd(te + k, a[k]);
    if (c == 0) touched[tok] = 1;
  }
}

// Pass 2: one warp per vocabulary row; a touched row is added into the
// gradient (model dtype, accumulating into what the head GEMM already put
// there) and its accumulator row and flag are cleared.  Untouched rows cost
// one byte read.
template <typename T>
__global__ void __launch_bounds__(256)
embedding_bwd_finish_kernel(float* __restrict__ acc, unsigned char* __restrict__ touched,
                            T* __restrict__ grad, long long V, int C, int accumulate) {
  ::msb::pdl_begin();
  const int lane = threadIdx.x & 31;
  for (long long t = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); t < V;
       t += (long long)gridDim.x * 8) {
    if (!touched[t]) continue;
    float* row = acc + t * C;
    T* g = grad + t * C;
    for (int c = lane * 8; c < C; c += 256) {
      float a[8], o[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        a[k] = row[c + k];
        row[c + k] = 0.f;
      }
      if (accumulate) {
        load8(g + c, o);
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] += a[k];
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = a[k];
      }
      store8(g + c, o);
    }
    __syncwarp();
    if (lane == 0) touched[t] = 0;
  }
}

// Position-embedding gradient: grad[p] (+)= sum over b of dout[b * T + p], in
// batch order (deterministic, no atomics); one thread per 8 columns of a row.
template <typename T>
__global__ void __launch_bounds__(256)
embedding_bwd_pos_kernel(const T* __restrict__ dout, T* __restrict__ grad, long long M,
                         int T_len, int C, int accumulate) {
  ::msb::pdl_begin();
  const int nvec = C >> 3;
  const long long total = (long long)T_len * nvec;
  const long long B = M / T_len;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long p = i / nvec;
    const int c = (int)(i % nvec) << 3;
    float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (long long b = 0; b < B; ++b) {
      float a[8];
      load8(dout + (b * T_len + p) * C + c, a);
#pragma unroll
      for (int k = 0; k < 8; ++k) s[k] += a[k];
    }
    if (accumulate) {
      float o[8];
      load8(grad + p * C + c, o);
#pragma unroll
      for (int k = 0; k < 8; ++k) s[k] += o[k];
    }
    store8(grad + p * C + c, s);
  }
}

// ----------------------------------------------------------------- RoPE
// x: [B, T, H, D] viewed with row stride `row_stride` elements between
// consecutive (b, t); rotates pairs (i, i + D/2) (the "rotate_half" form).
template <typename T>
__global__ void __launch_bounds__(256)
rope_kernel(T* __restrict__ x, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
            long long BT, int T_len, int H, int D, long long row_stride, int inverse) {
  ::msb::pdl_begin();
  const int half = D >> 1;
  const long long total = BT * H * half;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int j = (int)(i % half);
    const long long hb = i / half;
    const int h = (int)(hb % H);
    const long long bt = hb / H;
    const int t = (int)(bt % T_len);
    T* p = x + bt * row_stride + (long long)h * D;
    const float c = cos_t[(size_t)t * half + j];
    const float s = inverse ? -sin_t[(size_t)t * half + j] : sin_t[(size_t)t * half + j];
    const float a = to_f32(p[j]), b = to_f32(p[j + half]);
    p[j] = from_f32<T>(a * c - b * s);
    p[j + half] = from_f32<T>(b * c + a * s);
  }
}

}  // namespace

// =============================================================== host API
// Blocks of `kernel` resident on the whole GPU at once (its registers and
// shared memory per block); a row-looping kernel launches that many.
template <typename K>
static int resident_blocks(K kernel, int threads, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, size_t>, int> cache;
  const auto key = std::make_tuple(reinterpret_cast<const void*>(kernel), threads, smem);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int per_sm = 0;
  check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem),
             "occupancy");
  return cache[key] = std::max(1, per_sm) * kNumSMs;
}

template <typename T, int NVV>
static void launch_norm_fwd(const void* x, const void* delta, const void* w, const void* b,
                            void* s_out, void* y, float* mean, float* rstd, int M, int C,
                            float eps, bool rms, int blocks, cudaStream_t st) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if constexpr (NVV <= 8 && !std::is_same<T, float>::value) {
    if (C % 8 == 0 && al(x) && al(y) && (delta == nullptr || al(delta)) &&
        (s_out == nullptr || al(s_out))) {
      // as many blocks of 8 warps as are resident at once, each looping
      // over groups of 8 rows
      const size_t smem = (rms ? 1 : 2) * (size_t)C * sizeof(float);
      auto kern = rms ? add_norm_fwd_rows_kernel<T, NVV, true>
                      : add_norm_fwd_rows_kernel<T, NVV, false>;
      const int grid = std::min(blocks, resident_blocks(kern, 256, smem));
      ::msb::launch(kern, grid, 256, smem, st, (const T*)x, (const T*)delta, (const T*)w,
                    (const T*)b, (T*)s_out, (T*)y, mean, rstd, M, C, eps);
      return;
    }
  }
  if (rms)
    ::msb::launch(add_norm_fwd_kernel<T, NVV, true>, blocks, 256, 0, st, 
        (const T*)x, (const T*)delta, (const T*)w, (const T*)b, (T*)s_out, (T*)y, mean, rstd, M,
        C, eps);
  else
    ::msb::launch(add_norm_fwd_kernel<T, NVV, false>, blocks, 256, 0, st, 
        (const T*)x, (const T*)delta, (const T*)w, (const T*)b, (T*)s_out, (T*)y, mean, rstd, M,
        C, eps);
}

void add_norm_fwd(const void* x, const void* delta, const void* w, const void* b, void* s_out,
                  void* y, float* mean, float* rstd, int M, int C, float eps, bool rms,
                  int dtype, cudaStream_t st) {
  const int nv = (C / 8 + 31) / 32;
  const int blocks = (M + 7) / 8;
  MSB_DISPATCH_FLOAT(dtype, T, {
    if (nv <= 1) launch_norm_fwd<T, 1>(x, delta, w, b, s_out, y, mean, rstd, M, C, eps, rms, blocks, st);
    else if (nv <= 2) launch_norm_fwd<T, 2>(x, delta, w, b, s_out, y, mean, rstd, M, C, eps, rms, blocks, st);
    else if (nv <= 3) launch_norm_fwd<T, 3>(x, delta, w, b, s_out, y, mean, rstd, M, C, eps, rms, blocks, st);
    else if (nv <= 4) launch_norm_fwd<T, 4>(x, delta, w, b, s_out, y, mean, rstd, M, C, eps, rms, blocks, st);
    else if (nv <= 8) launch_norm_fwd<T, 8>(x, delta, w, b, s_out, y, mean, rstd, M, C, eps, rms, blocks, st);
    else if (nv <= 16) launch_norm_fwd<T, 16>(x, delta, w, b, s_out, y, mean, rstd, M, C, eps, rms, blocks, st);
    else throw std::runtime_error("norm: hidden size too large");
  });
  MSB_CHECK_LAUNCH("add_norm_fwd");
}

template <typename T, int NVV>
static void launch_norm_dx(const void* dy, const void* s, const void* w, const float* mean,
                           const float* rstd, const void* dres, void* dx, int M, int C, bool rms,
                           cudaStream_t st) {
  const int blocks = grid_for((M + 7) / 8, 1, kNumSMs * 16);
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if constexpr (NVV <= 8 && !std::is_same<T, float>::value) {
    if (C % 8 == 0 && al(dy) && al(s) && al(dx) && (dres == nullptr || al(dres))) {
      // as many blocks of 4 warps as are resident at once, each looping
      // over groups of 4 rows
      const size_t smem = (size_t)C * sizeof(float);
      auto kern = rms ? norm_dx_prefetch_kernel<T, NVV, true> : norm_dx_prefetch_kernel<T, NVV, false>;
      const int grid = std::min((M + 3) / 4, resident_blocks(kern, 128, smem));
      ::msb::launch(kern, grid, 128, smem, st, (const T*)dy, (const T*)s, (const T*)w, mean, rstd,
                    (const T*)dres, (T*)dx, M, C);
      return;
    }
  }
  if (rms)
    ::msb::launch(norm_dx_kernel<T, NVV, true>, blocks, 256, 0, st, (const T*)dy, (const T*)s, (const T*)w,
                                                          mean, rstd, (const T*)dres, (T*)dx, M, C);
  else
    ::msb::launch(norm_dx_kernel<T, NVV, false>, blocks, 256, 0, st, (const T*)dy, (const T*)s, (const T*)w,
                                                           mean, rstd, (const T*)dres, (T*)dx, M,
                                                           C);
}

template <typename T, int NVV>
static bool launch_norm_fused(const void* dy, const void* s, const void* w, const float* mean,
                              const float* rstd, const void* dres, void* dx, float* dw_part,
                              float* db_part, int M, int C, bool rms, int blocks,
                              cudaStream_t st) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  // the accumulators take 16 registers per vector group: up to 1024 columns
  // the kernel stays without spills
  if constexpr (NVV <= 4) {
    if (C % 8 == 0 && al(dy) && al(s) && al(dx) && (dres == nullptr || al(dres))) {
      if (rms)
        ::msb::launch(norm_bwd_fused_kernel<T, NVV, true>, blocks, 256, 0, st, (const T*)dy,
                      (const T*)s, (const T*)w, mean, rstd, (const T*)dres, (T*)dx, dw_part,
                      (float*)nullptr, M, C);
      else
        ::msb::launch(norm_bwd_fused_kernel<T, NVV, false>, blocks, 256, 0, st, (const T*)dy,
                      (const T*)s, (const T*)w, mean, rstd, (const T*)dres, (T*)dx, dw_part,
                      db_part, M, C);
      return true;
    }
  }
  return false;
}

int norm_bwd(const void* dy, const void* s, const void* w, const float* mean, const float* rstd,
             const void* dres, void* dx, float* dw_part, float* db_part, int M, int C, bool rms,
             int dtype, int max_blocks, cudaStream_t st) {
  const int nv = (C / 8 + 31) / 32;
  // one pass (dx and the dw/db partials) when the rows allow 16-byte access
  const int fused_blocks = std::max(1, std::min({max_blocks, 2 * kNumSMs, (M + 7) / 8}));
  bool fused = false;
  MSB_DISPATCH_FLOAT(dtype, T, {
    if (nv <= 1) fused = launch_norm_fused<T, 1>(dy, s, w, mean, rstd, dres, dx, dw_part, db_part, M, C, rms, fused_blocks, st);
    else if (nv <= 2) fused = launch_norm_fused<T, 2>(dy, s, w, mean, rstd, dres, dx, dw_part, db_part, M, C, rms, fused_blocks, st);
    else if (nv <= 3) fused = launch_norm_fused<T, 3>(dy, s, w, mean, rstd, dres, dx, dw_part, db_part, M, C, rms, fused_blocks, st);
    else if (nv <= 4) fused = launch_norm_fused<T, 4>(dy, s, w, mean, rstd, dres, dx, dw_part, db_part, M, C, rms, fused_blocks, st);
  });
  if (fused) {
    MSB_CHECK_LAUNCH("norm_bwd_fused");
    return fused_blocks;
  }
  int chunks = std::min(max_blocks, std::max(1, (M + 63) / 64));
  const int rpb = (M + chunks - 1) / chunks;
  chunks = (M + rpb - 1) / rpb;
  dim3 grid((C + 255) / 256, chunks);
  MSB_DISPATCH_FLOAT(dtype, T, {
    if (nv <= 1) launch_norm_dx<T, 1>(dy, s, w, mean, rstd, dres, dx, M, C, rms, st);
    else if (nv <= 2) launch_norm_dx<T, 2>(dy, s, w, mean, rstd, dres, dx, M, C, rms, st);
    else if (nv <= 3) launch_norm_dx<T, 3>(dy, s, w, mean, rstd, dres, dx, M, C, rms, st);
    else if (nv <= 4) launch_norm_dx<T, 4>(dy, s, w, mean, rstd, dres, dx, M, C, rms, st);
    else if (nv <= 8) launch_norm_dx<T, 8>(dy, s, w, mean, rstd, dres, dx, M, C, rms, st);
    else if (nv <= 16) launch_norm_dx<T, 16>(dy, s, w, mean, rstd, dres, dx, M, C, rms, st);
    else throw std::runtime_error("norm_bwd: hidden size too large");
    MSB_CHECK_LAUNCH("norm_dx");
    if (rms)
      ::msb::launch(norm_dwdb_partial_kernel<T, true>, grid, 256, 0, st, (const T*)dy, (const T*)s, mean,
                                                             rstd, dw_part, nullptr, M, C, rpb);
    else
      ::msb::launch(norm_dwdb_partial_kernel<T, false>, grid, 256, 0, st, (const T*)dy, (const T*)s, mean,
                                                              rstd, dw_part, db_part, M, C, rpb);
  });
  MSB_CHECK_LAUNCH("norm_dwdb_partial");
  return chunks;
}

int colsum_partial(const void* a, float* part, int M, int N, long long ld, int dtype,
                   int max_chunks, cudaStream_t st) {
  int chunks = min(max_chunks, max(1, (M + 63) / 64));
  const int rpb = (M + chunks - 1) / chunks;
  chunks = (M + rpb - 1) / rpb;
  dim3 grid((N + 255) / 256, chunks);
  MSB_DISPATCH_FLOAT(dtype, T, {
    ::msb::launch(colsum_partial_kernel<T>, grid, 256, 0, st, (const T*)a, part, M, N, ld, rpb);
  });
  MSB_CHECK_LAUNCH("colsum_partial");
  return chunks;
}

void colsum_finish(const float* part, int nparts, int N, void* out, int dtype, int accumulate,
                   cudaStream_t st) {
  MSB_DISPATCH_FLOAT(dtype, T, {
    ::msb::launch(colsum_finish_kernel<T>, (N + 31) / 32, 256, 0, st, part, nparts, N, (T*)out, accumulate);
  });
  MSB_CHECK_LAUNCH("colsum_finish");
}

void colsum_finish_many(const ColsumJob* jobs, int njobs, int dtype, cudaStream_t st) {
  for (int j0 = 0; j0 < njobs; j0 += kMaxColsumJobs) {
    ColsumBatch b;
    b.njobs = std::min(kMaxColsumJobs, njobs - j0);
    int blocks = 0;
    for (int j = 0; j < b.njobs; ++j) {
      b.job[j] = jobs[j0 + j];
      b.first[j] = blocks;
      blocks += (jobs[j0 + j].N + 31) / 32;
    }
    b.first[b.njobs] = blocks;
    if (blocks == 0) continue;
    MSB_DISPATCH_FLOAT(dtype, T, {
      ::msb::launch(colsum_finish_many_kernel<T>, blocks, 256, 0, st, b);
    });
    MSB_CHECK_LAUNCH("colsum_finish_many");
  }
}

void accum_cast(const float* src, void* dst, long long n, int dtype, int accumulate,
                cudaStream_t st) {
  const int blocks = grid_for(n, 256, kNumSMs * 16);
  MSB_DISPATCH_FLOAT(dtype, T, {
    ::msb::launch(accum_cast_kernel<T>, blocks, 256, 0, st, src, (T*)dst, n, accumulate);
  });
  MSB_CHECK_LAUNCH("accum_cast");
}

void bias_gelu_fwd(void* u, const void* bias, void* h, long long total, int N, int dtype,
                   cudaStream_t st) {
  const int blocks = grid_for(total / 8, 256, kNumSMs * 16);
  MSB_DISPATCH_FLOAT(dtype, T, {
    ::msb::launch(bias_gelu_fwd_kernel<T>, blocks, 256, 0, st, (T*)u, (const T*)bias, (T*)h, total, N);
  });
  MSB_CHECK_LAUNCH("bias_gelu_fwd");
}

void gelu_bwd(const void* dh, const void* u, void* du, long long total, int dtype,
              cudaStream_t st) {
  const int blocks = grid_for(total / 8, 256, kNumSMs * 16);
  MSB_DISPATCH_FLOAT(dtype, T, {
    ::msb::launch(gelu_bwd_kernel<T>, blocks, 256, 0, st, (const T*)dh, (const T*)u, (T*)du, total);
  });
  MSB_CHECK_LAUNCH("gelu_bwd");
}

void swiglu_fwd(const void* gu, void* h, long long rows, int F, int dtype, cudaStream_t st) {
  const int blocks = grid_for(rows * (F / 8), 256, kNumSMs * 16);
  MSB_DISPATCH_FLOAT(dtype, T, {
    ::msb::launch(swiglu_fwd_kernel<T>, blocks, 256, 0, st, (const T*)gu, (T*)h, rows, F);
  });
  MSB_CHECK_LAUNCH("swiglu_fwd");
}

void swiglu_bwd(const void* dh, const void* gu, void* dgu, long long rows, int F, int dtype,
                cudaStream_t st) {
  const int blocks = grid_for(rows * (F / 8), 256, kNumSMs * 16);
  MSB_DISPATCH_FLOAT(dtype, T, {
    ::msb::launch(swiglu_bwd_kernel<T>, blocks, 256, 0, st, (const T*)dh, (const T*)gu, (T*)dgu, rows, F);
  });
  MSB_CHECK_LAUNCH("swiglu_bwd");
}

void cross_entropy_fwd(const void* logits, const long long* tgt, float* lse, float* loss_rows,
                       float* loss, float* inv_count, long long M, int V, long long ld,
                       long long ignore_index, int dtype, cudaStream_t st) {
  MSB_DISPATCH_FLOAT(dtype, T, {
    ::msb::launch(ce_fwd_kernel<T>, (unsigned)M, 512, 0, st, (const T*)logits, tgt, lse, loss_rows, V, ld,
                                                 ignore_index);
  });
  MSB_CHECK_LAUNCH("ce_fwd");
  ::msb::launch(ce_reduce_kernel, 1, 1024, 0, st, loss_rows, tgt, M, V, ignore_index, loss, inv_count);
  MSB_CHECK_LAUNCH("ce_reduce");
}

void cross_entropy_bwd(void* logits, const long long* tgt, const float* lse,
                       const float* grad_out, const float* inv_count, long long M, int V,
                       long long ld, long long ignore_index, int dtype, cudaStream_t st) {
  MSB_DISPATCH_FLOAT(dtype, T, {
    ::msb::launch(ce_bwd_kernel<T>, (unsigned)M, 512, 0, st, (T*)logits, tgt, lse, grad_out, inv_count, V,
                                                 ld, ignore_index);
  });
  MSB_CHECK_LAUNCH("ce_bwd");
}

void cross_entropy_fwd_grad(void* logits, const long long* tgt, float* lse, float* loss_rows,
                            float* loss, float* inv_count, const float* g_hint, long long M, int V,
                            long long ld, long long ignore_index, int dtype, cudaStream_t st) {
  ::msb::launch(ce_count_kernel, 1, 1024, 0, st, tgt, M, V, ignore_index, inv_count);
  MSB_DISPATCH_FLOAT(dtype, T, {
    ::msb::launch(ce_fwd_grad_kernel<T>, (unsigned)M, 512, 0, st, (T*)logits, tgt, lse,
                  loss_rows, V, ld, ignore_index, g_hint, (const float*)inv_count);
  });
  ::msb::launch(ce_reduce_kernel, 1, 1024, 0, st, (const float*)loss_rows, tgt, M, V,
                ignore_index, loss, inv_count);
  MSB_CHECK_LAUNCH("ce_fwd_grad");
}

void cross_entropy_grad_rescale(void* dlogits, long long M, int V, long long ld,
                                const float* grad_out, const float* g_hint, int dtype,
                                cudaStream_t st) {
  MSB_DISPATCH_FLOAT(dtype, T, {
    ::msb::launch(ce_grad_rescale_kernel<T>, grid_for(M, 1, kNumSMs * 8), 256, 0, st, (T*)dlogits,
                  M, V, ld, grad_out, g_hint);
  });
  MSB_CHECK_LAUNCH("ce_grad_rescale");
}

void embedding_fwd(const long long* idx, const void* wte, const void* wpe, void* out, long long M,
                   int T_len, int C, long long V, int dtype, cudaStream_t st) {
  const int blocks = grid_for(M * (C / 8), 256, kNumSMs * 16);
  MSB_DISPATCH_FLOAT(dtype, T, {
    ::msb::launch(embedding_fwd_kernel<T>, blocks, 256, 0, st, idx, (const T*)wte, (const T*)wpe, (T*)out,
                                                    M, T_len, C, V);
  });
  MSB_CHECK_LAUNCH("embedding_fwd");
}

void embedding_bwd(const void* dout, const long long* idx, float* acc, unsigned char* touched,
                   void* dwte, int acc_wte, void* dwpe, int acc_wpe, long long M, int T_len,
                   int C, long long V, int dtype, cudaStream_t st) {
  MSB_DISPATCH_FLOAT(dtype, T, {
    ::msb::launch(embedding_bwd_tok_kernel<T>, grid_for(M * (C / 8), 256, kNumSMs * 16), 256, 0, st, 
        (const T*)dout, idx, acc, touched, M, C, V);
    ::msb::launch(embedding_bwd_finish_kernel<T>, grid_for(V, 8, kNumSMs * 16), 256, 0, st, 
        acc, touched, (T*)dwte, V, C, acc_wte);
    if (dwpe != nullptr)
      ::msb::launch(embedding_bwd_pos_kernel<T>, grid_for((long long)T_len * (C / 8), 256, kNumSMs * 8), 256, 0, st, (const T*)dout, (T*)dwpe, M, T_len, C, acc_wpe);
  });
  MSB_CHECK_LAUNCH("embedding_bwd");
}

void rope(void* x, const float* cos_t, const float* sin_t, long long BT, int T_len, int H, int D,
          long long row_stride, bool inverse, int dtype, cudaStream_t st) {
  const int blocks = grid_for(BT * H * (D / 2), 256, kNumSMs * 16);
  MSB_DISPATCH_FLOAT(dtype, T, {
    ::msb::launch(rope_kernel<T>, blocks, 256, 0, st, (T*)x, cos_t, sin_t, BT, T_len, H, D, row_stride,
                                           inverse ? 1 : 0);
  });
  MSB_CHECK_LAUNCH("rope");
}

MSB_BOUNDS_TU(nn)

}  // namespace msb
