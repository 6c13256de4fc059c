// Persistent warp-specialized GEMM for sm_100a on the 5th-generation tensor
// cores (tcgen05 + tensor memory).
//
//   C[M,N] (+)= A[M,K] * B[N,K]^T (+ bias[N]),  fp16/bf16 in, fp32 accumulate
//
// Operands may be K-major (K contiguous) or MN-major (M resp. N contiguous),
// which covers the three products of a linear layer without transposes:
// forward (both K-major), dgrad (B MN-major) and wgrad (both MN-major).
//
// CTA = 6 warps, one CTA per SM, persistent over output tiles (128 x BN):
//   warp 0     TMA producer: 64-deep K slices of A and B into a 4-stage
//              shared-memory ring (128-byte swizzle), one mbarrier per stage
//   warp 1     owns the tensor memory (allocates 2 x BN fp32 columns) and
//              issues tcgen05.mma (M=128, N=BN, K=16) from one thread;
//              tcgen05.commit frees a ring stage once its MMAs retire and
//              signals "accumulator full" after a tile's last K slice
//   warps 2-5  epilogue: tcgen05.ld 32 columns at a time (one TMEM lane =
//              one output row per thread), bias, cast, store; release the
//              accumulator buffer so the MMA warp can start the tile after
//              next while this one drains (double-buffered accumulators)
//
// Split-K (for wgrad products whose output has too few tiles to fill 148
// SMs) writes fp32 partial tiles to a workspace reduced by a second kernel.
//
// Every mbarrier wait is bounded (globaltimer): past the limit the kernel
// records an error code, raises a CTA-wide abort flag that every role polls,
// waits (bounded) for its TMA loads and MMAs in flight, frees its tensor
// memory and returns.  The host reads the error word.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <string>

#include "common.cuh"

namespace msb {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 x 16-bit = 128 bytes = one swizzle row
constexpr int STAGES = 4;
constexpr int kThreads = 192;

struct Params {
  int M, N, K;
  int kb_total;      // ceil(K / BK)
  int kb_per_split;  // K slices per split
  int splits;
  int tiles_m, tiles_n, units;
  void* C;
  long long ldc;
  const void* bias;
  float* ws;         // [splits][M][N] fp32 when splits > 1
  int a_mn, b_mn;    // 1 = MN-major operand
  int accumulate;    // C += result
  uint32_t idesc;
  unsigned* err;
  unsigned long long timeout_ns;
};

// ---------------------------------------------------------------- PTX
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t gtime() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor (tcgen05 "UMMA" form): start address,
// leading / stride byte offsets (16-byte units), version 1, 128-byte swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// Operand tile of ROWS x BK at `base` (1024-byte aligned) as written by TMA:
//   K-major : ROWS rows of 128 B (8-row swizzle atoms of 1024 B); the k-th
//             16-element step starts 32 B further into each row.
//   MN-major: ROWS/64 chunks of [BK K-rows x 128 B]; chunks are 8 KB apart
//             (leading offset), 8-row K groups 1024 B apart (stride offset);
//             the k-th 16-row step starts 2048 B further.
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int mn_major, int kstep) {
  if (mn_major) return smem_desc(base + kstep * 2048, BK * 128, 1024);
  return smem_desc(base + kstep * 32, 16, 1024);
}

struct alignas(8) Barriers {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

// Bounded wait: returns false when the CTA aborted or the limit passed.
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, volatile int* abort,
                                         const Params& p, unsigned code) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = gtime();
  while (true) {
    if (mbar_try(bar, parity)) return true;
    if (*abort) return false;
    if (gtime() - t0 > p.timeout_ns) {
      *abort = 1;
      atomicCAS(p.err, 0u, code);
      return false;
    }
  }
}

template <int BN>
__device__ __forceinline__ void unit_coords(const Params& p, int u, int& m0, int& n0, int& kb0,
                                            int& kb1, int& split) {
  const int tiles = p.tiles_m * p.tiles_n;
  split = u / tiles;
  const int t = u - split * tiles;
  m0 = (t % p.tiles_m) * BM;
  n0 = (t / p.tiles_m) * BN;
  kb0 = split * p.kb_per_split;
  kb1 = min(p.kb_total, kb0 + p.kb_per_split);
}

template <typename T>
__device__ __forceinline__ void store_row_chunk(const Params& p, int row, int col, const float* v,
                                                int nvalid) {
  T* c = static_cast<T*>(p.C) + (long long)row * p.ldc + col;
  const T* bias = static_cast<const T*>(p.bias);
  float o[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    float x = v[j];
    if (bias != nullptr && j < nvalid) x += to_f32(bias[col + j]);
    o[j] = x;
  }
  const bool vec = nvalid == 32 && (reinterpret_cast<uintptr_t>(c) & 15) == 0;
  if (vec) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 pack;
      T* h = reinterpret_cast<T*>(&pack);
      if (p.accumulate) {
        uint4 old = *reinterpret_cast<const uint4*>(c + q * 8);
        const T* oh = reinterpret_cast<const T*>(&old);
#pragma unroll
        for (int j = 0; j < 8; ++j) h[j] = from_f32<T>(o[q * 8 + j] + to_f32(oh[j]));
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) h[j] = from_f32<T>(o[q * 8 + j]);
      }
      *reinterpret_cast<uint4*>(c + q * 8) = pack;
    }
  } else {
    for (int j = 0; j < nvalid; ++j) {
      float x = o[j];
      if (p.accumulate) x += to_f32(c[j]);
      c[j] = from_f32<T>(x);
    }
  }
}

template <typename T, int BN>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const Params p) {
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int B_BYTES = BN * BK * 2;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  Barriers* bars = reinterpret_cast<Barriers*>(sB + STAGES * B_BYTES);
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&bars->full[s]), 1);
      mbar_init(smem_u32(&bars->empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&bars->tfull[b]), 1);
      mbar_init(smem_u32(&bars->tempty[b]), 4);
    }
    mbar_init(smem_u32(&bars->drain), 1);
    bars->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&bars->tmem_base), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------ TMA producer
    int stage = 0;
    uint32_t phase = 0;
    int pending[STAGES];
#pragma unroll
    for (int s = 0; s < STAGES; ++s) pending[s] = -1;
    bool ok = true;
    for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
      int m0, n0, kb0, kb1, split;
      unit_coords<BN>(p, u, m0, n0, kb0, kb1, split);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!wait_bar(smem_u32(&bars->empty[stage]), phase ^ 1, abort, p, 1)) {
          ok = false;
          break;
        }
        const uint32_t full = smem_u32(&bars->full[stage]);
        mbar_expect_tx(full, A_BYTES + B_BYTES);
        const uint32_t a_dst = smem_u32(sA + stage * A_BYTES);
        const uint32_t b_dst = smem_u32(sB + stage * B_BYTES);
        const int k0 = kb * BK;
        if (p.a_mn) {
#pragma unroll
          for (int j = 0; j < BM / 64; ++j) tma_load_2d(a_dst + j * 8192, &tmA, full, m0 + 64 * j, k0);
        } else {
          tma_load_2d(a_dst, &tmA, full, k0, m0);
        }
        if (p.b_mn) {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * 8192, &tmB, full, n0 + 64 * j, k0);
        } else {
          tma_load_2d(b_dst, &tmB, full, k0, n0);
        }
        pending[stage] = static_cast<int>(phase);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    // loads still landing must finish before the CTA may exit
    for (int s = 0; s < STAGES; ++s) {
      if (pending[s] < 0) continue;
      const uint32_t bar = smem_u32(&bars->full[s]);
      const uint64_t t0 = gtime();
      while (!mbar_try(bar, static_cast<uint32_t>(pending[s])) &&
             gtime() - t0 < p.timeout_ns) {
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------- MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++it) {
      int m0, n0, kb0, kb1, split;
      unit_coords<BN>(p, u, m0, n0, kb0, kb1, split);
      const int buf = it & 1;
      const uint32_t tphase = (it >> 1) & 1;
      if (!wait_bar(smem_u32(&bars->tempty[buf]), tphase ^ 1, abort, p, 2)) break;
      tc_fence_after();
      const uint32_t d = tmem_base + buf * BN;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!wait_bar(smem_u32(&bars->full[stage]), phase, abort, p, 3)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA + stage * A_BYTES);
        const uint32_t b_base = smem_u32(sB + stage * B_BYTES);
#pragma unroll
        for (int ks = 0; ks < BK / 16; ++ks) {
          umma_f16(d, operand_desc(a_base, p.a_mn, ks), operand_desc(b_base, p.b_mn, ks), p.idesc,
                   (kb > kb0 || ks > 0) ? 1u : 0u);
        }
        umma_commit(smem_u32(&bars->empty[stage]));
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (ok) umma_commit(smem_u32(&bars->tfull[buf]));
    }
    // every MMA issued by this thread retires before tensor memory is freed
    umma_commit(smem_u32(&bars->drain));
    const uint64_t t0 = gtime();
    while (!mbar_try(smem_u32(&bars->drain), 0) && gtime() - t0 < p.timeout_ns) {
    }
  } else if (warp >= 2) {
    // ---------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int row_in_tile = quarter * 32 + lane;
    int it = 0;
    for (int u = blockIdx.x; u < p.units; u += gridDim.x, ++it) {
      int m0, n0, kb0, kb1, split;
      unit_coords<BN>(p, u, m0, n0, kb0, kb1, split);
      const int buf = it & 1;
      const uint32_t tphase = (it >> 1) & 1;
      // one lane polls; the warp follows it as a unit (tcgen05.ld is .sync.aligned)
      int ok = lane == 0 ? (wait_bar(smem_u32(&bars->tfull[buf]), tphase, abort, p, 4) ? 1 : 0) : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const int row = m0 + row_in_tile;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_base + ((quarter * 32) << 16) + buf * BN + c * 32, r);
        tmem_ld_wait();
        const int col = n0 + c * 32;
        if (row < p.M && col < p.N) {
          const int nvalid = min(32, p.N - col);
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          if (p.splits > 1) {
            float* w = p.ws + ((long long)split * p.M + row) * p.N + col;
            if (nvalid == 32 && (reinterpret_cast<uintptr_t>(w) & 15) == 0) {
#pragma unroll
              for (int q = 0; q < 8; ++q)
                reinterpret_cast<float4*>(w)[q] =
                    make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
            } else {
              for (int j = 0; j < nvalid; ++j) w[j] = v[j];
            }
          } else {
            store_row_chunk<T>(p, row, col, v, nvalid);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars->tempty[buf]));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// C = sum_s ws[s] (+ bias) (+ C)
template <typename T>
__global__ void __launch_bounds__(256)
splitk_reduce_kernel(const float* __restrict__ ws, int splits, int M, int N, T* __restrict__ C,
                     long long ldc, const T* __restrict__ bias, int accumulate) {
  const long long total = (long long)M * N;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(i / N), n = (int)(i % N);
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) acc += ws[(long long)s * total + i];
    if (bias != nullptr) acc += to_f32(bias[n]);
    T* c = C + (long long)m * ldc + n;
    if (accumulate) acc += to_f32(*c);
    *c = from_f32<T>(acc);
  }
}

// ------------------------------------------------------------------ host
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    check_cuda(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q),
               "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
    if (ptr == nullptr || q != cudaDriverEntryPointSuccess)
      throw std::runtime_error("cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 2-D map over a row-major matrix [outer, inner] with row stride ld elements.
CUtensorMap make_map(const void* ptr, int dtype, long long inner, long long outer, long long ld,
                     int box_inner, int box_outer) {
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0)
    throw std::runtime_error("gemm operand must be 16-byte aligned");
  if ((ld * 2) % 16 != 0) throw std::runtime_error("gemm operand row stride must be 16-byte aligned");
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                           2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return m;
}

template <int BN>
constexpr size_t smem_bytes() {
  return 1024 + STAGES * (BM + BN) * BK * 2 + sizeof(Barriers);
}

template <typename T, int BN>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, int grid,
            cudaStream_t st) {
  auto kern = gemm_kernel<T, BN>;
  static bool attr_set = false;
  if (!attr_set) {
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)smem_bytes<BN>()),
               "gemm smem attribute");
    attr_set = true;
  }
  kern<<<grid, kThreads, smem_bytes<BN>(), st>>>(ta, tb, p);
}

}  // namespace tc

// Pick the N tile (256 or 128) and the split-K factor from a simple time
// model: waves * K-slices * per-slice time, plus the fp32 workspace round
// trip of split-K.  Returns the workspace floats the plan needs.
long long gemm_plan(int M, int N, int K, int num_sms, int* bn_out, int* splits_out) {
  const int kb = (K + tc::BK - 1) / tc::BK;
  double best = 1e30;
  int best_bn = N > 128 ? 256 : 128, best_s = 1;
  for (int bn : {256, 128}) {
    if (bn == 256 && N <= 128) continue;
    const double t_slice = bn == 256 ? 0.27 : 0.15;  // us per 64-deep K slice
    const long long tiles = (long long)((M + tc::BM - 1) / tc::BM) * ((N + bn - 1) / bn);
    for (int s = 1; s <= 16; ++s) {
      const int per = (kb + s - 1) / s;
      if (s > 1 && per < 4) break;
      if ((kb + per - 1) / per != s) continue;
      const double waves = std::ceil((double)(tiles * s) / num_sms);
      double t = waves * per * t_slice;
      if (s > 1) t += (2.0 * s * (double)M * N * 4.0 + (double)M * N * 2.0) / 6.0e12 * 1e6 + 3.0;
      if (t < best - 1e-9) {
        best = t;
        best_bn = bn;
        best_s = s;
      }
    }
  }
  *bn_out = best_bn;
  *splits_out = best_s;
  return best_s > 1 ? (long long)best_s * M * N : 0;
}

void gemm_tcgen05(const void* A, long long lda, int a_mn, const void* B, long long ldb, int b_mn,
                  void* C, long long ldc, const void* bias, int M, int N, int K, int dtype,
                  int accumulate, float* ws, long long ws_floats, unsigned* err,
                  double timeout_s, cudaStream_t st) {
  using namespace tc;
  int bn, splits;
  const long long need = gemm_plan(M, N, K, kNumSMs, &bn, &splits);
  if (need > ws_floats || ws == nullptr) {
    splits = 1;
    bn = N > 128 ? 256 : 128;
  }
  Params p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.kb_total = (K + BK - 1) / BK;
  p.kb_per_split = (p.kb_total + splits - 1) / splits;
  p.splits = (p.kb_total + p.kb_per_split - 1) / p.kb_per_split;
  p.tiles_m = (M + BM - 1) / BM;
  p.tiles_n = (N + bn - 1) / bn;
  p.units = p.tiles_m * p.tiles_n * p.splits;
  p.C = C;
  p.ldc = ldc;
  p.bias = p.splits > 1 ? nullptr : bias;
  p.ws = ws;
  p.a_mn = a_mn;
  p.b_mn = b_mn;
  p.accumulate = p.splits > 1 ? 0 : accumulate;
  const uint32_t fmt = dtype == kBF16 ? 1u : 0u;
  p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | (static_cast<uint32_t>(a_mn) << 15) |
            (static_cast<uint32_t>(b_mn) << 16) | (static_cast<uint32_t>(bn >> 3) << 17) |
            (static_cast<uint32_t>(BM >> 4) << 24);
  p.err = err;
  p.timeout_ns = static_cast<unsigned long long>(timeout_s * 1e9);

  // operand maps: K-major [rows, K] -> box {64, rows-tile}; MN-major [K, rows] -> box {64, 64}
  const CUtensorMap ta = a_mn ? make_map(A, dtype, M, K, lda, 64, 64)
                              : make_map(A, dtype, K, M, lda, 64, BM);
  const CUtensorMap tb = b_mn ? make_map(B, dtype, N, K, ldb, 64, 64)
                              : make_map(B, dtype, K, N, ldb, 64, bn);
  const int grid = std::min(p.units, kNumSMs);
  if (dtype == kF16) {
    if (bn == 256) launch<__half, 256>(ta, tb, p, grid, st);
    else launch<__half, 128>(ta, tb, p, grid, st);
  } else if (dtype == kBF16) {
    if (bn == 256) launch<__nv_bfloat16, 256>(ta, tb, p, grid, st);
    else launch<__nv_bfloat16, 128>(ta, tb, p, grid, st);
  } else {
    throw std::runtime_error("tcgen05 gemm takes fp16/bf16 operands");
  }
  MSB_CHECK_LAUNCH("gemm_tcgen05");
  if (p.splits > 1) {
    const int blocks = grid_for((long long)M * N, 256, kNumSMs * 8);
    if (dtype == kF16)
      splitk_reduce_kernel<__half><<<blocks, 256, 0, st>>>(
          ws, p.splits, M, N, static_cast<__half*>(C), ldc, static_cast<const __half*>(bias),
          accumulate);
    else
      splitk_reduce_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
          ws, p.splits, M, N, static_cast<__nv_bfloat16*>(C), ldc,
          static_cast<const __nv_bfloat16*>(bias), accumulate);
    MSB_CHECK_LAUNCH("splitk_reduce");
  }
}

}  // namespace msb
