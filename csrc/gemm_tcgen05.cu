// Persistent warp-specialized GEMM for sm_100a on the 5th-generation tensor
// cores (tcgen05 + tensor memory).
//
//   C[M,N] (+)= A[M,K] * B[N,K]^T (+ bias[N]),  fp16/bf16 in, fp32 accumulate
//
// Operands may be K-major (K contiguous) or MN-major (M resp. N contiguous),
// which covers the three products of a linear layer without transposes:
// forward (both K-major), dgrad (B MN-major) and wgrad (both MN-major).
//
// CTA = 10 warps, one CTA per SM, persistent over output tiles (128 x BN):
//   warp 0     TMA producer: 64-deep K slices of A and B into a 4-stage
//              shared-memory ring (128-byte swizzle), one mbarrier per stage
//   warp 1     owns the tensor memory (allocates 2 x BN fp32 columns) and
//              issues tcgen05.mma (M=128, N=BN, K=16);
//              tcgen05.commit frees a ring stage once its MMAs retire and
//              signals "accumulator full" after a tile's last K slice
//   Warps 0 and 1 run their loops as whole warps: every lane polls the
//   barriers and votes, one elected lane issues (a lone issuing thread in a
//   diverged warp measured up to a third slower per MMA).
//   warps 2-9  epilogue: tcgen05.ld 32 columns at a time (one TMEM lane =
//              one output row per thread), bias, activation, cast; each
//              32 x 32 chunk is staged in shared memory and written by a TMA
//              bulk tensor store; then release the accumulator buffer so the
//              MMA warp can start the tile after next while this one drains
//              (double-buffered accumulators)
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
#include <cstdlib>
#include <string>

#include "common.cuh"
#include "tcgen05.cuh"

namespace msb {
namespace tc {

using namespace ::msb::ptx;

constexpr int BM = 128;
constexpr int BK = 64;  // 64 x 16-bit = 128 bytes = one swizzle row
constexpr int STAGES = 4;
constexpr int kEpiWarps = 8;  // two warps per TMEM lane quarter
constexpr int kThreads = 64 + 32 * kEpiWarps;

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
  int c_vec;         // C base and row stride allow 16-byte stores
  int ws_vec;        // workspace rows allow 16-byte stores
  int nfast;         // tile order: 1 = all N tiles of an M block back to back
  int mode;          // 0 plain, 1 bias+GELU (C = u, aux = gelu(u)), 2 C = acc * gelu'(aux)
  void* aux;         // second output (mode 1) or input (mode 2), row stride ld_aux
  long long ld_aux;
  int aux_vec;
  int staged;        // epilogue through shared memory + TMA stores (tmC / tmX valid)
  // stream-K (2-CTA kernel): the tiles x kb_total K slices are cut into one
  // contiguous range per pair (sk_per slices, one more for the first
  // sk_extra pairs); a tile shared by several pairs is finished by the pair
  // holding its first slice, after the others' fp32 partials (ws: one
  // 256 x 256 slot per pair) and arrivals (sk_ctr[tile]) are in
  int sk;
  int sk_per, sk_extra;
  int* sk_ctr;
  // split-K with in-kernel fixup (pair kernel, all units resident at once):
  // splits 0..S-2 of a tile store fp32 partials (ws slot split * tiles +
  // tile) and arrive on sk_ctr[tile]; split S-1 adds them and finishes
  int fix;
  // mode 2: column sums of the stored output (the fc bias gradient), one
  // fp32 partial row per 32 output rows: [ceil(M / 32), N]
  float* colsum_part;
  long long ws_floats;  // workspace and counter sizes (bounds checks of the debug build)
  long long sk_ctr_n;
  uint32_t idesc;
  unsigned* err;
  unsigned long long timeout_ns;
};

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
// the k-th step's descriptor is the 0-th's plus k times this (start address, 16-byte units)
__device__ __forceinline__ uint32_t operand_step(int mn_major) { return mn_major ? 128u : 2u; }

struct alignas(8) Barriers {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

// Bounded wait of a whole converged warp (see warp_wait_all): false when the
// CTA aborted or the limit passed.
__device__ __forceinline__ bool wait_bar_w(uint32_t bar, uint32_t parity, volatile int* abort,
                                           const Params& p, unsigned code, int lane) {
  return warp_wait_all(bar, parity, abort, p.err, code, p.timeout_ns, lane);
}

template <int BN, int TM = BM>
__device__ __forceinline__ void unit_coords(const Params& p, int u, int& m0, int& n0, int& kb0,
                                            int& kb1, int& split) {
  const int tiles = p.tiles_m * p.tiles_n;
  split = u / tiles;
  const int t = u - split * tiles;
  // Walk along the operand that is re-read less: with nfast the CTAs that run
  // together share one row block of A (the larger operand) through L2.
  if (p.nfast) {
    m0 = (t / p.tiles_n) * TM;
    n0 = (t % p.tiles_n) * BN;
  } else {
    m0 = (t % p.tiles_m) * TM;
    n0 = (t / p.tiles_m) * BN;
  }
  kb0 = split * p.kb_per_split;
  kb1 = min(p.kb_total, kb0 + p.kb_per_split);
}

// Stream-K work of a pair: K-slice range [b, e) of the tiles * kb_total
// slices, and the pair that holds slice `it`.
__device__ __forceinline__ void sk_range(const Params& p, int pair, long long& b, long long& e) {
  b = (long long)pair * p.sk_per + min(pair, p.sk_extra);
  e = b + p.sk_per + (pair < p.sk_extra ? 1 : 0);
}
__device__ __forceinline__ int sk_pair_of(const Params& p, long long it) {
  const long long big = (long long)p.sk_extra * (p.sk_per + 1);
  if (it < big) return (int)(it / (p.sk_per + 1));
  return p.sk_extra + (int)((it - big) / p.sk_per);
}

// The k-th work item of a pair: a tile and its K-slice range.  Units mode:
// unit pair + k * npairs (unit_coords).  Stream-K: the k-th tile the pair's
// slice range touches, cut to that range.
template <int BN, int TM>
__device__ __forceinline__ bool work_item(const Params& p, int pair, int npairs, int k, int& m0,
                                          int& n0, int& kb0, int& kb1, int& split, int& tile) {
  if (!p.sk) {
    const int u = pair + k * npairs;
    if (u >= p.units) return false;
    unit_coords<BN, TM>(p, u, m0, n0, kb0, kb1, split);
    tile = u % (p.tiles_m * p.tiles_n);
    return true;
  }
  long long b, e;
  sk_range(p, pair, b, e);
  const long long t = b / p.kb_total + k;
  const long long lo = max(b, t * p.kb_total), hi = min(e, (t + 1) * p.kb_total);
  if (lo >= hi) return false;
  tile = (int)t;
  kb0 = (int)(lo - t * p.kb_total);
  kb1 = (int)(hi - t * p.kb_total);
  split = 0;
  if (p.nfast) {
    m0 = (tile / p.tiles_n) * TM;
    n0 = (tile % p.tiles_n) * BN;
  } else {
    m0 = (tile % p.tiles_m) * TM;
    n0 = (tile / p.tiles_m) * BN;
  }
  return true;
}

// 32 consecutive values of one row, 16-byte accesses when `vec`
template <typename T>
__device__ __forceinline__ void store32(T* c, bool vec, const float (&v)[32], int nvalid,
                                        int accumulate) {
  if (nvalid == 32 && vec) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 pack;
      T* h = reinterpret_cast<T*>(&pack);
      if (accumulate) {
        const uint4 old = *reinterpret_cast<const uint4*>(c + q * 8);
        const T* oh = reinterpret_cast<const T*>(&old);
#pragma unroll
        for (int j = 0; j < 8; ++j) h[j] = from_f32<T>(v[q * 8 + j] + to_f32(oh[j]));
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) h[j] = from_f32<T>(v[q * 8 + j]);
      }
      *reinterpret_cast<uint4*>(c + q * 8) = pack;
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (j < nvalid) {
      float x = v[j];
      if (accumulate) x += to_f32(c[j]);
      c[j] = from_f32<T>(x);
    }
  }
}

template <typename T>
__device__ __forceinline__ void load32(const T* a, bool vec, float (&v)[32], int nvalid) {
  if (nvalid == 32 && vec) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 pack = *reinterpret_cast<const uint4*>(a + q * 8);
      const T* h = reinterpret_cast<const T*>(&pack);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[q * 8 + j] = to_f32(h[j]);
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = j < nvalid ? to_f32(a[j]) : 0.f;
}

// Epilogue of one 32-column chunk of an output row (v = acc + bias).
template <typename T>
__device__ __forceinline__ void store_chunk(const Params& p, int row, int col, float (&v)[32],
                                            int nvalid) {
  T* c = static_cast<T*>(p.C) + (long long)row * p.ldc + col;
  if (p.mode == 1) {
    // pre-activation u is stored in the model dtype; GELU sees the rounded u
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = to_f32(from_f32<T>(v[j]));
    store32<T>(c, p.c_vec, v, nvalid, 0);
    float h[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) h[j] = gelu_f(v[j]);
    store32<T>(static_cast<T*>(p.aux) + (long long)row * p.ld_aux + col, p.aux_vec, h, nvalid, 0);
    return;
  }
  if (p.mode == 2) {
    float u[32];
    load32<T>(static_cast<const T*>(p.aux) + (long long)row * p.ld_aux + col, p.aux_vec, u, nvalid);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = to_f32(from_f32<T>(v[j])) * gelu_grad_f(u[j]);
  }
  store32<T>(c, p.c_vec, v, nvalid, p.accumulate);
}

// ------------------------------------------------ staged (TMA-store) epilogue
// Each epilogue warp owns two 2 KB staging buffers: one 32-row x 32-column
// chunk of the output in the model dtype, 64 bytes per row, 16-byte pieces
// XOR-swizzled by bits 7-8 of the address (the tensor map's 64-byte swizzle;
// the eight rows one 16-byte store phase touches land in eight different
// bank groups).  Lane 0 writes the chunk to global memory with one TMA bulk
// tensor store: whole 128-byte lines, asynchronous, off the load/store unit.
constexpr int kStageBytes = 2048;
constexpr int kEpiStageBytes = kEpiWarps * 2 * kStageBytes;

template <typename T>
__device__ __forceinline__ void stage_row(uint8_t* buf, int r, const float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 pack;
    T* h = reinterpret_cast<T*>(&pack);
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = from_f32<T>(v[j * 8 + e]);
    *reinterpret_cast<uint4*>(buf + r * 64 + ((j ^ ((r >> 1) & 3)) << 4)) = pack;
  }
}

// v += bias[col .. col+31]; every lane reads the same addresses (broadcast)
template <typename T>
__device__ __forceinline__ void add_bias(const Params& p, int col, int nvalid, float (&v)[32]) {
  const T* b = static_cast<const T*>(p.bias) + col;
  if (nvalid == 32 && (reinterpret_cast<uintptr_t>(b) & 15) == 0) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 pack = *reinterpret_cast<const uint4*>(b + q * 8);
      const T* h = reinterpret_cast<const T*>(&pack);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[q * 8 + j] += to_f32(h[j]);
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j < nvalid) v[j] += to_f32(b[j]);
}

// One 32 x 32 chunk of C, rows row0.. and columns col.. all inside C (warp-
// uniform), through the staging buffers.  Modes as store_chunk; with
// accumulate (mode 0) the TMA unit adds the chunk into C (bulk reduce-add:
// the product is rounded to the 16-bit type, then added).  Split-K never
// comes here.  sbuf alternates the two buffers in modes 0 and 2.
template <typename T>
__device__ __forceinline__ void staged_chunk(const Params& p, const CUtensorMap* tmC,
                                             const CUtensorMap* tmX, uint8_t* stg, int& sbuf,
                                             int row0, int lane, int col, int nvalid,
                                             float (&v)[32]) {
  const int row = row0 + lane;
  if (p.mode == 1) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = to_f32(from_f32<T>(v[j]));
    float h[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) h[j] = gelu_f(v[j]);
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
    stage_row<T>(stg, lane, v);
    stage_row<T>(stg + kStageBytes, lane, h);
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmC, smem_u32(stg), col, row0);
      tma_store_2d(tmX, smem_u32(stg + kStageBytes), col, row0);
      bulk_commit();
    }
    return;
  }
  if (p.mode == 2) {
    float u[32];
    load32<T>(static_cast<const T*>(p.aux) + (long long)row * p.ld_aux + col, p.aux_vec, u, nvalid);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = to_f32(from_f32<T>(v[j])) * gelu_grad_f(u[j]);
  }
  if (lane == 0) bulk_wait_read<1>();
  __syncwarp();
  uint8_t* buf = stg + sbuf * kStageBytes;
  stage_row<T>(buf, lane, v);
  fence_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (p.accumulate) tma_reduce_add_2d(tmC, smem_u32(buf), col, row0);
    else tma_store_2d(tmC, smem_u32(buf), col, row0);
    bulk_commit();
  }
  sbuf ^= 1;
}

// Column sums of one 32 x 32 output chunk (lane = row) into its partial
// row: the values as stored (rounded to the model dtype), rows past M as
// zero.  A transpose-reduce: at each of five steps every lane sends the half
// of its remaining columns that its partner keeps and adds the half it
// receives (31 shuffles); lane j ends with column j's sum.
template <typename T>
__device__ __forceinline__ void chunk_colsum(const Params& p, int row0, int col, int nvalid,
                                             bool valid_row, const float (&v)[32], int lane) {
  float x[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) x[j] = valid_row ? to_f32(from_f32<T>(v[j])) : 0.f;
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const bool up = (lane & w) != 0;
#pragma unroll
    for (int j = 0; j < w; ++j) {
      const float send = up ? x[j] : x[j + w];
      const float keep = up ? x[j + w] : x[j];
      x[j] = keep + __shfl_xor_sync(0xffffffffu, send, w);
    }
  }
  const long long ci = (long long)(row0 >> 5) * p.N + col + lane;
  if (lane < nvalid && MSB_INB(ci, (long long)((p.M + 31) >> 5) * p.N, kSiteGemmColsum))
    p.colsum_part[ci] = x[0];
}

__device__ __forceinline__ void store_ws_chunk(const Params& p, int split, int row, int col,
                                               const float (&v)[32], int nvalid) {
  const long long wi = ((long long)split * p.M + row) * p.N + col;
  if (!MSB_INB(wi + nvalid - 1, p.ws_floats, kSiteGemmSlot)) return;
  float* w = p.ws + wi;
  if (nvalid == 32 && p.ws_vec) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
      reinterpret_cast<float4*>(w)[q] = make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
    return;
  }
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j < nvalid) w[j] = v[j];
}

template <typename T, int BN>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmX,
            const Params p) {
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int B_BYTES = BN * BK * 2;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sStage = sB + STAGES * B_BYTES;
  Barriers* bars = reinterpret_cast<Barriers*>(sStage + kEpiStageBytes);
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&bars->full[s]), 1);
      mbar_init(smem_u32(&bars->empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&bars->tfull[b]), 1);
      mbar_init(smem_u32(&bars->tempty[b]), kEpiWarps);
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
  // set-up above touches shared and tensor memory only: it overlaps the
  // previous kernel's tail (programmatic dependent launch)
  ::msb::pdl_begin();

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    // the whole warp runs the loop; one elected lane issues (tma_load_2d_w)
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
        if (!wait_bar_w(smem_u32(&bars->empty[stage]), phase ^ 1, abort, p, 1, lane)) {
          ok = false;
          break;
        }
        const uint32_t full = smem_u32(&bars->full[stage]);
        mbar_expect_tx_w(full, A_BYTES + B_BYTES);
        const uint32_t a_dst = smem_u32(sA + stage * A_BYTES);
        const uint32_t b_dst = smem_u32(sB + stage * B_BYTES);
        const int k0 = kb * BK;
        if (p.a_mn) {
#pragma unroll
          for (int j = 0; j < BM / 64; ++j) tma_load_2d_w(a_dst + j * 8192, &tmA, full, m0 + 64 * j, k0);
        } else {
          tma_load_2d_w(a_dst, &tmA, full, k0, m0);
        }
        if (p.b_mn) {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) tma_load_2d_w(b_dst + j * 8192, &tmB, full, n0 + 64 * j, k0);
        } else {
          tma_load_2d_w(b_dst, &tmB, full, k0, n0);
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
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    // the whole warp runs the loop; one elected lane issues (umma_*_w)
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true;
    const uint32_t a_step = operand_step(p.a_mn), b_step = operand_step(p.b_mn);
    for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++it) {
      int m0, n0, kb0, kb1, split;
      unit_coords<BN>(p, u, m0, n0, kb0, kb1, split);
      const int buf = it & 1;
      const uint32_t tphase = (it >> 1) & 1;
      if (!wait_bar_w(smem_u32(&bars->tempty[buf]), tphase ^ 1, abort, p, 2, lane)) break;
      tc_fence_after();
      const uint32_t d = tmem_base + buf * BN;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!wait_bar_w(smem_u32(&bars->full[stage]), phase, abort, p, 3, lane)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = operand_desc(smem_u32(sA + stage * A_BYTES), p.a_mn, 0);
        const uint64_t bd = operand_desc(smem_u32(sB + stage * B_BYTES), p.b_mn, 0);
#pragma unroll
        for (int ks = 0; ks < BK / 16; ++ks)
          umma_f16_w(d, ad + ks * a_step, bd + ks * b_step, p.idesc, (kb > kb0 || ks > 0) ? 1u : 0u);
        umma_commit_w(smem_u32(&bars->empty[stage]));
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (ok) umma_commit_w(smem_u32(&bars->tfull[buf]));
    }
    // every MMA issued by this warp retires before tensor memory is freed
    umma_commit_w(smem_u32(&bars->drain));
    const uint64_t t0 = gtime();
    while (!mbar_try(smem_u32(&bars->drain), 0) && gtime() - t0 < p.timeout_ns) {
    }
  } else if (warp >= 2) {
    // ---------------------------------------------------------- epilogue
    const int quarter = warp & 3;           // TMEM lanes this warp may access
    const int half = (warp - 2) / 4;        // which interleaved half of the chunks
    const int row_in_tile = quarter * 32 + lane;
    const bool has_bias = p.bias != nullptr && p.splits == 1;
    uint8_t* stg = sStage + (warp - 2) * 2 * kStageBytes;
    int sbuf = 0;
    int it = 0;
    for (int u = blockIdx.x; u < p.units; u += gridDim.x, ++it) {
      int m0, n0, kb0, kb1, split;
      unit_coords<BN>(p, u, m0, n0, kb0, kb1, split);
      const int buf = it & 1;
      const uint32_t tphase = (it >> 1) & 1;
      // one lane polls; the warp follows it as a unit (tcgen05.ld is .sync.aligned)
      if (!wait_bar_w(smem_u32(&bars->tfull[buf]), tphase, abort, p, 4, lane)) break;
      tc_fence_after();
      const int row0 = m0 + quarter * 32;
      const int row = m0 + row_in_tile;
#pragma unroll 1
      for (int c = half; c < BN / 32; c += 2) {
        uint32_t r[32];
        tmem_ld32(tmem_base + ((quarter * 32) << 16) + buf * BN + c * 32, r);
        tmem_ld_wait();
        const int col = n0 + c * 32;  // warp-uniform
        if (col >= p.N || row0 >= p.M) continue;
        const int nvalid = min(32, p.N - col);
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (has_bias) add_bias<T>(p, col, nvalid, v);
        // TMA stores only for chunks wholly inside C: ragged edges are
        // stored per thread, so no write depends on the map's bound clipping
        if (p.staged && nvalid == 32 && row0 + 32 <= p.M) {
          staged_chunk<T>(p, &tmC, &tmX, stg, sbuf, row0, lane, col, nvalid, v);
        } else if (row < p.M) {
          if (p.splits > 1) store_ws_chunk(p, split, row, col, v, nvalid);
          else store_chunk<T>(p, row, col, v, nvalid);
        }
        if (p.colsum_part != nullptr) chunk_colsum<T>(p, row0, col, nvalid, row < p.M, v, lane);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars->tempty[buf]));
    }
    // the staging buffers are read and the stores performed before exit
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}


// ======================================================================
// 2-CTA variant: a cluster of two CTAs on two SMs computes a 256 x 256
// tile with tcgen05.mma.cta_group::2 (M = 256 split over the pair's tensor
// memories).  Each CTA stages only its 128 rows of A and its 128 rows of B
// per K slice, so the L2 -> SM traffic per FLOP is 2/3 of the 1-CTA kernel
// and six ring stages fit in shared memory.  The even CTA ("leader") issues
// the MMAs; both CTAs' TMA loads signal the leader's stage barrier
// (.cta_group::2 form), each commit is sent to both CTAs' barriers, and both
// epilogues release the accumulator on the leader's barrier.  Every TMA load
// is a plain per-CTA tile load.
// ======================================================================
namespace pair {

constexpr int TM = 256;        // M rows per CTA pair
constexpr int BN2 = 256;       // N columns per tile
constexpr int HALF = 128;      // rows of A and of B staged per CTA
constexpr int STAGES2 = 6;
constexpr int A2_BYTES = HALF * BK * 2;
constexpr int B2_BYTES = HALF * BK * 2;

__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
__device__ __forceinline__ void remote_arrive(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ bool try_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded cluster-scope wait of a whole converged warp: every lane polls and
// votes (see warp_wait_all); false when the CTA aborted or the limit passed.
__device__ __forceinline__ bool wait2_w(uint32_t bar, uint32_t parity, volatile int* abort,
                                        const Params& p, unsigned code, int lane) {
  if (__all_sync(0xffffffffu, try_cluster(bar, parity))) return true;
  const uint64_t t0 = gtime();
  while (true) {
    if (__all_sync(0xffffffffu, try_cluster(bar, parity))) return true;
    int stop = 0;
    if (lane == 0) {
      if (*abort) {
        stop = 1;
      } else if (gtime() - t0 > p.timeout_ns) {
        *abort = 1;
        atomicCAS(p.err, 0u, code);
        stop = 1;
      }
    }
    if (__shfl_sync(0xffffffffu, stop, 0)) return false;
  }
}
__device__ __forceinline__ void tma_load_pair_w(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                                int x, int y) {
  if (!MSB_CHECK((x & 7) == 0, kSiteTmaLoadX, x, 8)) x &= ~7;   // as tma_load_2d_w
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.cta_group::2"
      " [%0], [%1, {%2, %3}], [%4];\n\t}" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void alloc2(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// arrive (when the issued MMAs retire) on the barrier at this offset in
// both CTAs of the pair: one commit per barrier, the peer's addressed
// through its shared::cluster window
// warp-wide forms (one elected lane issues; see umma_f16_w)
__device__ __forceinline__ void mma2_w(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void commit2_to_w(uint32_t cluster_bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          cluster_bar)
      : "memory");
}
__device__ __forceinline__ void commit2_both_w(uint32_t bar) {
  commit2_to_w(bar);
  commit2_to_w(mapa(bar, 1));
}

struct alignas(8) Bars2 {
  uint64_t full[STAGES2];
  uint64_t empty[STAGES2];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

// Bounded wait of a whole warp until *ctr >= target (lane 0 polls with
// acquire loads; the warp then proceeds together).  False on abort/timeout.
__device__ __forceinline__ bool sk_wait_w(int* ctr, int target, volatile int* abort,
                                          const Params& p, unsigned code, int lane) {
  int stop = 0;
  if (lane == 0) {
    const uint64_t t0 = gtime();
    while (true) {
      int v;
      asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
      if (v >= target) break;
      if (*abort) {
        stop = 1;
        break;
      }
      if (gtime() - t0 > p.timeout_ns) {
        *abort = 1;
        atomicCAS(p.err, 0u, code);
        stop = 1;
        break;
      }
    }
  }
  stop = __shfl_sync(0xffffffffu, stop, 0);
  __syncwarp();
  return stop == 0;
}

constexpr size_t smem_bytes2() {
  return 1024 + STAGES2 * (A2_BYTES + B2_BYTES) + kEpiStageBytes + sizeof(Bars2);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
             const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmX,
             const Params p) {
  constexpr uint32_t TMEM_COLS = 2 * BN2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES2 * A2_BYTES;
  uint8_t* sStage = sB + STAGES2 * B2_BYTES;
  Bars2* bars = reinterpret_cast<Bars2*>(sStage + kEpiStageBytes);
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cta_rank();
  const bool leader = rank == 0;
  const int pair_id = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES2; ++s) {
      mbar_init(smem_u32(&bars->full[s]), 1);
      mbar_init(smem_u32(&bars->empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&bars->tfull[b]), 1);
      mbar_init(smem_u32(&bars->tempty[b]), 2 * kEpiWarps);
    }
    mbar_init(smem_u32(&bars->drain), 1);
    bars->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  // both CTAs are running and their barriers initialised before any remote use
  cluster_sync();
  if (warp == 1) {
    alloc2(smem_u32(&bars->tmem_base), TMEM_COLS);
    relinquish2();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  // set-up above touches shared and tensor memory only: it overlaps the
  // previous kernel's tail (programmatic dependent launch)
  ::msb::pdl_begin();

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    int stage = 0;
    uint32_t phase = 0;
    int pending[STAGES2];
#pragma unroll
    for (int s = 0; s < STAGES2; ++s) pending[s] = -1;
    bool ok = true;
    int m0, n0, kb0, kb1, split, tile;
    for (int k = 0; ok && work_item<BN2, TM>(p, pair_id, npairs, k, m0, n0, kb0, kb1, split, tile);
         ++k) {
      const int am = m0 + HALF * rank, bn = n0 + HALF * rank;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!wait2_w(smem_u32(&bars->empty[stage]), phase ^ 1, abort, p, 11, lane)) {
          ok = false;
          break;
        }
        const uint32_t full_local = smem_u32(&bars->full[stage]);
        const uint32_t full_leader = mapa(full_local, 0);
        if (leader) mbar_expect_tx_w(full_local, 2 * (A2_BYTES + B2_BYTES));
        const uint32_t a_dst = smem_u32(sA + stage * A2_BYTES);
        const uint32_t b_dst = smem_u32(sB + stage * B2_BYTES);
        const int k0 = kb * BK;
        if (p.a_mn) {
          tma_load_pair_w(a_dst, &tmA, full_leader, am, k0);
          tma_load_pair_w(a_dst + 8192, &tmA, full_leader, am + 64, k0);
        } else {
          tma_load_pair_w(a_dst, &tmA, full_leader, k0, am);
        }
        if (p.b_mn) {
          tma_load_pair_w(b_dst, &tmB, full_leader, bn, k0);
          tma_load_pair_w(b_dst + 8192, &tmB, full_leader, bn + 64, k0);
        } else {
          tma_load_pair_w(b_dst, &tmB, full_leader, k0, bn);
        }
        pending[stage] = static_cast<int>(phase);
        if (++stage == STAGES2) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    if (leader) {
      // the leader's stage barriers count both CTAs' bytes: wait for them
      for (int s = 0; s < STAGES2; ++s) {
        if (pending[s] < 0) continue;
        const uint64_t t0 = gtime();
        while (!try_cluster(smem_u32(&bars->full[s]), static_cast<uint32_t>(pending[s])) &&
               gtime() - t0 < p.timeout_ns) {
        }
      }
    }
  } else if (warp == 1 && leader) {
    // ------------------------------------------------------- MMA issuer
    // the whole warp runs the loop; one elected lane issues (mma2_w)
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true;
    const uint32_t a_step = operand_step(p.a_mn), b_step = operand_step(p.b_mn);
    int m0, n0, kb0, kb1, split, tile;
    for (int k = 0; ok && work_item<BN2, TM>(p, pair_id, npairs, k, m0, n0, kb0, kb1, split, tile);
         ++k, ++it) {
      const int buf = it & 1;
      const uint32_t tphase = (it >> 1) & 1;
      if (!wait2_w(smem_u32(&bars->tempty[buf]), tphase ^ 1, abort, p, 12, lane)) break;
      tc_fence_after();
      const uint32_t d = tmem_base + buf * BN2;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!wait2_w(smem_u32(&bars->full[stage]), phase, abort, p, 13, lane)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = operand_desc(smem_u32(sA + stage * A2_BYTES), p.a_mn, 0);
        const uint64_t bd = operand_desc(smem_u32(sB + stage * B2_BYTES), p.b_mn, 0);
#pragma unroll
        for (int ks = 0; ks < BK / 16; ++ks)
          mma2_w(d, ad + ks * a_step, bd + ks * b_step, p.idesc, (kb > kb0 || ks > 0) ? 1u : 0u);
        commit2_both_w(smem_u32(&bars->empty[stage]));
        if (++stage == STAGES2) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (ok) commit2_both_w(smem_u32(&bars->tfull[buf]));
    }
    commit2_to_w(smem_u32(&bars->drain));   // this CTA's own barrier (the elected lane issued)
    const uint64_t t0 = gtime();
    while (!mbar_try(smem_u32(&bars->drain), 0) && gtime() - t0 < p.timeout_ns) {
    }
  } else if (warp >= 2) {
    // ---------------------------------------------------------- epilogue
    const int quarter = warp & 3;
    const int half = (warp - 2) / 4;
    const int row_in_tile = HALF * rank + quarter * 32 + lane;
    const bool has_bias = p.bias != nullptr && (p.splits == 1 || p.fix);
    const uint32_t tempty_leader0 = mapa(smem_u32(&bars->tempty[0]), 0);
    const uint32_t tempty_leader1 = mapa(smem_u32(&bars->tempty[1]), 0);
    uint8_t* stg = sStage + (warp - 2) * 2 * kStageBytes;
    int sbuf = 0;
    int it = 0;
    int m0, n0, kb0, kb1, split, tile;
    for (int k = 0; work_item<BN2, TM>(p, pair_id, npairs, k, m0, n0, kb0, kb1, split, tile);
         ++k, ++it) {
      const int buf = it & 1;
      const uint32_t tphase = (it >> 1) & 1;
      if (!wait2_w(smem_u32(&bars->tfull[buf]), tphase, abort, p, 14, lane)) break;
      tc_fence_after();
      // stream-K: a pair's first item may continue a tile another pair
      // started (contribute the partial); its last item may start a tile
      // that later pairs continue (finish it once their partials are in)
      // split-K fixup: the last split of a tile finishes it from the others
      const int ntiles = p.tiles_m * p.tiles_n;
      const bool contrib = (p.sk && kb0 > 0) || (p.fix && split < p.splits - 1);
      const bool finish =
          (p.sk && kb0 == 0 && kb1 < p.kb_total) || (p.fix && split == p.splits - 1);
      const long long my_slot = p.fix ? (long long)split * ntiles + tile : pair_id;
      int ncontrib = 0;
      if (finish) {
        ncontrib = p.fix ? p.splits - 1
                         : sk_pair_of(p, (long long)(tile + 1) * p.kb_total - 1) - pair_id;
        // all 16 epilogue warps of each contributing pair have arrived
        if (MSB_INB(tile, p.sk_ctr_n, kSiteGemmCounter) &&
            !sk_wait_w(p.sk_ctr + tile, 16 * ncontrib, abort, p, 15, lane))
          break;
      }
      const int row0 = m0 + HALF * rank + quarter * 32;
      const int row = m0 + row_in_tile;
#pragma unroll 1
      for (int c = half; c < BN2 / 32; c += 2) {
        uint32_t r[32];
        tmem_ld32(tmem_base + ((quarter * 32) << 16) + buf * BN2 + c * 32, r);
        tmem_ld_wait();
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        // a partial tile is stored chunk by chunk in register order: float4
        // q of lane l of chunk (row block, c) at ((rb * 8 + c) * 8 + q) * 32
        // + l, so every warp-wide store and load moves 512 contiguous bytes
        const long long slot_off =
            (((long long)(row_in_tile >> 5) * (BN2 / 32) + c) * 8) * 32 + lane;
        if (contrib) {
          // the whole 32-column piece of the row, in or out of C: the
          // finisher reads back exactly what it needs
          float4* w = reinterpret_cast<float4*>(p.ws + my_slot * (TM * BN2)) + slot_off;
          if (MSB_INB(my_slot * (TM * BN2) + (slot_off + 7 * 32) * 4 + 3, p.ws_floats,
                      kSiteGemmSlot)) {
#pragma unroll
            for (int q = 0; q < 8; ++q)
              w[q * 32] = make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
          }
          continue;
        }
        const int col = n0 + c * 32;
        if (col >= p.N || row0 >= p.M) continue;
        if (finish) {
          for (int j = 1; j <= ncontrib; ++j) {
            const long long slot =
                p.fix ? (long long)(j - 1) * ntiles + tile : (long long)(pair_id + j);
            const float4* w = reinterpret_cast<const float4*>(p.ws + slot * (TM * BN2)) + slot_off;
            if (!MSB_INB(slot * (TM * BN2) + (slot_off + 7 * 32) * 4 + 3, p.ws_floats,
                         kSiteGemmSlot))
              continue;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 x = __ldcg(w + q * 32);
              v[q * 4] += x.x;
              v[q * 4 + 1] += x.y;
              v[q * 4 + 2] += x.z;
              v[q * 4 + 3] += x.w;
            }
          }
        }
        const int nvalid = min(32, p.N - col);
        if (has_bias) add_bias<T>(p, col, nvalid, v);
        // TMA stores only for chunks wholly inside C: ragged edges are
        // stored per thread, so no write depends on the map's bound clipping
        if (p.staged && nvalid == 32 && row0 + 32 <= p.M) {
          staged_chunk<T>(p, &tmC, &tmX, stg, sbuf, row0, lane, col, nvalid, v);
        } else if (row < p.M) {
          if (p.splits > 1 && !p.fix) store_ws_chunk(p, split, row, col, v, nvalid);
          else store_chunk<T>(p, row, col, v, nvalid);
        }
        if (p.colsum_part != nullptr) chunk_colsum<T>(p, row0, col, nvalid, row < p.M, v, lane);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) remote_arrive(buf ? tempty_leader1 : tempty_leader0);
      if (contrib) {
        // release: this warp's partial rows are visible before its arrival
        __threadfence();
        __syncwarp();
        if (lane == 0 && MSB_INB(tile, p.sk_ctr_n, kSiteGemmCounter)) atomicAdd(p.sk_ctr + tile, 1);
      } else if (finish) {
        // the 16 finishing warps count out; the last one clears the counter
        // for the next launch
        __syncwarp();
        if (lane == 0 && MSB_INB(tile, p.sk_ctr_n, kSiteGemmCounter) &&
            atomicAdd(p.sk_ctr + tile, 1) == 16 * ncontrib + 15)
          atomicExch(p.sk_ctr + tile, 0);
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  // every role of both CTAs is done before tensor memory is released and
  // before either CTA's shared memory can go away
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    dealloc2(tmem_base, TMEM_COLS);
  }
}

}  // namespace pair

// C = sum_s ws[s] (+ bias) (+ C); 4 columns per thread (16-byte workspace loads)
template <typename T>
__global__ void __launch_bounds__(256)
splitk_reduce_kernel(const float* __restrict__ ws, int splits, int M, int N, T* __restrict__ C,
                     long long ldc, const T* __restrict__ bias, int accumulate) {
  ::msb::pdl_begin();
  const long long total = (long long)M * N;
  const int nq = N >> 2;  // N % 4 == 0 on this path
  const long long quads = (long long)M * nq;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < quads;
       i += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(i / nq), n = (int)(i % nq) * 4;
    const long long e = (long long)m * N + n;
    float4 acc = *reinterpret_cast<const float4*>(ws + e);
    for (int s = 1; s < splits; ++s) {
      const float4 w = *reinterpret_cast<const float4*>(ws + (long long)s * total + e);
      acc.x += w.x;
      acc.y += w.y;
      acc.z += w.z;
      acc.w += w.w;
    }
    float a[4] = {acc.x, acc.y, acc.z, acc.w};
    T* c = C + (long long)m * ldc + n;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float x = a[k];
      if (bias != nullptr) x += to_f32(bias[n + k]);
      if (accumulate) x += to_f32(c[k]);
      c[k] = from_f32<T>(x);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
splitk_reduce_scalar_kernel(const float* __restrict__ ws, int splits, int M, int N,
                            T* __restrict__ C, long long ldc, const T* __restrict__ bias,
                            int accumulate) {
  ::msb::pdl_begin();
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

template <typename T>
void launch_reduce(const float* ws, int splits, int M, int N, void* C, long long ldc,
                   const void* bias, int accumulate, cudaStream_t st) {
  if (N % 4 == 0 && (reinterpret_cast<uintptr_t>(ws) & 15) == 0) {
    const int blocks = grid_for((long long)M * N / 4, 256, kNumSMs * 8);
    ::msb::launch(splitk_reduce_kernel<T>, blocks, 256, 0, st, ws, splits, M, N, static_cast<T*>(C), ldc,
                                                    static_cast<const T*>(bias), accumulate);
  } else {
    const int blocks = grid_for((long long)M * N, 256, kNumSMs * 8);
    ::msb::launch(splitk_reduce_scalar_kernel<T>, blocks, 256, 0, st, ws, splits, M, N, static_cast<T*>(C),
                                                           ldc, static_cast<const T*>(bias),
                                                           accumulate);
  }
}

// ------------------------------------------------------------------ host
template <int BN>
constexpr size_t smem_bytes() {
  return 1024 + STAGES * (BM + BN) * BK * 2 + kEpiStageBytes + sizeof(Barriers);
}

template <typename T, int BN>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
            const CUtensorMap& tx, const Params& p, int grid, cudaStream_t st) {
  auto kern = gemm_kernel<T, BN>;
  static bool attr_set = false;
  if (!attr_set) {
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)smem_bytes<BN>()),
               "gemm smem attribute");
    attr_set = true;
  }
  ::msb::launch(kern, grid, kThreads, smem_bytes<BN>(), st, ta, tb, tc, tx, p);
}

template <typename T>
int pair_capacity(const Params& p, cudaStream_t st) {
  // how many 2-CTA clusters of this kernel can be resident at once
  static int cached = -1;
  if (cached < 0) {
    auto kern = pair::gemm2_kernel<T>;
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)pair::smem_bytes2()),
               "gemm2 smem attribute");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 74);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = pair::smem_bytes2();
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    check_cuda(cudaOccupancyMaxActiveClusters(&n, kern, &cfg), "gemm2 occupancy");
    cached = n > 0 ? n : 1;
  }
  (void)p;
  return cached;
}

template <typename T>
void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                 const CUtensorMap& tx, const Params& p, int npairs, cudaStream_t st) {
  auto kern = pair::gemm2_kernel<T>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * npairs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = pair::smem_bytes2();
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  check_cuda(cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, tx, p), "gemm2 launch");
  count_launch();
}

}  // namespace tc

// Pick the N tile (256 or 128) and the split-K factor from a simple time
// model: waves * K-slices * per-slice time, plus the fp32 workspace round
// trip of split-K.  Returns the workspace floats the plan needs.
// bn_out = 256 or 128 (one CTA per tile) or 512 (a 2-CTA pair per 256 x 256 tile).
long long gemm_plan(int M, int N, int K, int num_sms, int* bn_out, int* splits_out) {
  const int kb = (K + tc::BK - 1) / tc::BK;
  double best = 1e30;
  int best_bn = N > 128 ? 256 : 128, best_s = 1;
  const char* force = std::getenv("MSB_GEMM_VARIANT");
  for (int bn : {512, 256, 128}) {
    if (force != nullptr) {
      if (std::string(force) == "1cta" && bn == 512) continue;
      if (std::string(force) == "2cta" && bn != 512) continue;
    }
    if (bn == 256 && N <= 128) continue;
    // us per 64-deep K slice per tile; the pair kernel moves 2/3 of the bytes
    const double t_slice = bn == 512 ? 0.22 : (bn == 256 ? 0.27 : 0.15);
    const int tm = bn == 512 ? 256 : tc::BM;
    const int tn = bn == 512 ? 256 : bn;
    const int slots = bn == 512 ? num_sms / 2 : num_sms;
    const long long tiles = (long long)((M + tm - 1) / tm) * ((N + tn - 1) / tn);
    for (int s = 1; s <= 16; ++s) {
      const int per = (kb + s - 1) / s;
      if (s > 1 && per < 4) break;
      if ((kb + per - 1) / per != s) continue;
      const double waves = std::ceil((double)(tiles * s) / slots);
      double t = waves * per * t_slice;
      if (s > 1) t += (2.0 * s * (double)M * N * 4.0 + (double)M * N * 4.0) / 4.0e12 * 1e6 + 5.0;
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
                  int accumulate, int mode, void* aux, long long ld_aux, float* ws,
                  long long ws_floats, unsigned* err, double timeout_s, cudaStream_t st,
                  int force_bn, int force_splits, int* sk_ctr, long long sk_ctr_n,
                  float* colsum_part) {
  using namespace tc;
  int bn, splits;
  const long long need = gemm_plan(M, N, K, kNumSMs, &bn, &splits);
  bool stream_k = false;
  if (force_bn > 0) {
    bn = force_bn;
    stream_k = force_splits == -1 && bn == 512;
    splits = force_splits > 0 ? force_splits : 1;
    if (splits > 1 && (long long)splits * M * N > ws_floats) splits = 1;
  }
  if ((splits > 1 && (ws == nullptr || (long long)splits * M * N > ws_floats)) || mode != 0) {
    splits = 1;
    if (bn != 512) bn = N > 128 ? 256 : 128;
  }
  const bool two_cta = bn == 512;
  const int tm = two_cta ? 256 : BM;
  const int tn = two_cta ? 256 : bn;
  Params p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.kb_total = (K + BK - 1) / BK;
  p.kb_per_split = (p.kb_total + splits - 1) / splits;
  p.splits = (p.kb_total + p.kb_per_split - 1) / p.kb_per_split;
  p.tiles_m = (M + tm - 1) / tm;
  p.tiles_n = (N + tn - 1) / tn;
  p.nfast = (long long)M > (long long)N ? 1 : 0;  // A (M x K) larger than B (N x K)
  p.units = p.tiles_m * p.tiles_n * p.splits;
  // split-K on the pair kernel finishes in the kernel (no reduce launch)
  // when every unit is resident at once and the tile counters and the
  // per-tile partial slots are available
  p.fix = 0;
  if (two_cta && p.splits > 1 && sk_ctr != nullptr && ws != nullptr) {
    const int cap = dtype == kF16 ? pair_capacity<__half>(p, st)
                                  : pair_capacity<__nv_bfloat16>(p, st);
    const long long tiles = (long long)p.tiles_m * p.tiles_n;
    if (p.units <= cap && tiles <= sk_ctr_n &&
        ws_floats >= (long long)(p.splits - 1) * tiles * pair::TM * pair::BN2)
      p.fix = 1;
  }
  const bool reduce_launch = p.splits > 1 && !p.fix;
  p.C = C;
  p.ldc = ldc;
  p.bias = reduce_launch ? nullptr : bias;
  p.ws = ws;
  p.a_mn = a_mn;
  p.b_mn = b_mn;
  p.accumulate = reduce_launch ? 0 : accumulate;
  p.c_vec = ((reinterpret_cast<uintptr_t>(C) & 15) == 0 && (ldc % 8) == 0) ? 1 : 0;
  p.mode = mode;
  p.aux = aux;
  p.ld_aux = ld_aux;
  p.aux_vec = ((reinterpret_cast<uintptr_t>(aux) & 15) == 0 && (ld_aux % 8) == 0) ? 1 : 0;
  p.ws_vec = ((reinterpret_cast<uintptr_t>(ws) & 15) == 0 && (N % 4) == 0) ? 1 : 0;
  const uint32_t fmt = dtype == kBF16 ? 1u : 0u;
  p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | (static_cast<uint32_t>(a_mn) << 15) |
            (static_cast<uint32_t>(b_mn) << 16) | (static_cast<uint32_t>(tn >> 3) << 17) |
            (static_cast<uint32_t>(tm >> 4) << 24);
  p.err = err;
  p.timeout_ns = static_cast<unsigned long long>(timeout_s * 1e9);
  p.ws_floats = ws != nullptr ? ws_floats : 0;
  p.sk_ctr_n = sk_ctr != nullptr ? sk_ctr_n : 0;

  // operand maps: K-major [rows, K] -> box {64, rows staged per CTA};
  // MN-major [K, rows] -> box {64, 64}
  const int a_rows = two_cta ? pair::HALF : BM;
  const int b_rows = two_cta ? pair::HALF : bn;
  const CUtensorMap ta = a_mn ? make_map(A, dtype, M, K, lda, 64, 64)
                              : make_map(A, dtype, K, M, lda, 64, a_rows);
  const CUtensorMap tb = b_mn ? make_map(B, dtype, N, K, ldb, 64, 64)
                              : make_map(B, dtype, K, N, ldb, 64, b_rows);
  // output maps for the staged epilogue: 32 x 32 boxes, 64-byte swizzle
  // (plain and GELU/dGELU outputs; accumulation and split-K store per thread)
  p.staged = (!reduce_launch && p.c_vec && (mode != 1 || p.aux_vec) &&
              (!p.accumulate || mode == 0))
                 ? 1 : 0;
  const CUtensorMap tcm = p.staged ? make_map(C, dtype, N, M, ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)
                                   : ta;
  const CUtensorMap txm = (p.staged && mode == 1)
                              ? make_map(aux, dtype, N, M, ld_aux, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)
                              : ta;
  const int grid = std::min(p.units, kNumSMs);
  p.sk = 0;
  p.sk_per = 0;
  p.sk_extra = 0;
  p.sk_ctr = p.fix ? sk_ctr : nullptr;
  p.colsum_part = mode == 2 ? colsum_part : nullptr;
  if (two_cta) {
    const int cap = dtype == kF16 ? pair_capacity<__half>(p, st)
                                  : pair_capacity<__nv_bfloat16>(p, st);
    int npairs = std::min(p.units, cap);
    if (stream_k) {
      // every pair must be resident at once (a finishing pair waits for
      // pairs after it): one pair per resident slot, each with >= 1 slice
      const long long tiles = (long long)p.tiles_m * p.tiles_n;
      const long long total = tiles * p.kb_total;
      npairs = cap;
      if (total >= npairs && tiles <= sk_ctr_n && sk_ctr != nullptr && ws != nullptr &&
          ws_floats >= (long long)npairs * pair::TM * pair::BN2 && p.splits == 1) {
        p.sk = 1;
        p.sk_per = static_cast<int>(total / npairs);
        p.sk_extra = static_cast<int>(total % npairs);
        p.sk_ctr = sk_ctr;
        p.ws = ws;
      } else {
        npairs = std::min(p.units, cap);
      }
    }
    if (dtype == kF16) {
      launch_pair<__half>(ta, tb, tcm, txm, p, npairs, st);
    } else if (dtype == kBF16) {
      launch_pair<__nv_bfloat16>(ta, tb, tcm, txm, p, npairs, st);
    } else {
      throw std::runtime_error("tcgen05 gemm takes fp16/bf16 operands");
    }
  } else if (dtype == kF16) {
    if (bn == 256) launch<__half, 256>(ta, tb, tcm, txm, p, grid, st);
    else launch<__half, 128>(ta, tb, tcm, txm, p, grid, st);
  } else if (dtype == kBF16) {
    if (bn == 256) launch<__nv_bfloat16, 256>(ta, tb, tcm, txm, p, grid, st);
    else launch<__nv_bfloat16, 128>(ta, tb, tcm, txm, p, grid, st);
  } else {
    throw std::runtime_error("tcgen05 gemm takes fp16/bf16 operands");
  }
  MSB_CHECK_LAUNCH("gemm_tcgen05");
  if (reduce_launch) {
    if (dtype == kF16)
      launch_reduce<__half>(ws, p.splits, M, N, C, ldc, bias, accumulate, st);
    else
      launch_reduce<__nv_bfloat16>(ws, p.splits, M, N, C, ldc, bias, accumulate, st);
    MSB_CHECK_LAUNCH("splitk_reduce");
  }
}

MSB_BOUNDS_TU(gemm)

}  // namespace msb
