// Causal flash attention, forward, for sm_100a (tcgen05 + tensor memory).
//
//   O[b, t, h, :] = softmax_t'<=t (q_t . k_t' / sqrt(D)) v_t'     (GQA: kv head h / (H/Hkv))
//
// Reads Q, K and V straight out of the fused projection output: a row-major
// [B*T, W] matrix whose row holds every head's q, k and v (column offsets
// q_col + h*D, k_col + g*D, v_col + g*D), so no head-major copies are made.
// Writes O as [B*T, H*D] (the layout the output projection consumes) and the
// per-row log-sum-exp (base 2) for the backward pass.
//
// One CTA computes one 128-row query tile of one (batch, head):
//   warp 0     TMA: the Q tile once, then K and V tiles of 128 keys into a
//              two-stage ring (separate barriers, so S can start before V lands)
//   warp 1     tensor memory owner and MMA issuer:
//                S  = Q K^T        (M=128, N=128, K=D; A, B from shared memory)
//                O += P V          (M=128, N=D, K=128; A = P from tensor memory,
//                                   B = V MN-major from shared memory)
//   warps 2-5  softmax, one thread per query row: tcgen05.ld its 128 scores,
//              causal mask, running max, exp2, row sum; P is written back over
//              the S columns as packed 16-bit pairs (tcgen05.st); O is
//              rescaled in tensor memory only when the row max grew by more
//              than 8 (log2 units) since the last rescale, so P <= 2^8 always
//              fits the 16-bit type and most tiles skip the O round trip.
//              After the last tile: O / l, stored to global memory.
// Tensor memory: 128 columns S/P + D columns O (256 columns), so two CTAs
// share an SM and one's softmax overlaps the other's MMAs.
// Causal tile skip: query tile i visits key tiles 0..i only; the diagonal
// tile is masked per element.  Query tiles are scheduled longest first.
//
// Every wait is bounded (globaltimer): past the limit the CTA records an
// error code, raises its abort flag, waits (bounded) for copies and MMAs in
// flight, frees its tensor memory and returns.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <type_traits>

#include "common.cuh"
#include "tcgen05.cuh"

// Phase tracing for tuning (off unless compiled with -DMSB_ATTN_TRACE): the
// cycles each role spends per phase, summed over CTAs into g_attn_trace.
#ifdef MSB_ATTN_TRACE
__device__ unsigned long long g_attn_trace[64];
#define ATTN_T0(v) const long long v = clock64()
#define ATTN_ADD(id, v) atomicAdd(&g_attn_trace[id], (unsigned long long)(clock64() - (v)))
#else
#define ATTN_T0(v)
#define ATTN_ADD(id, v)
#endif

namespace msb {
namespace attn {

using namespace ::msb::ptx;

constexpr int BQ = 128;        // query rows per tile
constexpr int BKV = 128;       // keys per tile
constexpr int KV_MAX = 3;      // K/V ring stages: 3 for D = 64, 2 for D = 128 (shared memory)
template <int D>
constexpr int kv_stages() { return D == 64 ? 3 : 2; }
constexpr int kThreads = 320;  // 10 warps
constexpr float kRescaleLog2 = 8.f;

struct Params {
  int B, T, H, Hkv;
  int q_col, k_col, v_col;   // column of head 0's q / k / v in the qkv row
  void* out;
  long long ld_out;
  float* lse;                // [B*H, T], base-2 log-sum-exp of the scaled scores
  float scale_log2;          // log2(e) / sqrt(D)
  int n_qtiles, n_pairs;
  uint32_t idesc_s, idesc_o;
  unsigned* err;
  unsigned long long timeout_ns;
  int poly;                  // of every 4 exponentials of P, how many exp2_poly computes (0-2)
};

template <int D>
struct Smem {
  static constexpr int Q_BYTES = BQ * D * 2;
  static constexpr int KV_BYTES = BKV * D * 2;
  static constexpr int CHUNK = BQ * 128;   // one 64-column (128-byte) slab of a tile
};

struct alignas(8) Bars {
  uint64_t q_full;
  uint64_t k_full[KV_MAX], k_empty[KV_MAX];
  uint64_t v_full[KV_MAX], v_empty[KV_MAX];
  uint64_t s_full[2];    // S of tile t in tensor memory
  uint64_t s_free[2];    // S of tile t read into registers (4 warps arrive; separate-P layout)
  uint64_t p_full[2];    // P of tile t written, O of tile t corrected (4 warps arrive)
  uint64_t pv_done[2];   // O_t += P_t V retired: S_t/P_t columns free again
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

template <int D>
constexpr size_t smem_bytes() {
  return 1024 + 2 * Smem<D>::Q_BYTES + kv_stages<D>() * 2 * Smem<D>::KV_BYTES + sizeof(Bars);
}

__device__ __forceinline__ bool wait_b(uint32_t bar, uint32_t parity, volatile int* abort,
                                       const Params& p, unsigned code) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = gtime();
  while (true) {
    if (mbar_try_for(bar, parity, 1000000u)) return true;
    if (*abort) return false;
    if (gtime() - t0 > p.timeout_ns) {
      *abort = 1;
      atomicCAS(p.err, 0u, code);
      return false;
    }
  }
}

__device__ __forceinline__ bool warp_wait_f(uint32_t bar, uint32_t parity, volatile int* abort,
                                            const Params& p, unsigned code, int lane) {
  return warp_wait_all(bar, parity, abort, p.err, code, p.timeout_ns, lane);
}

// K-major operand (rows x D, 64-column slabs CHUNK bytes apart), k-th 16-wide step
template <int D>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int ks) {
  return smem_desc(base + (ks >> 2) * Smem<D>::CHUNK + (ks & 3) * 32, 16, 1024);
}
// V (128 keys x D, MN-major: D contiguous), k-th 16-key step
template <int D>
__device__ __forceinline__ uint64_t v_desc(uint32_t base, int ks) {
  return smem_desc(base + ks * 2048, Smem<D>::CHUNK, 1024);
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// explicit shared-memory accesses (a pointer that went through the CTA's
// alignment round-up is generic to the compiler, and generic accesses wait
// on the long scoreboard)
__device__ __forceinline__ float4 lds_f4(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(a));
  return v;
}
__device__ __forceinline__ void sts_u4(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}
__device__ __forceinline__ void sts_f(uint32_t a, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}

#ifndef MSB_EXP2_POLY
#define MSB_EXP2_POLY 0   // of every 4 backward exponentials, how many use exp2_poly
#endif

// exp2_poly (2^x on the FMA and integer pipes) lives in common.cuh.

// One CTA: query tiles 2c and 2c+1 of one (batch, head).  The MMA warp
// alternates between them (ping-pong): while warps 2-5 run the softmax of
// tile 0's scores, the tensor core computes tile 1's, and the other way
// round.  Each softmax thread holds its row's 128 scores in registers
// (one batched tensor-memory load, one pass).
template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
attn_fwd_kernel(const __grid_constant__ CUtensorMap tm, const Params p) {
  using S = Smem<D>;
  constexpr int KV_STAGES = kv_stages<D>();
  constexpr uint32_t TMEM_COLS = 512;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                               // two tiles
  uint8_t* sK = sQ + 2 * S::Q_BYTES;
  uint8_t* sV = sK + KV_STAGES * S::KV_BYTES;
  Bars* bars = reinterpret_cast<Bars*>(sV + KV_STAGES * S::KV_BYTES);
  volatile int* abort = &bars->abort;

  ATTN_T0(t_cta);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // blocks are dispatched x-fastest: every head's last pair (the most key
  // tiles) first, then the next-to-last, ...
  const int c = p.n_pairs - 1 - blockIdx.y;
  const int bh = blockIdx.x;
  const int b = bh / p.H, h = bh % p.H;
  const int g = h / (p.H / p.Hkv);
  const int row0 = b * p.T;
  const int n_kv_all = (p.T + BKV - 1) / BKV;
  const int qt0 = 2 * c, qt1 = 2 * c + 1;
  const bool has1 = qt1 < p.n_qtiles;
  const int nkv0 = min(n_kv_all, qt0 + 1);
  const int nkv1 = has1 ? min(n_kv_all, qt1 + 1) : 0;
  const int nkv = max(nkv0, nkv1);

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bars->q_full), 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(smem_u32(&bars->k_full[s]), 1);
      mbar_init(smem_u32(&bars->k_empty[s]), 1);
      mbar_init(smem_u32(&bars->v_full[s]), 1);
      mbar_init(smem_u32(&bars->v_empty[s]), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(smem_u32(&bars->s_full[t]), 1);
      mbar_init(smem_u32(&bars->s_free[t]), 4);
      mbar_init(smem_u32(&bars->p_full[t]), 4);
      mbar_init(smem_u32(&bars->pv_done[t]), 1);
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
  const uint32_t tmem = bars->tmem_base;
  // set-up above touches shared and tensor memory only: it overlaps the
  // previous kernel's tail (programmatic dependent launch)
  ::msb::pdl_begin();
  // Tensor memory.  D = 64: S of tile t at 128t, P at 256 + 64t, O at 384 + 64t,
  // so the next scores of a tile can be computed while its softmax still
  // runs.  D = 128: no room for that; P overwrites S (its next S waits for P V).
  constexpr bool SEP_P = D == 64;
  auto col_s = [](int t) { return (uint32_t)(128 * t); };
  auto col_p = [](int t) { return SEP_P ? (uint32_t)(256 + 64 * t) : (uint32_t)(128 * t); };
  auto col_o = [](int t) { return SEP_P ? (uint32_t)(384 + 64 * t) : (uint32_t)(256 + D * t); };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA
    // (the whole warp; one elected lane issues the copies)
    const uint32_t qb = smem_u32(&bars->q_full);
    mbar_expect_tx_w(qb, (has1 ? 2 : 1) * S::Q_BYTES);
#pragma unroll
    for (int cc = 0; cc < D / 64; ++cc) {
      tma_load_2d_w(smem_u32(sQ) + cc * S::CHUNK, &tm, qb, p.q_col + h * D + 64 * cc,
                  row0 + qt0 * BQ);
      if (has1)
        tma_load_2d_w(smem_u32(sQ + S::Q_BYTES) + cc * S::CHUNK, &tm, qb,
                    p.q_col + h * D + 64 * cc, row0 + qt1 * BQ);
    }
    int kpend[KV_STAGES], vpend[KV_STAGES];
#pragma unroll
    for (int s = 0; s < KV_STAGES; ++s) kpend[s] = vpend[s] = -1;
    for (int j = 0; j < nkv; ++j) {
      const int st = j % KV_STAGES;
      const uint32_t ph = (j / KV_STAGES) & 1;
      const int y = row0 + j * BKV;
      if (!warp_wait_f(smem_u32(&bars->k_empty[st]), ph ^ 1, abort, p, 21, lane)) break;
      const uint32_t kb = smem_u32(&bars->k_full[st]);
      mbar_expect_tx_w(kb, S::KV_BYTES);
#pragma unroll
      for (int cc = 0; cc < D / 64; ++cc)
        tma_load_2d_w(smem_u32(sK + st * S::KV_BYTES) + cc * S::CHUNK, &tm, kb,
                    p.k_col + g * D + 64 * cc, y);
      kpend[st] = (int)ph;
      if (!warp_wait_f(smem_u32(&bars->v_empty[st]), ph ^ 1, abort, p, 22, lane)) break;
      const uint32_t vb = smem_u32(&bars->v_full[st]);
      mbar_expect_tx_w(vb, S::KV_BYTES);
#pragma unroll
      for (int cc = 0; cc < D / 64; ++cc)
        tma_load_2d_w(smem_u32(sV + st * S::KV_BYTES) + cc * S::CHUNK, &tm, vb,
                    p.v_col + g * D + 64 * cc, y);
      vpend[st] = (int)ph;
    }
    // copies in flight land before the CTA may exit
    const uint64_t t0 = gtime();
    while (!mbar_try(qb, 0) && gtime() - t0 < p.timeout_ns) {
    }
    for (int s = 0; s < KV_STAGES; ++s) {
      if (kpend[s] >= 0)
        while (!mbar_try(smem_u32(&bars->k_full[s]), (uint32_t)kpend[s]) &&
               gtime() - t0 < p.timeout_ns) {
        }
      if (vpend[s] >= 0)
        while (!mbar_try(smem_u32(&bars->v_full[s]), (uint32_t)vpend[s]) &&
               gtime() - t0 < p.timeout_ns) {
        }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA
    // Event loop over the two tiles: issue whichever MMA is ready (S of
    // tile t for key tile js[t], P V of tile t for key tile jp[t]), so one
    // tile's softmax never holds up the other's tensor-core work.  The whole
    // warp runs it (every lane probes the barriers, a vote keeps it
    // converged) and issues through the warp-wide umma_*_w forms.
    auto ready = [&](uint32_t bar, uint32_t parity) -> bool { return warp_test(bar, parity); };
    auto qbase = [&](int t) { return smem_u32(sQ + t * S::Q_BYTES); };
    auto nk = [&](int t) { return t == 0 ? nkv0 : nkv1; };
    int js[2] = {0, 0}, jp[2] = {0, 0};
    int kfree = 0, vfree = 0;               // next key tile whose K / V slot to release
    bool ok = warp_wait_f(smem_u32(&bars->q_full), 0, abort, p, 23, lane);
    uint64_t t_idle = 0;
    while (ok) {
      bool progress = false, pending = false;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        // ---- S_t(js): K landed, and tile t's S columns free (its softmax read
        // the previous S, or, when P overwrites S, the previous P V retired)
        const int j = t == 0 ? js[0] : js[1];
        if (j < nk(t)) {
          pending = true;
          const int st = j % KV_STAGES;
          const bool s_ok = j == 0 || (SEP_P ? ready(smem_u32(&bars->s_free[t]), (j - 1) & 1)
                                             : ready(smem_u32(&bars->pv_done[t]), (j - 1) & 1));
          if (s_ok && ready(smem_u32(&bars->k_full[st]), (j / KV_STAGES) & 1)) {
            tc_fence_after();
            const uint32_t kb = smem_u32(sK + st * S::KV_BYTES);
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks)
              umma_f16_w(tmem + col_s(t), kmajor_desc<D>(qbase(t), ks), kmajor_desc<D>(kb, ks),
                         p.idesc_s, ks > 0 ? 1u : 0u);
            umma_commit_w(smem_u32(&bars->s_full[t]));
            if (t == 0) ++js[0]; else ++js[1];
            progress = true;
          }
        }
        // ---- P_t V(jp): P written and V landed (S of that key tile issued)
        const int jj = t == 0 ? jp[0] : jp[1];
        if (jj < nk(t)) {
          pending = true;
          const int st = jj % KV_STAGES;
          if (jj < (t == 0 ? js[0] : js[1]) && ready(smem_u32(&bars->p_full[t]), jj & 1) &&
              ready(smem_u32(&bars->v_full[st]), (jj / KV_STAGES) & 1)) {
            tc_fence_after();
            const uint32_t vbase = smem_u32(sV + st * S::KV_BYTES);
#pragma unroll
            for (int ks = 0; ks < BKV / 16; ++ks)
              umma_f16_ts_w(tmem + col_o(t), tmem + col_p(t) + ks * 8, v_desc<D>(vbase, ks),
                            p.idesc_o, (jj > 0 || ks > 0) ? 1u : 0u);
            umma_commit_w(smem_u32(&bars->pv_done[t]));
            if (t == 0) ++jp[0]; else ++jp[1];
            progress = true;
          }
        }
      }
      // release K / V slots once every tile that reads them has issued its MMA
      while (kfree < nkv && (kfree < js[0] || kfree >= nkv0) && (kfree < js[1] || kfree >= nkv1)) {
        umma_commit_w(smem_u32(&bars->k_empty[kfree % KV_STAGES]));
        ++kfree;
      }
      while (vfree < nkv && (vfree < jp[0] || vfree >= nkv0) && (vfree < jp[1] || vfree >= nkv1)) {
        umma_commit_w(smem_u32(&bars->v_empty[vfree % KV_STAGES]));
        ++vfree;
      }
      if (!pending) break;
      if (progress) {
        t_idle = 0;
      } else {
        // lane 0 decides, so the warp leaves together
        int stop = 0;
        if (lane == 0) {
          const uint64_t now = gtime();
          if (*abort) {
            stop = 1;
          } else if (t_idle == 0) {
            t_idle = now;
          } else if (now - t_idle > p.timeout_ns) {
            *abort = 1;
            atomicCAS(p.err, 0u, 26u);
            stop = 1;
          }
        }
        if (__shfl_sync(0xffffffffu, stop, 0)) break;
      }
    }
    umma_commit_w(smem_u32(&bars->drain));
    const uint64_t t0 = gtime();
    while (!mbar_try(smem_u32(&bars->drain), 0) && gtime() - t0 < p.timeout_ns) {
    }
  } else if (warp >= 2) {
    // -------------------------------------------------------- softmax
    const int t = (warp - 2) >> 2;                    // which query tile
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;                // row of the tile = TMEM lane
    const int qt = t == 0 ? qt0 : qt1;
    const int nk = t == 0 ? nkv0 : nkv1;
    const int q = qt * BQ + r;                        // query position
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const uint32_t cs = col_s(t), cp = col_p(t), co = col_o(t);
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nk; ++j) {
      ATTN_T0(t_s);
      int w = lane == 0 ? (wait_b(smem_u32(&bars->s_full[t]), j & 1, abort, p, 28) ? 1 : 0) : 0;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) { ok = false; break; }
      if (warp == 2 && lane == 0) ATTN_ADD(0, t_s);
      tc_fence_after();
      ATTN_T0(t_p1);
      // raw scores of this thread's row (scaled on use, fused into the exp's FMA)
      uint32_t sv[BKV];
#pragma unroll
      for (int cc = 0; cc < BKV / 32; ++cc)
        tmem_ld32(lane_base + cs + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(sv + cc * 32));
      tmem_ld_wait();
      if (SEP_P) {
        // the scores are in registers: the tensor core may overwrite them
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bars->s_free[t]));
      }
      const int kv0 = j * BKV;
      // keys past the query (diagonal tile) or past the sequence are masked
      const int lim = min(q, p.T - 1) - kv0;          // last visible key offset in this tile
      if (lim < BKV - 1) {
#pragma unroll
        for (int e = 0; e < BKV; ++e)
          if (e > lim) sv[e] = __float_as_uint(-INFINITY);
      }
      float mx = -INFINITY;
#pragma unroll
      for (int e = 0; e < BKV; ++e) mx = fmaxf(mx, __uint_as_float(sv[e]));
      mx *= p.scale_log2;
      if (warp == 2 && lane == 0) ATTN_ADD(1, t_p1);
      ATTN_T0(t_rs);
      // lazy rescale: move the reference max only when it grew by > 2^8
      const bool grow = mx > m_used + kRescaleLog2;
      const float m_new = grow ? mx : m_used;
      const float alpha = grow ? ex2(m_used - m_new) : 1.f;   // 0 on the first visible tile
      l *= alpha;
      m_used = m_new;
      if (warp == 2 && lane == 0) ATTN_ADD(2, t_rs);
      ATTN_T0(t_p2);
      const float mref = m_used == -INFINITY ? 0.f : m_used;
      // P = 2^(s - m) as packed 16-bit pairs, first into registers: the
      // exponentials do not depend on the tile's previous P V, only the
      // store of P into its (single) tensor-memory buffer does, so they run
      // while that P V is still on the tensor core.  A share of them (p.poly
      // of every 4, off by default) can go to exp2_poly on the FMA pipe.
      uint32_t pk[64];
      auto make_p = [&](auto share) {
        constexpr int PC = decltype(share)::value;
#pragma unroll
        for (int e = 0; e < 64; ++e) {
          const float xa = fmaf(__uint_as_float(sv[2 * e]), p.scale_log2, -mref);
          const float xb = fmaf(__uint_as_float(sv[2 * e + 1]), p.scale_log2, -mref);
          const float a = ex2(xa);
          const float bb = (PC >= 2 || (PC == 1 && (e & 1))) ? exp2_poly(xb) : ex2(xb);
          l += a + bb;
          pk[e] = pack2<T>(a, bb);
        }
      };
      if (p.poly <= 0) make_p(std::integral_constant<int, 0>{});
      else if (p.poly == 1) make_p(std::integral_constant<int, 1>{});
      else make_p(std::integral_constant<int, 2>{});
      if (SEP_P && j > 0) {
        // P and O of this tile are free once its previous P V retired
        if (!warp_wait_f(smem_u32(&bars->pv_done[t]), (j - 1) & 1, abort, p, 30, lane)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
#pragma unroll
      for (int hh = 0; hh < 4; ++hh)
        tmem_st16(lane_base + cp + hh * 16, *reinterpret_cast<uint32_t(*)[16]>(pk + hh * 16));
      if (__any_sync(0xffffffffu, grow && j > 0)) {
        // O is stable: this tile's previous P V retired (waited for above, or
        // before its S was issued), and its next P V waits for p_full
#pragma unroll
        for (int cc = 0; cc < D / 32; ++cc) {
          uint32_t v[32];
          tmem_ld32(lane_base + co + cc * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
          tmem_st32(lane_base + co + cc * 32, v);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars->p_full[t]));
      if (warp == 2 && lane == 0) ATTN_ADD(3, t_p2);
    }
    if (ok && nk > 0) {
      int w = lane == 0 ? (wait_b(smem_u32(&bars->pv_done[t]), (nk - 1) & 1, abort, p, 29) ? 1 : 0)
                        : 0;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (w) {
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        T* orow = static_cast<T*>(p.out) + (long long)(row0 + q) * p.ld_out + (long long)h * D;
#pragma unroll
        for (int cc = 0; cc < D / 32; ++cc) {
          uint32_t v[32];
          tmem_ld32(lane_base + co + cc * 32, v);
          tmem_ld_wait();
          if (q < p.T) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              uint4 pack;
              uint32_t* pw = reinterpret_cast<uint32_t*>(&pack);
#pragma unroll
              for (int e = 0; e < 4; ++e)
                pw[e] = pack2<T>(__uint_as_float(v[u * 8 + 2 * e]) * inv,
                                 __uint_as_float(v[u * 8 + 2 * e + 1]) * inv);
              *reinterpret_cast<uint4*>(orow + cc * 32 + u * 8) = pack;
            }
          }
        }
        if (q < p.T) p.lse[(long long)bh * p.T + q] = m_used + __log2f(l);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (threadIdx.x == 0) ATTN_ADD(8, t_cta);
}

template <typename T, int D>
void launch_fwd(const CUtensorMap& tm, const Params& p, int B, int H, cudaStream_t st) {
  auto kern = attn_fwd_kernel<T, D>;
  static bool attr = false;
  if (!attr) {
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)smem_bytes<D>()),
               "attn smem attribute");
    attr = true;
  }
  dim3 grid(B * H, p.n_pairs);
  ::msb::launch(kern, grid, kThreads, smem_bytes<D>(), st, tm, p);
}

// ======================================================================
// Backward.  One CTA owns one 128-key tile of one (batch, kv head) and loops
// over the query heads of its group and over the query tiles at or after
// the diagonal.  Per (head, query tile):
//   S^T  = K Q^T,  dP^T = V dO^T                (keys on the tensor-memory lanes)
//   P^T  = 2^(S^T * scale*log2e - lse),  dS^T = P^T (dP^T - delta)   (warps 2-5)
//   dV  += P^T dO,  dK += dS^T Q                (A = P^T / dS^T from tensor memory;
//                                                accumulated across the whole loop)
//   dQ   = dS K                                 (A = dS^T from shared memory)
// and warps 6-9 add the dQ partial into an fp32 accumulator with TMA
// reduce-adds (several key tiles contribute to one query tile).  delta =
// rowsum(dO * O) and the zeroed accumulator come from attn_delta_kernel; the
// 16-bit dQ (times the softmax scale) from attn_dq_convert_kernel.
// Tensor memory: S^T/P^T 128, dP^T/dS^T 128, dV D, dK D, dQ D columns.
namespace bwd {

struct Params {
  int B, T, H, Hkv;
  int q_col, k_col, v_col;
  void* dqkv;
  long long ld_dqkv;
  const float* lse;
  const float* delta;
  float scale_log2, scale;
  int n_q;
  int rep, nbh;          // H / Hkv, B * Hkv
  uint32_t idesc_s, idesc_kv, idesc_q;
  unsigned* err;
  unsigned long long timeout_ns;
};

// operand whose rows (the K index of the MMA) are 128-byte swizzled rows of
// 64 contiguous M/N elements, slabs of 64 columns 16 KB apart
__device__ __forceinline__ uint64_t mn_desc(uint32_t base, int ks) {
  return smem_desc(base + ks * 2048, 128 * 128, 1024);
}
// K-major operand: rows of 64 contiguous K elements (128-byte swizzle), k-th 16-wide step
__device__ __forceinline__ uint64_t k_desc(uint32_t base, int ks) {
  return smem_desc(base + ks * 32, 16, 1024);
}

// ---------------------------------------------------------------- head dim 64
// Persistent: one CTA per SM walks work items w = blockIdx.x, + gridDim.x, ...
// An item is one 128-key block j of one (batch, kv head); items are ordered
// by key block, so the ones with the most query tiles come first.  Per item
// the CTA walks the 64-row query tiles from the diagonal down, for every
// query head that shares the kv head.  Per query tile t (score buffer t & 1):
//   S^T = K Q_t^T, dP^T = V dO_t^T       M = 128 keys, N = 64 queries -> buffer
//   softmax warps: P^T = exp2(S^T * scale_log2 - lse), dS^T = P^T (dP^T - delta);
//                  P^T -> tensor memory (packed 16-bit), dS^T -> shared memory
//   dV += P^T dO_t (A from tensor memory), dK += dS^T Q_t (A from shared memory)
//   every second tile: dQ = dS K over the pair's 128 queries (M = 128), read
//                  out by the dQ warps and reduce-added into an fp32 buffer
// The MMA warp issues tile t+2's scores as soon as the softmax of tile t is
// done, then tile t's gradient MMAs, so the tensor core works on one tile
// while the softmax warps work on the other.  Tiles are numbered across the
// CTA's items, so the next item's K/V loads and first scores overlap the end
// of the current one; K/V are double-buffered, dK/dV are read out of tensor
// memory by the softmax warps after the next item's first tile.
// Tensor memory (512 columns): S^T 0/128, dP^T 64/192 (buffer 0/1), P^T
// 256/288, dV 320, dK 384, dQ 448.
// Warps: 0 TMA, 1 MMA, 2-9 softmax (thread = key row, warp = 32 queries),
// 10-13 dQ read-out (thread = query row).  The TMA and MMA warps run their
// loops as whole warps (every lane polls the barriers, one elected lane
// issues), which keeps the MMA issue rate at the tensor core's.  The
// barrier protocol is modelled on the CPU in tests/test_kernel_protocols.py.
constexpr int kThreadsB = 448;
constexpr int kStages64 = 5;   // Q / dO tiles in flight

struct alignas(8) Bars {
  uint64_t kv_full[2], kv_empty[2];
  uint64_t qo_full[kStages64], qo_empty[kStages64];
  uint64_t st_full[2];   // scores of a tile in buffer b
  uint64_t ds_ready[2];  // softmax of a tile done: P^T / dS^T written, buffer b read (8 warps)
  uint64_t p_free[2];    // gradient MMAs of a tile retired (and every MMA before them)
  uint64_t dq_full;      // dQ of a tile pair in tensor memory
  uint64_t dq_free;      // dQ read out (4 warps)
  uint64_t acc_full;     // dK / dV of an item complete
  uint64_t acc_free;     // dK / dV read out (8 warps)
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

struct Layout64 {
  static constexpr int KV = 128 * 128;   // 128 rows x 128 bytes
  static constexpr int QT = 64 * 128;    // 64 rows x 128 bytes
  static constexpr int KV_OFF = 0;                          // 2 buffers x (K, V)
  static constexpr int Q_OFF = 4 * KV;
  static constexpr int DO_OFF = Q_OFF + kStages64 * QT;
  static constexpr int DS_OFF = DO_OFF + kStages64 * QT;   // 2 pair slots x 2 tiles x [128 keys][64 q]
  static constexpr int STG_OFF = DS_OFF + 4 * KV;          // dQ staging: 4 warps x 32 rows x 16 fp32
  static constexpr int STG_WARP = 32 * 16 * 4;
  static constexpr int LSE_OFF = STG_OFF + 4 * STG_WARP;   // 8 softmax warps x 32 floats
  static constexpr int DELTA_OFF = LSE_OFF + 8 * 128;
  static constexpr int BARS_OFF = DELTA_OFF + 8 * 128;
  static constexpr size_t BYTES = 1024 + BARS_OFF + sizeof(Bars);
  static_assert(BYTES <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ bool wait_b(uint32_t bar, uint32_t parity, volatile int* abort,
                                       const Params& p, unsigned code) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = gtime();
  while (true) {
    if (mbar_try_for(bar, parity, 1000000u)) return true;
    if (*abort) return false;
    if (gtime() - t0 > p.timeout_ns) {
      *abort = 1;
      atomicCAS(p.err, 0u, code);
      return false;
    }
  }
}
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                                          const Params& p, unsigned code, int lane) {
  return warp_wait_all(bar, parity, abort, p.err, code, p.timeout_ns, lane);
}

// A CTA's position in its sequence of work items and their query tiles
// (counters only: no divisions per tile).
struct Cursor {
  int k;      // item ordinal within the CTA
  int j, b, g;
  int n_i;    // 64-row query tiles per query head (even)
  int nit;    // query tiles of the item (all heads of the group)
  int t;      // tile within the item
  int ti, hh; // t = hh * n_i + ti
  bool valid;
  __device__ __forceinline__ void load(const Params& p) {
    const int w = blockIdx.x + k * gridDim.x;
    valid = w < p.n_q * p.nbh;
    t = ti = hh = 0;
    if (!valid) return;
    j = w / p.nbh;
    const int bh = w - j * p.nbh;
    b = bh / p.Hkv;
    g = bh - b * p.Hkv;
    n_i = 2 * (p.n_q - j);
    nit = p.rep * n_i;
  }
  __device__ __forceinline__ void start(const Params& p) {
    k = 0;
    load(p);
  }
  __device__ __forceinline__ void next(const Params& p) {
    ++t;
    if (++ti == n_i) {
      ti = 0;
      ++hh;
    }
    if (t == nit) {
      ++k;
      load(p);
    }
  }
  __device__ __forceinline__ int head(const Params& p) const { return g * p.rep + hh; }
  __device__ __forceinline__ int q0() const { return j * 128 + ti * 64; }
};

// slot and phase of a kStages64-deep ring
struct Ring {
  int s = 0;
  uint32_t ph = 0;
  __device__ __forceinline__ void next() {
    if (++s == kStages64) {
      s = 0;
      ph ^= 1;
    }
  }
};

__device__ __forceinline__ int cta_tiles(const Params& p) {
  Cursor c;
  c.start(p);
  int n = 0;
  while (c.valid) {
    n += c.nit;
    ++c.k;
    c.load(p);
  }
  return n;
}

// P^T and dS^T of 32 queries (one row of keys) from their scores and dP^T.
// MASK: causal / sequence-end mask (diagonal and last tiles only).
template <typename T, bool MASK>
__device__ __forceinline__ void softmax_bwd_row(const uint32_t (&sv)[32], const uint32_t (&dv)[32],
                                                uint32_t wl, uint32_t wd, float scale_log2,
                                                int qbase, int kj, int seq, uint32_t (&pk)[16],
                                                uint32_t (&dk)[16]) {
#pragma unroll
  for (int e4 = 0; e4 < 8; ++e4) {
    const float4 lv = lds_f4(wl + e4 * 16), dl = lds_f4(wd + e4 * 16);
    const float la[4] = {lv.x, lv.y, lv.z, lv.w};
    const float da[4] = {dl.x, dl.y, dl.z, dl.w};
    float pp[4], dd[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int c = 4 * e4 + u;
      // half of the exponentials on the special-function unit, half on the FMA pipe
      const float x = fmaf(__uint_as_float(sv[c]), scale_log2, -la[u]);
      float pr = u < 4 - MSB_EXP2_POLY ? ex2(x) : exp2_poly(x);
      if (MASK) {
        const int qi = qbase + c;
        pr = (qi >= kj && qi < seq) ? pr : 0.f;
      }
      pp[u] = pr;
      dd[u] = pr * (__uint_as_float(dv[c]) - da[u]);
    }
    pk[2 * e4] = pack2<T>(pp[0], pp[1]);
    pk[2 * e4 + 1] = pack2<T>(pp[2], pp[3]);
    dk[2 * e4] = pack2<T>(dd[0], dd[1]);
    dk[2 * e4 + 1] = pack2<T>(dd[2], dd[3]);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreadsB, 1)
attn_bwd64_kernel(const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ CUtensorMap tm_q,
                  const __grid_constant__ CUtensorMap tm_do, const __grid_constant__ CUtensorMap tm_dq,
                  const Params p) {
  using L = Layout64;
  constexpr int D = 64;
  constexpr uint32_t TMEM_COLS = 512;
  constexpr uint32_t C_P = 256, C_DV = 320, C_DK = 384, C_DQ = 448;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + L::BARS_OFF);
  float* sLse = reinterpret_cast<float*>(smem + L::LSE_OFF);
  float* sDelta = reinterpret_cast<float*>(smem + L::DELTA_OFF);
  volatile int* abort = &bars->abort;
  const uint32_t sbase = smem_u32(smem);

  ATTN_T0(t_cta);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = cta_tiles(p);   // query tiles over all of this CTA's items (even)

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&bars->kv_full[s]), 1);
      mbar_init(smem_u32(&bars->kv_empty[s]), 1);
      mbar_init(smem_u32(&bars->st_full[s]), 1);
      mbar_init(smem_u32(&bars->ds_ready[s]), 8);
      mbar_init(smem_u32(&bars->p_free[s]), 1);
    }
    for (int s = 0; s < kStages64; ++s) {
      mbar_init(smem_u32(&bars->qo_full[s]), 1);
      mbar_init(smem_u32(&bars->qo_empty[s]), 1);
    }
    mbar_init(smem_u32(&bars->dq_full), 1);
    mbar_init(smem_u32(&bars->dq_free), 4);
    mbar_init(smem_u32(&bars->acc_full), 1);
    mbar_init(smem_u32(&bars->acc_free), 8);
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
  const uint32_t tmem = bars->tmem_base;
  // set-up above touches shared and tensor memory only: it overlaps the
  // previous kernel's tail (programmatic dependent launch)
  ::msb::pdl_begin();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA
    // (the whole warp; one elected lane issues the copies)
    Cursor c, kc;   // next tile to load; next item whose K / V to load
    c.start(p);
    kc.start(p);
    uint32_t used = 0, phases = 0;   // buffers loaded, and the phase of each one's last load
    Ring ring;
    // K and V of item kc into buffer kc.k & 1 once the item two back is done
    // with it (wait: block until then; otherwise return if it is still busy)
    auto load_kv = [&](bool wait) -> bool {
      const int kb = kc.k & 1;
      const uint32_t eb = smem_u32(&bars->kv_empty[kb]), par = ((kc.k - 2) >> 1) & 1;
      if (kc.k >= 2) {
        if (wait) {
          if (!warp_wait(eb, par, abort, p, 40, lane)) return false;
        } else if (!warp_test(eb, par)) {
          return true;
        }
      }
      const uint32_t fb = smem_u32(&bars->kv_full[kb]);
      const int row = kc.b * p.T + kc.j * 128;
      mbar_expect_tx_w(fb, 2 * L::KV);
      tma_load_2d_w(sbase + L::KV_OFF + kb * 2 * L::KV, &tm_kv, fb, p.k_col + kc.g * D, row);
      tma_load_2d_w(sbase + L::KV_OFF + kb * 2 * L::KV + L::KV, &tm_kv, fb, p.v_col + kc.g * D, row);
      used |= 1u << (kStages64 + kb);
      phases = (phases & ~(1u << (kStages64 + kb))) | ((uint32_t)((kc.k >> 1) & 1) << (kStages64 + kb));
      ++kc.k;
      kc.load(p);
      return true;
    };
    bool ok = true;
    for (int t = 0; t < total && ok; ++t, c.next(p)) {
      if (kc.valid && kc.k <= c.k && !load_kv(true)) break;   // this item's K / V
      const int s = ring.s;
      const uint32_t ph = ring.ph;
      ring.next();
      const uint32_t eb = smem_u32(&bars->qo_empty[s]);
      // while the ring slot is busy, load the next item's K / V if its buffer frees
      const uint64_t t0 = gtime();
      while (!__all_sync(0xffffffffu, mbar_try_for(eb, ph ^ 1, 2000u))) {
        if (kc.valid && kc.k == c.k + 1 && !load_kv(false)) ok = false;
        int stop = 0;
        if (lane == 0) {
          if (!ok || *abort) {
            stop = 1;
          } else if (gtime() - t0 > p.timeout_ns) {
            *abort = 1;
            atomicCAS(p.err, 0u, 41u);
            stop = 1;
          }
        }
        if (__shfl_sync(0xffffffffu, stop, 0)) {
          ok = false;
          break;
        }
      }
      if (!ok) break;
      const uint32_t fb = smem_u32(&bars->qo_full[s]);
      const int row = c.b * p.T + c.q0(), h = c.head(p);
      mbar_expect_tx_w(fb, 2 * L::QT);
      tma_load_2d_w(sbase + L::Q_OFF + s * L::QT, &tm_q, fb, p.q_col + h * D, row);
      tma_load_2d_w(sbase + L::DO_OFF + s * L::QT, &tm_do, fb, h * D, row);
      used |= 1u << s;
      phases = (phases & ~(1u << s)) | (ph << s);
      if (kc.valid && kc.k == c.k + 1) load_kv(false);
    }
    // let every load this warp issued land before the CTA exits
    const uint64_t t0 = gtime();
    for (int s = 0; s < kStages64 + 2; ++s) {
      if (!(used >> s & 1)) continue;
      const uint32_t bar = s < kStages64 ? smem_u32(&bars->qo_full[s])
                                         : smem_u32(&bars->kv_full[s - kStages64]);
      while (!mbar_try(bar, (phases >> s) & 1) && gtime() - t0 < p.timeout_ns) {
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA
    // The whole warp runs this loop (waits, descriptors, cursors) and issues
    // through the warp-wide umma_*_w forms (one elected lane issues).
    const bool issuer = lane == 0;
    bool ok = true;
    Cursor sc, gc;   // the tile whose scores are issued next; whose gradients are issued next
    Ring rs, rg;     // their Q / dO ring slots
    // operand descriptors built once: a buffer or k-step offset adds to the
    // start-address field (16-byte units: a 128 x 128-byte tile is 1024, a
    // K-major k-step 2, an MN-major k-step 128)
    const uint64_t kd_kv = k_desc(sbase + L::KV_OFF, 0), md_kv = mn_desc(sbase + L::KV_OFF, 0);
    const uint64_t kd_q = k_desc(sbase + L::Q_OFF, 0), md_q = mn_desc(sbase + L::Q_OFF, 0);
    const uint64_t kd_o = k_desc(sbase + L::DO_OFF, 0), md_o = mn_desc(sbase + L::DO_OFF, 0);
    const uint64_t kd_s = k_desc(sbase + L::DS_OFF, 0), md_s = mn_desc(sbase + L::DS_OFF, 0);
    constexpr uint32_t U_KV = L::KV / 16, U_QT = L::QT / 16;
    sc.start(p);
    gc.start(p);
    // gradient MMAs of global tile v (cursor gc), whose softmax is done (and,
    // after a pair's second tile, the pair's dQ; after an item's last tile,
    // its dK / dV and K / V buffers are released)
    auto grads = [&](int v) -> bool {
      const int bv = v & 1, sv = rg.s, kvb = gc.k & 1;
      rg.next();
      if (gc.t == 0 && gc.k > 0 &&
          !warp_wait(smem_u32(&bars->acc_free), (gc.k - 1) & 1, abort, p, 44, lane))
        return false;
      tc_fence_after();
      ATTN_T0(t_g1);
      const uint64_t b_o = md_o + sv * U_QT, b_q = md_q + sv * U_QT;
      const uint64_t a_ds = kd_s + (((v >> 1) & 1) * 2 + (v & 1)) * U_KV;
      const uint32_t first = gc.t == 0 ? 0u : 1u;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint32_t acc = ks > 0 ? 1u : first;
        umma_f16_ts_w(tmem + C_DV, tmem + C_P + bv * 32 + ks * 8, b_o + 128 * ks, p.idesc_kv, acc);
        umma_f16_w(tmem + C_DK, a_ds + 2 * ks, b_q + 128 * ks, p.idesc_kv, acc);
      }
      umma_commit_w(smem_u32(&bars->qo_empty[sv]));
      umma_commit_w(smem_u32(&bars->p_free[bv]));
      if (issuer) ATTN_ADD(25, t_g1);
      if (v & 1) {
        const int pr = v >> 1;
        ATTN_T0(t_dqf);
        if (pr > 0 && !warp_wait(smem_u32(&bars->dq_free), (pr - 1) & 1, abort, p, 46, lane))
          return false;
        if (issuer) ATTN_ADD(15, t_dqf);
        tc_fence_after();
        ATTN_T0(t_g2);
        const uint64_t a_s = md_s + (pr & 1) * 2 * U_KV, b_k = md_kv + kvb * 2 * U_KV;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_f16_w(tmem + C_DQ, a_s + 128 * ks, b_k + 128 * ks, p.idesc_q, ks > 0 ? 1u : 0u);
        umma_commit_w(smem_u32(&bars->dq_full));
        if (issuer) ATTN_ADD(26, t_g2);
      }
      if (gc.t == gc.nit - 1) {
        umma_commit_w(smem_u32(&bars->acc_full));
        umma_commit_w(smem_u32(&bars->kv_empty[kvb]));
      }
      gc.next(p);
      return true;
    };
    // S^T and dP^T of global tile u (cursor sc) into buffer u & 1
    auto issue_s = [&](int u) {
      ATTN_T0(t_is);
      const int bt = u & 1, st = rs.s, kvb = sc.k & 1;
      rs.next();
      const uint64_t a_k = kd_kv + kvb * 2 * U_KV, a_v = a_k + U_KV;
      const uint64_t b_q = kd_q + st * U_QT, b_o = kd_o + st * U_QT;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        umma_f16_w(tmem + bt * 128, a_k + 2 * ks, b_q + 2 * ks, p.idesc_s, ks > 0 ? 1u : 0u);
        umma_f16_w(tmem + bt * 128 + 64, a_v + 2 * ks, b_o + 2 * ks, p.idesc_s, ks > 0 ? 1u : 0u);
      }
      umma_commit_w(smem_u32(&bars->st_full[bt]));
      if (issuer) ATTN_ADD(24, t_is);
      sc.next(p);
    };
    // non-blocking probe, the same answer in every lane
    auto ready = [&](uint32_t bar, uint32_t parity) -> bool { return warp_test(bar, parity); };
    // step u: once the softmax of tile u-2 is done, its score buffer takes
    // tile u, and tile u-2's gradient MMAs are issued
    for (int u = 0; u < total + 2 && ok; ++u) {
      if (u >= 2) {
        ATTN_T0(t_ds);
        if (!warp_wait(smem_u32(&bars->ds_ready[u & 1]), ((u - 2) >> 1) & 1, abort, p, 45, lane)) {
          ok = false;
          break;
        }
        if (issuer) ATTN_ADD(14, t_ds);
        tc_fence_after();
      }
      // tile u's scores go first when its K / V and Q / dO are in; otherwise
      // tile u-2's gradient MMAs go first and the scores follow
      bool pend = u < total;
      if (pend && (sc.t > 0 || ready(smem_u32(&bars->kv_full[sc.k & 1]), (sc.k >> 1) & 1)) &&
          ready(smem_u32(&bars->qo_full[rs.s]), rs.ph)) {
        tc_fence_after();
        issue_s(u);
        pend = false;
      }
      if (u >= 2 && !grads(u - 2)) {
        ok = false;
        break;
      }
      if (pend) {
        ATTN_T0(t_q);
        if ((sc.t == 0 && !warp_wait(smem_u32(&bars->kv_full[sc.k & 1]), (sc.k >> 1) & 1, abort,
                                     p, 42, lane)) ||
            !warp_wait(smem_u32(&bars->qo_full[rs.s]), rs.ph, abort, p, 43, lane)) {
          ok = false;
          break;
        }
        if (issuer) ATTN_ADD(12, t_q);
        tc_fence_after();
        issue_s(u);
      }
    }
    umma_commit_w(smem_u32(&bars->drain));
    const uint64_t t0 = gtime();
    while (!mbar_try(smem_u32(&bars->drain), 0) && gtime() - t0 < p.timeout_ns) {
    }
  } else if (warp >= 2 && warp < 10) {
    // ------------------- P^T, dS^T (thread = key, warp = 32 of the 64 queries)
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lb = tmem + ((uint32_t)(quarter * 32) << 16);
    const uint32_t sdS = sbase + L::DS_OFF;
    // this warp's copy of its 32 queries' lse / delta, loaded one tile ahead
    const uint32_t wLse = smem_u32(sLse + (warp - 2) * 32);
    const uint32_t wDelta = smem_u32(sDelta + (warp - 2) * 32);
    auto gload = [&](const Cursor& c, float& l, float& d) {
      const int qi = c.q0() + half * 32 + lane;
      const long long lrow = (long long)(c.b * p.H + c.head(p)) * p.T;
      l = qi < p.T ? p.lse[lrow + qi] : 0.f;
      d = qi < p.T ? p.delta[lrow + qi] : 0.f;
    };
    // dK (times the softmax scale) and dV of item ep_k: the warps of half 0
    // store dK, those of half 1 dV
    int ep_k = -1, ep_b = 0, ep_j = 0, ep_g = 0;
    auto epilogue = [&]() -> bool {
      ATTN_T0(t_ep);
      if (!warp_wait(smem_u32(&bars->acc_full), ep_k & 1, abort, p, 48, lane)) return false;
      tc_fence_after();
      const uint32_t col0 = half == 0 ? C_DK : C_DV;
      uint32_t v[64];
      tmem_ld32(lb + col0, *reinterpret_cast<uint32_t(*)[32]>(v));
      tmem_ld32(lb + col0 + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars->acc_free));
      const int kj = ep_j * 128 + r;
      if (kj < p.T) {
        const float f = half == 0 ? p.scale : 1.f;
        T* dst = static_cast<T*>(p.dqkv) + (long long)(ep_b * p.T + kj) * p.ld_dqkv +
                 (half == 0 ? p.k_col : p.v_col) + ep_g * D;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          uint4 pack;
          uint32_t* pw = reinterpret_cast<uint32_t*>(&pack);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            pw[e] = pack2<T>(__uint_as_float(v[u * 8 + 2 * e]) * f,
                             __uint_as_float(v[u * 8 + 2 * e + 1]) * f);
          *reinterpret_cast<uint4*>(dst + u * 8) = pack;
        }
      }
      ep_k = -1;
      if (warp == 2 && lane == 0) ATTN_ADD(13, t_ep);
      return true;
    };
    Cursor c, nc;
    c.start(p);
    nc = c;
    float gl = 0.f, gd = 0.f;
    if (total > 0) gload(c, gl, gd);
    bool ok = true;
    for (int t = 0; t < total; ++t, c.next(p)) {
      const int bt = t & 1, ti = c.ti;
      const int kj = c.j * 128 + r;
      const int qbase = c.q0() + half * 32;
      __syncwarp();
      sts_f(wLse + lane * 4, gl);
      sts_f(wDelta + lane * 4, gd);
      __syncwarp();
      nc.next(p);
      if (t + 1 < total) gload(nc, gl, gd);
      ATTN_T0(t_st);
      if (!warp_wait(smem_u32(&bars->st_full[bt]), (t >> 1) & 1, abort, p, 47, lane)) {
        ok = false;
        break;
      }
      if (warp == 2 && lane == 0) ATTN_ADD(10, t_st);
      ATTN_T0(t_sm);
      tc_fence_after();
      uint32_t sv[32], dv[32];
      tmem_ld32(lb + bt * 128 + half * 32, sv);
      tmem_ld32(lb + bt * 128 + 64 + half * 32, dv);
      tmem_ld_wait();
      if (warp == 2 && lane == 0) ATTN_ADD(20, t_sm);
      ATTN_T0(t_c1);
      uint32_t pk[16], dk[16];
      if (ti < 2 || qbase - half * 32 + 64 > p.T)
        softmax_bwd_row<T, true>(sv, dv, wLse, wDelta, p.scale_log2, qbase, kj, p.T, pk, dk);
      else
        softmax_bwd_row<T, false>(sv, dv, wLse, wDelta, p.scale_log2, qbase, kj, p.T, pk, dk);
#ifdef MSB_ATTN_TRACE
      __syncwarp();
      if (warp == 2 && lane == 0) ATTN_ADD(21, t_c1);
#endif
      ATTN_T0(t_c2);
      // P^T columns of buffer bt and the dS^T slab of tile t are free once the
      // gradient MMAs of tile t-2 retired (and with them the dQ MMA of the
      // pair that last used the slab)
      if (t >= 2 && !warp_wait(smem_u32(&bars->p_free[bt]), ((t - 2) >> 1) & 1, abort, p, 50,
                               lane)) {
        ok = false;
        break;
      }
      if (warp == 2 && lane == 0) ATTN_ADD(22, t_c2);
      ATTN_T0(t_c3);
      tc_fence_after();
      tmem_st16(lb + C_P + bt * 32 + half * 16, pk);
      // dS^T row r, queries half*32 .. +31 of the tile: 16-byte pieces 4*half .. 4*half+3
      const uint32_t rowp = sdS + (((t >> 1) & 1) * 2 + (t & 1)) * L::KV + r * 128;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int piece = (half * 4 + u) ^ (r & 7);
        sts_u4(rowp + piece * 16, dk[4 * u], dk[4 * u + 1], dk[4 * u + 2], dk[4 * u + 3]);
      }
      tmem_st_wait();
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars->ds_ready[bt]));
      if (warp == 2 && lane == 0) ATTN_ADD(11, t_sm);
      if (warp == 2 && lane == 0) ATTN_ADD(23, t_c3);
      // the previous item's dK / dV once this tile's softmax is out (its last
      // gradient MMAs ran meanwhile)
      if (ep_k >= 0 && !epilogue()) {
        ok = false;
        break;
      }
      if (c.t == c.nit - 1) {
        ep_k = c.k;
        ep_b = c.b;
        ep_j = c.j;
        ep_g = c.g;
      }
    }
    if (ok && ep_k >= 0) epilogue();
  } else if (warp >= 10) {
    // ------------------------------------- dQ of a tile pair -> fp32 accumulator
    const int quarter = warp & 3;
    const uint32_t lb = tmem + ((uint32_t)(quarter * 32) << 16);
    uint8_t* stg = smem + L::STG_OFF + (warp - 10) * L::STG_WARP;
    Cursor c;
    c.start(p);
    for (int pr = 0; pr < total / 2; ++pr, c.next(p), c.next(p)) {
      const int h = c.head(p), row = c.b * p.T + c.q0() + quarter * 32;
      ATTN_T0(t_dq);
      if (!warp_wait(smem_u32(&bars->dq_full), pr & 1, abort, p, 49, lane)) break;
      if (warp == 10 && lane == 0) ATTN_ADD(16, t_dq);
      ATTN_T0(t_dqe);
      tc_fence_after();
      uint32_t v[D];
      tmem_ld32(lb + C_DQ, *reinterpret_cast<uint32_t(*)[32]>(v));
      tmem_ld32(lb + C_DQ + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars->dq_free));
      if (warp == 10 && lane == 0) ATTN_ADD(17, t_dqe);
      // four 16-column boxes of 32 rows x 64 bytes (64-byte swizzle) through
      // one staging buffer
#pragma unroll
      for (int cc = 0; cc < D / 16; ++cc) {
        ATTN_T0(t_bw);
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
        if (warp == 10 && lane == 0) ATTN_ADD(18, t_bw);
        const uint32_t rowp = smem_u32(stg) + lane * 64;
#pragma unroll
        for (int u = 0; u < 4; ++u)
          sts_u4(rowp + ((u ^ ((lane >> 1) & 3)) << 4), v[cc * 16 + 4 * u], v[cc * 16 + 4 * u + 1],
                 v[cc * 16 + 4 * u + 2], v[cc * 16 + 4 * u + 3]);
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_2d<4>(&tm_dq, smem_u32(stg), h * D + 16 * cc, row);
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (threadIdx.x == 0) ATTN_ADD(19, t_cta);
}

// delta[b, h, t] = sum_d dO * O (fp32) and a zeroed dQ accumulator row.
// Eight lanes per (row, head), each on its own 16-byte pieces, so a warp's
// loads and stores cover whole contiguous segments.
template <typename T, int D>
__global__ void __launch_bounds__(256)
attn_delta_kernel(const T* __restrict__ dout, long long ld_do, const T* __restrict__ out,
                  long long ld_o, float* __restrict__ delta, float* __restrict__ dq_acc, int BT,
                  int seq, int H) {
  ::msb::pdl_begin();
  constexpr int V = D / 64;   // 16-byte pieces of a head row per lane
  const long long n = (long long)BT * H;
  const int sub = threadIdx.x & 7;
  // a warp takes four consecutive (row, head) items per pass; the loop bound
  // is the warp's, so every lane reaches the shuffles
  const long long step = ((long long)gridDim.x * blockDim.x) >> 3;
  for (long long w0 = (((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * 4; w0 < n;
       w0 += step) {
    const long long idx = w0 + ((threadIdx.x & 31) >> 3);
    const bool valid = idx < n;
    const int row = valid ? (int)(idx / H) : 0, h = valid ? (int)(idx % H) : 0;
    const uint4* a = reinterpret_cast<const uint4*>(dout + (long long)row * ld_do + h * D);
    const uint4* o = reinterpret_cast<const uint4*>(out + (long long)row * ld_o + h * D);
    float acc = 0.f;
#pragma unroll
    for (int q = 0; q < V && valid; ++q) {
      const uint4 x = a[sub + 8 * q], y = o[sub + 8 * q];
      const T* xh = reinterpret_cast<const T*>(&x);
      const T* yh = reinterpret_cast<const T*>(&y);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc += to_f32(xh[e]) * to_f32(yh[e]);
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 4);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    if (!valid) continue;
    const int b = row / seq, t = row % seq;
    if (sub == 0) delta[((long long)b * H + h) * seq + t] = acc;
    float4* z = reinterpret_cast<float4*>(dq_acc + (long long)row * H * D + h * D);
#pragma unroll
    for (int q = 0; q < D / 32; ++q) z[sub + 8 * q] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// dqkv[:, q_col + h*D + d] = dq_acc * scale
template <typename T>
__global__ void __launch_bounds__(256)
attn_dq_convert_kernel(const float* __restrict__ dq_acc, int BT, int HD, T* __restrict__ dqkv,
                       long long ld_dqkv, int q_col, float scale) {
  ::msb::pdl_begin();
  const long long n = (long long)BT * HD / 8;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long e0 = idx * 8;
    const int row = (int)(e0 / HD), col = (int)(e0 % HD);
    const float4 x = reinterpret_cast<const float4*>(dq_acc)[idx * 2];
    const float4 y = reinterpret_cast<const float4*>(dq_acc)[idx * 2 + 1];
    uint4 pack;
    uint32_t* pw = reinterpret_cast<uint32_t*>(&pack);
    pw[0] = pack2<T>(x.x * scale, x.y * scale);
    pw[1] = pack2<T>(x.z * scale, x.w * scale);
    pw[2] = pack2<T>(y.x * scale, y.y * scale);
    pw[3] = pack2<T>(y.z * scale, y.w * scale);
    *reinterpret_cast<uint4*>(dqkv + (long long)row * ld_dqkv + q_col + col) = pack;
  }
}

template <typename T>
void launch_bwd64(const CUtensorMap& tkv, const CUtensorMap& tq, const CUtensorMap& td,
                  const CUtensorMap& tdq, const Params& p, cudaStream_t st) {
  auto kern = attn_bwd64_kernel<T>;
  static bool attr = false;
  if (!attr) {
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)Layout64::BYTES),
               "attn bwd smem attribute");
    attr = true;
  }
  const int items = p.n_q * p.B * p.Hkv;
  ::msb::launch(kern, std::min(items, kNumSMs), kThreadsB, Layout64::BYTES, st, tkv, tq, td, tdq, p);
}


// ---------------------------------------------------------------- head dim 128
// Tensor memory is full with S^T, dP^T, dV and dK (128 columns each), so P^T
// and dS^T are packed in place over the scores they come from (one thread per
// key row walks its row front to back and only overwrites columns it has
// already read) and the dQ partial goes, as two 64-column halves, into the
// columns the packing freed.  The dS^T tile in shared memory doubles as the
// fp32 staging of the dQ reduce-adds once the dQ MMA has read it.
// Warps: 0 TMA, 1 MMA, 2-5 P^T/dS^T (thread = key), 6-9 dQ (thread = query).
constexpr int kThreads128 = 320;

struct alignas(8) Bars128 {
  uint64_t kv_full;
  uint64_t qo_full[2], qo_empty[2];
  uint64_t st_full, ds_ready, mma2_done, dq_full, dq_free, stg_free, lse_full, drain;
  uint32_t tmem_base;
  int abort;
};

struct Layout128 {
  static constexpr int TILE = 128 * 128 * 2;
  static constexpr int CH = 128 * 128;
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = TILE;
  static constexpr int Q_OFF = 2 * TILE;        // two stages
  static constexpr int DO_OFF = 4 * TILE;       // two stages
  static constexpr int DS_OFF = 6 * TILE;       // dS^T; later the dQ staging
  static constexpr int LSE_OFF = 7 * TILE;
  static constexpr int DELTA_OFF = LSE_OFF + 512;
  static constexpr int BARS_OFF = DELTA_OFF + 512;
  static constexpr size_t BYTES = 1024 + BARS_OFF + sizeof(Bars128);
};

template <typename T>
__global__ void __launch_bounds__(kThreads128, 1)
attn_bwd128_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                   const __grid_constant__ CUtensorMap tm_do,
                   const __grid_constant__ CUtensorMap tm_dq, const Params p) {
  constexpr int D = 128;
  using L = Layout128;
  constexpr uint32_t TMEM_COLS = 512;
  constexpr uint32_t C_S = 0, C_DP = 128, C_DV = 256, C_DK = 384;
  constexpr uint32_t C_DQ0 = C_S + 64, C_DQ1 = C_DP + 64;   // freed by the packing
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Bars128* bars = reinterpret_cast<Bars128*>(smem + L::BARS_OFF);
  float* sLse = reinterpret_cast<float*>(smem + L::LSE_OFF);
  float* sDelta = reinterpret_cast<float*>(smem + L::DELTA_OFF);
  volatile int* abort = &bars->abort;
  const uint32_t sbase = smem_u32(smem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // blocks are dispatched x-fastest: every kv head's key block 0 (the most
  // query tiles) first, then key block 1, ...
  const int j = blockIdx.y;
  const int b = blockIdx.x / p.Hkv, g = blockIdx.x % p.Hkv;
  const int rep = p.H / p.Hkv;
  const int n_i = p.n_q - j;
  const int nit = rep * n_i;
  const int row0 = b * p.T;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bars->kv_full), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&bars->qo_full[s]), 1);
      mbar_init(smem_u32(&bars->qo_empty[s]), 1);
    }
    mbar_init(smem_u32(&bars->st_full), 1);
    mbar_init(smem_u32(&bars->ds_ready), 4);
    mbar_init(smem_u32(&bars->mma2_done), 1);
    mbar_init(smem_u32(&bars->dq_full), 1);
    mbar_init(smem_u32(&bars->dq_free), 4);
    mbar_init(smem_u32(&bars->stg_free), 4);
    mbar_init(smem_u32(&bars->lse_full), 4);
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
  const uint32_t tmem = bars->tmem_base;
  // set-up above touches shared and tensor memory only: it overlaps the
  // previous kernel's tail (programmatic dependent launch)
  ::msb::pdl_begin();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA
    // (the whole warp; one elected lane issues the copies)
    const uint32_t kvb = smem_u32(&bars->kv_full);
    mbar_expect_tx_w(kvb, 2 * L::TILE);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      tma_load_2d_w(sbase + L::K_OFF + c * L::CH, &tm_qkv, kvb, p.k_col + g * D + 64 * c,
                  row0 + j * 128);
      tma_load_2d_w(sbase + L::V_OFF + c * L::CH, &tm_qkv, kvb, p.v_col + g * D + 64 * c,
                  row0 + j * 128);
    }
    int pend[2] = {-1, -1};
    for (int it = 0; it < nit; ++it) {
      const int st = it & 1;
      const uint32_t ph = (it >> 1) & 1;
      const int h = g * rep + it / n_i, i = j + it % n_i;
      if (!warp_wait(smem_u32(&bars->qo_empty[st]), ph ^ 1, abort, p, 51, lane)) break;
      const uint32_t fb = smem_u32(&bars->qo_full[st]);
      mbar_expect_tx_w(fb, 2 * L::TILE);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tma_load_2d_w(sbase + L::Q_OFF + st * L::TILE + c * L::CH, &tm_qkv, fb,
                    p.q_col + h * D + 64 * c, row0 + i * 128);
        tma_load_2d_w(sbase + L::DO_OFF + st * L::TILE + c * L::CH, &tm_do, fb, h * D + 64 * c,
                    row0 + i * 128);
      }
      pend[st] = (int)ph;
    }
    const uint64_t t0 = gtime();
    while (!mbar_try(kvb, 0) && gtime() - t0 < p.timeout_ns) {
    }
    for (int s = 0; s < 2; ++s)
      if (pend[s] >= 0)
        while (!mbar_try(smem_u32(&bars->qo_full[s]), (uint32_t)pend[s]) &&
               gtime() - t0 < p.timeout_ns) {
        }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA
    // (the whole warp; lane 0 waits, umma_*_w issue from one elected lane)
    bool ok = warp_wait(smem_u32(&bars->kv_full), 0, abort, p, 52, lane);
    const uint32_t kb = sbase + L::K_OFF, vb = sbase + L::V_OFF, dsb = sbase + L::DS_OFF;
    for (int it = 0; it < nit && ok; ++it) {
      const int st = it & 1;
      const uint32_t ph = (it >> 1) & 1;
      ATTN_T0(t_a);
      if (!warp_wait(smem_u32(&bars->qo_full[st]), ph, abort, p, 53, lane)) break;
      if (lane == 0) ATTN_ADD(27, t_a);
      ATTN_T0(t_b);
      // S^T / dP^T columns (and the dQ halves inside them) are free once the
      // last MMAs retired and the dQ partial was read
      if (it > 0 && !warp_wait(smem_u32(&bars->mma2_done), (it - 1) & 1, abort, p, 54, lane)) break;
      if (it > 0 && !warp_wait(smem_u32(&bars->dq_free), (it - 1) & 1, abort, p, 55, lane)) break;
      if (lane == 0) ATTN_ADD(28, t_b);
      ATTN_T0(t_c);
      tc_fence_after();
      const uint32_t qb = sbase + L::Q_OFF + st * L::TILE, ob = sbase + L::DO_OFF + st * L::TILE;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        umma_f16_w(tmem + C_S, kmajor_desc<D>(kb, ks), kmajor_desc<D>(qb, ks), p.idesc_s,
                 ks > 0 ? 1u : 0u);
        umma_f16_w(tmem + C_DP, kmajor_desc<D>(vb, ks), kmajor_desc<D>(ob, ks), p.idesc_s,
                 ks > 0 ? 1u : 0u);
      }
      umma_commit_w(smem_u32(&bars->st_full));
      if (lane == 0) ATTN_ADD(30, t_c);
      ATTN_T0(t_d);
      if (!warp_wait(smem_u32(&bars->ds_ready), it & 1, abort, p, 56, lane)) break;
      if (lane == 0) ATTN_ADD(31, t_d);
      ATTN_T0(t_e);
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        umma_f16_ts_w(tmem + C_DV, tmem + C_S + ks * 8, mn_desc(ob, ks), p.idesc_kv,
                    (it > 0 || ks > 0) ? 1u : 0u);
        umma_f16_ts_w(tmem + C_DK, tmem + C_DP + ks * 8, mn_desc(qb, ks), p.idesc_kv,
                    (it > 0 || ks > 0) ? 1u : 0u);
      }
      if (lane == 0) ATTN_ADD(29, t_e);
      ATTN_T0(t_e2);
      // dQ = dS K in two 64-column halves (idesc_q has N = 64)
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        umma_f16_w(tmem + C_DQ0, mn_desc(dsb, ks), mn_desc(kb, ks), p.idesc_q, ks > 0 ? 1u : 0u);
        umma_f16_w(tmem + C_DQ1, mn_desc(dsb, ks), mn_desc(kb + L::CH, ks), p.idesc_q,
                 ks > 0 ? 1u : 0u);
      }
      umma_commit_w(smem_u32(&bars->qo_empty[st]));
      umma_commit_w(smem_u32(&bars->mma2_done));
      umma_commit_w(smem_u32(&bars->dq_full));
      if (lane == 0) ATTN_ADD(32, t_e2);
    }
    umma_commit_w(smem_u32(&bars->drain));
    const uint64_t t0 = gtime();
    while (!mbar_try(smem_u32(&bars->drain), 0) && gtime() - t0 < p.timeout_ns) {
    }
  } else if (warp >= 2 && warp < 6) {
    // ------------------------------------------ P^T, dS^T (thread = key row)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int kj = j * 128 + r;
    const uint32_t lb = tmem + ((uint32_t)(quarter * 32) << 16);
    uint8_t* sdS = smem + L::DS_OFF;
    const uint32_t lse_s = smem_u32(sLse), delta_s = smem_u32(sDelta);
    bool ok = true;
    for (int it = 0; it < nit; ++it) {
      const int h = g * rep + it / n_i, i = j + it % n_i;
      const long long lrow = (long long)(b * p.H + h) * p.T;
      // the shared lse / delta of the previous tile were read by every warp
      ATTN_T0(t_f);
      if (it > 0 && !warp_wait(smem_u32(&bars->ds_ready), (it - 1) & 1, abort, p, 57, lane)) {
        ok = false;
        break;
      }
      {
        const int qi = i * 128 + quarter * 32 + lane;
        sLse[quarter * 32 + lane] = qi < p.T ? p.lse[lrow + qi] : 0.f;
        sDelta[quarter * 32 + lane] = qi < p.T ? p.delta[lrow + qi] : 0.f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars->lse_full));
      if (!warp_wait(smem_u32(&bars->lse_full), it & 1, abort, p, 58, lane) ||
          !warp_wait(smem_u32(&bars->st_full), it & 1, abort, p, 59, lane) ||
          (it > 0 && !warp_wait(smem_u32(&bars->stg_free), (it - 1) & 1, abort, p, 60, lane))) {
        ok = false;
        break;
      }
      if (warp == 2 && lane == 0) ATTN_ADD(33, t_f);
      ATTN_T0(t_g);
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t sv[32], dv[32];
        tmem_ld32(lb + C_S + c * 32, sv);
        tmem_ld32(lb + C_DP + c * 32, dv);
        tmem_ld_wait();
        uint32_t pk[16], dk[16];
        // the causal / sequence-end mask only on the diagonal and last tiles
        if (i == j || i * 128 + 128 > p.T)
          softmax_bwd_row<T, true>(sv, dv, lse_s + c * 128, delta_s + c * 128, p.scale_log2,
                                   i * 128 + c * 32, kj, p.T, pk, dk);
        else
          softmax_bwd_row<T, false>(sv, dv, lse_s + c * 128, delta_s + c * 128, p.scale_log2,
                                    i * 128 + c * 32, kj, p.T, pk, dk);
        // packed in place: columns 16c..16c+15, all read by this thread already
        tmem_st16(lb + C_S + c * 16, pk);
        tmem_st16(lb + C_DP + c * 16, dk);
        const uint32_t rowp = smem_u32(sdS) + (c >> 1) * L::CH + r * 128;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int piece = ((c & 1) * 4 + u) ^ (r & 7);
          sts_u4(rowp + piece * 16, dk[4 * u], dk[4 * u + 1], dk[4 * u + 2], dk[4 * u + 3]);
        }
      }
      tmem_st_wait();
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars->ds_ready));
      if (warp == 2 && lane == 0) ATTN_ADD(34, t_g);
    }
    // dK (times the softmax scale) and dV of this key tile
    if (ok && nit > 0 && warp_wait(smem_u32(&bars->mma2_done), (nit - 1) & 1, abort, p, 61, lane)) {
      tc_fence_after();
      T* drow = static_cast<T*>(p.dqkv) + (long long)(row0 + kj) * p.ld_dqkv;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        const uint32_t col0 = which == 0 ? C_DK : C_DV;
        const float f = which == 0 ? p.scale : 1.f;
        T* dst = drow + (which == 0 ? p.k_col : p.v_col) + g * D;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(lb + col0 + c * 32, v);
          tmem_ld_wait();
          if (kj < p.T) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              uint4 pack;
              uint32_t* pw = reinterpret_cast<uint32_t*>(&pack);
#pragma unroll
              for (int e = 0; e < 4; ++e)
                pw[e] = pack2<T>(__uint_as_float(v[u * 8 + 2 * e]) * f,
                                 __uint_as_float(v[u * 8 + 2 * e + 1]) * f);
              *reinterpret_cast<uint4*>(dst + c * 32 + u * 8) = pack;
            }
          }
        }
      }
    }
  } else if (warp >= 6) {
    // ------------------------------------- dQ partial -> fp32 accumulator
    const int quarter = warp & 3;
    const uint32_t lb = tmem + ((uint32_t)(quarter * 32) << 16);
    // staging: this warp's 32 rows x 64 fp32 columns (two 32 x 32 boxes) in the dS^T tile
    uint8_t* stg = smem + L::DS_OFF + (warp - 6) * 8192;
    for (int it = 0; it < nit; ++it) {
      const int h = g * rep + it / n_i, i = j + it % n_i;
      ATTN_T0(t_h);
      if (!warp_wait(smem_u32(&bars->dq_full), it & 1, abort, p, 62, lane)) break;
      if (warp == 6 && lane == 0) ATTN_ADD(35, t_h);
      ATTN_T0(t_i);
      tc_fence_after();
      uint32_t v[128];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tmem_ld32(lb + C_DQ0 + c * 32, *reinterpret_cast<uint32_t(*)[32]>(v + c * 32));
        tmem_ld32(lb + C_DQ1 + c * 32, *reinterpret_cast<uint32_t(*)[32]>(v + 64 + c * 32));
      }
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars->dq_free));
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        if (half == 1) {
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
        }
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint8_t* rowp = stg + c * 4096 + lane * 128;
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int e0 = half * 64 + c * 32 + 4 * u;
            *reinterpret_cast<uint4*>(rowp + ((u ^ (lane & 7)) << 4)) =
                make_uint4(v[e0], v[e0 + 1], v[e0 + 2], v[e0 + 3]);
          }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
#pragma unroll
          for (int c = 0; c < 2; ++c)
            tma_reduce_add_2d<4>(&tm_dq, smem_u32(stg + c * 4096), h * D + half * 64 + 32 * c,
                              row0 + i * 128 + quarter * 32);
          bulk_commit();
        }
      }
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars->stg_free));
      if (warp == 6 && lane == 0) ATTN_ADD(36, t_i);
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

template <typename T>
void launch_bwd128(const CUtensorMap& tq, const CUtensorMap& td, const CUtensorMap& tdq,
                   const Params& p, cudaStream_t st) {
  auto kern = attn_bwd128_kernel<T>;
  static bool attr = false;
  if (!attr) {
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)Layout128::BYTES),
               "attn bwd128 smem attribute");
    attr = true;
  }
  dim3 grid(p.B * p.Hkv, p.n_q);
  ::msb::launch(kern, grid, kThreads128, Layout128::BYTES, st, tq, td, tdq, p);
}

}  // namespace bwd
}  // namespace attn

// The q, k and v heads are read with TMA at column q_col + h*D (k_col, v_col
// alike).  A TMA copy's innermost coordinate must be a multiple of 16 bytes
// (8 16-bit elements): an unaligned one is an illegal instruction, not an
// error the kernel can report, so it is refused here.  Each head range must
// also lie inside the row.
static void check_head_columns(const char* what, long long n_cols, int q_col, int k_col,
                               int v_col, int H, int Hkv, int D) {
  const long long cols[3] = {q_col, k_col, v_col};
  const long long widths[3] = {(long long)H * D, (long long)Hkv * D, (long long)Hkv * D};
  for (int i = 0; i < 3; ++i) {
    if (cols[i] < 0 || cols[i] % 8 != 0)
      throw std::runtime_error(std::string(what) +
                               ": q/k/v column offsets must be non-negative multiples of 8");
    if (cols[i] + widths[i] > n_cols)
      throw std::runtime_error(std::string(what) + ": q/k/v heads extend past the row");
  }
}

void attention_fwd(const void* qkv, long long ld_qkv, long long n_cols, int q_col, int k_col,
                   int v_col, void* out, long long ld_out, float* lse, int B, int T, int H,
                   int Hkv, int D, int dtype, float scale, unsigned* err, double timeout_s,
                   cudaStream_t st) {
  using namespace attn;
  if (D != 64 && D != 128) throw std::runtime_error("attention: head dim must be 64 or 128");
  if (H % Hkv != 0) throw std::runtime_error("attention: H must be a multiple of Hkv");
  check_head_columns("attention", n_cols, q_col, k_col, v_col, H, Hkv, D);
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (ld_out % 8))
    throw std::runtime_error("attention: output must allow 16-byte row stores");
  Params p;
  p.B = B;
  p.T = T;
  p.H = H;
  p.Hkv = Hkv;
  p.q_col = q_col;
  p.k_col = k_col;
  p.v_col = v_col;
  p.out = out;
  p.ld_out = ld_out;
  p.lse = lse;
  // share of the forward's exponentials on the FMA pipe (MSB_ATTN_POLY=0-2 of
  // 4; off by default: on B16 T1024 H12 D64 one and two of four measured
  // 0.090 and 0.104 ms against 0.087 ms with none)
  static const int poly_share = [] {
    const char* v = std::getenv("MSB_ATTN_POLY");
    const int n = v ? std::atoi(v) : 0;
    return n < 0 ? 0 : (n > 2 ? 2 : n);
  }();
  p.poly = poly_share;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.n_qtiles = (T + BQ - 1) / BQ;
  p.n_pairs = (p.n_qtiles + 1) / 2;
  const uint32_t fmt = dtype == kBF16 ? 1u : 0u;
  // S = Q K^T: both K-major, N = 128, M = 128
  p.idesc_s = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(BKV >> 3) << 17) |
              ((uint32_t)(BQ >> 4) << 24);
  // O += P V: A (tensor memory) K-major, B = V MN-major, N = D, M = 128
  p.idesc_o = (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 16) | ((uint32_t)(D >> 3) << 17) |
              ((uint32_t)(BQ >> 4) << 24);
  p.err = err;
  p.timeout_ns = static_cast<unsigned long long>(timeout_s * 1e9);
  const CUtensorMap tm = make_map(qkv, dtype, n_cols, (long long)B * T, ld_qkv, 64, 128);
  if (dtype == kF16) {
    if (D == 64) launch_fwd<__half, 64>(tm, p, B, H, st);
    else launch_fwd<__half, 128>(tm, p, B, H, st);
  } else if (dtype == kBF16) {
    if (D == 64) launch_fwd<__nv_bfloat16, 64>(tm, p, B, H, st);
    else launch_fwd<__nv_bfloat16, 128>(tm, p, B, H, st);
  } else {
    throw std::runtime_error("attention takes fp16/bf16");
  }
  MSB_CHECK_LAUNCH("attention_fwd");
}


void attention_bwd(const void* qkv, long long ld_qkv, long long n_cols, int q_col, int k_col,
                   int v_col, const void* out, long long ld_out, const void* dout, long long ld_do,
                   const float* lse, float* delta, float* dq_acc, void* dqkv, long long ld_dqkv,
                   int B, int T, int H, int Hkv, int D, int dtype, float scale, unsigned* err,
                   double timeout_s, cudaStream_t st) {
  using namespace attn::bwd;
  if (D != 64 && D != 128) throw std::runtime_error("attention backward: head dim 64 or 128");
  if (H % Hkv != 0) throw std::runtime_error("attention: H must be a multiple of Hkv");
  check_head_columns("attention backward", n_cols, q_col, k_col, v_col, H, Hkv, D);
  auto aligned = [](const void* ptr, long long ld) {
    return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && ld % 8 == 0;
  };
  if (!aligned(out, ld_out) || !aligned(dout, ld_do) || !aligned(dqkv, ld_dqkv))
    throw std::runtime_error("attention backward: operands must allow 16-byte row access");
  const int BT = B * T;
  const int T_seq = T;
  const int blocks = grid_for((long long)BT * H * 8, 256, kNumSMs * 8);
  const int blocks_c = grid_for((long long)BT * H * D / 8, 256, kNumSMs * 8);
  attn::bwd::Params p;
  p.B = B;
  p.T = T;
  p.H = H;
  p.Hkv = Hkv;
  p.q_col = q_col;
  p.k_col = k_col;
  p.v_col = v_col;
  p.dqkv = dqkv;
  p.ld_dqkv = ld_dqkv;
  p.lse = lse;
  p.delta = delta;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.n_q = (T + 127) / 128;
  p.rep = H / Hkv;
  p.nbh = B * Hkv;
  const uint32_t fmt = dtype == kBF16 ? 1u : 0u;
  // S^T = K Q^T, dP^T = V dO^T: N = 128 queries (head dim 128), 64 (head dim 64)
  p.idesc_s = (1u << 4) | (fmt << 7) | (fmt << 10) | ((D == 128 ? 16u : 8u) << 17) | (8u << 24);
  p.idesc_kv = (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 16) | ((uint32_t)(D >> 3) << 17) |
               (8u << 24);
  // dQ = dS K: N = D (head dim 128: two N = 64 halves)
  const uint32_t nq = D == 128 ? 64u : (uint32_t)D;
  p.idesc_q = (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 15) | (1u << 16) | ((nq >> 3) << 17) |
              (8u << 24);
  p.err = err;
  p.timeout_ns = static_cast<unsigned long long>(timeout_s * 1e9);
  const CUtensorMap tq = make_map(qkv, dtype, n_cols, (long long)BT, ld_qkv, 64, 128);
  const CUtensorMap td = make_map(dout, dtype, (long long)H * D, (long long)BT, ld_do, 64, 128);
  const CUtensorMap tq64 = make_map(qkv, dtype, n_cols, (long long)BT, ld_qkv, 64, 64);
  const CUtensorMap td64 = make_map(dout, dtype, (long long)H * D, (long long)BT, ld_do, 64, 64);
  const CUtensorMap tdq = make_map_f32(dq_acc, (long long)H * D, (long long)BT, (long long)H * D,
                                       32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tdq16 = make_map_f32(dq_acc, (long long)H * D, (long long)BT, (long long)H * D,
                                         16, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  auto run = [&](auto tag) {
    using T = decltype(tag);
    if (D == 64)
      ::msb::launch(attn_delta_kernel<T, 64>, blocks, 256, 0, st, static_cast<const T*>(dout), ld_do,
                                                       static_cast<const T*>(out), ld_out, delta,
                                                       dq_acc, BT, T_seq, H);
    else
      ::msb::launch(attn_delta_kernel<T, 128>, blocks, 256, 0, st, static_cast<const T*>(dout), ld_do,
                                                        static_cast<const T*>(out), ld_out, delta,
                                                        dq_acc, BT, T_seq, H);
    if (D == 64) launch_bwd64<T>(tq, tq64, td64, tdq16, p, st);
    else launch_bwd128<T>(tq, td, tdq, p, st);
    ::msb::launch(attn_dq_convert_kernel<T>, blocks_c, 256, 0, st, dq_acc, BT, H * D, static_cast<T*>(dqkv),
                                                        ld_dqkv, q_col, scale);
  };
  if (dtype == kF16) {
    run(__half());
  } else if (dtype == kBF16) {
    run(__nv_bfloat16());
  } else {
    throw std::runtime_error("attention takes fp16/bf16");
  }
  MSB_CHECK_LAUNCH("attention_bwd");
}

MSB_BOUNDS_TU(attention)

}  // namespace msb
