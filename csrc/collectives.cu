// Fused step-pipeline collectives over NVLink peer memory.
//
// Every rank owns one device buffer (the "peer heap") whose layout is the
// same on all ranks; each rank maps every peer's heap (CUDA IPC) and passes
// the table of heap base addresses to these kernels, which then load from
// and store to peer HBM directly over NVLink 5 / NVSwitch.  Plain loads and
// stores only: no multimem, no TMA.
//
//   peer_barrier      every rank signals an epoch to every peer and waits
//                     (bounded) until all peers signalled it
//   rs_stats          reduce-scatter fused with unscale/average and the
//                     gradient statistics: rank r sums its shard of every
//                     peer's model-dtype gradient arena in fp32 in rank
//                     order (deterministic), scales by 1/(loss_scale*W),
//                     writes the fp32 shard (optionally also into every
//                     peer's full fp32 buffer: the all-reduce of stage 0)
//                     and emits per-block (sum of squares, inf/nan) partials
//   stats_exchange    all-gather of each rank's [flag, sumsq] through a
//                     board in every heap; summed in rank order so every
//                     rank computes the bitwise-identical global norm
//   adamw_fanout      AdamW on this rank's shard whose fp16/bf16 cast is
//                     stored into the parameter arena of EVERY rank (the
//                     parameter all-gather fused into the update)
//   gather_range      stage-3 parameter gather: a range of the local arena <-
//                     the owning peers' model-dtype shards (gather_pull: all)
//
// Waits use %globaltimer bounds; on expiry a kernel records an error code in
// a local status word and returns, leaving the context usable.
#include "common.cuh"

namespace msb {
namespace {

__device__ __forceinline__ uint64_t gtime_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Sync area at `sync_off` in every heap:
//   uint32 flags[kMaxRanks]         flags[q] = last epoch rank q signalled
//   Board  board[kMaxRanks]         board[q] = rank q's step statistics
constexpr int kMaxRanks = 16;
struct Board {
  unsigned epoch;
  float flag;
  float sumsq;
  unsigned pad;
};

__device__ __forceinline__ unsigned* flags_of(char* heap, long long sync_off) {
  return reinterpret_cast<unsigned*>(heap + sync_off);
}
__device__ __forceinline__ Board* board_of(char* heap, long long sync_off) {
  return reinterpret_cast<Board*>(heap + sync_off + kMaxRanks * sizeof(unsigned) * 4);
}

// Epochs come from a per-rank device counter that every barrier-type kernel
// advances by one: all ranks run the same sequence of barriers, so the
// counters agree, and a kernel replayed from a CUDA graph uses the next epoch
// rather than the one current at capture time.
__global__ void peer_barrier_kernel(char* const* heaps, long long sync_off, int rank, int world,
                                    unsigned* ctr, unsigned long long timeout_ns,
                                    unsigned* status) {
  ::msb::pdl_begin();
  // make this device's earlier writes (local and peer stores of preceding
  // kernels) visible system-wide before announcing the epoch
  __threadfence_system();
  __shared__ unsigned s_epoch;
  const int t = threadIdx.x;
  if (t == 0) s_epoch = *ctr + 1u;
  __syncthreads();
  const unsigned epoch = s_epoch;
  if (t < world) st_release_sys(flags_of(heaps[t], sync_off) + rank, epoch);
  __syncthreads();
  if (t < world) {
    const unsigned* mine = flags_of(heaps[rank], sync_off) + t;
    const uint64_t t0 = gtime_ns();
    while (static_cast<int>(ld_acquire_sys(mine) - epoch) < 0) {
      if (gtime_ns() - t0 > timeout_ns) {
        atomicCAS(status, 0u, 0x100u | static_cast<unsigned>(t));
        break;
      }
    }
  }
  __syncthreads();
  if (t == 0) *ctr = epoch;
  __threadfence_system();
}

template <typename T, int VEC>
__global__ void __launch_bounds__(256, 2)
rs_stats_kernel(char* const* heaps, long long grad_off, long long s0, long long n, int world,
                float mul_host, const float* __restrict__ mul_dev, float* __restrict__ out,
                long long fanout_off, float* __restrict__ partials,
                unsigned* __restrict__ pflags) {
  ::msb::pdl_begin();
  // the multiplier (1 / (loss scale * world)) may live on the device, so a
  // launch replayed from a CUDA graph follows the current loss scale
  const float mul = mul_dev != nullptr ? mul_host * *mul_dev : mul_host;
  float ss = 0.f;
  unsigned bad = 0u;
  const long long nvec = n / VEC;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    float acc[VEC];
#pragma unroll
    for (int k = 0; k < VEC; ++k) acc[k] = 0.f;
    for (int q = 0; q < world; ++q) {
      const T* src = reinterpret_cast<const T*>(heaps[q] + grad_off) + s0 + i * VEC;
      if (VEC == 8) {
        const uint4 raw = *reinterpret_cast<const uint4*>(src);
        const T* h = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int k = 0; k < VEC; ++k) acc[k] += to_f32(h[k]);
      } else {
#pragma unroll
        for (int k = 0; k < VEC; ++k) acc[k] += to_f32(src[k]);
      }
    }
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
      const float v = acc[k] * mul;
      bad |= finite_f32(v) ? 0u : 1u;
      ss = fmaf(v, v, ss);
      acc[k] = v;
    }
    float* o = out + i * VEC;
    if (VEC == 8) {
      // out is a fresh fp32 buffer (16-byte aligned): two 16-byte stores
      reinterpret_cast<float4*>(o)[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      reinterpret_cast<float4*>(o)[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    } else {
#pragma unroll
      for (int k = 0; k < VEC; ++k) o[k] = acc[k];
    }
    if (fanout_off >= 0) {
      for (int q = 0; q < world; ++q) {
        float* dst = reinterpret_cast<float*>(heaps[q] + fanout_off) + s0 + i * VEC;
#pragma unroll
        for (int k = 0; k < VEC; ++k) dst[k] = acc[k];
      }
    }
  }
  for (long long i = nvec * VEC + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    float a = 0.f;
    for (int q = 0; q < world; ++q)
      a += to_f32(reinterpret_cast<const T*>(heaps[q] + grad_off)[s0 + i]);
    const float v = a * mul;
    bad |= finite_f32(v) ? 0u : 1u;
    ss = fmaf(v, v, ss);
    out[i] = v;
    if (fanout_off >= 0)
      for (int q = 0; q < world; ++q) reinterpret_cast<float*>(heaps[q] + fanout_off)[s0 + i] = v;
  }
  if (fanout_off >= 0) __threadfence_system();
  __shared__ float s_ss[8];
  __shared__ unsigned s_bad[8];
  ss = warp_sum(ss);
  bad = warp_or(bad);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    s_ss[warp] = ss;
    s_bad[warp] = bad;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    ss = lane < nw ? s_ss[lane] : 0.f;
    bad = lane < nw ? s_bad[lane] : 0u;
    ss = warp_sum(ss);
    bad = warp_or(bad);
    if (lane == 0) {
      partials[blockIdx.x] = ss;
      pflags[blockIdx.x] = bad;
    }
  }
}

__global__ void stats_exchange_kernel(char* const* heaps, long long sync_off, int rank, int world,
                                      unsigned* ctr, float* out, double max_norm,
                                      unsigned long long timeout_ns, unsigned* status) {
  ::msb::pdl_begin();
  if (threadIdx.x == 0) {
    const unsigned epoch = *ctr + 1u;
    *ctr = epoch;
    const float flag = out[0], sumsq = out[1];
    for (int q = 0; q < world; ++q) {
      Board* b = board_of(heaps[q], sync_off) + rank;
      b->flag = flag;
      b->sumsq = sumsq;
    }
    __threadfence_system();
    for (int q = 0; q < world; ++q) st_release_sys(&(board_of(heaps[q], sync_off) + rank)->epoch, epoch);
    Board* mine = board_of(heaps[rank], sync_off);
    double total = 0.0;
    float any = 0.f;
    bool ok = true;
    for (int q = 0; q < world && ok; ++q) {
      const uint64_t t0 = gtime_ns();
      while (ld_acquire_sys(&mine[q].epoch) != epoch) {
        if (gtime_ns() - t0 > timeout_ns) {
          atomicCAS(status, 0u, 0x200u | static_cast<unsigned>(q));
          ok = false;
          break;
        }
      }
    }
    if (ok) {
      // rank order: every rank adds the same numbers in the same order
      for (int q = 0; q < world; ++q) {
        const volatile Board* b = &mine[q];
        total += (double)b->sumsq;
        any = fmaxf(any, b->flag);
      }
    } else {
      any = 1.f;  // a timed-out step is never applied
    }
    out[0] = any > 0.f ? 1.f : 0.f;
    out[1] = (float)total;
    const float norm = sqrtf(out[1]);
    out[2] = norm;
    float coef = 1.f;
    if (max_norm > 0.0 && (double)norm > max_norm) coef = (float)(max_norm / ((double)norm + 1e-6));
    out[3] = coef;
  }
}

struct AdamArgs2 {
  float lr_neg, wd_term, b1, omb1, b2, omb2, bc1, bc2, eps, grad_mul;
};

__device__ __forceinline__ float adam_one(float& p, float& mm, float& vv, float graw, float coef,
                                          const AdamArgs2& a) {
  float g = graw * a.grad_mul;
  g = g * coef;
  if (a.wd_term != 0.f) p = p + a.wd_term * p;
  mm = mm * a.b1 + a.omb1 * g;
  vv = vv * a.b2 + a.omb2 * g * g;
  const float denom = sqrtf(vv / a.bc2) + a.eps;
  p = p + a.lr_neg * ((mm / a.bc1) / denom);
  return p;
}

// VECLOAD: master/m/v/grad are 16-byte aligned -> float4 accesses.  Each
// thread updates 16 bytes' worth of parameters (8 x 16-bit or 4 x fp32) and
// stores them to every rank with one 16-byte store per rank; the rank order
// starts at a different peer in each block, so the stores of one moment
// spread over all peers' links instead of queueing on rank 0's.
template <typename P, bool VECLOAD>
__global__ void __launch_bounds__(256)
adamw_fanout_kernel(float* __restrict__ master, float* __restrict__ m, float* __restrict__ v,
                    const float* __restrict__ grad, char* const* heaps, long long param_off,
                    long long s0, long long n, int world, const float* __restrict__ stats,
                    AdamArgs2 a) {
  ::msb::pdl_begin();
  if (stats[0] != 0.f) return;  // overflow: nothing changes on any rank
  const float coef = stats[3];
  constexpr int VEC = 16 / static_cast<int>(sizeof(P));
  const long long groups = (n + VEC - 1) / VEC;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const int q0 = (int)(blockIdx.x % (unsigned)world);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < groups; i += stride) {
    const long long e0 = i * VEC;
    const int cnt = (int)min((long long)VEC, n - e0);
    alignas(16) P outv[VEC];
    if (VECLOAD && cnt == VEC) {
#pragma unroll
      for (int h = 0; h < VEC / 4; ++h) {
        const long long e = e0 + 4 * h;
        float4 p4 = *reinterpret_cast<const float4*>(master + e);
        float4 m4 = *reinterpret_cast<const float4*>(m + e);
        float4 v4 = *reinterpret_cast<const float4*>(v + e);
        const float4 g4 = *reinterpret_cast<const float4*>(grad + e);
        outv[4 * h + 0] = from_f32<P>(adam_one(p4.x, m4.x, v4.x, g4.x, coef, a));
        outv[4 * h + 1] = from_f32<P>(adam_one(p4.y, m4.y, v4.y, g4.y, coef, a));
        outv[4 * h + 2] = from_f32<P>(adam_one(p4.z, m4.z, v4.z, g4.z, coef, a));
        outv[4 * h + 3] = from_f32<P>(adam_one(p4.w, m4.w, v4.w, g4.w, coef, a));
        *reinterpret_cast<float4*>(master + e) = p4;
        *reinterpret_cast<float4*>(m + e) = m4;
        *reinterpret_cast<float4*>(v + e) = v4;
      }
    } else {
#pragma unroll
      for (int k = 0; k < VEC; ++k) {
        if (k < cnt) {
          const long long e = e0 + k;
          float p = master[e], mm = m[e], vv = v[e];
          outv[k] = from_f32<P>(adam_one(p, mm, vv, grad[e], coef, a));
          master[e] = p;
          m[e] = mm;
          v[e] = vv;
        }
      }
    }
    for (int j = 0; j < world; ++j) {
      int q = q0 + j;
      if (q >= world) q -= world;
      P* dst = reinterpret_cast<P*>(heaps[q] + param_off) + s0 + e0;
      if (cnt == VEC && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(outv);
      } else {
#pragma unroll
        for (int k = 0; k < VEC; ++k)
          if (k < cnt) dst[k] = outv[k];
      }
    }
  }
  __threadfence_system();
}

// dst[i] = owner(i)'s shard element, for flat indices i in [lo, hi); owner
// q holds [q*shard, (q+1)*shard).  VEC elements (16 bytes) per access when the
// shard size, lo and both bases are 16-byte aligned (a vector then never
// crosses two owners).
template <typename T, int VEC>
__global__ void __launch_bounds__(256)
gather_range_kernel(char* const* heaps, long long shard_off, long long shard, long long lo,
                    long long hi, T* __restrict__ dst) {
  ::msb::pdl_begin();
  const long long nv = (hi - lo) / VEC;
  for (long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x; v < nv;
       v += (long long)gridDim.x * blockDim.x) {
    const long long i = lo + v * VEC;
    const int q = (int)(i / shard);
    const long long j = i - (long long)q * shard;
    const T* src = reinterpret_cast<const T*>(heaps[q] + shard_off) + j;
    if (VEC == 8) {
      *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(src);
    } else {
      dst[i] = *src;
    }
  }
}

}  // namespace

// ------------------------------------------------------------- host API
void peer_barrier(char* const* heaps, long long sync_off, int rank, int world, unsigned* ctr,
                  double timeout_s, unsigned* status, cudaStream_t st) {
  ::msb::launch(peer_barrier_kernel, 1, 32, 0, st, heaps, sync_off, rank, world, ctr,
                                        (unsigned long long)(timeout_s * 1e9), status);
  MSB_CHECK_LAUNCH("peer_barrier");
}

// threads: 256, or 128 for reductions that run beside other kernels (a
// 128 x 32-register block fits next to any of this library's large CTAs)
int rs_stats(char* const* heaps, long long grad_off, int dtype, long long s0, long long n,
             int world, float mul, const float* mul_dev, float* out, long long fanout_off,
             float* partials, unsigned* pflags, int max_blocks, bool aligned16, cudaStream_t st,
             int threads) {
  int blocks = 1;
  if (threads != 128) threads = 256;
  MSB_DISPATCH_FLOAT(dtype, T, {
    constexpr int V = 16 / sizeof(T);
    // vector loads need 16-byte aligned sources, vector stores an aligned out
    if (aligned16 && V == 8 && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
      blocks = grid_for(n / V, threads, max_blocks);
      ::msb::launch(rs_stats_kernel<T, 8>, blocks, threads, 0, st, heaps, grad_off, s0, n, world, mul,
                                                        mul_dev, out, fanout_off, partials, pflags);
    } else {
      blocks = grid_for(n, threads, max_blocks);
      ::msb::launch(rs_stats_kernel<T, 1>, blocks, threads, 0, st, heaps, grad_off, s0, n, world, mul,
                                                        mul_dev, out, fanout_off, partials, pflags);
    }
  });
  MSB_CHECK_LAUNCH("rs_stats");
  return blocks;
}

void stats_exchange(char* const* heaps, long long sync_off, int rank, int world, unsigned* ctr,
                    float* out, double max_norm, double timeout_s, unsigned* status,
                    cudaStream_t st) {
  ::msb::launch(stats_exchange_kernel, 1, 32, 0, st, heaps, sync_off, rank, world, ctr, out, max_norm,
                                          (unsigned long long)(timeout_s * 1e9), status);
  MSB_CHECK_LAUNCH("stats_exchange");
}

void adamw_fanout(float* master, float* m, float* v, const float* grad, char* const* heaps,
                  long long param_off, int pdtype, long long s0, long long n, int world,
                  const float* stats, double lr, double beta1, double beta2, double eps,
                  double wd, double bc1, double bc2, double grad_mul, cudaStream_t st) {
  AdamArgs2 a;
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
  const int per = pdtype == kF32 ? 4 : 8;
  const int blocks = grid_for(n / per + 1, 256, kNumSMs * 16);
  auto al = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  const bool vl = al(master) && al(m) && al(v) && al(grad);
#define MSB_FANOUT(P)                                                                        \
  if (vl)                                                                                    \
    ::msb::launch(adamw_fanout_kernel<P, true>, blocks, 256, 0, st, master, m, v, grad, heaps, param_off, \
                                                         s0, n, world, stats, a);            \
  else                                                                                       \
    ::msb::launch(adamw_fanout_kernel<P, false>, blocks, 256, 0, st, master, m, v, grad, heaps,         \
                                                          param_off, s0, n, world, stats, a);
  if (pdtype == kF16) {
    MSB_FANOUT(__half)
  } else if (pdtype == kBF16) {
    MSB_FANOUT(__nv_bfloat16)
  } else {
    MSB_FANOUT(float)
  }
#undef MSB_FANOUT
  MSB_CHECK_LAUNCH("adamw_fanout");
}

void gather_range(char* const* heaps, long long shard_off, long long shard, long long lo,
                  long long hi, void* dst, int dtype, bool aligned16, cudaStream_t st) {
  if (hi <= lo) return;
  MSB_DISPATCH_FLOAT(dtype, T, {
    constexpr int V = 16 / sizeof(T);
    if (aligned16 && V == 8 && shard % V == 0 && lo % V == 0 && hi % V == 0) {
      const int blocks = grid_for((hi - lo) / V, 256, kNumSMs * 8);
      ::msb::launch(gather_range_kernel<T, 8>, blocks, 256, 0, st, heaps, shard_off, shard, lo, hi,
                                                        static_cast<T*>(dst));
    } else {
      const int blocks = grid_for(hi - lo, 256, kNumSMs * 16);
      ::msb::launch(gather_range_kernel<T, 1>, blocks, 256, 0, st, heaps, shard_off, shard, lo, hi,
                                                        static_cast<T*>(dst));
    }
  });
  MSB_CHECK_LAUNCH("gather_range");
}

void gather_pull(char* const* heaps, long long shard_off, long long shard, int world, void* dst,
                 int dtype, bool aligned16, cudaStream_t st) {
  gather_range(heaps, shard_off, shard, 0, shard * world, dst, dtype, aligned16, st);
}

// --------------------------------------------------------- peer heap
void* peer_alloc(size_t bytes) {
  void* p = nullptr;
  check_cuda(cudaMalloc(&p, bytes), "peer heap cudaMalloc");
  check_cuda(cudaMemset(p, 0, bytes), "peer heap memset");
  return p;
}
void peer_free(void* p) { check_cuda(cudaFree(p), "peer heap cudaFree"); }
void peer_handle(void* p, char out[64]) {
  cudaIpcMemHandle_t h;
  check_cuda(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
  memcpy(out, &h, sizeof(h));
}
void* peer_open(const char handle[64]) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  check_cuda(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return p;
}
void peer_close(void* p) { check_cuda(cudaIpcCloseMemHandle(p), "cudaIpcCloseMemHandle"); }

}  // namespace msb
