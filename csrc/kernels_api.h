// Host entry points of the CUDA kernels (raw pointers + stream).  Implemented
// in the .cu files of this directory; called from bindings.cpp.
#pragma once

#include <cuda_runtime.h>

// C entry point that allocates nothing (msb_colsum_noalloc); no counterpart
// in the reference
#include "colsum_noalloc.h"

namespace msb {

enum DType : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

long long launch_count();
void count_launch(int n);

// ---- bounds-checked debug build (-DMSB_BOUNDS_CHECK: the extension
// minispeed_b200._C_debug).  Every translation unit with checks keeps one
// record on the device: how many checks failed, and the site, index and
// limit of the first failure.  A failed check skips its access (a TMA load
// moves its x coordinate down to the aligned one, so its barrier still
// completes) and the kernel runs on; nothing traps.  The release build
// compiles every check away.
enum BoundsSite : int {
  kSiteNone = 0,
  kSiteEmbeddingToken = 1,  // token id outside [0, vocab) (embedding forward / backward)
  kSiteTarget = 2,          // cross-entropy target outside [0, V), not ignore_index
  kSiteTmaLoadX = 3,        // TMA load whose x coordinate is not 16-byte aligned
  kSiteTmaStoreXY = 4,      // TMA store / reduce at a negative or unaligned coordinate
  kSiteGemmSlot = 5,        // split-K / stream-K partial beyond the workspace
  kSiteGemmCounter = 6,     // stream-K / fixup tile counter beyond the counter array
  kSiteGemmColsum = 7,      // dGELU column-sum partial beyond [ceil(M / 32), N]
  kSiteCount = 8
};
struct BoundsRecord {
  unsigned long long count;
  long long site, index, limit;
};
bool bounds_check_build();
// one per translation unit: copy its record out, zero it when reset
void bounds_read_nn(BoundsRecord* out, bool reset);
void bounds_read_gemm(BoundsRecord* out, bool reset);
void bounds_read_attention(BoundsRecord* out, bool reset);

// ---- step pipeline (step_kernels.cu)
int grad_stats(const void* x, int dtype, long long n, float mul, float* partials,
               unsigned* flags, int max_blocks, cudaStream_t stream);
void stats_finalize(const float* partials, const unsigned* flags, int n, float* out,
                    double max_norm, bool epilogue, cudaStream_t stream);
void stats_epilogue(float* out, double max_norm, cudaStream_t stream);
void adamw(float* master, float* m, float* v, const void* grad, int gdtype, void* param_out,
           int pdtype, long long n, const float* stats, double lr, double beta1, double beta2,
           double eps, double wd, double bc1, double bc2, double grad_mul, cudaStream_t stream);
void cast_scale(const void* src, int sdtype, void* dst, int ddtype, long long n, float mul,
                cudaStream_t stream);

// ---- model kernels (nn_kernels.cu)
void add_norm_fwd(const void* x, const void* delta, const void* w, const void* b, void* s_out,
                  void* y, float* mean, float* rstd, int M, int C, float eps, bool rms,
                  int dtype, cudaStream_t st);
int norm_bwd(const void* dy, const void* s, const void* w, const float* mean, const float* rstd,
             const void* dres, void* dx, float* dw_part, float* db_part, int M, int C, bool rms,
             int dtype, int max_blocks, cudaStream_t st);
int colsum_partial(const void* a, float* part, int M, int N, long long ld, int dtype,
                   int max_chunks, cudaStream_t st);
void colsum_finish(const float* part, int nparts, int N, void* out, int dtype, int accumulate,
                   cudaStream_t st);
// One finish of a column-sum reduction: out[c] (+)= sum over the nparts fp32
// partial rows part[p * N + c].  colsum_finish_many runs up to
// kMaxColsumJobs of them (one output dtype) per launch; the jobs travel as
// the kernel's parameter, so a captured CUDA graph holds them by value.
struct ColsumJob {
  const float* part;
  void* out;
  int nparts;
  int N;
  int accumulate;
};
constexpr int kMaxColsumJobs = 48;
void colsum_finish_many(const ColsumJob* jobs, int njobs, int dtype, cudaStream_t st);
void accum_cast(const float* src, void* dst, long long n, int dtype, int accumulate,
                cudaStream_t st);
void bias_gelu_fwd(void* u, const void* bias, void* h, long long total, int N, int dtype,
                   cudaStream_t st);
void gelu_bwd(const void* dh, const void* u, void* du, long long total, int dtype,
              cudaStream_t st);
void swiglu_fwd(const void* gu, void* h, long long rows, int F, int dtype, cudaStream_t st);
void swiglu_bwd(const void* dh, const void* gu, void* dgu, long long rows, int F, int dtype,
                cudaStream_t st);
void cross_entropy_fwd(const void* logits, const long long* tgt, float* lse, float* loss_rows,
                       float* loss, float* inv_count, long long M, int V, long long ld,
                       long long ignore_index, int dtype, cudaStream_t st);
void cross_entropy_bwd(void* logits, const long long* tgt, const float* lse,
                       const float* grad_out, const float* inv_count, long long M, int V,
                       long long ld, long long ignore_index, int dtype, cudaStream_t st);
// forward + gradient for an expected upstream gradient *g_hint (logits are
// overwritten by the gradient); the rescale corrects it in backward when the
// real upstream gradient differs
void cross_entropy_fwd_grad(void* logits, const long long* tgt, float* lse, float* loss_rows,
                            float* loss, float* inv_count, const float* g_hint, long long M, int V,
                            long long ld, long long ignore_index, int dtype, cudaStream_t st);
void cross_entropy_grad_rescale(void* dlogits, long long M, int V, long long ld,
                                const float* grad_out, const float* g_hint, int dtype,
                                cudaStream_t st);
void embedding_fwd(const long long* idx, const void* wte, const void* wpe, void* out, long long M,
                   int T_len, int C, long long V, int dtype, cudaStream_t st);
// acc [V, C] fp32 and touched [V] must be all zero on entry and are left so
void embedding_bwd(const void* dout, const long long* idx, float* acc, unsigned char* touched,
                   void* dwte, int acc_wte, void* dwpe, int acc_wpe, long long M, int T_len,
                   int C, long long V, int dtype, cudaStream_t st);
void rope(void* x, const float* cos_t, const float* sin_t, long long BT, int T_len, int H, int D,
          long long row_stride, bool inverse, int dtype, cudaStream_t st);

// ---- tcgen05 GEMM (gemm_tcgen05.cu)
long long gemm_plan(int M, int N, int K, int num_sms, int* bn_out, int* splits_out);
// ---- attention (attention_tcgen05.cu): qkv is a row-major [B*T, n_cols] matrix
void attention_fwd(const void* qkv, long long ld_qkv, long long n_cols, int q_col, int k_col,
                   int v_col, void* out, long long ld_out, float* lse, int B, int T, int H,
                   int Hkv, int D, int dtype, float scale, unsigned* err, double timeout_s,
                   cudaStream_t st);
void attention_bwd(const void* qkv, long long ld_qkv, long long n_cols, int q_col, int k_col,
                   int v_col, const void* out, long long ld_out, const void* dout, long long ld_do,
                   const float* lse, float* delta, float* dq_acc, void* dqkv, long long ld_dqkv,
                   int B, int T, int H, int Hkv, int D, int dtype, float scale, unsigned* err,
                   double timeout_s, cudaStream_t st);

void gemm_tcgen05(const void* A, long long lda, int a_mn, const void* B, long long ldb, int b_mn,
                  void* C, long long ldc, const void* bias, int M, int N, int K, int dtype,
                  int accumulate, int mode, void* aux, long long ld_aux, float* ws,
                  long long ws_floats, unsigned* err, double timeout_s, cudaStream_t st,
                  int force_bn = 0, int force_splits = 0, int* sk_ctr = nullptr,
                  long long sk_ctr_n = 0, float* colsum_part = nullptr);
// colsum_part (mode 2 only): fp32 [ceil(M / 32), N] column sums of the stored
// output, one row per 32 output rows (finished by colsum_finish)
// stream-K (force_bn 512, force_splits -1): fp32 slots ws >= kStreamKSlotFloats
// per resident pair, and zeroed per-tile counters (left zero again)
constexpr long long kStreamKSlotFloats = 256LL * 256;
constexpr long long kStreamKCounters = 1LL << 16;

// ---- NVLink peer heap + fused collectives (collectives.cu)
// barrier-type kernels take this rank's device epoch counter (advanced by one each)
void peer_barrier(char* const* heaps, long long sync_off, int rank, int world, unsigned* ctr,
                  double timeout_s, unsigned* status, cudaStream_t st);
int rs_stats(char* const* heaps, long long grad_off, int dtype, long long s0, long long n,
             int world, float mul, const float* mul_dev, float* out, long long fanout_off,
             float* partials, unsigned* pflags, int max_blocks, bool aligned16, cudaStream_t st,
             int threads = 256);
void stats_exchange(char* const* heaps, long long sync_off, int rank, int world, unsigned* ctr,
                    float* out, double max_norm, double timeout_s, unsigned* status,
                    cudaStream_t st);
void adamw_fanout(float* master, float* m, float* v, const float* grad, char* const* heaps,
                  long long param_off, int pdtype, long long s0, long long n, int world,
                  const float* stats, double lr, double beta1, double beta2, double eps,
                  double wd, double bc1, double bc2, double grad_mul, cudaStream_t st);
void gather_pull(char* const* heaps, long long shard_off, long long shard, int world, void* dst,
                 int dtype, bool aligned16, cudaStream_t st);
void gather_range(char* const* heaps, long long shard_off, long long shard, long long lo,
                  long long hi, void* dst, int dtype, bool aligned16, cudaStream_t st);
void* peer_alloc(size_t bytes);
void peer_free(void* p);
void peer_handle(void* p, char out[64]);
void* peer_open(const char handle[64]);
void peer_close(void* p);

}  // namespace msb
