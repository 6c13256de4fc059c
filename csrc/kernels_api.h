// Host entry points of the CUDA kernels (raw pointers + stream).  Implemented
// in the .cu files of this directory; called from bindings.cpp.
#pragma once

#include <cuda_runtime.h>

namespace msb {

enum DType : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

long long launch_count();

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

}  // namespace msb
