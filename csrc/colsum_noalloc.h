/* Column sums without device allocation: the C declaration.
 *
 * This entry point has no counterpart in the reference (minispeed has no
 * native code); it is an addition of this library, implemented in
 * colsum_noalloc.cu and exported from the extension's shared object.
 *
 * It is for callers that cannot call cudaMalloc (or any allocator) when they
 * run the operation: a runtime that plans all device memory once at start-up
 * and forbids allocation afterwards; code inside a process whose device
 * memory belongs to another framework's allocator, where a direct cudaMalloc
 * would escape that allocator's accounting; a caller that reaches this
 * library only through a C ABI with device pointers it already owns.
 *
 * out[c] (+)= sum over rows r of a[r, c] for a row-major [M, N] matrix with
 * row stride ld elements.  dtype: 0 fp32, 1 fp16, 2 bf16 (input and output
 * share it).  stream is a cudaStream_t (NULL: the legacy default stream).
 *
 * Scratch is a fixed 4 MiB array inside the library (every GPU that loads
 * the library holds it until exit), so N is limited to
 * MSB_COLSUM_NOALLOC_MAX_N columns.  The first call on a device, with that
 * device current, looks up the array's device address; make that call
 * before capturing any stream.  All calls share the array: calls that
 * overlap on the GPU (other streams, other host threads) race on it, so
 * serialize them.
 */
#ifndef MSB_COLSUM_NOALLOC_H
#define MSB_COLSUM_NOALLOC_H

#ifdef __cplusplus
extern "C" {
#endif

#define MSB_COLSUM_NOALLOC_MAX_N (1LL << 20)

/* return codes */
#define MSB_NOALLOC_OK 0
#define MSB_NOALLOC_BAD_ARGS (-1)   /* null pointer, M or N < 1, ld < N, unknown dtype */
#define MSB_NOALLOC_TOO_WIDE (-2)   /* N > MSB_COLSUM_NOALLOC_MAX_N; nothing launched */
#define MSB_NOALLOC_CUDA_ERROR (-3) /* device lookup, symbol lookup or launch failed */

int msb_colsum_noalloc(const void* a, int dtype, long long M, long long N, long long ld,
                       void* out, int accumulate, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MSB_COLSUM_NOALLOC_H */
