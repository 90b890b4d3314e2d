/* GLINT H-TILE dequant-GEMM / GEMV C ABI (libglint_encode.so).
 *
 * y[M,N] = x[M,K] * W^T with W[n,k] = GLINT_CELLS[hole][plug] * absmax[(n*K+k)/blocksize],
 * W packed over the flattened [N, K] index (lo nibble first), x BF16 [M, K] and
 * y [M, N] row-major, y overwritten.  Device pointers, enqueued on `stream`.
 *
 * The two reference entry points keep their signatures (Jadon-Fox/glint
 * include/glint_htile.h:11-19, cuda/glint_htile.cu:165-187) and f32-class
 * accuracy: every dequantised weight reaches the tensor cores as a BF16 hi/lo
 * pair, so y matches an f32 dot product to about 1e-6 relative.  Any M, N, K,
 * blocksize and pointer alignment is accepted.
 * Return codes: 0 ok, -1 null pointer or negative size, -2 blocksize <= 0,
 * -3 launch failure.
 */
#ifndef GLINT_HTILE_H_
#define GLINT_HTILE_H_
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif
int launch_glint_htile_s3_f32_stream(
    const uint8_t *d_hole, const uint8_t *d_plug, const float *d_absmax,
    const __nv_bfloat16 *d_x, float *d_y,
    int M, int N, int K, int blocksize, cudaStream_t stream);
/* Same on the legacy default stream. */
int launch_glint_htile_s3_f32(
    const uint8_t *d_hole, const uint8_t *d_plug, const float *d_absmax,
    const __nv_bfloat16 *d_x, float *d_y,
    int M, int N, int K, int blocksize);

/* ---- additive (no counterpart in the reference ABI) ----------------------- */
/* y dtype: GLINT_Y_F32 or GLINT_Y_BF16.  mode: GLINT_HTILE_PRECISE (as above) or
 * GLINT_HTILE_FAST, one BF16 value per weight (relative error <= 2^-9 per
 * weight; within max|y - y_ref| <= 1e-2 * max(1, max|y_ref|) of an f32
 * dequant-then-matmul at the shapes GLINT serves). */
#define GLINT_Y_F32 0
#define GLINT_Y_BF16 1
#define GLINT_HTILE_PRECISE 0
#define GLINT_HTILE_FAST 1
int glint_htile_stream(
    const uint8_t *d_hole, const uint8_t *d_plug, const float *d_absmax,
    const __nv_bfloat16 *d_x, void *d_y, int y_dtype,
    int M, int N, int K, int blocksize, int mode, cudaStream_t stream);

/* Same contract as glint_htile_stream for decode shapes, for callers that cannot
 * let a library allocate device memory (for example a serving process whose own
 * allocator already owns all free HBM, or an integration whose memory budget is
 * fixed before the first call).  No counterpart in the reference ABI.
 * It allocates nothing: the split-K partial sums and counters live in one 4 MiB
 * array compiled into the library, which every GPU that loads the library holds
 * until the process exits.  The first call on a device looks the array's device
 * address up; make that first call before any stream capture.  All calls share
 * the array, so calls that overlap on the GPU (other streams, other threads) race
 * and give wrong results; serialise them.  Limits: M <= 32, blocksize == 64,
 * K % 256 == 0, 16-byte aligned pointers (-1 otherwise), N <= 65536 and the
 * partial sums within the array (-5 GLINT_ERR_SCRATCH otherwise). */
#define GLINT_ERR_SCRATCH (-5)
int glint_htile_stream_noalloc(
    const uint8_t *d_hole, const uint8_t *d_plug, const float *d_absmax,
    const __nv_bfloat16 *d_x, void *d_y, int y_dtype,
    int M, int N, int K, int blocksize, int mode, cudaStream_t stream);
#ifdef __cplusplus
}
#endif
#endif
