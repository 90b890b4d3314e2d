/* GLINT H-TILE dequant-GEMM / GEMV C ABI (libglint_encode.so).
 *
 * y[M,N] = x[M,K] * W^T with W[n,k] = GLINT_CELLS[hole][plug] * absmax[(n*K+k)/blocksize],
 * W packed over the flattened [N, K] index (lo nibble first), x BF16 [M, K] and
 * y [M, N] row-major, y overwritten.  Device pointers, enqueued on `stream`.
 *
 * The two reference entry points keep their signatures (Jadon-Fox/glint
 * include/glint_htile.h:11-19, cuda/glint_htile.cu:165-187) and f32-class
 * accuracy: each codebook cell reaches the tensor cores as a BF16 hi/lo pair
 * (about 17 significant bits), every 64-k absmax block is summed in a fresh
 * accumulator and the blocks are scaled and added in f32, so y is within
 * 1e-5 * (1 + |y|) of an f32 dot product on the reference's device-test shapes
 * and within 1e-5 * max(1, max|y|) at K up to 14336.  Any M, N, K, blocksize and
 * pointer alignment is accepted.
 * Return codes: 0 ok, -1 null pointer or negative size, -2 blocksize <= 0,
 * -3 launch failure.
 */
#ifndef GLINT_HTILE_H_
#define GLINT_HTILE_H_
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
/* BF16 activations are passed by pointer.  C++ (CUDA) callers see exactly the
 * reference's __nv_bfloat16; cuda_bf16.h declares that type for C++ only, so C
 * translation units get its 16-bit storage struct, which has the same layout. */
#ifdef __cplusplus
typedef __nv_bfloat16 glint_bf16_t;
#else
typedef __nv_bfloat16_raw glint_bf16_t;
#endif
#ifdef __cplusplus
extern "C" {
#endif
int launch_glint_htile_s3_f32_stream(
    const uint8_t *d_hole, const uint8_t *d_plug, const float *d_absmax,
    const glint_bf16_t *d_x, float *d_y,
    int M, int N, int K, int blocksize, cudaStream_t stream);
/* Same on the legacy default stream. */
int launch_glint_htile_s3_f32(
    const uint8_t *d_hole, const uint8_t *d_plug, const float *d_absmax,
    const glint_bf16_t *d_x, float *d_y,
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
    const glint_bf16_t *d_x, void *d_y, int y_dtype,
    int M, int N, int K, int blocksize, int mode, cudaStream_t stream);

/* Same contract as glint_htile_stream for decode shapes, for callers that cannot
 * let a library allocate device memory (for example a serving process whose own
 * allocator already owns all free HBM, or an integration whose memory budget is
 * fixed before the first call).  No counterpart in the reference ABI.
 * It allocates nothing: the split-K partial sums and counters live in one 4 MiB
 * array compiled into the library, which every GPU that loads the library holds
 * until the process exits.  The first call on a device (and the first after a
 * device reset) looks the array's device address up; make that first call before
 * any stream capture.  All calls share the array, so calls that overlap on the
 * GPU (other streams, other threads) race and give wrong results; serialise them.
 * Limits: M <= 32, blocksize == 64, K % 256 == 0, 16-byte aligned pointers (-1
 * otherwise); N <= 65536, else -5 GLINT_ERR_SCRATCH.
 * Only stream-K shapes use the array: N < 16, N > 224 x SMs (33152 on a B200's
 * 148 SMs), or N < 16 x SMs with K > 8192; the others need no scratch.  Those
 * return -5 unless their partial sums fit 4 MiB - 64 KiB:
 *   rb x parts x 256 x 8 MT x 4 bytes <= 4128768, where
 *   MT = 1 (M <= 8), 2 (M <= 16), 4 (M <= 32); ku = K / 256 (M <= 16) or K / 128;
 *   rb = ceil(N / 256); units = rb x ku; ctas = min(units, SMs);
 *   parts = min(ctas, ceil(ku / max(1, floor(units / ctas))) + 1).
 * On 148 SMs, for example: M <= 8 covers N up to about 64000 at any K; M = 4,
 * N = 1024, K = 14336 fits (1.9 MB); M = 16, N = 1024, K = 16384 (4.3 MB) and
 * M = 1, N = 65536, K = 4096 (4.2 MB) return -5. */
#define GLINT_ERR_SCRATCH (-5)
int glint_htile_stream_noalloc(
    const uint8_t *d_hole, const uint8_t *d_plug, const float *d_absmax,
    const glint_bf16_t *d_x, void *d_y, int y_dtype,
    int M, int N, int K, int blocksize, int mode, cudaStream_t stream);

/* Column-parallel decode with the all-gather fused in (one process per GPU; no
 * counterpart in the reference, which runs on one device).  This rank holds rows
 * [n0, n0 + N) of a weight with ld_y rows in all; the call computes them and
 * stores them straight into every rank's y[M, ld_y] (d_y_ranks[r]: rank r's
 * buffer as mapped in this process, this rank's own at d_y_ranks[rank]) over
 * NVLink, then signals every rank (d_flag_ranks[r]: rank r's counters, 9
 * zero-initialised uint32 per rank) and waits for one signal from every rank.
 * When the call completes on `stream`, this rank's y holds every rank's rows.
 * Every rank must make every gathered call of the group, in the same order (a
 * missing rank makes the others give up after about a second with
 * glint_kernel_error() = 1); the same launch may be replayed in a CUDA graph.
 * Peer buffers come from glint_device_alloc and are shared with
 * glint_ipc_handle / glint_ipc_open.
 * Covers bs == 64, K % 256 == 0, 16-byte aligned operands, world <= 8, and
 * 1 <= M <= 32 (the decode kernels, either mode) or M >= 128 in fast mode (the
 * prefill GEMM, whose epilogue stores each finished tile into every rank's y
 * while later tiles compute); else GLINT_ERR_UNSUPPORTED.  The calls of a group
 * go on one stream per rank. */
#define GLINT_ERR_UNSUPPORTED (-6)
int glint_htile_gather_stream(
    const uint8_t *d_hole, const uint8_t *d_plug, const float *d_absmax,
    const glint_bf16_t *d_x, void *const *d_y_ranks, unsigned int *const *d_flag_ranks,
    int world, int rank, int y_dtype, int M, int N, int K, int ld_y, int n0,
    int blocksize, int mode, cudaStream_t stream);
/* A column shard gathered into every rank's buffer, on the same counters and with the
 * same rules as glint_htile_gather_stream: src [M, cols] (row stride ld_src elements,
 * elem_bytes 2 or 4) is stored into columns [n0, n0 + cols) of every rank's
 * y [M, ld_y]; when the call completes on `stream`, this rank's y holds every rank's
 * columns.  For activations that feed a column-parallel linear (e.g. the heads of an
 * attention output).  -6 for another element size. */
int glint_gather_stream(const void *d_src, int elem_bytes, int M, int cols, int ld_src, void *const *d_y_ranks,
                        unsigned int *const *d_flag_ranks, int world, int rank, int ld_y, int n0,
                        cudaStream_t stream);
/* Zero-initialised device memory that can be shared with other processes
 * (cudaMalloc'd, so glint_ipc_handle covers exactly this range). */
int glint_device_alloc(size_t bytes, void **d_ptr);
int glint_device_free(void *d_ptr);
/* CUDA IPC: a 64-byte handle for a glint_device_alloc pointer, and its mapping in
 * another process on the same node (peer access enabled on open). */
int glint_ipc_handle(const void *d_ptr, void *handle_out);
int glint_ipc_open(const void *handle, void **d_ptr);
int glint_ipc_close(void *d_ptr);
#ifdef __cplusplus
}
#endif
#endif
