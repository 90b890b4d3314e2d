/* Host-side launchers shared between the kernel files and the C ABI (abi.cu). */
#ifndef GLINT_B200_INTERNAL_H_
#define GLINT_B200_INTERNAL_H_

#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace glint {

/* One tensor of an encode: BF16 bits (or f32) in, packed planes + absmax out. */
struct EncodeJob {
    const void *w;
    int64_t n;
    uint8_t *hole;
    uint8_t *plug;
    float *absmax;
};

/* One tensor of an expand: packed planes + absmax in, BF16 bits or f32 out. */
struct ExpandJob {
    const uint8_t *hole;
    const uint8_t *plug;
    const float *absmax;
    int64_t n;
    void *out;
};

enum OutKind : int { kOutF32 = 0, kOutBF16 = 1 };

/* H-TILE arithmetic: kPrecise splits every dequantised weight into a BF16 pair
 * (hi + lo) so the tensor-core sums match an f32 dot product to ~1e-6; kFast uses
 * one BF16 value per weight (relative error 2^-9 per weight). */
enum HtileMode : int { kPrecise = 0, kFast = 1 };

/* Launch the encode of `count` tensors with one blocksize on `stream`.  Returns a
 * Status (0 ok).  Device pointers; nothing is allocated. */
int encode_launch(const EncodeJob *jobs, int count, int blocksize, bool f32_in, cudaStream_t stream);

/* Launch the expand of `count` tensors. */
int expand_launch(const ExpandJob *jobs, int count, int blocksize, OutKind out, cudaStream_t stream);

/* Squared dequantisation error of one encoded tensor (or chunk): sq_error_grid(n)
 * f64 partial sums into `partial`, whose in-order total is
 * sum_i ((double)w_i - (double)(CELLS[h_i][p_i] * absmax[i / bs]))^2. */
constexpr int kSqErrThreads = 256;
constexpr int kMaxSqErrPartials = 1024;
int sq_error_grid(int64_t n);
int sq_error_launch(const void *w, bool f32_in, const uint8_t *hole, const uint8_t *plug, const float *absmax,
                    int64_t n, int blocksize, double *partial, cudaStream_t stream);

/* y[M,N] = x[M,K] . W^T with W dequantised from hole/plug/absmax. */
int htile_launch(const uint8_t *hole, const uint8_t *plug, const float *absmax, const __nv_bfloat16 *x,
                 void *y, OutKind y_kind, int M, int N, int K, int blocksize, HtileMode mode, cudaStream_t stream);

/* Decode-shaped path (tensor-core GEMV for K % 64 == 0 and bs % 64 == 0, generic otherwise). */
int htile_gemv_launch(const uint8_t *hole, const uint8_t *plug, const float *absmax, const __nv_bfloat16 *x,
                      void *y, OutKind y_kind, int M, int N, int K, int blocksize, HtileMode mode,
                      cudaStream_t stream);

/* Prefill-shaped path on tcgen05 tensor cores (GLINT_HTILE_FAST arithmetic). */
bool htile_gemm_supported(const uint8_t *hole, const uint8_t *plug, const float *absmax, const __nv_bfloat16 *x,
                          const void *y, bool y_bf16, int M, int N, int K, int blocksize);
int htile_gemm_launch(const uint8_t *hole, const uint8_t *plug, const float *absmax, const __nv_bfloat16 *x, void *y,
                      bool y_bf16, int M, int N, int K, int blocksize, cudaStream_t stream);
/* The same with the output gathered into every rank's y over peer memory (the
 * epilogue stores each tile into every rank's y[M, ldy] at column n0 + n). */
int htile_gemm_gather_launch(const uint8_t *hole, const uint8_t *plug, const float *absmax, const __nv_bfloat16 *x,
                             void *const *y_ranks, uint32_t *const *flag_ranks, int world, int rank, bool y_bf16,
                             int M, int N, int K, int ldy, int n0, cudaStream_t stream);
/* The same shapes in precise mode (f32-class: a fresh accumulator per 64-k block,
 * BF16 hi + lo weight halves, the blocks scaled and added in f32). */
int htile_gemm_precise_launch(const uint8_t *hole, const uint8_t *plug, const float *absmax, const __nv_bfloat16 *x,
                              void *y, bool y_bf16, int M, int N, int K, cudaStream_t stream);
/* The INT8 W8A8 GEMM (int8_mma_gemm contract, no fused plug) on tcgen05 kind::i8:
 * M > 64, K % 128 == 0, 16-byte aligned int8 operands; y (+)= bit for bit what the
 * mma.sync path gives. */
bool int8_tc_supported(const int8_t *xq, const int8_t *wq, const uint8_t *pq4, int M, int K);
cudaError_t int8_tc_gemm_launch(const int8_t *xq, const float *sx, const int8_t *wq, const float *sw,
                                const uint8_t *pq4, const float *psc, float *y, int M, int N, int K, int accumulate,
                                cudaStream_t stream); /* cudaErrorNotSupported: not launched */
/* Sticky error words written by kernels whose bounded waits ran out (0 = none),
 * one per kernel file; read_kernel_error ORs them. */
int read_kernel_error(bool clear);
int encode_error_word(bool clear);
int expand_error_word(bool clear);
int decode_error_word(bool clear);
int km_error_word(bool clear);
/* Decode-shaped path streamed through TMA (bs == 64, K % 256 == 0, M <= 32). */
bool htile_decode_supported(const uint8_t *hole, const uint8_t *plug, const float *absmax, const __nv_bfloat16 *x,
                            int M, int N, int K, int blocksize);
int htile_decode_launch(const uint8_t *hole, const uint8_t *plug, const float *absmax, const __nv_bfloat16 *x,
                        void *y, OutKind y_kind, int M, int N, int K, HtileMode mode, cudaStream_t stream);
/* The same decode path on the library's fixed per-device scratch array (no allocation). */
int htile_decode_launch_noalloc(const uint8_t *hole, const uint8_t *plug, const float *absmax,
                                const __nv_bfloat16 *x, void *y, OutKind y_kind, int M, int N, int K,
                                HtileMode mode, cudaStream_t stream);

/* Decode with the output gathered into every rank's y over peer memory
 * (1 <= M <= 32; kUnsupported otherwise). */
bool htile_gather_supported(int M, int N);
int htile_decode_gather_launch(const uint8_t *hole, const uint8_t *plug, const float *absmax,
                               const __nv_bfloat16 *x, void *const *y_ranks, uint32_t *const *flag_ranks,
                               int world, int rank, OutKind y_kind, int M, int N, int K, int ldy, int n0,
                               HtileMode mode, cudaStream_t stream);

/* K-major layout, parent-only decode GEMV and activation-selected plug correction
 * (kmajor.cu): n % 8 == 0, K % 64 == 0, K <= kKmMaxK, blocksize 64, 16-byte
 * aligned planes and scales. */
constexpr int kKmMaxK = 65536;
bool km_supported(int n, int K, const void *hole_k, const void *scales_k);
int km_layout_launch(const uint8_t *hole, const uint8_t *plug, const float *absmax, int n, int K, uint8_t *hole_k,
                     uint8_t *plug_k, float *scales_k, cudaStream_t stream);
int km_gemv_launch(const uint8_t *hole_k, const float *scales_k, const __nv_bfloat16 *x, float *y, int n, int K,
                   cudaStream_t stream);
int km_select_launch(const __nv_bfloat16 *x, int K, int nsel, int *idx, int *cnt, cudaStream_t stream);
int km_corr_launch(const uint8_t *hole_k, const uint8_t *plug_k, const float *scales_k, const __nv_bfloat16 *x,
                   const int *idx, const int *cnt, float *y, int n, int K, cudaStream_t stream);
int km_gemv_select_launch(const uint8_t *hole_k, const uint8_t *plug_k, const float *scales_k,
                          const __nv_bfloat16 *x, float *y, int n, int K, int nsel, int *idx, int *cnt,
                          cudaStream_t stream);

/* cuTensorMapEncodeTiled through the runtime's driver entry point (nullptr when the
 * driver does not offer it); looked up once. */
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

/* A [M, cols] column shard stored into every rank's y [M, ldy] at column n0 over
 * peer memory, with the gathered decode's completion protocol. */
int gather_copy_launch(const void *src, int elem_bytes, int M, int cols, int ld_src, void *const *y_ranks,
                       uint32_t *const *flag_ranks, int world, int rank, int ldy, int n0, cudaStream_t stream);

/* SM count of the current device (cached per device). */
int sm_count();
/* Raise a kernel's dynamic shared memory limit once per device. */
bool ensure_smem(const void *kernel, int bytes);

} // namespace glint

#endif
