/* INT8 W8A8 GEMM over a bf16_to_int8_pin_v1 linear, with the res4 late plug
 * (libglint_encode.so).  The declarations are the reference's
 * (Jadon-Fox/glint include/int8_mma_gemm.h:1-66, shipped there in libp7_kernels.so),
 * so callers compiled against that header link this library instead:
 *
 *   int8_mma_gemm            Y = X W^T, X quantized per (row, 64-block) on the fly
 *   int8_mma_gemm_plug       + the res4 plug as a second accumulating pass (scratch plug_i8)
 *   int8_mma_gemm_plug_fused the same sum in one pass (base and plug terms per block)
 *   int8_mma_gemm_resolve    + the activation's quantization residual as a second pass
 *
 * A linear: q I8 [n_out, k_in] row-major, scale F32 [n_out * k_in / 64]
 * (w[n, k] = q[n, k] * scale[n * (k_in / 64) + k / 64]).  Activations: s = amax / 127
 * of each 64-block of a row (1 for an all-zero block), xq = rint(x / s) clamped to
 * +-127.  Per 64-block, the int8 products are summed exactly in int32 and added to
 * the f32 result as ((float)sum * sx) * sw, blocks in K order; a plug nibble is
 * (nibble - 8), element 2i in the low nibble, with its own per-64 scale.
 * Requires k_in % 64 == 0 (and k_in >= 64), m, n_out >= 1, 16-byte aligned q, x and
 * scratch; cudaErrorInvalidValue otherwise.  y is fp32 [m, n_out] row-major.
 */
#ifndef GLINT_INT8_MMA_GEMM_H
#define GLINT_INT8_MMA_GEMM_H

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define INT8_MMA_BLOCK 64

typedef struct {
    const int8_t *q;
    const float *scale;
    int n_out;
    int k_in;
} Int8MmaLinear;

/* caller scratch for the activation quantization: xq [m, k_in] bytes, sx [m, k_in / 64] floats */
static inline size_t int8_mma_xq_bytes(int m, int k_in) { return (size_t)m * (size_t)k_in; }
static inline size_t int8_mma_sx_bytes(int m, int k_in)
{
    return (size_t)m * (size_t)(k_in / INT8_MMA_BLOCK) * sizeof(float);
}

cudaError_t int8_mma_gemm(const __nv_bfloat16 *x, Int8MmaLinear w, float *y, int m, int8_t *xq, float *sx,
                          cudaStream_t stream);
/* plug_q4: ceil(n_out * k_in / 2) bytes, plug_scale: one F32 per 64 weights, plug_i8:
 * n_out * k_in bytes of caller scratch */
cudaError_t int8_mma_gemm_plug(const __nv_bfloat16 *x, Int8MmaLinear w, const uint8_t *plug_q4,
                               const float *plug_scale, float *y, int m, int8_t *xq, float *sx, int8_t *plug_i8,
                               cudaStream_t stream);
cudaError_t int8_mma_gemm_plug_fused(const __nv_bfloat16 *x, Int8MmaLinear w, const uint8_t *plug_q4,
                                     const float *plug_scale, float *y, int m, int8_t *xq, float *sx,
                                     cudaStream_t stream);
/* rq/sr: scratch the size of xq/sx; the plug pointers are all NULL or all set */
cudaError_t int8_mma_gemm_resolve(const __nv_bfloat16 *x, Int8MmaLinear w, const uint8_t *plug_q4,
                                  const float *plug_scale, float *y, int m, int8_t *xq, float *sx, int8_t *rq,
                                  float *sr, int8_t *plug_i8, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif
