/* GLINT encode / expand C ABI (libglint_encode.so built from glint_b200/csrc).
 *
 * The first six declarations keep the reference's signatures unchanged
 * (Jadon-Fox/glint include/glint_encode.h:11-29, implemented there in
 * cuda/glint_encode.cu:128-262), so glint_cuda.py's ctypes bindings and C callers
 * link against this library as they are.  The rest are additive: stream-ordered
 * device-pointer entry points, a BF16 expand, batched calls over many tensors
 * and 64-bit size helpers.
 *
 * Return codes: 0 ok; -1 bad argument or host<->device copy failure; -3 device
 * allocation, launch or device error.  (-2 / -4, the reference's codebook-upload
 * failures, cannot occur: the codebook is compiled into the kernels.)
 */
#ifndef GLINT_ENCODE_H_
#define GLINT_ENCODE_H_
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif
struct CUstream_st;

/* Host pointers in and out; synchronous.  Input is streamed to the current GPU in
 * chunks, encoded and copied back with the copies overlapped; page-locked buffers
 * are read and written by DMA directly.  Replaces glint_encode.h:11-13. */
int glint_encode_bf16_host(
    const uint16_t *w_bf16, int64_t n, int blocksize,
    uint8_t *hole_packed, uint8_t *plug_packed, float *absmax);
/* f32 input, otherwise as above.  Replaces glint_encode.h:14-16. */
int glint_encode_f32_host(
    const float *w, int64_t n, int blocksize,
    uint8_t *hole_packed, uint8_t *plug_packed, float *absmax);
/* ceil(n / blocksize) (0 for blocksize <= 0), ceil(n / 2).  Return int like the
 * reference (glint_encode.h:17-18); see the *64 variants for larger tensors. */
int glint_encode_n_absmax(int64_t n, int blocksize);
int glint_encode_n_packed(int64_t n);
/* Host pointers; f32 out.  Replaces glint_encode.h:20-22. */
int glint_expand_packed_to_f32_host(
    const uint8_t *hole_packed, const uint8_t *plug_packed, const float *absmax,
    int64_t n, int blocksize, float *out_f32);
/* Device pointers, asynchronous on `stream`; f32 out.  n <= 0 returns 0.
 * Replaces glint_encode.h:26-29. */
int glint_expand_packed_to_f32_device(
    const uint8_t *d_hole_packed, const uint8_t *d_plug_packed, const float *d_absmax,
    int64_t n, int blocksize, float *d_out_f32, struct CUstream_st *stream);

/* ---- additive entry points (no counterpart in the reference ABI) ---------- */

int64_t glint_encode_n_absmax64(int64_t n, int blocksize);
int64_t glint_encode_n_packed64(int64_t n);

/* Device pointers, asynchronous on `stream`: the reference's encode without the
 * host round trip (its encode_dev_f32, cuda/glint_encode.cu:134-168, allocates
 * and copies back on every call). */
int glint_encode_bf16_device(
    const uint16_t *d_w_bf16, int64_t n, int blocksize,
    uint8_t *d_hole_packed, uint8_t *d_plug_packed, float *d_absmax, struct CUstream_st *stream);
int glint_encode_f32_device(
    const float *d_w, int64_t n, int blocksize,
    uint8_t *d_hole_packed, uint8_t *d_plug_packed, float *d_absmax, struct CUstream_st *stream);

/* Expand to BF16 (round to nearest even; a NaN absmax gives (bits >> 16) | 0x40),
 * the bytes glint_unpin.py writes (glint_unpin.py:25-31). */
int glint_expand_packed_to_bf16_device(
    const uint8_t *d_hole_packed, const uint8_t *d_plug_packed, const float *d_absmax,
    int64_t n, int blocksize, uint16_t *d_out_bf16, struct CUstream_st *stream);
int glint_expand_packed_to_bf16_host(
    const uint8_t *hole_packed, const uint8_t *plug_packed, const float *absmax,
    int64_t n, int blocksize, uint16_t *out_bf16);

/* One tensor of a batched call.  For encode, `dense` is the BF16 (or f32) input;
 * for expand it is the BF16 (or f32) output. */
typedef struct GlintTensorDesc {
    void *dense;
    uint8_t *hole_packed;
    uint8_t *plug_packed;
    float *absmax;
    int64_t n;
} GlintTensorDesc;

/* Encode / expand `count` tensors (device pointers) with few launches; the
 * descriptor array itself is host memory and is read before the call returns. */
int glint_encode_bf16_device_batch(
    const GlintTensorDesc *tensors, int count, int blocksize, struct CUstream_st *stream);
int glint_expand_packed_to_bf16_device_batch(
    const GlintTensorDesc *tensors, int count, int blocksize, struct CUstream_st *stream);

/* glint_encode_bf16_host / glint_encode_f32_host that also return, in *sum_sq_err,
 * the f64 sum over the n weights of (w - dequant(w))^2, dequant(w) being the f32
 * product GLINT_CELLS[h][p] * absmax that expand writes.  sqrt(*sum_sq_err / n)
 * is the rmse the reference pin tool reports per linear (glint_pin.py:66-72, from
 * glint_np.rmse of glint_np.expand, glint_np.py:93-95), here computed on the GPU
 * while the tensor streams through; the sum's order is fixed, so repeated calls
 * on one GPU give the same bits.  A null sum_sq_err returns -1. */
int glint_encode_bf16_host_sqerr(
    const uint16_t *w_bf16, int64_t n, int blocksize,
    uint8_t *hole_packed, uint8_t *plug_packed, float *absmax, double *sum_sq_err);
int glint_encode_f32_host_sqerr(
    const float *w, int64_t n, int blocksize,
    uint8_t *hole_packed, uint8_t *plug_packed, float *absmax, double *sum_sq_err);

/* Copies the compiled codebook GLINT_CELLS (16 x 16 f32, row-major: the pin's
 * `_glint_cells` tensor, glint_pin.py:158-159) into out[256]; returns 256, or -1
 * for a null out.  Needs no GPU. */
int glint_cells_f32(float *out);

#ifdef __cplusplus
}
#endif
#endif
