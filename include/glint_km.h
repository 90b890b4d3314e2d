/* K-major GLINT decode: parent-only GEMV plus an activation-selected plug
 * correction (libglint_encode.so; additive, no counterpart in the reference's C
 * ABI).  Each entry point replaces one kernel of the reference's Mojo decoders
 * (Jadon-Fox/glint), with the same layout, rule and argument meaning:
 *
 *   glint_kmajor_from_rowmajor  transpose_plug (mojo/p7_glint_select_decode.mojo:120-135)
 *                               for hole and plug, transpose_scales
 *                               (mojo/p7_select_device.mojo:197-208)
 *   glint_gemv_km_stream        glint_gemv_km + gemv_km_combine
 *                               (mojo/p7_glint_gemv_km.mojo:17-95)
 *   glint_select_topk_stream    select_topk, default rule (mojo/p7_select_device.mojo:15-153)
 *   glint_apply_corr_k_stream   gather_rows_d + apply_corr_k (mojo/p7_select_device.mojo:
 *                               155-165, 210-238), the plug rows read in place
 *   glint_gemv_select_stream    the three above as one decode step
 *                               (p7_glint_select_decode.mojo's linear with kmaj)
 *
 * Layout of a weight [n, K] (n rows = outputs, K input channels, bs 64):
 *   plane_k[c * n/2 + r/2]: row r of channel c in nibble r & 1 (low nibble first),
 *   for the hole and the plug plane; scales_k[(c / 64) * n + r] = absmax[r * K/64 + c/64].
 * Arithmetic: y[r] = sum_c PARENT[h] * scale * x[c] (parent-only, M = 1); the
 * correction adds, over the selected channels c, (CELLS[h][p] - PARENT[h]) * scale
 * * x[c].  Selecting every channel gives the full GLINT GEMV.  f32 sums in a fixed
 * order (deterministic), not the reference's order: within 1e-5 * max(1, max|y|)
 * of an f64 sum.
 * Selection: key = BF16 bits & 0x7FFF; T = the largest key such that at least
 * nsel keys are >= T (0 if K < nsel); every channel with key >= T is kept, ties
 * included, indices ascending into d_idx (K ints), the count into *d_cnt (device);
 * nsel == 0 keeps none.
 * Limits: n % 8 == 0, K % 64 == 0, 64 <= K <= 65536, blocksize 64, 16-byte aligned
 * planes and scales; -1 otherwise (-2 for blocksize != 64).  plug_k may be device
 * memory or pinned (page-locked, mapped) host memory, whose device mapping the call
 * looks up; other host memory is refused with -1.  Only the selected channels'
 * plug rows are read.  All calls are asynchronous on `stream`;
 * the GEMV and correction use a per-stream scratch area (allocated on first use). */
#ifndef GLINT_KM_H_
#define GLINT_KM_H_
#include <cuda_runtime.h>
#include <stdint.h>

#include "glint_htile.h"
#ifdef __cplusplus
extern "C" {
#endif
int glint_kmajor_from_rowmajor(const uint8_t *d_hole, const uint8_t *d_plug, const float *d_absmax, int n, int K,
                               int blocksize, uint8_t *d_hole_k, uint8_t *d_plug_k, float *d_scales_k,
                               cudaStream_t stream);
int glint_gemv_km_stream(const uint8_t *d_hole_k, const float *d_scales_k, const glint_bf16_t *d_x, float *d_y,
                         int n, int K, cudaStream_t stream);
int glint_select_topk_stream(const glint_bf16_t *d_x, int K, int nsel, int *d_idx, int *d_cnt, cudaStream_t stream);
int glint_apply_corr_k_stream(const uint8_t *d_hole_k, const uint8_t *plug_k, const float *d_scales_k,
                              const glint_bf16_t *d_x, const int *d_idx, const int *d_cnt, float *d_y, int n, int K,
                              cudaStream_t stream);
int glint_gemv_select_stream(const uint8_t *d_hole_k, const uint8_t *plug_k, const float *d_scales_k,
                             const glint_bf16_t *d_x, float *d_y, int n, int K, int nsel, int *d_idx, int *d_cnt,
                             cudaStream_t stream);
#ifdef __cplusplus
}
#endif
#endif
