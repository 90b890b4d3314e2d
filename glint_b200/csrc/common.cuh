/* Shared pieces of the GLINT sm_100a library: error codes, tables, small
 * device helpers.  Kernels live in encode.cu, expand.cu, htile_gemv.cu and
 * htile_gemm.cu; the C ABI in abi.cu.
 */
#ifndef GLINT_B200_COMMON_CUH_
#define GLINT_B200_COMMON_CUH_

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/glint_cells.h"
#include "glint_codec.cuh"
#include "glint_lut.inc"

namespace glint {

/* Return codes shared with the reference ABI (cuda/glint_encode.cu:134-262,
 * cuda/glint_htile.cu:170-179): 0 ok, -1 bad argument / host-device copy,
 * -2 blocksize, -3 allocation / launch / device error, -4 codebook. */
enum Status : int {
    kOk = 0,
    kBadArg = -1,
    kBadBlocksize = -2,
    kLaunch = -3,
    kCodebook = -4,
    kScratch = -5, /* the fixed scratch area is too small for this call */
    kUnsupported = -6, /* a shape or rank layout the gathered call does not cover */
};

/* Encode lookup table: {threshold bits, base code} per grid cell, generated at
 * build time by gen_lut.cpp (see glint_codec.cuh).  Each translation unit keeps
 * its own copy; kernels stage it into shared memory. */
static __device__ const uint2 g_encode_lut[kNumCells] = GLINT_LUT_INIT;
/* The codebook, GLINT_CELLS[hole][plug]. */
static __device__ const float g_cells[16][16] = GLINT_CELLS_INIT;

/* 32-bit index of a shared-memory address for inline PTX. */
__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }

/* Warp-shuffle max over aligned groups of G lanes (G a power of two <= 32).
 * fmaxf ignores NaN, as the reference absmax does ((NaN > m) is false). */
template <int G>
__device__ __forceinline__ float group_max(float v)
{
#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
    return v;
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
        v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
    return v;
}

inline bool aligned_to(const void *p, uintptr_t a) { return ((uintptr_t)p & (a - 1)) == 0; }

/* Read-and-clear of a kernel error word as one device atomic, so a bit that a
 * still-running kernel sets between a read and a reset cannot be lost. */
static __global__ void take_word_kernel(int *word, int *out) { *out = atomicExch(word, 0); }

/* Value of the __device__ int `word` of the calling translation unit; with `clear`,
 * taken and zeroed atomically (through `taken`, another __device__ int of that
 * unit).  Synchronous on the legacy default stream; -1 on a CUDA error. */
template <class W>
inline int read_error_word(W &word, W &taken, bool clear)
{
    int v = 0;
    if (!clear)
        return cudaMemcpyFromSymbol(&v, word, sizeof(int)) == cudaSuccess ? v : -1;
    void *pw = nullptr, *pt = nullptr;
    if (cudaGetSymbolAddress(&pw, word) != cudaSuccess || cudaGetSymbolAddress(&pt, taken) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    take_word_kernel<<<1, 1, 0, 0>>>(static_cast<int *>(pw), static_cast<int *>(pt));
    if (cudaGetLastError() != cudaSuccess || cudaMemcpyFromSymbol(&v, taken, sizeof(int)) != cudaSuccess)
        return -1;
    return v;
}

} // namespace glint

#endif
