/* GLINT codec arithmetic shared by the sm_100a kernels and by host code.
 *
 * Everything here is __host__ __device__ so that the exact same source decides
 * codes on the GPU and in the host-side table builder / exhaustive checker.
 *
 * Encode rule (reference cuda/glint_encode.cu:80-102, glint_np.py:63-83):
 *   s = max |w| over the block (NaN skipped), v = (s == 0) ? 0 : RN(w / s),
 *   hole = first-minimum nearest of v among GLINT_PARENT,
 *   plug = first-minimum nearest of v within GLINT_CELLS[hole].
 * The combined code 16*hole + plug is a non-decreasing step function of v, so
 * it is fully described by 255 f32 thresholds.  A uniform grid of 513 cells over
 * [-1, 1] (cell = RN(256 v + 256)) holds at most one threshold per cell, so
 *   code(v) = cell_base[c] + (v >= cell_thr[c])
 * with one table read.  The tables are built on the host from the scan itself
 * (gen_lut.cpp) and checked against the CPU oracle over every f32 in [-1, 1].
 *
 * The divide uses Markstein's correction with a correctly rounded reciprocal
 * (P. Markstein, "Computation of elementary functions on the IBM RISC
 * System/6000 processor", IBM J. Res. Dev. 34(1), 1990): with y = RN(1/s) and
 * q = RN(w*y) within 1 ulp of w/s, r = w - q*s is exact (one fma) and RN(q + r*y)
 * equals RN(w/s) when nothing underflows.  Blocks whose s lies outside
 * [2^-60, 2^60] use the IEEE divide instead.  Quotients too small for the
 * theorem (|w/s| < 2^-20) still come out far below the smallest threshold
 * (|T| > 2.4e-3), where the code is constant.
 */
#ifndef GLINT_B200_CODEC_CUH_
#define GLINT_B200_CODEC_CUH_

#include <stdint.h>
#include <string.h>
#include <math.h>

#if defined(__CUDACC__)
#define GLINT_HD __host__ __device__ __forceinline__
#else
#define GLINT_HD static inline
#endif

namespace glint {

/* grid of the code lookup: cell_of(v) in [0, 2*kCellScale], 1/kCellScale wide in v */
constexpr int kCellScale = 256;
constexpr int kNumCells = 2 * kCellScale + 1; /* 513 */
/* 1.5 * 2^23: adding it to a value in [0, 2^22) leaves RN(value) in the low mantissa bits */
constexpr float kMagic = 12582912.0f;
constexpr uint32_t kMagicBits = 0x4B400000u;
/* blocks whose absmax lies in [kMarksteinLo, kMarksteinHi] use the reciprocal divide */
constexpr float kMarksteinLo = 8.67361737988403547206e-19f; /* 2^-60 */
constexpr float kMarksteinHi = 1.15292150460684697600e+18f; /* 2^60 */

GLINT_HD uint32_t f2u(float f)
{
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
#endif
}
GLINT_HD float u2f(uint32_t u)
{
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float f;
    memcpy(&f, &u, 4);
    return f;
#endif
}
GLINT_HD float fma_rn(float a, float b, float c)
{
#if defined(__CUDA_ARCH__)
    return __fmaf_rn(a, b, c);
#else
    return fmaf(a, b, c);
#endif
}
GLINT_HD float mul_rn(float a, float b)
{
#if defined(__CUDA_ARCH__)
    return __fmul_rn(a, b);
#else
    volatile float p = a * b; /* keeps the host compiler from contracting it */
    return p;
#endif
}
GLINT_HD float div_rn(float a, float b)
{
#if defined(__CUDA_ARCH__)
    return __fdiv_rn(a, b);
#else
    volatile float q = a / b;
    return q;
#endif
}
GLINT_HD float bf16_bits_to_f32(uint32_t b16) { return u2f(b16 << 16); }

/* Grid cell of a normalised value in [-1, 1]: key = RN(256 v + 256 + 1.5*2^23),
 * cell = bits(key) - bits(1.5*2^23) = RN(256 v + 256) in [0, 512].  One fma; the
 * kernels use it directly where v is known to lie in [-1, 1] (Markstein's
 * quotient of |w| <= s). */
GLINT_HD float cell_key(float v) { return fma_rn(v, (float)kCellScale, kMagic + (float)kCellScale); }

/* Clamped form for any v: NaN maps to -1 (code 0, what the reference scan gives
 * NaN), finite values outside [-1, 1] to the nearer end (the scan's answer too). */
GLINT_HD uint32_t cell_of(float v)
{
    return f2u(cell_key(fminf(fmaxf(v, -1.0f), 1.0f))) - kMagicBits;
}

/* One cell of the lookup table: the code at the cell's lowest value and the one
 * threshold inside the cell (+inf when there is none). */
struct CellEntry {
    float thr;
    uint32_t base;
};

GLINT_HD uint32_t code_from_entry(float v, CellEntry e)
{
    return e.base + (v >= e.thr ? 1u : 0u);
}

/* v = RN(w / s) for a block whose s passed the Markstein range check, y = RN(1/s). */
GLINT_HD float quotient_markstein(float w, float s, float y)
{
    float q = mul_rn(w, y);
    float r = fma_rn(-q, s, w);
    return fma_rn(r, y, q);
}

/* f32 -> BF16 bits, round to nearest even; NaN keeps its top bits and is quietened
 * (reference glint_np.py:25-31). */
GLINT_HD uint32_t f32_to_bf16_bits(float f)
{
    uint32_t u = f2u(f);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u)
        return (u >> 16) | 0x40u;
    return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}

} // namespace glint

#endif
