/* GLINT CPU oracle — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's kernel-exact GLINT codec, used as the
 * checker for the CUDA library in tests/, in __graft_entry__.smoke() and as the
 * timed CPU baseline in bench.py.  Nothing in the product (glint_b200/) links,
 * loads or calls this file.
 *
 * Every function follows one reference function, cited as path:line inside
 * Jadon-Fox/glint:
 *   - block absmax        cuda/glint_encode.cu:41-66, glint_np.py:32-40
 *   - nearest16           cuda/glint_encode.cu:67-79 (first minimum, strict <),
 *                         glint_np.py:41-52
 *   - encode (pack)       cuda/glint_encode.cu:80-102, glint_np.py:53-83
 *   - BF16 widening       cuda/glint_encode.cu:35-40, glint_np.py:16-19
 *   - expand (f32)        cuda/glint_encode.cu:103-114, glint_np.py:84-92
 *   - f32 -> BF16 RNE     glint_np.py:25-31, dtype_io.py:32-42
 *   - H-TILE reference    cuda/glint_htile.cu:124-164 (weights dequantised in
 *                         f32, products accumulated in f64 as in
 *                         tests/test_htile_k_bounds_device.cu:90-95)
 *   - INT8 W8A8 GEMM, res4 plug cuda/int8_mma_gemm.cu:10-240 (activation quantization,
 *                         per-block int32 dots, f32 scaling order); checked on the GPU
 *                         against that file built unchanged for sm_100a (oracle/_ref)
 *   - K-major layout, parent-only GEMV, channel selection, plug correction
 *                         mojo/p7_glint_select_decode.mojo:120-143,
 *                         mojo/p7_glint_gemv_km.mojo:17-95,
 *                         mojo/p7_select_device.mojo:15-153, 197-238
 *                         (no Mojo toolchain here and no reference vectors: the sum
 *                         parent + full correction is pinned to the H-TILE goldens;
 *                         the parent-only values and the selection rule are parity
 *                         unpinned against the reference's own outputs)
 * Parity is pinned against golden vectors that tests/golden/make_golden.py wrote
 * by running the reference's own glint_np.py / glint_htile_sim.py.
 *
 * Build (oracle/Makefile): gcc -O2 -fopenmp -shared -fPIC.  Never with
 * -ffast-math: the divide must stay IEEE round-to-nearest and denormals must
 * not be flushed.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif
#include "../include/glint_cells.h"

static int g_threads = 1;

void orc_set_threads(int t) { g_threads = t > 0 ? t : 1; }
int orc_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_num_procs();
#else
    return 1;
#endif
}

/* cuda/glint_encode.cu:67-79: linear scan, strict < so the first minimum wins.
 * NaN v makes every comparison false and returns 0. */
static inline int nearest16(const float *tab, float v)
{
    int best = 0;
    float bd = fabsf(v - tab[0]);
    for (int k = 1; k < 16; ++k) {
        float d = fabsf(v - tab[k]);
        if (d < bd) {
            bd = d;
            best = k;
        }
    }
    return best;
}

/* Combined code 16*hole + plug of one normalised value v (glint_encode.cu:91-92). */
int orc_code(float v)
{
    int h = nearest16(GLINT_PARENT, v);
    int p = nearest16(GLINT_CELLS[h], v);
    return (h << 4) | p;
}

/* Codes for a contiguous range of f32 bit patterns [lo, lo+count). */
void orc_codes_for_bits(uint32_t lo, int64_t count, uint8_t *out)
{
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (int64_t i = 0; i < count; ++i) {
        uint32_t u = lo + (uint32_t)i;
        float v;
        memcpy(&v, &u, 4);
        out[i] = (uint8_t)orc_code(v);
    }
}

static inline float bf16_to_f32(uint16_t b)
{
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* glint_np.py:25-31: round to nearest even; NaN keeps its top bits and is quietened. */
uint16_t orc_f32_to_bf16(float f)
{
    uint32_t u;
    memcpy(&u, &f, 4);
    if (isnan(f))
        return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

/* cuda/glint_encode.cu:41-66: max |w| over each block, NaN skipped because
 * (NaN > m) is false; the last block is padded with zeros. */
static void block_absmax_f32(const float *w, int64_t n, int bs, float *am)
{
    int64_t nb = (n + bs - 1) / bs;
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (int64_t b = 0; b < nb; ++b) {
        float m = 0.f;
        int64_t e = (b + 1) * (int64_t)bs < n ? (b + 1) * (int64_t)bs : n;
        for (int64_t i = b * (int64_t)bs; i < e; ++i) {
            float a = fabsf(w[i]);
            if (a > m)
                m = a;
        }
        am[b] = m;
    }
}

/* One weight: v = (s == 0) ? 0 : w / s (IEEE f32 divide), then the two scans
 * (cuda/glint_encode.cu:89-92). */
static inline int encode_one(float w, float s)
{
    float v = (s == 0.f) ? 0.f : (w / s);
    return orc_code(v);
}

/* cuda/glint_encode.cu:80-102 over the whole tensor: byte e holds element 2e in
 * the low nibble and element 2e+1 in the high nibble; the pad nibble of an odd n
 * is 0 in both planes. */
static void encode_pack_f32(const float *w, int64_t n, int bs, const float *am,
                            uint8_t *hole, uint8_t *plug)
{
    int64_t npack = (n + 1) / 2;
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (int64_t e = 0; e < npack; ++e) {
        int64_t i0 = 2 * e, i1 = i0 + 1;
        int c0 = encode_one(w[i0], am[i0 / bs]);
        int c1 = 0;
        if (i1 < n)
            c1 = encode_one(w[i1], am[i1 / bs]);
        hole[e] = (uint8_t)(((c0 >> 4) & 15) | (((c1 >> 4) & 15) << 4));
        plug[e] = (uint8_t)((c0 & 15) | ((c1 & 15) << 4));
    }
}

/* glint_np.encode_f32 (glint_np.py:63-83). Returns 0, or -1 for bs <= 0. */
int orc_encode_f32(const float *w, int64_t n, int bs, uint8_t *hole, uint8_t *plug, float *am)
{
    if (bs <= 0)
        return -1;
    if (n <= 0)
        return 0;
    block_absmax_f32(w, n, bs, am);
    encode_pack_f32(w, n, bs, am, hole, plug);
    return 0;
}

/* glint_np.encode_f32(glint_np.dense_to_f32("BF16", raw, n), bs): the BF16 bits
 * are widened exactly (glint_np.py:17-19, cuda/glint_encode.cu:35-40), then the
 * f32 encode runs block by block without a full f32 copy. */
int orc_encode_bf16(const uint16_t *wb, int64_t n, int bs, uint8_t *hole, uint8_t *plug, float *am)
{
    if (bs <= 0)
        return -1;
    if (n <= 0)
        return 0;
    int64_t nb = (n + bs - 1) / bs;
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (int64_t b = 0; b < nb; ++b) {
        float m = 0.f;
        int64_t e = (b + 1) * (int64_t)bs < n ? (b + 1) * (int64_t)bs : n;
        for (int64_t i = b * (int64_t)bs; i < e; ++i) {
            float a = fabsf(bf16_to_f32(wb[i]));
            if (a > m)
                m = a;
        }
        am[b] = m;
    }
    int64_t npack = (n + 1) / 2;
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (int64_t e = 0; e < npack; ++e) {
        int64_t i0 = 2 * e, i1 = i0 + 1;
        int c0 = encode_one(bf16_to_f32(wb[i0]), am[i0 / bs]);
        int c1 = 0;
        if (i1 < n)
            c1 = encode_one(bf16_to_f32(wb[i1]), am[i1 / bs]);
        hole[e] = (uint8_t)(((c0 >> 4) & 15) | (((c1 >> 4) & 15) << 4));
        plug[e] = (uint8_t)((c0 & 15) | ((c1 & 15) << 4));
    }
    return 0;
}

static inline float dequant(const uint8_t *hole, const uint8_t *plug, const float *am, int64_t i, int bs)
{
    int sh = (int)(i & 1) * 4;
    int h = (hole[i >> 1] >> sh) & 15;
    int p = (plug[i >> 1] >> sh) & 15;
    return GLINT_CELLS[h][p] * am[i / bs];
}

/* cuda/glint_encode.cu:103-114 / glint_np.py:84-92: out[i] = cells[h][p] * absmax[i / bs],
 * one f32 multiply. */
int orc_expand_f32(const uint8_t *hole, const uint8_t *plug, const float *am, int64_t n, int bs, float *out)
{
    if (bs <= 0)
        return -1;
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (int64_t i = 0; i < n; ++i)
        out[i] = dequant(hole, plug, am, i, bs);
    return 0;
}

/* glint_unpin._expand for BF16 (glint_unpin.py:25-31): f32 expand, then RNE to BF16. */
int orc_expand_bf16(const uint8_t *hole, const uint8_t *plug, const float *am, int64_t n, int bs, uint16_t *out)
{
    if (bs <= 0)
        return -1;
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (int64_t i = 0; i < n; ++i)
        out[i] = orc_f32_to_bf16(dequant(hole, plug, am, i, bs));
    return 0;
}

/* H-TILE reference: y[m,n] = sum_k cells[h][p]*absmax[(nK+k)/bs] * x[m,k]
 * (cuda/glint_htile.cu:147-158), x BF16 row-major [M,K], W packed over the
 * flattened [N,K] index, y f32 row-major [M,N].  The dequantised weight is the
 * f32 product (as the kernel forms it); the sum runs in f64 with k ascending. */
int orc_htile(const uint8_t *hole, const uint8_t *plug, const float *am, const uint16_t *x,
              float *y, int M, int N, int K, int bs)
{
    if (bs <= 0)
        return -2;
#pragma omp parallel for num_threads(g_threads) schedule(static) collapse(2)
    for (int m = 0; m < M; ++m) {
        for (int nn = 0; nn < N; ++nn) {
            double acc = 0.0;
            for (int k = 0; k < K; ++k) {
                int64_t i = (int64_t)nn * K + k;
                acc += (double)dequant(hole, plug, am, i, bs) * (double)bf16_to_f32(x[(int64_t)m * K + k]);
            }
            y[(int64_t)m * N + nn] = (float)acc;
        }
    }
    return 0;
}

/* ---- K-major layout, parent-only GEMV, activation-selected plug correction ----
 * The reference's Mojo decoders (mojo/p7_glint_gemv_km.mojo, mojo/p7_select_device.mojo,
 * mojo/p7_glint_select_decode.mojo).  A weight [n, K] (bs 64, K % 64 == 0, n even)
 * in K-major form: plane_k[c * n/2 + r/2] holds row r of input channel c in nibble
 * r & 1 (low nibble first); scales_k[(c / 64) * n + r] = absmax[r * K/64 + c / 64]. */

/* transpose_plug (mojo/p7_glint_select_decode.mojo:120-135), applied to both planes,
 * and transpose_scales (mojo/p7_select_device.mojo:197-208). */
int orc_to_kmajor(const uint8_t *hole, const uint8_t *plug, const float *am, int n, int K, uint8_t *hole_k,
                  uint8_t *plug_k, float *scales_k)
{
    if (n <= 0 || K <= 0 || (n & 1) || K % 64)
        return -1;
    const int64_t half = n / 2;
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (int64_t g = 0; g < (int64_t)K * half; ++g) {
        const int64_t c = g / half, b = g - c * half;
        const int64_t j0 = (2 * b) * (int64_t)K + c, j1 = (2 * b + 1) * (int64_t)K + c;
        hole_k[g] = (uint8_t)(((hole[j0 >> 1] >> (4 * (j0 & 1))) & 15) | (((hole[j1 >> 1] >> (4 * (j1 & 1))) & 15) << 4));
        if (plug && plug_k)
            plug_k[g] =
                (uint8_t)(((plug[j0 >> 1] >> (4 * (j0 & 1))) & 15) | (((plug[j1 >> 1] >> (4 * (j1 & 1))) & 15) << 4));
    }
    const int cb_n = K / 64;
    for (int64_t g = 0; g < (int64_t)n * cb_n; ++g) {
        const int64_t r = g / cb_n, cb = g - r * cb_n;
        scales_k[cb * n + r] = am[g];
    }
    return 0;
}

static inline int nib_k(const uint8_t *plane_k, int64_t half, int64_t c, int64_t r)
{
    return (plane_k[c * half + (r >> 1)] >> (4 * (r & 1))) & 15;
}

/* glint_gemv_km + gemv_km_combine (mojo/p7_glint_gemv_km.mojo:17-95): y[r] =
 * sum_c (PARENT[h] * scales_k[c/64][r]) * x[c], M = 1, in the reference's order:
 * channels ascending within each of ksg equal slices (f32, one product rounded,
 * then the multiply by x, then the add), slices added in order.  The reference
 * takes its 16 parent values from a table built as t0[h*16 + p] = PARENT[h]
 * (make_tables, mojo/p7_glint_select_decode.mojo:136-143). */
int orc_gemv_km(const uint8_t *hole_k, const float *scales_k, const uint16_t *x, float *y, int n, int K, int ksg)
{
    if (n <= 0 || K <= 0 || (n % 8) || ksg <= 0 || K % (64 * ksg))
        return -1;
    const int64_t half = n / 2;
    const int kslice = K / ksg;
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (int r = 0; r < n; ++r) {
        float tot = 0.f;
        for (int s = 0; s < ksg; ++s) {
            float a = 0.f;
            for (int c = s * kslice; c < (s + 1) * kslice; ++c) {
                const float t = GLINT_PARENT[nib_k(hole_k, half, c, r)] * scales_k[(int64_t)(c / 64) * n + r];
                a += t * bf16_to_f32(x[c]);
            }
            tot = s == 0 ? a : tot + a;
        }
        y[r] = tot;
    }
    return 0;
}

/* select_topk with its default rule (mojo/p7_select_device.mojo:15-153, tkey = 0,
 * nfloor = 0): key = BF16 bits & 0x7FFF; T = the largest 15-bit value such that at
 * least nsel keys are >= T (T = 0 when fewer than nsel channels exist); nsel == 0
 * selects nothing.  Every channel with key >= T is kept (ties all kept), indices
 * ascending.  Returns the count, or -1 for nsel < 0. */
int orc_select_topk(const uint16_t *x, int K, int nsel, int32_t *idx)
{
    if (nsel < 0 || K < 0)
        return -1;
    int thr = 0;
    for (int bi = 0; bi < 15; ++bi) {
        const int cand = thr | (1 << (14 - bi));
        int c = 0;
        for (int i = 0; i < K; ++i)
            c += (x[i] & 0x7FFF) >= cand;
        if (c >= nsel)
            thr = cand;
    }
    if (nsel == 0)
        thr = 32768;
    int cnt = 0;
    for (int i = 0; i < K; ++i)
        if ((x[i] & 0x7FFF) >= thr)
            idx[cnt++] = i;
    return cnt;
}

/* apply_corr_k (mojo/p7_select_device.mojo:210-238) with the staged plug rows read
 * in place from plug_k: y[r] = y[r] + sum_{i < cnt} (delta[h][p] * scales_k[c/64][r])
 * * x[c], c = idx[i] in list order, f32, delta = CELLS[h][p] - PARENT[h] (make_tables,
 * mojo/p7_glint_select_decode.mojo:136-143). */
int orc_apply_corr_k(const uint8_t *hole_k, const uint8_t *plug_k, const float *scales_k, const uint16_t *x,
                     const int32_t *idx, int cnt, float *y, int n, int K)
{
    if (n <= 0 || K <= 0 || (n & 1) || cnt < 0)
        return -1;
    const int64_t half = n / 2;
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (int r = 0; r < n; ++r) {
        float acc = 0.f;
        for (int i = 0; i < cnt; ++i) {
            const int64_t c = idx[i];
            const int h = nib_k(hole_k, half, c, r), p = nib_k(plug_k, half, c, r);
            const float d = GLINT_CELLS[h][p] - GLINT_PARENT[h];
            acc += (d * scales_k[(c / 64) * n + r]) * bf16_to_f32(x[c]);
        }
        y[r] = y[r] + acc;
    }
    return 0;
}

/* ---- INT8 W8A8 GEMM and the res4 late plug (cuda/int8_mma_gemm.cu) ------------ */

/* k_quant_act (cuda/int8_mma_gemm.cu:10-29); with xq_prev, k_quant_act_resid
 * (:170-189), whose x - xq * sx the reference's compiler fuses into one step.  Per
 * (row, 64-block): s = amax / 127 (1 when amax == 0), q = rint(w / s) clamped to
 * +-127. */
int orc_int8_quant(const uint16_t *x, const int8_t *xq_prev, const float *sx_prev, int m, int k, int8_t *q,
                   float *s)
{
    if (m < 1 || k < 64 || k % 64)
        return -1;
    const int nkb = k / 64;
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (int item = 0; item < m * nkb; ++item) {
        const int row = item / nkb, kb = item % nkb;
        float w[64], am = 0.f;
        for (int j = 0; j < 64; ++j) {
            const int64_t i = (int64_t)row * k + kb * 64 + j;
            w[j] = bf16_to_f32(x[i]);
            if (xq_prev)
                w[j] = fmaf(-(float)xq_prev[i], sx_prev[item], w[j]);
            am = fmaxf(am, fabsf(w[j]));
        }
        const float sc = am > 0.f ? am / 127.f : 1.f;
        s[item] = sc;
        for (int j = 0; j < 64; ++j) {
            int v = (int)rintf(w[j] / sc);
            v = v > 127 ? 127 : (v < -127 ? -127 : v);
            q[(int64_t)row * k + kb * 64 + j] = (int8_t)v;
        }
    }
    return 0;
}

/* k_int8_mma_gemm (cuda/int8_mma_gemm.cu:40-156): per 64-block the exact int32 dot,
 * then acc = fma((float)dot * sx, sw, acc) (the reference's `acc += (dot * x0) * w0`
 * as its compiler emits it), the fused plug's term (nibble - 8, element 2i in the low
 * nibble) right after the base's; y = (accumulate ? y : 0) + acc. */
int orc_int8_gemm(const int8_t *xq, const float *sx, const int8_t *wq, const float *sw, float *y, int m, int n, int k,
                  int accumulate, const uint8_t *pq4, const float *psc)
{
    if (m < 1 || n < 1 || k < 64 || k % 64)
        return -1;
    const int nkb = k / 64;
#pragma omp parallel for num_threads(g_threads) schedule(static) collapse(2)
    for (int r = 0; r < m; ++r) {
        for (int c = 0; c < n; ++c) {
            float acc = 0.f;
            for (int kb = 0; kb < nkb; ++kb) {
                int ic = 0, ip = 0;
                for (int j = 0; j < 64; ++j) {
                    const int64_t kk = (int64_t)kb * 64 + j, wi = (int64_t)c * k + kk;
                    ic += (int)xq[(int64_t)r * k + kk] * (int)wq[wi];
                    if (pq4)
                        ip += (int)xq[(int64_t)r * k + kk] * ((int)((pq4[wi >> 1] >> ((wi & 1) * 4)) & 15) - 8);
                }
                const float xs = sx[(int64_t)r * nkb + kb];
                acc = fmaf((float)ic * xs, sw[(int64_t)c * nkb + kb], acc);
                if (pq4)
                    acc = fmaf((float)ip * xs, psc[(int64_t)c * nkb + kb], acc);
            }
            float *yy = y + (int64_t)r * n + c;
            *yy = (accumulate ? *yy : 0.f) + acc;
        }
    }
    return 0;
}
