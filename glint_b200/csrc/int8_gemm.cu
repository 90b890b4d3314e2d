/* INT8 W8A8 GEMM over a bf16_to_int8_pin_v1 linear, with the res4 late plug
 * (include/int8_mma_gemm.h; the reference's cuda/int8_mma_gemm.cu contract).
 *
 *   activations  s = amax / 127 per (row, 64-block), 1 for an all-zero block;
 *                xq = rint(x / s) clamped to +-127 (reference k_quant_act); the
 *                resolve pass quantizes x - xq * s the same way (k_quant_act_resid)
 *   product      per 64-block: the int8 dot of the block in int32 (exact), then
 *                acc = fma((float)sum * sx, sw, acc) in f32, blocks in K order, the
 *                plug's term (nibble - 8, its own scale) right after the base's in
 *                the fused form; y = (accumulate ? y : 0) + acc
 * The f32 steps are the reference's, in its order (one rounded product, then one
 * fused multiply-add per block and output), so the outputs match it bit for bit
 * whatever the tiling.
 *
 * On sm_100a, prefill shapes (M > 64, K % 128 == 0) run the tcgen05 kind::i8 kernel of
 * htile_gemm.cu (TMA operands, int32 block sums in TMEM, a fused plug unpacked to int8
 * in shared memory, the same f32 steps in the epilogue); the rest run `mma.sync` m16n8k32 s8 tiles (64 activation rows x 128 weight rows
 * with a three-stage ring, or for M <= 16, 16 x 64 with an eight-stage ring), 8 warps,
 * shared-memory rings filled with 16-byte asynchronous copies (later K slices land
 * while this one multiplies), plug nibbles unpacked in shared memory.  No split over
 * K: each output's blocks are added in K order, as the reference adds them.  No kernel here waits on
 * another CTA, so nothing can hang.
 */
#include <algorithm>

#include "../../include/int8_mma_gemm.h"
#include "common.cuh"
#include "glint_internal.h"
#include "ptx.cuh"

namespace glint {
namespace {

constexpr int kIBM = 64, kIBN = 128, kIBK = 64;
constexpr int kIPad = 80; /* shared row stride in bytes: 64 + 16 keeps the fragment loads conflict-free */
constexpr int kIThreads = 256;

/* one warp per (row, 64-block): lane owns elements 2 lane, 2 lane + 1 */
__global__ void __launch_bounds__(256) quant_act_kernel(const __nv_bfloat16 *__restrict__ x, const int8_t *xq_prev,
                                                        const float *sx_prev, int m, int k, int8_t *__restrict__ q,
                                                        float *__restrict__ s)
{
    const int nkb = k / kIBK;
    const int item = (int)blockIdx.x * 8 + (int)(threadIdx.x >> 5), lane = (int)(threadIdx.x & 31);
    if (item >= m * nkb)
        return;
    const int row = item / nkb, kb = item - row * nkb;
    const int64_t i = (int64_t)row * k + (int64_t)kb * kIBK + 2 * lane;
    float w0 = __bfloat162float(x[i]), w1 = __bfloat162float(x[i + 1]);
    if (xq_prev) {
        /* the residual of the first quantization (reference: x - xq * sx, one fused step) */
        const float sp = sx_prev[item];
        w0 = __fmaf_rn(-(float)xq_prev[i], sp, w0);
        w1 = __fmaf_rn(-(float)xq_prev[i + 1], sp, w1);
    }
    float a = fmaxf(fabsf(w0), fabsf(w1));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, o));
    const float sc = a > 0.f ? __fdiv_rn(a, 127.f) : 1.f;
    if (lane == 0)
        s[item] = sc;
    int v0 = (int)rintf(__fdiv_rn(w0, sc)), v1 = (int)rintf(__fdiv_rn(w1, sc));
    v0 = v0 > 127 ? 127 : (v0 < -127 ? -127 : v0);
    v1 = v1 > 127 ? 127 : (v1 < -127 ? -127 : v1);
    q[i] = (int8_t)v0;
    q[i + 1] = (int8_t)v1;
}

/* res4 plug -> int8 scratch: element 2i in the low nibble, value nibble - 8 */
__global__ void unpack_res4_kernel(const uint8_t *__restrict__ q4, int8_t *__restrict__ out, int64_t n)
{
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n)
        out[i] = (int8_t)(((q4[i >> 1] >> ((i & 1) * 4)) & 15) - 8);
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool full)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr(dst)), "l"(src), "r"(full ? 16 : 0)
                 : "memory");
}
/* 4-byte asynchronous copy (zero-filled when !full) */
__device__ __forceinline__ void cp_async4(void *dst, const void *src, bool full)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(saddr(dst)), "l"(src), "r"(full ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct Int8Args {
    const int8_t *xq;
    const float *sx;
    const int8_t *wq;
    const float *sw;
    float *y;
    int m, n, k;
    int accumulate;
    const uint8_t *pq4; /* fused plug, or null */
    const float *psc;
};

/* one K slice of a tile: x rows, weight rows, packed plug nibbles, the slice's scales */
template <int BM, int BN>
struct __align__(16) Int8Stage {
    int8_t a[BM][kIPad];
    int8_t b[BN][kIPad];
    uint8_t pp[BN][32];
    float sx[BM], sw[BN], sp[BN];
};

/* the 64-wide K slice kb of this tile into stage st, all by asynchronous copies
 * zero-filled past m / n (x, weights, packed plug: 16 bytes; scales: 4 bytes), so no
 * thread waits on a global load before the slice's barrier */
template <bool PLUG, int BM, int BN>
__device__ __forceinline__ void load_slice(const Int8Args &a, Int8Stage<BM, BN> &st, int m0, int n0, int kb, int nkb)
{
    const int tid = (int)threadIdx.x;
    for (int idx = tid; idx < BM * 4; idx += kIThreads) {
        const int r = idx >> 2, c = (idx & 3) * 16;
        const bool ok = m0 + r < a.m;
        cp_async16(&st.a[r][c], ok ? a.xq + (int64_t)(m0 + r) * a.k + (int64_t)kb * kIBK + c : a.xq, ok);
    }
    for (int idx = tid; idx < BN * 4; idx += kIThreads) {
        const int r = idx >> 2, c = (idx & 3) * 16;
        const bool ok = n0 + r < a.n;
        cp_async16(&st.b[r][c], ok ? a.wq + (int64_t)(n0 + r) * a.k + (int64_t)kb * kIBK + c : a.wq, ok);
    }
    if (PLUG) {
        for (int idx = tid; idx < BN * 2; idx += kIThreads) {
            const int r = idx >> 1, c = (idx & 1) * 16;
            const bool ok = n0 + r < a.n;
            cp_async16(&st.pp[r][c], ok ? a.pq4 + (((int64_t)(n0 + r) * a.k + (int64_t)kb * kIBK) >> 1) + c : a.pq4,
                       ok);
        }
    }
    if (tid < BM) {
        const bool ok = m0 + tid < a.m;
        cp_async4(&st.sx[tid], ok ? a.sx + (int64_t)(m0 + tid) * nkb + kb : a.sx, ok);
    }
    if (tid < BN) {
        const bool ok = n0 + tid < a.n;
        cp_async4(&st.sw[tid], ok ? a.sw + (int64_t)(n0 + tid) * nkb + kb : a.sw, ok);
        if (PLUG)
            cp_async4(&st.sp[tid], ok ? a.psc + (int64_t)(n0 + tid) * nkb + kb : a.psc, ok);
    }
}

/* Tiles of BM activation rows x BN weight rows; the 8 warps split them into BM / 16
 * row groups x (8 / (BM / 16)) column groups of NTW 8-column MMA tiles; STAGES K
 * slices in flight.  Large M: 64 x 128, 3 stages; decode (M <= 16): 16 x 64, 8
 * stages, so that there are enough CTAs and bytes in flight to stream the weights.
 * One barrier per slice (two with a plug, whose unpacked copy is shared). */
template <bool PLUG, int BM, int BN, int STAGES>
__global__ void __launch_bounds__(kIThreads) int8_gemm_kernel(const Int8Args a)
{
    constexpr int MW = BM / 16, NW = 8 / MW, NTW = BN / NW / 8;
    static_assert(MW * NW == 8 && NTW >= 1, "warp layout");
    using Stage = Int8Stage<BM, BN>;
    extern __shared__ __align__(16) uint8_t smem[];
    Stage *stages = reinterpret_cast<Stage *>(smem);
    __shared__ __align__(16) int8_t sP[PLUG ? BN : 1][kIPad]; /* the slice's plug, unpacked */
    const int tid = (int)threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int m0 = (int)blockIdx.y * BM, n0 = (int)blockIdx.x * BN;
    const int rb = (warp % MW) * 16, cb = (warp / MW) * (NTW * 8); /* this warp's 16 x 8 NTW */
    const int nkb = a.k / kIBK;

    float acc[NTW][4];
#pragma unroll
    for (int i = 0; i < NTW; ++i)
        acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

#pragma unroll
    for (int s0 = 0; s0 < STAGES - 1; ++s0) {
        if (s0 < nkb)
            load_slice<PLUG, BM, BN>(a, stages[s0], m0, n0, s0, nkb);
        cp_async_commit();
    }
    for (int kb = 0; kb < nkb; ++kb) {
        Stage &st = stages[kb % STAGES];
        cp_async_wait<STAGES - 2>(); /* this slice's copies have landed */
        /* every thread's copies of slice kb are visible, and every thread is done with
         * slice kb - 1, whose stage the next load reuses */
        __syncthreads();
        if (kb + STAGES - 1 < nkb)
            load_slice<PLUG, BM, BN>(a, stages[(kb + STAGES - 1) % STAGES], m0, n0, kb + STAGES - 1, nkb);
        cp_async_commit();
        if (PLUG) {
            /* unpack: row r, packed byte b -> elements 2b (low nibble), 2b + 1 */
            for (int i = tid; i < BN * 32; i += kIThreads) {
                const int r = i >> 5, b = i & 31;
                const uint32_t v = st.pp[r][b];
                sP[r][2 * b] = (int8_t)((int)(v & 15u) - 8);
                sP[r][2 * b + 1] = (int8_t)((int)(v >> 4) - 8);
            }
            __syncthreads();
        }
        int ic[NTW][4], ip[NTW][4];
#pragma unroll
        for (int i = 0; i < NTW; ++i) {
            ic[i][0] = ic[i][1] = ic[i][2] = ic[i][3] = 0;
            ip[i][0] = ip[i][1] = ip[i][2] = ip[i][3] = 0;
        }
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
            const uint32_t a0 = *reinterpret_cast<const uint32_t *>(&st.a[rb + g][ks * 32 + t * 4]);
            const uint32_t a1 = *reinterpret_cast<const uint32_t *>(&st.a[rb + g + 8][ks * 32 + t * 4]);
            const uint32_t a2 = *reinterpret_cast<const uint32_t *>(&st.a[rb + g][ks * 32 + 16 + t * 4]);
            const uint32_t a3 = *reinterpret_cast<const uint32_t *>(&st.a[rb + g + 8][ks * 32 + 16 + t * 4]);
#pragma unroll
            for (int nt = 0; nt < NTW; ++nt) {
                const int nr = cb + nt * 8 + g;
                mma_s8(ic[nt], a0, a1, a2, a3, *reinterpret_cast<const uint32_t *>(&st.b[nr][ks * 32 + t * 4]),
                       *reinterpret_cast<const uint32_t *>(&st.b[nr][ks * 32 + 16 + t * 4]));
                if (PLUG)
                    mma_s8(ip[nt], a0, a1, a2, a3, *reinterpret_cast<const uint32_t *>(&sP[nr][ks * 32 + t * 4]),
                           *reinterpret_cast<const uint32_t *>(&sP[nr][ks * 32 + 16 + t * 4]));
            }
        }
        const float x0 = st.sx[rb + g], x1 = st.sx[rb + g + 8];
#pragma unroll
        for (int nt = 0; nt < NTW; ++nt) {
            const int c = cb + nt * 8 + t * 2;
            const float w0 = st.sw[c], w1 = st.sw[c + 1];
            acc[nt][0] = __fmaf_rn(__fmul_rn((float)ic[nt][0], x0), w0, acc[nt][0]);
            acc[nt][1] = __fmaf_rn(__fmul_rn((float)ic[nt][1], x0), w1, acc[nt][1]);
            acc[nt][2] = __fmaf_rn(__fmul_rn((float)ic[nt][2], x1), w0, acc[nt][2]);
            acc[nt][3] = __fmaf_rn(__fmul_rn((float)ic[nt][3], x1), w1, acc[nt][3]);
            if (PLUG) {
                const float q0 = st.sp[c], q1 = st.sp[c + 1];
                acc[nt][0] = __fmaf_rn(__fmul_rn((float)ip[nt][0], x0), q0, acc[nt][0]);
                acc[nt][1] = __fmaf_rn(__fmul_rn((float)ip[nt][1], x0), q1, acc[nt][1]);
                acc[nt][2] = __fmaf_rn(__fmul_rn((float)ip[nt][2], x1), q0, acc[nt][2]);
                acc[nt][3] = __fmaf_rn(__fmul_rn((float)ip[nt][3], x1), q1, acc[nt][3]);
            }
        }
    }
    cp_async_wait<0>();
#pragma unroll
    for (int nt = 0; nt < NTW; ++nt) {
        const int col = n0 + cb + nt * 8 + t * 2;
        const int r0 = m0 + rb + g, r1 = r0 + 8;
        float *y0 = a.y + (int64_t)r0 * a.n + col, *y1 = a.y + (int64_t)r1 * a.n + col;
        if (r0 < a.m) {
            if (col < a.n)
                y0[0] = (a.accumulate ? y0[0] : 0.f) + acc[nt][0];
            if (col + 1 < a.n)
                y0[1] = (a.accumulate ? y0[1] : 0.f) + acc[nt][1];
        }
        if (r1 < a.m) {
            if (col < a.n)
                y1[0] = (a.accumulate ? y1[0] : 0.f) + acc[nt][2];
            if (col + 1 < a.n)
                y1[1] = (a.accumulate ? y1[1] : 0.f) + acc[nt][3];
        }
    }
}

template <bool PLUG, int BM, int BN, int STAGES>
cudaError_t launch_gemm(const Int8Args &a, cudaStream_t st)
{
    constexpr int smem = STAGES * (int)sizeof(Int8Stage<BM, BN>);
    auto kern = int8_gemm_kernel<PLUG, BM, BN, STAGES>;
    if (!ensure_smem((const void *)kern, smem))
        return cudaErrorInvalidValue;
    kern<<<dim3((a.n + BN - 1) / BN, (a.m + BM - 1) / BM), kIThreads, smem, st>>>(a);
    return cudaGetLastError();
}

cudaError_t quant(const __nv_bfloat16 *x, const int8_t *xq_prev, const float *sx_prev, int m, int k, int8_t *q,
                  float *s, cudaStream_t st)
{
    const int items = m * (k / kIBK);
    quant_act_kernel<<<(items + 7) / 8, 256, 0, st>>>(x, xq_prev, sx_prev, m, k, q, s);
    return cudaGetLastError();
}

cudaError_t gemm(const int8_t *xq, const float *sx, const int8_t *wq, const float *sw, float *y, int m, int n, int k,
                 int accumulate, const uint8_t *pq4, const float *psc, cudaStream_t st)
{
    /* prefill shapes: tcgen05 kind::i8 (the same bits) */
    if (int8_tc_supported(xq, wq, pq4, m, k)) {
        const cudaError_t e = int8_tc_gemm_launch(xq, sx, wq, sw, pq4, psc, y, m, n, k, accumulate, st);
        if (e != cudaErrorNotSupported)
            return e;
    }
    Int8Args a{xq, sx, wq, sw, y, m, n, k, accumulate, pq4, psc};
    if (m <= 16)
        return pq4 ? launch_gemm<true, 16, 64, 8>(a, st) : launch_gemm<false, 16, 64, 8>(a, st);
    if (m <= 32)
        return pq4 ? launch_gemm<true, 32, 64, 8>(a, st) : launch_gemm<false, 32, 64, 8>(a, st);
    return pq4 ? launch_gemm<true, 64, 128, 3>(a, st) : launch_gemm<false, 64, 128, 3>(a, st);
}

cudaError_t unpack(const uint8_t *q4, int8_t *out, int64_t n, cudaStream_t st)
{
    unpack_res4_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(q4, out, n);
    return cudaGetLastError();
}

bool valid(const __nv_bfloat16 *x, const Int8MmaLinear &w, const float *y, int m, const int8_t *xq, const float *sx)
{
    return x && y && xq && sx && w.q && w.scale && m >= 1 && w.n_out >= 1 && w.k_in >= kIBK && w.k_in % kIBK == 0 &&
           aligned_to(w.q, 16) && aligned_to(xq, 16);
}

} // namespace
} // namespace glint

using namespace glint;

extern "C" {

cudaError_t int8_mma_gemm(const __nv_bfloat16 *x, Int8MmaLinear w, float *y, int m, int8_t *xq, float *sx,
                          cudaStream_t stream)
{
    if (!valid(x, w, y, m, xq, sx))
        return cudaErrorInvalidValue;
    cudaError_t e = quant(x, nullptr, nullptr, m, w.k_in, xq, sx, stream);
    return e != cudaSuccess ? e : gemm(xq, sx, w.q, w.scale, y, m, w.n_out, w.k_in, 0, nullptr, nullptr, stream);
}

cudaError_t int8_mma_gemm_plug(const __nv_bfloat16 *x, Int8MmaLinear w, const uint8_t *plug_q4,
                               const float *plug_scale, float *y, int m, int8_t *xq, float *sx, int8_t *plug_i8,
                               cudaStream_t stream)
{
    if (!valid(x, w, y, m, xq, sx) || !plug_q4 || !plug_scale || !plug_i8 || !aligned_to(plug_i8, 16))
        return cudaErrorInvalidValue;
    const int64_t n = (int64_t)w.n_out * w.k_in;
    cudaError_t e = quant(x, nullptr, nullptr, m, w.k_in, xq, sx, stream);
    if (e == cudaSuccess)
        e = gemm(xq, sx, w.q, w.scale, y, m, w.n_out, w.k_in, 0, nullptr, nullptr, stream);
    if (e == cudaSuccess)
        e = unpack(plug_q4, plug_i8, n, stream);
    /* the plug shares the base's activation quantization and adds into y */
    if (e == cudaSuccess)
        e = gemm(xq, sx, plug_i8, plug_scale, y, m, w.n_out, w.k_in, 1, nullptr, nullptr, stream);
    return e;
}

cudaError_t int8_mma_gemm_plug_fused(const __nv_bfloat16 *x, Int8MmaLinear w, const uint8_t *plug_q4,
                                     const float *plug_scale, float *y, int m, int8_t *xq, float *sx,
                                     cudaStream_t stream)
{
    if (!valid(x, w, y, m, xq, sx) || !plug_q4 || !plug_scale || !aligned_to(plug_q4, 16))
        return cudaErrorInvalidValue;
    cudaError_t e = quant(x, nullptr, nullptr, m, w.k_in, xq, sx, stream);
    return e != cudaSuccess ? e : gemm(xq, sx, w.q, w.scale, y, m, w.n_out, w.k_in, 0, plug_q4, plug_scale, stream);
}

cudaError_t int8_mma_gemm_resolve(const __nv_bfloat16 *x, Int8MmaLinear w, const uint8_t *plug_q4,
                                  const float *plug_scale, float *y, int m, int8_t *xq, float *sx, int8_t *rq,
                                  float *sr, int8_t *plug_i8, cudaStream_t stream)
{
    if (!valid(x, w, y, m, xq, sx) || !rq || !sr || !aligned_to(rq, 16) || (plug_q4 != nullptr) != (plug_i8 != nullptr) ||
        (plug_q4 != nullptr) != (plug_scale != nullptr) || (plug_i8 && !aligned_to(plug_i8, 16)))
        return cudaErrorInvalidValue;
    const int64_t n = (int64_t)w.n_out * w.k_in;
    const int k = w.k_in;
    cudaError_t e = quant(x, nullptr, nullptr, m, k, xq, sx, stream);
    if (e == cudaSuccess)
        e = quant(x, xq, sx, m, k, rq, sr, stream);
    if (e == cudaSuccess)
        e = gemm(xq, sx, w.q, w.scale, y, m, w.n_out, k, 0, nullptr, nullptr, stream);
    if (e == cudaSuccess)
        e = gemm(rq, sr, w.q, w.scale, y, m, w.n_out, k, 1, nullptr, nullptr, stream);
    if (plug_q4) {
        if (e == cudaSuccess)
            e = unpack(plug_q4, plug_i8, n, stream);
        if (e == cudaSuccess)
            e = gemm(xq, sx, plug_i8, plug_scale, y, m, w.n_out, k, 1, nullptr, nullptr, stream);
        if (e == cudaSuccess)
            e = gemm(rq, sr, plug_i8, plug_scale, y, m, w.n_out, k, 1, nullptr, nullptr, stream);
    }
    return e;
}

} /* extern "C" */
