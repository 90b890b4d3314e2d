/* The C ABI of libglint_encode.so: the reference's entry points
 * (include/glint_encode.h:11-29, include/glint_htile.h:11-19, cuda/p7_abi.c:3-11
 * of Jadon-Fox/glint) plus additive device-pointer, BF16 and batched calls.
 *
 * Host-pointer calls (glint_encode_*_host, glint_expand_*_host) keep the
 * reference's synchronous contract but do not allocate per call: each device
 * keeps three grow-only slots of device memory (and of page-locked staging, only
 * if a caller passes pageable buffers), and a tensor is streamed through them in
 * chunks so that the host-to-device copy of one chunk, the kernel of the next
 * and the device-to-host copy of a third overlap.  Page-locked caller buffers are
 * read and written by DMA directly.  Calls on one device are serialised by a
 * per-device mutex; the reference's unguarded `static int once` codebook upload
 * (cuda/glint_encode.cu:115-127) has no counterpart because the codebook is
 * compiled into the kernels, so every device sees it.
 */
#include <algorithm>
#include <condition_variable>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include <unistd.h>

#include "../../include/glint_b200.h"
#include "../../include/glint_encode.h"
#include "../../include/glint_htile.h"
#include "../../include/glint_km.h"
#include "common.cuh"
#include "glint_internal.h"

#ifndef GLINT_B200_VERSION
#define GLINT_B200_VERSION "0.1.0"
#endif

namespace glint {
namespace {

constexpr int kMaxDevices = 64;
constexpr int kSlots = 3;
constexpr int64_t kChunkWeights = int64_t(1) << 24;    /* at most 16 Mi weights per pipeline chunk */
constexpr int64_t kMinChunkWeights = int64_t(1) << 21; /* at least 2 Mi (unless the tensor is smaller) */

struct Buffer {
    void *p = nullptr;
    size_t cap = 0;
};

struct DevState {
    std::mutex mu;       /* host pipelines */
    std::mutex attr_mu;  /* kernel attributes */
    int sms = 0;
    std::vector<const void *> smem_done;
    bool streams_ready = false;
    cudaStream_t st[kSlots] = {};
    cudaEvent_t done[kSlots] = {};
    Buffer dbuf[kSlots];
    Buffer hbuf[kSlots];
};

DevState g_dev[kMaxDevices];

int current_device()
{
    int d = -1;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDevices)
        return -1;
    return d;
}

bool grow_device(Buffer &b, size_t need)
{
    if (b.cap >= need)
        return true;
    if (b.p)
        cudaFree(b.p);
    b.p = nullptr;
    b.cap = 0;
    if (cudaMalloc(&b.p, need) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    b.cap = need;
    return true;
}

bool grow_pinned(Buffer &b, size_t need)
{
    if (b.cap >= need)
        return true;
    if (b.p)
        cudaFreeHost(b.p);
    b.p = nullptr;
    b.cap = 0;
    if (cudaMallocHost(&b.p, need) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    b.cap = need;
    return true;
}

bool ensure_streams(DevState &S)
{
    if (S.streams_ready)
        return true;
    for (int i = 0; i < kSlots; ++i) {
        if (cudaStreamCreateWithFlags(&S.st[i], cudaStreamNonBlocking) != cudaSuccess)
            return false;
        if (cudaEventCreateWithFlags(&S.done[i], cudaEventDisableTiming) != cudaSuccess)
            return false;
    }
    S.streams_ready = true;
    return true;
}

/* Host memcpy split with a few persistent threads (at most 8 with the caller), for
 * the pipeline's copies between pageable caller memory and pinned staging: one
 * thread moves ~5-10 GB/s, and first-touch page faults of a memory-mapped input
 * are taken in parallel too.  Workers take fixed parts of one copy at a time
 * (copies are serialised), so every worker sees every copy exactly once.  The pool
 * is never destroyed: idle workers block on a condition variable until exit. */
class CopyPool {
  public:
    static CopyPool &get()
    {
        static CopyPool *pool = new CopyPool();
        return *pool;
    }
    void copy(void *dst, const void *src, size_t bytes)
    {
        /* a forked child has the pool's state but not its threads */
        if (bytes < kMinSplit || workers_ == 0 || getpid() != pid_) {
            std::memcpy(dst, src, bytes);
            return;
        }
        std::lock_guard<std::mutex> one(call_mu_);
        const size_t parts = (size_t)workers_ + 1;
        {
            std::lock_guard<std::mutex> lk(mu_);
            dst_ = static_cast<char *>(dst);
            src_ = static_cast<const char *>(src);
            bytes_ = bytes;
            part_ = ((bytes + parts - 1) / parts + 4095) & ~size_t(4095);
            done_ = 0;
            ++gen_;
        }
        cv_.notify_all();
        run_part(0);
        std::unique_lock<std::mutex> lk(mu_);
        done_cv_.wait(lk, [&] { return done_ == workers_; });
    }

  private:
    static constexpr size_t kMinSplit = size_t(4) << 20;
    CopyPool() : pid_(getpid())
    {
        const unsigned hw = std::thread::hardware_concurrency();
        workers_ = (int)std::min(7u, hw > 1 ? hw - 1 : 0u);
        for (int i = 0; i < workers_; ++i)
            std::thread([this, i] { loop(i + 1); }).detach();
    }
    void run_part(int k)
    {
        const size_t off = (size_t)k * part_;
        if (off < bytes_)
            std::memcpy(dst_ + off, src_ + off, std::min(part_, bytes_ - off));
    }
    void loop(int k)
    {
        uint64_t seen = 0;
        for (;;) {
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return gen_ != seen; });
                seen = gen_;
            }
            run_part(k);
            {
                std::lock_guard<std::mutex> lk(mu_);
                ++done_;
            }
            done_cv_.notify_one();
        }
    }
    pid_t pid_;
    int workers_ = 0;
    std::mutex call_mu_, mu_;
    std::condition_variable cv_, done_cv_;
    char *dst_ = nullptr;
    const char *src_ = nullptr;
    size_t bytes_ = 0, part_ = 0;
    int done_ = 0;
    uint64_t gen_ = 0;
};

void host_copy(void *dst, const void *src, size_t bytes) { CopyPool::get().copy(dst, src, bytes); }

bool is_pinned(const void *p)
{
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

int64_t gcd64(int64_t a, int64_t b)
{
    while (b) {
        int64_t t = a % b;
        a = b;
        b = t;
    }
    return a;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

/* Chunk length: a multiple of the blocksize (blocks never straddle chunks) and of
 * 512 (plane offsets stay 256-byte aligned). */
int64_t chunk_len(int64_t n, int bs)
{
    const int64_t unit = (int64_t)bs / gcd64(bs, 512) * 512;
    /* about eight chunks per tensor, 2-16 Mi weights each: the copy-in, kernel and
     * copy-out of neighbouring chunks overlap, so only ~1/8 of a mid-size tensor's
     * transfer is left unoverlapped at its start and end (one 33 MB chunk left all
     * of it); below 2 Mi weights the per-chunk call overhead would dominate */
    const int64_t target = std::min(kChunkWeights, std::max(kMinChunkWeights, (n + 7) / 8));
    const int64_t c = std::max(unit, (target + unit - 1) / unit * unit);
    const int64_t need = (n + unit - 1) / unit * unit;
    return std::min(c, need);
}

struct Layout {
    size_t dense, planes, am, err, total; /* bytes of each part of a slot, in this order */
};
Layout slot_layout(int64_t chunk, int bs, size_t dense_elem, bool with_err)
{
    Layout L;
    L.dense = align256((size_t)chunk * dense_elem);
    L.planes = align256((size_t)(chunk / 2));
    L.am = align256((size_t)(chunk / bs) * sizeof(float));
    L.err = with_err ? align256((size_t)kMaxSqErrPartials * sizeof(double)) : 0;
    L.total = L.dense + 2 * L.planes + L.am + L.err;
    return L;
}

/* Encode (to_planes) or expand (!to_planes) a host tensor through the slots.
 * dense: host input (encode) or output (expand) of n elements of dense_elem bytes.
 * sq_err (encode only, may be null): the f64 squared dequantisation error of the
 * whole tensor, each chunk's partials added in order on the host, then the chunks
 * in order. */
int host_pipeline(bool to_planes, bool f32_dense, void *dense, int64_t n, int bs, uint8_t *hole, uint8_t *plug,
                  float *am, double *sq_err = nullptr)
{
    const int dev = current_device();
    if (dev < 0)
        return kLaunch;
    DevState &S = g_dev[dev];
    std::lock_guard<std::mutex> lk(S.mu);
    if (!ensure_streams(S))
        return kLaunch;
    const size_t de = f32_dense ? 4 : 2;
    const int64_t chunk = chunk_len(n, bs);
    const bool want_err = to_planes && sq_err;
    const Layout L = slot_layout(chunk, bs, de, want_err);
    const size_t err_off = L.dense + 2 * L.planes + L.am;
    const int64_t nb_total = (n + bs - 1) / bs;
    const bool pin_dense = is_pinned(dense);
    const bool pin_planes = is_pinned(hole) && is_pinned(plug) && is_pinned(am);
    for (int s = 0; s < kSlots; ++s) {
        if (!grow_device(S.dbuf[s], L.total))
            return to_planes ? kBadArg : kLaunch;
        if ((!pin_dense || !pin_planes || want_err) && !grow_pinned(S.hbuf[s], L.total))
            return kLaunch;
    }
    const int64_t nchunks = (n + chunk - 1) / chunk;
    std::vector<int64_t> pending(kSlots, -1); /* chunk whose results still sit in a staging slot */
    std::vector<double> chunk_err(want_err ? nchunks : 0, 0.0);
    int rc = kOk;

    auto span = [&](int64_t ci, int64_t &off, int64_t &cn, int64_t &bytes_pk, int64_t &nam) {
        off = ci * chunk;
        cn = std::min(chunk, n - off);
        bytes_pk = (cn + 1) / 2;
        nam = std::min((cn + bs - 1) / bs, nb_total - off / bs);
    };
    /* move a finished chunk's results from staging to the caller (pageable output) */
    auto drain = [&](int s) -> int {
        if (pending[s] < 0)
            return kOk;
        if (cudaEventSynchronize(S.done[s]) != cudaSuccess)
            return kLaunch;
        int64_t off, cn, bpk, nam;
        span(pending[s], off, cn, bpk, nam);
        char *h = static_cast<char *>(S.hbuf[s].p);
        if (to_planes && !pin_planes) {
            host_copy(hole + off / 2, h + L.dense, bpk);
            host_copy(plug + off / 2, h + L.dense + L.planes, bpk);
            host_copy(am + off / bs, h + L.dense + 2 * L.planes, nam * sizeof(float));
        }
        if (!to_planes && !pin_dense)
            host_copy(static_cast<char *>(dense) + off * de, h, cn * de);
        if (want_err) {
            const double *part = reinterpret_cast<const double *>(h + err_off);
            double e = 0.0;
            for (int g = 0, G = sq_error_grid(cn); g < G; ++g)
                e += part[g];
            chunk_err[pending[s]] = e;
        }
        pending[s] = -1;
        return kOk;
    };

    for (int64_t ci = 0; ci < nchunks && rc == kOk; ++ci) {
        const int s = (int)(ci % kSlots);
        if (ci >= kSlots) {
            if (cudaEventSynchronize(S.done[s]) != cudaSuccess) {
                rc = kLaunch;
                break;
            }
            if ((rc = drain(s)) != kOk)
                break;
        }
        int64_t off, cn, bpk, nam;
        span(ci, off, cn, bpk, nam);
        char *d = static_cast<char *>(S.dbuf[s].p);
        char *h = static_cast<char *>(S.hbuf[s].p);
        uint8_t *d_hole = reinterpret_cast<uint8_t *>(d + L.dense);
        uint8_t *d_plug = reinterpret_cast<uint8_t *>(d + L.dense + L.planes);
        float *d_am = reinterpret_cast<float *>(d + L.dense + 2 * L.planes);
        cudaStream_t st = S.st[s];
        if (to_planes) {
            const char *src = static_cast<const char *>(dense) + off * de;
            if (!pin_dense) {
                host_copy(h, src, cn * de);
                src = h;
            }
            if (cudaMemcpyAsync(d, src, cn * de, cudaMemcpyHostToDevice, st) != cudaSuccess) {
                rc = kBadArg;
                break;
            }
            EncodeJob j{d, cn, d_hole, d_plug, d_am};
            if ((rc = encode_launch(&j, 1, bs, f32_dense, st)) != kOk)
                break;
            if (want_err) {
                double *d_err = reinterpret_cast<double *>(d + err_off);
                if ((rc = sq_error_launch(d, f32_dense, d_hole, d_plug, d_am, cn, bs, d_err, st)) != kOk)
                    break;
                if (cudaMemcpyAsync(h + err_off, d_err, (size_t)sq_error_grid(cn) * sizeof(double),
                                    cudaMemcpyDeviceToHost, st) != cudaSuccess) {
                    rc = kLaunch;
                    break;
                }
            }
            uint8_t *oh = pin_planes ? hole + off / 2 : reinterpret_cast<uint8_t *>(h + L.dense);
            uint8_t *op = pin_planes ? plug + off / 2 : reinterpret_cast<uint8_t *>(h + L.dense + L.planes);
            float *oa = pin_planes ? am + off / bs : reinterpret_cast<float *>(h + L.dense + 2 * L.planes);
            if (cudaMemcpyAsync(oh, d_hole, bpk, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
                cudaMemcpyAsync(op, d_plug, bpk, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
                cudaMemcpyAsync(oa, d_am, nam * sizeof(float), cudaMemcpyDeviceToHost, st) != cudaSuccess) {
                rc = kLaunch;
                break;
            }
        } else {
            const uint8_t *sh = hole + off / 2, *sp = plug + off / 2;
            const float *sa = am + off / bs;
            if (!pin_planes) {
                host_copy(h + L.dense, sh, bpk);
                host_copy(h + L.dense + L.planes, sp, bpk);
                host_copy(h + L.dense + 2 * L.planes, sa, nam * sizeof(float));
                sh = reinterpret_cast<uint8_t *>(h + L.dense);
                sp = reinterpret_cast<uint8_t *>(h + L.dense + L.planes);
                sa = reinterpret_cast<float *>(h + L.dense + 2 * L.planes);
            }
            if (cudaMemcpyAsync(d_hole, sh, bpk, cudaMemcpyHostToDevice, st) != cudaSuccess ||
                cudaMemcpyAsync(d_plug, sp, bpk, cudaMemcpyHostToDevice, st) != cudaSuccess ||
                cudaMemcpyAsync(d_am, sa, nam * sizeof(float), cudaMemcpyHostToDevice, st) != cudaSuccess) {
                rc = kBadArg;
                break;
            }
            ExpandJob j{d_hole, d_plug, d_am, cn, d};
            if ((rc = expand_launch(&j, 1, bs, f32_dense ? kOutF32 : kOutBF16, st)) != kOk)
                break;
            char *dst = pin_dense ? static_cast<char *>(dense) + off * de : h;
            if (cudaMemcpyAsync(dst, d, cn * de, cudaMemcpyDeviceToHost, st) != cudaSuccess) {
                rc = kLaunch;
                break;
            }
        }
        if (cudaEventRecord(S.done[s], st) != cudaSuccess) {
            rc = kLaunch;
            break;
        }
        pending[s] = ((to_planes && !pin_planes) || (!to_planes && !pin_dense) || want_err) ? ci : -1;
    }
    /* finish every slot, also after an error, so no copy into caller memory outlives the call */
    for (int s = 0; s < kSlots; ++s) {
        if (cudaStreamSynchronize(S.st[s]) != cudaSuccess && rc == kOk)
            rc = kLaunch;
        if (rc == kOk) {
            int r = drain(s);
            if (r != kOk)
                rc = r;
        }
    }
    if (cudaGetLastError() != cudaSuccess && rc == kOk)
        rc = kLaunch;
    if (want_err && rc == kOk) {
        double e = 0.0;
        for (double c : chunk_err)
            e += c;
        *sq_err = e;
    }
    return rc;
}

int encode_host(const void *w, int64_t n, int bs, uint8_t *hole, uint8_t *plug, float *am, bool f32,
                double *sq_err = nullptr)
{
    if (n < 0 || bs <= 0)
        return kBadArg;
    if (n == 0) {
        if (sq_err)
            *sq_err = 0.0;
        return kOk;
    }
    if (!w || !hole || !plug || !am)
        return kBadArg;
    return host_pipeline(true, f32, const_cast<void *>(w), n, bs, hole, plug, am, sq_err);
}

int expand_host(const uint8_t *hole, const uint8_t *plug, const float *am, int64_t n, int bs, void *out, bool f32)
{
    if (n < 0 || bs <= 0)
        return kBadArg;
    if (n == 0)
        return kOk;
    if (!hole || !plug || !am || !out)
        return kBadArg;
    return host_pipeline(false, f32, out, n, bs, const_cast<uint8_t *>(hole), const_cast<uint8_t *>(plug),
                         const_cast<float *>(am));
}

} // namespace

int sm_count()
{
    const int d = current_device();
    if (d < 0)
        return 148;
    DevState &S = g_dev[d];
    if (S.sms <= 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || v <= 0)
            v = 148;
        S.sms = v;
    }
    return S.sms;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

bool ensure_smem(const void *kernel, int bytes)
{
    const int d = current_device();
    if (d < 0)
        return false;
    DevState &S = g_dev[d];
    std::lock_guard<std::mutex> lk(S.attr_mu);
    if (std::find(S.smem_done.begin(), S.smem_done.end(), kernel) != S.smem_done.end())
        return true;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    S.smem_done.push_back(kernel);
    return true;
}

int htile_launch(const uint8_t *hole, const uint8_t *plug, const float *am, const __nv_bfloat16 *x, void *y,
                 OutKind yk, int M, int N, int K, int bs, HtileMode mode, cudaStream_t st)
{
    if (!hole || !plug || !am || !x || !y)
        return kBadArg;
    if (bs <= 0)
        return kBadBlocksize;
    if (M < 0 || N < 0 || K < 0)
        return kBadArg;
    if (M == 0 || N == 0)
        return kOk;
    if (K == 0) {
        const size_t bytes = (size_t)M * N * (yk == kOutBF16 ? 2 : 4);
        return cudaMemsetAsync(y, 0, bytes, st) == cudaSuccess ? kOk : kLaunch;
    }
    if (htile_gemm_supported(hole, plug, am, x, y, yk == kOutBF16, M, N, K, bs))
        return mode == kFast ? htile_gemm_launch(hole, plug, am, x, y, yk == kOutBF16, M, N, K, bs, st)
                             : htile_gemm_precise_launch(hole, plug, am, x, y, yk == kOutBF16, M, N, K, st);
    return htile_gemv_launch(hole, plug, am, x, y, yk, M, N, K, bs, mode, st);
}

} // namespace glint

using namespace glint;

extern "C" {

const char *p7_abi_version(void) { return "p7_attach_abi_v1"; }
int glint_kernel_error(int clear) { return read_kernel_error(clear != 0); }
const char *glint_b200_version(void) { return "glint_b200 " GLINT_B200_VERSION " sm_100a"; }

int glint_encode_n_absmax(int64_t n, int blocksize)
{
    if (blocksize <= 0)
        return 0;
    return (int)((n + blocksize - 1) / blocksize);
}
int glint_encode_n_packed(int64_t n) { return (int)((n + 1) / 2); }
int64_t glint_encode_n_absmax64(int64_t n, int blocksize)
{
    if (blocksize <= 0 || n <= 0)
        return 0;
    return (n + blocksize - 1) / blocksize;
}
int64_t glint_encode_n_packed64(int64_t n) { return n <= 0 ? 0 : (n + 1) / 2; }

int glint_encode_bf16_host(const uint16_t *w_bf16, int64_t n, int blocksize, uint8_t *hole_packed,
                           uint8_t *plug_packed, float *absmax)
{
    return encode_host(w_bf16, n, blocksize, hole_packed, plug_packed, absmax, false);
}
int glint_encode_f32_host(const float *w, int64_t n, int blocksize, uint8_t *hole_packed, uint8_t *plug_packed,
                          float *absmax)
{
    return encode_host(w, n, blocksize, hole_packed, plug_packed, absmax, true);
}
int glint_encode_bf16_host_sqerr(const uint16_t *w_bf16, int64_t n, int blocksize, uint8_t *hole_packed,
                                 uint8_t *plug_packed, float *absmax, double *sum_sq_err)
{
    if (!sum_sq_err)
        return kBadArg;
    return encode_host(w_bf16, n, blocksize, hole_packed, plug_packed, absmax, false, sum_sq_err);
}
int glint_encode_f32_host_sqerr(const float *w, int64_t n, int blocksize, uint8_t *hole_packed, uint8_t *plug_packed,
                                float *absmax, double *sum_sq_err)
{
    if (!sum_sq_err)
        return kBadArg;
    return encode_host(w, n, blocksize, hole_packed, plug_packed, absmax, true, sum_sq_err);
}
int glint_cells_f32(float *out)
{
    static const float kCells[16][16] = GLINT_CELLS_INIT;
    if (!out)
        return kBadArg;
    memcpy(out, kCells, sizeof(kCells));
    return 256;
}
int glint_expand_packed_to_f32_host(const uint8_t *hole_packed, const uint8_t *plug_packed, const float *absmax,
                                    int64_t n, int blocksize, float *out_f32)
{
    return expand_host(hole_packed, plug_packed, absmax, n, blocksize, out_f32, true);
}
int glint_expand_packed_to_bf16_host(const uint8_t *hole_packed, const uint8_t *plug_packed, const float *absmax,
                                     int64_t n, int blocksize, uint16_t *out_bf16)
{
    return expand_host(hole_packed, plug_packed, absmax, n, blocksize, out_bf16, false);
}

static int device_encode(const void *w, int64_t n, int bs, uint8_t *h, uint8_t *p, float *a, bool f32,
                         struct CUstream_st *stream)
{
    if (n < 0 || bs <= 0)
        return kBadArg;
    if (n == 0)
        return kOk;
    if (!w || !h || !p || !a)
        return kBadArg;
    EncodeJob j{w, n, h, p, a};
    return encode_launch(&j, 1, bs, f32, (cudaStream_t)stream);
}
int glint_encode_bf16_device(const uint16_t *d_w_bf16, int64_t n, int blocksize, uint8_t *d_hole_packed,
                             uint8_t *d_plug_packed, float *d_absmax, struct CUstream_st *stream)
{
    return device_encode(d_w_bf16, n, blocksize, d_hole_packed, d_plug_packed, d_absmax, false, stream);
}
int glint_encode_f32_device(const float *d_w, int64_t n, int blocksize, uint8_t *d_hole_packed,
                            uint8_t *d_plug_packed, float *d_absmax, struct CUstream_st *stream)
{
    return device_encode(d_w, n, blocksize, d_hole_packed, d_plug_packed, d_absmax, true, stream);
}

static int device_expand(const uint8_t *h, const uint8_t *p, const float *a, int64_t n, int bs, void *out, OutKind k,
                         struct CUstream_st *stream)
{
    if (!h || !p || !a || !out || bs <= 0)
        return kBadArg;
    if (n <= 0)
        return kOk;
    ExpandJob j{h, p, a, n, out};
    return expand_launch(&j, 1, bs, k, (cudaStream_t)stream);
}
int glint_expand_packed_to_f32_device(const uint8_t *d_hole_packed, const uint8_t *d_plug_packed,
                                      const float *d_absmax, int64_t n, int blocksize, float *d_out_f32,
                                      struct CUstream_st *stream)
{
    return device_expand(d_hole_packed, d_plug_packed, d_absmax, n, blocksize, d_out_f32, kOutF32, stream);
}
int glint_expand_packed_to_bf16_device(const uint8_t *d_hole_packed, const uint8_t *d_plug_packed,
                                       const float *d_absmax, int64_t n, int blocksize, uint16_t *d_out_bf16,
                                       struct CUstream_st *stream)
{
    return device_expand(d_hole_packed, d_plug_packed, d_absmax, n, blocksize, d_out_bf16, kOutBF16, stream);
}

int glint_encode_bf16_device_batch(const GlintTensorDesc *t, int count, int blocksize, struct CUstream_st *stream)
{
    if (count < 0 || (count > 0 && !t) || blocksize <= 0)
        return kBadArg;
    std::vector<EncodeJob> jobs((size_t)count);
    for (int i = 0; i < count; ++i) {
        if (t[i].n < 0)
            return kBadArg;
        jobs[i] = EncodeJob{t[i].dense, t[i].n, t[i].hole_packed, t[i].plug_packed, t[i].absmax};
    }
    return encode_launch(jobs.data(), count, blocksize, false, (cudaStream_t)stream);
}
int glint_expand_packed_to_bf16_device_batch(const GlintTensorDesc *t, int count, int blocksize,
                                             struct CUstream_st *stream)
{
    if (count < 0 || (count > 0 && !t) || blocksize <= 0)
        return kBadArg;
    std::vector<ExpandJob> jobs((size_t)count);
    for (int i = 0; i < count; ++i) {
        if (t[i].n < 0)
            return kBadArg;
        jobs[i] = ExpandJob{t[i].hole_packed, t[i].plug_packed, t[i].absmax, t[i].n, t[i].dense};
    }
    return expand_launch(jobs.data(), count, blocksize, kOutBF16, (cudaStream_t)stream);
}

int launch_glint_htile_s3_f32_stream(const uint8_t *d_hole, const uint8_t *d_plug, const float *d_absmax,
                                     const __nv_bfloat16 *d_x, float *d_y, int M, int N, int K, int blocksize,
                                     cudaStream_t stream)
{
    return htile_launch(d_hole, d_plug, d_absmax, d_x, d_y, kOutF32, M, N, K, blocksize, kPrecise, stream);
}
int launch_glint_htile_s3_f32(const uint8_t *d_hole, const uint8_t *d_plug, const float *d_absmax,
                              const __nv_bfloat16 *d_x, float *d_y, int M, int N, int K, int blocksize)
{
    return launch_glint_htile_s3_f32_stream(d_hole, d_plug, d_absmax, d_x, d_y, M, N, K, blocksize, 0);
}
int glint_htile_stream(const uint8_t *d_hole, const uint8_t *d_plug, const float *d_absmax,
                       const __nv_bfloat16 *d_x, void *d_y, int y_dtype, int M, int N, int K, int blocksize,
                       int mode, cudaStream_t stream)
{
    if ((y_dtype != GLINT_Y_F32 && y_dtype != GLINT_Y_BF16) || (mode != GLINT_HTILE_PRECISE && mode != GLINT_HTILE_FAST))
        return kBadArg;
    return htile_launch(d_hole, d_plug, d_absmax, d_x, d_y, y_dtype == GLINT_Y_BF16 ? kOutBF16 : kOutF32, M, N, K,
                        blocksize, mode == GLINT_HTILE_FAST ? kFast : kPrecise, stream);
}

int glint_htile_gather_stream(const uint8_t *d_hole, const uint8_t *d_plug, const float *d_absmax,
                              const __nv_bfloat16 *d_x, void *const *d_y_ranks, unsigned int *const *d_flag_ranks,
                              int world, int rank, int y_dtype, int M, int N, int K, int ld_y, int n0,
                              int blocksize, int mode, cudaStream_t stream)
{
    if (!d_hole || !d_plug || !d_absmax || !d_x || !d_y_ranks || !d_flag_ranks || world < 1 || rank < 0 ||
        rank >= world)
        return kBadArg;
    for (int r = 0; r < world; ++r)
        if (!d_y_ranks[r] || !d_flag_ranks[r])
            return kBadArg;
    if ((y_dtype != GLINT_Y_F32 && y_dtype != GLINT_Y_BF16) || (mode != GLINT_HTILE_PRECISE && mode != GLINT_HTILE_FAST))
        return kBadArg;
    if (blocksize <= 0)
        return kBadBlocksize;
    if (M <= 0 || N <= 0 || K <= 0 || n0 < 0 || ld_y < n0 + N)
        return kBadArg;
    const bool bf16 = y_dtype == GLINT_Y_BF16;
    if (htile_decode_supported(d_hole, d_plug, d_absmax, d_x, M, N, K, blocksize) && htile_gather_supported(M, N))
        return htile_decode_gather_launch(d_hole, d_plug, d_absmax, d_x, d_y_ranks, d_flag_ranks, world, rank,
                                          bf16 ? kOutBF16 : kOutF32, M, N, K, ld_y, n0,
                                          mode == GLINT_HTILE_FAST ? kFast : kPrecise, stream);
    /* prefill shapes: the tcgen05 GEMM stores its tiles into every rank's y */
    if (mode == GLINT_HTILE_FAST && htile_gemm_supported(d_hole, d_plug, d_absmax, d_x, nullptr, bf16, M, N, K, blocksize))
        return htile_gemm_gather_launch(d_hole, d_plug, d_absmax, d_x, d_y_ranks, d_flag_ranks, world, rank, bf16, M,
                                        N, K, ld_y, n0, stream);
    return kUnsupported;
}

int glint_gather_stream(const void *d_src, int elem_bytes, int M, int cols, int ld_src, void *const *d_y_ranks,
                        unsigned int *const *d_flag_ranks, int world, int rank, int ld_y, int n0,
                        cudaStream_t stream)
{
    if (!d_src || !d_y_ranks || !d_flag_ranks || world < 1 || rank < 0 || rank >= world || M < 1 || cols < 1 ||
        ld_src < cols || n0 < 0 || ld_y < n0 + cols)
        return kBadArg;
    for (int r = 0; r < world; ++r)
        if (!d_y_ranks[r] || !d_flag_ranks[r])
            return kBadArg;
    return gather_copy_launch(d_src, elem_bytes, M, cols, ld_src, d_y_ranks, d_flag_ranks, world, rank, ld_y, n0,
                              stream);
}

int glint_device_alloc(size_t bytes, void **d_ptr)
{
    if (!d_ptr || bytes == 0)
        return kBadArg;
    *d_ptr = nullptr;
    if (cudaMalloc(d_ptr, bytes) != cudaSuccess || cudaMemset(*d_ptr, 0, bytes) != cudaSuccess) {
        if (*d_ptr)
            cudaFree(*d_ptr);
        *d_ptr = nullptr;
        cudaGetLastError();
        return kLaunch;
    }
    return kOk;
}
int glint_device_free(void *d_ptr) { return d_ptr && cudaFree(d_ptr) != cudaSuccess ? kLaunch : kOk; }
int glint_ipc_handle(const void *d_ptr, void *handle_out)
{
    if (!d_ptr || !handle_out)
        return kBadArg;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, const_cast<void *>(d_ptr)) != cudaSuccess) {
        cudaGetLastError();
        return kLaunch;
    }
    std::memcpy(handle_out, &h, sizeof(h));
    return kOk;
}
int glint_ipc_open(const void *handle, void **d_ptr)
{
    if (!handle || !d_ptr)
        return kBadArg;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    *d_ptr = nullptr;
    if (cudaIpcOpenMemHandle(d_ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        *d_ptr = nullptr;
        return kLaunch;
    }
    return kOk;
}
int glint_ipc_close(void *d_ptr)
{
    if (!d_ptr)
        return kBadArg;
    if (cudaIpcCloseMemHandle(d_ptr) != cudaSuccess) {
        cudaGetLastError();
        return kLaunch;
    }
    return kOk;
}

int glint_htile_stream_noalloc(const uint8_t *d_hole, const uint8_t *d_plug, const float *d_absmax,
                               const __nv_bfloat16 *d_x, void *d_y, int y_dtype, int M, int N, int K,
                               int blocksize, int mode, cudaStream_t stream)
{
    if (!d_hole || !d_plug || !d_absmax || !d_x || !d_y)
        return kBadArg;
    if ((y_dtype != GLINT_Y_F32 && y_dtype != GLINT_Y_BF16) || (mode != GLINT_HTILE_PRECISE && mode != GLINT_HTILE_FAST))
        return kBadArg;
    if (blocksize <= 0)
        return kBadBlocksize;
    if (M <= 0 || N <= 0 || K <= 0 || !htile_decode_supported(d_hole, d_plug, d_absmax, d_x, M, N, K, blocksize))
        return kBadArg;
    return htile_decode_launch_noalloc(d_hole, d_plug, d_absmax, d_x, d_y, y_dtype == GLINT_Y_BF16 ? kOutBF16 : kOutF32,
                                       M, N, K, mode == GLINT_HTILE_FAST ? kFast : kPrecise, stream);
}

/* ---- K-major decode (include/glint_km.h) ---- */
/* The device address of a plug plane: device or managed memory as given, pinned
 * host memory through its mapping; nullptr for memory the device cannot read
 * (never handed to a kernel). */
static const uint8_t *device_view(const uint8_t *p)
{
    cudaPointerAttributes at{};
    if (!p || cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged)
        return p;
    if (at.type == cudaMemoryTypeHost && at.devicePointer)
        return static_cast<const uint8_t *>(at.devicePointer);
    return nullptr;
}

int glint_kmajor_from_rowmajor(const uint8_t *d_hole, const uint8_t *d_plug, const float *d_absmax, int n, int K,
                               int blocksize, uint8_t *d_hole_k, uint8_t *d_plug_k, float *d_scales_k,
                               cudaStream_t stream)
{
    if (!d_hole || !d_absmax || !d_hole_k || !d_scales_k || (!d_plug) != (!d_plug_k))
        return kBadArg;
    if (blocksize != 64)
        return kBadBlocksize;
    if (!km_supported(n, K, d_hole_k, d_scales_k) || (d_plug_k && !aligned_to(d_plug_k, 16)))
        return kBadArg;
    return km_layout_launch(d_hole, d_plug, d_absmax, n, K, d_hole_k, d_plug_k, d_scales_k, stream);
}
int glint_gemv_km_stream(const uint8_t *d_hole_k, const float *d_scales_k, const __nv_bfloat16 *d_x, float *d_y,
                         int n, int K, cudaStream_t stream)
{
    if (!d_hole_k || !d_scales_k || !d_x || !d_y || !km_supported(n, K, d_hole_k, d_scales_k))
        return kBadArg;
    return km_gemv_launch(d_hole_k, d_scales_k, d_x, d_y, n, K, stream);
}
int glint_select_topk_stream(const __nv_bfloat16 *d_x, int K, int nsel, int *d_idx, int *d_cnt, cudaStream_t stream)
{
    if (!d_x || !d_idx || !d_cnt || K < 1 || K > kKmMaxK || nsel < 0)
        return kBadArg;
    return km_select_launch(d_x, K, nsel, d_idx, d_cnt, stream);
}
int glint_apply_corr_k_stream(const uint8_t *d_hole_k, const uint8_t *plug_k, const float *d_scales_k,
                              const __nv_bfloat16 *d_x, const int *d_idx, const int *d_cnt, float *d_y, int n, int K,
                              cudaStream_t stream)
{
    const uint8_t *pk = device_view(plug_k);
    if (!d_hole_k || !pk || !d_scales_k || !d_x || !d_idx || !d_cnt || !d_y ||
        !km_supported(n, K, d_hole_k, d_scales_k) || !aligned_to(pk, 16))
        return kBadArg;
    return km_corr_launch(d_hole_k, pk, d_scales_k, d_x, d_idx, d_cnt, d_y, n, K, stream);
}
int glint_gemv_select_stream(const uint8_t *d_hole_k, const uint8_t *plug_k, const float *d_scales_k,
                             const __nv_bfloat16 *d_x, float *d_y, int n, int K, int nsel, int *d_idx, int *d_cnt,
                             cudaStream_t stream)
{
    const uint8_t *pk = device_view(plug_k);
    if (!d_hole_k || !pk || !d_scales_k || !d_x || !d_y || !d_idx || !d_cnt || nsel < 0 ||
        !km_supported(n, K, d_hole_k, d_scales_k) || !aligned_to(pk, 16))
        return kBadArg;
    return km_gemv_select_launch(d_hole_k, pk, d_scales_k, d_x, d_y, n, K, nsel, d_idx, d_cnt, stream);
}

} /* extern "C" */
