/* GLINT plug streamer: per-layer plug planes in pinned host memory, streamed
 * into a two-slot VRAM ring one layer ahead of the compute stream.
 *
 * Reference behaviour: include/glint_plug_streamer.h:11-61 and
 * cuda/glint_plug_streamer.cu:27-215 (same calls, ordering rules and return
 * codes).  The host side is laid out for a B200 node:
 *   - one pinned arena for all layers (4 KiB-aligned offsets) and one device
 *     allocation for both slots, instead of an allocation per layer;
 *   - copy completion and slot reuse are ordered by events created without
 *     timing (cheaper to record and wait on); only the stall brackets on
 *     compute_stream carry timestamps, for the stats;
 *   - one cudaMemcpyAsync per layer: a single large pinned copy already runs
 *     the PCIe link at its rate, and the ring depth of two hides it behind a
 *     layer's compute whenever the copy is the shorter of the two;
 *   - set_host_data splits large layers over host threads (pinned writes of
 *     ~100 MB layers are memory-bandwidth work);
 *   - calls on one streamer are serialised by a mutex, so serving threads may
 *     share it (the reference leaves threading to the caller).
 */
#include <algorithm>
#include <cstring>
#include <mutex>
#include <new>
#include <thread>
#include <vector>

#include "../../include/glint_plug_streamer.h"

namespace {
constexpr int kMaxLayers = 64;
constexpr uint64_t kHostAlign = 4096;
constexpr uint64_t kParallelCopyBytes = 64ull << 20;

uint64_t round_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

/* memcpy split over up to 8 host threads for large buffers */
void host_copy(void *dst, const void *src, uint64_t bytes)
{
    if (bytes < kParallelCopyBytes) {
        std::memcpy(dst, src, (size_t)bytes);
        return;
    }
    const unsigned hw = std::max(1u, std::min(8u, std::thread::hardware_concurrency()));
    const uint64_t part = round_up((bytes + hw - 1) / hw, kHostAlign);
    std::vector<std::thread> th;
    for (unsigned t = 0; t < hw; ++t) {
        const uint64_t o = (uint64_t)t * part;
        if (o >= bytes)
            break;
        const uint64_t n = std::min(part, bytes - o);
        th.emplace_back([=] {
            std::memcpy(static_cast<uint8_t *>(dst) + o, static_cast<const uint8_t *>(src) + o, (size_t)n);
        });
    }
    for (auto &t : th)
        t.join();
}
} // namespace

struct GlintPlugStreamer {
    std::mutex mu;
    int n_layers = 0;
    uint64_t layer_bytes[kMaxLayers] = {};
    uint64_t host_off[kMaxLayers] = {};
    uint64_t max_bytes = 0;
    uint8_t *host = nullptr;  /* pinned arena */
    uint8_t *device = nullptr; /* both slots */
    uint8_t *slot[2] = {nullptr, nullptr};
    cudaStream_t copy_stream = nullptr;
    cudaStream_t compute_stream = nullptr;
    cudaEvent_t copied[kMaxLayers] = {};  /* layer's copy complete (no timing) */
    cudaEvent_t stall_b[kMaxLayers] = {}; /* compute_stream before / after waiting for it */
    cudaEvent_t stall_e[kMaxLayers] = {};
    bool stalled[kMaxLayers] = {};        /* the stall pair was recorded this pass */
    cudaEvent_t slot_free[2] = {nullptr, nullptr};
    int acquired_through = -1;
    int released_through = -1;
    GlintStreamerStats stats{};
};

namespace {
void release_all(GlintPlugStreamer *s)
{
    for (int b = 0; b < 2; ++b)
        if (s->slot_free[b])
            cudaEventDestroy(s->slot_free[b]);
    for (int l = 0; l < s->n_layers; ++l) {
        if (s->copied[l])
            cudaEventDestroy(s->copied[l]);
        if (s->stall_b[l])
            cudaEventDestroy(s->stall_b[l]);
        if (s->stall_e[l])
            cudaEventDestroy(s->stall_e[l]);
    }
    if (s->device)
        cudaFree(s->device);
    if (s->host)
        cudaFreeHost(s->host);
    cudaGetLastError();
    delete s;
}

/* queue layer l's copy into its slot behind the slot's last release */
int queue_copy(GlintPlugStreamer *s, int l, int e_wait, int e_copy, int e_record)
{
    const int b = l & 1;
    if (cudaStreamWaitEvent(s->copy_stream, s->slot_free[b], 0) != cudaSuccess)
        return e_wait;
    if (cudaMemcpyAsync(s->slot[b], s->host + s->host_off[l], (size_t)s->layer_bytes[l], cudaMemcpyHostToDevice,
                        s->copy_stream) != cudaSuccess)
        return e_copy;
    if (cudaEventRecord(s->copied[l], s->copy_stream) != cudaSuccess)
        return e_record;
    s->stats.total_h2d_bytes += s->layer_bytes[l];
    return 0;
}
} // namespace

extern "C" {

int glint_plug_streamer_create(GlintPlugStreamer **out, int n_layers, const uint64_t *layer_bytes,
                               cudaStream_t copy_stream, cudaStream_t compute_stream)
{
    if (!out || n_layers <= 0 || n_layers > kMaxLayers || !layer_bytes)
        return -1;
    GlintPlugStreamer *s = new (std::nothrow) GlintPlugStreamer();
    if (!s)
        return -2;
    s->n_layers = n_layers;
    s->copy_stream = copy_stream;
    s->compute_stream = compute_stream;
    uint64_t total = 0;
    for (int l = 0; l < n_layers; ++l) {
        s->layer_bytes[l] = layer_bytes[l];
        s->max_bytes = std::max(s->max_bytes, layer_bytes[l]);
        s->host_off[l] = total;
        total += round_up(std::max<uint64_t>(layer_bytes[l], 1), kHostAlign);
    }
    const uint64_t slot_bytes = round_up(std::max<uint64_t>(s->max_bytes, 1), 256);
    if (cudaMalloc(reinterpret_cast<void **>(&s->device), (size_t)(2 * slot_bytes)) != cudaSuccess) {
        s->device = nullptr;
        release_all(s);
        return -3;
    }
    s->slot[0] = s->device;
    s->slot[1] = s->device + slot_bytes;
    for (int b = 0; b < 2; ++b)
        if (cudaEventCreateWithFlags(&s->slot_free[b], cudaEventDisableTiming) != cudaSuccess) {
            s->slot_free[b] = nullptr;
            release_all(s);
            return -3;
        }
    if (cudaHostAlloc(reinterpret_cast<void **>(&s->host), (size_t)total, cudaHostAllocDefault) != cudaSuccess) {
        s->host = nullptr;
        release_all(s);
        return -4;
    }
    for (int l = 0; l < n_layers; ++l) {
        if (cudaEventCreateWithFlags(&s->copied[l], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreate(&s->stall_b[l]) != cudaSuccess || cudaEventCreate(&s->stall_e[l]) != cudaSuccess) {
            release_all(s);
            return -5;
        }
    }
    /* no pass in flight: start() may begin one */
    s->acquired_through = n_layers - 1;
    s->released_through = n_layers - 1;
    s->stats.n_layers = n_layers;
    *out = s;
    return 0;
}

void glint_plug_streamer_destroy(GlintPlugStreamer *s)
{
    if (!s)
        return;
    /* copies out of the pinned arena and reads of the slots must be done first */
    cudaStreamSynchronize(s->copy_stream);
    cudaStreamSynchronize(s->compute_stream);
    release_all(s);
}

int glint_plug_streamer_set_host_data(GlintPlugStreamer *s, int layer, const void *host_src, uint64_t bytes)
{
    if (!s || layer < 0 || layer >= s->n_layers || !host_src)
        return -1;
    if (bytes != s->layer_bytes[layer])
        return -2;
    std::lock_guard<std::mutex> lk(s->mu);
    host_copy(s->host + s->host_off[layer], host_src, bytes);
    return 0;
}

uint8_t *glint_plug_streamer_host_buffer(GlintPlugStreamer *s, int layer)
{
    if (!s || layer < 0 || layer >= s->n_layers)
        return nullptr;
    return s->host + s->host_off[layer];
}

int glint_plug_streamer_start(GlintPlugStreamer *s)
{
    if (!s || s->n_layers <= 0)
        return -1;
    std::lock_guard<std::mutex> lk(s->mu);
    if (s->released_through != s->n_layers - 1)
        return -6;
    const int rc = queue_copy(s, 0, -5, -3, -4);
    if (rc)
        return rc;
    for (int l = 0; l < s->n_layers; ++l)
        s->stalled[l] = false;
    s->acquired_through = -1;
    s->released_through = -1;
    return 0;
}

int glint_plug_streamer_acquire(GlintPlugStreamer *s, int layer, const uint8_t **out_dev_plug)
{
    if (!s || layer < 0 || layer >= s->n_layers || !out_dev_plug)
        return -1;
    std::lock_guard<std::mutex> lk(s->mu);
    if (s->released_through != layer - 1)
        return -10;
    if (layer + 1 < s->n_layers) {
        const int rc = queue_copy(s, layer + 1, -2, -4, -5);
        if (rc)
            return rc;
    }
    if (cudaEventRecord(s->stall_b[layer], s->compute_stream) != cudaSuccess)
        return -6;
    if (cudaStreamWaitEvent(s->compute_stream, s->copied[layer], 0) != cudaSuccess)
        return -7;
    if (cudaEventRecord(s->stall_e[layer], s->compute_stream) != cudaSuccess)
        return -8;
    s->stalled[layer] = true;
    s->acquired_through = layer;
    *out_dev_plug = s->slot[layer & 1];
    return 0;
}

int glint_plug_streamer_release(GlintPlugStreamer *s, int layer)
{
    if (!s || layer < 0 || layer >= s->n_layers)
        return -1;
    std::lock_guard<std::mutex> lk(s->mu);
    if (layer != s->released_through + 1 || layer != s->acquired_through)
        return -11;
    if (cudaEventRecord(s->slot_free[layer & 1], s->compute_stream) != cudaSuccess)
        return -2;
    s->released_through = layer;
    return 0;
}

int glint_plug_streamer_get_stats(GlintPlugStreamer *s, GlintStreamerStats *stats)
{
    if (!s || !stats)
        return -1;
    std::lock_guard<std::mutex> lk(s->mu);
    cudaStreamSynchronize(s->copy_stream);
    cudaStreamSynchronize(s->compute_stream);
    double total = 0.0;
    for (int l = 0; l < s->n_layers; ++l) {
        float ms = 0.f;
        if (!s->stalled[l] || cudaEventElapsedTime(&ms, s->stall_b[l], s->stall_e[l]) != cudaSuccess)
            ms = 0.f;
        s->stats.per_layer_stall_ms[l] = (double)ms;
        total += (double)ms;
    }
    cudaGetLastError();
    s->stats.total_stall_ms = total;
    *stats = s->stats;
    return 0;
}

void glint_plug_streamer_reset_stats(GlintPlugStreamer *s)
{
    if (!s)
        return;
    std::lock_guard<std::mutex> lk(s->mu);
    cudaStreamSynchronize(s->copy_stream);
    cudaStreamSynchronize(s->compute_stream);
    s->stats.total_h2d_bytes = 0;
    s->stats.total_stall_ms = 0.0;
    std::memset(s->stats.per_layer_stall_ms, 0, sizeof(s->stats.per_layer_stall_ms));
}

} // extern "C"
