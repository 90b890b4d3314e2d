/* GLINT plug streamer C ABI (libglint_encode.so): per-layer plug planes kept in
 * pinned host memory and streamed into a two-slot VRAM ring ahead of the layer
 * that reads them, so only the hole planes and absmax stay resident on the GPU.
 *
 * Same declarations, call order and return codes as the reference streamer
 * (Jadon-Fox/glint include/glint_plug_streamer.h:11-61,
 * cuda/glint_plug_streamer.cu:27-215):
 *   create      0 ok, -1 bad arguments (n_layers outside [1, 64]), -2 out of host
 *               memory, -3 device slots, -4 pinned host memory, -5 events;
 *   set_host_data  -1 bad arguments, -2 size differs from the layer's;
 *   start       -6 the previous pass did not release its last layer (no state
 *               change, so a failed start can be retried), other negatives are
 *               CUDA failures while queueing layer 0's copy;
 *   acquire     -10 unless layer - 1 was released (or layer == 0 after start);
 *   release     -11 unless `layer` was acquired and layer - 1 released.
 * Layer l lives in slot l & 1.  acquire(l) queues the copy of layer l + 1 on
 * copy_stream behind the last release of its slot, and makes compute_stream wait
 * for layer l's copy; release(l) marks the point on compute_stream after which
 * slot l & 1 may be overwritten, so every read of the slot must be enqueued on
 * compute_stream before it.  A pass that stops early is finished by acquiring and
 * releasing the remaining layers in order (there is no abort).
 */
#ifndef GLINT_PLUG_STREAMER_H_
#define GLINT_PLUG_STREAMER_H_
#include <cuda_runtime.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct GlintPlugStreamer GlintPlugStreamer;

typedef struct {
    uint64_t total_h2d_bytes;      /* bytes queued host -> device since the last reset */
    double total_stall_ms;         /* sum of per_layer_stall_ms */
    double per_layer_stall_ms[64]; /* compute_stream time spent waiting for the layer's copy */
    int n_layers;
} GlintStreamerStats;

int glint_plug_streamer_create(GlintPlugStreamer **out, int n_layers, const uint64_t *layer_bytes,
                               cudaStream_t copy_stream, cudaStream_t compute_stream);
void glint_plug_streamer_destroy(GlintPlugStreamer *s);
/* Copy a layer's plug bytes into the streamer's pinned host memory. */
int glint_plug_streamer_set_host_data(GlintPlugStreamer *s, int layer, const void *host_src, uint64_t bytes);
/* Queue layer 0's copy (slot 0) before the layer loop. */
int glint_plug_streamer_start(GlintPlugStreamer *s);
int glint_plug_streamer_acquire(GlintPlugStreamer *s, int layer, const uint8_t **out_dev_plug);
int glint_plug_streamer_release(GlintPlugStreamer *s, int layer);
/* Waits for both streams, then reports bytes and per-layer stalls of the last pass. */
int glint_plug_streamer_get_stats(GlintPlugStreamer *s, GlintStreamerStats *stats);
/* Waits for both streams and zeroes the counters. */
void glint_plug_streamer_reset_stats(GlintPlugStreamer *s);

/* ---- additive (no counterpart in the reference ABI) ----------------------- */
/* The pinned host buffer of a layer (layer_bytes[layer] bytes), so a producer
 * such as glint_encode_bf16_host can write plugs there without a staging copy;
 * NULL for a bad layer.  Writes must finish before the pass that copies it. */
uint8_t *glint_plug_streamer_host_buffer(GlintPlugStreamer *s, int layer);

/* the reference's P7 names */
typedef GlintPlugStreamer P7PlugStreamer;
typedef GlintStreamerStats P7StreamerStats;
#define p7_plug_streamer_create glint_plug_streamer_create
#define p7_plug_streamer_destroy glint_plug_streamer_destroy
#define p7_plug_streamer_set_host_data glint_plug_streamer_set_host_data
#define p7_plug_streamer_start glint_plug_streamer_start
#define p7_plug_streamer_acquire glint_plug_streamer_acquire
#define p7_plug_streamer_release glint_plug_streamer_release
#define p7_plug_streamer_get_stats glint_plug_streamer_get_stats
#define p7_plug_streamer_reset_stats glint_plug_streamer_reset_stats

#ifdef __cplusplus
}
#endif
#endif /* GLINT_PLUG_STREAMER_H_ */
