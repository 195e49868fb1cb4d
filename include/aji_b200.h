/*
 * aji_b200.h — the native hot path of this engine as a C ABI: the fused 3x3 conv kernels, the
 * 1x1 concat kernel, the colour pre/post passes, the on-device image tiler, the native model
 * (a plan of fused conv steps) and its executor. Plain pointers and sizes only; device pointers
 * are CUDA device addresses on the current device, `stream` is a cudaStream_t (NULL = legacy
 * default stream).
 *
 * Each declaration names the reference interface it replaces (the-database/animejanai-inference,
 * file:line). The reference exposes these as C++ functions inside its backend library; a caller
 * that wants the kernels alone (a test, a benchmark, another front-end) binds them here.
 *
 * Return codes: AJIB_OK (0) or a negative AJIB_ERR_*.
 */
#ifndef AJI_B200_H
#define AJI_B200_H

#include <stddef.h>
#include <stdint.h>

#include "aji.h"
#include "aji_image.h"

#ifdef __cplusplus
extern "C" {
#endif

#define AJIB_EXPORT __attribute__((visibility("default")))

enum ajib_status {
    AJIB_OK = 0,
    AJIB_ERR = -1,
    AJIB_ERR_ARGS = -2,        /* a bad pointer, size or shape */
    AJIB_ERR_UNSUPPORTED = -3, /* no kernel for this combination */
    AJIB_ERR_CUDA = -4,        /* a CUDA call failed */
    AJIB_ERR_NO_MEM = -5,      /* a device or host allocation failed */
    AJIB_ERR_TIMEOUT = -6,     /* a kernel gave up waiting on its own pipeline (ajib_kernel_status) */
};

/* ---- op vocabulary (reference src/native/ops.h:13-21; same integer values) ---- */
enum ajib_input { AJIB_IN_NHWC = 0, AJIB_IN_NCHW3 = 1, AJIB_IN_NCHW3_UNSHUFFLE2 = 2 };
enum ajib_act { AJIB_ACT_NONE = 0, AJIB_ACT_RELU = 1, AJIB_ACT_PRELU = 2, AJIB_ACT_SILU = 3 };
enum ajib_gate { AJIB_GATE_NONE = 0, AJIB_GATE_RESIDUAL = 1, AJIB_GATE_TANH1X1 = 2, AJIB_GATE_SIGMOID_HALF = 3 };
enum ajib_output { AJIB_OUT_NHWC = 0, AJIB_OUT_D2S2 = 1, AJIB_OUT_D2S4 = 2, AJIB_OUT_D2S1 = 3, AJIB_OUT_D2S3 = 4 };

/* ---- conv weights (reference src/native/conv.h:34-49, upload/release) ----
 * w: [taps][cin][cout] fp16 bit patterns (ONNX OIHW transposed to HWIO), bias: cout floats,
 * slope: cout floats (PReLU) or NULL. taps is 9 (3x3) or 1 (1x1). Packed on the host into the
 * tensor-core operand image the kernels copy to shared memory, and uploaded to the current
 * device. */
typedef struct ajib_weights ajib_weights;
AJIB_EXPORT int ajib_weights_upload(ajib_weights **out, const uint16_t *w, const float *bias, const float *slope,
                                    int taps, int cin, int cout);
AJIB_EXPORT void ajib_weights_release(ajib_weights **w);
AJIB_EXPORT size_t ajib_weights_bytes(const ajib_weights *w);

/* ---- one fused 3x3 conv (reference src/native/conv.h:53-66, struct Conv3x3) ----
 * Logical channel counts: an NCHW3 input has cin 3, a pixel-unshuffled one (NCHW3_UNSHUFFLE2,
 * channel c * 4 + ry * 2 + rx of the input [3][2H][2W]) 12; a D2S1/2/3/4 output has cout
 * 3/12/27/48. AJIB_GATE_TANH1X1 computes (x + fp16(o)) * tanh(att(fp16(o))), att the 1x1 conv in
 * `att` (uploaded with taps 1, cin = cout = the op's cout). */
typedef struct ajib_conv {
    int in, act, gate, out; /* enum ajib_input / ajib_act / ajib_gate / ajib_output */
    int cin, cout;
    const ajib_weights *w;
    const ajib_weights *att; /* AJIB_GATE_TANH1X1: the 1x1 cout -> cout attention conv */
    int in_norm;             /* NCHW3 input: load (x - in_mean[c]) * in_scale[c] */
    float in_mean[3], in_scale[3];
    int out_clamp; /* depth-to-space outputs: clamp to [0, 1] after the model input is added */
} ajib_conv;

/* Whether a kernel exists for op (reference src/native/conv.h:86, supported); why (may be NULL)
 * receives the reason for a refusal. Returns 1 or 0. */
AJIB_EXPORT int ajib_conv_supported(const ajib_conv *op, char *why, size_t why_size);

/* Feature maps (the NHWC tensors between steps) are stored strip-chunked: each row of a C-channel
 * map (C a multiple of 8) is cut into S = ajib_feature_strips(W) strips of 128 pixels, and each
 * (row, strip) is one contiguous block of C/8 chunks of 130 columns of 8 fp16 channels — the
 * strip's pixels and a halo column on each side. Element (y, x, c), x in strip s = x / 128, is the
 * fp16 at index
 *   ((((y * S + s) * C/8 + c/8) * 130 + x - 128 s + 1) * 8 + c % 8,
 * and a strip's halo columns (0 and 129) hold copies of the neighbouring strips' edge pixels; the
 * columns at the image's edges (column 0 of strip 0, and every column past W) must hold zeros
 * (clear the buffer once; the kernels never write them). A staged input row is then one
 * contiguous block the kernels copy in one piece. ajib_feature_bytes gives the buffer size. */
/* The 1x1 convolution over the concatenation of nsrc (2..4) strip-chunked maps of c channels (c a
 * multiple of 8, 8..64) into a strip-chunked map of c channels, plus bias (SPAN's concat + conv;
 * replaces the reference's ConcatConv1x1 / k_concat1x1, src/native/conv.h:38-102 and
 * conv_kernels.cuh:351-407). w: 1x1 weights uploaded with taps 1, cin nsrc * c, cout c (K index
 * k * c + i is channel i of source k). Rows [row_begin, row_end) (row_end <= 0: all). */
AJIB_EXPORT int ajib_concat1x1_launch(const ajib_weights *w, int nsrc, const void *const *srcs, int c, void *dst,
                                      int H, int W, int row_begin, int row_end, void *stream);
AJIB_EXPORT int ajib_feature_strips(int W);
AJIB_EXPORT size_t ajib_feature_bytes(int H, int W, int C);

/* Launch op at conv resolution H x W on output rows [row_begin, row_end) (row_end <= 0: all
 * rows) (reference src/native/conv.h:91, launch). src: a strip-chunked map [H][cin] or the NCHW
 * fp16 model input [3][H][W] ([3][2H][2W] pixel-unshuffled). resid: gates read the block input x
 * as a strip-chunked map [H][cout]; depth-to-space outputs add the NCHW model input [3][H][W]
 * (nearest upsampled) when resid is not NULL (not with a pixel-unshuffled input: AJIB_ERR_ARGS).
 * dst: a strip-chunked map [H][cout] or NCHW [3][R*H][R*W]. Rows outside the range are neither
 * read beyond the one-row halo nor written, so a frame can be run as bands. */
AJIB_EXPORT int ajib_conv3x3_launch(const ajib_conv *op, const void *src, const void *resid, void *dst, int H, int W,
                                    int row_begin, int row_end, void *stream);

/* The same over nimg images of img_h rows stacked along H (H = nimg * img_h): each image is
 * convolved on its own, zero-padded at its own top and bottom rows. One launch for a batch of
 * equal-size tiles (the image tiler); no reference counterpart (the reference runs tiles one by
 * one, src/aji_img_trt.cpp:980-1011). */
AJIB_EXPORT int ajib_conv3x3_launch_images(const ajib_conv *op, const void *src, const void *resid, void *dst,
                                           int nimg, int img_h, int W, int row_begin, int row_end, void *stream);

/* Strip-chunked convs with cin == cout at 32, 48 or 64 padded channels and an activation, or at
 * 32 or 48 and a SPAN gate, can run on SM pairs (one tcgen05 MMA over a cluster of two CTAs, each
 * SM holding half of the weights) instead of the one-SM kernel. Off by default (slower on B200 as
 * built); mode 1 / 0 turns pairs on / off for the process (the environment variable AJIB_PAIR=1
 * sets the initial state to on); any other value only queries. Returns the mode now in force. Both
 * kernels compute the same sums; results may differ in the last bits of the fp32 accumulation
 * order. */
AJIB_EXPORT int ajib_conv_pair_mode(int mode);
/* 1 when op runs on SM pairs in the current mode, else 0. */
AJIB_EXPORT int ajib_conv_on_pairs(const ajib_conv *op);
/* How many SM pairs (clusters of two CTAs) of the 64-channel pair kernel the current device runs
 * at once, or a negative AJIB_ERR_*. */
AJIB_EXPORT int ajib_conv_pair_clusters(void);

/* ---- colour passes (reference src/kernels.h:12-78; same names, arguments and semantics) ----
 * Normalisation constants in raw container units (P010 samples are 10 bits in the high bits of
 * 16, so its scales include the << 6): y = (raw - yoff) / yscale, c = (raw - coff) / cscale. */
typedef struct aji_csp {
    float kr, kb;
    float yoff, yscale;
    float coff, cscale;
} aji_csp;

/* reference src/kernels.h:21 (constants: src/resample.h:100-129) */
AJIB_EXPORT aji_csp aji_make_csp(int format, int matrix, int range);

typedef struct aji_plan aji_plan;
enum { AJI_FILTER_SPLINE36 = 0, AJI_FILTER_BILINEAR = 1 };

/* Resampling plans (reference src/kernels.h:46-49): the filter tables of zimg's compute_filter
 * for 4:2:0 chroma at luma size w x h and the given siting, uploaded to the current device.
 * Runs must use the same device. NULL on failure. */
AJIB_EXPORT aji_plan *aji_pre_plan_create(int format, int w, int h, int siting, int filter);
AJIB_EXPORT aji_plan *aji_post_plan_create(int format, int w, int h, int siting, int filter);
AJIB_EXPORT void aji_plan_destroy(aji_plan *p);
/* Spline36 resize plan, sw x sh -> dw x dh (reference src/kernels.h:48, zimg semantics: kernel
 * stretched by 1/scale when downscaling, mirrored borders). NULL on failure. */
AJIB_EXPORT aji_plan *aji_resize_plan_create(int sw, int sh, int dw, int dh);
/* Resize fp16 NCHW RGB [3][sh][sw] -> [3][dh][dw] with a resize plan (reference src/kernels.h:
 * 77-78): horizontal then vertical pass, fp32 between them, one rounding to fp16. One kernel.
 * Returns 0 or a cudaError_t. */
AJIB_EXPORT int aji_run_resize(aji_plan *p, const void *src_f16, void *dst_f16, void *stream);

/* NV12/P010 -> fp16 NCHW RGB [3][h][w] (reference src/kernels.h:52-55): chroma upsampled with
 * the plan's filter, then the matrix; fp32 throughout, one rounding to fp16. One kernel. Returns
 * 0 or a cudaError_t. */
AJIB_EXPORT int aji_run_pre(aji_plan *p, const void *y_plane, ptrdiff_t y_stride, const void *uv_plane,
                            ptrdiff_t uv_stride, const aji_csp *csp, void *dst_f16, void *stream);

/* fp16 NCHW RGB [3][h][w] -> NV12/P010 (reference src/kernels.h:58-60): matrix, luma quantised,
 * chroma downsampled (horizontal then vertical, fp32) and quantised. P010 quantises at 10 bits
 * then shifts. One kernel. Returns 0 or a cudaError_t. */
AJIB_EXPORT int aji_run_post(aji_plan *p, const void *src_f16, const aji_csp *csp, void *y_plane, ptrdiff_t y_stride,
                             void *uv_plane, ptrdiff_t uv_stride, void *stream);

/* 4:4:4 16-bit planar variants, matrix only (reference src/kernels.h:64-75). */
AJIB_EXPORT int aji_run_post444(int format, int w, int h, const void *src_f16, const aji_csp *csp, void *y_plane,
                                ptrdiff_t y_stride, void *cb_plane, ptrdiff_t cb_stride, void *cr_plane,
                                ptrdiff_t cr_stride, void *stream);
AJIB_EXPORT int aji_run_pre444(int w, int h, const void *y_plane, ptrdiff_t y_stride, const void *cb_plane,
                               ptrdiff_t cb_stride, const void *cr_plane, ptrdiff_t cr_stride, const aji_csp *csp,
                               void *dst_f16, void *stream);

/* The filter table the plans upload, computed on the host alone (no device): zimg's
 * compute_filter (reference src/resample.h:53-84) for src -> dst samples with the given shift.
 * Returns taps; start [dst] and wt [dst][taps] are filled when both are not NULL. */
AJIB_EXPORT int ajib_filter_table(int src, int dst, double shift, int filter, int *start, float *wt);

/* The plan's filter tables as the host computed them (for tests): which = 0 horizontal, 1
 * vertical. Copies up to max_dst entries of start and max_dst * taps weights; returns taps. */
AJIB_EXPORT int ajib_plan_table(const aji_plan *p, int which, int *start, float *wt, int max_dst);

/* Which kernel a colour plan's runs use (for tests and profiles; no reference counterpart, the
 * reference has one kernel form): 1 = the streaming form (blocks walk column strips downwards,
 * each source row staged once by asynchronous copies; chosen at plan creation when the filter
 * tables are 2:1 with one set of weights and the width is a multiple of 8), 0 = the tiled form
 * (serves every plan), -1 = bad plan. Each run checks its buffers' alignment again and uses the
 * tiled form for unaligned buffers. */
AJIB_EXPORT int ajib_plan_kernel(const aji_plan *p);

/* ---- the image tiler on the GPU ----
 * Geometry of the reference's cover (src/core/tiling.cpp:17-103: tile origins flush to the far
 * edge or even tiles, reflect padding, linear blend ramps across a 16-pixel band at the centre of
 * each overlap, normalised per axis), uploaded for one image shape. Replaces the reference's
 * gpu_tile_extract / gpu_tile_blend / gpu_band_flush (src/core/tiling_gpu.h:49-67):
 *  - extract cuts tiles [k0, k0 + n) (k = tile row * nx + tile column) of the device image
 *    (W x H x ci, packed, 8-bit) into fp16 [3][n * th][tw] (tiles stacked along H), v / 255;
 *  - compose blends the model outputs of all tiles, fp16 [3][nx * ny * th * S][tw * S], into the
 *    8-bit output (H * S) x (W * S) x ci, bit-identical to blending each tile into an fp32 band
 *    in tile order and flushing it. */
typedef struct ajib_tiler ajib_tiler;
AJIB_EXPORT int ajib_tiler_create(int W, int H, int ci, int scale, int tile_w, int tile_h, int overlap, int even,
                                  ajib_tiler **out);
AJIB_EXPORT int ajib_tiler_info(const ajib_tiler *t, int *nx, int *ny, int *tw, int *th);
AJIB_EXPORT int ajib_tiler_extract(ajib_tiler *t, const uint8_t *img, int k0, int n, void *dst, void *stream);
AJIB_EXPORT int ajib_tiler_compose(ajib_tiler *t, const void *tiles, uint8_t *out, void *stream);
AJIB_EXPORT void ajib_tiler_release(ajib_tiler **t);

/* Compose without allocating device memory. This entry point has no counterpart in the
 * reference; it exists for callers that may not call cudaMalloc, such as a host application
 * whose device memory all comes from its own allocator or budget, or a real-time frame path
 * where cudaMalloc / cudaFree would synchronise the device. It does what ajib_tiler_create +
 * ajib_tiler_compose + ajib_tiler_release do for one image shape (same arguments, same bytes
 * out), but the geometry tables go into a fixed 1 MiB area inside this library that every GPU
 * loading it holds until the process exits; the tables of outputs up to about 24K x 24K pixels
 * fit. The caller passes the tiles and the output, both device memory.
 * Returns AJIB_OK, AJIB_ERR_ARGS for bad arguments, AJIB_ERR_UNSUPPORTED when the shape's tables
 * exceed the 1 MiB area, AJIB_ERR_CUDA on a CUDA error.
 * The first call on a device looks up the area's device address (with that device current).
 * Every call on a device uses the same area and
 * leaves its tables there: calls that overlap on the GPU (other streams, or the next call before
 * this one's kernel has run on another stream) race; calls on one stream are ordered by it. Each
 * call uploads its tables by a copy from host memory inside this library, which may wait for
 * earlier work on `stream` before the call returns. */
AJIB_EXPORT int ajib_tiler_compose_static(int W, int H, int ci, int scale, int tile_w, int tile_h, int overlap,
                                          int even, const void *tiles, uint8_t *out, void *stream);

/* ---- several GPUs for one image ----
 * An image context over n devices (aji_img_device.id values; 0 = the first device), used like one
 * from aji_img_create with the rest of include/aji_image.h. The reference's image ABI has one
 * device per context (aji_img_create, include/aji_image.h:124-125); this additive entry point is
 * what its dispatcher would probe, like the reference's optional 0.24+ additions
 * (aji_image.h:220-222). aji_img_upscale splits the output rows into one band per device at tile
 * row boundaries: each device uploads the image, runs the tile rows covering its band (the tile
 * row before the band, whose blend reaches into it, runs on both neighbours) and blends and
 * downloads only its band, so no data crosses devices and the bytes equal the one-device result.
 * Progress is reported per finished band. */
AJIB_EXPORT aji_img_ctx *ajib_img_create_multi(const aji_img_create_params *p, const uint64_t *device_ids, int n,
                                               char *err, size_t err_size);
/* The bands ajib_img_create_multi's upscale gives ndev devices for one image shape (host only):
 * returns the number of bands used (min(ndev, tile rows)); band d owns output rows
 * [y0[d], y1[d]) and runs tile rows [j0[d], j1[d]]. Arrays hold ndev entries. -1: bad arguments. */
AJIB_EXPORT int ajib_img_shares(int W, int H, int ci, int scale, int tile_w, int tile_h, int overlap, int even, int ndev,
                                int *y0, int *y1, int *j0, int *j1);

/* ---- several GPUs for one video stream ----
 * One stream upscaled frame-parallel on n devices of this host (CUDA ordinals, no duplicates):
 * frame k (ticket k + 1) runs on device k mod n, each device with its own video context built
 * from the same create params (direct or conf mode, see aji.h), its own upload, compute and
 * download streams and a ring of `depth` (1..16) frame slots; results complete in submission
 * order, as a one-device player sees them (the reference harness's one-stream loop,
 * src/harness.c:646-700). The reference's video ABI serves one device per context (aji_create,
 * include/aji.h:149-160); this additive entry point is what its dispatcher would probe, like the
 * image ABI's optional 0.24+ additions (aji_image.h:220-222). No data crosses devices.
 *
 * Frames here are HOST memory: aji_frame.plane[] are host addresses (page-locked for
 * asynchronous copies at link speed; pageable memory works, staged by the driver), stride[] in
 * bytes. submit copies the input into the next device's slot, enqueues aji_infer and the copy of
 * the result into the caller's output planes, and returns the frame's ticket (> 0) or a negative
 * AJIB_ERR_*; it blocks only while that device's ring is full. Both buffers must stay untouched
 * until the ticket finishes: wait(t) blocks until t and every earlier ticket have finished
 * (their outputs are in host memory), done(t) asks without blocking (1 finished, 0 not yet).
 * Driven by one host thread, like aji_ctx. configure sizes every device's chain for w x h input
 * (aji_configure) and waits for frames in flight first. */
typedef struct ajib_video_multi ajib_video_multi;
AJIB_EXPORT ajib_video_multi *ajib_video_create_multi(const aji_create_params *p, const int *devices, int n, int depth,
                                                      char *err, size_t err_size);
AJIB_EXPORT int ajib_video_multi_configure(ajib_video_multi *m, int w, int h, double fps, int *out_w, int *out_h);
AJIB_EXPORT int64_t ajib_video_multi_submit(ajib_video_multi *m, const aji_frame *in, const aji_frame *out);
AJIB_EXPORT int ajib_video_multi_wait(ajib_video_multi *m, int64_t ticket);
AJIB_EXPORT int ajib_video_multi_done(ajib_video_multi *m, int64_t ticket);
AJIB_EXPORT int ajib_video_multi_devices(const ajib_video_multi *m);
AJIB_EXPORT const char *ajib_video_multi_error(const ajib_video_multi *m);
AJIB_EXPORT void ajib_video_multi_destroy(ajib_video_multi **m);
/* Device timing for benchmarks: after timing(m, 1) (which waits for frames in flight), each
 * device records a CUDA event before its first upload and after every download; device_ms waits
 * for everything in flight and gives, per device in the order given at creation, the device time
 * from its first upload's start to its last download's end (0 for a device that ran nothing). */
AJIB_EXPORT int ajib_video_multi_timing(ajib_video_multi *m, int on);
AJIB_EXPORT int ajib_video_multi_device_ms(ajib_video_multi *m, double *ms, int n);
/* The frame order alone (host only, for tests): nframes frames over ndev devices with ring depth
 * depth get device_of / slot_of and the ticket each must wait for before reusing its slot
 * (reuse_of, 0: none); then the tickets finish in finish_order (a permutation of 1..nframes) and
 * completed_after[i] is the count of tickets finished in order after the i-th of them. */
AJIB_EXPORT int ajib_selftest_frame_order(int ndev, int depth, int nframes, const int64_t *finish_order, int *device_of,
                                          int *slot_of, int64_t *reuse_of, int64_t *completed_after);

/* ---- the native model and its executor ----
 * A model is a plan of fused conv steps (reference src/native/lower.h:38-77, Plan), read from
 * this engine's model file (format: animejanai-inference_b200/csrc/model.cpp). An executor is
 * the model instantiated for one input size on the current device (reference
 * src/native/executor.h:21-60): weights uploaded, feature buffers allocated, run() only launches
 * kernels (no allocation, no host synchronisation). */
typedef struct ajib_model ajib_model;
typedef struct ajib_exec ajib_exec;

AJIB_EXPORT int ajib_model_load(const char *path, ajib_model **out, char *err, size_t err_size);
AJIB_EXPORT int ajib_model_from_memory(const void *data, size_t size, ajib_model **out, char *err, size_t err_size);
/* ajib_model_load / ajib_model_from_memory take this engine's model file or an ONNX model, which
 * is lowered to a plan (reference src/native/lower.h:80-100, lower(); src/native/onnx_graph.h,
 * parse_onnx): the SRVGG Compact / SuperUltraCompact and SPAN families; anything the kernels
 * cannot run refuses the model with the reason. ajib_model_save writes the model (lowered or not)
 * as this engine's model file: *size gets its length; buf is filled when cap is large enough. */
AJIB_EXPORT int ajib_model_save(const ajib_model *m, void *buf, size_t cap, size_t *size);
AJIB_EXPORT void ajib_model_release(ajib_model **m);
/* scale (depth-to-space), steps, algorithmic FLOPs per input pixel; description into desc */
AJIB_EXPORT int ajib_model_info(const ajib_model *m, int *scale, int *steps, double *flops_per_px, char *desc,
                                size_t desc_size);

AJIB_EXPORT int ajib_exec_create(const ajib_model *m, int w, int h, ajib_exec **out, char *err, size_t err_size);
AJIB_EXPORT void ajib_exec_release(ajib_exec **e);
/* in: NCHW fp16 [3][h][w]; out: NCHW fp16 [3][R*h][R*w] (device pointers). */
AJIB_EXPORT int ajib_exec_run(ajib_exec *e, const void *in, void *out, void *stream);
/* The same on nimg images of img_h rows stacked along H, each convolved on its own: in
 * [3][nimg * img_h][w], out [3][R * nimg * img_h][R * w], nimg * img_h no more than the executor's
 * height. One launch per step for a whole batch of tiles (the image tiler's); no reference
 * counterpart (the reference runs tiles one at a time, src/aji_img_trt.cpp:980-1011). */
AJIB_EXPORT int ajib_exec_run_images(ajib_exec *e, const void *in, void *out, int w, int img_h, int nimg, void *stream);
/* Run the net as `bands` horizontal bands (1 = whole frame per step): each band runs every step,
 * its rows shifted down one per step, so a band's activations stay in L2 between steps. */
AJIB_EXPORT int ajib_exec_set_bands(ajib_exec *e, int bands);
/* Step timing for benchmarks: while on, each step's launch is bracketed by CUDA events on the run's
 * stream; profile_read synchronises and fills per-step summed milliseconds and run counts. */
AJIB_EXPORT int ajib_exec_profile(ajib_exec *e, int on);
AJIB_EXPORT int ajib_exec_profile_read(ajib_exec *e, double *ms, int *counts, int nsteps);
/* The same for the executor inside a configured video context (aji.h): the chain's last model. */
AJIB_EXPORT int ajib_video_profile(aji_ctx *c, int on);
AJIB_EXPORT int ajib_video_profile_read(aji_ctx *c, double *ms, int *counts, int nsteps);
/* device bytes held, launches per run */
AJIB_EXPORT int ajib_exec_info(const ajib_exec *e, size_t *device_bytes, size_t *weight_bytes, int *launches);

/* Reads and optionally clears the current device's kernel status word: 0, or the code of the
 * first pipeline wait that timed out in a kernel of this library. There is one word per device,
 * shared by every context and executor on it: a code may come from another context's kernels,
 * and a read that clears it clears it for all of them. */
AJIB_EXPORT int ajib_kernel_status(int clear);

/* A one-CTA check of the tensor-core operand encodings the conv kernels use (a: [130][32] fp16,
 * b: [2n][32] fp16, out: [2][128][n] fp32 = A[shift:shift+128] x B-halves^T). For tests. */
AJIB_EXPORT int ajib_selftest_umma(const void *a, const void *b, float *out, int n, int shift, int collector, int *err,
                                   void *stream);
/* Self-test of the colour post pass's division by a constant (a reciprocal and one FMA correction
 * in place of a division per sample): every float of magnitude in [2^-80, 2^18) (the pass's
 * dividends are zero or in [2^-52, 2^18)) divided by 2 (1 - k[i]),
 * i < nk <= 8, against the IEEE division; *mismatches counts differing quotients, *first_bits the
 * first dividend's bits (0xFFFFFFFF: none). No reference counterpart (the reference divides). */
AJIB_EXPORT int ajib_selftest_division(const float *k, int nk, unsigned long long *mismatches, unsigned int *first_bits);
/* The same check for the given divisors d[i], i < nd <= 8 (the pre pass divides by the colour
 * space's luma and chroma scales). */
AJIB_EXPORT int ajib_selftest_division_by(const float *d, int nd, unsigned long long *mismatches,
                                          unsigned int *first_bits);

#ifdef __cplusplus
}
#endif

#endif /* AJI_B200_H */
