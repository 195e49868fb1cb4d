/*
 * aji.h — the video C ABI (version 9) of libaji, as this B200 engine exports it.
 *
 * Players and encoders (mpv's vf_animejanai, aji_encode, aji_harness) dlopen libaji.so and bind
 * these symbols. The types, enum values, struct layouts and function signatures are those of the
 * reference header (the-database/animejanai-inference include/aji.h:45-501), so a caller built
 * against that header loads this library unchanged. Only the native conv path (SRVGG Compact,
 * SuperUltraCompact, SPAN, SPANF3) is implemented, with Spline36 resizing (aji_resize_frame and
 * conf chains' resize-before-upscale steps); RIFE, temporal models and aji_resize answer as an
 * inactive feature does (0, or AJI_ERR with aji_last_error set).
 *
 * Frames: aji_frame.plane[] are CUDA device pointers (CUdeviceptr), stride[] in bytes.
 * aji_infer enqueues on the caller's CUDA stream and returns before the GPU finishes; aji_flush
 * returns a ticket that completes once everything enqueued before it has.
 *
 * Modes:
 *  - direct mode (conf_path NULL): engine_path names a model file (this engine's native format
 *    or an ONNX SRVGG / SPAN export, see aji_b200.h, ajib_model_load); aji_configure(w, h) sizes
 *    it for w x h.
 *  - conf mode (conf_path set): an animejanai.conf; aji_configure picks the slot's chain for the
 *    stream's size and fps and builds it from the models in model_dir (the conf's directory when
 *    NULL): resize steps and models one after another, or passthrough when no chain matches.
 */
#ifndef AJI_H
#define AJI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define AJI_EXPORT __declspec(dllexport)
#else
#define AJI_EXPORT __attribute__((visibility("default")))
#endif

#define AJI_API_VERSION 9

typedef struct aji_ctx aji_ctx;

/* reference include/aji.h:49-62 */
enum aji_format {
    AJI_FMT_NV12 = 1,          /* 8-bit 4:2:0, CbCr interleaved in one half-height plane */
    AJI_FMT_P010 = 2,          /* 10 bits in the high bits of 16, 4:2:0, CbCr interleaved */
    AJI_FMT_YUV444P16 = 3,     /* 16-bit planar 4:4:4 */
    AJI_FMT_RGB10A2 = 4,       /* packed RGB (DirectML input only; refused here) */
    AJI_FMT_YUV444P10MSB = 5,  /* 10 bits in the high bits of 16, planar 4:4:4 */
    AJI_FMT_YUV444P12MSB = 6,  /* 12 bits in the high bits of 16, planar 4:4:4 */
};

static inline int aji_format_is_444(int format)
{
    return format == AJI_FMT_YUV444P16 || format == AJI_FMT_YUV444P10MSB || format == AJI_FMT_YUV444P12MSB;
}

/* reference include/aji.h:71-86 */
enum aji_matrix { AJI_MATRIX_BT601 = 1, AJI_MATRIX_BT709 = 2, AJI_MATRIX_BT2020 = 3 };
enum aji_range { AJI_RANGE_LIMITED = 1, AJI_RANGE_FULL = 2 };
enum aji_siting { AJI_SITING_LEFT = 1, AJI_SITING_CENTER = 2, AJI_SITING_TOPLEFT = 3 };

/* reference include/aji.h:88-97 */
enum aji_status {
    AJI_OK = 0,
    AJI_SCENE = 1,
    AJI_ERR = -1,
    AJI_ERR_SHAPE = -2,
    AJI_ERR_FORMAT = -3,
    AJI_ERR_CUDA = -4,
    AJI_ERR_ENGINE = -5,
    AJI_ERR_CONF = -6,
};

typedef void (*aji_log_fn)(void *opaque, int level, const char *msg);

/* reference include/aji.h:101-132 (same field order and types) */
typedef struct aji_create_params {
    uint32_t api_version;  /* AJI_API_VERSION */
    void *cuda_context;    /* CUcontext to run in; NULL = the primary context of device 0 */
    const char *conf_path; /* an animejanai.conf (conf mode); NULL = direct mode */
    const char *model_dir;
    const char *trtexec;
    const char *trtexec_env;
    int slot;
    const char *rife_model_dir;
    int async_build;
    void *d3d11_device;
    const char *engine_path; /* direct mode: the native model file */
    int max_width, max_height;
    aji_log_fn log;
    void *log_opaque;
} aji_create_params;

/* reference include/aji.h:134-145 */
typedef struct aji_frame {
    int width, height; /* luma size */
    int format;        /* enum aji_format */
    int matrix;        /* enum aji_matrix */
    int range;         /* enum aji_range */
    int siting;        /* enum aji_siting */
    void *plane[3];    /* device pointers: Y, CbCr (4:2:0) or Y, Cb, Cr (4:4:4) */
    ptrdiff_t stride[3];
} aji_frame;

/* reference include/aji.h:274-283 */
typedef struct aji_frame_diff_result {
    float max_tile;
    float region_mean[16];
} aji_frame_diff_result;

AJI_EXPORT int aji_stream_policy_version(void);
AJI_EXPORT aji_ctx *aji_create(const aji_create_params *params);
AJI_EXPORT int aji_set_slot(aji_ctx *c, int slot);
/* Size the model for w x h input: returns 1 and the output size (scale * input). */
AJI_EXPORT int aji_configure(aji_ctx *c, int w, int h, double fps, int *out_w, int *out_h);
/* Upscale one frame: pre-pass (YUV -> RGB), the conv net, post-pass (RGB -> YUV), enqueued on
 * cu_stream. Output format NV12 / P010 / 4:4:4, independent of the input's. */
AJI_EXPORT int aji_infer(aji_ctx *c, const aji_frame *in, const aji_frame *out, void *cu_stream);
AJI_EXPORT uint64_t aji_flush(aji_ctx *c, void *cu_stream);
AJI_EXPORT int aji_done(aji_ctx *c, uint64_t ticket);
AJI_EXPORT int aji_wait(aji_ctx *c, uint64_t ticket);
AJI_EXPORT const char *aji_current_log(aji_ctx *c);
AJI_EXPORT int aji_scale_factor(aji_ctx *c);
AJI_EXPORT int aji_rife_factor(aji_ctx *c, int *num, int *den);
AJI_EXPORT int aji_rife_before_upscale(aji_ctx *c);
AJI_EXPORT int aji_pre_resize(aji_ctx *c, int *work_w, int *work_h);
AJI_EXPORT int aji_resize(aji_ctx *c, const aji_frame *in, const aji_frame *out, void *cu_stream);
AJI_EXPORT int aji_resize_frame(aji_ctx *c, const aji_frame *in, const aji_frame *out, void *cu_stream);
AJI_EXPORT int aji_frame_diff(aji_ctx *c, const aji_frame *a, const aji_frame *b, aji_frame_diff_result *out,
                              void *cu_stream);
AJI_EXPORT int aji_poll(aji_ctx *c);
AJI_EXPORT int aji_infer_rife(aji_ctx *c, const aji_frame *a, const aji_frame *b, double t, const aji_frame *out,
                              void *cu_stream);
AJI_EXPORT int aji_temporal_radius(aji_ctx *c);
AJI_EXPORT int aji_ingest(aji_ctx *c, const aji_frame *in, uint64_t seq, void *cu_stream);
AJI_EXPORT int aji_infer_seq(aji_ctx *c, uint64_t seq, const aji_frame *out, void *cu_stream);
AJI_EXPORT void aji_temporal_reset(aji_ctx *c);
AJI_EXPORT const char *aji_last_error(aji_ctx *c);
AJI_EXPORT void aji_destroy(aji_ctx **c);
AJI_EXPORT int aji_copy_frame(aji_ctx *c, const aji_frame *in, const aji_frame *out);

#ifdef __cplusplus
}
#endif

#endif /* AJI_H */
