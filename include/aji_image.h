/*
 * aji_image.h — the still-image C ABI (version 1) of libaji, as this B200 engine exports it.
 *
 * Image tools (MangaJaNai, the aji_image CLI) bind these symbols. Types, enum values, struct
 * layouts and signatures are those of the reference header (the-database/animejanai-inference
 * include/aji_image.h:50-276). 8-bit gray or RGB images travel in host memory; tiling, overlap
 * blending and dtype conversion run on the GPU. Models are native model files (aji_b200.h,
 * ajib_model_load) passed as onnx_path.
 *
 * Multi-GPU (additive): aji_img_create_multi spreads each image's tiles over several devices of
 * one box, with results bit-identical to one device (aji_b200.h).
 */
#ifndef AJI_IMAGE_H
#define AJI_IMAGE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define AJI_IMG_EXPORT __declspec(dllexport)
#else
#define AJI_IMG_EXPORT __attribute__((visibility("default")))
#endif

#define AJI_IMAGE_API_VERSION 1

typedef struct aji_img_ctx aji_img_ctx;
typedef struct aji_img_model aji_img_model;

/* reference include/aji_image.h:50-67; this engine serves the CUDA value */
enum aji_img_backend { AJI_IMG_TENSORRT = 1, AJI_IMG_DIRECTML = 2, AJI_IMG_TENSORRT_RTX = 3, AJI_IMG_VULKAN = 4 };

/* reference include/aji_image.h:67-74 */
enum aji_img_status {
    AJI_IMG_OK = 0,
    AJI_IMG_ERR = -1,
    AJI_IMG_ERR_ARGS = -2,
    AJI_IMG_NOT_READY = -3,
    AJI_IMG_CANCELLED = -4,
    AJI_IMG_ERR_NO_MEM = -5,
};

enum aji_img_model_state { AJI_IMG_STATE_READY = 0, AJI_IMG_STATE_BUILDING = 1, AJI_IMG_STATE_FAILED = -1 };

typedef void (*aji_img_log_fn)(void *opaque, int level, const char *msg);
/* nonzero cancels; called between tiles */
typedef int (*aji_img_progress_fn)(void *opaque, int tiles_done, int tiles_total);

/* reference include/aji_image.h:88-97 */
typedef struct aji_img_device {
    uint64_t id; /* PCI domain/bus/device */
    char name[128];
    uint64_t vram_bytes;
    int sm_major, sm_minor;
} aji_img_device;

AJI_IMG_EXPORT int aji_img_enum_devices(int backend, aji_img_device *out, int max);

/* reference include/aji_image.h:107-121 */
typedef struct aji_img_create_params {
    uint32_t api_version;
    int backend;
    uint64_t device_id; /* aji_img_device.id; 0 = first device */
    const char *cache_dir;
    const char *trtexec;
    const char *trtexec_env;
    aji_img_log_fn log;
    void *log_opaque;
} aji_img_create_params;

AJI_IMG_EXPORT aji_img_ctx *aji_img_create(const aji_img_create_params *p, char *err, size_t err_size);

enum aji_img_load_flags { AJI_IMG_LOAD_ASYNC_BUILD = 1, AJI_IMG_LOAD_EVEN_TILES = 2 };

/* reference include/aji_image.h:148-161 */
typedef struct aji_img_model_params {
    const char *onnx_path; /* a native model file */
    int tile_w, tile_h;    /* input-pixel tile; 0 = 512 */
    int overlap;           /* input-pixel overlap between tiles; 0 = 128 */
    int flags;
} aji_img_model_params;

AJI_IMG_EXPORT aji_img_model *aji_img_load(aji_img_ctx *c, const aji_img_model_params *p);
AJI_IMG_EXPORT int aji_img_model_state(aji_img_model *m);

/* reference include/aji_image.h:173-180 */
typedef struct aji_img_model_info {
    int scale;
    int in_channels;
    int out_channels;
    int tile_w, tile_h;
    int overlap;
} aji_img_model_info;

AJI_IMG_EXPORT int aji_img_model_info_get(aji_img_model *m, aji_img_model_info *info);

/* reference include/aji_image.h:186-191 */
typedef struct aji_img_buffer {
    int width, height;
    int channels; /* 1 = gray, 3 = RGB */
    ptrdiff_t stride;
    uint8_t *data;
} aji_img_buffer;

AJI_IMG_EXPORT int aji_img_upscale(aji_img_model *m, const aji_img_buffer *in, const aji_img_buffer *out,
                                   aji_img_progress_fn progress, void *opaque);
AJI_IMG_EXPORT void aji_img_release(aji_img_model **m);
AJI_IMG_EXPORT const char *aji_img_last_error(aji_img_ctx *c);
AJI_IMG_EXPORT void aji_img_destroy(aji_img_ctx **c);
AJI_IMG_EXPORT int aji_img_release_device(int backend, uint64_t device_id);

/* reference include/aji_image.h:225-262 */
typedef struct aji_img_memory {
    uint64_t device_free;
    uint64_t device_total;
    uint64_t ctx_activations;
    uint64_t ctx_scratch;
    uint64_t model_weights;
    uint64_t model_activations;
    uint64_t model_buffers;
    int activations_shared;
} aji_img_memory;

AJI_IMG_EXPORT int aji_img_memory_get(aji_img_ctx *c, aji_img_model *m, aji_img_memory *out);
AJI_IMG_EXPORT int aji_img_native_probe(aji_img_ctx *c, const aji_img_model_params *p, aji_img_memory *out);

#ifdef __cplusplus
}
#endif

#endif /* AJI_IMAGE_H */
