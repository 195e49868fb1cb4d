/*
 * video.cpp — the video C ABI (include/aji.h) over the native path: pre-pass, the conv net on
 * the executor, post-pass, all enqueued on the caller's stream. Reference behaviour followed:
 * aji_create direct mode (src/aji_trt.cpp:1088-1190), aji_configure (:1202-1225), aji_infer's
 * checks (:1892-1944), run_pre / run_post / run_chain (:1947-2171), tickets aji_flush / aji_done /
 * aji_wait (:2770-2840). The reference runs its native kernels only in conf mode and TensorRT in
 * direct mode; this engine has no TensorRT, so direct mode's engine_path names a native model
 * file. Features outside the native conv path answer as an inactive feature does.
 */
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>

#include "cuctx.h"
#include "plan.h"
#include "../../include/aji.h"
#include "../../include/aji_b200.h"

using namespace ajib;

struct aji_ctx {
    CUcontext cu = nullptr;
    CUdevice dev = 0;
    bool owns_primary = false;
    aji_log_fn log = nullptr;
    void *log_opaque = nullptr;
    std::string err, current_log, model_path;
    Plan plan;
    std::unique_ptr<Executor> exec;
    int max_w = 0, max_h = 0, in_w = 0, in_h = 0, out_w = 0, out_h = 0, scale = 0, bands = 1;
    bool active = false;
    aji_plan *pre = nullptr, *post = nullptr;
    int pre_key[4] = {0, 0, 0, 0}, post_key[4] = {0, 0, 0, 0};
    void *rgb_in = nullptr, *rgb_out = nullptr;
    // tickets: a ring of events, ticket t tracked by slot t % kRing
    static constexpr int kRing = 64;
    cudaEvent_t ev[kRing] = {};
    uint64_t next = 1, completed = 0;

    void set_error(const char *fmt, ...)
    {
        char b[512];
        va_list ap;
        va_start(ap, fmt);
        std::vsnprintf(b, sizeof(b), fmt, ap);
        va_end(ap);
        err = b;
        if (log) log(log_opaque, 2, b);
    }
    void free_frame_state()
    {
        aji_plan_destroy(pre);
        aji_plan_destroy(post);
        pre = post = nullptr;
        std::memset(pre_key, 0, sizeof(pre_key));
        std::memset(post_key, 0, sizeof(post_key));
        cudaFree(rgb_in);
        cudaFree(rgb_out);
        rgb_in = rgb_out = nullptr;
        exec.reset();
        active = false;
    }
};

namespace {

bool supported_in(int f) { return f == AJI_FMT_NV12 || f == AJI_FMT_P010 || aji_format_is_444(f); }

int run_pre(aji_ctx *c, const aji_frame *in, cudaStream_t s)
{
    const aji_csp csp = aji_make_csp(in->format, in->matrix, in->range);
    int e;
    if (aji_format_is_444(in->format)) {
        e = aji_run_pre444(in->width, in->height, in->plane[0], in->stride[0], in->plane[1], in->stride[1], in->plane[2],
                           in->stride[2], &csp, c->rgb_in, s);
    } else {
        const int key[4] = {in->format, in->width, in->height, in->siting};
        if (!c->pre || std::memcmp(key, c->pre_key, sizeof(key)) != 0) {
            aji_plan_destroy(c->pre);
            c->pre = aji_pre_plan_create(in->format, in->width, in->height, in->siting, AJI_FILTER_SPLINE36);
            if (!c->pre) {
                c->set_error("pre plan creation failed");
                return AJI_ERR_CUDA;
            }
            std::memcpy(c->pre_key, key, sizeof(key));
        }
        e = aji_run_pre(c->pre, in->plane[0], in->stride[0], in->plane[1], in->stride[1], &csp, c->rgb_in, s);
    }
    if (e) {
        c->set_error("pre-kernel failed: %s", cudaGetErrorString((cudaError_t)e));
        return AJI_ERR_CUDA;
    }
    return AJI_OK;
}

// The output keeps the input's matrix and range; 4:2:0 output is subsampled with left siting,
// as the reference pipeline's final resize does (src/aji_trt.cpp:2111-2118).
int run_post(aji_ctx *c, int matrix, int range, const aji_frame *out, cudaStream_t s)
{
    const aji_csp csp = aji_make_csp(out->format, matrix, range);
    int e;
    if (aji_format_is_444(out->format)) {
        e = aji_run_post444(out->format, c->out_w, c->out_h, c->rgb_out, &csp, out->plane[0], out->stride[0],
                            out->plane[1], out->stride[1], out->plane[2], out->stride[2], s);
    } else {
        const int key[4] = {out->format, c->out_w, c->out_h, AJI_SITING_LEFT};
        if (!c->post || std::memcmp(key, c->post_key, sizeof(key)) != 0) {
            aji_plan_destroy(c->post);
            c->post = aji_post_plan_create(out->format, c->out_w, c->out_h, AJI_SITING_LEFT, AJI_FILTER_SPLINE36);
            if (!c->post) {
                c->set_error("post plan creation failed");
                return AJI_ERR_CUDA;
            }
            std::memcpy(c->post_key, key, sizeof(key));
        }
        e = aji_run_post(c->post, c->rgb_out, &csp, out->plane[0], out->stride[0], out->plane[1], out->stride[1], s);
    }
    if (e) {
        c->set_error("post-kernel failed: %s", cudaGetErrorString((cudaError_t)e));
        return AJI_ERR_CUDA;
    }
    return AJI_OK;
}

}  // namespace

extern "C" int aji_stream_policy_version(void) { return 0; }

extern "C" aji_ctx *aji_create(const aji_create_params *params)
{
    if (!params || params->api_version != AJI_API_VERSION) return nullptr;
    try {
        auto c = std::make_unique<aji_ctx>();
        c->log = params->log;
        c->log_opaque = params->log_opaque;
        const Driver &d = driver();
        if (!d.ok || d.init(0) != CUDA_SUCCESS) return nullptr;
        if (params->conf_path && params->conf_path[0]) {
            c->set_error("conf mode is not supported by this engine: pass a native model as engine_path");
            return nullptr;
        }
        if (!params->engine_path || params->max_width < 2 || params->max_height < 2) return nullptr;
        if (params->cuda_context) {
            c->cu = (CUcontext)params->cuda_context;
        } else {
            if (d.device_get(&c->dev, 0) != CUDA_SUCCESS || d.primary_retain(&c->cu, c->dev) != CUDA_SUCCESS) return nullptr;
            c->owns_primary = true;
        }
        CtxGuard g(c->cu);
        if (!g.ok) return nullptr;
        if (!c->owns_primary && d.ctx_get_device(&c->dev) != CUDA_SUCCESS) return nullptr;
        // the kernels are built for sm_100a only: refuse any other device up front
        int rdev = 0, major = 0;
        if (cudaGetDevice(&rdev) != cudaSuccess ||
            cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, rdev) != cudaSuccess || major != 10) {
            if (c->log) c->log(c->log_opaque, 2, "this engine runs on B200-class (sm_100) devices only");
            if (c->owns_primary) d.primary_release(c->dev);
            return nullptr;
        }
        std::string why;
        if (!load_model_file(params->engine_path, &c->plan, &why)) {
            if (c->log) c->log(c->log_opaque, 2, why.c_str());
            if (c->owns_primary) d.primary_release(c->dev);
            return nullptr;
        }
        c->model_path = params->engine_path;
        c->max_w = params->max_width;
        c->max_h = params->max_height;
        c->scale = c->plan.depth_to_space;
        if (const char *b = std::getenv("AJIB_BANDS")) c->bands = std::max(1, std::atoi(b));
        return c.release();
    } catch (...) {
        return nullptr;
    }
}

extern "C" int aji_set_slot(aji_ctx *c, int slot) { return (!c || slot < 0) ? AJI_ERR : AJI_OK; }

extern "C" int aji_configure(aji_ctx *c, int w, int h, double fps, int *out_w, int *out_h)
{
    (void)fps;
    if (!c || w < 2 || h < 2 || (w & 1) || (h & 1)) return AJI_ERR_SHAPE;
    if (w > c->max_w || h > c->max_h) {
        c->set_error("input %dx%d exceeds direct-mode max %dx%d", w, h, c->max_w, c->max_h);
        return AJI_ERR_SHAPE;
    }
    CtxGuard g(c->cu);
    if (!g.ok) {
        c->set_error("cannot make the CUDA context current");
        return AJI_ERR_CUDA;
    }
    try {
        cudaDeviceSynchronize();  // in-flight work may use the state freed here
        c->free_frame_state();
        std::string why;
        c->exec = Executor::create(c->plan, w, h, &why);
        if (!c->exec) {
            c->set_error("native model refused at %dx%d: %s", w, h, why.c_str());
            return AJI_ERR_ENGINE;
        }
        c->exec->set_bands(c->bands);
        c->in_w = w;
        c->in_h = h;
        c->out_w = w * c->scale;
        c->out_h = h * c->scale;
        if (cudaMalloc(&c->rgb_in, (size_t)3 * w * h * 2) != cudaSuccess ||
            cudaMalloc(&c->rgb_out, (size_t)3 * c->out_w * c->out_h * 2) != cudaSuccess) {
            cudaGetLastError();
            c->free_frame_state();
            c->set_error("frame buffer allocation failed");
            return AJI_ERR_CUDA;
        }
        c->active = true;
        char b[512];
        std::snprintf(b, sizeof(b), "Native model: %s\nInput %dx%d -> output %dx%d\n\n1. %s (native, sm_100a)\n",
                      c->model_path.c_str(), w, h, c->out_w, c->out_h, describe(c->plan).c_str());
        c->current_log = b;
        if (out_w) *out_w = c->out_w;
        if (out_h) *out_h = c->out_h;
        return 1;
    } catch (...) {
        c->set_error("configure failed (host allocation)");
        return AJI_ERR;
    }
}

extern "C" int aji_infer(aji_ctx *c, const aji_frame *in, const aji_frame *out, void *cu_stream)
{
    if (!c || !in || !out) return AJI_ERR;
    if (!c->active) {
        c->set_error("aji_infer without an active configuration");
        return AJI_ERR;
    }
    if (!supported_in(in->format)) {
        c->set_error("unsupported input format %d", in->format);
        return AJI_ERR_FORMAT;
    }
    if (!supported_in(out->format)) {
        c->set_error("unsupported output format %d (nv12/p010/planar 444)", out->format);
        return AJI_ERR_FORMAT;
    }
    if (in->width != c->in_w || in->height != c->in_h || out->width != c->out_w || out->height != c->out_h) {
        c->set_error("frame dims %dx%d->%dx%d do not match configured %dx%d->%dx%d", in->width, in->height, out->width,
                     out->height, c->in_w, c->in_h, c->out_w, c->out_h);
        return AJI_ERR_SHAPE;
    }
    CtxGuard g(c->cu);
    if (!g.ok) {
        c->set_error("cannot make the CUDA context current");
        return AJI_ERR_CUDA;
    }
    cudaStream_t s = (cudaStream_t)cu_stream;
    int rc = run_pre(c, in, s);
    if (rc != AJI_OK) return rc;
    const int e = c->exec->run(c->rgb_in, c->rgb_out, s);
    if (e != AJIB_OK) {
        c->set_error("native kernels failed (%d)", e);
        return AJI_ERR_CUDA;
    }
    return run_post(c, in->matrix, in->range, out, s);
}

extern "C" uint64_t aji_flush(aji_ctx *c, void *cu_stream)
{
    if (!c) return 0;
    CtxGuard g(c->cu);
    if (!g.ok) return 0;
    cudaEvent_t &ev = c->ev[c->next % aji_ctx::kRing];
    if (!ev && cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
        c->set_error("ticket event creation failed");
        return 0;
    }
    if (c->next > (uint64_t)aji_ctx::kRing) {
        // the slot's previous ticket must be retired before its event is reused
        if (cudaEventSynchronize(ev) != cudaSuccess) {
            c->set_error("ticket event sync failed");
            return 0;
        }
        c->completed = std::max(c->completed, c->next - aji_ctx::kRing);
    }
    if (cudaEventRecord(ev, (cudaStream_t)cu_stream) != cudaSuccess) {
        c->set_error("ticket event record failed");
        return 0;
    }
    return c->next++;
}

extern "C" int aji_done(aji_ctx *c, uint64_t ticket)
{
    if (!c) return AJI_ERR;
    if (ticket <= c->completed) return 1;
    if (ticket >= c->next) return AJI_ERR;
    CtxGuard g(c->cu);
    if (!g.ok) return AJI_ERR_CUDA;
    const cudaError_t e = cudaEventQuery(c->ev[ticket % aji_ctx::kRing]);
    if (e == cudaSuccess) {
        c->completed = std::max(c->completed, ticket);
        return 1;
    }
    if (e == cudaErrorNotReady) return 0;
    c->set_error("ticket query failed: %s", cudaGetErrorString(e));
    return AJI_ERR_CUDA;
}

extern "C" int aji_wait(aji_ctx *c, uint64_t ticket)
{
    if (!c) return AJI_ERR;
    if (ticket <= c->completed) return AJI_OK;
    if (ticket >= c->next) return AJI_ERR;
    CtxGuard g(c->cu);
    if (!g.ok) return AJI_ERR_CUDA;
    if (cudaEventSynchronize(c->ev[ticket % aji_ctx::kRing]) != cudaSuccess) {
        c->set_error("ticket wait failed");
        return AJI_ERR_CUDA;
    }
    // a kernel that gave up on its own pipeline leaves a code in the status word
    const int st = ajib_kernel_status(1);
    if (st != 0) {
        c->set_error("a native kernel timed out waiting on its pipeline (code %d)", st);
        return AJI_ERR_CUDA;
    }
    c->completed = std::max(c->completed, ticket);
    return AJI_OK;
}

extern "C" int ajib_video_profile(aji_ctx *c, int on)
{
    if (!c || !c->exec) return AJIB_ERR_ARGS;
    return c->exec->profile(on != 0);
}

extern "C" int ajib_video_profile_read(aji_ctx *c, double *ms, int *counts, int nsteps)
{
    if (!c || !c->exec || !ms || !counts) return AJIB_ERR_ARGS;
    CtxGuard g(c->cu);
    if (!g.ok) return AJIB_ERR_CUDA;
    return c->exec->profile_read(ms, counts, nsteps);
}

extern "C" const char *aji_current_log(aji_ctx *c) { return c ? c->current_log.c_str() : ""; }
extern "C" int aji_scale_factor(aji_ctx *c) { return c ? c->scale : 0; }
extern "C" const char *aji_last_error(aji_ctx *c) { return c ? c->err.c_str() : "no context"; }

// ---- features outside the native conv path: inactive ----
extern "C" int aji_rife_factor(aji_ctx *, int *, int *) { return 0; }
extern "C" int aji_rife_before_upscale(aji_ctx *) { return 0; }
extern "C" int aji_pre_resize(aji_ctx *, int *, int *) { return 0; }
extern "C" int aji_poll(aji_ctx *) { return 0; }
extern "C" int aji_temporal_radius(aji_ctx *) { return 0; }
extern "C" void aji_temporal_reset(aji_ctx *) {}

static int inactive(aji_ctx *c, const char *what)
{
    if (c) c->set_error("%s is not supported by this engine (native conv path only)", what);
    return AJI_ERR;
}
extern "C" int aji_resize(aji_ctx *c, const aji_frame *, const aji_frame *, void *) { return inactive(c, "aji_resize"); }
extern "C" int aji_resize_frame(aji_ctx *c, const aji_frame *, const aji_frame *, void *)
{
    return inactive(c, "aji_resize_frame");
}
extern "C" int aji_frame_diff(aji_ctx *c, const aji_frame *, const aji_frame *, aji_frame_diff_result *, void *)
{
    return inactive(c, "aji_frame_diff");
}
extern "C" int aji_infer_rife(aji_ctx *c, const aji_frame *, const aji_frame *, double, const aji_frame *, void *)
{
    return inactive(c, "RIFE");
}
extern "C" int aji_ingest(aji_ctx *c, const aji_frame *, uint64_t, void *) { return inactive(c, "temporal models"); }
extern "C" int aji_infer_seq(aji_ctx *c, uint64_t, const aji_frame *, void *) { return inactive(c, "temporal models"); }
extern "C" int aji_copy_frame(aji_ctx *c, const aji_frame *, const aji_frame *) { return inactive(c, "aji_copy_frame"); }

extern "C" void aji_destroy(aji_ctx **pc)
{
    if (!pc || !*pc) return;
    aji_ctx *c = *pc;
    {
        CtxGuard g(c->cu);
        if (g.ok) {
            cudaDeviceSynchronize();
            c->free_frame_state();
            for (cudaEvent_t &e : c->ev)
                if (e) cudaEventDestroy(e);
        }
    }
    if (c->owns_primary) driver().primary_release(c->dev);
    delete c;
    *pc = nullptr;
}
