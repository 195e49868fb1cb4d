/*
 * video.cpp — the video C ABI (include/aji.h) over the native path: pre-pass, the conv net on
 * the executor, post-pass, all enqueued on the caller's stream. Reference behaviour followed:
 * aji_create direct mode (src/aji_trt.cpp:1088-1190), aji_configure (:1202-1225), aji_infer's
 * checks (:1892-1944), run_pre / run_post / run_chain (:1947-2171), tickets aji_flush / aji_done /
 * aji_wait (:2770-2840). The reference runs its native kernels only in conf mode and TensorRT in
 * direct mode; this engine has no TensorRT, so direct mode's engine_path names a native model
 * file, and conf mode (animejanai.conf, conf.h) picks a chain of native model files per
 * resolution and fps (:1202-1660): Spline36 resize steps before models that ask for one, the
 * models one after another, each at the size the previous step produced. Features outside the
 * native conv path (RIFE, temporal models) answer as an inactive feature does.
 */
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>

#include <vector>

#include "conf.h"
#include "cuctx.h"
#include "plan.h"
#include "../../include/aji.h"
#include "../../include/aji_b200.h"

using namespace ajib;

// One step of the active chain: a Spline36 resize, or a model run on the executor.
struct ChainStep {
    bool resize = false;
    int in_w = 0, in_h = 0, out_w = 0, out_h = 0;
    aji_plan *rs = nullptr;           // resize
    std::unique_ptr<Executor> exec;   // model
    std::string name;
};

struct aji_ctx {
    CUcontext cu = nullptr;
    CUdevice dev = 0;
    bool owns_primary = false;
    aji_log_fn log = nullptr;
    void *log_opaque = nullptr;
    std::string err, current_log, model_path;
    // direct mode: one model; conf mode: the configuration, its model directory and slot
    bool conf_mode = false;
    Plan plan;
    Conf conf;
    std::string model_dir;
    int slot = 0;
    int max_w = 0, max_h = 0, in_w = 0, in_h = 0, out_w = 0, out_h = 0, scale = 0, bands = 1;
    bool active = false;
    std::vector<ChainStep> steps;
    Executor *exec = nullptr;  // the first model step's executor (step profiling)
    aji_plan *pre = nullptr, *post = nullptr;
    int pre_key[4] = {0, 0, 0, 0}, post_key[4] = {0, 0, 0, 0};
    void *buf[2] = {nullptr, nullptr};  // RGB fp16 ping-pong buffers, each the largest step size
    void *rgb_out = nullptr;            // the chain's result (one of buf)
    // aji_resize_frame's plans and buffers, per size, apart from the chain's
    aji_plan *rf_pre = nullptr, *rf_rs = nullptr, *rf_post = nullptr;
    int rf_key[4] = {0, 0, 0, 0}, rf_pre_key[4] = {0, 0, 0, 0}, rf_post_key[4] = {0, 0, 0, 0};
    void *rf_buf[2] = {nullptr, nullptr};
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
        for (ChainStep &st : steps) aji_plan_destroy(st.rs);
        steps.clear();
        exec = nullptr;
        cudaFree(buf[0]);
        cudaFree(buf[1]);
        buf[0] = buf[1] = nullptr;
        rgb_out = nullptr;
        active = false;
    }
    // the resize plan and buffers of aji_resize_frame's last size pair
    void free_resize_frame_size()
    {
        aji_plan_destroy(rf_rs);
        rf_rs = nullptr;
        std::memset(rf_key, 0, sizeof(rf_key));
        cudaFree(rf_buf[0]);
        cudaFree(rf_buf[1]);
        rf_buf[0] = rf_buf[1] = nullptr;
    }
    void free_resize_frame_state()
    {
        free_resize_frame_size();
        aji_plan_destroy(rf_pre);
        aji_plan_destroy(rf_post);
        rf_pre = rf_post = nullptr;
        std::memset(rf_pre_key, 0, sizeof(rf_pre_key));
        std::memset(rf_post_key, 0, sizeof(rf_post_key));
    }
};

namespace {

bool supported_in(int f) { return f == AJI_FMT_NV12 || f == AJI_FMT_P010 || aji_format_is_444(f); }

// in (NV12 / P010 / 4:4:4) -> fp16 NCHW RGB dst at the frame's size; *plan / key cache the
// 4:2:0 filter plan per format, size and siting. With pk (4:2:0 only), the pass also writes the
// first model's head input map (the executor's own input pack, fused into this pass).
int run_pre(aji_ctx *c, const aji_frame *in, void *dst, aji_plan **plan, int *key, cudaStream_t s,
            const InputPack *pk = nullptr)
{
    const aji_csp csp = aji_make_csp(in->format, in->matrix, in->range);
    int e;
    if (aji_format_is_444(in->format)) {
        e = aji_run_pre444(in->width, in->height, in->plane[0], in->stride[0], in->plane[1], in->stride[1], in->plane[2],
                           in->stride[2], &csp, dst, s);
    } else {
        const int k[4] = {in->format, in->width, in->height, in->siting};
        if (!*plan || std::memcmp(k, key, sizeof(k)) != 0) {
            aji_plan_destroy(*plan);
            *plan = aji_pre_plan_create(in->format, in->width, in->height, in->siting, AJI_FILTER_SPLINE36);
            if (!*plan) {
                c->set_error("pre plan creation failed");
                return AJI_ERR_CUDA;
            }
            std::memcpy(key, k, sizeof(k));
        }
        e = pk ? run_pre_packed(*plan, in->plane[0], in->stride[0], in->plane[1], in->stride[1], &csp, dst, *pk, s)
               : aji_run_pre(*plan, in->plane[0], in->stride[0], in->plane[1], in->stride[1], &csp, dst, s);
    }
    if (e) {
        c->set_error("pre-kernel failed: %s", cudaGetErrorString((cudaError_t)e));
        return AJI_ERR_CUDA;
    }
    return AJI_OK;
}

// fp16 NCHW RGB src at the output frame's size -> out. The output keeps the input's matrix and
// range; 4:2:0 output is subsampled with left siting, as the reference pipeline's final resize
// does (src/aji_trt.cpp:2111-2118).
int run_post(aji_ctx *c, const void *src, int matrix, int range, const aji_frame *out, aji_plan **plan, int *key,
             cudaStream_t s)
{
    const aji_csp csp = aji_make_csp(out->format, matrix, range);
    int e;
    if (aji_format_is_444(out->format)) {
        e = aji_run_post444(out->format, out->width, out->height, src, &csp, out->plane[0], out->stride[0],
                            out->plane[1], out->stride[1], out->plane[2], out->stride[2], s);
    } else {
        const int k[4] = {out->format, out->width, out->height, AJI_SITING_LEFT};
        if (!*plan || std::memcmp(k, key, sizeof(k)) != 0) {
            aji_plan_destroy(*plan);
            *plan = aji_post_plan_create(out->format, out->width, out->height, AJI_SITING_LEFT, AJI_FILTER_SPLINE36);
            if (!*plan) {
                c->set_error("post plan creation failed");
                return AJI_ERR_CUDA;
            }
            std::memcpy(key, k, sizeof(k));
        }
        e = aji_run_post(*plan, src, &csp, out->plane[0], out->stride[0], out->plane[1], out->stride[1], s);
    }
    if (e) {
        c->set_error("post-kernel failed: %s", cudaGetErrorString((cudaError_t)e));
        return AJI_ERR_CUDA;
    }
    return AJI_OK;
}

bool load_plan(aji_ctx *c, const std::string &path, Plan *plan)
{
    std::string why;
    if (!load_model_file(path, plan, &why)) {
        c->set_error("%s", why.c_str());
        return false;
    }
    return true;
}

// A resize step to (nw, nh) after the current size (*cw, *ch).
bool push_resize(aji_ctx *c, int *cw, int *ch, int nw, int nh)
{
    ChainStep st;
    st.resize = true;
    st.in_w = *cw;
    st.in_h = *ch;
    st.out_w = nw;
    st.out_h = nh;
    st.rs = aji_resize_plan_create(*cw, *ch, nw, nh);
    if (!st.rs) {
        c->set_error("resize plan %dx%d -> %dx%d failed", *cw, *ch, nw, nh);
        return false;
    }
    c->steps.push_back(std::move(st));
    *cw = nw;
    *ch = nh;
    return true;
}

// A model step at the current size.
bool push_model(aji_ctx *c, const Plan &plan, const std::string &name, int *cw, int *ch)
{
    std::string why;
    ChainStep st;
    st.name = name;
    st.in_w = *cw;
    st.in_h = *ch;
    st.exec = Executor::create(plan, *cw, *ch, &why);
    if (!st.exec) {
        c->set_error("native model %s refused at %dx%d: %s", name.c_str(), *cw, *ch, why.c_str());
        return false;
    }
    st.exec->set_bands(c->bands);
    st.out_w = st.exec->out_w();
    st.out_h = st.exec->out_h();
    *cw = st.out_w;
    *ch = st.out_h;
    c->steps.push_back(std::move(st));
    return true;
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
        c->conf_mode = params->conf_path && params->conf_path[0];
        if (!c->conf_mode && (!params->engine_path || params->max_width < 2 || params->max_height < 2)) return nullptr;
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
        if (c->conf_mode) {
            if (!load_conf(params->conf_path, &c->conf, &why)) {
                if (c->log) c->log(c->log_opaque, 2, why.c_str());
                if (c->owns_primary) d.primary_release(c->dev);
                return nullptr;
            }
            if (params->model_dir && params->model_dir[0]) {
                c->model_dir = params->model_dir;
            } else {
                // default: the configuration file's directory
                const std::string cp = params->conf_path;
                const size_t sl = cp.find_last_of('/');
                c->model_dir = sl == std::string::npos ? "." : cp.substr(0, sl);
            }
            c->slot = params->slot;
        } else {
            if (!load_model_file(params->engine_path, &c->plan, &why)) {
                if (c->log) c->log(c->log_opaque, 2, why.c_str());
                if (c->owns_primary) d.primary_release(c->dev);
                return nullptr;
            }
            c->model_path = params->engine_path;
            c->max_w = params->max_width;
            c->max_h = params->max_height;
            c->scale = model_scale(c->plan);
        }
        if (const char *b = std::getenv("AJIB_BANDS")) c->bands = std::max(1, std::atoi(b));
        return c.release();
    } catch (...) {
        return nullptr;
    }
}

extern "C" int aji_set_slot(aji_ctx *c, int slot)
{
    if (!c || slot < 0) return AJI_ERR;
    c->slot = slot;
    return AJI_OK;
}

extern "C" int aji_configure(aji_ctx *c, int w, int h, double fps, int *out_w, int *out_h)
{
    if (!c || w < 2 || h < 2 || (w & 1) || (h & 1)) return AJI_ERR_SHAPE;
    if (!c->conf_mode && (w > c->max_w || h > c->max_h)) {
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
        int cw = w, ch = h;
        std::string log;
        char b[512];
        if (!c->conf_mode) {
            if (!push_model(c, c->plan, c->model_path, &cw, &ch)) return AJI_ERR_ENGINE;
            std::snprintf(b, sizeof(b), "Native model: %s\nInput %dx%d -> output %dx%d\n\n1. %s (native, sm_100a)\n",
                          c->model_path.c_str(), w, h, cw, ch, describe(c->plan).c_str());
            log = b;
        } else {
            // the first chain of the slot matching the stream (src/aji_conf.cpp:355-382)
            std::vector<std::string> skipped;
            const ChainConf *chain = select_chain(c->conf, c->slot, c->model_dir, w, h, fps, &skipped);
            for (const std::string &sk : skipped) log += sk + "\n";
            if (!chain || chain->models.empty()) {
                log += "No chain for " + std::to_string(w) + "x" + std::to_string(h) + ": passthrough\n";
                c->current_log = log;
                if (out_w) *out_w = w;
                if (out_h) *out_h = h;
                c->in_w = c->out_w = w;
                c->in_h = c->out_h = h;
                c->scale = 1;
                return 0;
            }
            if (chain->temporal) {
                c->set_error("chain %d uses a temporal model, which this engine does not serve", chain->index);
                return AJI_ERR_CONF;
            }
            std::snprintf(b, sizeof(b), "Profile: %s, chain %d\n",
                          c->conf.slots.at(c->slot).profile_name.c_str(), chain->index);
            log += b;
            if (chain->rife) log += "RIFE is not served by this engine: inactive\n";
            // the model loop of the reference's configure (src/aji_trt.cpp:1407-1455)
            for (const ModelConf &m : chain->models) {
                const double factor = m.resize_height != 0 ? 100.0 : m.resize_factor;
                if (factor != 100.0) {
                    const int nw = round_even(cw * factor / 100.0), nh = round_even(ch * factor / 100.0);
                    if (nw >= 2 && nh >= 2 && (nw != cw || nh != ch)) {
                        if (!push_resize(c, &cw, &ch, nw, nh)) return AJI_ERR_CUDA;
                        std::snprintf(b, sizeof(b), "Applied Resize Factor Before Upscale: %g%%;    New Video Resolution: %dx%d\n",
                                      factor, cw, ch);
                        log += b;
                    }
                }
                if (m.resize_height != 0 && (int)m.resize_height != ch) {
                    int nw, nh;
                    fit_box(cw, ch, m.resize_height * 16.0 / 9.0, m.resize_height, &nw, &nh);
                    if (!push_resize(c, &cw, &ch, nw, nh)) return AJI_ERR_CUDA;
                    std::snprintf(b, sizeof(b), "Applied Resize Height Before Upscale: %gpx;    New Video Resolution: %dx%d\n",
                                  m.resize_height, cw, ch);
                    log += b;
                }
                if (m.name.empty()) continue;
                Plan plan;
                if (!load_plan(c, model_file(c->model_dir, m.name), &plan)) return AJI_ERR_ENGINE;
                if (!push_model(c, plan, m.name, &cw, &ch)) return AJI_ERR_ENGINE;
                std::snprintf(b, sizeof(b), "Applied Model: %s (native, %s);    New Video Resolution: %dx%d\n",
                              m.name.c_str(), describe(plan).c_str(), cw, ch);
                log += b;
            }
        }
        // two RGB buffers, each as large as the largest image the chain holds
        size_t most = (size_t)3 * w * h * 2;
        for (const ChainStep &st : c->steps) most = std::max(most, (size_t)3 * st.out_w * st.out_h * 2);
        if (cudaMalloc(&c->buf[0], most) != cudaSuccess || cudaMalloc(&c->buf[1], most) != cudaSuccess) {
            cudaGetLastError();
            c->free_frame_state();
            c->set_error("frame buffer allocation failed");
            return AJI_ERR_CUDA;
        }
        for (ChainStep &st : c->steps)
            if (!st.resize && !c->exec) c->exec = st.exec.get();
        c->in_w = w;
        c->in_h = h;
        c->out_w = cw;
        c->out_h = ch;
        c->scale = cw / w;
        c->rgb_out = c->buf[c->steps.size() % 2];
        c->active = true;
        c->current_log = log;
        if (out_w) *out_w = cw;
        if (out_h) *out_h = ch;
        return 1;
    } catch (...) {
        c->free_frame_state();
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
    // a chain that starts with a model whose head reads the plain NCHW input: the 4:2:0 pre pass
    // writes that head's input map as well, so the executor skips its own pack launch
    InputPack pk;
    const bool fused = !c->steps.empty() && !c->steps[0].resize && !aji_format_is_444(in->format) &&
                       c->steps[0].exec->input_pack(&pk);
    int rc = run_pre(c, in, c->buf[0], &c->pre, c->pre_key, s, fused ? &pk : nullptr);
    if (rc != AJI_OK) return rc;
    // the chain's steps, ping-ponging between the two buffers
    for (size_t i = 0; i < c->steps.size(); i++) {
        const ChainStep &st = c->steps[i];
        void *src = c->buf[i % 2], *dst = c->buf[(i + 1) % 2];
        const int e = st.resize             ? aji_run_resize(st.rs, src, dst, s)
                      : (i == 0 && fused) ? st.exec->run_packed(src, dst, s)
                                          : st.exec->run(src, dst, s);
        if (e != 0) {
            c->set_error("%s failed (%d)", st.resize ? "resize kernel" : "native kernels", e);
            return AJI_ERR_CUDA;
        }
    }
    return run_post(c, c->rgb_out, in->matrix, in->range, out, &c->post, c->post_key, s);
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

// The model step profiled: the chain's last model (in a chain, the largest and costliest).
namespace {
Executor *profiled_exec(aji_ctx *c)
{
    for (auto it = c->steps.rbegin(); it != c->steps.rend(); ++it)
        if (it->exec) return it->exec.get();
    return c->exec;
}
}  // namespace

extern "C" int ajib_video_profile(aji_ctx *c, int on)
{
    if (!c) return AJIB_ERR_ARGS;
    Executor *e = profiled_exec(c);
    return e ? e->profile(on != 0) : AJIB_ERR_ARGS;
}

extern "C" int ajib_video_profile_read(aji_ctx *c, double *ms, int *counts, int nsteps)
{
    if (!c || !ms || !counts) return AJIB_ERR_ARGS;
    Executor *e = profiled_exec(c);
    if (!e) return AJIB_ERR_ARGS;
    CtxGuard g(c->cu);
    if (!g.ok) return AJIB_ERR_CUDA;
    return e->profile_read(ms, counts, nsteps);
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
// in -> fp16 RGB -> Spline36 -> out (src/aji_trt.cpp, aji_resize_frame): any sizes, same format
// family; plans and buffers per size, apart from the chain's.
extern "C" int aji_resize_frame(aji_ctx *c, const aji_frame *in, const aji_frame *out, void *cu_stream)
{
    if (!c || !in || !out) return AJI_ERR;
    if (!supported_in(in->format) || !supported_in(out->format)) {
        c->set_error("aji_resize_frame: unsupported format");
        return AJI_ERR_FORMAT;
    }
    if (in->width < 2 || in->height < 2 || out->width < 2 || out->height < 2) return AJI_ERR_SHAPE;
    CtxGuard g(c->cu);
    if (!g.ok) {
        c->set_error("cannot make the CUDA context current");
        return AJI_ERR_CUDA;
    }
    cudaStream_t s = (cudaStream_t)cu_stream;
    const int key[4] = {in->width, in->height, out->width, out->height};
    if (!c->rf_rs || std::memcmp(key, c->rf_key, sizeof(key)) != 0) {
        cudaStreamSynchronize(s);  // earlier calls may still use the buffers freed here
        c->free_resize_frame_size();
        c->rf_rs = aji_resize_plan_create(in->width, in->height, out->width, out->height);
        if (!c->rf_rs || cudaMalloc(&c->rf_buf[0], (size_t)3 * in->width * in->height * 2) != cudaSuccess ||
            cudaMalloc(&c->rf_buf[1], (size_t)3 * out->width * out->height * 2) != cudaSuccess) {
            cudaGetLastError();
            c->free_resize_frame_size();
            c->set_error("aji_resize_frame: plan or buffer allocation failed");
            return AJI_ERR_CUDA;
        }
        std::memcpy(c->rf_key, key, sizeof(key));
    }
    int rc = run_pre(c, in, c->rf_buf[0], &c->rf_pre, c->rf_pre_key, s);
    if (rc != AJI_OK) return rc;
    const int e = aji_run_resize(c->rf_rs, c->rf_buf[0], c->rf_buf[1], s);
    if (e) {
        c->set_error("resize kernel failed: %s", cudaGetErrorString((cudaError_t)e));
        return AJI_ERR_CUDA;
    }
    return run_post(c, c->rf_buf[1], in->matrix, in->range, out, &c->rf_post, c->rf_post_key, s);
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
            c->free_resize_frame_state();
            for (cudaEvent_t &e : c->ev)
                if (e) cudaEventDestroy(e);
        }
    }
    if (c->owns_primary) driver().primary_release(c->dev);
    delete c;
    *pc = nullptr;
}
