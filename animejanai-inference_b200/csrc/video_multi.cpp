/*
 * video_multi.cpp — one video stream upscaled frame-parallel on several GPUs of one host
 * (ajib_video_create_multi and the calls after it, include/aji_b200.h).
 *
 * The reference serves a stream from one device (aji_create, src/aji_trt.cpp:1088-1190); its
 * frames are independent, so here frame k runs on device k mod n (frame_order.h), each device
 * with its own video context (the same model chain, video.cpp), three non-blocking streams
 * (upload, compute, download) and a ring of `depth` device frame slots. A submitted frame is
 * copied from the caller's host planes into its slot, upscaled by aji_infer and copied back into
 * the caller's host output planes, each step ordered after the previous one by events, so the
 * copies of neighbouring frames overlap the compute of this one on every device. No data crosses
 * devices and nothing is collective. Results complete in submission order: ticket t counts as
 * finished only when every earlier ticket has, as a one-device player sees them.
 *
 * Host buffers should be page-locked (cudaHostAlloc / cudaHostRegister) for the copies to run
 * asynchronously at link speed; pageable buffers work, with the driver staging them on the
 * submitting thread.
 */
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <deque>
#include <memory>
#include <string>
#include <vector>

#include "cuctx.h"
#include "frame_order.h"
#include "../../include/aji.h"
#include "../../include/aji_b200.h"

using namespace ajib;

namespace {

struct Slot {
    void *in[3] = {nullptr, nullptr, nullptr};
    void *out[3] = {nullptr, nullptr, nullptr};
    size_t in_cap = 0, out_cap = 0;  // bytes of each buffer (one allocation per frame, planes inside)
    cudaEvent_t up = nullptr, done = nullptr, down = nullptr;
};

struct Dev {
    int ordinal = 0;
    CUdevice cudev = 0;
    CUcontext cu = nullptr;
    bool retained = false;
    aji_ctx *ctx = nullptr;
    cudaStream_t s_up = nullptr, s_comp = nullptr, s_down = nullptr;
    std::vector<Slot> ring;
    cudaEvent_t t0 = nullptr, t1 = nullptr;  // timing: first upload start, last download end
    bool t0_set = false, t1_set = false;
};

// The planes of a frame of the given format at w x h: count, rows and row bytes of each.
int frame_planes(int format, int w, int h, int rows[3], size_t row_bytes[3])
{
    if (format == AJI_FMT_NV12 || format == AJI_FMT_P010) {
        const size_t es = format == AJI_FMT_P010 ? 2 : 1;
        rows[0] = h;
        rows[1] = h / 2;
        row_bytes[0] = row_bytes[1] = (size_t)w * es;
        return 2;
    }
    if (aji_format_is_444(format)) {
        for (int p = 0; p < 3; p++) {
            rows[p] = h;
            row_bytes[p] = (size_t)w * 2;
        }
        return 3;
    }
    return 0;
}

}  // namespace

struct ajib_video_multi {
    std::vector<Dev> devs;
    std::unique_ptr<FrameOrder> order;
    int depth = 2;
    int in_w = 0, in_h = 0, out_w = 0, out_h = 0;
    bool configured = false, timing = false;
    // a submit failed after its ticket was issued: later calls refuse until the next configure
    bool broken = false;
    // frames in flight, in submission order: (ticket, device index, slot)
    struct Pending {
        int64_t ticket;
        int dev, slot;
    };
    std::deque<Pending> pending;
    std::string err;

    int fail(int code, const char *fmt, ...)
    {
        char b[512];
        va_list ap;
        va_start(ap, fmt);
        std::vsnprintf(b, sizeof(b), fmt, ap);
        va_end(ap);
        err = b;
        return code;
    }
    // Waits for the oldest frame in flight and retires it.
    int retire_front(bool block)
    {
        if (pending.empty()) return fail(AJIB_ERR, "a ticket was lost: an earlier submit failed");
        const Pending p = pending.front();
        Dev &d = devs[p.dev];
        CtxGuard g(d.cu);
        if (!g.ok) return fail(AJIB_ERR_CUDA, "cannot make device %d's context current", d.ordinal);
        const cudaEvent_t ev = d.ring[p.slot].down;
        const cudaError_t e = block ? cudaEventSynchronize(ev) : cudaEventQuery(ev);
        if (e == cudaErrorNotReady) return 0;
        if (e != cudaSuccess) return fail(AJIB_ERR_CUDA, "device %d: frame %lld failed: %s", d.ordinal,
                                          (long long)p.ticket, cudaGetErrorString(e));
        const int st = ajib_kernel_status(1);
        if (st != 0)
            return fail(AJIB_ERR_TIMEOUT, "device %d: a native kernel timed out waiting on its pipeline (code %d)",
                        d.ordinal, st);
        order->mark_done(p.ticket);
        pending.pop_front();
        return 1;
    }
    void free_ring(Dev &d)
    {
        for (Slot &s : d.ring) {
            cudaFree(s.in[0]);
            cudaFree(s.out[0]);
            if (s.up) cudaEventDestroy(s.up);
            if (s.done) cudaEventDestroy(s.done);
            if (s.down) cudaEventDestroy(s.down);
            s = Slot{};
        }
    }
    // Everything in flight finished (on every device); the host may reuse every buffer.
    int drain()
    {
        while (!pending.empty()) {
            const int rc = retire_front(true);
            if (rc < 0) return rc;
        }
        return AJIB_OK;
    }
};

namespace {

void destroy_devs(ajib_video_multi *m)
{
    const Driver &drv = driver();
    for (Dev &d : m->devs) {
        if (d.cu) {
            CtxGuard g(d.cu);
            if (g.ok) {
                cudaDeviceSynchronize();
                m->free_ring(d);
                if (d.t0) cudaEventDestroy(d.t0);
                if (d.t1) cudaEventDestroy(d.t1);
                if (d.s_up) cudaStreamDestroy(d.s_up);
                if (d.s_comp) cudaStreamDestroy(d.s_comp);
                if (d.s_down) cudaStreamDestroy(d.s_down);
            }
        }
        if (d.ctx) aji_destroy(&d.ctx);
        if (d.retained) drv.primary_release(d.cudev);
    }
    m->devs.clear();
}

}  // namespace

extern "C" ajib_video_multi *ajib_video_create_multi(const aji_create_params *params, const int *devices, int n,
                                                     int depth, char *err, size_t err_size)
{
    auto fail = [&](const char *msg) -> ajib_video_multi * {
        if (err && err_size) std::snprintf(err, err_size, "%s", msg);
        return nullptr;
    };
    if (!params || params->api_version != AJI_API_VERSION) return fail("bad create params or API version");
    if (!devices || n < 1 || n > 64) return fail("need 1..64 devices");
    if (depth < 1 || depth > 16) return fail("ring depth must be 1..16");
    for (int i = 0; i < n; i++)
        for (int j = 0; j < i; j++)
            if (devices[i] == devices[j]) return fail("a device is listed twice");
    const Driver &drv = driver();
    if (!drv.ok || drv.init(0) != CUDA_SUCCESS) return fail("no CUDA driver");
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess) return fail("no CUDA device");
    try {
        auto m = std::make_unique<ajib_video_multi>();
        m->depth = depth;
        m->devs.resize(n);
        for (int i = 0; i < n; i++) {
            Dev &d = m->devs[i];
            d.ordinal = devices[i];
            if (d.ordinal < 0 || d.ordinal >= count) {
                destroy_devs(m.get());
                return fail("no such CUDA device");
            }
            if (drv.device_get(&d.cudev, d.ordinal) != CUDA_SUCCESS || drv.primary_retain(&d.cu, d.cudev) != CUDA_SUCCESS) {
                destroy_devs(m.get());
                return fail("cannot retain a device's primary context");
            }
            d.retained = true;
            aji_create_params p = *params;
            p.cuda_context = d.cu;
            d.ctx = aji_create(&p);
            if (!d.ctx) {
                destroy_devs(m.get());
                return fail("aji_create refused the parameters on a device (model, conf or device type)");
            }
            CtxGuard g(d.cu);
            if (!g.ok || cudaStreamCreateWithFlags(&d.s_up, cudaStreamNonBlocking) != cudaSuccess ||
                cudaStreamCreateWithFlags(&d.s_comp, cudaStreamNonBlocking) != cudaSuccess ||
                cudaStreamCreateWithFlags(&d.s_down, cudaStreamNonBlocking) != cudaSuccess ||
                cudaEventCreate(&d.t0) != cudaSuccess || cudaEventCreate(&d.t1) != cudaSuccess) {
                destroy_devs(m.get());
                return fail("stream or event creation failed");
            }
        }
        m->order = std::make_unique<FrameOrder>(n, depth);
        return m.release();
    } catch (...) {
        return fail("out of host memory");
    }
}

extern "C" int ajib_video_multi_configure(ajib_video_multi *m, int w, int h, double fps, int *out_w, int *out_h)
{
    if (!m) return AJIB_ERR_ARGS;
    int rc = m->drain();
    if (rc < 0) return rc;
    int ow = 0, oh = 0;
    for (size_t i = 0; i < m->devs.size(); i++) {
        Dev &d = m->devs[i];
        int w1 = 0, h1 = 0;
        const int c = aji_configure(d.ctx, w, h, fps, &w1, &h1);
        if (c < 0) return m->fail(c, "device %d: %s", d.ordinal, aji_last_error(d.ctx));
        if (i == 0) {
            ow = w1;
            oh = h1;
        } else if (w1 != ow || h1 != oh) {
            return m->fail(AJIB_ERR, "devices disagree on the output size");
        }
        CtxGuard g(d.cu);
        if (!g.ok) return m->fail(AJIB_ERR_CUDA, "cannot make device %d's context current", d.ordinal);
        m->free_ring(d);
        d.ring.assign(m->depth, Slot{});
        for (Slot &s : d.ring)
            if (cudaEventCreateWithFlags(&s.up, cudaEventDisableTiming) != cudaSuccess ||
                cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming) != cudaSuccess ||
                cudaEventCreateWithFlags(&s.down, cudaEventDisableTiming) != cudaSuccess)
                return m->fail(AJIB_ERR_CUDA, "event creation failed");
    }
    m->in_w = w;
    m->in_h = h;
    m->out_w = ow;
    m->out_h = oh;
    m->configured = true;
    m->broken = false;
    m->order = std::make_unique<FrameOrder>((int)m->devs.size(), m->depth);
    if (out_w) *out_w = ow;
    if (out_h) *out_h = oh;
    return AJIB_OK;
}

extern "C" int64_t ajib_video_multi_submit(ajib_video_multi *m, const aji_frame *in, const aji_frame *out)
{
    if (!m || !in || !out) return AJIB_ERR_ARGS;
    if (!m->configured) return m->fail(AJIB_ERR, "submit before configure");
    if (in->width != m->in_w || in->height != m->in_h || out->width != m->out_w || out->height != m->out_h)
        return m->fail(AJIB_ERR_ARGS, "frame dims %dx%d->%dx%d do not match configured %dx%d->%dx%d", in->width,
                       in->height, out->width, out->height, m->in_w, m->in_h, m->out_w, m->out_h);
    int in_rows[3], out_rows[3];
    size_t in_rb[3], out_rb[3];
    const int npi = frame_planes(in->format, in->width, in->height, in_rows, in_rb);
    const int npo = frame_planes(out->format, out->width, out->height, out_rows, out_rb);
    if (!npi || !npo) return m->fail(AJIB_ERR_ARGS, "unsupported frame format (NV12, P010 or 16-bit 4:4:4)");
    for (int p = 0; p < npi; p++)
        if (!in->plane[p] || in->stride[p] < (ptrdiff_t)in_rb[p]) return m->fail(AJIB_ERR_ARGS, "bad input plane %d", p);
    for (int p = 0; p < npo; p++)
        if (!out->plane[p] || out->stride[p] < (ptrdiff_t)out_rb[p])
            return m->fail(AJIB_ERR_ARGS, "bad output plane %d", p);

    if (m->broken) return m->fail(AJIB_ERR, "an earlier submit failed; configure again");
    const FrameOrder::Place pl = m->order->next();
    m->broken = true;  // until this frame is fully enqueued
    // the slot's previous frame must have finished before its buffers are reused: retire frames in
    // order until it has
    while (pl.reuse && !m->order->finished(pl.reuse)) {
        const int rc = m->retire_front(true);
        if (rc < 0) return rc;
    }
    Dev &d = m->devs[pl.device];
    Slot &s = d.ring[pl.slot];
    CtxGuard g(d.cu);
    if (!g.ok) return m->fail(AJIB_ERR_CUDA, "cannot make device %d's context current", d.ordinal);
    size_t in_need = 0, out_need = 0, in_off[3], out_off[3];
    for (int p = 0; p < npi; p++) {
        in_off[p] = in_need;
        in_need += (in_rb[p] * in_rows[p] + 255) / 256 * 256;
    }
    for (int p = 0; p < npo; p++) {
        out_off[p] = out_need;
        out_need += (out_rb[p] * out_rows[p] + 255) / 256 * 256;
    }
    if (in_need > s.in_cap) {
        cudaFree(s.in[0]);
        s.in[0] = nullptr;
        s.in_cap = 0;
        if (cudaMalloc(&s.in[0], in_need) != cudaSuccess) {
            cudaGetLastError();
            return m->fail(AJIB_ERR_NO_MEM, "device %d: frame buffer allocation failed", d.ordinal);
        }
        s.in_cap = in_need;
    }
    if (out_need > s.out_cap) {
        cudaFree(s.out[0]);
        s.out[0] = nullptr;
        s.out_cap = 0;
        if (cudaMalloc(&s.out[0], out_need) != cudaSuccess) {
            cudaGetLastError();
            return m->fail(AJIB_ERR_NO_MEM, "device %d: frame buffer allocation failed", d.ordinal);
        }
        s.out_cap = out_need;
    }
    aji_frame din = *in, dout = *out;
    for (int p = 0; p < 3; p++) {
        din.plane[p] = p < npi ? (char *)s.in[0] + in_off[p] : nullptr;
        din.stride[p] = p < npi ? (ptrdiff_t)in_rb[p] : 0;
        dout.plane[p] = p < npo ? (char *)s.out[0] + out_off[p] : nullptr;
        dout.stride[p] = p < npo ? (ptrdiff_t)out_rb[p] : 0;
    }
    if (m->timing && !d.t0_set) {
        if (cudaEventRecord(d.t0, d.s_up) != cudaSuccess) return m->fail(AJIB_ERR_CUDA, "timing event failed");
        d.t0_set = true;
    }
    // upload
    for (int p = 0; p < npi; p++)
        if (cudaMemcpy2DAsync(din.plane[p], in_rb[p], in->plane[p], in->stride[p], in_rb[p], in_rows[p],
                              cudaMemcpyHostToDevice, d.s_up) != cudaSuccess)
            return m->fail(AJIB_ERR_CUDA, "device %d: upload failed", d.ordinal);
    if (cudaEventRecord(s.up, d.s_up) != cudaSuccess || cudaStreamWaitEvent(d.s_comp, s.up, 0) != cudaSuccess)
        return m->fail(AJIB_ERR_CUDA, "device %d: event failed", d.ordinal);
    // compute: the device's video context, on its compute stream
    const int rc = aji_infer(d.ctx, &din, &dout, d.s_comp);
    if (rc != AJI_OK) return m->fail(AJIB_ERR, "device %d: %s", d.ordinal, aji_last_error(d.ctx));
    if (cudaEventRecord(s.done, d.s_comp) != cudaSuccess || cudaStreamWaitEvent(d.s_down, s.done, 0) != cudaSuccess)
        return m->fail(AJIB_ERR_CUDA, "device %d: event failed", d.ordinal);
    // download
    for (int p = 0; p < npo; p++)
        if (cudaMemcpy2DAsync(out->plane[p], out->stride[p], dout.plane[p], out_rb[p], out_rb[p], out_rows[p],
                              cudaMemcpyDeviceToHost, d.s_down) != cudaSuccess)
            return m->fail(AJIB_ERR_CUDA, "device %d: download failed", d.ordinal);
    if (cudaEventRecord(s.down, d.s_down) != cudaSuccess) return m->fail(AJIB_ERR_CUDA, "device %d: event failed", d.ordinal);
    if (m->timing) {
        if (cudaEventRecord(d.t1, d.s_down) != cudaSuccess) return m->fail(AJIB_ERR_CUDA, "timing event failed");
        d.t1_set = true;
    }
    m->pending.push_back({pl.ticket, pl.device, pl.slot});
    m->broken = false;
    return pl.ticket;
}

extern "C" int ajib_video_multi_wait(ajib_video_multi *m, int64_t ticket)
{
    if (!m) return AJIB_ERR_ARGS;
    if (ticket < 1 || ticket > m->order->issued()) return m->fail(AJIB_ERR_ARGS, "no such ticket");
    while (m->order->completed() < ticket) {
        const int rc = m->retire_front(true);
        if (rc < 0) return rc;
    }
    return AJIB_OK;
}

extern "C" int ajib_video_multi_done(ajib_video_multi *m, int64_t ticket)
{
    if (!m) return AJIB_ERR_ARGS;
    if (ticket < 1 || ticket > m->order->issued()) return m->fail(AJIB_ERR_ARGS, "no such ticket");
    while (m->order->completed() < ticket && !m->pending.empty()) {
        const int rc = m->retire_front(false);
        if (rc < 0) return rc;
        if (rc == 0) break;
    }
    return m->order->completed() >= ticket ? 1 : 0;
}

extern "C" int ajib_video_multi_devices(const ajib_video_multi *m) { return m ? (int)m->devs.size() : 0; }

extern "C" int ajib_video_multi_timing(ajib_video_multi *m, int on)
{
    if (!m) return AJIB_ERR_ARGS;
    const int rc = m->drain();
    if (rc < 0) return rc;
    m->timing = on != 0;
    for (Dev &d : m->devs) d.t0_set = d.t1_set = false;
    return AJIB_OK;
}

extern "C" int ajib_video_multi_device_ms(ajib_video_multi *m, double *ms, int n)
{
    if (!m || !ms || n < (int)m->devs.size()) return AJIB_ERR_ARGS;
    const int rc = m->drain();
    if (rc < 0) return rc;
    for (size_t i = 0; i < m->devs.size(); i++) {
        Dev &d = m->devs[i];
        ms[i] = 0.0;
        if (!d.t0_set || !d.t1_set) continue;
        CtxGuard g(d.cu);
        float t = 0.f;
        if (!g.ok || cudaEventElapsedTime(&t, d.t0, d.t1) != cudaSuccess)
            return m->fail(AJIB_ERR_CUDA, "device %d: timing read failed", d.ordinal);
        ms[i] = t;
    }
    return AJIB_OK;
}

extern "C" const char *ajib_video_multi_error(const ajib_video_multi *m) { return m ? m->err.c_str() : "no context"; }

extern "C" void ajib_video_multi_destroy(ajib_video_multi **pm)
{
    if (!pm || !*pm) return;
    destroy_devs(*pm);
    delete *pm;
    *pm = nullptr;
}

// ---- the frame order alone, for tests on machines without a GPU ----
extern "C" int ajib_selftest_frame_order(int ndev, int depth, int nframes, const int64_t *finish_order, int *device_of,
                                         int *slot_of, int64_t *reuse_of, int64_t *completed_after)
{
    if (ndev < 1 || depth < 1 || nframes < 0 || (nframes && (!finish_order || !device_of || !slot_of || !reuse_of ||
                                                               !completed_after)))
        return AJIB_ERR_ARGS;
    try {
        FrameOrder o(ndev, depth);
        for (int k = 0; k < nframes; k++) {
            const FrameOrder::Place p = o.next();
            device_of[k] = p.device;
            slot_of[k] = p.slot;
            reuse_of[k] = p.reuse;
        }
        for (int k = 0; k < nframes; k++) completed_after[k] = o.mark_done(finish_order[k]);
        return AJIB_OK;
    } catch (...) {
        return AJIB_ERR_NO_MEM;
    }
}
