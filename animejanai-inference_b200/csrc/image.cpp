/*
 * image.cpp — the still-image C ABI (include/aji_image.h) over the native path: the image goes to
 * the GPU once, every tile is cut out in one batched launch, the whole batch runs through the
 * conv net together (tiles stacked along H, each convolved on its own), and one pass blends the
 * tiles into the 8-bit output, which comes back to the caller's buffer.
 *
 * Reference behaviour followed (the-database/animejanai-inference): device enumeration and ids
 * (src/aji_img_trt.cpp:69-73, :497-517), context creation (:520-560), argument checks of
 * upscale_tiled (src/core/tiling.cpp:119-140), tile geometry and blend (tiling.cpp:17-289,
 * tiling_gpu.cu), one upscale at a time per context (:1065), progress callback between tiles
 * with cancellation (:1006-1010), memory report (:1184-1216). Models are this engine's native
 * model files, passed as onnx_path; there is no engine to build, so a load is READY at once.
 */
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>

#include "plan.h"
#include "tiler.h"
#include "../../include/aji_b200.h"
#include "../../include/aji_image.h"

using namespace ajib;

namespace {

uint64_t pci_id(const cudaDeviceProp &p)
{
    return (1ull << 63) | ((uint64_t)(uint32_t)p.pciDomainID << 32) | ((uint64_t)(uint32_t)p.pciBusID << 8) |
           (uint64_t)(p.pciDeviceID & 0xff);
}

bool backend_ok(int b) { return b == AJI_IMG_TENSORRT || b == AJI_IMG_TENSORRT_RTX; }

std::mutex g_open_mu;
int g_open[64] = {};  // open contexts per CUDA ordinal

constexpr int kMaxBatch = 256;  // tiles per net launch

}  // namespace

struct aji_img_model;

struct aji_img_ctx {
    int device = 0;
    aji_img_log_fn log = nullptr;
    void *log_opaque = nullptr;
    std::string err;
    std::mutex run_mu;
    cudaStream_t stream = nullptr;
    std::vector<aji_img_model *> models;
    // scratch shared by the context's models, grown on demand
    uint8_t *d_img = nullptr, *d_out = nullptr;
    void *d_tin = nullptr, *d_tout = nullptr;
    size_t img_cap = 0, out_cap = 0, tin_cap = 0, tout_cap = 0;
    std::unique_ptr<DeviceTiler> tiler;  // the last geometry's tables
    int tiler_key[8] = {0, 0, 0, 0, 0, 0, 0, 0};

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
    size_t scratch_bytes() const { return img_cap + out_cap + tin_cap + tout_cap + (tiler ? tiler->table_bytes() : 0); }
};

struct aji_img_model {
    aji_img_ctx *ctx = nullptr;
    Plan plan;
    std::unique_ptr<Executor> exec;
    int capacity = 0;  // tiles the executor holds at once
    int tile_w = 512, tile_h = 512, overlap = 128, flags = 0, scale = 1;
};

namespace {

bool grow(void **p, size_t *cap, size_t need)
{
    if (need <= *cap) return true;
    cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    if (cudaMalloc(p, need) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    *cap = need;
    return true;
}

// The executor sized for n tiles of the model's tile (grown, never shrunk).
bool ensure_exec(aji_img_model *m, int n)
{
    if (m->exec && m->capacity >= n) return true;
    m->exec.reset();
    std::string why;
    m->exec = Executor::create(m->plan, m->tile_w, m->tile_h * n, &why);
    if (!m->exec) {
        m->ctx->set_error("native model refused at %d tiles of %dx%d: %s", n, m->tile_w, m->tile_h, why.c_str());
        m->capacity = 0;
        return false;
    }
    m->capacity = n;
    return true;
}

int device_ordinal(uint64_t id, int *out)
{
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n < 1) return -1;
    for (int d = 0; d < n; d++) {
        cudaDeviceProp p;
        if (cudaGetDeviceProperties(&p, d) == cudaSuccess && (id == 0 || pci_id(p) == id)) {
            *out = d;
            return 0;
        }
    }
    return -1;
}

}  // namespace

extern "C" int aji_img_enum_devices(int backend, aji_img_device *out, int max)
{
    if (!backend_ok(backend)) return -1;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    for (int d = 0; d < n && out && d < max; d++) {
        cudaDeviceProp p;
        if (cudaGetDeviceProperties(&p, d) != cudaSuccess) return -1;
        aji_img_device &o = out[d];
        std::memset(&o, 0, sizeof(o));
        o.id = pci_id(p);
        std::snprintf(o.name, sizeof(o.name), "%.127s", p.name);
        o.vram_bytes = p.totalGlobalMem;
        o.sm_major = p.major;
        o.sm_minor = p.minor;
    }
    return n;
}

extern "C" aji_img_ctx *aji_img_create(const aji_img_create_params *p, char *err, size_t err_size)
{
    auto fail = [&](const char *m) -> aji_img_ctx * {
        if (err && err_size) std::snprintf(err, err_size, "%s", m);
        return nullptr;
    };
    if (!p || p->api_version != AJI_IMAGE_API_VERSION) return fail("bad create params or API version");
    if (!backend_ok(p->backend)) return fail("this engine serves the CUDA backends only");
    try {
        auto c = std::make_unique<aji_img_ctx>();
        c->log = p->log;
        c->log_opaque = p->log_opaque;
        if (device_ordinal(p->device_id, &c->device) != 0) return fail("no such CUDA device");
        cudaDeviceProp prop;
        if (cudaSetDevice(c->device) != cudaSuccess || cudaGetDeviceProperties(&prop, c->device) != cudaSuccess)
            return fail("cannot use the CUDA device");
        if (prop.major != 10) return fail("this engine runs on Blackwell datacenter GPUs (sm_100) only");
        if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) return fail("cannot create a stream");
        {
            std::lock_guard<std::mutex> lk(g_open_mu);
            g_open[c->device & 63]++;
        }
        return c.release();
    } catch (...) {
        return fail("out of host memory");
    }
}

extern "C" aji_img_model *aji_img_load(aji_img_ctx *c, const aji_img_model_params *p)
{
    if (!c) return nullptr;
    if (!p || !p->onnx_path) {
        c->set_error("aji_img_load: no model path");
        return nullptr;
    }
    try {
        cudaSetDevice(c->device);
        auto m = std::make_unique<aji_img_model>();
        m->ctx = c;
        std::string why;
        if (!load_model_file(p->onnx_path, &m->plan, &why)) {
            c->set_error("%s", why.c_str());
            return nullptr;
        }
        m->tile_w = p->tile_w > 0 ? p->tile_w : 512;
        m->tile_h = p->tile_h > 0 ? p->tile_h : 512;
        m->overlap = p->overlap > 0 ? p->overlap : 128;
        m->flags = p->flags;
        m->scale = m->plan.depth_to_space;
        if (!ensure_exec(m.get(), 1)) return nullptr;
        c->models.push_back(m.get());
        return m.release();
    } catch (...) {
        c->set_error("out of host memory");
        return nullptr;
    }
}

extern "C" int aji_img_model_state(aji_img_model *m) { return m ? AJI_IMG_STATE_READY : AJI_IMG_STATE_FAILED; }

extern "C" int aji_img_model_info_get(aji_img_model *m, aji_img_model_info *info)
{
    if (!m || !info) return AJI_IMG_ERR_ARGS;
    info->scale = m->scale;
    info->in_channels = 3;
    info->out_channels = 3;
    info->tile_w = m->tile_w;
    info->tile_h = m->tile_h;
    info->overlap = m->overlap;
    return AJI_IMG_OK;
}

extern "C" int aji_img_upscale(aji_img_model *m, const aji_img_buffer *in, const aji_img_buffer *out,
                               aji_img_progress_fn progress, void *opaque)
{
    if (!m) return AJI_IMG_ERR_ARGS;
    aji_img_ctx *c = m->ctx;
    std::lock_guard<std::mutex> lk(c->run_mu);
    // argument checks of upscale_tiled (src/core/tiling.cpp:119-140)
    if (!in || !out || !in->data || !out->data) {
        c->set_error("null image buffer");
        return AJI_IMG_ERR_ARGS;
    }
    const int W = in->width, H = in->height, s = m->scale, ci = in->channels;
    if (W < 1 || H < 1 || (ci != 1 && ci != 3) || out->channels != ci) {
        c->set_error("image must be 1 or 3 channels, same on both sides");
        return AJI_IMG_ERR_ARGS;
    }
    if (out->width != W * s || out->height != H * s) {
        c->set_error("output must be %dx%d (scale %d)", W * s, H * s, s);
        return AJI_IMG_ERR_ARGS;
    }
    if (in->stride < (ptrdiff_t)W * ci || out->stride < (ptrdiff_t)W * s * ci) {
        c->set_error("stride smaller than a row");
        return AJI_IMG_ERR_ARGS;
    }
    try {
        if (cudaSetDevice(c->device) != cudaSuccess) {
            c->set_error("cannot use the CUDA device");
            return AJI_IMG_ERR;
        }
        cudaStream_t st = c->stream;
        const bool even = (m->flags & AJI_IMG_LOAD_EVEN_TILES) != 0;
        const int key[8] = {W, H, ci, s, m->tile_w, m->tile_h, m->overlap, even ? 1 : 0};
        if (!c->tiler || std::memcmp(key, c->tiler_key, sizeof(key)) != 0) {
            auto t = std::make_unique<DeviceTiler>();
            if (!t->init(make_geometry(W, H, ci, s, m->tile_w, m->tile_h, m->overlap, even))) {
                cudaGetLastError();
                c->set_error("out of device memory for the tile tables");
                return AJI_IMG_ERR_NO_MEM;
            }
            c->tiler = std::move(t);
            std::memcpy(c->tiler_key, key, sizeof(key));
        }
        const TileGeometry &g = c->tiler->geometry();
        const int count = g.count(), tw = g.tw, th = g.th, batch = std::min(count, kMaxBatch);
        const size_t tile_in = (size_t)3 * tw * th * 2, tile_out = tile_in * s * s;
        const size_t OW = (size_t)W * s, OH = (size_t)H * s;
        // with more tiles than one batch, each batch's output is staged after its input and then
        // copied into its place in the full stack
        const size_t staging = batch < count ? tile_out * batch : 0;
        if (!ensure_exec(m, batch)) return AJI_IMG_ERR_NO_MEM;
        if (!grow((void **)&c->d_img, &c->img_cap, (size_t)W * H * ci) || !grow((void **)&c->d_out, &c->out_cap, OW * OH * ci) ||
            !grow(&c->d_tin, &c->tin_cap, tile_in * batch + staging) || !grow(&c->d_tout, &c->tout_cap, tile_out * count)) {
            c->set_error("out of device memory for the tiling buffers");
            return AJI_IMG_ERR_NO_MEM;
        }
        if (cudaMemcpy2DAsync(c->d_img, (size_t)W * ci, in->data, in->stride, (size_t)W * ci, H, cudaMemcpyHostToDevice,
                              st) != cudaSuccess) {
            c->set_error("image upload failed");
            return AJI_IMG_ERR;
        }
        // every tile through the net, a batch at a time; a batch's output lands in its tiles'
        // place of the full stack ([3][count * th * s][tw * s])
        const size_t plane_all = (size_t)count * th * s * tw * s;
        for (int k0 = 0; k0 < count; k0 += batch) {
            const int n = std::min(batch, count - k0);
            const bool direct = n == count;
            void *dst = direct ? c->d_tout : (char *)c->d_tin + tile_in * batch;
            if (c->tiler->extract(c->d_img, k0, n, c->d_tin, st) != cudaSuccess ||
                m->exec->run_images(c->d_tin, dst, tw, th, n, st) != AJIB_OK) {
                c->set_error("tile kernels failed");
                return AJI_IMG_ERR;
            }
            if (!direct) {
                const size_t plane_n = (size_t)n * th * s * tw * s;
                for (int ch = 0; ch < 3; ch++)
                    if (cudaMemcpyAsync((uint16_t *)c->d_tout + ch * plane_all + (size_t)k0 * th * s * tw * s,
                                        (const uint16_t *)dst + ch * plane_n, plane_n * 2, cudaMemcpyDeviceToDevice,
                                        st) != cudaSuccess) {
                        c->set_error("tile output copy failed");
                        return AJI_IMG_ERR;
                    }
            }
            if (progress) {
                if (cudaStreamSynchronize(st) != cudaSuccess) {
                    c->set_error("tile kernels failed");
                    return AJI_IMG_ERR;
                }
                if (progress(opaque, k0 + n, count)) {
                    c->set_error("cancelled");
                    return AJI_IMG_CANCELLED;
                }
            }
        }
        if (c->tiler->compose(c->d_tout, c->d_out, st) != cudaSuccess ||
            cudaMemcpy2DAsync(out->data, out->stride, c->d_out, OW * ci, OW * ci, OH, cudaMemcpyDeviceToHost, st) !=
                cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess) {
            c->set_error("compose or download failed: %s", cudaGetErrorString(cudaGetLastError()));
            return AJI_IMG_ERR;
        }
        const int ks = ajib_kernel_status(1);
        if (ks != 0) {
            c->set_error("a native kernel timed out waiting on its pipeline (code %d)", ks);
            return AJI_IMG_ERR;
        }
        return AJI_IMG_OK;
    } catch (...) {
        c->set_error("out of host memory");
        return AJI_IMG_ERR_NO_MEM;
    }
}

extern "C" void aji_img_release(aji_img_model **pm)
{
    if (!pm || !*pm) return;
    aji_img_model *m = *pm;
    aji_img_ctx *c = m->ctx;
    {
        std::lock_guard<std::mutex> lk(c->run_mu);
        cudaSetDevice(c->device);
        c->models.erase(std::remove(c->models.begin(), c->models.end(), m), c->models.end());
        delete m;
    }
    *pm = nullptr;
}

extern "C" const char *aji_img_last_error(aji_img_ctx *c) { return c ? c->err.c_str() : "no context"; }

extern "C" void aji_img_destroy(aji_img_ctx **pc)
{
    if (!pc || !*pc) return;
    aji_img_ctx *c = *pc;
    cudaSetDevice(c->device);
    for (aji_img_model *m : c->models) delete m;
    c->models.clear();
    c->tiler.reset();
    cudaFree(c->d_img);
    cudaFree(c->d_out);
    cudaFree(c->d_tin);
    cudaFree(c->d_tout);
    if (c->stream) cudaStreamDestroy(c->stream);
    {
        std::lock_guard<std::mutex> lk(g_open_mu);
        g_open[c->device & 63]--;
    }
    delete c;
    *pc = nullptr;
}

extern "C" int aji_img_release_device(int backend, uint64_t device_id)
{
    if (!backend_ok(backend)) return 0;
    int d = 0;
    if (device_ordinal(device_id, &d) != 0) return -1;
    {
        std::lock_guard<std::mutex> lk(g_open_mu);
        if (g_open[d & 63] > 0) return -1;
    }
    // this engine keeps no per-device state beyond the CUDA context, which belongs to the
    // process's CUDA runtime: nothing to free here
    return 0;
}

extern "C" int aji_img_memory_get(aji_img_ctx *c, aji_img_model *m, aji_img_memory *out)
{
    if (!c || !out) return AJI_IMG_ERR_ARGS;
    std::memset(out, 0, sizeof(*out));
    cudaSetDevice(c->device);
    size_t fr = 0, tot = 0;
    if (cudaMemGetInfo(&fr, &tot) != cudaSuccess) return AJI_IMG_ERR;
    out->device_free = fr;
    out->device_total = tot;
    out->ctx_scratch = c->scratch_bytes();
    if (m && m->exec) {
        out->model_weights = m->exec->weight_bytes();
        out->model_activations = m->exec->device_bytes() - m->exec->weight_bytes();
        out->activations_shared = 0;
    }
    return AJI_IMG_OK;
}

extern "C" int aji_img_native_probe(aji_img_ctx *c, const aji_img_model_params *p, aji_img_memory *out)
{
    if (!c) return AJI_IMG_ERR_ARGS;
    aji_img_model *m = aji_img_load(c, p);
    if (!m) return AJI_IMG_ERR;
    int rc = AJI_IMG_OK;
    if (out) {
        rc = aji_img_memory_get(c, m, out);
        if (rc == AJI_IMG_OK) out->device_free += m->exec ? m->exec->device_bytes() : 0;
    }
    aji_img_release(&m);
    return rc;
}
