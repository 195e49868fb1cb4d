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
#include <thread>
#include <vector>

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
// A share's tile rows run in up to kWaves waves: the output rows a wave completes are composed and
// downloaded (on a second stream) while the next wave's tiles go through the net.
constexpr int kWaves = 4;

}  // namespace

struct aji_img_model;

// One device of a context: its stream, scratch and the tile tables of the last geometry.
struct ImgDev {
    int device = 0;
    cudaStream_t stream = nullptr;
    cudaStream_t copy = nullptr;      // the output bands' downloads
    cudaEvent_t band[kWaves] = {};    // a band composed on `stream`
    uint8_t *d_img = nullptr, *d_out = nullptr;
    void *d_tin = nullptr, *d_tout = nullptr;
    size_t img_cap = 0, out_cap = 0, tin_cap = 0, tout_cap = 0;
    std::unique_ptr<DeviceTiler> tiler;
    int tiler_key[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    size_t scratch_bytes() const { return img_cap + out_cap + tin_cap + tout_cap + (tiler ? tiler->table_bytes() : 0); }
};

struct aji_img_ctx {
    std::vector<ImgDev> devs;  // one for aji_img_create; several for ajib_img_create_multi
    int device = 0;            // devs[0].device
    aji_img_log_fn log = nullptr;
    void *log_opaque = nullptr;
    std::string err;
    std::mutex run_mu;
    std::vector<aji_img_model *> models;

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
    size_t scratch_bytes() const
    {
        size_t n = 0;
        for (const ImgDev &d : devs) n += d.scratch_bytes();
        return n;
    }
};

// The model instantiated on each of the context's devices.
struct ImgExec {
    std::unique_ptr<Executor> exec;
    int capacity = 0;  // tiles the executor holds at once
};

struct aji_img_model {
    aji_img_ctx *ctx = nullptr;
    Plan plan;
    std::vector<ImgExec> execs;  // per device of the context
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

// The executor of device index di sized for n tiles of the model's tile (grown, never shrunk).
// The device must be current. *why on failure.
bool ensure_exec(aji_img_model *m, size_t di, int n, std::string *why)
{
    ImgExec &x = m->execs[di];
    if (x.exec && x.capacity >= n) return true;
    x.exec.reset();
    std::string r;
    x.exec = Executor::create(m->plan, m->tile_w, m->tile_h * n, &r);
    if (!x.exec) {
        char b[512];
        std::snprintf(b, sizeof(b), "native model refused at %d tiles of %dx%d: %s", n, m->tile_w, m->tile_h, r.c_str());
        *why = b;
        x.capacity = 0;
        return false;
    }
    x.capacity = n;
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

// Open device ordinal d for a context: sm_100 only, a non-blocking stream. *why on failure.
bool open_dev(int d, ImgDev *out, const char **why)
{
    cudaDeviceProp prop;
    if (cudaSetDevice(d) != cudaSuccess || cudaGetDeviceProperties(&prop, d) != cudaSuccess) {
        *why = "cannot use the CUDA device";
        return false;
    }
    if (prop.major != 10) {
        *why = "this engine runs on Blackwell datacenter GPUs (sm_100) only";
        return false;
    }
    out->device = d;
    if (cudaStreamCreateWithFlags(&out->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&out->copy, cudaStreamNonBlocking) != cudaSuccess) {
        *why = "cannot create a stream";
        return false;
    }
    for (cudaEvent_t &e : out->band)
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
            *why = "cannot create an event";
            return false;
        }
    std::lock_guard<std::mutex> lk(g_open_mu);
    g_open[d & 63]++;
    return true;
}

void close_dev(ImgDev &d)
{
    cudaSetDevice(d.device);
    d.tiler.reset();
    cudaFree(d.d_img);
    cudaFree(d.d_out);
    cudaFree(d.d_tin);
    cudaFree(d.d_tout);
    if (d.stream) cudaStreamDestroy(d.stream);
    if (d.copy) cudaStreamDestroy(d.copy);
    for (cudaEvent_t &e : d.band)
        if (e) cudaEventDestroy(e);
    d.stream = d.copy = nullptr;
    std::lock_guard<std::mutex> lk(g_open_mu);
    g_open[d.device & 63]--;
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

namespace {

aji_img_ctx *create_ctx(const aji_img_create_params *p, const int *ordinals, int n, char *err, size_t err_size)
{
    auto fail = [&](const char *m) -> aji_img_ctx * {
        if (err && err_size) std::snprintf(err, err_size, "%s", m);
        return nullptr;
    };
    auto c = std::make_unique<aji_img_ctx>();
    c->log = p->log;
    c->log_opaque = p->log_opaque;
    for (int i = 0; i < n; i++) {
        for (int k = 0; k < i; k++)
            if (ordinals[k] == ordinals[i]) {
                for (ImgDev &d : c->devs) close_dev(d);
                return fail("a device is listed twice");
            }
        ImgDev d;
        const char *why = nullptr;
        if (!open_dev(ordinals[i], &d, &why)) {
            for (ImgDev &o : c->devs) close_dev(o);
            return fail(why);
        }
        c->devs.push_back(std::move(d));
    }
    c->device = c->devs[0].device;
    return c.release();
}

}  // namespace

extern "C" aji_img_ctx *aji_img_create(const aji_img_create_params *p, char *err, size_t err_size)
{
    auto fail = [&](const char *m) -> aji_img_ctx * {
        if (err && err_size) std::snprintf(err, err_size, "%s", m);
        return nullptr;
    };
    if (!p || p->api_version != AJI_IMAGE_API_VERSION) return fail("bad create params or API version");
    if (!backend_ok(p->backend)) return fail("this engine serves the CUDA backends only");
    try {
        int d = 0;
        if (device_ordinal(p->device_id, &d) != 0) return fail("no such CUDA device");
        return create_ctx(p, &d, 1, err, err_size);
    } catch (...) {
        return fail("out of host memory");
    }
}

extern "C" aji_img_ctx *ajib_img_create_multi(const aji_img_create_params *p, const uint64_t *device_ids, int n, char *err,
                                              size_t err_size)
{
    auto fail = [&](const char *m) -> aji_img_ctx * {
        if (err && err_size) std::snprintf(err, err_size, "%s", m);
        return nullptr;
    };
    if (!p || p->api_version != AJI_IMAGE_API_VERSION) return fail("bad create params or API version");
    if (!backend_ok(p->backend)) return fail("this engine serves the CUDA backends only");
    if (!device_ids || n < 1 || n > 64) return fail("need 1..64 device ids");
    try {
        std::vector<int> ord(n);
        for (int i = 0; i < n; i++)
            if (device_ordinal(device_ids[i], &ord[i]) != 0) return fail("no such CUDA device");
        return create_ctx(p, ord.data(), n, err, err_size);
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
        m->scale = ajib::model_scale(m->plan);
        m->execs.resize(c->devs.size());
        for (size_t i = 0; i < c->devs.size(); i++) {
            cudaSetDevice(c->devs[i].device);
            if (!ensure_exec(m.get(), i, 1, &why)) {
                c->set_error("%s", why.c_str());
                return nullptr;
            }
        }
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

namespace {

// One device's share of an upscale: the output rows [Y0, Y1), from tile rows [j0, j1]. Runs with
// the device current; the first failure is reported through *why (and its status returned).
struct Share {
    int Y0 = 0, Y1 = 0, j0 = 0, j1 = -1;
    int tiles() const { return j1 >= j0 ? j1 - j0 + 1 : 0; }
};

std::vector<Share> make_shares(const TileGeometry &g, int ndev)
{
    const int ny = g.ny(), nd = std::max(1, std::min(ndev, ny)), s = g.scale;
    std::vector<Share> shares(nd);
    for (int d = 0; d < nd; d++) {
        const int ga = (int)((long)d * ny / nd), gb = (int)((long)(d + 1) * ny / nd) - 1;
        Share &sh = shares[d];
        sh.Y0 = d == 0 ? 0 : g.oy[ga] * s;
        sh.Y1 = d == nd - 1 ? g.H * s : g.oy[gb + 1] * s;
        tile_rows_covering(g, sh.Y0, sh.Y1, &sh.j0, &sh.j1);
    }
    return shares;
}

int run_share(aji_img_model *m, size_t di, const Share &sh, const aji_img_buffer *in, const aji_img_buffer *out,
              bool even, aji_img_progress_fn progress, void *opaque, std::string *why)
{
    aji_img_ctx *c = m->ctx;
    ImgDev &D = c->devs[di];
    const int W = in->width, H = in->height, s = m->scale, ci = in->channels;
    if (cudaSetDevice(D.device) != cudaSuccess) {
        *why = "cannot use the CUDA device";
        return AJI_IMG_ERR;
    }
    cudaStream_t st = D.stream;
    const int key[8] = {W, H, ci, s, m->tile_w, m->tile_h, m->overlap, even ? 1 : 0};
    if (!D.tiler || std::memcmp(key, D.tiler_key, sizeof(key)) != 0) {
        auto t = std::make_unique<DeviceTiler>();
        if (!t->init(make_geometry(W, H, ci, s, m->tile_w, m->tile_h, m->overlap, even))) {
            cudaGetLastError();
            *why = "out of device memory for the tile tables";
            return AJI_IMG_ERR_NO_MEM;
        }
        D.tiler = std::move(t);
        std::memcpy(D.tiler_key, key, sizeof(key));
    }
    const TileGeometry &g = D.tiler->geometry();
    const int nx = g.nx(), k0 = sh.j0 * nx, count = sh.tiles() * nx, tw = g.tw, th = g.th;
    // waves: contiguous groups of the share's tile rows
    const int nrows = sh.tiles(), nw = std::max(1, std::min(kWaves, nrows));
    const int wave_tiles = (nrows + nw - 1) / nw * nx;
    const int batch = std::min(wave_tiles, kMaxBatch);
    const size_t tile_in = (size_t)3 * tw * th * 2, tile_out = tile_in * s * s;
    const size_t OW = (size_t)W * s, rows = (size_t)(sh.Y1 - sh.Y0);
    if (!ensure_exec(m, di, batch, why)) return AJI_IMG_ERR_NO_MEM;
    if (!grow((void **)&D.d_img, &D.img_cap, (size_t)W * H * ci) || !grow((void **)&D.d_out, &D.out_cap, OW * rows * ci) ||
        !grow(&D.d_tin, &D.tin_cap, tile_in * batch) || !grow(&D.d_tout, &D.tout_cap, tile_out * count)) {
        *why = "out of device memory for the tiling buffers";
        return AJI_IMG_ERR_NO_MEM;
    }
    // no download may still be writing the caller's buffer when this returns
    auto fail = [&](int rc, const std::string &w) {
        cudaStreamSynchronize(D.copy);
        cudaStreamSynchronize(st);
        *why = w;
        return rc;
    };
    // the whole input on every device (tiles reflect across the image edges)
    if (cudaMemcpy2DAsync(D.d_img, (size_t)W * ci, in->data, in->stride, (size_t)W * ci, H, cudaMemcpyHostToDevice, st) !=
        cudaSuccess)
        return fail(AJI_IMG_ERR, "image upload failed");
    // The share's tiles stack as [3][count * th * s][tw * s] (the compose's layout); each batch's
    // net output lands in its tiles' place, its planes plane_all elements apart. After a wave,
    // the output rows before the next tile row's first are final: composed on `stream`, then
    // downloaded on `copy` while the next wave runs.
    Executor &ex = *m->execs[di].exec;
    const size_t plane_all = (size_t)count * th * s * tw * s, tile_elems = (size_t)th * s * tw * s;
    uint8_t *host_rows = (uint8_t *)out->data + (ptrdiff_t)sh.Y0 * out->stride;
    int y_done = sh.Y0, tiles_done = 0;
    for (int w = 0; w < nw; w++) {
        const int ja = sh.j0 + (int)((long)w * nrows / nw), jb = sh.j0 + (int)((long)(w + 1) * nrows / nw) - 1;
        for (int b0 = ja * nx; b0 < (jb + 1) * nx; b0 += batch) {
            const int n = std::min(batch, (jb + 1) * nx - b0);
            if (D.tiler->extract(D.d_img, b0, n, D.d_tin, st) != cudaSuccess ||
                ex.run_images(D.d_tin, (uint16_t *)D.d_tout + (size_t)(b0 - k0) * tile_elems, tw, th, n, st, plane_all) !=
                    AJIB_OK)
                return fail(AJI_IMG_ERR, "tile kernels failed");
            tiles_done += n;
        }
        const int y_end = w == nw - 1 ? sh.Y1 : std::min(sh.Y1, std::max(y_done, g.oy[jb + 1] * s));
        if (y_end > y_done) {
            const size_t off = (size_t)(y_done - sh.Y0);
            if (D.tiler->compose_rows(D.d_tout, k0, count, y_done, y_end, D.d_out + off * OW * ci, st) != cudaSuccess ||
                cudaEventRecord(D.band[w], st) != cudaSuccess || cudaStreamWaitEvent(D.copy, D.band[w], 0) != cudaSuccess ||
                cudaMemcpy2DAsync(host_rows + (ptrdiff_t)off * out->stride, out->stride, D.d_out + off * OW * ci, OW * ci,
                                  OW * ci, (size_t)(y_end - y_done), cudaMemcpyDeviceToHost, D.copy) != cudaSuccess)
                return fail(AJI_IMG_ERR, std::string("compose or download failed: ") + cudaGetErrorString(cudaGetLastError()));
            y_done = y_end;
        }
        if (progress) {
            if (cudaStreamSynchronize(st) != cudaSuccess) return fail(AJI_IMG_ERR, "tile kernels failed");
            if (progress(opaque, tiles_done, count)) return fail(AJI_IMG_CANCELLED, "cancelled");
        }
    }
    if (cudaStreamSynchronize(st) != cudaSuccess || cudaStreamSynchronize(D.copy) != cudaSuccess)
        return fail(AJI_IMG_ERR, std::string("compose or download failed: ") + cudaGetErrorString(cudaGetLastError()));
    const int ks = ajib_kernel_status(1);
    if (ks != 0) {
        *why = "a native kernel timed out waiting on its pipeline (code " + std::to_string(ks) + ")";
        return AJI_IMG_ERR;
    }
    return AJI_IMG_OK;
}

}  // namespace

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
        const bool even = (m->flags & AJI_IMG_LOAD_EVEN_TILES) != 0;
        const TileGeometry g = make_geometry(W, H, ci, s, m->tile_w, m->tile_h, m->overlap, even);
        // shares: contiguous groups of tile rows per device; a device owns the output rows from
        // the start of its first tile row to the start of the next device's, and also runs the
        // tile row before its group whose blend reaches into those rows (no data crosses devices;
        // every output pixel is blended in the one-device order, so the bytes are the same)
        const std::vector<Share> shares = make_shares(g, (int)c->devs.size());
        const int nd = (int)shares.size();
        if (nd == 1) {
            std::string why;
            const int rc = run_share(m, 0, shares[0], in, out, even, progress, opaque, &why);
            if (rc != AJI_IMG_OK) c->set_error("%s", why.c_str());
            return rc;
        }
        // several devices: one host thread each; progress reports whole shares as they finish
        std::vector<int> rcs(nd, AJI_IMG_OK);
        std::vector<std::string> whys(nd);
        std::vector<std::thread> threads;
        for (int d = 0; d < nd; d++)
            threads.emplace_back([&, d] { rcs[d] = run_share(m, d, shares[d], in, out, even, nullptr, nullptr, &whys[d]); });
        int total = 0, done = 0;
        for (const Share &sh : shares) total += sh.tiles() * g.nx();
        bool cancel = false;
        for (int d = 0; d < nd; d++) {
            threads[d].join();
            done += shares[d].tiles() * g.nx();
            if (progress && !cancel && rcs[d] == AJI_IMG_OK && progress(opaque, done, total)) cancel = true;
        }
        for (int d = 0; d < nd; d++)
            if (rcs[d] != AJI_IMG_OK) {
                c->set_error("device %d: %s", c->devs[d].device, whys[d].c_str());
                return rcs[d];
            }
        if (cancel) {
            c->set_error("cancelled");
            return AJI_IMG_CANCELLED;
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
        c->models.erase(std::remove(c->models.begin(), c->models.end(), m), c->models.end());
        for (size_t i = 0; i < m->execs.size(); i++) {
            cudaSetDevice(c->devs[i].device);
            m->execs[i].exec.reset();
        }
        delete m;
    }
    *pm = nullptr;
}

extern "C" const char *aji_img_last_error(aji_img_ctx *c) { return c ? c->err.c_str() : "no context"; }

extern "C" void aji_img_destroy(aji_img_ctx **pc)
{
    if (!pc || !*pc) return;
    aji_img_ctx *c = *pc;
    while (!c->models.empty()) {
        aji_img_model *m = c->models.back();
        aji_img_release(&m);
    }
    for (ImgDev &d : c->devs) close_dev(d);
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
    // the first device's figures (the reference reports one device per context)
    cudaSetDevice(c->devs[0].device);
    size_t fr = 0, tot = 0;
    if (cudaMemGetInfo(&fr, &tot) != cudaSuccess) return AJI_IMG_ERR;
    out->device_free = fr;
    out->device_total = tot;
    out->ctx_scratch = c->devs[0].scratch_bytes();
    if (m && !m->execs.empty() && m->execs[0].exec) {
        out->model_weights = m->execs[0].exec->weight_bytes();
        out->model_activations = m->execs[0].exec->device_bytes() - m->execs[0].exec->weight_bytes();
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
        if (rc == AJI_IMG_OK && m->execs[0].exec) out->device_free += m->execs[0].exec->device_bytes();
    }
    aji_img_release(&m);
    return rc;
}

extern "C" int ajib_img_shares(int W, int H, int ci, int scale, int tile_w, int tile_h, int overlap, int even, int ndev,
                               int *y0, int *y1, int *j0, int *j1)
{
    if (W < 1 || H < 1 || (ci != 1 && ci != 3) || scale < 1 || tile_w < 1 || tile_h < 1 || overlap < 0 || ndev < 1)
        return -1;
    try {
        const std::vector<Share> sh = make_shares(make_geometry(W, H, ci, scale, tile_w, tile_h, overlap, even != 0), ndev);
        for (size_t d = 0; d < sh.size(); d++) {
            if (y0) y0[d] = sh[d].Y0;
            if (y1) y1[d] = sh[d].Y1;
            if (j0) j0[d] = sh[d].j0;
            if (j1) j1[d] = sh[d].j1;
        }
        return (int)sh.size();
    } catch (...) {
        return -1;
    }
}
