/*
 * api_native.cpp — C ABI over the native model and executor (include/aji_b200.h). No C++
 * exception crosses the ABI (the reference's guarded() barrier, src/native/guard.h:13-24).
 */
#include <cstdio>
#include <cstring>
#include <exception>
#include <new>

#include "plan.h"

struct ajib_model {
    ajib::Plan plan;
};
struct ajib_exec {
    std::unique_ptr<ajib::Executor> ex;
};

namespace {

void put(char *dst, size_t n, const std::string &s)
{
    if (dst && n) std::snprintf(dst, n, "%s", s.c_str());
}

template <typename F>
int guarded(char *err, size_t n, F &&fn)
{
    try {
        return fn();
    } catch (const std::bad_alloc &) {
        put(err, n, "out of host memory");
        return AJIB_ERR_NO_MEM;
    } catch (const std::exception &e) {
        put(err, n, e.what());
        return AJIB_ERR;
    } catch (...) {
        put(err, n, "unknown exception");
        return AJIB_ERR;
    }
}

}  // namespace

extern "C" int ajib_model_load(const char *path, ajib_model **out, char *err, size_t err_size)
{
    if (!path || !out) return AJIB_ERR_ARGS;
    *out = nullptr;
    return guarded(err, err_size, [&] {
        auto m = std::make_unique<ajib_model>();
        std::string why;
        if (!ajib::load_model_file(path, &m->plan, &why)) {
            put(err, err_size, why);
            return (int)AJIB_ERR;
        }
        *out = m.release();
        return (int)AJIB_OK;
    });
}

extern "C" int ajib_model_from_memory(const void *data, size_t size, ajib_model **out, char *err, size_t err_size)
{
    if (!data || !out) return AJIB_ERR_ARGS;
    *out = nullptr;
    return guarded(err, err_size, [&] {
        auto m = std::make_unique<ajib_model>();
        std::string why;
        if (!ajib::load_model_bytes(data, size, &m->plan, &why)) {
            put(err, err_size, why);
            return (int)AJIB_ERR;
        }
        *out = m.release();
        return (int)AJIB_OK;
    });
}

extern "C" void ajib_model_release(ajib_model **m)
{
    if (!m || !*m) return;
    delete *m;
    *m = nullptr;
}

extern "C" int ajib_model_save(const ajib_model *m, void *buf, size_t cap, size_t *size)
{
    if (!m) return AJIB_ERR_ARGS;
    return guarded(nullptr, 0, [&] {
        const std::vector<uint8_t> b = ajib::serialize_model(m->plan);
        if (size) *size = b.size();
        if (buf && cap >= b.size()) std::memcpy(buf, b.data(), b.size());
        return (buf && cap < b.size()) ? (int)AJIB_ERR_ARGS : (int)AJIB_OK;
    });
}

extern "C" int ajib_model_info(const ajib_model *m, int *scale, int *steps, double *flops_per_px, char *desc,
                               size_t desc_size)
{
    if (!m) return AJIB_ERR_ARGS;
    if (scale) *scale = ajib::model_scale(m->plan);
    if (steps) *steps = (int)m->plan.steps.size();
    if (flops_per_px) *flops_per_px = ajib::flops_per_pixel(m->plan);
    put(desc, desc_size, ajib::describe(m->plan));
    return AJIB_OK;
}

extern "C" int ajib_exec_create(const ajib_model *m, int w, int h, ajib_exec **out, char *err, size_t err_size)
{
    if (!m || !out) return AJIB_ERR_ARGS;
    *out = nullptr;
    return guarded(err, err_size, [&] {
        std::string why;
        auto ex = ajib::Executor::create(m->plan, w, h, &why);
        if (!ex) {
            put(err, err_size, why);
            return (int)AJIB_ERR;
        }
        auto e = std::make_unique<ajib_exec>();
        e->ex = std::move(ex);
        *out = e.release();
        return (int)AJIB_OK;
    });
}

extern "C" void ajib_exec_release(ajib_exec **e)
{
    if (!e || !*e) return;
    delete *e;
    *e = nullptr;
}

extern "C" int ajib_exec_run(ajib_exec *e, const void *in, void *out, void *stream)
{
    if (!e || !e->ex) return AJIB_ERR_ARGS;
    return e->ex->run(in, out, (cudaStream_t)stream);
}

extern "C" int ajib_exec_run_images(ajib_exec *e, const void *in, void *out, int w, int img_h, int nimg, void *stream)
{
    if (!e || !e->ex) return AJIB_ERR_ARGS;
    return e->ex->run_images(in, out, w, img_h, nimg, (cudaStream_t)stream);
}

extern "C" int ajib_exec_set_bands(ajib_exec *e, int bands)
{
    if (!e || !e->ex || bands < 1) return AJIB_ERR_ARGS;
    e->ex->set_bands(bands);
    return AJIB_OK;
}

extern "C" int ajib_exec_info(const ajib_exec *e, size_t *device_bytes, size_t *weight_bytes, int *launches)
{
    if (!e || !e->ex) return AJIB_ERR_ARGS;
    if (device_bytes) *device_bytes = e->ex->device_bytes();
    if (weight_bytes) *weight_bytes = e->ex->weight_bytes();
    if (launches) *launches = e->ex->launches_per_run();
    return AJIB_OK;
}

extern "C" int ajib_exec_profile(ajib_exec *e, int on)
{
    if (!e || !e->ex) return AJIB_ERR_ARGS;
    return e->ex->profile(on != 0);
}

extern "C" int ajib_exec_profile_read(ajib_exec *e, double *ms, int *counts, int nsteps)
{
    if (!e || !e->ex || !ms || !counts || nsteps < 0) return AJIB_ERR_ARGS;
    return e->ex->profile_read(ms, counts, nsteps);
}
