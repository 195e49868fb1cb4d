// tiler_api.cpp — C ABI over the GPU tiler (include/aji_b200.h, ajib_tiler_*).
#include <memory>
#include <new>

#include "tiler.h"
#include "../../include/aji_b200.h"

struct ajib_tiler {
    ajib::DeviceTiler t;
};

extern "C" int ajib_tiler_create(int W, int H, int ci, int scale, int tile_w, int tile_h, int overlap, int even,
                                 ajib_tiler **out)
{
    if (!out || W < 1 || H < 1 || (ci != 1 && ci != 3) || scale < 1 || tile_w < 1 || tile_h < 1 || overlap < 0)
        return AJIB_ERR_ARGS;
    *out = nullptr;
    auto *t = new (std::nothrow) ajib_tiler();
    if (!t) return AJIB_ERR_NO_MEM;
    if (!t->t.init(ajib::make_geometry(W, H, ci, scale, tile_w, tile_h, overlap, even != 0))) {
        delete t;
        return AJIB_ERR_CUDA;
    }
    *out = t;
    return AJIB_OK;
}

extern "C" int ajib_tiler_info(const ajib_tiler *t, int *nx, int *ny, int *tw, int *th)
{
    if (!t) return AJIB_ERR_ARGS;
    const ajib::TileGeometry &g = t->t.geometry();
    if (nx) *nx = g.nx();
    if (ny) *ny = g.ny();
    if (tw) *tw = g.tw;
    if (th) *th = g.th;
    return AJIB_OK;
}

extern "C" int ajib_tiler_extract(ajib_tiler *t, const uint8_t *img, int k0, int n, void *dst, void *stream)
{
    if (!t || !img || !dst || k0 < 0 || n < 1 || k0 + n > t->t.geometry().count()) return AJIB_ERR_ARGS;
    return t->t.extract(img, k0, n, dst, (cudaStream_t)stream) == cudaSuccess ? AJIB_OK : AJIB_ERR_CUDA;
}

extern "C" int ajib_tiler_compose(ajib_tiler *t, const void *tiles, uint8_t *out, void *stream)
{
    if (!t || !tiles || !out) return AJIB_ERR_ARGS;
    return t->t.compose(tiles, out, (cudaStream_t)stream) == cudaSuccess ? AJIB_OK : AJIB_ERR_CUDA;
}

extern "C" void ajib_tiler_release(ajib_tiler **t)
{
    if (!t || !*t) return;
    delete *t;
    *t = nullptr;
}
