// reftiling_shim.cpp — C entry points over the reference's CPU tiler (src/core/tiling.cpp:
// tile_origins, even_origins, reflect, axis_weights, upscale_tiled) with the reference test's mock
// models (sanity/tiling_test.cpp: Nearest pixel replication, Constant), compiled from the
// reference sources by build.sh into oracle/_ref/libref_tiling.so. Test infrastructure only.
#include <cstring>
#include <string>
#include <vector>

#include "tiling.h"

using namespace ajicore;

extern "C" int ref_tile_origins(int len, int tile, int overlap, int *out, int max)
{
    const std::vector<int> o = tile_origins(len, tile, overlap);
    for (size_t i = 0; i < o.size() && (int)i < max; i++) out[i] = o[i];
    return (int)o.size();
}

extern "C" int ref_even_origins(int n, int max_tile, int overlap, int *tile, int *out, int max)
{
    const std::vector<int> o = even_origins(n, max_tile, overlap, tile);
    for (size_t i = 0; i < o.size() && (int)i < max; i++) out[i] = o[i];
    return (int)o.size();
}

extern "C" int ref_reflect(int i, int n) { return reflect(i, n); }

// weights of all tiles concatenated: out[t * span * scale + u]
extern "C" int ref_axis_weights(const int *org, int n, int len, int tile, int scale, float *out)
{
    const std::vector<int> o(org, org + n);
    const auto w = axis_weights(o, len, tile, scale);
    size_t k = 0;
    for (const auto &row : w)
        for (float v : row) out[k++] = v;
    return (int)k;
}

namespace {
// A tile model the host drives: kind 0 nearest replication, 1 constant, 2 a callback.
typedef void (*tile_fn)(void *opaque, const float *in, float *out, int tw, int th, int scale);
class Mock : public TileModel {
public:
    int kind = 0;
    float value = 0.6f;
    tile_fn fn = nullptr;
    void *opaque = nullptr;
    int run_tile(const float *in, float *out, std::string *) override
    {
        const int s = scale, ow = tile_w * s, oh = tile_h * s;
        if (kind == 2) {
            fn(opaque, in, out, tile_w, tile_h, s);
            return AJI_IMG_OK;
        }
        for (int c = 0; c < out_ch; c++)
            for (int y = 0; y < oh; y++)
                for (int x = 0; x < ow; x++)
                    out[((size_t)c * oh + y) * ow + x] =
                        kind == 1 ? value : in[((size_t)(in_ch == 1 ? 0 : c) * tile_h + y / s) * tile_w + x / s];
        return AJI_IMG_OK;
    }
};
}  // namespace

extern "C" int ref_upscale_tiled(int kind, float value, tile_fn fn, void *opaque, int tile_w, int tile_h, int scale,
                                 int overlap, const uint8_t *in, int w, int h, int ch, uint8_t *out)
{
    Mock m;
    m.kind = kind;
    m.value = value;
    m.fn = fn;
    m.opaque = opaque;
    m.tile_w = tile_w;
    m.tile_h = tile_h;
    m.scale = scale;
    aji_img_buffer bi{w, h, ch, (ptrdiff_t)w * ch, const_cast<uint8_t *>(in)};
    aji_img_buffer bo{w * scale, h * scale, ch, (ptrdiff_t)w * scale * ch, out};
    std::string err;
    return upscale_tiled(m, overlap, &bi, &bo, nullptr, nullptr, &err);
}
