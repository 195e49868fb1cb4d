// reftiling_gpu_shim.cu — C entry points over the reference's GPU tiler kernels
// (src/core/tiling_gpu.cu: gpu_tile_extract, gpu_tile_blend, gpu_band_flush), compiled for sm_100a
// from the reference sources by build.sh into oracle/_ref/libref_tiling_gpu.so: the bit-exact
// checker of this engine's tiler kernels. Test infrastructure only.
#include <cstdint>

#include "tiling_gpu.h"

using namespace ajicore;

extern "C" int ref_tile_extract_f16(const uint8_t *img, int W, int H, int ci, int ox, int oy, int tw, int th,
                                    void *dst, void *stream)
{
    return (int)gpu_tile_extract(img, W, H, ci, ox, oy, tw, th, 3, 1.0f / 255.0f, dst, GpuDtype::F16, (cudaStream_t)stream);
}

extern "C" int ref_tile_blend_f16(const void *tile, int tow, int toh, const float *wx, const float *wy, int cols,
                                  int rows, int ux0, int uy0, float *band, int co, int band_rows, int OW, void *stream)
{
    return (int)gpu_tile_blend(tile, GpuDtype::F16, 3, tow, toh, wx, wy, cols, rows, ux0, uy0, band, co, band_rows, OW,
                               (cudaStream_t)stream);
}

extern "C" int ref_band_flush(float *band, int co, int band_rows, int OW, int y0, int n, uint8_t *dst, void *stream)
{
    return (int)gpu_band_flush(band, co, band_rows, OW, y0, n, dst, (cudaStream_t)stream);
}
