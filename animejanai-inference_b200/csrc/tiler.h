/*
 * tiler.h — the still-image tiler on the GPU (internal; C ABI in include/aji_b200.h).
 *
 * Geometry (host): tile origins with the last tile flush to the far edge, optional even tiles,
 * reflect padding, and per-axis linear blend ramps across a 16-pixel band at the centre of each
 * overlap, normalised so the tiles covering a position sum to one — the reference's cover
 * (src/core/tiling.cpp:17-103). The weights must be bit-identical to the reference's for the
 * output to be, so their float arithmetic follows the same steps.
 *
 * Device: tiles are cut out of the 8-bit image as a batch stacked along H (one launch for all
 * tiles of a batch, fp16 NCHW, the net's input), and after the net the output is composed in one
 * pass: each output pixel gathers the at most few tiles covering it, in the reference's blend
 * order (tile rows, then tiles) with the same separately-rounded multiplies and adds, and is
 * quantised to 8 bits. The reference instead blends each tile into an fp32 band and flushes the
 * band per tile row (src/core/tiling_gpu.cu:98-134); the result is the same, bit for bit, without
 * the band's HBM round trip.
 */
#pragma once

#include <cstdint>
#include <vector>

#include <cuda_runtime.h>

namespace ajib {

constexpr int kTileAlign = 16, kMinTile = 32, kBlendWidth = 16;

std::vector<int> tile_origins(int len, int tile, int overlap);
std::vector<int> even_origins(int n, int max_tile, int overlap, int *tile);
int reflect_index(int i, int n);
// w[t * span * scale + u], span = min(tile, len)
std::vector<float> axis_weights(const std::vector<int> &org, int len, int tile, int scale);

struct TileGeometry {
    int W = 0, H = 0, ci = 0, scale = 1;  // the image, 1 or 3 channels
    int tw = 0, th = 0;                   // tile (input pixels)
    std::vector<int> ox, oy;              // origins
    int nx() const { return (int)ox.size(); }
    int ny() const { return (int)oy.size(); }
    int count() const { return nx() * ny(); }
};

TileGeometry make_geometry(int W, int H, int ci, int scale, int tile_w, int tile_h, int overlap, bool even);
// The tile rows [*j0, *j1] whose outputs cover any of the output rows [Y0, Y1) (Y0 < Y1).
void tile_rows_covering(const TileGeometry &g, int Y0, int Y1, int *j0, int *j1);

// Device tables for one geometry (origins, weights, per-output-pixel covering tile ranges).
class DeviceTiler {
public:
    ~DeviceTiler();
    bool init(const TileGeometry &g);
    const TileGeometry &geometry() const { return g_; }
    // tiles [k0, k0 + n) of img (device, W x H x ci packed) -> dst fp16 [3][n * th][tw]
    cudaError_t extract(const uint8_t *img, int k0, int n, void *dst, cudaStream_t s) const;
    // all tiles' model outputs tiles fp16 [3][count * th * S][tw * S] -> out u8 [H*S][W*S][ci]
    cudaError_t compose(const void *tiles, uint8_t *out, cudaStream_t s) const;
    // output rows [Y0, Y1) into out u8 [Y1 - Y0][W*S][ci], from the outputs of tiles
    // [k0, k0 + ntiles) (fp16 [3][ntiles * th * S][tw * S]), which must hold every tile covering
    // those rows
    cudaError_t compose_rows(const void *tiles, int k0, int ntiles, int Y0, int Y1, uint8_t *out, cudaStream_t s) const;
    size_t table_bytes() const { return bytes_; }

private:
    TileGeometry g_;
    int *d_ox_ = nullptr, *d_oy_ = nullptr;
    float *d_wx_ = nullptr, *d_wy_ = nullptr;
    int2 *d_cx_ = nullptr, *d_cy_ = nullptr;  // per output column / row: first covering tile, count
    size_t bytes_ = 0;
};

}  // namespace ajib
