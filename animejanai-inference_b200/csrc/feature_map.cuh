/*
 * feature_map.cuh — the strip-chunked layout of the feature maps between conv steps (device
 * helpers shared by the conv, concat and colour kernels).
 *
 * Each row of a C-channel map (C a multiple of 8) is cut into strips of 128 pixels, and each
 * (row, strip) is one contiguous block of C/8 chunks of 130 columns of 8 fp16 channels: the
 * strip's pixels and a halo column on each side holding a copy of the neighbouring strip's edge
 * pixel (zero at the image's edges and past the width). A conv's staged input row is then one
 * contiguous bulk copy.
 */
#pragma once

#include <cuda_fp16.h>

#include <cstddef>
#include <cstdint>

namespace ajib {

constexpr int kTileM = 128;  // pixels per strip (the conv MMA's M)

// Strip-chunked feature maps: 128-pixel strips per row, and columns per strip (the strip and a
// halo column on each side).
constexpr int kStripW = kTileM + 2;
__host__ __device__ constexpr int feature_strips(int W) { return (W + kTileM - 1) / kTileM; }

// Half index of column u (0 .. 129) of chunk `chunk` of strip `strip` of row y in a map of cc
// chunks and nstrips strips per row.
__device__ __forceinline__ size_t map_at(int y, int strip, int chunk, int u, int nstrips, int cc)
{
    return ((((size_t)y * nstrips + strip) * cc + chunk) * kStripW + u) * 8;
}

// Store one pixel's 8-channel chunk (pixel x < W of row y) at its column and, at a strip edge, into
// the neighbouring strip's halo column.
__device__ __forceinline__ void store_px(__half *map, int y, int x, int chunk, int nstrips, int cc, uint4 v)
{
    const int s = x >> 7, u = (x & (kTileM - 1)) + 1;
    *reinterpret_cast<uint4 *>(map + map_at(y, s, chunk, u, nstrips, cc)) = v;
    if (u == 1 && s > 0) *reinterpret_cast<uint4 *>(map + map_at(y, s - 1, chunk, kStripW - 1, nstrips, cc)) = v;
    if (u == kTileM && s + 1 < nstrips) *reinterpret_cast<uint4 *>(map + map_at(y, s + 1, chunk, 0, nstrips, cc)) = v;
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b)
{
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

}  // namespace ajib
