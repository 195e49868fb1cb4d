// tiler_geom.cpp — host tile geometry (see tiler.h). Restates src/core/tiling.cpp:17-103 of the
// reference step for step: the blend weights must come out bit-identical. Compiled without
// floating-point contraction.
#include <algorithm>

#include "tiler.h"

namespace ajib {

std::vector<int> tile_origins(int len, int tile, int overlap)
{
    if (len <= tile) return {0};
    const int step = std::max(1, tile - overlap);
    const int n = std::max(1, (len - overlap + step - 1) / step);
    std::vector<int> o;
    for (int i = 0; i < n; i++) {
        const int p = std::min(i * step, len - tile);
        if (o.empty() || p != o.back()) o.push_back(p);
    }
    return o;
}

std::vector<int> even_origins(int n, int max_tile, int overlap, int *tile)
{
    const auto up = [](int v) { return (v + kTileAlign - 1) / kTileAlign * kTileAlign; };
    const int T = max_tile / kTileAlign * kTileAlign;
    if (T < kMinTile) {
        *tile = max_tile;
        return tile_origins(n, max_tile, overlap);
    }
    if (n <= T) {
        *tile = std::max(kMinTile, up(n));
        return {0};
    }
    const int O = std::max(0, std::min(overlap, T / 2));
    for (int k = std::max(2, (n - O + (T - O) - 1) / (T - O));; k++) {
        const int t = std::max(kMinTile, up((n + (k - 1) * O + k - 1) / k));
        if (t > T) continue;
        std::vector<int> o;
        for (int i = 0; i < k; i++) o.push_back((int)((long long)i * (n - t) / (k - 1)));
        *tile = t;
        return o;
    }
}

int reflect_index(int i, int n)
{
    if (n == 1) return 0;
    const int period = 2 * (n - 1);
    i %= period;
    if (i < 0) i += period;
    return i < n ? i : period - i;
}

std::vector<float> axis_weights(const std::vector<int> &org, int len, int tile, int scale)
{
    const int span = std::min(tile, len), n = (int)org.size(), S = span * scale;
    std::vector<float> w((size_t)n * S, 1.0f);
    for (int t = 0; t < n; t++) {
        const int ol = t > 0 ? (org[t - 1] + span - org[t]) * scale : 0;
        const int orr = t + 1 < n ? (org[t] + span - org[t + 1]) * scale : 0;
        const int bl = std::min(ol, kBlendWidth * scale), br = std::min(orr, kBlendWidth * scale);
        const int l0 = (ol - bl) / 2, r0 = (orr - br) / 2;
        for (int u = 0; u < S; u++) {
            float v = 1.0f;
            if (u < ol) v = std::min(v, u < l0 ? 0.0f : (u - l0 + 0.5f) / bl);
            if (u >= S - orr) {
                const int d = S - u - 1;
                v = std::min(v, d < r0 ? 0.0f : (d - r0 + 0.5f) / br);
            }
            w[(size_t)t * S + u] = std::min(v, 1.0f);
        }
    }
    std::vector<float> sum((size_t)len * scale, 0.0f);
    for (int t = 0; t < n; t++)
        for (int u = 0; u < S; u++) sum[(size_t)org[t] * scale + u] += w[(size_t)t * S + u];
    for (int t = 0; t < n; t++)
        for (int u = 0; u < S; u++) w[(size_t)t * S + u] /= sum[(size_t)org[t] * scale + u];
    return w;
}

TileGeometry make_geometry(int W, int H, int ci, int scale, int tile_w, int tile_h, int overlap, bool even)
{
    TileGeometry g;
    g.W = W;
    g.H = H;
    g.ci = ci;
    g.scale = scale;
    if (even) {
        g.ox = even_origins(W, tile_w, overlap, &g.tw);
        g.oy = even_origins(H, tile_h, overlap, &g.th);
    } else {
        g.tw = tile_w;
        g.th = tile_h;
        g.ox = tile_origins(W, tile_w, overlap);
        g.oy = tile_origins(H, tile_h, overlap);
    }
    return g;
}

void tile_rows_covering(const TileGeometry &g, int Y0, int Y1, int *j0, int *j1)
{
    const int s = g.scale, span = std::min(g.th, g.H);
    *j0 = g.ny();
    *j1 = -1;
    for (int j = 0; j < g.ny(); j++)
        if (g.oy[j] * s < Y1 && (g.oy[j] + span) * s > Y0) {
            *j0 = std::min(*j0, j);
            *j1 = std::max(*j1, j);
        }
}

}  // namespace ajib
