/*
 * oracle_tiling.c — CPU restatement of the reference's still-image tiler (test infrastructure
 * only; see oracle.h): src/core/tiling.cpp:17-103 (tile_origins, even_origins, reflect,
 * axis_weights) and :115-289 (upscale_tiled) with the model as a callback. Float arithmetic as
 * the reference host path: separate multiplies and adds (this file is compiled with
 * -ffp-contract=off), blend in tile-row-major, tile-minor order into a float band, 8-bit output
 * as (uint8)(v * 255 + 0.5) clamped.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

enum { TILE_ALIGN = 16, MIN_TILE = 32, BLEND_WIDTH = 16 };

static int imin(int a, int b) { return a < b ? a : b; }
static int imax(int a, int b) { return a > b ? a : b; }

/* src/core/tiling.cpp:17-30 */
int orc_tile_origins(int len, int tile, int overlap, int *out, int max)
{
    if (len <= tile) {
        if (max > 0) out[0] = 0;
        return 1;
    }
    const int step = imax(1, tile - overlap);
    const int n = imax(1, (len - overlap + step - 1) / step);
    int k = 0, last = -1;
    for (int i = 0; i < n; i++) {
        const int p = imin(i * step, len - tile);
        if (k == 0 || p != last) {
            if (k < max) out[k] = p;
            k++;
            last = p;
        }
    }
    return k;
}

/* src/core/tiling.cpp:32-55 */
int orc_even_origins(int n, int max_tile, int overlap, int *tile, int *out, int max)
{
    const int T = max_tile / TILE_ALIGN * TILE_ALIGN;
    if (T < MIN_TILE) {
        *tile = max_tile;
        return orc_tile_origins(n, max_tile, overlap, out, max);
    }
    if (n <= T) {
        const int up = (n + TILE_ALIGN - 1) / TILE_ALIGN * TILE_ALIGN;
        *tile = imax(MIN_TILE, up);
        if (max > 0) out[0] = 0;
        return 1;
    }
    const int O = imax(0, imin(overlap, T / 2));
    for (int k = imax(2, (n - O + (T - O) - 1) / (T - O));; k++) {
        const int want = (n + (k - 1) * O + k - 1) / k;
        const int t = imax(MIN_TILE, (want + TILE_ALIGN - 1) / TILE_ALIGN * TILE_ALIGN);
        if (t > T) continue;
        for (int i = 0; i < k && i < max; i++) out[i] = (int)((long long)i * (n - t) / (k - 1));
        *tile = t;
        return k;
    }
}

/* src/core/tiling.cpp:57-66 */
int orc_reflect(int i, int n)
{
    if (n == 1) return 0;
    const int period = 2 * (n - 1);
    i %= period;
    if (i < 0) i += period;
    return i < n ? i : period - i;
}

/* src/core/tiling.cpp:68-103: w[t * span * scale + u] */
int orc_axis_weights(const int *org, int n, int len, int tile, int scale, float *w)
{
    const int span = imin(tile, len), S = span * scale;
    for (int t = 0; t < n; t++) {
        const int ol = t > 0 ? (org[t - 1] + span - org[t]) * scale : 0;
        const int orr = t + 1 < n ? (org[t] + span - org[t + 1]) * scale : 0;
        const int bl = imin(ol, BLEND_WIDTH * scale), br = imin(orr, BLEND_WIDTH * scale);
        const int l0 = (ol - bl) / 2, r0 = (orr - br) / 2;
        for (int u = 0; u < S; u++) {
            float v = 1.0f;
            if (u < ol) v = fminf(v, u < l0 ? 0.0f : (u - l0 + 0.5f) / bl);
            if (u >= S - orr) {
                const int d = S - u - 1;
                v = fminf(v, d < r0 ? 0.0f : (d - r0 + 0.5f) / br);
            }
            w[(size_t)t * S + u] = fminf(v, 1.0f);
        }
    }
    float *sum = calloc((size_t)len * scale, sizeof(float));
    if (!sum) return -1;
    for (int t = 0; t < n; t++)
        for (int u = 0; u < S; u++) sum[(size_t)org[t] * scale + u] += w[(size_t)t * S + u];
    for (int t = 0; t < n; t++)
        for (int u = 0; u < S; u++) w[(size_t)t * S + u] /= sum[(size_t)org[t] * scale + u];
    free(sum);
    return n * S;
}

static uint8_t to_u8(float v)
{
    const float f = v * 255.0f + 0.5f;
    return f <= 0.0f ? 0 : f >= 255.0f ? 255 : (uint8_t)f;
}

/* src/core/tiling.cpp:115-289 for a 3-channel model: run(opaque, in [3][th][tw], out
 * [3][th*s][tw*s]) returns 0 on success. in / out: interleaved 8-bit images, ci == co in {1, 3},
 * strides in bytes. even != 0 takes the even-tile origins and tile sides of the GPU image path
 * (src/aji_img_trt.cpp:899-916; tw / th are then the largest tile, and the tiles passed to run
 * have the sides orc_even_origins returns). Returns 0, -2 for bad arguments, or the model's error. */
int orc_upscale_tiled(int (*run)(void *opaque, const float *in, float *out), void *opaque, int tw, int th, int s,
                      int overlap, int even, const uint8_t *in, int W, int H, int ci, ptrdiff_t in_stride,
                      uint8_t *out, ptrdiff_t out_stride)
{
    if (!in || !out || W < 1 || H < 1 || (ci != 1 && ci != 3) || s < 1) return -2;
    const int co = ci;
    int ox[4096], oy[4096], nx, ny;
    if (even) {
        nx = orc_even_origins(W, tw, overlap, &tw, ox, 4096);
        ny = orc_even_origins(H, th, overlap, &th, oy, 4096);
    } else {
        nx = orc_tile_origins(W, tw, overlap, ox, 4096);
        ny = orc_tile_origins(H, th, overlap, oy, 4096);
    }
    if (nx > 4096 || ny > 4096) return -2;
    const int spw = imin(tw, W), sph = imin(th, H), OW = W * s, OH = H * s;
    const int tow = tw * s, toh = th * s, band_rows = sph * s;
    const size_t in_plane = (size_t)tw * th, out_plane = (size_t)tow * toh;
    float *wx = malloc(sizeof(float) * (size_t)nx * spw * s), *wy = malloc(sizeof(float) * (size_t)ny * sph * s);
    float *tin = malloc(sizeof(float) * in_plane * 3), *tout = malloc(sizeof(float) * out_plane * 3);
    float *band = calloc((size_t)co * band_rows * OW, sizeof(float));
    if (!wx || !wy || !tin || !tout || !band) return -5;
    orc_axis_weights(ox, nx, W, tw, s, wx);
    orc_axis_weights(oy, ny, H, th, s, wy);
    const float inv255 = 1.0f / 255.0f;
    int band_y0 = 0, rc = 0;
    for (int j = 0; j < ny && !rc; j++) {
        for (int i = 0; i < nx && !rc; i++) {
            for (int y = 0; y < th; y++) {
                const uint8_t *row = in + (ptrdiff_t)orc_reflect(oy[j] + y, H) * in_stride;
                for (int x = 0; x < tw; x++) {
                    const uint8_t *p = row + (size_t)orc_reflect(ox[i] + x, W) * ci;
                    const int g = ci == 1;
                    tin[(size_t)y * tw + x] = p[0] * inv255;
                    tin[(size_t)y * tw + x + in_plane] = p[g ? 0 : 1] * inv255;
                    tin[(size_t)y * tw + x + 2 * in_plane] = p[g ? 0 : 2] * inv255;
                }
            }
            rc = run(opaque, tin, tout);
            if (rc) break;
            const int ux0 = ox[i] * s, uy0 = oy[j] * s, vrows = sph * s, cols = spw * s;
            const float *wxi = wx + (size_t)i * spw * s, *wyj = wy + (size_t)j * sph * s;
            for (int c = 0; c < co; c++)
                for (int v = 0; v < vrows; v++) {
                    const int mc = co == 1 ? 0 : c;
                    const float *srow = tout + mc * out_plane + (size_t)v * tow;
                    const float wv = wyj[v];
                    const int r = (uy0 + v) % band_rows;
                    float *brow = band + ((size_t)c * band_rows + r) * OW + ux0;
                    for (int u = 0; u < cols; u++) brow[u] += wv * wxi[u] * srow[u];
                }
        }
        if (rc) break;
        const int next_y0 = j + 1 < ny ? oy[j + 1] * s : OH;
        for (int Y = band_y0; Y < next_y0; Y++) {
            uint8_t *orow = out + (ptrdiff_t)Y * out_stride;
            const int r = Y % band_rows;
            for (int c = 0; c < co; c++) {
                float *b = band + ((size_t)c * band_rows + r) * OW;
                for (int X = 0; X < OW; X++) {
                    orow[(size_t)X * co + c] = to_u8(b[X]);
                    b[X] = 0.0f;
                }
            }
        }
        band_y0 = next_y0;
    }
    free(wx);
    free(wy);
    free(tin);
    free(tout);
    free(band);
    return rc;
}
