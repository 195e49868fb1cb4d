/*
 * oracle_colour.c — CPU restatement of the colour passes on the native path (test
 * infrastructure only; see oracle.h): the zimg filter tables of src/resample.h:53-98, the
 * constants of src/resample.h:100-129, and the pre / post / 4:4:4 kernels of
 * src/kernels.cu:89-320 and their runs :441-497, computed unfused (first filter pass into a
 * float plane, second pass from it), one output at a time, in the same fp32 operation order.
 * Multiply-adds that the CUDA compiler fuses are written as fmaf (correctly rounded); this file
 * is compiled with -ffp-contract=off so nothing else is fused.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

enum { FMT_NV12 = 1, FMT_P010 = 2, FMT_444P16 = 3, FMT_444P10 = 5, FMT_444P12 = 6 };
enum { MAT_601 = 1, MAT_709 = 2, MAT_2020 = 3 };
enum { RANGE_FULL = 2 };
enum { SIT_LEFT = 1, SIT_CENTER = 2, SIT_TOPLEFT = 3 };

/* src/resample.h:31-45 (the Spline36 kernel) */
static double spline36(double x)
{
    x = fabs(x);
    if (x < 1.0) return ((13.0 / 11.0 * x - 453.0 / 209.0) * x - 3.0 / 209.0) * x + 1.0;
    if (x < 2.0) {
        x -= 1.0;
        return ((-6.0 / 11.0 * x + 270.0 / 209.0) * x - 156.0 / 209.0) * x;
    }
    if (x < 3.0) {
        x -= 2.0;
        return ((1.0 / 11.0 * x - 45.0 / 209.0) * x + 26.0 / 209.0) * x;
    }
    return 0.0;
}

static double bilinear(double x)
{
    x = fabs(x);
    return x < 1.0 ? 1.0 - x : 0.0;
}

int orc_filter(int src, int dst, double shift, int filter, int *start, float *wt)
{
    const double scale = (double)dst / src;
    const double step = scale < 1.0 ? scale : 1.0;
    const double support = filter == 1 ? 1.0 : 3.0;
    int taps = (int)ceil(support / step) * 2;
    if (taps < 1) taps = 1;
    if (!start || !wt) return taps;
    double row[64];
    if (taps > 64) return -1;
    for (int i = 0; i < dst; i++) {
        const double pos = (i + 0.5) / scale + shift;
        const double begin = floor(pos - taps / 2.0 + 0.5) + 0.5;
        double sum = 0.0;
        for (int j = 0; j < taps; j++) {
            row[j] = filter == 1 ? bilinear((begin + j - pos) * step) : spline36((begin + j - pos) * step);
            sum += row[j];
        }
        start[i] = (int)(begin - 0.5);
        for (int j = 0; j < taps; j++) wt[(size_t)i * taps + j] = (float)(row[j] / sum);
    }
    return taps;
}

/* src/resample.h:89-98 */
void orc_chroma_shift(int siting, int up, double *sx, double *sy)
{
    if (up) {
        *sx = siting == SIT_CENTER ? 0.0 : 0.25;
        *sy = siting == SIT_TOPLEFT ? 0.25 : 0.0;
    } else {
        *sx = siting == SIT_CENTER ? 0.0 : -0.5;
        *sy = siting == SIT_TOPLEFT ? -0.5 : 0.0;
    }
}

static int is444(int f) { return f == FMT_444P16 || f == FMT_444P10 || f == FMT_444P12; }

/* src/resample.h:100-129 */
void orc_make_csp(int format, int matrix, int range, float *csp)
{
    float kr, kb;
    if (matrix == MAT_601) {
        kr = 0.299f;
        kb = 0.114f;
    } else if (matrix == MAT_2020) {
        kr = 0.2627f;
        kb = 0.0593f;
    } else {
        kr = 0.2126f;
        kb = 0.0722f;
    }
    const float m = (format == FMT_P010 || is444(format)) ? 256.0f : 1.0f;
    const float maxraw = (format == FMT_P010 || format == FMT_444P10) ? 65472.0f
                         : format == FMT_444P12                       ? 65520.0f
                         : format == FMT_444P16                       ? 65535.0f
                                                                      : 255.0f;
    csp[0] = kr;
    csp[1] = kb;
    if (range == RANGE_FULL) {
        csp[2] = 0.0f;
        csp[3] = maxraw;
        csp[4] = m == 256.0f ? 32768.0f : 128.0f;
        csp[5] = maxraw;
    } else {
        csp[2] = 16.0f * m;
        csp[3] = 219.0f * m;
        csp[4] = 128.0f * m;
        csp[5] = 224.0f * m;
    }
}

/* src/kernels.cu:89-94 */
static int mirr(int i, int n)
{
    i = i < 0 ? -i - 1 : i;
    i = i >= n ? 2 * n - 1 - i : i;
    return i < 0 ? 0 : i > n - 1 ? n - 1 : i;
}

/* src/kernels.cu:96-99 */
static float quant(float v, float qdiv, float qmax)
{
    return fminf(fmaxf(rintf(v / qdiv), 0.0f), qmax) * qdiv;
}

static float sample_at(const uint8_t *base, ptrdiff_t stride, int y, int x, int bytes)
{
    const uint8_t *row = base + (size_t)y * stride;
    return bytes == 1 ? (float)row[x] : (float)((const uint16_t *)row)[x];
}

/* aji_run_pre (src/kernels.cu:441-465): k_uv_h (:105-128) then k_pre_v_combine (:130-164) */
int orc_pre(int format, int w, int h, int siting, int filter, const void *y_plane, ptrdiff_t ys, const void *uv_plane,
            ptrdiff_t uvs, const float *csp, uint16_t *dst)
{
    if (format != FMT_NV12 && format != FMT_P010) return -1;
    const int cw = w / 2, ch = h / 2, bytes = format == FMT_P010 ? 2 : 1;
    double sx, sy;
    orc_chroma_shift(siting, 1, &sx, &sy);
    const int th = orc_filter(cw, w, sx, filter, 0, 0), tv = orc_filter(ch, h, sy, filter, 0, 0);
    int *hs = malloc(sizeof(int) * w), *vs = malloc(sizeof(int) * h);
    float *hw = malloc(sizeof(float) * w * th), *vw = malloc(sizeof(float) * h * tv);
    float *tmp = malloc(sizeof(float) * 2 * (size_t)w * ch);
    if (!hs || !vs || !hw || !vw || !tmp) return -1;
    orc_filter(cw, w, sx, filter, hs, hw);
    orc_filter(ch, h, sy, filter, vs, vw);
    const size_t tplane = (size_t)w * ch;
    for (int y = 0; y < ch; y++)
        for (int x = 0; x < w; x++) {
            float u = 0.0f, v = 0.0f;
            for (int j = 0; j < th; j++) {
                const int sxi = mirr(hs[x] + j, cw);
                u = fmaf(hw[(size_t)x * th + j], sample_at(uv_plane, uvs, y, 2 * sxi, bytes), u);
                v = fmaf(hw[(size_t)x * th + j], sample_at(uv_plane, uvs, y, 2 * sxi + 1, bytes), v);
            }
            tmp[(size_t)y * w + x] = u;
            tmp[tplane + (size_t)y * w + x] = v;
        }
    const float kr = csp[0], kb = csp[1], yoff = csp[2], yscale = csp[3], coff = csp[4], cscale = csp[5];
    const float kg = 1.0f - kr - kb;
    const size_t plane = (size_t)w * h;
    for (int y = 0; y < h; y++)
        for (int x = 0; x < w; x++) {
            float u = 0.0f, v = 0.0f;
            for (int j = 0; j < tv; j++) {
                const size_t pos = (size_t)mirr(vs[y] + j, ch) * w + x;
                u = fmaf(vw[(size_t)y * tv + j], tmp[pos], u);
                v = fmaf(vw[(size_t)y * tv + j], tmp[tplane + pos], v);
            }
            const float Y = (sample_at(y_plane, ys, y, x, bytes) - yoff) / yscale;
            const float U = (u - coff) / cscale;
            const float V = (v - coff) / cscale;
            const float r = fmaf(2.0f * (1.0f - kr), V, Y);
            const float b = fmaf(2.0f * (1.0f - kb), U, Y);
            const float g = Y - fmaf(2.0f * kb * (1.0f - kb), U, 2.0f * kr * (1.0f - kr) * V) / kg;
            const size_t idx = (size_t)y * w + x;
            dst[idx] = orc_f2h(r);
            dst[plane + idx] = orc_f2h(g);
            dst[2 * plane + idx] = orc_f2h(b);
        }
    free(hs);
    free(vs);
    free(hw);
    free(vw);
    free(tmp);
    return 0;
}

static void put_sample(uint8_t *base, ptrdiff_t stride, int y, int x, int bytes, float v)
{
    uint8_t *row = base + (size_t)y * stride;
    if (bytes == 1)
        row[x] = (uint8_t)v;
    else
        ((uint16_t *)row)[x] = (uint16_t)v;
}

/* aji_run_post (src/kernels.cu:467-497): k_post_matrix (:170-190), k_h_f32 (:193-207),
 * k_uv_v_store (:211-231); output siting as given (the video path always passes left). */
int orc_post(int format, int w, int h, int siting, int filter, const uint16_t *src, const float *csp, void *y_plane,
             ptrdiff_t ys, void *uv_plane, ptrdiff_t uvs)
{
    if (format != FMT_NV12 && format != FMT_P010) return -1;
    const int cw = w / 2, ch = h / 2, bytes = format == FMT_P010 ? 2 : 1;
    const float qdiv = format == FMT_P010 ? 64.0f : 1.0f, qmax = format == FMT_P010 ? 1023.0f : 255.0f;
    double sx, sy;
    orc_chroma_shift(siting, 0, &sx, &sy);
    const int th = orc_filter(w, cw, sx, filter, 0, 0), tv = orc_filter(h, ch, sy, filter, 0, 0);
    int *hs = malloc(sizeof(int) * cw), *vs = malloc(sizeof(int) * ch);
    float *hw = malloc(sizeof(float) * cw * th), *vw = malloc(sizeof(float) * ch * tv);
    float *t0 = malloc(sizeof(float) * 2 * (size_t)w * h), *t1 = malloc(sizeof(float) * 2 * (size_t)cw * h);
    if (!hs || !vs || !hw || !vw || !t0 || !t1) return -1;
    orc_filter(w, cw, sx, filter, hs, hw);
    orc_filter(h, ch, sy, filter, vs, vw);
    const float kr = csp[0], kb = csp[1], yoff = csp[2], yscale = csp[3], coff = csp[4], cscale = csp[5];
    const size_t plane = (size_t)w * h;
    for (int y = 0; y < h; y++)
        for (int x = 0; x < w; x++) {
            const size_t idx = (size_t)y * w + x;
            const float r = orc_h2f(src[idx]), g = orc_h2f(src[plane + idx]), b = orc_h2f(src[2 * plane + idx]);
            const float Y = fmaf(kb, b, fmaf(kr, r, (1.0f - kr - kb) * g));
            put_sample(y_plane, ys, y, x, bytes, quant(fmaf(Y, yscale, yoff), qdiv, qmax));
            t0[idx] = (b - Y) / (2.0f * (1.0f - kb));
            t0[plane + idx] = (r - Y) / (2.0f * (1.0f - kr));
        }
    for (int z = 0; z < 2; z++)
        for (int y = 0; y < h; y++)
            for (int x = 0; x < cw; x++) {
                float a = 0.0f;
                for (int j = 0; j < th; j++)
                    a = fmaf(hw[(size_t)x * th + j], t0[(size_t)z * plane + (size_t)y * w + mirr(hs[x] + j, w)], a);
                t1[(size_t)z * cw * h + (size_t)y * cw + x] = a;
            }
    const size_t p1 = (size_t)cw * h;
    for (int y = 0; y < ch; y++)
        for (int x = 0; x < cw; x++) {
            float u = 0.0f, v = 0.0f;
            for (int j = 0; j < tv; j++) {
                const size_t row = (size_t)mirr(vs[y] + j, h) * cw + x;
                u = fmaf(vw[(size_t)y * tv + j], t1[row], u);
                v = fmaf(vw[(size_t)y * tv + j], t1[p1 + row], v);
            }
            put_sample(uv_plane, uvs, y, 2 * x, bytes, quant(fmaf(u, cscale, coff), qdiv, qmax));
            put_sample(uv_plane, uvs, y, 2 * x + 1, bytes, quant(fmaf(v, cscale, coff), qdiv, qmax));
        }
    free(hs);
    free(vs);
    free(hw);
    free(vw);
    free(t0);
    free(t1);
    return 0;
}

/* aji_run_post444 (src/kernels.cu:235-280) */
int orc_post444(int format, int w, int h, const uint16_t *src, const float *csp, uint16_t *yp, uint16_t *cbp,
                uint16_t *crp)
{
    const float qdiv = format == FMT_444P10 ? 64.0f : format == FMT_444P12 ? 16.0f : 1.0f;
    const float qmax = format == FMT_444P10 ? 1023.0f : format == FMT_444P12 ? 4095.0f : 65535.0f;
    const float kr = csp[0], kb = csp[1], yoff = csp[2], yscale = csp[3], coff = csp[4], cscale = csp[5];
    const size_t plane = (size_t)w * h;
    for (size_t idx = 0; idx < plane; idx++) {
        const float r = orc_h2f(src[idx]), g = orc_h2f(src[plane + idx]), b = orc_h2f(src[2 * plane + idx]);
        const float Y = fmaf(kb, b, fmaf(kr, r, (1.0f - kr - kb) * g));
        const float U = (b - Y) / (2.0f * (1.0f - kb));
        const float V = (r - Y) / (2.0f * (1.0f - kr));
        yp[idx] = (uint16_t)quant(fmaf(Y, yscale, yoff), qdiv, qmax);
        cbp[idx] = (uint16_t)quant(fmaf(U, cscale, coff), qdiv, qmax);
        crp[idx] = (uint16_t)quant(fmaf(V, cscale, coff), qdiv, qmax);
    }
    return 0;
}

/* aji_run_pre444 (src/kernels.cu:282-320) */
int orc_pre444(int w, int h, const uint16_t *yp, const uint16_t *cbp, const uint16_t *crp, const float *csp,
               uint16_t *dst)
{
    const float kr = csp[0], kb = csp[1], yoff = csp[2], yscale = csp[3], coff = csp[4], cscale = csp[5];
    const float kg = 1.0f - kr - kb;
    const size_t plane = (size_t)w * h;
    for (size_t idx = 0; idx < plane; idx++) {
        const float Y = ((float)yp[idx] - yoff) / yscale;
        const float U = ((float)cbp[idx] - coff) / cscale;
        const float V = ((float)crp[idx] - coff) / cscale;
        dst[idx] = orc_f2h(fmaf(2.0f * (1.0f - kr), V, Y));
        dst[2 * plane + idx] = orc_f2h(fmaf(2.0f * (1.0f - kb), U, Y));
        dst[plane + idx] = orc_f2h(Y - fmaf(2.0f * kb * (1.0f - kb), U, 2.0f * kr * (1.0f - kr) * V) / kg);
    }
    return 0;
}

/* src/kernels.cu:322-354 + :416-431, :499-508 (aji_resize_plan_create / aji_run_resize): Spline36
 * resize of fp16 NCHW RGB [3][sh][sw] (bits) -> [3][dh][dw] (bits). Horizontal pass into an fp32
 * plane, vertical pass, each sum accumulated as fmaf(weight, sample, sum) in tap order (the CUDA
 * compiler contracts the reference's a += w * x), one rounding to fp16. Returns 0 or -1. */
int orc_resize(const uint16_t *src, int sw, int sh, int dw, int dh, uint16_t *dst)
{
    if (!src || !dst || sw < 1 || sh < 1 || dw < 1 || dh < 1) return -1;
    const int th = orc_filter(sw, dw, 0.0, 0, 0, 0), tv = orc_filter(sh, dh, 0.0, 0, 0, 0);
    int *hs = malloc(sizeof(int) * dw), *vs = malloc(sizeof(int) * dh);
    float *hw = malloc(sizeof(float) * (size_t)dw * th), *vw = malloc(sizeof(float) * (size_t)dh * tv);
    float *tmp = malloc(sizeof(float) * (size_t)3 * dw * sh);
    if (!hs || !vs || !hw || !vw || !tmp) return -1;
    orc_filter(sw, dw, 0.0, 0, hs, hw);
    orc_filter(sh, dh, 0.0, 0, vs, vw);
    for (int c = 0; c < 3; c++)
        for (int y = 0; y < sh; y++)
            for (int x = 0; x < dw; x++) {
                float a = 0.0f;
                for (int j = 0; j < th; j++)
                    a = fmaf(hw[(size_t)x * th + j], orc_h2f(src[((size_t)c * sh + y) * sw + mirr(hs[x] + j, sw)]), a);
                tmp[((size_t)c * sh + y) * dw + x] = a;
            }
    for (int c = 0; c < 3; c++)
        for (int y = 0; y < dh; y++)
            for (int x = 0; x < dw; x++) {
                float a = 0.0f;
                for (int j = 0; j < tv; j++)
                    a = fmaf(vw[(size_t)y * tv + j], tmp[((size_t)c * sh + mirr(vs[y] + j, sh)) * dw + x], a);
                dst[((size_t)c * dh + y) * dw + x] = orc_f2h(a);
            }
    free(hs);
    free(vs);
    free(hw);
    free(vw);
    free(tmp);
    return 0;
}
