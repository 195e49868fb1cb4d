/*
 * oracle_conv.c — the CPU reference net of the native conv path (test infrastructure only; see
 * oracle.h). Restates sanity/native_ref.h:24-122 (ajiref::run_plan) step by step: every
 * product in fp32, accumulated in double from the bias, activations and gates in fp32, each
 * stored feature map rounded to fp16 as the GPU kernels store it.
 */
#include "oracle.h"

#include <math.h>
#include <string.h>
#include "par.h"

/* src/native/pack.cpp:69-92 (float_to_half_bits): round to nearest even, overflow to inf */
uint16_t orc_f2h(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
    if (ax < 0x38800000u) {
        if (ax < 0x33000000u) return (uint16_t)sign;
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const int shift = 126 - (int)(ax >> 23);
        uint32_t r = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1u))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t r = (ax - 0x38000000u) >> 13;
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    return (uint16_t)(sign | r);
}

/* src/native/pack.cpp:94-111 (half_bits_to_float) */
float orc_h2f(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {
            const float f = ldexpf((float)m, -24);
            memcpy(&x, &f, 4);
            x |= sign;
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

static inline float f16r(float x) { return orc_h2f(orc_f2h(x)); }

void orc_round_f16(float *x, size_t n)
{
    for (size_t i = 0; i < n; i++) x[i] = f16r(x[i]);
}
void orc_f2h_array(const float *x, uint16_t *out, size_t n)
{
    for (size_t i = 0; i < n; i++) out[i] = orc_f2h(x[i]);
}
void orc_h2f_array(const uint16_t *h, float *out, size_t n)
{
    for (size_t i = 0; i < n; i++) out[i] = orc_h2f(h[i]);
}

static inline float input_at(int in_mode, const float *src, int H, int W, int cin, int y, int x, int c)
{
    if (y < 0 || y >= H || x < 0 || x >= W) return 0.f;  /* pad 1 with zeros */
    if (in_mode == 0) return src[((size_t)y * W + x) * cin + c];
    if (in_mode == 1) return src[((size_t)c * H + y) * W + x];  /* NCHW model input */
    /* the model input [3][2H][2W] pixel-unshuffled by 2: channel c = cc * 4 + ry * 2 + rx
     * (sanity/native_ref.h:66-67) */
    const int cc = c / 4, ry = (c / 2) % 2, rx = c % 2;
    return src[((size_t)cc * 2 * H + 2 * y + ry) * 2 * W + 2 * x + rx];
}

struct conv_job {
    int in_mode, H, W, cin, cout, act, gate, R, out_clamp;
    const float *src, *w, *bias, *slope, *resid, *att_w, *att_bias, *model_in;
    float *dst;
};

static void conv_row(void *ctx, int y)
{
    const struct conv_job *j = (const struct conv_job *)ctx;
    const int H = j->H, W = j->W, cin = j->cin, cout = j->cout, R = j->R;
    const int OW = R * W, OH = R * H;
    double acc[256];
    for (int x = 0; x < W; x++) {
        for (int n = 0; n < cout; n++) acc[n] = j->bias[n];
        for (int t = 0; t < 9; t++)
            for (int c = 0; c < cin; c++) {
                const float v = input_at(j->in_mode, j->src, H, W, cin, y + t / 3 - 1, x + t % 3 - 1, c);
                if (v == 0.f) continue;
                const float *wr = j->w + ((size_t)t * cin + c) * cout;
                for (int n = 0; n < cout; n++) acc[n] += (double)v * wr[n];
            }
        const size_t p = (size_t)y * W + x;
        float o[256];
        for (int n = 0; n < cout; n++) {
            float v = (float)acc[n];
            if (j->act == 1) v = fmaxf(v, 0.f);
            if (j->act == 2) v = v >= 0.f ? v : v * j->slope[n];
            if (j->act == 3) v = v / (1.f + expf(-v));
            o[n] = v;
        }
        /* the tanh 1x1 gate's attention: att_bias + att_w^T fp16(o), in double (native_ref.h:93-99) */
        float ga[256];
        if (j->gate == 2)
            for (int n = 0; n < cout; n++) {
                double a = j->att_bias[n];
                for (int k = 0; k < cout; k++) a += (double)f16r(o[k]) * j->att_w[(size_t)k * cout + n];
                ga[n] = (float)a;
            }
        for (int n = 0; n < cout; n++) {
            float v = o[n];
            if (j->gate == 1) v = j->resid[p * cout + n] + v;
            if (j->gate == 2) v = (j->resid[p * cout + n] + f16r(v)) * tanhf(ga[n]);
            if (j->gate == 3) v = (j->resid[p * cout + n] + v) * (1.f / (1.f + expf(-v)) - 0.5f);
            if (R == 0) {
                j->dst[p * cout + n] = f16r(v);
            } else if (n < 3 * R * R) {
                const int c3 = n / (R * R), ry = (n / R) % R, rx = n % R;
                const float add = j->model_in ? j->model_in[((size_t)c3 * H + y) * W + x] : 0.f;
                float out = v + add;
                if (j->out_clamp) out = fminf(fmaxf(out, 0.f), 1.f);
                j->dst[((size_t)c3 * OH + (size_t)R * y + ry) * OW + (size_t)R * x + rx] = f16r(out);
            }
        }
    }
}

int orc_conv3x3_ex(int in_mode, const float *src, int H, int W, int cin, const float *w, const float *bias,
                   const float *slope, int cout, int act, int gate, const float *resid, const float *att_w,
                   const float *att_bias, int R, const float *model_in, int out_clamp, float *dst, int nthreads)
{
    if (!src || !w || !bias || !dst || H < 1 || W < 1 || cin < 1 || cout < 1 || cout > 256) return -1;
    if (in_mode < 0 || in_mode > 2 || (in_mode == 1 && cin != 3) || (in_mode == 2 && cin != 12)) return -1;
    if (gate && !resid) return -1;
    if (gate == 2 && (!att_w || !att_bias)) return -1;
    if (act == 2 && !slope) return -1;
    if (R < 0 || R > 4 || (R > 0 && cout < 3 * R * R)) return -1;
    if (in_mode == 2 && model_in) return -1; /* no skip from an unshuffled input */
    struct conv_job j = {in_mode, H,     W,        cin,      cout,     act, gate,  R, out_clamp, src, w, bias, slope,
                         resid,   att_w, att_bias, model_in, dst};
    orc_par_for(H, nthreads, conv_row, &j);
    return 0;
}

int orc_conv3x3(int in_mode, const float *src, int H, int W, int cin, const float *w, const float *bias,
                const float *slope, int cout, int act, int gate, const float *resid, int R, const float *model_in,
                int out_clamp, float *dst, int nthreads)
{
    if (gate == 2) return -1;
    return orc_conv3x3_ex(in_mode, src, H, W, cin, w, bias, slope, cout, act, gate, resid, NULL, NULL, R, model_in,
                          out_clamp, dst, nthreads);
}

struct cat_job {
    const float *const *srcs;
    int nsrc, c;
    const float *w, *bias;
    float *dst;
};

static void cat_px(void *ctx, int p)
{
    const struct cat_job *j = (const struct cat_job *)ctx;
    const int c = j->c;
    for (int n = 0; n < c; n++) {
        double acc = j->bias[n];
        for (int q = 0; q < j->nsrc; q++) {
            const float *f = j->srcs[q] + (size_t)p * c;
            for (int k = 0; k < c; k++) acc += (double)f[k] * j->w[(size_t)(q * c + k) * c + n];
        }
        j->dst[(size_t)p * c + n] = f16r((float)acc);
    }
}

int orc_concat1x1(const float *const *srcs, int nsrc, int npx, int c, const float *w, const float *bias, float *dst,
                  int nthreads)
{
    if (!srcs || nsrc < 1 || nsrc > 4 || npx < 1 || c < 1 || c > 256 || !w || !bias || !dst) return -1;
    struct cat_job j = {srcs, nsrc, c, w, bias, dst};
    orc_par_for(npx, nthreads, cat_px, &j);
    return 0;
}
