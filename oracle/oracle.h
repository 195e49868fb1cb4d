/*
 * oracle.h — CPU restatement of the reference's algorithms on the native conv path, in plain C.
 *
 * TEST INFRASTRUCTURE ONLY. The product (animejanai-inference_b200/) never links, loads or calls
 * this code; tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it as the
 * checker. Pinned against the reference itself: tests/golden/ holds vectors produced by the
 * reference's own sources compiled here (oracle/_ref, recipe in oracle/ref/), and the CPU tests
 * compare this restatement against them.
 *
 * Every function cites the reference file:line it follows (the-database/animejanai-inference).
 */
#ifndef AJI_ORACLE_H
#define AJI_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* fp32 <-> fp16 bits, round to nearest even (src/native/pack.cpp:69-111). */
uint16_t orc_f2h(float f);
float orc_h2f(uint16_t h);
/* x[i] = fp16(x[i]) for n values (sanity/native_ref.h:22, f16r). */
void orc_round_f16(float *x, size_t n);
void orc_f2h_array(const float *x, uint16_t *out, size_t n);
void orc_h2f_array(const uint16_t *h, float *out, size_t n);

/* One fused 3x3 conv step of a lowered plan (sanity/native_ref.h:53-118), at conv resolution
 * H x W. in_mode 0: src NHWC [H][W][cin]; 1: src NCHW [3][H][W] (the model input, cin 3);
 * 2: src NCHW [3][2H][2W] pixel-unshuffled by 2 (cin 12, channel c * 4 + ry * 2 + rx).
 * w: [9][cin][cout] (fp16-valued floats), bias [cout], slope [cout] (act 2) or NULL.
 * act 0 none, 1 ReLU, 2 PReLU, 3 SiLU; gate 0 none, 1 residual, 2 tanh 1x1
 * ((x + fp16(o)) * tanh(att_bias + att_w^T fp16(o)), att_w [cout][cout] fp16-valued), 3
 * sigmoid-half, with resid NHWC [H][W][cout]. R == 0: dst NHWC [H][W][cout], each value
 * rounded to fp16. R in 1..4: depth-to-space (CRD) into dst NCHW [3][R*H][R*W] plus model_in
 * NCHW [3][H][W] (nearest upsampled) when not NULL (in_mode 0 and 1 only), clamped to [0,1] if
 * out_clamp, rounded to fp16. Accumulates in double. nthreads <= 0: all cores. Returns 0, or -1
 * on bad arguments. orc_conv3x3 is the same without the attention weights (gate 2 refused). */
int orc_conv3x3_ex(int in_mode, const float *src, int H, int W, int cin, const float *w, const float *bias,
                   const float *slope, int cout, int act, int gate, const float *resid, const float *att_w,
                   const float *att_bias, int R, const float *model_in, int out_clamp, float *dst, int nthreads);
int orc_conv3x3(int in_mode, const float *src, int H, int W, int cin, const float *w, const float *bias,
                const float *slope, int cout, int act, int gate, const float *resid, int R, const float *model_in,
                int out_clamp, float *dst, int nthreads);

/* 1x1 conv over the channel concat of nsrc NHWC [npx][c] maps (sanity/native_ref.h:41-52):
 * w [nsrc*c][c], bias [c]; dst NHWC [npx][c] rounded to fp16. */
int orc_concat1x1(const float *const *srcs, int nsrc, int npx, int c, const float *w, const float *bias, float *dst,
                  int nthreads);

/* ---- colour passes (src/resample.h, src/kernels.cu) ---- */
/* zimg filter table (src/resample.h:53-84): returns taps; start [dst] and wt [dst][taps] filled
 * when both are given. filter 0 Spline36, 1 bilinear. */
int orc_filter(int src, int dst, double shift, int filter, int *start, float *wt);
void orc_chroma_shift(int siting, int up, double *sx, double *sy);
/* csp = {kr, kb, yoff, yscale, coff, cscale} (src/resample.h:100-129) */
void orc_make_csp(int format, int matrix, int range, float *csp);
/* NV12/P010 -> fp16 bits NCHW [3][h][w] (src/kernels.cu:105-164, :441-465) */
int orc_pre(int format, int w, int h, int siting, int filter, const void *y_plane, ptrdiff_t ys, const void *uv_plane,
            ptrdiff_t uvs, const float *csp, uint16_t *dst);
/* fp16 bits NCHW [3][h][w] -> NV12/P010 (src/kernels.cu:170-231, :467-497) */
int orc_post(int format, int w, int h, int siting, int filter, const uint16_t *src, const float *csp, void *y_plane,
             ptrdiff_t ys, void *uv_plane, ptrdiff_t uvs);
int orc_post444(int format, int w, int h, const uint16_t *src, const float *csp, uint16_t *yp, uint16_t *cbp,
                uint16_t *crp);
int orc_pre444(int w, int h, const uint16_t *yp, const uint16_t *cbp, const uint16_t *crp, const float *csp,
               uint16_t *dst);

/* ---- the still-image tiler (src/core/tiling.cpp) ---- */
int orc_tile_origins(int len, int tile, int overlap, int *out, int max);
int orc_even_origins(int n, int max_tile, int overlap, int *tile, int *out, int max);
int orc_reflect(int i, int n);
/* w[t][u] for n tiles, u < min(tile, len) * scale */
int orc_axis_weights(const int *org, int n, int len, int tile, int scale, float *w);
/* upscale_tiled with the model as a callback (3-channel model): see oracle_tiling.c */
int orc_upscale_tiled(int (*run)(void *opaque, const float *in, float *out), void *opaque, int tw, int th, int s,
                      int overlap, int even, const uint8_t *in, int W, int H, int ci, ptrdiff_t in_stride,
                      uint8_t *out, ptrdiff_t out_stride);

int orc_resize(const uint16_t *src, int sw, int sh, int dw, int dh, uint16_t *dst);

#ifdef __cplusplus
}
#endif

#endif
