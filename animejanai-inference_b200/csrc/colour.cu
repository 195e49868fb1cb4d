/*
 * colour.cu — the YUV <-> RGB passes around the conv net: NV12/P010 -> fp16 NCHW RGB before the
 * first conv and fp16 NCHW RGB -> NV12/P010 after the last one, plus the 4:4:4 matrix-only
 * variants (C ABI in include/aji_b200.h, named as the reference's src/kernels.h).
 *
 * The reference runs the pre-pass as two kernels with an fp32 chroma plane between them and the
 * post-pass as three kernels with two fp32 planes between them (src/kernels.cu:105-231,
 * :441-497). Here each pass is one kernel over a 2-D tile: the separable filter's first pass is
 * computed for the tile's halo into shared memory and the second pass reads it from there, so
 * the intermediate planes never reach HBM. Every output keeps the same fp32 operation sequence
 * as the reference (taps accumulated in order with fused multiply-adds, IEEE divisions in the
 * normalisation, rintf quantisation), which is what makes the results bit-identical.
 */
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <new>

#include "colour_math.cuh"
#include "feature_map.cuh"
#include "plan.h"
#include "resample.h"
#include "../../include/aji_b200.h"

using namespace ajib;

struct DevPass {
    int taps, src, dst;
    const int *start;
    const float *wt;
    int step2;  // start[i] = start[0] + 2 i for every output i (a 2:1 table)
};

// The streaming post pass's launch (k_post_roll): table offsets and weights (one set per
// direction), chroma rows per block.
struct PostRoll {
    int w, h, cw, ch;
    int oh, ov;  // start[0] of the horizontal and vertical tables (output i starts at o + 2 i)
    int seg;     // chroma rows per block (a multiple of kPsG)
    float wh[16], wv[16];
};

// The streaming pre pass's launch (k_pre_roll): first taps and weights of outputs 0 and 1 of each
// table (output 2k + i starts at s_i + k with output i's weights), luma rows per block.
struct PreRoll {
    int w, h, cw, ch;
    int sh0, sh1, sv0, sv1;
    int seg;  // a multiple of kPrG
    float whe[8], who[8], wve[8], wvo[8];
};

struct aji_plan {
    enum Kind { PRE, POST, RESIZE } kind;
    int format = 0, w = 0, h = 0;
    int dw = 0, dh = 0;  // RESIZE: output size
    FilterTable th, tv;  // host copies (tests)
    DevPass ph{}, pv{};
    int max_rows = 0, max_cols = 0;  // staged halo extents (checked against the kernel's capacity)
    int roll_taps = 0;               // the streaming kernel serves the plan (its taps), else 0
    PostRoll roll{};                 // POST: k_post_roll's launch
    PreRoll proll{};                 // PRE: k_pre_roll's launch
    dim3 roll_grid{};
};

extern "C" aji_csp aji_make_csp(int format, int matrix, int range)
{
    aji_csp c{};
    switch (matrix) {
    case AJI_MATRIX_BT601:
        c.kr = 0.299f;
        c.kb = 0.114f;
        break;
    case AJI_MATRIX_BT2020:
        c.kr = 0.2627f;
        c.kb = 0.0593f;
        break;
    default:
        c.kr = 0.2126f;
        c.kb = 0.0722f;
        break;
    }
    // 16-bit containers hold MSB-aligned samples: limited-range points scale by 256; full-range
    // peaks are the container's largest value at the sample depth.
    const bool wide = format == AJI_FMT_P010 || aji_format_is_444(format);
    const float m = wide ? 256.0f : 1.0f;
    const float maxraw = (format == AJI_FMT_P010 || format == AJI_FMT_YUV444P10MSB) ? 65472.0f
                         : format == AJI_FMT_YUV444P12MSB                           ? 65520.0f
                         : format == AJI_FMT_YUV444P16                              ? 65535.0f
                                                                                    : 255.0f;
    if (range == AJI_RANGE_FULL) {
        c.yoff = 0.0f;
        c.yscale = maxraw;
        c.coff = wide ? 32768.0f : 128.0f;
        c.cscale = maxraw;
    } else {
        c.yoff = 16.0f * m;
        c.yscale = 219.0f * m;
        c.coff = 128.0f * m;
        c.cscale = 224.0f * m;
    }
    return c;
}

namespace {

// mirror an index into [0, n): -1 -> 0, -2 -> 1, n -> n - 1 (then clamp for far-out indices)
__device__ __forceinline__ int mirror_index(int i, int n)
{
    i = i < 0 ? -i - 1 : i;
    i = i >= n ? 2 * n - 1 - i : i;
    return min(max(i, 0), n - 1);
}

// rintf(v / qdiv) clamped and scaled back. qdiv is 1, 16 or 64 (a power of two), so v / qdiv is
// exactly v * qinv with qinv = 1 / qdiv.
__device__ __forceinline__ float quantize(float v, float qdiv, float qinv, float qmax)
{
    return __fmul_rn(fminf(fmaxf(rintf(__fmul_rn(v, qinv)), 0.0f), qmax), qdiv);
}

// ---------------- pre: NV12/P010 -> fp16 NCHW RGB ----------------
constexpr int kPreTW = 64, kPreTH = 16, kPreRows = 24;
constexpr int kPreMaxTaps = 8;  // taps per pass the kernel holds (plans with more are refused)

// The head conv's input, written by the pre pass as well when it is fused with it (PACK): the
// fp16 RGB of each pixel, normalised as the conv's input ((x - mean) * scale, rounded to fp16)
// when the model asks for it, as chunk 0 {r, g, b, 0 x 5} of an 8-channel strip-chunked map —
// the bytes the executor's own pack of the NCHW input (conv.cu, k_pack_input) writes. With
// unshuffle set (the streaming kernel only), the map is the 2x pixel-unshuffled input at half
// width and height: 16 channels, c * 4 + ry * 2 + rx for colour c and the pixel's row and column
// parity, the 12 real ones in chunk 0 and the first half of chunk 1.
struct PreMap {
    __half *map;
    int nstrips, in_norm, unshuffle;
    float mean[3], scale[3];
};

template <typename T, bool PACK>
__global__ void __launch_bounds__(256) k_pre(const uint8_t *yp, ptrdiff_t ys, const uint8_t *uvp, ptrdiff_t uvs,
                                             DevPass ph, DevPass pv, aji_csp csp, __half *dst, int w, int h, PreMap pm)
{
    __shared__ float2 uvh[kPreRows][kPreTW];  // horizontally resampled (u, v) per staged chroma row
    const int x0 = blockIdx.x * kPreTW, y0 = blockIdx.y * kPreTH;
    const int tid = threadIdx.x;
    const int ylast = min(y0 + kPreTH, h) - 1;
    const int lo = pv.start[y0], hi = pv.start[ylast] + pv.taps - 1;
    const int nrows = hi - lo + 1;  // <= kPreRows (checked at plan creation)
    const int ch = pv.src;

    // pass 1: horizontal resample of the staged chroma rows (interleaved CbCr). A thread keeps its
    // column's taps and weights in registers and walks the rows, each row's samples loaded before
    // its FMA chain.
    {
        const int tx = tid % kPreTW, x = x0 + tx;
        if (x < w) {
            const int taps = ph.taps;
            const float *wtp = ph.wt + (size_t)x * taps;
            const int s0 = ph.start[x];
            float wt[kPreMaxTaps];
            int sx[kPreMaxTaps];
#pragma unroll
            for (int j = 0; j < kPreMaxTaps; j++) {
                wt[j] = j < taps ? wtp[j] : 0.0f;
                sx[j] = mirror_index(s0 + min(j, taps - 1), ph.src);
            }
            for (int rr = tid / kPreTW; rr < nrows; rr += 256 / kPreTW) {
                const T *row = reinterpret_cast<const T *>(uvp + (size_t)mirror_index(lo + rr, ch) * uvs);
                float cu[kPreMaxTaps], cv[kPreMaxTaps];
#pragma unroll
                for (int j = 0; j < kPreMaxTaps; j++) {
                    if (j < taps) {
                        cu[j] = (float)row[2 * sx[j]];
                        cv[j] = (float)row[2 * sx[j] + 1];
                    }
                }
                float u = 0.0f, v = 0.0f;
#pragma unroll
                for (int j = 0; j < kPreMaxTaps; j++) {
                    if (j < taps) {
                        u = __fmaf_rn(wt[j], cu[j], u);
                        v = __fmaf_rn(wt[j], cv[j], v);
                    }
                }
                uvh[rr][tx] = make_float2(u, v);
            }
        }
    }
    __syncthreads();

    // pass 2: vertical resample + matrix, one pixel per thread and row
    const int tx = tid % kPreTW, x = x0 + tx;
    if (x >= w) return;
    const size_t plane = (size_t)w * h;
    const float kg = __fsub_rn(__fsub_rn(1.0f, csp.kr), csp.kb);
    const float cr = __fmul_rn(2.0f, __fsub_rn(1.0f, csp.kr));   // 2 (1 - kr)
    const float cb = __fmul_rn(2.0f, __fsub_rn(1.0f, csp.kb));   // 2 (1 - kb)
    const float gb = __fmul_rn(__fmul_rn(2.0f, csp.kb), __fsub_rn(1.0f, csp.kb));  // 2 kb (1 - kb)
    const float gr = __fmul_rn(__fmul_rn(2.0f, csp.kr), __fsub_rn(1.0f, csp.kr));  // 2 kr (1 - kr)
    // (x / yscale and x / cscale by dev::div_by: bit-identical to the IEEE division over these
    // dividends, ajib_selftest_division_by)
    const float ry = __frcp_rn(csp.yscale), rc = __frcp_rn(csp.cscale);
    // the thread's four rows: luma loads first, then independent FMA chains
    constexpr int kG = 256 / kPreTW, kN = kPreTH / kG;
    const int taps = pv.taps;
    float lraw[kN];
#pragma unroll
    for (int k = 0; k < kN; k++) {
        const int y = min(y0 + tid / kPreTW + k * kG, h - 1);
        lraw[k] = (float)reinterpret_cast<const T *>(yp + (size_t)y * ys)[x];
    }
    float uu[kN], vv[kN];
#pragma unroll
    for (int k = 0; k < kN; k++) {
        const int y = min(y0 + tid / kPreTW + k * kG, h - 1);
        const float *wt = pv.wt + (size_t)y * taps;
        const int s0 = pv.start[y] - lo;
        float u = 0.0f, v = 0.0f;
#pragma unroll
        for (int j = 0; j < kPreMaxTaps; j++) {
            if (j < taps) {
                const float2 q = uvh[s0 + j][tx];
                u = __fmaf_rn(wt[j], q.x, u);
                v = __fmaf_rn(wt[j], q.y, v);
            }
        }
        uu[k] = u;
        vv[k] = v;
    }
#pragma unroll
    for (int k = 0; k < kN; k++) {
        const int ty = tid / kPreTW + k * kG;
        const int y = y0 + ty;
        if (y >= h) break;
        const float u = uu[k], v = vv[k];
        const float raw = lraw[k];
        const float Y = dev::div_by(__fsub_rn(raw, csp.yoff), csp.yscale, ry);
        const float U = dev::div_by(__fsub_rn(u, csp.coff), csp.cscale, rc);
        const float V = dev::div_by(__fsub_rn(v, csp.coff), csp.cscale, rc);
        const float r = __fmaf_rn(cr, V, Y);
        const float b = __fmaf_rn(cb, U, Y);
        const float g = __fsub_rn(Y, __fdiv_rn(__fmaf_rn(gb, U, __fmul_rn(gr, V)), kg));
        const size_t idx = (size_t)y * w + x;
        const __half hr = __float2half_rn(r), hg = __float2half_rn(g), hb = __float2half_rn(b);
        dst[idx] = hr;
        dst[plane + idx] = hg;
        dst[2 * plane + idx] = hb;
        if constexpr (PACK) {
            float v[3] = {__half2float(hr), __half2float(hg), __half2float(hb)};
            if (pm.in_norm) {
#pragma unroll
                for (int c = 0; c < 3; c++) v[c] = (v[c] - pm.mean[c]) * pm.scale[c];
            }
            store_px(pm.map, y, x, 0, pm.nstrips, 1, make_uint4(pack_h2(v[0], v[1]), pack_h2(v[2], 0.f), 0u, 0u));
        }
    }
}

// ---------------- post: fp16 NCHW RGB -> NV12/P010 ----------------
// A tile is 64 x 16 chroma samples (128 x 32 luma pixels). Staging: each staged (mirrored) luma
// pixel of the tile's filter halo is read once, its colour differences (b - Y) / db and
// (r - Y) / dr go to shared memory split by column parity (so the horizontal taps of 32
// consecutive outputs, two source columns apart, are 32 consecutive words), and where the pixel
// is one of the tile's own, its quantised luma is stored. Then the horizontal pass (each thread
// keeps one output column's weights in registers and walks rows), then the vertical pass.
constexpr int kPostTW = 64, kPostTH = 16;          // chroma samples per tile
constexpr int kPostRows = 44, kPostCols = 140;     // staged luma halo capacity
constexpr int kPostHalf = kPostCols / 2;           // words per staged row of one parity
constexpr int kPostPar = kPostRows * kPostHalf + 16;  // one parity plane (+16: the other parity on other banks)
constexpr int kPostMaxTaps = 16;
constexpr size_t kPostSmem = (size_t)(4 * kPostPar + 2 * kPostRows * kPostTW + kPostTH * kPostMaxTaps) * sizeof(float);

template <typename T>
__global__ void __launch_bounds__(256) k_post(const __half *src, int w, int h, DevPass ph, DevPass pv, aji_csp csp,
                                              float qdiv, float qmax, uint8_t *yp, ptrdiff_t ys, uint8_t *uvp,
                                              ptrdiff_t uvs)
{
    extern __shared__ float post_sm[];
    float *su = post_sm;                            // [2 parities][kPostRows][kPostHalf] (b - Y) / db
    float *sv = su + 2 * kPostPar;                  // the same for (r - Y) / dr
    float *hu = sv + 2 * kPostPar;                  // [kPostRows][kPostTW] after the horizontal pass
    float *hv = hu + kPostRows * kPostTW;
    float *swv = hv + kPostRows * kPostTW;          // [kPostTH][kPostMaxTaps] vertical weights of the tile
    const int cx0 = blockIdx.x * kPostTW, cy0 = blockIdx.y * kPostTH;
    const int cw = ph.dst, chh = pv.dst;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cxl = min(cx0 + kPostTW, cw) - 1, cyl = min(cy0 + kPostTH, chh) - 1;
    const int xlo = ph.start[cx0], xhi = ph.start[cxl] + ph.taps - 1;
    const int ylo = pv.start[cy0], yhi = pv.start[cyl] + pv.taps - 1;
    const int ncols = xhi - xlo + 1, nrows = yhi - ylo + 1;
    const size_t plane = (size_t)w * h;
    const float kg = __fsub_rn(__fsub_rn(1.0f, csp.kr), csp.kb);
    const float db = __fmul_rn(2.0f, __fsub_rn(1.0f, csp.kb));
    const float dr = __fmul_rn(2.0f, __fsub_rn(1.0f, csp.kr));
    const float rdb = __frcp_rn(db), rdr = __frcp_rn(dr);  // (x / db and x / dr by dev::div_by)
    const float qinv = __frcp_rn(qdiv);
    // the tile's own luma pixels, and whether the staged halo holds all of them
    const int lx0 = 2 * cx0, lx1 = min(2 * (cx0 + kPostTW), w), ly0 = 2 * cy0, ly1 = min(2 * (cy0 + kPostTH), h);
    const bool covered = xlo <= lx0 && xhi >= lx1 - 1 && ylo <= ly0 && yhi >= ly1 - 1;

    for (int i = tid; i < kPostTH * pv.taps; i += 256) {
        const int ty = i / pv.taps, j = i % pv.taps;
        swv[ty * kPostMaxTaps + j] = cy0 + ty < chh ? pv.wt[(size_t)(cy0 + ty) * pv.taps + j] : 0.0f;
    }
    // staging: one warp per staged row, lanes along it; a row's pixels are all loaded before any
    // is converted, so their global loads are in flight together
    constexpr int kPostIt = (kPostCols + 31) / 32;
    for (int rr = warp; rr < nrows; rr += 8) {
        const int gy = ylo + rr, my = mirror_index(gy, h);
        const bool own_row = covered && gy == my && gy >= ly0 && gy < ly1;
        const __half *srow = src + (size_t)my * w;
        __half pr[kPostIt], pg[kPostIt], pb[kPostIt];
#pragma unroll
        for (int k = 0; k < kPostIt; k++) {
            const int cc = lane + 32 * k;
            if (cc < ncols) {
                const int mx = mirror_index(xlo + cc, w);
                pr[k] = srow[mx];
                pg[k] = srow[plane + mx];
                pb[k] = srow[2 * plane + mx];
            }
        }
#pragma unroll
        for (int k = 0; k < kPostIt; k++) {
            const int cc = lane + 32 * k;
            if (cc >= ncols) continue;
            const int gx = xlo + cc;
            const float r = __half2float(pr[k]), g = __half2float(pg[k]), b = __half2float(pb[k]);
            const float Y = __fmaf_rn(csp.kb, b, __fmaf_rn(csp.kr, r, __fmul_rn(kg, g)));
            const int at = (cc & 1) * kPostPar + rr * kPostHalf + (cc >> 1);
            su[at] = dev::div_by(__fsub_rn(b, Y), db, rdb);
            sv[at] = dev::div_by(__fsub_rn(r, Y), dr, rdr);
            if (own_row && gx == mirror_index(gx, w) && gx >= lx0 && gx < lx1)
                reinterpret_cast<T *>(yp + (size_t)gy * ys)[gx] = (T)quantize(__fmaf_rn(Y, csp.yscale, csp.yoff), qdiv, qinv, qmax);
        }
    }
    if (!covered) {
        // (no filter table of this engine gets here: a 2:1 table's halo always covers the tile)
        for (int i = tid; i < (lx1 - lx0) * (ly1 - ly0); i += 256) {
            const int ly = ly0 + i / (lx1 - lx0), lx = lx0 + i % (lx1 - lx0);
            const size_t idx = (size_t)ly * w + lx;
            const float r = __half2float(src[idx]), g = __half2float(src[plane + idx]), b = __half2float(src[2 * plane + idx]);
            const float Y = __fmaf_rn(csp.kb, b, __fmaf_rn(csp.kr, r, __fmul_rn(kg, g)));
            reinterpret_cast<T *>(yp + (size_t)ly * ys)[lx] = (T)quantize(__fmaf_rn(Y, csp.yscale, csp.yoff), qdiv, qinv, qmax);
        }
    }
    __syncthreads();
    // horizontal pass. For a 2:1 table (every output's taps start two staged columns after the
    // previous one's) a thread takes two adjacent outputs, whose twelve taps overlap in ten: the
    // union is seven words of each parity, loaded as float2 pairs (consecutive threads read
    // consecutive pairs, no bank conflicts), a third of the shared-memory loads of one output a
    // thread. Each output's FMAs run in tap order as below.
    const int tx = tid & (kPostTW - 1), grp = tid / kPostTW, cx = cx0 + tx;
    if (ph.step2) {
        const int t = tid & 31, rg = tid >> 5;  // output pair (2t, 2t + 1), row group
        const int ca = cx0 + 2 * t, cb = ca + 1;
        const int taps = ph.taps;
        float wa[kPostMaxTaps], wb[kPostMaxTaps];
#pragma unroll
        for (int j = 0; j < kPostMaxTaps; j++) {
            wa[j] = (j < taps && ca < cw) ? ph.wt[(size_t)ca * taps + j] : 0.0f;
            wb[j] = (j < taps && cb < cw) ? ph.wt[(size_t)cb * taps + j] : 0.0f;
        }
        // output a's taps start at staged column 4t (s0 = start[ca] - xlo), b's at 4t + 2: words
        // 2t .. 2t + taps / 2 of each parity plane (kPostHalf leaves room for the widest table)
        constexpr int kW = kPostMaxTaps / 2 + 2;  // words loaded per plane (float2 pairs)
        if (ca < cw) {
            for (int rr = rg; rr < nrows; rr += 256 / 32) {
#pragma unroll
                for (int q = 0; q < 2; q++) {
                    const float *pl = q == 0 ? su : sv;
                    float e[kW], o[kW];
#pragma unroll
                    for (int k = 0; k < kW; k += 2) {
                        const float2 pe = *reinterpret_cast<const float2 *>(pl + rr * kPostHalf + 2 * t + k);
                        const float2 po = *reinterpret_cast<const float2 *>(pl + kPostPar + rr * kPostHalf + 2 * t + k);
                        e[k] = pe.x;
                        e[k + 1] = pe.y;
                        o[k] = po.x;
                        o[k + 1] = po.y;
                    }
                    float xa = 0.0f, xb = 0.0f;
#pragma unroll
                    for (int j = 0; j < kPostMaxTaps; j++) {
                        if (j < taps) {
                            const float ta = (j & 1) ? o[j >> 1] : e[j >> 1];
                            const float tb = (j & 1) ? o[(j >> 1) + 1] : e[(j >> 1) + 1];
                            xa = __fmaf_rn(wa[j], ta, xa);
                            xb = __fmaf_rn(wb[j], tb, xb);
                        }
                    }
                    float *hq = q == 0 ? hu : hv;
                    *reinterpret_cast<float2 *>(hq + rr * kPostTW + 2 * t) = make_float2(xa, xb);
                }
            }
        }
    } else if (cx < cw) {
        float wt[kPostMaxTaps];
        const int taps = ph.taps;
#pragma unroll
        for (int j = 0; j < kPostMaxTaps; j++) wt[j] = j < taps ? ph.wt[(size_t)cx * taps + j] : 0.0f;
        const int s0 = ph.start[cx] - xlo;
        // two staged rows at a time (rr and rr + 4): four independent FMA chains per thread
        constexpr int kG = 256 / kPostTW;
        for (int rr = grp; rr < nrows; rr += 2 * kG) {
            const int r1 = rr + kG < nrows ? rr + kG : rr;
            float u0 = 0.0f, v0 = 0.0f, u1 = 0.0f, v1 = 0.0f;
#pragma unroll
            for (int j = 0; j < kPostMaxTaps; j++) {
                if (j < taps) {
                    const int c = s0 + j;
                    const int at = (c & 1) * kPostPar + (c >> 1);
                    u0 = __fmaf_rn(wt[j], su[at + rr * kPostHalf], u0);
                    v0 = __fmaf_rn(wt[j], sv[at + rr * kPostHalf], v0);
                    u1 = __fmaf_rn(wt[j], su[at + r1 * kPostHalf], u1);
                    v1 = __fmaf_rn(wt[j], sv[at + r1 * kPostHalf], v1);
                }
            }
            hu[rr * kPostTW + tx] = u0;
            hv[rr * kPostTW + tx] = v0;
            if (r1 != rr) {
                hu[r1 * kPostTW + tx] = u1;
                hv[r1 * kPostTW + tx] = v1;
            }
        }
    }
    __syncthreads();
    // vertical pass, quantise, interleave
    if (cx < cw) {
        const int taps = pv.taps;
        // the thread's four output rows at once (independent FMA chains)
        constexpr int kG = 256 / kPostTW, kN = kPostTH / kG;
        float u[kN], v[kN];
        int s0[kN];
#pragma unroll
        for (int k = 0; k < kN; k++) {
            const int cy = min(cy0 + grp + k * kG, chh - 1);
            s0[k] = pv.start[cy] - ylo;
            u[k] = 0.0f;
            v[k] = 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kPostMaxTaps; j++) {
            if (j < taps) {
#pragma unroll
                for (int k = 0; k < kN; k++) {
                    const float wj = swv[(grp + k * kG) * kPostMaxTaps + j];
                    u[k] = __fmaf_rn(wj, hu[(s0[k] + j) * kPostTW + tx], u[k]);
                    v[k] = __fmaf_rn(wj, hv[(s0[k] + j) * kPostTW + tx], v[k]);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < kN; k++) {
            const int cy = cy0 + grp + k * kG;
            if (cy >= chh) break;
            T *row = reinterpret_cast<T *>(uvp + (size_t)cy * uvs);
            row[2 * cx] = (T)quantize(__fmaf_rn(u[k], csp.cscale, csp.coff), qdiv, qinv, qmax);
            row[2 * cx + 1] = (T)quantize(__fmaf_rn(v[k], csp.cscale, csp.coff), qdiv, qinv, qmax);
        }
    }
}

// ---------------- post, streaming form ----------------
// For 2:1 tables whose outputs all share one set of weights (every table of a 4:2:0 post plan:
// zimg's positions are exact in double, so each output's taps sit at the same offsets) on
// frames whose width is a multiple of 8. The chroma plane is cut into strips of 64 columns (128
// luma pixels) and each strip into runs of chroma rows; a block walks its run downwards, eight
// chroma rows (sixteen luma rows) a step:
//  - the next step's sixteen luma rows (3 planes x a 16-byte-aligned window of 152 columns
//    around the strip's filter halo) are copied into a ring in shared memory by cp.async while
//    this step computes;
//  - each staged pixel's colour differences (u, v) are computed once and kept as a pair, split by
//    column parity as in k_post; for the block's own pixels the quantised luma is stored, two
//    pixels a store;
//  - the horizontal pass turns each staged luma row into one row of 64 (u, v) pairs in a ring of
//    32 rows, two adjacent outputs a thread (their taps overlap: 128-bit loads of the pairs);
//  - the vertical pass reads the ring, two output rows a thread.
// u and v share every tap position and weight, so each tap of both planes is one packed fp32 FMA
// (__ffma2_rn: two IEEE fp32 FMAs, each rounded as __fmaf_rn), and so are the colour matrix and
// the divisions of two adjacent pixels. Only the taps - 2 luma rows a run starts with are staged
// twice. Every output keeps the reference's operation sequence (the expressions of k_post), so
// the bytes are identical.
constexpr int kPsCols = 64;              // chroma columns per strip
constexpr int kPsG = 8;                  // chroma rows per step
constexpr int kPsLW = 152;               // staged luma columns per row and plane (19 x 16 bytes)
constexpr int kPsChunks = kPsLW / 8;     // 16-byte pieces per staged row and plane
constexpr int kPsRaw = 32;               // luma rows in the staging ring (two steps)
constexpr int kPsHR = 32;                // horizontally filtered rows in their ring
constexpr int kPsNW = kPsLW / 2;         // (u, v) pairs per staged row of one parity

struct PostRollSmem {
    __half raw[kPsRaw][3][kPsLW];        // staged fp16 RGB rows
    float2 d[2][2 * kPsG][kPsNW];        // [parity][row][word] ((b - Y) / db, (r - Y) / dr)
    float2 hr[kPsHR][kPsCols];           // horizontally filtered (u, v)
};
static_assert(sizeof(PostRoll::wh) / sizeof(float) == kPostMaxTaps, "PostRoll holds the widest table");

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait()
{
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }
// x / d for both lanes, as dev::div_by (fma(q0, -d, a) is fma(-q0, d, a): negation is exact)
__device__ __forceinline__ float2 div_by2(float2 a, float d, float r)
{
    const float2 q0 = __fmul2_rn(a, f2(r));
    const float2 e = __ffma2_rn(q0, f2(-d), a);
    return __ffma2_rn(e, f2(r), q0);
}

// The sample bits quantize() gives for v = t * qdiv in the streaming kernel's formats (P010: 10
// bits in the high bits of 16, qdiv 64; NV12: qdiv 1): round to nearest even with the result
// clamped to [0, qmax] in one conversion (negative values and NaN give 0, as fmaxf(., 0) does),
// then the shift that is the multiplication by qdiv.
template <typename T>
__device__ __forceinline__ uint32_t quant_bits(float t)
{
    uint32_t i;
    asm("cvt.rni.u32.f32 %0, %1;" : "=r"(i) : "f"(t));
    return sizeof(T) == 2 ? min(i, 1023u) << 6 : min(i, 255u);
}

template <typename T, int TAPS>
__global__ void __launch_bounds__(256, 3) k_post_roll(const __half *src, PostRoll pr, aji_csp csp, float qdiv,
                                                      float qmax, uint8_t *yp, ptrdiff_t ys, uint8_t *uvp, ptrdiff_t uvs)
{
    extern __shared__ __align__(16) unsigned char ps_smem[];
    PostRollSmem &sm = *reinterpret_cast<PostRollSmem *>(ps_smem);
    constexpr int kPro = TAPS - 2;  // luma rows staged before the first step
    // the row loops below cover rows tid / 64 + 4 k (k < 4) and tid / 32 + 8 k (k < 2): every
    // row of a pass of at most 2 kPsG rows
    static_assert(kPro <= 2 * kPsG, "the prologue's rows fit the row loops");
    const int tid = threadIdx.x;
    const int w = pr.w, h = pr.h;
    const int cx0 = blockIdx.x * kPsCols;
    const int cya = blockIdx.y * pr.seg, cyb = min(cya + pr.seg, pr.ch);
    const int cxl = min(cx0 + kPsCols, pr.cw) - 1;              // the strip's last real column
    const int xlo = 2 * cx0 + pr.oh;                             // staged column 0
    const int ncols = 2 * (cxl - cx0) + TAPS;                    // staged columns real outputs read
    const int xa = xlo & ~7;                                     // the aligned window's first column
    const int ylo = 2 * cya + pr.ov;                             // luma row of relative row 0
    const int nsteps = (cyb - cya + kPsG - 1) / kPsG;
    const size_t plane = (size_t)w * h;
    const float kg = __fsub_rn(__fsub_rn(1.0f, csp.kr), csp.kb);
    const float db = __fmul_rn(2.0f, __fsub_rn(1.0f, csp.kb));
    const float dr = __fmul_rn(2.0f, __fsub_rn(1.0f, csp.kr));
    const float rdb = __frcp_rn(db), rdr = __frcp_rn(dr);
    const float qinv = __frcp_rn(qdiv);
    const int lx1 = min(2 * (cx0 + kPsCols), w);                 // the block's own luma columns end
    const int ly0 = 2 * cya, ly1 = 2 * cyb;                      // and its own rows

    // staging: piece (plane, 16-byte chunk) tid & 63 of rows tid >> 6, + 4, + 8, + 12
    const int piece = tid & 63, sp = piece / kPsChunks, sj = piece - sp * kPsChunks;
    const int scol = xa + 8 * sj;
    const bool scopy = piece < 3 * kPsChunks && scol >= 0 && scol + 8 <= w;
    const __half *sbase = src + (scopy ? sp * plane + scol : 0);
    auto stage = [&](int rel0, int n) {
        if (!scopy) return;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int r = (tid >> 6) + 4 * k;
            if (r >= n) break;
            const int rel = rel0 + r;
            cp_async16(&sm.raw[rel & (kPsRaw - 1)][sp][8 * sj], sbase + (size_t)mirror_index(ylo + rel, h) * w);
        }
    };
    // one staged pixel's colour differences (the halo columns outside the strip's own 128, and
    // own columns past a partial strip's end): mirrored column
    auto diff_px = [&](int r, int rel, int gx) {
        const __half(*row)[kPsLW] = sm.raw[rel & (kPsRaw - 1)];
        const int at = min(max(mirror_index(gx, w) - xa, 0), kPsLW - 1);
        const float rr = __half2float(row[0][at]), gg = __half2float(row[1][at]), bb = __half2float(row[2][at]);
        const float Y = __fmaf_rn(csp.kb, bb, __fmaf_rn(csp.kr, rr, __fmul_rn(kg, gg)));
        const int c = gx - xlo;
        sm.d[c & 1][r][c >> 1] = make_float2(dev::div_by(__fsub_rn(bb, Y), db, rdb), dev::div_by(__fsub_rn(rr, Y), dr, rdr));
    };
    // halo pixels: the columns [xlo, 2 cx0) and [2 cx0 + 128, xlo + ncols), one per thread and row
    const int nhl = 2 * cx0 - xlo, nh = nhl + max(xlo + ncols - (2 * cx0 + 2 * kPsCols), 0);
    const int hrow = nh ? tid / nh : 2 * kPsG, hidx = nh ? tid - hrow * nh : 0;
    const int hgx = hidx < nhl ? xlo + hidx : 2 * cx0 + 2 * kPsCols + (hidx - nhl);
    // own columns: the pair (2 cx0 + 2p, + 1), p = tid & 63, rows tid >> 6, + 4, + 8, + 12
    const int pgx = 2 * cx0 + 2 * (tid & 63), pc = pgx - xlo;
    const bool pfast = pgx + 1 < w;
    auto differences = [&](int rel0, int n) {
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int r = (tid >> 6) + 4 * k;
            if (r >= n) break;
            const int rel = rel0 + r, gy = ylo + rel;
            if (pfast) {
                const __half(*row)[kPsLW] = sm.raw[rel & (kPsRaw - 1)];
                const int at = pgx - xa;
                const float2 r2 = __half22float2(*reinterpret_cast<const __half2 *>(&row[0][at]));
                const float2 g2 = __half22float2(*reinterpret_cast<const __half2 *>(&row[1][at]));
                const float2 b2 = __half22float2(*reinterpret_cast<const __half2 *>(&row[2][at]));
                const float2 Y = __ffma2_rn(f2(csp.kb), b2, __ffma2_rn(f2(csp.kr), r2, __fmul2_rn(f2(kg), g2)));
                // b - Y as fma(Y, -1, b): the product is exact, so the one rounding is the subtraction's
                const float2 U = div_by2(__ffma2_rn(Y, f2(-1.0f), b2), db, rdb);
                const float2 V = div_by2(__ffma2_rn(Y, f2(-1.0f), r2), dr, rdr);
                if (pc < ncols) sm.d[pc & 1][r][pc >> 1] = make_float2(U.x, V.x);
                if (pc + 1 < ncols) sm.d[(pc + 1) & 1][r][(pc + 1) >> 1] = make_float2(U.y, V.y);
                if (gy >= ly0 && gy < ly1 && pgx < lx1) {
                    const float2 t = __fmul2_rn(__ffma2_rn(Y, f2(csp.yscale), f2(csp.yoff)), f2(qinv));
                    const uint32_t q0 = quant_bits<T>(t.x), q1 = quant_bits<T>(t.y);
                    T *yrow = reinterpret_cast<T *>(yp + (size_t)gy * ys);
                    if constexpr (sizeof(T) == 2)
                        *reinterpret_cast<uint32_t *>(yrow + pgx) = q0 | (q1 << 16);
                    else
                        *reinterpret_cast<uint16_t *>(yrow + pgx) = (uint16_t)(q0 | (q1 << 8));
                }
            } else {
                if (pc < ncols) diff_px(r, rel, pgx);
                if (pc + 1 < ncols) diff_px(r, rel, pgx + 1);
            }
        }
        if (hrow < n) diff_px(hrow, rel0 + hrow, hgx);
    };
    // horizontal pass: outputs 2t and 2t + 1 of the strip (their taps start at staged columns 4t
    // and 4t + 2: pairs 2t .. 2t + TAPS / 2 of each parity), rows tid >> 5 and + 8
    constexpr int kW = (TAPS / 2 + 2) & ~1;  // pairs loaded per parity (two per 128-bit load)
    const int ht = tid & 31;
    auto horizontal = [&](int rel0, int n) {
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const int r = (tid >> 5) + 8 * k;
            if (r >= n) break;
            float2 e[kW], o[kW];
#pragma unroll
            for (int k = 0; k < kW; k += 2) {
                const float4 pe = *reinterpret_cast<const float4 *>(&sm.d[0][r][2 * ht + k]);
                const float4 po = *reinterpret_cast<const float4 *>(&sm.d[1][r][2 * ht + k]);
                e[k] = make_float2(pe.x, pe.y), e[k + 1] = make_float2(pe.z, pe.w);
                o[k] = make_float2(po.x, po.y), o[k + 1] = make_float2(po.z, po.w);
            }
            float2 a = make_float2(0.0f, 0.0f), b = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int j = 0; j < TAPS; j++) {
                a = __ffma2_rn(f2(pr.wh[j]), (j & 1) ? o[j >> 1] : e[j >> 1], a);
                b = __ffma2_rn(f2(pr.wh[j]), (j & 1) ? o[(j >> 1) + 1] : e[(j >> 1) + 1], b);
            }
            *reinterpret_cast<float4 *>(&sm.hr[(rel0 + r) & (kPsHR - 1)][2 * ht]) = make_float4(a.x, a.y, b.x, b.y);
        }
    };

    stage(0, kPro);
    cp_async_commit();
    stage(kPro, 2 * kPsG);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    differences(0, kPro);
    __syncthreads();
    horizontal(0, kPro);

    // vertical pass: column tid & 63 of the strip, output rows 2 (tid >> 6) and + 1 of the step
    const int vcol = tid & 63, vcx = cx0 + vcol, vrp = tid >> 6;
    for (int s = 0; s < nsteps; s++) {
        if (s + 1 < nsteps) stage(kPro + 2 * kPsG * (s + 1), 2 * kPsG);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        differences(kPro + 2 * kPsG * s, 2 * kPsG);
        __syncthreads();
        horizontal(kPro + 2 * kPsG * s, 2 * kPsG);
        __syncthreads();
        const int cyf = cya + kPsG * s + 2 * vrp;  // the first of this thread's two output rows
        const int rel0 = 2 * (cyf - cya);
        float2 v[2 + TAPS];
#pragma unroll
        for (int i = 0; i < 2 + TAPS; i++) v[i] = sm.hr[(rel0 + i) & (kPsHR - 1)][vcol];
        if (vcx < pr.cw) {
#pragma unroll
            for (int k = 0; k < 2; k++) {
                float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int j = 0; j < TAPS; j++) acc = __ffma2_rn(f2(pr.wv[j]), v[2 * k + j], acc);
                if (cyf + k < cyb) {
                    const float2 t = __fmul2_rn(__ffma2_rn(acc, f2(csp.cscale), f2(csp.coff)), f2(qinv));
                    const uint32_t qu = quant_bits<T>(t.x), qv = quant_bits<T>(t.y);
                    T *uvrow = reinterpret_cast<T *>(uvp + (size_t)(cyf + k) * uvs);
                    if constexpr (sizeof(T) == 2)
                        *reinterpret_cast<uint32_t *>(uvrow + 2 * vcx) = qu | (qv << 16);
                    else
                        *reinterpret_cast<uint16_t *>(uvrow + 2 * vcx) = (uint16_t)(qu | (qv << 8));
                }
            }
        }
    }
}

// ---------------- pre, streaming form ----------------
// For 2x tables with period 2 (output 2k + 2 starts one source sample after output 2k and uses
// its weights: every table of a 4:2:0 pre plan) on frames whose width is a multiple of 16. A
// block owns a strip of 128 luma columns (one strip of the head conv's map) and a run of luma
// rows, and walks it sixteen luma rows (eight chroma rows) a step:
//  - the next step's luma rows and new chroma rows (a 16-byte-aligned window of 80 (u, v) pairs,
//    mirrored at the frame's edges) are copied by cp.async while this step computes; each thread
//    converts the chroma piece it copied to fp32 pairs;
//  - the horizontal pass upsamples each new chroma row to the strip's 128 columns into a ring of
//    16 rows, two adjacent outputs a thread;
//  - the vertical pass, the colour matrix and the stores run two adjacent pixels a thread: their
//    u and v, and the two pixels of each matrix step, are packed fp32 operations (__ffma2_rn and
//    friends: two IEEE fp32 operations, each rounded as the scalar one), the output planes are
//    written two pixels a store, and the head conv's map (PACK) one pixel chunk a store.
// Only the taps - 1 (+1) chroma rows a run starts with are staged twice. Every output keeps the
// reference's operation sequence (the expressions of k_pre), so the bytes are identical.
constexpr int kPrCols = 128;  // luma columns per strip
constexpr int kPrG = 16;      // luma rows per step (eight chroma rows)
constexpr int kPrCW = 80;     // staged chroma (u, v) pairs per row
constexpr int kPrCR = 16;     // chroma rows in the rings
constexpr int kPrYR = 32;     // luma rows in the luma ring (two steps)

template <typename T>
struct PreRollSmem {
    T uvraw[kPrCR][2 * kPrCW];   // staged (u, v) samples
    float2 uvf[kPrCR][kPrCW];    // the same as fp32 pairs
    float2 hr[kPrCR][kPrCols];   // horizontally upsampled (u, v) of each luma column
    T yraw[kPrYR][kPrCols];      // staged luma rows
};

// Exact fp32 values of the two 16-bit samples in a word (low, high): 2^23 + v has v in its low
// mantissa bits, and subtracting 2^23 is exact.
__device__ __forceinline__ float2 u16x2_to_f2(uint32_t wd)
{
    return __fadd2_rn(make_float2(__uint_as_float(__byte_perm(wd, 0x4B00u, 0x5410)),
                                  __uint_as_float(__byte_perm(wd, 0x4B00u, 0x5432))),
                      f2(-8388608.0f));
}
// the same for bytes k and k + 1 of a word
template <int K>
__device__ __forceinline__ float2 u8x2_to_f2(uint32_t wd)
{
    return __fadd2_rn(make_float2(__uint_as_float(__byte_perm(wd, 0x4B000000u, 0x7440 + K)),
                                  __uint_as_float(__byte_perm(wd, 0x4B000000u, 0x7440 + K + 1))),
                      f2(-8388608.0f));
}

// PACK: 0 the NCHW RGB only; 1 also the head's map of the same pixels; 2 also the head's map of
// the 2x pixel-unshuffled pixels (PreMap)
template <typename T, int TAPS, int PACK>
__global__ void __launch_bounds__(256, 4) k_pre_roll(const uint8_t *yp, ptrdiff_t ys, const uint8_t *uvp, ptrdiff_t uvs,
                                                     PreRoll pr, aji_csp csp, __half *dst, PreMap pm)
{
    extern __shared__ __align__(16) unsigned char prs_smem[];
    PreRollSmem<T> &sm = *reinterpret_cast<PreRollSmem<T> *>(prs_smem);
    constexpr int kPpc = 16 / (2 * (int)sizeof(T));  // (u, v) pairs per 16-byte piece
    constexpr int kUvChunks = kPrCW / kPpc;          // pieces per staged chroma row
    constexpr int kYChunks = kPrCols * (int)sizeof(T) / 16;
    const int tid = threadIdx.x;
    const int w = pr.w, h = pr.h, cw = pr.cw, ch = pr.ch;
    const int x0 = blockIdx.x * kPrCols;
    const int ya = blockIdx.y * pr.seg, yb = min(ya + pr.seg, h);
    const int mv = min(pr.sv0, pr.sv1);
    const int ca = (x0 / 2 + min(pr.sh0, pr.sh1)) & ~(kPpc - 1);  // the window's first chroma column
    const int cbase = ya / 2 + mv;                                 // chroma row of relative row 0
    const int npro = TAPS - 1 + abs(pr.sv1 - pr.sv0);              // chroma rows staged before step 0
    const int nsteps = (yb - ya + kPrG - 1) / kPrG;
    const size_t plane = (size_t)w * h;

    // chroma staging: piece tid % kUvChunks of new row tid / kUvChunks (eight rows a step)
    const int ur = tid / kUvChunks, uj = tid - ur * kUvChunks, ucol = ca + uj * kPpc;
    const bool uin = ucol >= 0 && ucol + kPpc <= cw;  // inside the frame: copied; else mirrored loads
    auto stage_uv = [&](int crel0, int n) {
        if (ur >= n || !uin) return;
        const int crel = crel0 + ur;
        const T *row = reinterpret_cast<const T *>(uvp + (size_t)mirror_index(cbase + crel, ch) * uvs);
        cp_async16(&sm.uvraw[crel & (kPrCR - 1)][2 * uj * kPpc], row + 2 * ucol);
    };
    auto convert_uv = [&](int crel0, int n) {
        if (ur >= n) return;
        const int crel = crel0 + ur, slot = crel & (kPrCR - 1);
        float2 f[kPpc];
        if (uin) {
            const uint4 q = *reinterpret_cast<const uint4 *>(&sm.uvraw[slot][2 * uj * kPpc]);
            if constexpr (sizeof(T) == 2) {
                f[0] = u16x2_to_f2(q.x), f[1] = u16x2_to_f2(q.y), f[2] = u16x2_to_f2(q.z), f[3] = u16x2_to_f2(q.w);
            } else {
                f[0] = u8x2_to_f2<0>(q.x), f[1] = u8x2_to_f2<2>(q.x), f[2] = u8x2_to_f2<0>(q.y), f[3] = u8x2_to_f2<2>(q.y);
                f[4] = u8x2_to_f2<0>(q.z), f[5] = u8x2_to_f2<2>(q.z), f[6] = u8x2_to_f2<0>(q.w), f[7] = u8x2_to_f2<2>(q.w);
            }
        } else {
            const T *row = reinterpret_cast<const T *>(uvp + (size_t)mirror_index(cbase + crel, ch) * uvs);
#pragma unroll
            for (int k = 0; k < kPpc; k++) {
                const int c = mirror_index(ucol + k, cw);
                f[k] = make_float2((float)row[2 * c], (float)row[2 * c + 1]);
            }
        }
#pragma unroll
        for (int k = 0; k < kPpc; k += 2)
            *reinterpret_cast<float4 *>(&sm.uvf[slot][uj * kPpc + k]) = make_float4(f[k].x, f[k].y, f[k + 1].x, f[k + 1].y);
    };
    // luma staging: piece tid % kYChunks of row tid / kYChunks of the step
    const int yr = tid / kYChunks, yj = tid - yr * kYChunks;
    const bool ycopy = yr < kPrG && x0 + (yj + 1) * (16 / (int)sizeof(T)) <= w;
    auto stage_y = [&](int s) {
        const int y = ya + kPrG * s + yr;
        if (!ycopy || y >= h) return;
        cp_async16(&sm.yraw[(kPrG * s + yr) & (kPrYR - 1)][yj * (16 / sizeof(T))],
                   reinterpret_cast<const T *>(yp + (size_t)y * ys) + x0 + yj * (16 / sizeof(T)));
    };
    // horizontal pass: luma columns x0 + 2k and + 1 (k = tid & 63), new chroma rows tid >> 6, + 4
    const int hk = tid & 63;
    const int hbe = x0 / 2 + pr.sh0 + hk - ca, hbo = x0 / 2 + pr.sh1 + hk - ca;
    auto horizontal = [&](int crel0, int n) {
        for (int r = tid >> 6; r < n; r += 4) {
            const int slot = (crel0 + r) & (kPrCR - 1);
            const float2 *f = sm.uvf[slot];
            float2 e = make_float2(0.0f, 0.0f), o = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int j = 0; j < TAPS; j++) {
                e = __ffma2_rn(f2(pr.whe[j]), f[hbe + j], e);
                o = __ffma2_rn(f2(pr.who[j]), f[hbo + j], o);
            }
            *reinterpret_cast<float4 *>(&sm.hr[slot][2 * hk]) = make_float4(e.x, e.y, o.x, o.y);
        }
    };
    // vertical pass + matrix + stores: pixels (x0 + 2k, + 1), k = tid & 63, luma rows
    // 4 (tid >> 6) .. + 3 of the step
    const int vk = tid & 63, vx = x0 + 2 * vk, vg = tid >> 6;
    const float kg = __fsub_rn(__fsub_rn(1.0f, csp.kr), csp.kb);
    const float cr = __fmul_rn(2.0f, __fsub_rn(1.0f, csp.kr));
    const float cb = __fmul_rn(2.0f, __fsub_rn(1.0f, csp.kb));
    const float gb = __fmul_rn(__fmul_rn(2.0f, csp.kb), __fsub_rn(1.0f, csp.kb));
    const float gr = __fmul_rn(__fmul_rn(2.0f, csp.kr), __fsub_rn(1.0f, csp.kr));
    const float ry = __frcp_rn(csp.yscale), rc = __frcp_rn(csp.cscale);
    auto vertical = [&](int s) {
        if (vx >= w) return;
        __half2 er, eg, eb;  // PACK 2: the (even) upper row of the pair the odd row completes
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int yrel = kPrG * s + 4 * vg + i, y = ya + yrel;
            if (y >= yb) break;
            const int c0 = ((i & 1) ? pr.sv1 : pr.sv0) - mv + (yrel >> 1);  // relative row of tap 0
            float2 a0 = make_float2(0.0f, 0.0f), a1 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int j = 0; j < TAPS; j++) {
                const float4 q = *reinterpret_cast<const float4 *>(&sm.hr[(c0 + j) & (kPrCR - 1)][2 * vk]);
                const float wj = (i & 1) ? pr.wvo[j] : pr.wve[j];
                a0 = __ffma2_rn(f2(wj), make_float2(q.x, q.y), a0);
                a1 = __ffma2_rn(f2(wj), make_float2(q.z, q.w), a1);
            }
            float2 raw;
            if constexpr (sizeof(T) == 2)
                raw = u16x2_to_f2(*reinterpret_cast<const uint32_t *>(&sm.yraw[yrel & (kPrYR - 1)][2 * vk]));
            else
                raw = u8x2_to_f2<0>(*reinterpret_cast<const uint16_t *>(&sm.yraw[yrel & (kPrYR - 1)][2 * vk]));
            const float2 Y = div_by2(__fadd2_rn(raw, f2(-csp.yoff)), csp.yscale, ry);
            const float2 uv0 = div_by2(__fadd2_rn(a0, f2(-csp.coff)), csp.cscale, rc);  // (U, V) of pixel 0
            const float2 uv1 = div_by2(__fadd2_rn(a1, f2(-csp.coff)), csp.cscale, rc);
            const float2 U = make_float2(uv0.x, uv1.x), V = make_float2(uv0.y, uv1.y);
            const float2 r = __ffma2_rn(f2(cr), V, Y);
            const float2 b = __ffma2_rn(f2(cb), U, Y);
            const float2 gn = __ffma2_rn(f2(gb), U, __fmul2_rn(f2(gr), V));
            const float2 g = make_float2(__fsub_rn(Y.x, __fdiv_rn(gn.x, kg)), __fsub_rn(Y.y, __fdiv_rn(gn.y, kg)));
            const __half2 hr = __floats2half2_rn(r.x, r.y), hg = __floats2half2_rn(g.x, g.y),
                          hb = __floats2half2_rn(b.x, b.y);
            const size_t idx = (size_t)y * w + vx;
            *reinterpret_cast<__half2 *>(dst + idx) = hr;
            *reinterpret_cast<__half2 *>(dst + plane + idx) = hg;
            *reinterpret_cast<__half2 *>(dst + 2 * plane + idx) = hb;
            if constexpr (PACK == 1) {
#pragma unroll
                for (int p = 0; p < 2; p++) {
                    float v[3] = {p ? __high2float(hr) : __low2float(hr), p ? __high2float(hg) : __low2float(hg),
                                  p ? __high2float(hb) : __low2float(hb)};
                    if (pm.in_norm) {
#pragma unroll
                        for (int c = 0; c < 3; c++) v[c] = (v[c] - pm.mean[c]) * pm.scale[c];
                    }
                    store_px(pm.map, y, vx + p, 0, pm.nstrips, 1,
                             make_uint4(pack_h2(v[0], v[1]), pack_h2(v[2], 0.f), 0u, 0u));
                }
            } else if constexpr (PACK == 2) {
                // a run and every step start on an even row (seg and kPrG are even) and end on an
                // odd one (h is even), so rows i = 0, 1 and i = 2, 3 are the two rows of the
                // unshuffled pixel (y / 2, vx / 2): its word (c, ry) holds columns vx, vx + 1
                if (!(i & 1)) {
                    er = hr, eg = hg, eb = hb;
                } else {
                    __half2 q[6] = {er, hr, eg, hg, eb, hb};
                    if (pm.in_norm) {
#pragma unroll
                        for (int j = 0; j < 6; j++) {
                            const float2 f = __half22float2(q[j]);
                            const float m = pm.mean[j >> 1], sc = pm.scale[j >> 1];
                            q[j] = __floats2half2_rn((f.x - m) * sc, (f.y - m) * sc);
                        }
                    }
                    const uint32_t *u = reinterpret_cast<const uint32_t *>(q);
                    store_px(pm.map, y >> 1, vx >> 1, 0, pm.nstrips, 2, make_uint4(u[0], u[1], u[2], u[3]));
                    store_px(pm.map, y >> 1, vx >> 1, 1, pm.nstrips, 2, make_uint4(u[4], u[5], 0u, 0u));
                }
            }
        }
    };

    stage_uv(0, npro);
    cp_async_commit();
    for (int s = -1;; s++) {
        const int crel0 = s < 0 ? 0 : npro + (kPrG / 2) * s, n = s < 0 ? npro : kPrG / 2;
        cp_async_wait<0>();
        convert_uv(crel0, n);
        __syncthreads();
        if (s + 1 < nsteps) {
            stage_uv(npro + (kPrG / 2) * (s + 1), kPrG / 2);
            stage_y(s + 1);
        }
        cp_async_commit();
        horizontal(crel0, n);
        __syncthreads();
        if (s >= 0) vertical(s);
        if (s + 1 >= nsteps) break;
    }
}

// ---------------- resize: fp16 NCHW RGB -> fp16 NCHW RGB (Spline36) ----------------
// The reference's k_rs_h + k_rs_v (src/kernels.cu:322-354) in one kernel: a tile of 32 x 16
// output pixels of one plane runs the horizontal pass for the (mirrored) source rows its
// vertical taps read into shared memory, then the vertical pass; each pass accumulates
// fma(weight, sample, sum) in tap order in fp32 as the reference's, one rounding to fp16.
constexpr int kRsTW = 32, kRsTH = 16;

__global__ void __launch_bounds__(256) k_resize(const __half *src, int sw, int sh, DevPass ph, DevPass pv, __half *dst)
{
    extern __shared__ float rs_sm[];  // [rows][kRsTW]
    const int c = blockIdx.z, tx = threadIdx.x, ty = threadIdx.y;
    const int dw = ph.dst, dh = pv.dst;
    const int x0 = blockIdx.x * kRsTW, y0 = blockIdx.y * kRsTH, x = x0 + tx;
    const int ylo = pv.start[y0], yl = min(y0 + kRsTH, dh) - 1, nrows = pv.start[yl] + pv.taps - ylo;
    const __half *plane = src + (size_t)c * sw * sh;
    if (x < dw) {
        const float *wt = ph.wt + (size_t)x * ph.taps;
        const int s0 = ph.start[x];
        for (int rr = ty; rr < nrows; rr += blockDim.y) {
            const __half *row = plane + (size_t)mirror_index(ylo + rr, sh) * sw;
            float a = 0.0f;
            for (int j = 0; j < ph.taps; j++) a = __fmaf_rn(wt[j], __half2float(row[mirror_index(s0 + j, sw)]), a);
            rs_sm[rr * kRsTW + tx] = a;
        }
    }
    __syncthreads();
    if (x >= dw) return;
    for (int yy = ty; yy < kRsTH; yy += blockDim.y) {
        const int y = y0 + yy;
        if (y >= dh) break;
        const float *wt = pv.wt + (size_t)y * pv.taps;
        const int s0 = pv.start[y] - ylo;
        float a = 0.0f;
        for (int j = 0; j < pv.taps; j++) a = __fmaf_rn(wt[j], rs_sm[(s0 + j) * kRsTW + tx], a);
        dst[(size_t)c * dw * dh + (size_t)y * dw + x] = __float2half_rn(a);
    }
}

// ---------------- 4:4:4 16-bit planar, matrix only ----------------
__global__ void k_post444(const __half *src, int w, int h, aji_csp csp, float qdiv, float qmax, uint8_t *yp,
                          ptrdiff_t ys, uint8_t *cbp, ptrdiff_t cbs, uint8_t *crp, ptrdiff_t crs)
{
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y * blockDim.y + threadIdx.y;
    if (x >= w || y >= h) return;
    const float qinv = __frcp_rn(qdiv);
    const size_t plane = (size_t)w * h, idx = (size_t)y * w + x;
    const float r = __half2float(src[idx]), g = __half2float(src[plane + idx]), b = __half2float(src[2 * plane + idx]);
    const float kg = __fsub_rn(__fsub_rn(1.0f, csp.kr), csp.kb);
    const float Y = __fmaf_rn(csp.kb, b, __fmaf_rn(csp.kr, r, __fmul_rn(kg, g)));
    const float U = __fdiv_rn(__fsub_rn(b, Y), __fmul_rn(2.0f, __fsub_rn(1.0f, csp.kb)));
    const float V = __fdiv_rn(__fsub_rn(r, Y), __fmul_rn(2.0f, __fsub_rn(1.0f, csp.kr)));
    reinterpret_cast<uint16_t *>(yp + (size_t)y * ys)[x] = (uint16_t)quantize(__fmaf_rn(Y, csp.yscale, csp.yoff), qdiv, qinv, qmax);
    reinterpret_cast<uint16_t *>(cbp + (size_t)y * cbs)[x] = (uint16_t)quantize(__fmaf_rn(U, csp.cscale, csp.coff), qdiv, qinv, qmax);
    reinterpret_cast<uint16_t *>(crp + (size_t)y * crs)[x] = (uint16_t)quantize(__fmaf_rn(V, csp.cscale, csp.coff), qdiv, qinv, qmax);
}

__global__ void k_pre444(const uint8_t *yp, ptrdiff_t ys, const uint8_t *cbp, ptrdiff_t cbs, const uint8_t *crp,
                         ptrdiff_t crs, int w, int h, aji_csp csp, __half *dst)
{
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y * blockDim.y + threadIdx.y;
    if (x >= w || y >= h) return;
    const size_t plane = (size_t)w * h, idx = (size_t)y * w + x;
    const float Y = __fdiv_rn(__fsub_rn((float)reinterpret_cast<const uint16_t *>(yp + (size_t)y * ys)[x], csp.yoff), csp.yscale);
    const float U = __fdiv_rn(__fsub_rn((float)reinterpret_cast<const uint16_t *>(cbp + (size_t)y * cbs)[x], csp.coff), csp.cscale);
    const float V = __fdiv_rn(__fsub_rn((float)reinterpret_cast<const uint16_t *>(crp + (size_t)y * crs)[x], csp.coff), csp.cscale);
    const float kg = __fsub_rn(__fsub_rn(1.0f, csp.kr), csp.kb);
    const float cr = __fmul_rn(2.0f, __fsub_rn(1.0f, csp.kr)), cb = __fmul_rn(2.0f, __fsub_rn(1.0f, csp.kb));
    const float gb = __fmul_rn(__fmul_rn(2.0f, csp.kb), __fsub_rn(1.0f, csp.kb));
    const float gr = __fmul_rn(__fmul_rn(2.0f, csp.kr), __fsub_rn(1.0f, csp.kr));
    dst[idx] = __float2half_rn(__fmaf_rn(cr, V, Y));
    dst[2 * plane + idx] = __float2half_rn(__fmaf_rn(cb, U, Y));
    dst[plane + idx] = __float2half_rn(__fsub_rn(Y, __fdiv_rn(__fmaf_rn(gb, U, __fmul_rn(gr, V)), kg)));
}

bool upload_pass(DevPass *d, const FilterTable &t)
{
    int *s = nullptr;
    float *w = nullptr;
    if (cudaMalloc(&s, t.start.size() * sizeof(int)) != cudaSuccess) return false;
    if (cudaMalloc(&w, t.wt.size() * sizeof(float)) != cudaSuccess) {
        cudaFree(s);
        return false;
    }
    if (cudaMemcpy(s, t.start.data(), t.start.size() * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(w, t.wt.data(), t.wt.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(s);
        cudaFree(w);
        return false;
    }
    d->taps = t.taps;
    d->src = t.src;
    d->dst = t.dst;
    d->start = s;
    d->wt = w;
    d->step2 = 1;
    for (size_t i = 1; i < t.start.size(); i++)
        if (t.start[i] != t.start[0] + 2 * (int)i) d->step2 = 0;
    return true;
}

// largest number of source indices a tile of `tile` consecutive outputs spans
int span_of(const FilterTable &t, int tile)
{
    int m = 0;
    for (int i0 = 0; i0 < t.dst; i0 += tile) {
        const int i1 = std::min(i0 + tile, t.dst) - 1;
        m = std::max(m, t.start[i1] + t.taps - t.start[i0]);
    }
    return m;
}

int host_mirror(int i, int n)
{
    i = i < 0 ? -i - 1 : i;
    i = i >= n ? 2 * n - 1 - i : i;
    return std::min(std::max(i, 0), n - 1);
}

// Whether k_post_roll serves a post plan: 2:1 tables of the same tap count (12 for Spline36, 4 for
// bilinear) with one set of weights each and first taps in [2 - taps, 0] (so the staged rows and
// columns reach every own pixel), a width that is a multiple of 8 (every 16-byte piece of a row is
// wholly inside or outside the frame), and, for every strip, each mirrored column its real outputs
// read inside its staged window. Sets the launch (PostRoll, grid) when it does.
template <typename T, int TAPS>
bool post_roll_setup(aji_plan *p)
{
    const FilterTable &th = p->th, &tv = p->tv;
    if (th.taps != TAPS || tv.taps != TAPS || p->w % 8 != 0) return false;
    for (const FilterTable *t : {&th, &tv}) {
        if (t->start[0] > 0 || t->start[0] < 2 - TAPS) return false;
        for (int i = 0; i < t->dst; i++) {
            if (t->start[i] != t->start[0] + 2 * i) return false;
            if (std::memcmp(&t->wt[(size_t)i * TAPS], t->wt.data(), TAPS * sizeof(float)) != 0) return false;
        }
    }
    const int cw = p->w / 2, ch = p->h / 2;
    for (int cx0 = 0; cx0 < cw; cx0 += kPsCols) {
        const int cxl = std::min(cx0 + kPsCols, cw) - 1, xlo = 2 * cx0 + th.start[0], xa = xlo & ~7;
        for (int gx = xlo; gx <= 2 * cxl + th.start[0] + TAPS - 1; gx++) {
            const int mx = host_mirror(gx, p->w);
            if (mx < xa || mx - xa >= kPsLW) return false;
        }
    }
    // blocks: the strips times runs of chroma rows, about as many as fit on the device at once
    int dev = 0, sms = 0, per_sm = 0;
    const size_t smem = sizeof(PostRollSmem);
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaFuncSetAttribute(k_post_roll<T, TAPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_post_roll<T, TAPS>, 256, smem) != cudaSuccess ||
        per_sm < 1)
        return false;
    const int nstrips = (cw + kPsCols - 1) / kPsCols;
    const int nseg = std::max(1, sms * per_sm / nstrips);
    const int seg = ((ch + nseg - 1) / nseg + kPsG - 1) / kPsG * kPsG;
    PostRoll &r = p->roll;
    r.w = p->w;
    r.h = p->h;
    r.cw = cw;
    r.ch = ch;
    r.oh = th.start[0];
    r.ov = tv.start[0];
    r.seg = seg;
    for (int j = 0; j < kPostMaxTaps; j++) {
        r.wh[j] = j < TAPS ? th.wt[j] : 0.0f;
        r.wv[j] = j < TAPS ? tv.wt[j] : 0.0f;
    }
    p->roll_grid = dim3(nstrips, (ch + seg - 1) / seg);
    p->roll_taps = TAPS;
    return true;
}

// Whether k_pre_roll serves a pre plan: 2x tables of the same tap count (6 for Spline36, 2 for
// bilinear) with period 2 (output i + 2 starts one sample after output i, with its weights) and
// outputs 0 and 1 starting at most one sample apart, a width that is a multiple of 16 (every
// 16-byte piece of a luma or chroma row is wholly inside or outside the frame), and every tap of
// a strip's real outputs inside its staged window. Sets the launch (PreRoll, grid) when it does.
template <typename T, int TAPS, int PACK>
bool pre_roll_occupancy(int *per_sm)
{
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, k_pre_roll<T, TAPS, PACK>, 256,
                                                         sizeof(PreRollSmem<T>)) == cudaSuccess;
}

template <typename T, int TAPS>
bool pre_roll_setup(aji_plan *p)
{
    const FilterTable &th = p->th, &tv = p->tv;
    if (th.taps != TAPS || tv.taps != TAPS || p->w % 16 != 0 || th.dst < 2 || tv.dst < 2) return false;
    for (const FilterTable *t : {&th, &tv}) {
        if (std::abs(t->start[1] - t->start[0]) > 1) return false;
        for (int i = 2; i < t->dst; i++) {
            if (t->start[i] != t->start[i - 2] + 1) return false;
            if (std::memcmp(&t->wt[(size_t)i * TAPS], &t->wt[(size_t)(i - 2) * TAPS], TAPS * sizeof(float)) != 0)
                return false;
        }
    }
    constexpr int kPpc = 16 / (2 * (int)sizeof(T));
    const int cw = p->w / 2, ch = p->h / 2;
    for (int x0 = 0; x0 < p->w; x0 += kPrCols) {
        const int ca = (x0 / 2 + std::min(th.start[0], th.start[1])) & ~(kPpc - 1);
        for (int x = x0; x < std::min(x0 + kPrCols, p->w); x++)
            if (th.start[x] < ca || th.start[x] + TAPS > ca + kPrCW) return false;
    }
    int dev = 0, sms = 0, per_sm = 0, per_sm_pack = 0, per_sm_unsh = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        !pre_roll_occupancy<T, TAPS, 0>(&per_sm) || !pre_roll_occupancy<T, TAPS, 1>(&per_sm_pack) ||
        !pre_roll_occupancy<T, TAPS, 2>(&per_sm_unsh))
        return false;
    per_sm = std::min(per_sm, std::min(per_sm_pack, per_sm_unsh));
    if (per_sm < 1) return false;
    const int nstrips = (p->w + kPrCols - 1) / kPrCols;
    const int nseg = std::max(1, sms * per_sm / nstrips);
    const int seg = ((p->h + nseg - 1) / nseg + kPrG - 1) / kPrG * kPrG;
    PreRoll &r = p->proll;
    r.w = p->w;
    r.h = p->h;
    r.cw = cw;
    r.ch = ch;
    r.sh0 = th.start[0];
    r.sh1 = th.start[1];
    r.sv0 = tv.start[0];
    r.sv1 = tv.start[1];
    r.seg = seg;
    for (int j = 0; j < 8; j++) {
        r.whe[j] = j < TAPS ? th.wt[j] : 0.0f;
        r.who[j] = j < TAPS ? th.wt[TAPS + j] : 0.0f;
        r.wve[j] = j < TAPS ? tv.wt[j] : 0.0f;
        r.wvo[j] = j < TAPS ? tv.wt[TAPS + j] : 0.0f;
    }
    p->roll_grid = dim3(nstrips, (p->h + seg - 1) / seg);
    p->roll_taps = TAPS;
    return true;
}

aji_plan *plan_create(aji_plan::Kind kind, int format, int w, int h, int siting, int filter)
{
    if ((format != AJI_FMT_NV12 && format != AJI_FMT_P010) || w < 2 || h < 2 || (w & 1) || (h & 1)) return nullptr;
    auto *p = new (std::nothrow) aji_plan();
    if (!p) return nullptr;
    p->kind = kind;
    p->format = format;
    p->w = w;
    p->h = h;
    const int cw = w / 2, ch = h / 2;
    double sx, sy;
    chroma_shift(siting, kind == aji_plan::PRE, &sx, &sy);
    if (kind == aji_plan::PRE) {
        p->th = make_filter(cw, w, sx, filter);
        p->tv = make_filter(ch, h, sy, filter);
        p->max_rows = span_of(p->tv, kPreTH);
        if (p->max_rows > kPreRows || p->th.taps > kPreMaxTaps || p->tv.taps > kPreMaxTaps) {
            delete p;
            return nullptr;
        }
        if (format == AJI_FMT_P010) {
            if (!pre_roll_setup<uint16_t, 6>(p)) pre_roll_setup<uint16_t, 2>(p);
        } else {
            if (!pre_roll_setup<uint8_t, 6>(p)) pre_roll_setup<uint8_t, 2>(p);
        }
    } else {
        p->th = make_filter(w, cw, sx, filter);
        p->tv = make_filter(h, ch, sy, filter);
        p->max_rows = span_of(p->tv, kPostTH);
        p->max_cols = span_of(p->th, kPostTW);
        if (p->max_rows > kPostRows || p->max_cols > kPostCols || p->th.taps > kPostMaxTaps || p->tv.taps > kPostMaxTaps) {
            delete p;
            return nullptr;
        }
        if (format == AJI_FMT_P010) {
            if (!post_roll_setup<uint16_t, 12>(p)) post_roll_setup<uint16_t, 4>(p);
        } else {
            if (!post_roll_setup<uint8_t, 12>(p)) post_roll_setup<uint8_t, 4>(p);
        }
    }
    if (!upload_pass(&p->ph, p->th) || !upload_pass(&p->pv, p->tv)) {
        aji_plan_destroy(p);
        return nullptr;
    }
    return p;
}

}  // namespace

extern "C" aji_plan *aji_pre_plan_create(int format, int w, int h, int siting, int filter)
{
    return plan_create(aji_plan::PRE, format, w, h, siting, filter);
}

extern "C" aji_plan *aji_post_plan_create(int format, int w, int h, int siting, int filter)
{
    return plan_create(aji_plan::POST, format, w, h, siting, filter);
}

extern "C" aji_plan *aji_resize_plan_create(int sw, int sh, int dw, int dh)
{
    if (sw < 1 || sh < 1 || dw < 1 || dh < 1) return nullptr;
    auto *p = new (std::nothrow) aji_plan();
    if (!p) return nullptr;
    p->kind = aji_plan::RESIZE;
    p->w = sw;
    p->h = sh;
    p->dw = dw;
    p->dh = dh;
    p->th = make_filter(sw, dw, 0.0, kFilterSpline36);
    p->tv = make_filter(sh, dh, 0.0, kFilterSpline36);
    p->max_rows = span_of(p->tv, kRsTH);
    // the tile's staged rows must fit the shared memory of one block (downscales beyond ~16x do not)
    if ((size_t)p->max_rows * kRsTW * sizeof(float) > 96 * 1024 || !upload_pass(&p->ph, p->th) ||
        !upload_pass(&p->pv, p->tv)) {
        aji_plan_destroy(p);
        return nullptr;
    }
    return p;
}

extern "C" int aji_run_resize(aji_plan *p, const void *src_f16, void *dst_f16, void *stream)
{
    if (!p || p->kind != aji_plan::RESIZE || !src_f16 || !dst_f16) return (int)cudaErrorInvalidValue;
    const size_t smem = (size_t)p->max_rows * kRsTW * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(k_resize, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    const dim3 grid((p->dw + kRsTW - 1) / kRsTW, (p->dh + kRsTH - 1) / kRsTH, 3), block(kRsTW, 8);
    k_resize<<<grid, block, smem, (cudaStream_t)stream>>>((const __half *)src_f16, p->w, p->h, p->ph, p->pv,
                                                         (__half *)dst_f16);
    return (int)cudaGetLastError();
}

extern "C" void aji_plan_destroy(aji_plan *p)
{
    if (!p) return;
    cudaFree((void *)p->ph.start);
    cudaFree((void *)p->ph.wt);
    cudaFree((void *)p->pv.start);
    cudaFree((void *)p->pv.wt);
    delete p;
}

extern "C" int ajib_filter_table(int src, int dst, double shift, int filter, int *start, float *wt)
{
    if (src < 1 || dst < 1) return -1;
    const FilterTable t = make_filter(src, dst, shift, filter);
    if (start && wt) {
        std::memcpy(start, t.start.data(), t.start.size() * sizeof(int));
        std::memcpy(wt, t.wt.data(), t.wt.size() * sizeof(float));
    }
    return t.taps;
}

extern "C" int ajib_plan_table(const aji_plan *p, int which, int *start, float *wt, int max_dst)
{
    if (!p) return -1;
    const FilterTable &t = which ? p->tv : p->th;
    const int n = std::min(max_dst, t.dst);
    if (start) std::memcpy(start, t.start.data(), n * sizeof(int));
    if (wt) std::memcpy(wt, t.wt.data(), (size_t)n * t.taps * sizeof(float));
    return t.taps;
}

extern "C" int ajib_plan_kernel(const aji_plan *p)
{
    if (!p) return -1;
    return p->roll_taps ? 1 : 0;
}

namespace {

template <typename T, int TAPS>
void launch_pre_roll(const aji_plan *p, const uint8_t *yp, ptrdiff_t ys, const uint8_t *uvp, ptrdiff_t uvs,
                     const aji_csp &csp, __half *dst, const PreMap *pm, cudaStream_t s)
{
    const size_t smem = sizeof(PreRollSmem<T>);
    if (pm && pm->unshuffle)
        k_pre_roll<T, TAPS, 2><<<p->roll_grid, 256, smem, s>>>(yp, ys, uvp, uvs, p->proll, csp, dst, *pm);
    else if (pm)
        k_pre_roll<T, TAPS, 1><<<p->roll_grid, 256, smem, s>>>(yp, ys, uvp, uvs, p->proll, csp, dst, *pm);
    else
        k_pre_roll<T, TAPS, 0><<<p->roll_grid, 256, smem, s>>>(yp, ys, uvp, uvs, p->proll, csp, dst, PreMap{});
}

int launch_pre(aji_plan *p, const void *y_plane, ptrdiff_t y_stride, const void *uv_plane, ptrdiff_t uv_stride,
               const aji_csp *csp, void *dst_f16, const PreMap *pm, cudaStream_t s)
{
    const dim3 grid((p->w + kPreTW - 1) / kPreTW, (p->h + kPreTH - 1) / kPreTH);
    const PreMap m = pm ? *pm : PreMap{};
    const uint8_t *yp = (const uint8_t *)y_plane, *uvp = (const uint8_t *)uv_plane;
    __half *dst = (__half *)dst_f16;
    // the streaming kernel copies 16-byte pieces of the luma and chroma rows and stores two
    // pixels of each output plane at once
    if (p->roll_taps && ((uintptr_t)y_plane & 15) == 0 && (y_stride & 15) == 0 && ((uintptr_t)uv_plane & 15) == 0 &&
        (uv_stride & 15) == 0 && y_stride > 0 && uv_stride > 0 && ((uintptr_t)dst_f16 & 3) == 0) {
        const bool p010 = p->format == AJI_FMT_P010;
        if (p010 && p->roll_taps == 6) launch_pre_roll<uint16_t, 6>(p, yp, y_stride, uvp, uv_stride, *csp, dst, pm, s);
        else if (p010) launch_pre_roll<uint16_t, 2>(p, yp, y_stride, uvp, uv_stride, *csp, dst, pm, s);
        else if (p->roll_taps == 6) launch_pre_roll<uint8_t, 6>(p, yp, y_stride, uvp, uv_stride, *csp, dst, pm, s);
        else launch_pre_roll<uint8_t, 2>(p, yp, y_stride, uvp, uv_stride, *csp, dst, pm, s);
        return (int)cudaGetLastError();
    }
    if (pm && pm->unshuffle) {
        // the tiled kernel writes no unshuffled map: the NCHW RGB, then the executor's own pack
        const int e = launch_pre(p, y_plane, y_stride, uv_plane, uv_stride, csp, dst_f16, nullptr, s);
        if (e != (int)cudaSuccess) return e;
        const int rc = ajib::pack_model_input(dst_f16, p->h / 2, p->w / 2, 1, pm->in_norm != 0, pm->mean, pm->scale, 0,
                                              p->h / 2, pm->map, s);
        return rc == AJIB_OK ? (int)cudaSuccess : rc == AJIB_ERR_CUDA ? (int)cudaErrorLaunchFailure : (int)cudaErrorInvalidValue;
    }
    if (p->format == AJI_FMT_NV12) {
        if (pm)
            k_pre<uint8_t, true><<<grid, 256, 0, s>>>(yp, y_stride, uvp, uv_stride, p->ph, p->pv, *csp, dst, p->w, p->h, m);
        else
            k_pre<uint8_t, false><<<grid, 256, 0, s>>>(yp, y_stride, uvp, uv_stride, p->ph, p->pv, *csp, dst, p->w, p->h, m);
    } else {
        if (pm)
            k_pre<uint16_t, true><<<grid, 256, 0, s>>>(yp, y_stride, uvp, uv_stride, p->ph, p->pv, *csp, dst, p->w, p->h, m);
        else
            k_pre<uint16_t, false><<<grid, 256, 0, s>>>(yp, y_stride, uvp, uv_stride, p->ph, p->pv, *csp, dst, p->w, p->h, m);
    }
    return (int)cudaGetLastError();
}

}  // namespace

extern "C" int aji_run_pre(aji_plan *p, const void *y_plane, ptrdiff_t y_stride, const void *uv_plane,
                           ptrdiff_t uv_stride, const aji_csp *csp, void *dst_f16, void *stream)
{
    if (!p || p->kind != aji_plan::PRE || !y_plane || !uv_plane || !csp || !dst_f16) return (int)cudaErrorInvalidValue;
    return launch_pre(p, y_plane, y_stride, uv_plane, uv_stride, csp, dst_f16, nullptr, (cudaStream_t)stream);
}

namespace ajib {

int run_pre_packed(aji_plan *p, const void *y_plane, ptrdiff_t y_stride, const void *uv_plane, ptrdiff_t uv_stride,
                   const aji_csp *csp, void *dst_f16, const InputPack &pk, cudaStream_t s)
{
    if (!p || p->kind != aji_plan::PRE || !y_plane || !uv_plane || !csp || !dst_f16 || !pk.map) return (int)cudaErrorInvalidValue;
    if (((uintptr_t)pk.map & 15) != 0) return (int)cudaErrorInvalidValue;
    PreMap m{};
    m.map = (__half *)pk.map;
    m.unshuffle = pk.unshuffle ? 1 : 0;
    m.nstrips = feature_strips(pk.unshuffle ? p->w / 2 : p->w);
    m.in_norm = pk.in_norm ? 1 : 0;
    for (int c = 0; c < 3; c++) {
        m.mean[c] = pk.mean[c];
        m.scale[c] = pk.scale[c];
    }
    return launch_pre(p, y_plane, y_stride, uv_plane, uv_stride, csp, dst_f16, &m, s);
}

}  // namespace ajib

extern "C" int aji_run_post(aji_plan *p, const void *src_f16, const aji_csp *csp, void *y_plane, ptrdiff_t y_stride,
                            void *uv_plane, ptrdiff_t uv_stride, void *stream)
{
    if (!p || p->kind != aji_plan::POST || !src_f16 || !csp || !y_plane || !uv_plane) return (int)cudaErrorInvalidValue;
    const int cw = p->w / 2, ch = p->h / 2;
    const dim3 grid((cw + kPostTW - 1) / kPostTW, (ch + kPostTH - 1) / kPostTH);
    const size_t smem = kPostSmem;
    cudaStream_t s = (cudaStream_t)stream;
    const bool p010 = p->format == AJI_FMT_P010;
    const float qdiv = p010 ? 64.0f : 1.0f, qmax = p010 ? 1023.0f : 255.0f;
    // the streaming kernel stores two samples at once and copies 16-byte pieces of the RGB rows
    const size_t pair = p010 ? 4 : 2;
    if (p->roll_taps && ((uintptr_t)src_f16 & 15) == 0 && ((uintptr_t)y_plane % pair) == 0 && (y_stride % pair) == 0 &&
        ((uintptr_t)uv_plane % pair) == 0 && (uv_stride % pair) == 0 && y_stride > 0 && uv_stride > 0) {
        const size_t smem = sizeof(PostRollSmem);
        const __half *in = (const __half *)src_f16;
        uint8_t *yo = (uint8_t *)y_plane, *uvo = (uint8_t *)uv_plane;
        if (p010 && p->roll_taps == 12)
            k_post_roll<uint16_t, 12><<<p->roll_grid, 256, smem, s>>>(in, p->roll, *csp, qdiv, qmax, yo, y_stride, uvo, uv_stride);
        else if (p010)
            k_post_roll<uint16_t, 4><<<p->roll_grid, 256, smem, s>>>(in, p->roll, *csp, qdiv, qmax, yo, y_stride, uvo, uv_stride);
        else if (p->roll_taps == 12)
            k_post_roll<uint8_t, 12><<<p->roll_grid, 256, smem, s>>>(in, p->roll, *csp, qdiv, qmax, yo, y_stride, uvo, uv_stride);
        else
            k_post_roll<uint8_t, 4><<<p->roll_grid, 256, smem, s>>>(in, p->roll, *csp, qdiv, qmax, yo, y_stride, uvo, uv_stride);
        return (int)cudaGetLastError();
    }
    cudaError_t e;
    if (p010) {
        e = cudaFuncSetAttribute(k_post<uint16_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return (int)e;
        k_post<uint16_t><<<grid, 256, smem, s>>>((const __half *)src_f16, p->w, p->h, p->ph, p->pv, *csp, qdiv, qmax,
                                                 (uint8_t *)y_plane, y_stride, (uint8_t *)uv_plane, uv_stride);
    } else {
        e = cudaFuncSetAttribute(k_post<uint8_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return (int)e;
        k_post<uint8_t><<<grid, 256, smem, s>>>((const __half *)src_f16, p->w, p->h, p->ph, p->pv, *csp, qdiv, qmax,
                                                (uint8_t *)y_plane, y_stride, (uint8_t *)uv_plane, uv_stride);
    }
    return (int)cudaGetLastError();
}

extern "C" int aji_run_post444(int format, int w, int h, const void *src_f16, const aji_csp *csp, void *y_plane,
                               ptrdiff_t y_stride, void *cb_plane, ptrdiff_t cb_stride, void *cr_plane,
                               ptrdiff_t cr_stride, void *stream)
{
    if (w < 1 || h < 1 || !src_f16 || !csp || !y_plane || !cb_plane || !cr_plane) return (int)cudaErrorInvalidValue;
    const float qdiv = format == AJI_FMT_YUV444P10MSB ? 64.0f : format == AJI_FMT_YUV444P12MSB ? 16.0f : 1.0f;
    const float qmax = format == AJI_FMT_YUV444P10MSB ? 1023.0f : format == AJI_FMT_YUV444P12MSB ? 4095.0f : 65535.0f;
    k_post444<<<dim3((w + 31) / 32, (h + 7) / 8), dim3(32, 8), 0, (cudaStream_t)stream>>>(
        (const __half *)src_f16, w, h, *csp, qdiv, qmax, (uint8_t *)y_plane, y_stride, (uint8_t *)cb_plane, cb_stride,
        (uint8_t *)cr_plane, cr_stride);
    return (int)cudaGetLastError();
}

extern "C" int aji_run_pre444(int w, int h, const void *y_plane, ptrdiff_t y_stride, const void *cb_plane,
                              ptrdiff_t cb_stride, const void *cr_plane, ptrdiff_t cr_stride, const aji_csp *csp,
                              void *dst_f16, void *stream)
{
    if (w < 1 || h < 1 || !y_plane || !cb_plane || !cr_plane || !csp || !dst_f16) return (int)cudaErrorInvalidValue;
    k_pre444<<<dim3((w + 31) / 32, (h + 7) / 8), dim3(32, 8), 0, (cudaStream_t)stream>>>(
        (const uint8_t *)y_plane, y_stride, (const uint8_t *)cb_plane, cb_stride, (const uint8_t *)cr_plane, cr_stride, w,
        h, *csp, (__half *)dst_f16);
    return (int)cudaGetLastError();
}
