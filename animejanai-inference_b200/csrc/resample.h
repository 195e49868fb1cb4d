/*
 * resample.h — host-side resampling tables and colour-space constants for the colour passes.
 *
 * The tables follow zimg's compute_filter, which is what VapourSynth's resize (the reference
 * pipeline the-database/animejanai-inference matches) uses; the reference restates it in
 * src/resample.h:53-84. Per output sample i: position (i + 0.5) / scale + shift in the source,
 * a kernel stretched by 1/scale when downscaling (step = min(scale, 1)), taps =
 * ceil(support / step) * 2, the first tap centred at round_half_up(pos - taps/2) + 0.5, weights
 * computed in double and normalised to sum 1, then stored as float. Spline36 is the published
 * piecewise cubic of the Spline36 kernel (support 3); bilinear is the triangle (support 1).
 * Out-of-range source indices are mirrored by the kernels (mirror_index below).
 *
 * The colour constants (Kr, Kb per matrix; offsets and scales in raw container units, P010
 * values being 10 bits in the high bits of 16) are the standard BT.601 / BT.709 / BT.2020
 * values in the reference's convention (src/resample.h:100-129).
 */
#pragma once

#include <cmath>
#include <vector>

#include "../../include/aji.h"

namespace ajib {

enum { kFilterSpline36 = 0, kFilterBilinear = 1 };

struct FilterTable {
    int taps = 0, src = 0, dst = 0;
    std::vector<int> start;  // [dst] first source index (before mirroring)
    std::vector<float> wt;   // [dst][taps]
};

inline double spline36_kernel(double x)
{
    x = std::fabs(x);
    if (x < 1.0) return ((13.0 / 11.0 * x - 453.0 / 209.0) * x - 3.0 / 209.0) * x + 1.0;
    if (x < 2.0) {
        const double t = x - 1.0;
        return ((-6.0 / 11.0 * t + 270.0 / 209.0) * t - 156.0 / 209.0) * t;
    }
    if (x < 3.0) {
        const double t = x - 2.0;
        return ((1.0 / 11.0 * t - 45.0 / 209.0) * t + 26.0 / 209.0) * t;
    }
    return 0.0;
}

inline double triangle_kernel(double x)
{
    x = std::fabs(x);
    return x < 1.0 ? 1.0 - x : 0.0;
}

inline FilterTable make_filter(int src, int dst, double shift, int filter)
{
    FilterTable t;
    const double scale = (double)dst / src;
    const double step = scale < 1.0 ? scale : 1.0;
    const double support = filter == kFilterBilinear ? 1.0 : 3.0;
    int taps = (int)std::ceil(support / step) * 2;
    if (taps < 1) taps = 1;
    t.taps = taps;
    t.src = src;
    t.dst = dst;
    t.start.resize(dst);
    t.wt.resize((size_t)dst * taps);
    std::vector<double> k(taps);
    for (int i = 0; i < dst; i++) {
        const double pos = (i + 0.5) / scale + shift;
        const double first = std::floor(pos - taps / 2.0 + 0.5) + 0.5;  // centre of tap 0
        double sum = 0.0;
        for (int j = 0; j < taps; j++) {
            const double d = (first + j - pos) * step;
            k[j] = filter == kFilterBilinear ? triangle_kernel(d) : spline36_kernel(d);
            sum += k[j];
        }
        t.start[i] = (int)(first - 0.5);
        for (int j = 0; j < taps; j++) t.wt[(size_t)i * taps + j] = (float)(k[j] / sum);
    }
    return t;
}

// Extra source-plane offset of the chroma grid relative to plain (i + 0.5) / scale mapping, in
// zimg's convention: 4:2:0 chroma up to the luma grid (up = true) or luma down to 4:2:0 chroma.
inline void chroma_shift(int siting, bool up, double *sx, double *sy)
{
    if (up) {
        *sx = siting == AJI_SITING_CENTER ? 0.0 : 0.25;
        *sy = siting == AJI_SITING_TOPLEFT ? 0.25 : 0.0;
    } else {
        *sx = siting == AJI_SITING_CENTER ? 0.0 : -0.5;
        *sy = siting == AJI_SITING_TOPLEFT ? -0.5 : 0.0;
    }
}

}  // namespace ajib
