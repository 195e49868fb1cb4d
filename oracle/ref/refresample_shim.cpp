// refresample_shim.cpp — C entry points over the reference's host resampling math
// (src/resample.h: compute, chroma_shifts, make_csp), compiled from the reference sources by
// build.sh into oracle/_ref/libref_resample.so. Test infrastructure only.
#include <cstring>

#include "resample.h"

extern "C" int ref_filter(int src, int dst, double shift, int filter, int *start, float *wt)
{
    const aji_resample::weights w = aji_resample::compute(src, dst, shift, filter);
    if (start) std::memcpy(start, w.start.data(), w.start.size() * sizeof(int));
    if (wt) std::memcpy(wt, w.wt.data(), w.wt.size() * sizeof(float));
    return w.taps;
}

extern "C" void ref_chroma_shifts(int siting, int up, double *sx, double *sy) { aji_resample::chroma_shifts(siting, up != 0, sx, sy); }

extern "C" void ref_make_csp(int format, int matrix, int range, float *out)
{
    const aji_csp c = aji_resample::make_csp(format, matrix, range);
    std::memcpy(out, &c, sizeof(c));
}
