// refnet_shim.cpp — a C entry point over the reference's own CPU reference net
// (sanity/native_ref.h, ajiref::run_plan), compiled from the reference sources by build.sh into
// oracle/_ref/libref_net.so. Test and baseline infrastructure only (see oracle.h).
#include <cstring>
#include <thread>

#include "native_ref.h"
#include "refplan.h"

// in: NCHW [3][h][w]; out: NCHW [3][h * depth_to_space / unshuffle][w * depth_to_space / unshuffle]
extern "C" int ref_run_plan(const ref_step *steps, int nsteps, const int *channels, int nfeat, int depth_to_space,
                            int unshuffle, const float *in, int w, int h, float *out)
{
    const ajinative::Plan p = ref_plan_of(steps, nsteps, channels, nfeat, depth_to_space, unshuffle);
    std::vector<float> x(in, in + (size_t)3 * w * h);
    const std::vector<float> y = ajiref::run_plan(p, x, w, h);
    std::memcpy(out, y.data(), y.size() * sizeof(float));
    return 0;
}

extern "C" int ref_threads(void) { return (int)std::max(1u, std::thread::hardware_concurrency()); }
