// refnet_shim.cpp — a C entry point over the reference's own CPU reference net
// (sanity/native_ref.h, ajiref::run_plan), compiled from the reference sources by build.sh into
// oracle/_ref/libref_net.so. Test and baseline infrastructure only (see oracle.h).
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "native_ref.h"

struct ref_step {
    int kind, in, act, gate, out, cin, cout, src, resid, dst, c, nsrc, srcs[4], taps;
    const uint16_t *w;  // [taps][cin][cout]
    const float *bias;  // [cout]
    const float *slope; // [cout] or null
    const uint16_t *att_w;   // gate 2: the 1x1 attention conv [cout][cout], else null
    const float *att_bias;   // gate 2: [cout]
};

// in: NCHW [3][h][w]; out: NCHW [3][h * depth_to_space / unshuffle][w * depth_to_space / unshuffle]
extern "C" int ref_run_plan(const ref_step *steps, int nsteps, const int *channels, int nfeat, int depth_to_space,
                            int unshuffle, const float *in, int w, int h, float *out)
{
    ajinative::Plan p;
    p.unshuffle = unshuffle;
    p.depth_to_space = depth_to_space;
    p.channels.assign(channels, channels + nfeat);
    for (int i = 0; i < nsteps; i++) {
        const ref_step &r = steps[i];
        ajinative::PlanStep s;
        s.kind = r.kind ? ajinative::PlanStep::CONCAT : ajinative::PlanStep::CONV;
        s.in = r.in;
        s.act = r.act;
        s.gate = r.gate;
        s.out = r.out;
        s.cin = r.cin;
        s.cout = r.cout;
        s.src = r.src;
        s.resid = r.resid;
        s.dst = r.dst;
        s.c = r.c;
        s.nsrc = r.nsrc;
        for (int k = 0; k < 4; k++) s.srcs[k] = r.srcs[k];
        const int cin = r.kind ? r.nsrc * r.c : r.cin, cout = r.kind ? r.c : r.cout;
        s.w.taps = r.taps;
        s.w.cin = cin;
        s.w.cout = cout;
        s.w.w.assign(r.w, r.w + (size_t)r.taps * cin * cout);
        s.w.bias.assign(r.bias, r.bias + cout);
        if (r.slope) s.w.slope.assign(r.slope, r.slope + cout);
        if (r.att_w) {
            s.att.taps = 1;
            s.att.cin = s.att.cout = cout;
            s.att.w.assign(r.att_w, r.att_w + (size_t)cout * cout);
            s.att.bias.assign(r.att_bias, r.att_bias + cout);
        }
        p.steps.push_back(std::move(s));
    }
    std::vector<float> x(in, in + (size_t)3 * w * h);
    const std::vector<float> y = ajiref::run_plan(p, x, w, h);
    std::memcpy(out, y.data(), y.size() * sizeof(float));
    return 0;
}

extern "C" int ref_threads(void) { return (int)std::max(1u, std::thread::hardware_concurrency()); }
