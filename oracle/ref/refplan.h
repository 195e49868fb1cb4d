// refplan.h — the plan description the oracle/ref shims take over their C entry points, turned
// into the reference's own ajinative::Plan (src/native/lower.h:38-77). Shared by refnet_shim.cpp
// (the CPU reference net) and refexec_shim.cu (the reference's GPU executor). Test and baseline
// infrastructure only.
#pragma once

#include <cstdint>
#include <vector>

#include "native/lower.h"

struct ref_step {
    int kind, in, act, gate, out, cin, cout, src, resid, dst, c, nsrc, srcs[4], taps;
    const uint16_t *w;  // [taps][cin][cout]
    const float *bias;  // [cout]
    const float *slope; // [cout] or null
    const uint16_t *att_w;   // gate 2: the 1x1 attention conv [cout][cout], else null
    const float *att_bias;   // gate 2: [cout]
};

inline ajinative::Plan ref_plan_of(const ref_step *steps, int nsteps, const int *channels, int nfeat, int depth_to_space,
                                   int unshuffle)
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
    return p;
}
