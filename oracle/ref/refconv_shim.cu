// refconv_shim.cu — C entry points over the reference's native conv kernels
// (src/native/conv.cu: upload, launch, tile_variant), compiled for sm_100a from the reference
// sources by build.sh into oracle/_ref/libref_conv.so: the GPU bar the new kernels are measured
// against (the reference's mma.sync kernels recompiled for B200). Test/benchmark infrastructure only.
#include <cstdint>

#include "native/conv.h"

using namespace ajinative;

extern "C" void *ref_conv_upload(const uint16_t *w, const float *bias, const float *slope, int cin, int cin_pad,
                                 int cout, int cout_pad)
{
    auto *wt = new Weights();
    if (upload(*wt, w, bias, slope, 9, cin, cin_pad, cout, cout_pad) != cudaSuccess) {
        delete wt;
        return nullptr;
    }
    return wt;
}

extern "C" void ref_conv_release(void *w)
{
    if (!w) return;
    release(*static_cast<Weights *>(w));
    delete static_cast<Weights *>(w);
}

// variant < 0: the reference's own tile pick (tile_variant)
extern "C" int ref_conv_launch(void *w, int in, int act, int gate, int out, int cin, int cout, const void *src,
                               const void *resid, void *dst, int H, int W, int variant, void *stream)
{
    Conv3x3 op;
    op.in = (Input)in;
    op.act = (Act)act;
    op.gate = (Gate)gate;
    op.out = (Output)out;
    op.cin = cin;
    op.cout = cout;
    op.w = static_cast<Weights *>(w);
    Tensors t;
    t.src = src;
    t.resid = resid;
    t.dst = dst;
    if (!supported(op)) return -1;
    const int v = variant < 0 ? tile_variant(op) : variant;
    return (int)launch(op, t, H, W, v, (cudaStream_t)stream);
}
