/*
 * conv.cu — host side of the fused conv kernels: weight packing and upload, TMA tensor maps,
 * shape checks, instantiation dispatch and launch (the C ABI in include/aji_b200.h).
 *
 * Counterparts in the reference: src/native/conv.cu (kConv table :60-61, key_of :89-147,
 * upload :183-204, launch :231-270) and src/native/pack.cpp (pack_fragments :9). The packing
 * here targets a different consumer: the tcgen05 B operand, K-major without swizzle, stored
 * per tap as [K/8 chunks][N/8 row groups][8 rows][8 fp16] so that one MMA's B (N x 16) is two
 * K-adjacent chunks at a fixed leading-byte offset.
 */
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <new>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "concat_tc.cuh"
#include "conv_pair.cuh"
#include "conv_tc.cuh"
#include "plan.h"
#include "../../include/aji_b200.h"

struct ajib_weights {
    void *img = nullptr;     // packed B image (9 or 1 taps)
    float *bias = nullptr;   // npad floats
    float *slope = nullptr;  // npad floats or null
    int taps = 0, cin = 0, cout = 0, kpad = 0, npad = 0;
    size_t bytes = 0;
};

namespace ajib {

int pad_k(int cin) { return cin <= 16 ? 16 : (cin + 15) / 16 * 16; }
// 3x3 outputs pad to 16, 32, 48 or 64 columns. 48 channels (SPAN, SPANF3) keep their width: a
// row's stacked-tap MMA is then N = 144 rather than 192 (a quarter fewer tensor cycles), and the
// accumulator ring's slots start on 16-column TMEM boundaries, as every MMA, load and store here
// addresses TMEM in 16-column units. Up to 16 channels (the 2x tails' 12, depth-to-space of RGB)
// pad to 16: N = 48 stacked-tap MMAs, and both epilogue warps of a lane quarter hold real
// channels (with 32 columns the second warp's were all padding).
int pad_n(int cout) { return cout <= 16 ? 16 : cout <= 32 ? 32 : cout == 48 ? 48 : 64; }

// The B operand image. 3x3 weights (taps == 9) are stacked by tap row so that one MMA covers all
// three vertical taps of a horizontal tap dx: [dx][kc][ty][ng][n8][k8], B row ty * npad + n of
// (dx, K chunk kc) holding w[tap ty * 3 + dx][kc * 8 + k8][n]. 1x1 weights: [kc][ng][n8][k8].
// Entries past cin / cout are zero.
std::vector<uint16_t> pack_b_image(const uint16_t *w, int taps, int cin, int cout, int kpad, int npad)
{
    const int KC = kpad / 8, NG = npad / 8;
    std::vector<uint16_t> img((size_t)taps * kpad * npad, 0);
    for (int t = 0; t < taps; t++) {
        const int ty = taps == 9 ? t / 3 : 0, dx = taps == 9 ? t % 3 : 0;
        for (int kc = 0; kc < KC; kc++)
            for (int ng = 0; ng < NG; ng++)
                for (int n8 = 0; n8 < 8; n8++)
                    for (int k8 = 0; k8 < 8; k8++) {
                        const int k = kc * 8 + k8, n = ng * 8 + n8;
                        if (k >= cin || n >= cout) continue;
                        const size_t at = taps == 9 ? ((((size_t)dx * KC + kc) * 3 + ty) * NG + ng) * 64 + n8 * 8 + k8
                                                    : (((size_t)kc * NG + ng) * 64) + n8 * 8 + k8;
                        img[at] = w[((size_t)t * cin + k) * cout + n];
                    }
    }
    return img;
}

// ---- per-device status word (kernels record pipeline timeouts here) ----
namespace {
std::mutex g_status_mu;
int *g_status[64] = {};
}  // namespace

int *status_word()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_status_mu);
    if (!g_status[dev]) {
        int *p = nullptr;
        if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
        if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) {
            cudaFree(p);
            return nullptr;
        }
        g_status[dev] = p;
    }
    return g_status[dev];
}

int sm_count()
{
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return 148;
    return n;
}

namespace {

using ConvFn = cudaError_t (*)(const ConvDev &, int grid, cudaStream_t);

// Launch with programmatic stream serialisation: the kernel's set-up (barriers, TMEM, weight fetch)
// may run while the previous kernel in the stream drains; the kernel waits (griddepcontrol.wait)
// before it touches that kernel's outputs.
// AJIB_PDL=0 in the environment launches without the attribute (plain stream order)
bool pdl_enabled()
{
    static const bool pdl = [] {
        const char *e = std::getenv("AJIB_PDL");
        return !(e && e[0] == '0');
    }();
    return pdl;
}

template <typename Arg>
cudaError_t launch_pdl(void (*kernel)(Arg), int grid, int threads, int smem, cudaStream_t s, const Arg &arg)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, arg);
}

// Whether strip-chunked convs run on SM pairs (k_conv3x3_pair) where a pair kernel exists: off
// unless AJIB_PAIR=1 in the environment or ajib_conv_pair_mode(1). (Measured on one B200, the
// 64-channel body conv: 0.138-0.147 ms on pairs against 0.129-0.134 ms on the one-SM kernel.)
std::atomic<int> g_pair_mode{-1};
int pair_mode()
{
    int m = g_pair_mode.load();
    if (m < 0) {
        const char *e = std::getenv("AJIB_PAIR");
        m = (e && e[0] == '1') ? 1 : 0;
        int expect = -1;
        g_pair_mode.compare_exchange_strong(expect, m);
        m = g_pair_mode.load();
    }
    return m;
}

using PairFn = cudaError_t (*)(const ConvDev &, long tiles, cudaStream_t);

// The pair kernel on clusters of two CTAs, as many pairs as the device holds at once (one CTA per
// SM), each pair a run of tiles.
template <int KPAD, int NPAD, int EK>
cudaError_t run_conv_pair(const ConvDev &p, long tiles, cudaStream_t s)
{
    using Cf = PairCfg<KPAD, NPAD>;
    constexpr int smem = Cf::SMEM;
    void (*kern)(ConvDev) = k_conv3x3_pair<KPAD, NPAD, EK>;
    static std::atomic<uint64_t> done{0};
    static std::atomic<int> pairs[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(Cf::THREADS);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(done.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        cfg.gridDim = dim3(2 * (sm_count() / 2));
        int n = 0;
        e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
        if (e != cudaSuccess) return e;
        if (n < 1) return cudaErrorLaunchOutOfResources;
        pairs[dev & 63].store(n);
        done.fetch_or(bit);
    }
    const long grid = std::min<long>(2L * pairs[dev & 63].load(), (tiles + 1) / 2 * 2);
    cfg.gridDim = dim3((unsigned)grid);
    return cudaLaunchKernelEx(&cfg, kern, p);
}

// The pair kernels built: strip-chunked input and output, cin == cout at 32, 48 and 64 padded
// channels with an activation, and at 32 and 48 with a SPAN gate (the body convs of Compact,
// SuperUltraCompact and SPAN; a 64-channel gate variant would spill registers).
PairFn find_pair_fn(int kpad, int npad, int ek)
{
#define AJIB_P(KP, NP, EK) \
    if (kpad == KP && npad == NP && ek == EK) return &run_conv_pair<KP, NP, EK>;
    AJIB_P(32, 32, kEpiAct)
    AJIB_P(48, 48, kEpiAct)
    AJIB_P(64, 64, kEpiAct)
    AJIB_P(32, 32, kEpiGate)
    AJIB_P(48, 48, kEpiGate)
#undef AJIB_P
    return nullptr;
}

template <int KPAD, int NPAD, int EK, int IN>
cudaError_t run_conv(const ConvDev &p, int grid, cudaStream_t s)
{
    using Cf = ConvCfg<KPAD, NPAD, EK == kEpiAtt, EK == kEpiD2S, EK == kEpiGate>;
    // at least half the SM's shared memory, so one CTA holds an SM and its whole TMEM (a second
    // CTA on the SM would only wait in its TMEM allocation)
    constexpr int smem = Cf::SMEM > 117 * 1024 ? Cf::SMEM : 117 * 1024;
    static_assert(Cf::SMEM <= kMaxSmem, "shared memory budget");
    // the shared-memory opt-in is per device: set it once on each
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(done.load() & bit)) {
        const cudaError_t attr =
            cudaFuncSetAttribute(k_conv3x3_tc<KPAD, NPAD, EK, IN>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (attr != cudaSuccess) return attr;
        done.fetch_or(bit);
    }
    return launch_pdl(k_conv3x3_tc<KPAD, NPAD, EK, IN>, grid, kConvThreads, smem, s, p);
}

// The kernel instantiation for padded channel counts, epilogue kind and input mode. Built: every
// K x N (N 16, 32, 48 or 64) with the activation and depth-to-space epilogues; the SPAN gates and
// the SPANF3 tanh gate (cin == cout) at the five K x N pairs that cin == cout gives; the NCHW RGB
// model input, plain or pixel-unshuffled by 2 (K 16 both), with activation or depth-to-space.
ConvFn find_fn(int kpad, int npad, int ek, int in)
{
#define AJIB_K(KP, NP, EK, IN) \
    if (kpad == KP && npad == NP && ek == EK && in == IN) return &run_conv<KP, NP, EK, IN>;
#define AJIB_KN(KP, EK) AJIB_K(KP, 16, EK, kInRows) AJIB_K(KP, 32, EK, kInRows) AJIB_K(KP, 48, EK, kInRows) \
    AJIB_K(KP, 64, EK, kInRows)
#define AJIB_SQ(EK) AJIB_K(16, 16, EK, kInRows) AJIB_K(16, 32, EK, kInRows) AJIB_K(32, 32, EK, kInRows) \
    AJIB_K(48, 48, EK, kInRows) AJIB_K(64, 64, EK, kInRows)
#define AJIB_RGB(IN) AJIB_K(16, 16, kEpiAct, IN) AJIB_K(16, 32, kEpiAct, IN) AJIB_K(16, 48, kEpiAct, IN) \
    AJIB_K(16, 64, kEpiAct, IN) AJIB_K(16, 16, kEpiD2S, IN) AJIB_K(16, 32, kEpiD2S, IN) AJIB_K(16, 48, kEpiD2S, IN) \
    AJIB_K(16, 64, kEpiD2S, IN)
    AJIB_KN(16, kEpiAct)
    AJIB_KN(32, kEpiAct)
    AJIB_KN(48, kEpiAct)
    AJIB_KN(64, kEpiAct)
    AJIB_KN(16, kEpiD2S)
    AJIB_KN(32, kEpiD2S)
    AJIB_KN(48, kEpiD2S)
    AJIB_KN(64, kEpiD2S)
    AJIB_SQ(kEpiGate)
    AJIB_SQ(kEpiAtt)
    AJIB_RGB(kInRgb)
    AJIB_RGB(kInRgbUnshuffle2)
#undef AJIB_RGB
#undef AJIB_SQ
#undef AJIB_KN
#undef AJIB_K
    return nullptr;
}

int epi_kind(const ajib_conv *op)
{
    if (op->out != AJIB_OUT_NHWC) return kEpiD2S;
    if (op->gate == AJIB_GATE_TANH1X1) return kEpiAtt;
    return op->gate != AJIB_GATE_NONE ? kEpiGate : kEpiAct;
}

int in_kind(const ajib_conv *op)
{
    return op->in == AJIB_IN_NCHW3 ? kInRgb : op->in == AJIB_IN_NCHW3_UNSHUFFLE2 ? kInRgbUnshuffle2 : kInRows;
}

ConvFn op_fn(const ajib_conv *op) { return find_fn(op->w->kpad, op->w->npad, epi_kind(op), in_kind(op)); }

// The pair kernel for the op when pairs are on and one is built for it, else null.
PairFn pair_fn(const ajib_conv *op)
{
    if (!pair_mode() || op->in != AJIB_IN_NHWC || op->out != AJIB_OUT_NHWC) return nullptr;
    const int ek = epi_kind(op);
    if (ek != kEpiAct && ek != kEpiGate) return nullptr;
    return find_pair_fn(op->w->kpad, op->w->npad, ek);
}

int d2s_factor(int out) { return out == 1 ? 2 : out == 2 ? 4 : out == 3 ? 1 : out == 4 ? 3 : 0; }

bool fail(char *why, size_t n, const char *msg)
{
    if (why && n) std::snprintf(why, n, "%s", msg);
    return false;
}

// The shape checks of the reference key_of (src/native/conv.cu:89-147), for this engine's kernels.
bool check(const ajib_conv *op, char *why, size_t n)
{
    if (!op) return fail(why, n, "no op");
    if (!op->w) return fail(why, n, "no weights");
    if (op->w->taps != 9) return fail(why, n, "weights are not 3x3");
    if (op->w->cin != op->cin || op->w->cout != op->cout) return fail(why, n, "weights do not match the op's channels");
    switch (op->in) {
    case AJIB_IN_NHWC:
        if (op->cin % 8 || op->cin < 8 || op->cin > 64) return fail(why, n, "NHWC input channels must be a multiple of 8, 8..64");
        break;
    case AJIB_IN_NCHW3:
        if (op->cin != 3) return fail(why, n, "NCHW3 input has 3 channels");
        break;
    case AJIB_IN_NCHW3_UNSHUFFLE2:
        if (op->cin != 12) return fail(why, n, "a pixel-unshuffled NCHW3 input has 12 channels");
        break;
    default:
        return fail(why, n, "unknown input mode");
    }
    switch (op->out) {
    case AJIB_OUT_NHWC:
        if (op->cout % 8 || op->cout < 8 || op->cout > 64) return fail(why, n, "NHWC output channels must be a multiple of 8, 8..64");
        break;
    case AJIB_OUT_D2S2:
        if (op->cout != 12) return fail(why, n, "depth-to-space 2 output has 12 channels");
        break;
    case AJIB_OUT_D2S4:
        if (op->cout != 48) return fail(why, n, "depth-to-space 4 output has 48 channels");
        break;
    case AJIB_OUT_D2S1:
        if (op->cout != 3) return fail(why, n, "depth-to-space 1 output has 3 channels");
        break;
    case AJIB_OUT_D2S3:
        if (op->cout != 27) return fail(why, n, "depth-to-space 3 output has 27 channels");
        break;
    default:
        return fail(why, n, "unknown output mode");
    }
    if (op->act < 0 || op->act > 3) return fail(why, n, "unknown activation");
    if (op->gate < 0 || op->gate > 3) return fail(why, n, "unknown gate");
    if (op->gate != AJIB_GATE_NONE) {
        if (op->act != AJIB_ACT_NONE) return fail(why, n, "gates take no activation");
        if (op->in != AJIB_IN_NHWC || op->out != AJIB_OUT_NHWC || op->cin != op->cout)
            return fail(why, n, "gates need NHWC input and output with cin == cout");
        if (op->gate == AJIB_GATE_TANH1X1) {
            const ajib_weights *t = op->att;
            if (!t || t->taps != 1 || t->cin != op->cout || t->cout != op->cout)
                return fail(why, n, "the tanh 1x1 gate needs 1x1 cout -> cout attention weights");
            if (t->kpad > op->w->npad || t->npad > op->w->npad) return fail(why, n, "attention weights wider than the conv");
        }
    }
    if (op->act == AJIB_ACT_PRELU && !op->w->slope) return fail(why, n, "PReLU without slopes");
    if (!op_fn(op)) return fail(why, n, "no kernel for these channel counts");
    return true;
}

}  // namespace
}  // namespace ajib

using namespace ajib;

extern "C" int ajib_weights_upload(ajib_weights **out, const uint16_t *w, const float *bias, const float *slope, int taps,
                                   int cin, int cout)
{
    if (!out || !w || !bias || (taps != 9 && taps != 1) || cin < 1 || cout < 1 || cin > 256 || cout > 64) return AJIB_ERR_ARGS;
    *out = nullptr;
    auto *r = new (std::nothrow) ajib_weights();
    if (!r) return AJIB_ERR_NO_MEM;
    r->taps = taps;
    r->cin = cin;
    r->cout = cout;
    r->kpad = taps == 9 ? pad_k(cin) : (cin + 15) / 16 * 16;
    r->npad = taps == 9 ? pad_n(cout) : (cout + 15) / 16 * 16;
    const std::vector<uint16_t> img = pack_b_image(w, taps, cin, cout, r->kpad, r->npad);
    std::vector<float> b(r->npad, 0.f), s(r->npad, 0.f);
    for (int i = 0; i < cout; i++) {
        b[i] = bias[i];
        if (slope) s[i] = slope[i];
    }
    cudaError_t e = cudaMalloc(&r->img, img.size() * 2);
    if (e == cudaSuccess) e = cudaMemcpy(r->img, img.data(), img.size() * 2, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMalloc(&r->bias, r->npad * 4);
    if (e == cudaSuccess) e = cudaMemcpy(r->bias, b.data(), r->npad * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && slope) e = cudaMalloc(&r->slope, r->npad * 4);
    if (e == cudaSuccess && slope) e = cudaMemcpy(r->slope, s.data(), r->npad * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        ajib_weights_release(&r);
        cudaGetLastError();
        return e == cudaErrorMemoryAllocation ? AJIB_ERR_NO_MEM : AJIB_ERR_CUDA;
    }
    r->bytes = img.size() * 2 + r->npad * 4 * (slope ? 2 : 1);
    *out = r;
    return AJIB_OK;
}

extern "C" void ajib_weights_release(ajib_weights **w)
{
    if (!w || !*w) return;
    cudaFree((*w)->img);
    cudaFree((*w)->bias);
    cudaFree((*w)->slope);
    delete *w;
    *w = nullptr;
}

extern "C" size_t ajib_weights_bytes(const ajib_weights *w) { return w ? w->bytes : 0; }

extern "C" int ajib_conv_supported(const ajib_conv *op, char *why, size_t why_size)
{
    return check(op, why, why_size) ? 1 : 0;
}

extern "C" int ajib_conv3x3_launch(const ajib_conv *op, const void *src, const void *resid, void *dst, int H, int W,
                                   int row_begin, int row_end, void *stream)
{
    return ajib_conv3x3_launch_images(op, src, resid, dst, 1, H, W, row_begin, row_end, stream);
}

extern "C" int ajib_conv3x3_launch_images(const ajib_conv *op, const void *src, const void *resid, void *dst, int nimg,
                                          int img_h, int W, int row_begin, int row_end, void *stream)
{
    return ajib::conv3x3_launch_planes(op, src, resid, dst, nimg, img_h, W, row_begin, row_end, stream, 0);
}

int ajib::conv3x3_launch_planes(const ajib_conv *op, const void *src, const void *resid, void *dst, int nimg, int img_h,
                                int W, int row_begin, int row_end, void *stream, size_t dst_plane)
{
    if (!check(op, nullptr, 0)) return AJIB_ERR_UNSUPPORTED;
    if (nimg < 1 || img_h < 1 || (long)nimg * img_h > (1l << 30)) return AJIB_ERR_ARGS;
    const int H = nimg * img_h;
    if (!src || !dst || H < 1 || W < 1) return AJIB_ERR_ARGS;
    if (op->gate != AJIB_GATE_NONE && !resid) return AJIB_ERR_ARGS;
    // no model-input skip from a pixel-unshuffled input (its resolution is not the conv's)
    if (op->in == AJIB_IN_NCHW3_UNSHUFFLE2 && op->out != AJIB_OUT_NHWC && resid) return AJIB_ERR_ARGS;
    if (row_end <= 0 || row_end > H) row_end = H;
    if (row_begin < 0 || row_begin >= row_end) return row_begin == row_end ? AJIB_OK : AJIB_ERR_ARGS;
    // strip-chunked maps are read by bulk copies and written by 16-byte stores
    if (((uintptr_t)src & 15) || ((uintptr_t)dst & 15) || (resid && op->gate && ((uintptr_t)resid & 15)))
        return AJIB_ERR_ARGS;

    ConvDev p{};
    p.src = (const __half *)src;
    p.resid = (const __half *)resid;
    p.dst = (__half *)dst;
    p.wimg = (const unsigned char *)op->w->img;
    p.bias = op->w->bias;
    p.slope = op->w->slope;
    p.err = status_word();
    if (!p.err) return AJIB_ERR_CUDA;
    p.H = H;
    p.W = W;
    p.cin = op->cin;
    p.cout = op->cout;
    p.in_mode = op->in;
    p.act = op->act;
    p.gate = op->gate;
    p.R = d2s_factor(op->out);
    p.in_norm = op->in_norm && op->in != AJIB_IN_NHWC;
    p.out_clamp = op->out_clamp && op->out != AJIB_OUT_NHWC;
    for (int c = 0; c < 3; c++) {
        p.in_mean[c] = op->in_mean[c];
        p.in_scale[c] = op->in_scale[c];
    }
    p.row_begin = row_begin;
    p.row_end = row_end;
    p.nstrips = feature_strips(W);
    p.img_h = img_h;
    p.skip_smem = op->out != AJIB_OUT_NHWC && resid && op->in == AJIB_IN_NHWC && W % 8 == 0 &&
                  ((uintptr_t)resid & 15) == 0;
    if (dst_plane) {
        // a plane stride only for depth-to-space outputs, and at least one dense plane
        const size_t R = (size_t)p.R;
        if (op->out == AJIB_OUT_NHWC || dst_plane < R * H * R * W) return AJIB_ERR_ARGS;
    }
    p.dst_plane = dst_plane;
    if (op->gate == AJIB_GATE_TANH1X1) {
        p.att_img = (const unsigned char *)op->att->img;
        p.att_bias = op->att->bias;
        p.att_kpad = op->att->kpad;
        p.att_npad = op->att->npad;
    }
    const long strips = (W + kTileM - 1) / kTileM;
    const long tiles = strips * (row_end - row_begin);
    cudaError_t e;
    PairFn pf = pair_fn(op);
    if (pf) {
        e = pf(p, tiles, (cudaStream_t)stream);
    } else {
        const int grid = (int)std::min<long>(sm_count(), tiles);
        e = op_fn(op)(p, grid, (cudaStream_t)stream);
    }
    return e == cudaSuccess ? AJIB_OK : AJIB_ERR_CUDA;
}

extern "C" int ajib_conv_pair_mode(int mode)
{
    if (mode == 0 || mode == 1) g_pair_mode.store(mode);
    return pair_mode();
}

extern "C" int ajib_conv_on_pairs(const ajib_conv *op) { return check(op, nullptr, 0) && pair_fn(op) ? 1 : 0; }

extern "C" int ajib_conv_pair_clusters(void)
{
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(PairCfg<64, 64>::THREADS);
    cfg.dynamicSmemBytes = (size_t)PairCfg<64, 64>::SMEM;
    cfg.gridDim = dim3(2 * (sm_count() / 2));
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void (*kern)(ConvDev) = k_conv3x3_pair<64, 64, kEpiAct>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PairCfg<64, 64>::SMEM) != cudaSuccess)
        return AJIB_ERR_CUDA;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) return AJIB_ERR_CUDA;
    return n;
}

namespace ajib {
namespace {

template <int NPAD>
cudaError_t run_concat(const CatDev &p, int grid, int smem, cudaStream_t s)
{
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(done.load() & bit)) {
        const cudaError_t attr = cudaFuncSetAttribute(k_concat1x1<NPAD>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
        if (attr != cudaSuccess) return attr;
        done.fetch_or(bit);
    }
    return launch_pdl(k_concat1x1<NPAD>, grid, kCatThreads, smem, s, p);
}

}  // namespace
}  // namespace ajib

extern "C" int ajib_concat1x1_launch(const ajib_weights *w, int nsrc, const void *const *srcs, int c, void *dst, int H,
                                     int W, int row_begin, int row_end, void *stream)
{
    if (!w || !srcs || !dst || nsrc < 2 || nsrc > 4 || c < 8 || c > 64 || c % 8 || H < 1 || W < 1) return AJIB_ERR_ARGS;
    if (w->taps != 1 || w->cin != nsrc * c || w->cout != c) return AJIB_ERR_ARGS;
    if (((uintptr_t)dst & 15)) return AJIB_ERR_ARGS;
    for (int k = 0; k < nsrc; k++)
        if (!srcs[k] || ((uintptr_t)srcs[k] & 15)) return AJIB_ERR_ARGS;
    if (row_end <= 0 || row_end > H) row_end = H;
    if (row_begin < 0 || row_begin >= row_end) return row_begin == row_end ? AJIB_OK : AJIB_ERR_ARGS;
    CatDev p{};
    for (int k = 0; k < 4; k++) p.src[k] = k < nsrc ? (const __half *)srcs[k] : nullptr;
    p.dst = (__half *)dst;
    p.wimg = (const unsigned char *)w->img;
    p.bias = w->bias;
    p.err = status_word();
    if (!p.err) return AJIB_ERR_CUDA;
    p.nsrc = nsrc;
    p.c = c;
    p.H = H;
    p.W = W;
    p.nstrips = feature_strips(W);
    p.kpad = w->kpad;
    p.row_begin = row_begin;
    p.row_end = row_end;
    // as many stages as fit (2..4); at least 120 KB requested so that one CTA holds an SM (and its TMEM)
    const CatSmem one(w->kpad, w->npad, 0);
    const int fit = (kMaxSmem - one.total) / one.stage;
    p.ns = std::min(kCatMaxStages, fit);
    if (p.ns < 2) return AJIB_ERR_UNSUPPORTED;
    const int smem = std::max(CatSmem(w->kpad, w->npad, p.ns).total, 120 * 1024);
    const long tiles = (long)((W + kTileM - 1) / kTileM) * (row_end - row_begin);
    const int grid = (int)std::min<long>(sm_count(), tiles);
    cudaError_t e;
    switch (w->npad) {
    case 16: e = run_concat<16>(p, grid, smem, (cudaStream_t)stream); break;
    case 32: e = run_concat<32>(p, grid, smem, (cudaStream_t)stream); break;
    case 48: e = run_concat<48>(p, grid, smem, (cudaStream_t)stream); break;
    case 64: e = run_concat<64>(p, grid, smem, (cudaStream_t)stream); break;
    default: return AJIB_ERR_UNSUPPORTED;
    }
    return e == cudaSuccess ? AJIB_OK : AJIB_ERR_CUDA;
}

extern "C" int ajib_feature_strips(int W) { return W > 0 ? feature_strips(W) : 0; }

extern "C" size_t ajib_feature_bytes(int H, int W, int C)
{
    if (H < 1 || W < 1 || C < 8 || C % 8) return 0;
    return (size_t)H * feature_strips(W) * (C / 8) * kStripW * 16;
}

extern "C" int ajib_kernel_status(int clear)
{
    int *w = status_word();
    if (!w) return AJIB_ERR_CUDA;
    int v = 0;
    if (cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return AJIB_ERR_CUDA;
    if (clear && v && cudaMemset(w, 0, sizeof(int)) != cudaSuccess) return AJIB_ERR_CUDA;
    return v;
}

// ---- the model input packed into a strip-chunked map (the executor's head path) ----
namespace ajib {
namespace {

// One conv pixel per thread: the NCHW fp16 model input [3][H][W] -> chunk 0 {r, g, b, 0 x 5} of
// an 8-channel strip-chunked map; pixel-unshuffled by 2 ([3][2H][2W] -> channels c*4 + ry*2 + rx,
// then 4 zeros) -> chunks 0 and 1 of a 16-channel map. Normalised as the conv's own NCHW input
// path does it ((x - mean) * scale, rounded to fp16). Strip edge pixels also go to the
// neighbouring strips' halo columns; the image's edge columns are never written.
__global__ void __launch_bounds__(128) k_pack_input(const __half *src, int H, int W, int unshuffle, int in_norm,
                                                     float m0, float m1, float m2, float s0, float s1, float s2,
                                                     int nstrips, int row_begin, __half *dst)
{
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = row_begin + blockIdx.y;
    if (x >= W) return;
    const float mean[3] = {m0, m1, m2}, scale[3] = {s0, s1, s2};
    if (!unshuffle) {
        const size_t plane = (size_t)H * W, at = (size_t)y * W + x;
        float v[3];
#pragma unroll
        for (int c = 0; c < 3; c++) {
            v[c] = __half2float(__ldg(src + c * plane + at));
            if (in_norm) v[c] = (v[c] - mean[c]) * scale[c];
        }
        store_px(dst, y, x, 0, nstrips, 1, make_uint4(pack_h2(v[0], v[1]), pack_h2(v[2], 0.f), 0u, 0u));
        return;
    }
    const int IW = 2 * W;
    const size_t plane = (size_t)2 * H * IW;
    uint32_t q[6];
#pragma unroll
    for (int j = 0; j < 6; j++) {
        const int c = j >> 1, ry = j & 1;
        q[j] = __ldg(reinterpret_cast<const unsigned int *>(src + c * plane + (size_t)(2 * y + ry) * IW + 2 * x));
        if (in_norm) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&q[j]));
            q[j] = pack_h2((f.x - mean[c]) * scale[c], (f.y - mean[c]) * scale[c]);
        }
    }
    store_px(dst, y, x, 0, nstrips, 2, make_uint4(q[0], q[1], q[2], q[3]));
    store_px(dst, y, x, 1, nstrips, 2, make_uint4(q[4], q[5], 0u, 0u));
}

}  // namespace

int pack_model_input(const void *src, int H, int W, int unshuffle, bool in_norm, const float *mean, const float *scale,
                     int row_begin, int row_end, void *dst, cudaStream_t s)
{
    if (!src || !dst || H < 1 || W < 1 || row_begin < 0 || row_end > H || row_begin >= row_end) return AJIB_ERR_ARGS;
    if (((uintptr_t)src & 3) || ((uintptr_t)dst & 15)) return AJIB_ERR_ARGS;
    const dim3 grid((W + 127) / 128, row_end - row_begin);
    k_pack_input<<<grid, 128, 0, s>>>((const __half *)src, H, W, unshuffle ? 1 : 0, in_norm ? 1 : 0, mean[0], mean[1],
                                      mean[2], scale[0], scale[1], scale[2], feature_strips(W), row_begin, (__half *)dst);
    return cudaGetLastError() == cudaSuccess ? AJIB_OK : AJIB_ERR_CUDA;
}

}  // namespace ajib
