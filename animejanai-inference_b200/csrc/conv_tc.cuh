/*
 * conv_tc.cuh — the fused 3x3 convolution on Blackwell tensor cores (sm_100a), device code.
 *
 * Implicit GEMM with the output pixels as M: a tile is 128 consecutive pixels of one output row,
 * K is 9 taps x cin (cin padded to a multiple of 16). One staged input row (130 pixels: the tile
 * plus a one-pixel halo on each side) feeds every tap of the three output rows it touches. For
 * horizontal tap dx the A operand is the staged row starting dx pixels in: a 16-byte shift of the
 * shared-memory descriptor's start address, because the row is staged K-major without swizzle as
 * [cin/8][130][8 fp16].
 *
 * The three vertical taps share that A, so one MMA computes all three at once: B stacks the
 * weights of tap rows 0, 1, 2 along N (N = 3 x cout_pad, 192 for 64 channels), and the MMA's D
 * is three adjacent accumulators — those of output rows r+1, r and r-1 for input row r. The
 * accumulators live in a ring of TMEM slots in descending order (output j in slot S-1-(j mod S)),
 * so those three outputs are adjacent slots; where the window wraps around the ring the MMA is
 * split in two. A tensor-core MMA of N >= 128 runs at the full rate, while N = cout alone would
 * be bound by the operand fetch (about 48 cycles for an N = 64 MMA against 32 of math). Each
 * slot is zeroed by the epilogue after it reads it, so every MMA accumulates.
 *
 * Feature maps live in HBM strip-chunked: a row of a C-channel map is cut into 128-pixel strips,
 * and each (row, strip) is one contiguous block of C/8 chunks of 130 columns of 8 fp16 channels
 * — the strip's pixels plus a halo column on each side holding a copy of the neighbouring strip's
 * edge pixel (zero at the image's edges and past W). Element (y, x, c), x in strip s = x / 128,
 * is at ((((y * S + s) * C/8 + c/8) * 130 + x - 128 s + 1) * 8 + c % 8, S = ceil(W / 128). So the
 * staged row — a strip with its halo, all chunks, the MMA's A layout [C/8][130][8] — is one
 * contiguous bulk copy (8 chunk copies issued per row measured 4.6 % slower on the 64-channel
 * layer), and the epilogue's stores of one chunk for 32 consecutive pixels are one coalesced
 * 512-byte write (the strip's two edge pixels are also written into the neighbours' halos).
 *
 * A CTA is persistent on one SM and walks a contiguous run of (strip, row) tiles down a
 * 128-pixel-wide vertical strip, so each input row is fetched once. Roles:
 *   warps 0-3   producer: warp 0 issues the bulk copy of each input row (strip-chunked inputs),
 *               or all 128 threads convert the NCHW RGB model input
 *               into the same layout; lane 0 also waits for the accumulators a row starts to be
 *               free and writes the row's MMA plan beside the staged row, and after the last row
 *               fills one terminator stage (depth-to-space convs and inputs of up to 32 channels:
 *               warp 2 does the waits and plans, warp 0 only the copies); warp 3 copies each
 *               output's extra input row into shared memory ahead of the epilogue: the SPAN
 *               gate's block input, or the depth-to-space skip (the model input);
 *   warps 4-11  epilogue: TMEM -> registers (one pixel per thread, half a slot's channels per
 *               warp), bias, activation, SPAN gate or depth-to-space with the model-input skip,
 *               fp16 store; then zero the half slot;
 *   warp 12     idle, so that
 *   warp 13     the MMA issuer (one thread) and TMEM owner sits on the second sub-partition (warp
 *               % 4), away from the producer thread: sharing the first one's issue slots cost
 *               2-4 % on every conv. The tensor pipe queues only a few MMAs and a lone thread's
 *               bookkeeping is slow, so this thread only waits for a staged row, reads its plan
 *               and issues, straight-line per stage of two rows; the next stage's wait sits
 *               inside the second row's MMAs.
 * Weights for all 9 taps stay resident in shared memory for the CTA's lifetime.
 *
 * The semantics are those of the reference kernel k_conv3x3 (src/native/conv_kernels.cuh:100-350)
 * with fp32 accumulation and an fp32 epilogue instead of fp16 ones (one rounding to fp16 at the
 * store).
 */
#pragma once

#include <cuda_fp16.h>

#include <type_traits>

#include "feature_map.cuh"
#include "sm100.cuh"

namespace ajib {

constexpr int kHalo = kTileM + 2;  // staged input pixels per row
constexpr int kTmemCols = 512;     // the whole TMEM: the accumulator ring
constexpr int kProdWarps = 4;      // producer warps (all of them convert an NCHW model input)
constexpr int kEpiWarps = 8;       // epilogue warps: two per TMEM lane quarter, one per half slot
constexpr int kIdleWarp = kProdWarps + kEpiWarps;  // keeps the MMA warp off the producer's sub-partition
constexpr int kMmaWarp = kIdleWarp + 1;
constexpr int kConvThreads = (kMmaWarp + 1) * 32;
constexpr int kMaxSmem = 227 * 1024;

// Epilogue kinds, one kernel instantiation each (so each layer runs only the code it needs):
// strip-chunked output with an activation; strip-chunked output through a SPAN gate; depth-to-space
// into NCHW (with the model-input skip); strip-chunked output through the SPANF3 tanh gate, whose
// 1x1 attention conv is a second tensor-core GEMM in the epilogue.
enum { kEpiAct = 0, kEpiGate = 1, kEpiD2S = 2, kEpiAtt = 3 };

// Input modes: strip-chunked feature map (bulk copies); the NCHW RGB model input; the NCHW RGB
// model input pixel-unshuffled by 2 (12 channels at half resolution).
enum { kInRows = 0, kInRgb = 1, kInRgbUnshuffle2 = 2 };

// error codes written to the status word (which wait timed out)
enum { kErrProdEmpty = 101, kErrMmaFull = 102, kErrProdAccEmpty = 103, kErrEpiAccFull = 104, kErrWeights = 105,
       kErrDrain = 106, kErrAttFull = 107 };

struct ConvDev {
    const __half *src;    // strip-chunked map [H][cin] or NCHW [3][H][W]
    const __half *resid;  // gate: strip-chunked [H][cout]; depth-to-space: NCHW model input [3][H][W] or null
    __half *dst;          // strip-chunked [H][cout] or NCHW [3][R*H][R*W]
    const unsigned char *wimg;  // packed B operand image, all taps
    const float *bias;    // NPAD floats
    const float *slope;   // NPAD floats or null
    int *err;             // status word
    int H, W, cin, cout;
    int in_mode, act, gate, R;  // R = 0: strip-chunked output, else depth-to-space factor
    int in_norm, out_clamp;
    float in_mean[3], in_scale[3];
    int row_begin, row_end;
    int nstrips;          // S: 128-pixel strips per row of the strip-chunked maps
    int img_h;            // rows per image: H = n * img_h images stacked along H, convolved apart
    // tanh gate: the 1x1 attention conv's packed B image ([K/8][N/8][8][8] fp16, K = att_kpad,
    // N = att_npad) and bias (att_npad floats)
    const unsigned char *att_img;
    const float *att_bias;
    int att_kpad, att_npad;
    // depth-to-space with the skip: its rows reach shared memory by bulk copies (strip-chunked
    // input and W a multiple of 8, so every copy is 16-byte aligned), else the epilogue loads them
    int skip_smem;
    // depth-to-space: elements from one output plane to the next (0: the dense [3][R*H][R*W]), so
    // that a batch of tiles can land inside a larger stack of tiles
    size_t dst_plane;
};

// The input rows a segment of output rows [ya, yb) reads: one-row halos that stay inside the
// image (a stack of images of img_h rows each).
__device__ __forceinline__ void segment_rows(int ya, int yb, int img_h, int &r0, int &r1)
{
    r0 = (ya % img_h == 0) ? ya : ya - 1;
    r1 = (yb % img_h == 0) ? yb - 1 : yb;
}

constexpr int kGateSlots = 3;  // SPAN gate: block-input rows staged ahead of the epilogue

template <int KPAD, int NPAD, bool ATT = false, bool SKIP = false, bool GATE = false>
struct ConvCfg {
    static_assert(KPAD % 16 == 0 && NPAD % 16 == 0 && KPAD <= 64 && NPAD <= 64, "padded channel counts");
    static constexpr int KC = KPAD / 8;       // 8-channel chunks per pixel
    static constexpr int KS = KPAD / 16;      // MMA K steps per tap
    static constexpr int NG = NPAD / 8;       // 8-row core-matrix groups of one tap's B
    // the tanh gate's two attention accumulators (one per epilogue group) take their columns from
    // the ring
    static constexpr int S = (kTmemCols - (ATT ? 2 * NPAD : 0)) / NPAD;  // accumulator ring slots
    static constexpr int LBO_A = kHalo * 16;  // bytes between K chunks of a staged row
    static constexpr int LBO_B = 3 * NG * 128;  // bytes between K chunks of a stacked-tap B
    static constexpr int SLOT = (KC * LBO_A + 1023) / 1024 * 1024;
    static constexpr int WBYTES = 9 * KPAD * NPAD * 2;
    static constexpr int AOFF = (WBYTES + 1023) / 1024 * 1024;
    static constexpr int RP = 2;                     // staged rows per pipeline stage
    static constexpr int STAGE = RP * SLOT;
    // tanh gate: the attention conv's B (at most NPAD x NPAD) and one A tile per epilogue group
    // (the gate's fp16 input o, [NPAD/8][128 pixels][8])
    static constexpr int ATT_B = ATT ? NPAD * NPAD * 2 : 0;
    static constexpr int ATT_A = NPAD / 8 * kTileM * 16;
    static constexpr int ATT_BYTES = ATT ? ATT_B + 2 * ATT_A : 0;
    // depth-to-space: per ring slot the model-input row its output adds (3 planes x 128 pixels),
    // copied in by the producer's bulk copies
    static constexpr int SKIP_ROW = 3 * kTileM * 2;
    static constexpr int SKIP_BYTES = SKIP ? S * SKIP_ROW : 0;
    // SPAN gate: the block input's (row, strip) block of each of kGateSlots outputs, halo columns
    // included ([NPAD/8][130][8] fp16), copied in by the gate warp
    static constexpr int GATE_ROW = NPAD / 8 * kHalo * 16;
    static constexpr int GATE_BYTES = GATE ? kGateSlots * GATE_ROW : 0;
    static constexpr int FIXED = AOFF + ATT_BYTES + SKIP_BYTES + GATE_BYTES + 3 * 64 * 4 + 1024 + 1024 + 1024;
    static constexpr int NS_FIT = (kMaxSmem - FIXED) / STAGE;
    static constexpr int NS = NS_FIT > 6 ? 6 : NS_FIT;  // stages of RP rows: as many as fit, up to 6
    static_assert(NS >= 2 && S >= 4, "pipeline depth");
    static constexpr int ATOFF = AOFF + NS * STAGE;  // attention B, then A tiles 0 and 1
    static constexpr int SKOFF = ATOFF + ATT_BYTES;  // skip rows [S][3][128] fp16
    static constexpr int GOFF = SKOFF + SKIP_BYTES;  // gate rows [kGateSlots][NPAD/8][130][8] fp16
    static constexpr int POFF = GOFF + GATE_BYTES;   // bias[64], slope[64], attention bias[64] floats
    // mbarriers: full[NS], empty[NS], accf[S], acce[S], wbar, dbar, attf[2], skipf[S], landed[NS],
    // the TMEM address word, gatef[kGateSlots], gatee[kGateSlots]
    static constexpr int BOFF = POFF + 3 * 64 * 4;
    static constexpr int PLOFF = BOFF + 1024;       // RowPlan per staged row
    static constexpr int SMEM = BOFF + 1024 + 1024 + 1024;  // + alignment slack for the base
    static_assert((3 * NS + 3 * S + 5 + 2 * kGateSlots) * 8 <= 1024 && NS * RP * 48 <= 1024, "barrier and plan area");
    static_assert(SMEM <= kMaxSmem, "shared memory budget");
};

// The run of tiles a CTA owns, split into per-strip segments. All roles walk the same sequence.
struct SegIter {
    long L, L1;
    int rows, row_begin;
    __device__ SegIter(int W, int row_begin_, int row_end) : SegIter(W, row_begin_, row_end, blockIdx.x, gridDim.x) {}
    // the run of CTA `cta` of `ncta`
    __device__ SegIter(int W, int row_begin_, int row_end, int cta, int ncta)
    {
        row_begin = row_begin_;
        rows = row_end - row_begin_;
        const long strips = (W + kTileM - 1) / kTileM;
        const long T = strips * rows;
        L = (long)cta * T / ncta;
        L1 = (long)(cta + 1) * T / ncta;
    }
    // next segment: strip, output rows [ya, yb)
    __device__ bool next(int &strip, int &ya, int &yb)
    {
        if (L >= L1) return false;
        strip = (int)(L / rows);
        const int off = (int)(L % rows);
        const long n = min((long)(rows - off), L1 - L);
        ya = row_begin + off;
        yb = ya + (int)n;
        L += n;
        return true;
    }
};


// Depth-to-space by R into NCHW [3][R*H][R*W] (PixelShuffle / DepthToSpace CRD: channel
// c*R*R + ry*R + rx -> [c][R*y + ry][R*x + rx]), plus the nearest-upsampled model input when
// given, optionally clamped to [0, 1]; one rounding to fp16. v holds channels [C0, C0 + CW): the
// groups of R channels that lie wholly inside it are stored here.
template <int R, int CW, int C0>
__device__ __forceinline__ void store_d2s(const float (&v)[CW], const ConvDev &a, int o, int x, const float (&skip)[3])
{
    const int W = a.W, H = a.H;
    const size_t OW = (size_t)R * W, OH = (size_t)R * H, plane = a.dst_plane ? a.dst_plane : OH * OW;
#pragma unroll
    for (int c3 = 0; c3 < 3; c3++) {
        // skip the colour planes with no channel group inside [C0, C0 + CW)
        if (c3 * R * R + R > C0 + CW || c3 * R * R + R * R <= C0) continue;
        const float add = skip[c3];
#pragma unroll
        for (int ry = 0; ry < R; ry++) {
            const int n0 = c3 * R * R + ry * R - C0;
            if (n0 < 0 || n0 + R > CW) continue;
            __half *d = a.dst + (size_t)c3 * plane + ((size_t)R * o + ry) * OW + (size_t)R * x;
            float t[R];
#pragma unroll
            for (int rx = 0; rx < R; rx++) {
                float val = v[n0 + rx] + add;
                if (a.out_clamp) val = fminf(fmaxf(val, 0.f), 1.f);
                t[rx] = val;
            }
            if constexpr (R == 2) {
                *reinterpret_cast<uint32_t *>(d) = pack_h2(t[0], t[1]);
            } else if constexpr (R == 4) {
                uint2 u;
                u.x = pack_h2(t[0], t[1]);
                u.y = pack_h2(t[2], t[3]);
                *reinterpret_cast<uint2 *>(d) = u;
            } else {
#pragma unroll
                for (int rx = 0; rx < R; rx++) d[rx] = __float2half_rn(t[rx]);
            }
        }
    }
}

// The global inputs of one output row's epilogue, for pixel x and channels [C0, C0 + CW). They
// are loaded before the wait for the accumulator, so their latency overlaps it.
template <int CW>
struct EpiIn {
    float skip[3];       // depth-to-space: the model-input pixel (nearest-upsampled skip), or zeros
    uint4 gate[CW / 8];  // SPAN gate: the block input's chunks of this half
};

// The epilogue's inputs of the next rows, loaded PF rows ahead (a register ring: e[0] is the row
// being finished).
template <int PF, typename T>
struct EpiRing {
    T e[PF];
    __device__ __forceinline__ void push(const T &next)
    {
#pragma unroll
        for (int i = 0; i + 1 < PF; i++) e[i] = e[i + 1];
        e[PF - 1] = next;
    }
};

template <int EK, int CW, int C0>
__device__ __forceinline__ void epi_prefetch(EpiIn<CW> &in, const ConvDev &a, int o, int x)
{
    const int W = a.W, H = a.H;
    if constexpr (EK == kEpiD2S) {
#pragma unroll
        for (int c3 = 0; c3 < 3; c3++)
            in.skip[c3] = (a.resid && x < W) ? __half2float(__ldg(a.resid + ((size_t)c3 * H + o) * W + x)) : 0.f;
    } else if constexpr (EK == kEpiGate) {
        const int ccout = a.cout / 8;
        (void)W;
        // x may be past W in the last strip: those columns hold zeros
        const __half *xr = a.resid + map_at(o, x >> 7, 0, (x & (kTileM - 1)) + 1, a.nstrips, ccout);
#pragma unroll
        for (int c = 0; c < CW / 8; c++)
            in.gate[c] = (C0 / 8 + c < ccout) ? __ldg(reinterpret_cast<const uint4 *>(xr + (size_t)(C0 / 8 + c) * kStripW * 8))
                                              : make_uint4(0, 0, 0, 0);
    }
}

// The epilogue of one output row for pixel x and channels [C0, C0 + CW) (v already holds the bias:
// every accumulator starts from it): activation or SPAN gate into the strip-chunked map, or
// depth-to-space into NCHW. (Staging the row in shared memory for bulk stores measured slower
// than these coalesced 512-byte warp stores.)
template <int EK, int CW, int C0>
__device__ __forceinline__ void epi_store(float (&v)[CW], const ConvDev &a, const float *sslope_m1, int o, int x,
                                          const EpiIn<CW> &in)
{
    if (x >= a.W) return;
    const int ccout = a.cout / 8;  // 16-byte chunks per pixel
    if constexpr (EK == kEpiAct) {
        // ReLU in the rounding to fp16 (exact: max(round(v), 0) = round(max(v, 0))); PReLU as
        // v + min(v, 0) * (slope - 1), one FMA a channel
        uint32_t w[CW / 2];
        if (a.act == 1) {
#pragma unroll
            for (int j = 0; j < CW / 2; j++) w[j] = dev::pack_relu_h2(v[2 * j], v[2 * j + 1]);
        } else if (a.act == 2) {
            // the FMAs two channels at a time (__ffma2_rn: each lane rounded as fmaf)
#pragma unroll
            for (int n = 0; n < CW; n += 4) {
                const float4 s4 = *reinterpret_cast<const float4 *>(sslope_m1 + C0 + n);
                const float2 r01 = __ffma2_rn(make_float2(fminf(v[n], 0.f), fminf(v[n + 1], 0.f)), make_float2(s4.x, s4.y),
                                              make_float2(v[n], v[n + 1]));
                const float2 r23 = __ffma2_rn(make_float2(fminf(v[n + 2], 0.f), fminf(v[n + 3], 0.f)),
                                              make_float2(s4.z, s4.w), make_float2(v[n + 2], v[n + 3]));
                w[n / 2] = pack_h2(r01.x, r01.y);
                w[n / 2 + 1] = pack_h2(r23.x, r23.y);
            }
        } else {
            if (a.act == 3) {
                // SiLU v * sigmoid(v) = v * (0.5 tanh(v / 2) + 0.5), two channels per multiply and
                // FMA (__fmul2_rn / __ffma2_rn: each lane rounded as the scalar operation)
#pragma unroll
                for (int j = 0; j < CW / 2; j++) {
                    const float2 vv = make_float2(v[2 * j], v[2 * j + 1]);
                    const float2 hv = __fmul2_rn(make_float2(0.5f, 0.5f), vv);
                    const float2 t = make_float2(dev::tanh_fast(hv.x), dev::tanh_fast(hv.y));
                    const float2 r = __fmul2_rn(vv, __ffma2_rn(make_float2(0.5f, 0.5f), t, make_float2(0.5f, 0.5f)));
                    w[j] = pack_h2(r.x, r.y);
                }
            } else {
#pragma unroll
                for (int j = 0; j < CW / 2; j++) w[j] = pack_h2(v[2 * j], v[2 * j + 1]);
            }
        }
        // one 16-byte chunk per lane per store: 32 consecutive pixels = 512 contiguous bytes; the
        // row's address once, chunks kStripW x 8 halves apart, and the strip's edge pixels also
        // into the neighbour's halo column (store_px's layout; one address computation a row
        // instead of one a chunk: 1.9 % on the body conv, 3.1 % on the head)
        {
            const int st = x >> 7, u = (x & (kTileM - 1)) + 1;
            uint4 *p0 = reinterpret_cast<uint4 *>(a.dst + map_at(o, st, C0 / 8, u, a.nstrips, ccout));
            const bool hl = u == 1 && st > 0, hr = u == kTileM && st + 1 < a.nstrips;
            uint4 *ph = hl ? reinterpret_cast<uint4 *>(a.dst + map_at(o, st - 1, C0 / 8, kStripW - 1, a.nstrips, ccout))
                           : reinterpret_cast<uint4 *>(a.dst + map_at(o, st + 1, C0 / 8, 0, a.nstrips, ccout));
#pragma unroll
            for (int c = 0; c < CW / 8; c++) {
                if (C0 / 8 + c < ccout) {
                    const uint4 val = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
                    p0[c * kStripW] = val;
                    if (hl || hr) ph[c * kStripW] = val;
                }
            }
        }
        return;
    }
    if constexpr (EK == kEpiD2S) {
        switch (a.R) {
        case 1: store_d2s<1, CW, C0>(v, a, o, x, in.skip); break;
        case 2: store_d2s<2, CW, C0>(v, a, o, x, in.skip); break;
        case 3: store_d2s<3, CW, C0>(v, a, o, x, in.skip); break;
        default: store_d2s<4, CW, C0>(v, a, o, x, in.skip); break;
        }
        return;
    }
    if constexpr (EK == kEpiGate) {
#pragma unroll
        for (int c = 0; c < CW / 8; c++) {
            if (C0 / 8 + c < ccout) {
                const __half2 *h = reinterpret_cast<const __half2 *>(&in.gate[c]);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float2 f = __half22float2(h[j]);
                    const int n0 = c * 8 + 2 * j;
                    if (a.gate == 1) {
                        v[n0] = f.x + v[n0];
                        v[n0 + 1] = f.y + v[n0 + 1];
                    } else if (a.gate == 3) {
                        // (x + v) * (sigmoid(v) - 0.5) = (x + v) * 0.5 tanh(v / 2), two channels per
                        // operation (each lane rounded as the scalar one)
                        const float2 vv = make_float2(v[n0], v[n0 + 1]);
                        const float2 hv = __fmul2_rn(make_float2(0.5f, 0.5f), vv);
                        const float2 g = __fmul2_rn(make_float2(0.5f, 0.5f),
                                                    make_float2(dev::tanh_fast(hv.x), dev::tanh_fast(hv.y)));
                        const float2 r = __fmul2_rn(__fadd2_rn(f, vv), g);
                        v[n0] = r.x;
                        v[n0 + 1] = r.y;
                    }
                }
            }
        }
        // one 16-byte chunk per lane per store: 32 consecutive pixels = 512 contiguous bytes; the
        // row's address once, chunks kStripW x 8 halves apart (as in the activation epilogue)
        const int st = x >> 7, u = (x & (kTileM - 1)) + 1;
        uint4 *p0 = reinterpret_cast<uint4 *>(a.dst + map_at(o, st, C0 / 8, u, a.nstrips, ccout));
        const bool hl = u == 1 && st > 0, hr = u == kTileM && st + 1 < a.nstrips;
        uint4 *ph = hl ? reinterpret_cast<uint4 *>(a.dst + map_at(o, st - 1, C0 / 8, kStripW - 1, a.nstrips, ccout))
                       : reinterpret_cast<uint4 *>(a.dst + map_at(o, st + 1, C0 / 8, 0, a.nstrips, ccout));
#pragma unroll
        for (int c = 0; c < CW / 8; c++) {
            if (C0 / 8 + c < ccout) {
                uint4 w4;
                w4.x = pack_h2(v[c * 8 + 0], v[c * 8 + 1]);
                w4.y = pack_h2(v[c * 8 + 2], v[c * 8 + 3]);
                w4.z = pack_h2(v[c * 8 + 4], v[c * 8 + 5]);
                w4.w = pack_h2(v[c * 8 + 6], v[c * 8 + 7]);
                p0[c * kStripW] = w4;
                if (hl || hr) ph[c * kStripW] = w4;
            }
        }
    }
}

// The ring slot of the j-th output row a CTA produces, and its mbarrier phase parity.
template <int S>
__device__ __forceinline__ int ring_slot(uint32_t j) { return S - 1 - (int)(j % S); }
template <int S>
__device__ __forceinline__ uint32_t ring_phase(uint32_t j) { return (j / S) & 1u; }

// The input rows a CTA stages, in the order the producer and the MMA thread walk them: per
// segment (strip, output rows [ya, yb)) its input rows r0..r1, with the first row of the image
// that holds the current row.
struct RowWalk {
    SegIter seg;
    int img_h;
    int r = 0, r1 = -1, ya = 0, yb = 0, first = 0, strip = 0;
    uint32_t ot = 0, ot_next = 0;  // output index of row ya; of the next segment's first row
    __device__ RowWalk(int W, int row_begin, int row_end, int img_h_) : seg(W, row_begin, row_end), img_h(img_h_) {}
    __device__ bool next()
    {
        if (r < r1) {
            r++;
            if (r - first == img_h) first = r;
            return true;
        }
        int a_, b_;
        if (!seg.next(strip, a_, b_)) return false;
        ot = ot_next;
        ot_next += (uint32_t)(b_ - a_);
        ya = a_;
        yb = b_;
        int r0;
        segment_rows(ya, yb, img_h, r0, r1);
        r = r0;
        first = r0 / img_h * img_h;
        return true;
    }
};

// What one staged row's MMAs do: up to three pieces (runs of adjacent accumulators, one MMA each
// per tap column and K step) and the accumulator-full barriers the row completes. The producer
// writes it into shared memory beside the staged row, so the MMA thread only reads it.
struct RowPlan {
    uint32_t pd[3], pb[3], pi[3];
    uint32_t np;                  // pieces (0: no row); kPlanEnd in a stage's first plan: the walk is over
    uint32_t commit_a, commit_b;  // accumulator-full mbarrier addresses to commit after the row, or 0
};
static_assert(sizeof(RowPlan) == 48, "row plan layout");
constexpr uint32_t kPlanEnd = 0xFFFFFFFFu;

// The accumulator-free waits a row's plan depends on: up to two (mbarrier, parity) pairs.
struct RowWaits {
    bool w0 = false, w1 = false;
    uint32_t bar0 = 0, par0 = 0, bar1 = 0, par1 = 0;
    __device__ bool wait(int *err) const
    {
        bool ok = true;
        if (w0) ok = dev::mbar_wait(bar0, par0, err, kErrProdAccEmpty);
        if (w1 && ok) ok = dev::mbar_wait(bar1, par1, err, kErrProdAccEmpty);
        return ok;
    }
};

// The plan of the walk's current row, and the waits that must pass before its MMAs may run (the
// accumulators the row starts must be free).
template <int S, int NPAD, int NG>
__device__ __forceinline__ void plan_row(const RowWalk &w, uint32_t tmem, uint32_t accf0, uint32_t acce0, RowPlan &p,
                                         RowWaits &wt)
{
    const int r = w.r, ya = w.ya, yb = w.yb, first = w.first, last = first + w.img_h - 1;
    // the outputs this row feeds: r+1 (tap row 0), r (1), r-1 (2), those in [ya, yb) and in r's
    // image, grouped into pieces: runs of adjacent ring slots, one MMA each
    const bool v0 = r + 1 <= last && r + 1 >= ya && r + 1 < yb, v1 = r >= ya && r < yb,
               v2 = r - 1 >= first && r - 1 >= ya && r - 1 < yb;
    const uint32_t j0 = w.ot + (uint32_t)(r + 1 - ya);
    const int sl0 = ring_slot<S>(j0), sl1 = ring_slot<S>(j0 - 1u), sl2 = ring_slot<S>(j0 - 2u);
    // an output's first input row must find its slot free: r+1 always starts at r, and r starts at
    // r when r is its image's first row
    wt.w0 = v0;
    wt.bar0 = acce0 + 8 * sl0;
    wt.par0 = ring_phase<S>(j0) ^ 1u;
    wt.w1 = v1 && r == first;
    wt.bar1 = acce0 + 8 * sl1;
    wt.par1 = ring_phase<S>(j0 - 1u) ^ 1u;
    const bool c01 = v0 && v1 && sl1 == sl0 + 1, c12 = v1 && v2 && sl2 == sl1 + 1;
    const bool st0 = v0, st1 = v1 && !c01, st2 = v2 && !c12;
    const int len0 = 1 + (c01 ? 1 : 0) + ((c01 && c12) ? 1 : 0), len1 = 1 + (c12 ? 1 : 0);
    const uint32_t D0 = tmem + (uint32_t)(sl0 * NPAD), D1 = tmem + (uint32_t)(sl1 * NPAD), D2 = tmem + (uint32_t)(sl2 * NPAD);
    constexpr uint32_t B1 = (uint32_t)(1 * NG * 128) >> 4, B2 = (uint32_t)(2 * NG * 128) >> 4;
    const uint32_t I0 = dev::idesc_f16_f32(kTileM, len0 * NPAD), I1 = dev::idesc_f16_f32(kTileM, len1 * NPAD),
                   I2 = dev::idesc_f16_f32(kTileM, NPAD);
    p.pd[0] = D0; p.pb[0] = 0u; p.pi[0] = I0;
    p.pd[1] = D1; p.pb[1] = B1; p.pi[1] = I1;
    p.pd[2] = D2; p.pb[2] = B2; p.pi[2] = I2;
    const int mask = (st0 ? 1 : 0) | (st1 ? 2 : 0) | (st2 ? 4 : 0);
    // mask 7 (three pieces) would need two wraps in three adjacent slots: impossible for S >= 2.
    // The ring wraps inside a row's window in two ways: between r+1 and r (mask 3: pieces {r+1} and
    // {r, r-1}) and between r and r-1 (mask 5: pieces {r+1, r} and {r-1}). A split row's N = 64
    // piece goes first: its MMA fills the A collector and the N = 128 one reuses it, which runs as
    // fast as one N = 192 MMA (the other order measured 12 % slower per row).
    static_assert(S >= 2, "ring");
    p.np = 1;
    switch (mask) {
    case 1: break;
    case 2: p.pd[0] = D1; p.pb[0] = B1; p.pi[0] = I1; break;
    case 3: p.np = 2; break;
    case 4: p.pd[0] = D2; p.pb[0] = B2; p.pi[0] = I2; break;
    case 5: p.pd[0] = D2; p.pb[0] = B2; p.pi[0] = I2; p.pd[1] = D0; p.pb[1] = 0u; p.pi[1] = I0; p.np = 2; break;
    default: p.pd[0] = D1; p.pb[0] = B1; p.pi[0] = I1; p.pd[1] = D2; p.pb[1] = B2; p.pi[1] = I2; p.np = 2; break;
    }
    // outputs complete at their last input row: o + 1, or o at the image's last row
    p.commit_a = v2 ? accf0 + 8 * sl2 : 0u;
    p.commit_b = (v1 && r == last) ? accf0 + 8 * sl1 : 0u;
}

// One staged row's MMAs for tap columns [DX0, DX1): for each K step, one MMA per piece. Two
// pieces share their A operand (the same staged row and K step): the first fills the A collector
// buffer, the second reads it from there (an MMA's cost is bound by fetching A, so a split row
// costs little more than a whole one).
template <int NP, int DX0, int DX1, int KS, int KC, int NG, int LBO_A>
__device__ __forceinline__ void issue_taps(uint64_t adesc0, uint64_t bdesc0, const RowPlan &p)
{
#pragma unroll
    for (int dx = DX0; dx < DX1; dx++) {
#pragma unroll
        for (int kk = 0; kk < KS; kk++) {
            const uint64_t ad = adesc0 + (uint64_t)((kk * 2 * LBO_A + dx * 16) >> 4);
            const uint64_t bd = bdesc0 + (uint64_t)(((dx * KC + 2 * kk) * 3 * NG * 128) >> 4);
            if constexpr (NP == 1) {
                dev::mma_f16(p.pd[0], ad, bd + p.pb[0], p.pi[0], 1u, 0);
            } else {
                dev::mma_f16(p.pd[0], ad, bd + p.pb[0], p.pi[0], 1u, 1);  // collector::a::fill
                dev::mma_f16(p.pd[1], ad, bd + p.pb[1], p.pi[1], 1u, 3);  // collector::a::lastuse
            }
        }
    }
}

// A row's pieces are one or two: its (up to) three accumulators are adjacent ring slots except
// across the ring's one wrap.
template <int DX0, int DX1, int KS, int KC, int NG, int LBO_A>
__device__ __forceinline__ void issue_plan(uint64_t adesc0, uint64_t bdesc0, const RowPlan &p)
{
    if (p.np == 1)
        issue_taps<1, DX0, DX1, KS, KC, NG, LBO_A>(adesc0, bdesc0, p);
    else
        issue_taps<2, DX0, DX1, KS, KC, NG, LBO_A>(adesc0, bdesc0, p);
}

// TMEM columns [C0, C0 + CW) of this warp's lanes from taddr (a slot's base) in runs of 16 at
// 16-column boundaries and runs of 8 elsewhere, so every access is aligned to its own width (a
// 48-column slot splits 24 + 24 between its two epilogue warps).
template <int CW, int C0, int C = 0>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float (&v)[CW])
{
    if constexpr (C < CW) {
        if constexpr ((C0 + C) % 16 == 0 && C + 16 <= CW) {
            float t[16];
            dev::tmem_ld16(taddr + C0 + C, t);
#pragma unroll
            for (int j = 0; j < 16; j++) v[C + j] = t[j];
            tmem_ld_cols<CW, C0, C + 16>(taddr, v);
        } else {
            float t[8];
            dev::tmem_ld8(taddr + C0 + C, t);
#pragma unroll
            for (int j = 0; j < 8; j++) v[C + j] = t[j];
            tmem_ld_cols<CW, C0, C + 8>(taddr, v);
        }
    }
}

// v += TMEM columns [C0, C0 + CW) of this warp's lanes from taddr, loaded and added in runs of 16
// or 8 (few registers live beside v).
template <int CW, int C0, int C = 0>
__device__ __forceinline__ void tmem_add_cols(uint32_t taddr, float (&v)[CW])
{
    if constexpr (C < CW) {
        if constexpr ((C0 + C) % 16 == 0 && C + 16 <= CW) {
            float t[16];
            dev::tmem_ld16(taddr + C0 + C, t);
            dev::tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; j++) v[C + j] += t[j];
            tmem_add_cols<CW, C0, C + 16>(taddr, v);
        } else {
            float t[8];
            dev::tmem_ld8(taddr + C0 + C, t);
            dev::tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 8; j++) v[C + j] += t[j];
            tmem_add_cols<CW, C0, C + 8>(taddr, v);
        }
    }
}

template <int CW, int C0, int C = 0>
__device__ __forceinline__ void tmem_st_cols(uint32_t taddr, const uint32_t (&w)[CW])
{
    if constexpr (C < CW) {
        if constexpr ((C0 + C) % 16 == 0 && C + 16 <= CW) {
            uint32_t t[16];
#pragma unroll
            for (int j = 0; j < 16; j++) t[j] = w[C + j];
            dev::tmem_st16(taddr + C0 + C, t);
            tmem_st_cols<CW, C0, C + 16>(taddr, w);
        } else {
            uint32_t t[8];
#pragma unroll
            for (int j = 0; j < 8; j++) t[j] = w[C + j];
            dev::tmem_st8(taddr + C0 + C, t);
            tmem_st_cols<CW, C0, C + 8>(taddr, w);
        }
    }
}

template <int KPAD, int NPAD, int EK, int IN>
__global__ void __launch_bounds__(kConvThreads, 1) k_conv3x3_tc(const __grid_constant__ ConvDev a)
{
    constexpr bool ATT = EK == kEpiAtt;
    constexpr bool GATE = EK == kEpiGate;
    using C = ConvCfg<KPAD, NPAD, ATT, EK == kEpiD2S, GATE>;
    constexpr int S = C::S;
    extern __shared__ unsigned char smraw[];
    // 1024-byte aligned base (bulk-copy destinations and descriptor bases)
    unsigned char *sm = smraw + ((1024 - (dev::smem_u32(smraw) & 1023)) & 1023);
    const uint32_t sbase = dev::smem_u32(sm);
    const uint32_t wbase = sbase, abase = sbase + C::AOFF;
    float *sbias = reinterpret_cast<float *>(sm + C::POFF), *sslope = sbias + 64, *satt = sbias + 128;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + C::BOFF);
    const uint32_t full0 = dev::smem_u32(bars), empty0 = full0 + 8 * C::NS, accf0 = empty0 + 8 * C::NS,
                   acce0 = accf0 + 8 * S, wbar = acce0 + 8 * S, dbar = wbar + 8, attf0 = dbar + 8,
                   skipf0 = attf0 + 16, landed0 = skipf0 + 8 * S;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 3 * C::NS + 3 * S + 4);
    const uint32_t gatef0 = dev::smem_u32(bars + 3 * C::NS + 3 * S + 5), gatee0 = gatef0 + 8 * kGateSlots;
    RowPlan *plans = reinterpret_cast<RowPlan *>(sm + C::PLOFF);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr bool bulk_in = IN == kInRows;  // strip-chunked input by bulk copies, else the NCHW RGB model input
    // strip-chunked input copied by its own warp (see the producer)
    constexpr bool split_in = bulk_in && (EK == kEpiD2S || KPAD <= 32);
    const int H = a.H, W = a.W;

    // ---- set-up
    if (tid == 0) {
        for (int s = 0; s < C::NS; s++) {
            dev::mbar_init(full0 + 8 * s, bulk_in ? 1 : kProdWarps * 32);
            dev::mbar_init(empty0 + 8 * s, 1);
            dev::mbar_init(landed0 + 8 * s, 1);
        }
        for (int s = 0; s < S; s++) {
            dev::mbar_init(accf0 + 8 * s, 1);
            dev::mbar_init(skipf0 + 8 * s, 1);
            // the tanh gate's epilogue groups take alternate rows: four warps free each slot
            dev::mbar_init(acce0 + 8 * s, ATT ? kEpiWarps / 2 : kEpiWarps);
        }
        dev::mbar_init(wbar, 1);
        dev::mbar_init(dbar, 1);
        dev::mbar_init(attf0, 1);
        dev::mbar_init(attf0 + 8, 1);
        if (GATE) {
            for (int g = 0; g < kGateSlots; g++) {
                dev::mbar_init(gatef0 + 8 * g, 1);
                dev::mbar_init(gatee0 + 8 * g, kEpiWarps);
            }
        }
        dev::fence_mbar_init();
        // the weights were uploaded long before any kernel ran: fetch them before the wait below
        const uint32_t att_bytes = ATT ? (uint32_t)(a.att_kpad * a.att_npad * 2) : 0u;
        dev::mbar_arrive_expect_tx(wbar, C::WBYTES + att_bytes);
        dev::bulk_load(wbase, a.wimg, C::WBYTES, wbar);
        if (ATT) dev::bulk_load(sbase + C::ATOFF, a.att_img, att_bytes, wbar);
    }
    if (warp == kMmaWarp) dev::tmem_alloc(dev::smem_u32(tslot), kTmemCols);
    // K chunks the producer never writes (channel padding) are zero for the kernel's lifetime
    {
        const int written = bulk_in ? a.cin / 8 : IN == kInRgb ? 1 : 2;
        const int nz = (C::KC - written) * kHalo;
        for (int s = 0; s < C::NS * C::RP; s++)
            for (int i = tid; i < nz; i += kConvThreads)
                reinterpret_cast<uint4 *>(sm + C::AOFF + s * C::SLOT + written * C::LBO_A)[i] = make_uint4(0, 0, 0, 0);
    }
    for (int n = tid; n < 64; n += kConvThreads) {
        sbias[n] = n < NPAD ? a.bias[n] : 0.f;
        // PReLU slopes less one (the epilogue's v + min(v, 0) * (slope - 1))
        sslope[n] = ((n < NPAD && a.slope) ? a.slope[n] : 0.f) - 1.f;
        satt[n] = (ATT && n < a.att_npad) ? a.att_bias[n] : 0.f;
    }
    dev::fence_proxy_async();
    dev::tc_fence_before();
    __syncthreads();
    dev::tc_fence_after();
    const uint32_t tmem = *tslot;
    // launched with programmatic stream serialisation: the set-up above overlapped the previous
    // kernel's tail; its outputs (this kernel's inputs) are read only after this wait
    dev::griddep_launch_dependents();
    dev::griddep_wait();

    if (warp < kProdWarps) {
        // ================= producer: stages each input row and writes its MMA plan beside it,
        // after waiting for the accumulators the row starts to be free
        static_assert(!GATE || bulk_in, "the SPAN gate reads strip-chunked maps");
        if constexpr (bulk_in) {
            if constexpr (GATE) {
                if (warp == 3) {
                    // the gate warp: the block input's (row, strip) block of each output, in the
                    // epilogue's output order, into a ring of kGateSlots slots (one bulk copy each,
                    // completing gatef[slot]); a slot is reused once the epilogue's eight warps have
                    // read it (gatee). Reading the block input from global memory in the epilogue
                    // left each row waiting on DRAM latency (gate conv 157 us against 94 for the
                    // activation conv at 1080p, 48 channels).
                    const int ccout = a.cout / 8;
                    const uint32_t bytes = (uint32_t)ccout * kHalo * 16;
                    SegIter gseg(W, a.row_begin, a.row_end);
                    uint32_t ot = 0;
                    int strip, ya, yb;
                    bool ok = true;
                    while (ok && gseg.next(strip, ya, yb)) {
                        for (int o = ya; o < yb; o++, ot++) {
                            const uint32_t g = ot % kGateSlots, ph = (ot / kGateSlots) & 1u;
                            if (!(ok = dev::mbar_wait_warp(gatee0 + 8 * g, ph ^ 1u, a.err, kErrProdEmpty))) break;
                            if (lane == 0) {
                                dev::mbar_arrive_expect_tx(gatef0 + 8 * g, bytes);
                                dev::bulk_load(sbase + C::GOFF + g * C::GATE_ROW,
                                               a.resid + map_at(o, strip, 0, 0, a.nstrips, ccout), bytes, gatef0 + 8 * g);
                            }
                            __syncwarp();
                        }
                    }
                    // on an error exit, let the last copy land before the CTA can leave
                    if (!ok && ot > 0 && lane == 0)
                        dev::mbar_wait(gatef0 + 8 * ((ot - 1) % kGateSlots), ((ot - 1) / kGateSlots) & 1u, nullptr, 0);
                }
            }
            // Depth-to-space convs (skip rows to copy) and the narrow inputs (up to 32 channels:
            // a staged row's copy is 2-8 KB) split the producer in two warps on different SM
            // sub-partitions, walking the same rows in the same stages: warp 0 copies, warp 2
            // plans. One warp doing both spends ~2000 cycles of its own a stage there, more than
            // the stage's MMAs (tail 108 -> 96 us, head 86 -> 81 us, the 24-channel body 70.0 ->
            // 64.0 us at 1080p); the 64-channel body measured the same split and the 48-channel
            // one 6 % slower.
            if constexpr (split_in) {
                if (warp == 0) {
                    // the copier: once a stage's buffer is free, one bulk copy per staged row, all
                    // completing landed[s]; it waits for nothing else
                    const int kcin = a.cin / 8;
                    const uint32_t bytes = (uint32_t)kcin * kHalo * 16;
                    RowWalk walk(W, a.row_begin, a.row_end, a.img_h);
                    uint32_t pi = 0;  // stage fills so far (pairs of rows)
                    bool ok = true;
                    while (ok && walk.next()) {
                        const uint32_t s = pi % C::NS, ph = (pi / C::NS) & 1;
                        if (!(ok = dev::mbar_wait_warp(empty0 + 8 * s, ph ^ 1, a.err, kErrProdEmpty))) break;
                        int rr[C::RP], rs[C::RP];
                        int n = 0;
    #pragma unroll
                        for (int h = 0; h < C::RP; h++) {
                            if (h > 0 && (n < h || !walk.next())) break;
                            rr[h] = walk.r;
                            rs[h] = walk.strip;
                            n = h + 1;
                        }
                        if (lane == 0) {
                            dev::mbar_arrive_expect_tx(landed0 + 8 * s, (uint32_t)n * bytes);
    #pragma unroll
                            for (int h = 0; h < C::RP; h++)
                                if (h < n)
                                    // the (row, strip) block, halo columns included: the staged row as it is
                                    dev::bulk_load(abase + s * C::STAGE + h * C::SLOT,
                                                   a.src + map_at(rr[h], rs[h], 0, 0, a.nstrips, kcin), bytes, landed0 + 8 * s);
                        }
                        __syncwarp();
                        pi++;
                    }
                    if (ok) {
                        // the terminator stage lands at once (no bytes)
                        const uint32_t s = pi % C::NS, ph = (pi / C::NS) & 1;
                        if ((ok = dev::mbar_wait_warp(empty0 + 8 * s, ph ^ 1, a.err, kErrProdEmpty)) && lane == 0)
                            dev::mbar_arrive(landed0 + 8 * s);
                    }
                    // on an error exit, let the last copies land before the CTA can leave
                    if (!ok && pi > 0 && lane == 0) {
                        const uint32_t s = (pi - 1) % C::NS, ph = ((pi - 1) / C::NS) & 1;
                        dev::mbar_wait(landed0 + 8 * s, ph, nullptr, 0);
                    }
                } else if (warp == 2) {
                    // the planner: per staged row, waits for the accumulators the row starts to be free
                    // and writes the row's MMA plan beside it; one arrival on full[s] a stage, and after
                    // the last row one terminator stage. Every lane walks the same rows (warp-uniform
                    // control flow); lane 0 waits and writes.
                    RowWalk walk(W, a.row_begin, a.row_end, a.img_h);
                    uint32_t pi = 0;
                    bool ok = true;
                    while (ok && walk.next()) {
                        const uint32_t s = pi % C::NS, ph = (pi / C::NS) & 1;
                        // the stage's plans are free once its MMAs are done
                        if (!(ok = dev::mbar_wait_warp(empty0 + 8 * s, ph ^ 1, a.err, kErrProdEmpty))) break;
                        int h = 0;
    #pragma unroll
                        for (; h < C::RP; h++) {
                            if (h > 0 && !walk.next()) break;
                            RowPlan pl;
                            RowWaits wt;
                            plan_row<S, NPAD, C::NG>(walk, tmem, accf0, acce0, pl, wt);
                            bool good = true;
                            if (lane == 0) good = wt.wait(a.err);
                            if (!(ok = __shfl_sync(0xffffffffu, good, 0))) break;
                            if (lane == 0) plans[s * C::RP + h] = pl;
                            __syncwarp();
                        }
                        // a stage short of rows (the walk's end, or a wait that gave up) marks the rest
                        // empty: the MMA thread skips rows whose plan has no pieces
                        if (lane == 0) {
                            for (int e = h; e < C::RP; e++) plans[s * C::RP + e].np = 0;
                            dev::mbar_arrive(full0 + 8 * s);
                        }
                        pi++;
                    }
                    if (ok) {
                        // the terminator: one more stage whose first plan says the walk is over, so the
                        // MMA thread never walks the rows itself
                        const uint32_t s = pi % C::NS, ph = (pi / C::NS) & 1;
                        if ((ok = dev::mbar_wait_warp(empty0 + 8 * s, ph ^ 1, a.err, kErrProdEmpty)) && lane == 0) {
                            plans[s * C::RP].np = kPlanEnd;
                            dev::mbar_arrive(full0 + 8 * s);
                        }
                    }
                } else if (EK == kEpiD2S && warp == 3 && a.skip_smem) {
                    // the skip warp (depth-to-space): each output's model-input row (the
                    // nearest-upsampled skip it adds: 3 planes x the strip's 128 pixels) bulk-copied
                    // into its accumulator slot's skip buffer once the slot is free, in the
                    // epilogue's output order (the epilogue reads the buffer before it frees the
                    // slot). In the planner these copies made it the tail's slowest role (~1200
                    // cycles of its own a row).
                    SegIter kseg(W, a.row_begin, a.row_end);
                    uint32_t ot = 0;
                    int strip, ya, yb;
                    bool ok = true;
                    while (ok && kseg.next(strip, ya, yb)) {
                        const int x0 = strip * kTileM;
                        const uint32_t rb = (uint32_t)min(kTileM, W - x0) * 2;
                        for (int o = ya; o < yb; o++, ot++) {
                            const int sl = ring_slot<S>(ot);
                            if (!(ok = dev::mbar_wait_warp(acce0 + 8 * sl, ring_phase<S>(ot) ^ 1u, a.err, kErrProdAccEmpty)))
                                break;
                            if (lane == 0) dev::mbar_arrive_expect_tx(skipf0 + 8 * sl, 3 * rb);
                            __syncwarp();
                            if (lane < 3)
                                dev::bulk_load(sbase + C::SKOFF + sl * C::SKIP_ROW + lane * (kTileM * 2),
                                               a.resid + ((size_t)lane * H + o) * W + x0, rb, skipf0 + 8 * sl);
                            __syncwarp();
                        }
                    }
                    // on an error exit, let the last copies land before the CTA can leave
                    if (!ok && ot > 0 && lane == 0)
                        dev::mbar_wait(skipf0 + 8 * ring_slot<S>(ot - 1), ring_phase<S>(ot - 1), nullptr, 0);
                }
            } else {
                if (warp == 0) {
                    // warp 0: every lane walks the same rows (warp-uniform control flow); lane 0 issues
                    // each row's bulk copy, waits for the accumulators, writes the plan and arrives
                    const int kcin = a.cin / 8;
                    const uint32_t bytes = (uint32_t)kcin * kHalo * 16;
                    RowWalk walk(W, a.row_begin, a.row_end, a.img_h);
                    uint32_t pi = 0;  // stage fills so far (pairs of rows)
                    bool ok = true;
                    while (ok && walk.next()) {
                        const uint32_t s = pi % C::NS, ph = (pi / C::NS) & 1;
                        if (!(ok = dev::mbar_wait_warp(empty0 + 8 * s, ph ^ 1, a.err, kErrProdEmpty))) break;
                        // the stage's copies go out as soon as its buffer is free (waiting first for the
                        // accumulators the rows start, as the plans need, left the MMA thread waiting
                        // ~800 cycles a stage for data: the TMEM ring, not the stages, bounded how far
                        // ahead rows were fetched); then the accumulator waits, the plans and, for
                        // depth-to-space, the skip rows, whose buffers belong to the accumulator slots
                        RowPlan pl[C::RP];
                        RowWaits wts[C::RP];
                        int rows_r[C::RP], rows_strip[C::RP];
                        int n = 0;
    #pragma unroll
                        for (int h = 0; h < C::RP; h++) {
                            if (h > 0 && (n < h || !walk.next())) break;
                            plan_row<S, NPAD, C::NG>(walk, tmem, accf0, acce0, pl[h], wts[h]);
                            rows_r[h] = walk.r;
                            rows_strip[h] = walk.strip;
                            if (lane == 0) dev::mbar_expect_tx(full0 + 8 * s, bytes);
                            // the (row, strip) block, halo columns included: the staged row as it is
                            if (lane == 0)
                                dev::bulk_load(abase + s * C::STAGE + h * C::SLOT,
                                               a.src + map_at(walk.r, walk.strip, 0, 0, a.nstrips, kcin), bytes, full0 + 8 * s);
                            n = h + 1;
                        }
                        int h = 0;
    #pragma unroll
                        for (; h < C::RP; h++) {
                            if (h >= n) break;
                            const RowWaits &wt = wts[h];
                            bool good = true;
                            if (lane == 0) good = wt.wait(a.err);
                            if (!(ok = __shfl_sync(0xffffffffu, good, 0))) break;
                            if (lane == 0) plans[s * C::RP + h] = pl[h];
                            if constexpr (EK == kEpiD2S) {
                                // the skip rows of the outputs this row starts (r + 1; r at an image's
                                // first row), into their slots: lanes 8-10 and 11-13, one plane each
                                if (a.skip_smem) {
                                    const int x0 = rows_strip[h] * kTileM;
                                    const uint32_t rb = (uint32_t)min(kTileM, W - x0) * 2;
                                    const int k = lane - 8, which = k / 3, c3 = k % 3;
                                    const bool mine = k >= 0 && k < 6 && (which == 0 ? wt.w0 : wt.w1);
                                    const uint32_t sl = ((which == 0 ? wt.bar0 : wt.bar1) - acce0) / 8;
                                    const int orow = which == 0 ? rows_r[h] + 1 : rows_r[h];
                                    if ((k == 0 && wt.w0) || (k == 3 && wt.w1)) dev::mbar_arrive_expect_tx(skipf0 + 8 * sl, 3 * rb);
                                    __syncwarp();
                                    if (mine)
                                        dev::bulk_load(sbase + C::SKOFF + sl * C::SKIP_ROW + c3 * (kTileM * 2),
                                                       a.resid + ((size_t)c3 * H + orow) * W + x0, rb, skipf0 + 8 * sl);
                                }
                            }
                            __syncwarp();
                        }
                        // a stage short of rows (the walk's end, or a wait that gave up) marks the rest
                        // empty: the MMA thread skips rows whose plan has no pieces. One arrival per
                        // stage; it completes once the copies above have landed.
                        if (lane == 0) {
                            for (int e = h; e < C::RP; e++) plans[s * C::RP + e].np = 0;
                            dev::mbar_arrive(full0 + 8 * s);
                        }
                        pi++;
                    }
                    if (ok) {
                        // the terminator: one more stage whose first plan says the walk is over, so the
                        // MMA thread never walks the rows itself
                        const uint32_t s = pi % C::NS, ph = (pi / C::NS) & 1;
                        if ((ok = dev::mbar_wait_warp(empty0 + 8 * s, ph ^ 1, a.err, kErrProdEmpty)) && lane == 0) {
                            plans[s * C::RP].np = kPlanEnd;
                            dev::mbar_arrive(full0 + 8 * s);
                        }
                    }
                    // on an error exit, let the last copies land before the CTA can leave
                    if (!ok && pi > 0 && lane == 0) {
                        const uint32_t s = (pi - 1) % C::NS, ph = ((pi - 1) / C::NS) & 1;
                        dev::mbar_wait(full0 + 8 * s, ph, nullptr, 0);
                    }
                }
            }
        } else {
            // NCHW RGB model input -> the staged row. Plain: chunk 0 = {r, g, b, 0, 0, 0, 0, 0} per
            // pixel. Pixel-unshuffled by 2 (the input is [3][2H][2W]): channel c * 4 + ry * 2 + rx
            // is input pixel (2y + ry, 2x + rx) of plane c (PyTorch's pixel_unshuffle order), so the
            // pair (rx 0, 1) is one 4-byte load and chunks 0 and 1 hold pairs (c, ry) = (0, 0) ..
            // (2, 1), then zeros. Each thread holds pixels tid and tid + 128 of a row. Two stages'
            // pixels are kept in registers, loaded one stage ahead of their use, so the load latency
            // overlaps a whole stage of work.
            constexpr bool U2 = IN == kInRgbUnshuffle2;
            constexpr int NV = U2 ? 6 : 3;  // loads per pixel: fp16 values, or fp16 pairs (c, ry)
            RowWalk wl(W, a.row_begin, a.row_end, a.img_h), wp(W, a.row_begin, a.row_end, a.img_h);
            const int IW = U2 ? 2 * W : W;                 // input row length
            const size_t plane = (size_t)(U2 ? 2 * H : H) * IW;
            typedef uint32_t StagePix[C::RP][2][NV];
            // the next stage's pixels (walk wl), as raw fp16 bits; returns its row count
            auto prefetch = [&](StagePix &pv) -> int {
                int n = 0;
#pragma unroll
                for (int h = 0; h < C::RP; h++) {
                    if (n < h || !wl.next()) break;
                    const int x0 = wl.strip * kTileM, r = wl.r;
#pragma unroll
                    for (int k = 0; k < 2; k++) {
                        const int p = tid + k * kProdWarps * 32, x = x0 - 1 + p;
                        const bool in = p < kHalo && x >= 0 && x < W;
#pragma unroll
                        for (int j = 0; j < NV; j++) {
                            if constexpr (U2) {
                                const int c = j >> 1, ry = j & 1;
                                const __half *px = a.src + c * plane + (size_t)(2 * r + ry) * IW + 2 * (in ? x : 0);
                                pv[h][k][j] = in ? __ldg(reinterpret_cast<const unsigned int *>(px)) : 0u;
                            } else {
                                const __half *px = a.src + j * plane + (size_t)r * IW + (in ? x : 0);
                                pv[h][k][j] = in ? (uint32_t)__half_as_ushort(__ldg(px)) : 0u;
                            }
                        }
                    }
                    n = h + 1;
                }
                return n;
            };
            uint32_t pi = 0;
            bool ok = true;
            // stage pi from pv (n rows, walk wp): its plans, its pixels, one arrival
            auto fill = [&](const StagePix &pv, int n) {
                const uint32_t s = pi % C::NS, ph = (pi / C::NS) & 1;
                if (!(ok = dev::mbar_wait(empty0 + 8 * s, ph ^ 1, a.err, kErrProdEmpty))) return;
#pragma unroll
                for (int h = 0; h < C::RP; h++) {
                    if (h >= n) break;
                    wp.next();
                    if (tid == 0) {
                        RowPlan p;
                        RowWaits wt;
                        plan_row<S, NPAD, C::NG>(wp, tmem, accf0, acce0, p, wt);
                        ok = wt.wait(a.err) && ok;
                        if (!ok) p.np = 0;
                        plans[s * C::RP + h] = p;
                    }
                    unsigned char *dst = sm + C::AOFF + s * C::STAGE + h * C::SLOT;
#pragma unroll
                    for (int k = 0; k < 2; k++) {
                        const int p = tid + k * kProdWarps * 32;
                        if (p >= kHalo) continue;
                        // normalisation applies to image pixels; the zero padding stays zero
                        const int x = wp.strip * kTileM - 1 + p;
                        const bool norm = a.in_norm && x >= 0 && x < W;
                        if constexpr (U2) {
                            uint32_t q[6];
#pragma unroll
                            for (int j = 0; j < 6; j++) {
                                q[j] = pv[h][k][j];
                                if (norm) {
                                    const int c = j >> 1;
                                    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&q[j]));
                                    q[j] = pack_h2((f.x - a.in_mean[c]) * a.in_scale[c], (f.y - a.in_mean[c]) * a.in_scale[c]);
                                }
                            }
                            reinterpret_cast<uint4 *>(dst)[p] = make_uint4(q[0], q[1], q[2], q[3]);
                            reinterpret_cast<uint4 *>(dst + C::LBO_A)[p] = make_uint4(q[4], q[5], 0u, 0u);
                        } else {
                            float v[3];
#pragma unroll
                            for (int c = 0; c < 3; c++) {
                                v[c] = __half2float(__ushort_as_half((unsigned short)pv[h][k][c]));
                                if (norm) v[c] = __half2float(__float2half_rn((v[c] - a.in_mean[c]) * a.in_scale[c]));
                            }
                            uint4 q;
                            q.x = pack_h2(v[0], v[1]);
                            q.y = pack_h2(v[2], 0.f);
                            q.z = 0u;
                            q.w = 0u;
                            reinterpret_cast<uint4 *>(dst)[p] = q;
                        }
                    }
                }
                if (tid == 0)
                    for (int e = n; e < C::RP; e++) plans[s * C::RP + e].np = 0;
                dev::fence_proxy_async();
                dev::mbar_arrive(full0 + 8 * s);
                pi++;
            };
            StagePix pa, pb;
            int na = prefetch(pa), nb = prefetch(pb);
            while (ok && na > 0) {
                fill(pa, na);
                if (!ok || nb == 0) break;
                na = prefetch(pa);
                fill(pb, nb);
                if (!ok) break;
                nb = prefetch(pb);
            }
            if (ok) {
                // the terminator stage (every producer thread arrives, as for a filled stage)
                const uint32_t s = pi % C::NS, ph = (pi / C::NS) & 1;
                if (dev::mbar_wait(empty0 + 8 * s, ph ^ 1, a.err, kErrProdEmpty)) {
                    if (tid == 0) plans[s * C::RP].np = kPlanEnd;
                    dev::mbar_arrive(full0 + 8 * s);
                }
            }
        }
    } else if (warp == kIdleWarp) {
        // no work: see kIdleWarp
    } else if (ATT && warp < kMmaWarp) {
      if constexpr (ATT) {
        // ================= epilogue of the tanh gate (x + o) * tanh(att_bias + W_att^T o), o the conv
        // output in fp16 (the reference's semantics). Group g (warps 4 + 4g .. 7 + 4g) takes the
        // output rows of parity g, its warp q TMEM lanes 32q.. (pixels) and whole slots. Per row the
        // group writes o into its A tile, one thread issues the attention GEMM (M 128 pixels, N and
        // K the channels) into the group's own TMEM accumulator, and the group finishes the row when
        // it completes, while the other group works on its own row.
        const int q = warp & 3, g = (warp - kProdWarps) >> 2;
        const uint32_t lanes = (uint32_t)(q * 32) << 16;
        // group g zeroes the slots of parity g, whole (16 columns at a 16-column boundary)
        for (int sl = g; sl < S; sl += 2)
#pragma unroll
            for (int c = 0; c < NPAD; c += 16) dev::tmem_zero16(tmem + lanes + (uint32_t)(sl * NPAD + c));
        dev::tmem_wait_st();
        dev::tc_fence_before();
        dev::named_bar_sync(1, (kEpiWarps + 1) * 32);

        const int px = q * 32 + lane;  // the tile pixel (TMEM lane) of this thread
        unsigned char *atile = sm + C::ATOFF + C::ATT_B + g * C::ATT_A;
        const bool issuer = q == 0 && lane == 0;
        // A: the group's tile, K-major without swizzle: K chunks 128 x 16 bytes apart, 8-pixel groups
        // 128 bytes apart. B: the packed 1x1 weights, K chunks (att_npad / 8) x 128 bytes apart.
        const uint32_t att_lbo_b = (uint32_t)(a.att_npad / 8 * 128);
        const uint64_t att_adesc = dev::sdesc(sbase + C::ATOFF + C::ATT_B + g * C::ATT_A, kTileM * 16, 128);
        const uint64_t att_bdesc = dev::sdesc(sbase + C::ATOFF, att_lbo_b, 128);
        const uint32_t att_idesc = dev::idesc_f16_f32(kTileM, a.att_npad);
        const int att_ks = a.att_kpad / 16;
        const uint32_t att_d = tmem + (uint32_t)((S + g) * NPAD);
        const int ccout = a.cout / 8;
        SegIter seg(W, a.row_begin, a.row_end);
        uint32_t ot = 0, na = 0;  // outputs so far (both groups); this group's rows so far
        int strip, ya, yb;
        bool alive = true;  // the group's verdict: every warp of it had every wait pass
        bool good = true;   // this warp's last attention wait passed
        while (alive && seg.next(strip, ya, yb)) {
            const int x = strip * kTileM + px;
            for (int o = ya; o < yb; o++, ot++) {
                if ((int)(ot & 1u) != g) continue;
                const int slot = ring_slot<S>(ot);
                // the block input x: loaded before the waits, so its latency overlaps them
                EpiIn<NPAD> in;
                epi_prefetch<kEpiGate, NPAD, 0>(in, a, o, x);
                bool ok = good && dev::mbar_wait_warp(accf0 + 8 * slot, ring_phase<S>(ot), a.err, kErrEpiAccFull);
                if (ok) {
                    __syncwarp();
                    dev::tc_fence_after();
                    const uint32_t taddr = tmem + lanes + (uint32_t)(slot * NPAD);
                    // 16 columns at a time, straight to fp16 into the A tile (few registers live
                    // beside the block input)
#pragma unroll
                    for (int c = 0; c < NPAD; c += 16) {
                        // the attention GEMM's K columns only (the output channels padded to 16; the
                        // slot's other columns accumulate zero products and are never read)
                        if (c >= a.att_kpad) break;
                        float t[16];
                        dev::tmem_ld16(taddr + c, t);
                        dev::tmem_wait_ld();
                        uint32_t oh[8];  // fp16(o + bias), channel pairs c .. c + 15
#pragma unroll
                        for (int j = 0; j < 16; j += 2) oh[j / 2] = pack_h2(t[j] + sbias[c + j], t[j + 1] + sbias[c + j + 1]);
#pragma unroll
                        for (int h2 = 0; h2 < 2; h2++)
                            *reinterpret_cast<uint4 *>(atile + (c / 8 + h2) * (kTileM * 16) + px * 16) =
                                make_uint4(oh[4 * h2], oh[4 * h2 + 1], oh[4 * h2 + 2], oh[4 * h2 + 3]);
                    }
#pragma unroll
                    for (int c = 0; c < NPAD; c += 16)
                        if (c < a.att_kpad) dev::tmem_zero16(taddr + c);
                    dev::tmem_wait_st();
                    dev::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) dev::mbar_arrive(acce0 + 8 * slot);
                }
                // the tile is read by the tensor core (the async proxy) once the whole group wrote it
                dev::fence_proxy_async();
                dev::tc_fence_before();
                alive = dev::named_bar_red_and(2 + g, kEpiWarps / 2 * 32, ok);
                if (!alive) break;
                if (issuer) {
                    dev::tc_fence_after();
                    for (int kk = 0; kk < att_ks; kk++)
                        dev::mma_f16(att_d, att_adesc + (uint64_t)((kk * 2 * kTileM * 16) >> 4),
                                     att_bdesc + (uint64_t)((kk * 2 * att_lbo_b) >> 4), att_idesc, kk > 0 ? 1u : 0u, 0);
                    dev::mma_commit(attf0 + 8 * g);
                }
                // a failed wait ends the group at its next barrier (never splits it before one)
                good = dev::mbar_wait_warp(attf0 + 8 * g, na & 1u, a.err, kErrAttFull);
                na++;
                if (!good) continue;
                __syncwarp();
                dev::tc_fence_after();
#pragma unroll
                for (int c16 = 0; c16 < NPAD / 16; c16++) {
                    if (c16 * 16 >= a.cout) break;
                    float ga[16];
                    dev::tmem_ld16(tmem + lanes + (uint32_t)((S + g) * NPAD + c16 * 16), ga);
                    dev::tmem_wait_ld();
#pragma unroll
                    for (int c8 = 0; c8 < 2; c8++) {
                        const int c = c16 * 2 + c8;
                        if (c >= ccout || x >= W) continue;
                        const __half2 *xh = reinterpret_cast<const __half2 *>(&in.gate[c]);
                        uint32_t w4[4];
                        // fp16(o) back from the tile (the tensor core only read it)
                        const uint4 o4 = *reinterpret_cast<const uint4 *>(atile + c * (kTileM * 16) + px * 16);
                        const __half2 *oh2 = reinterpret_cast<const __half2 *>(&o4);
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const int n = c * 8 + 2 * j;
                            const float2 xf = __half22float2(xh[j]);
                            const float2 of = __half22float2(oh2[j]);
                            const float t0 = dev::tanh_fast(ga[c8 * 8 + 2 * j] + satt[n]);
                            const float t1 = dev::tanh_fast(ga[c8 * 8 + 2 * j + 1] + satt[n + 1]);
                            w4[j] = pack_h2((xf.x + of.x) * t0, (xf.y + of.y) * t1);
                        }
                        store_px(a.dst, o, x, c, a.nstrips, ccout, make_uint4(w4[0], w4[1], w4[2], w4[3]));
                    }
                }
                dev::tc_fence_before();
            }
        }
      }
    } else if (warp < kMmaWarp) {
      if constexpr (!ATT) {
        // ================= epilogue: warp (q, h) takes TMEM lanes 32q.. (pixels) and half h of
        // each slot's columns (NPAD / 2: 16, 24 or 32); depth-to-space by 3 (groups of 3 channels
        // across the halves) has half 0 take the whole slot
        const int q = warp & 3, h = (warp - kProdWarps) >> 2;
        const uint32_t lanes = (uint32_t)(q * 32) << 16;
        const bool whole = EK == kEpiD2S && a.R == 3;
        constexpr int CWA = NPAD / 2, CWB = NPAD - CWA;
        auto run_half = [&](auto cw_tag, auto c0_tag) {
            constexpr int CW = decltype(cw_tag)::value, C0 = decltype(c0_tag)::value;
            // every accumulator starts from its channel's bias, so the epilogue adds none: this warp's
            // columns of the bias as TMEM words, written into each slot it hands back (the MMA warp
            // waits on named barrier 1 for the first fill)
            uint32_t bz[CW];
#pragma unroll
            for (int c = 0; c < CW; c++) bz[c] = __float_as_uint(sbias[C0 + c]);
            // taddr: a slot's base (the warp's lanes)
            auto fill_bias = [&](uint32_t taddr) { tmem_st_cols<CW, C0>(taddr, bz); };
            for (int sl = 0; sl < S; sl++) fill_bias(tmem + lanes + (uint32_t)(sl * NPAD));
            dev::tmem_wait_st();
            dev::tc_fence_before();
            dev::named_bar_sync(1, (kEpiWarps + 1) * 32);

            SegIter seg(W, a.row_begin, a.row_end);
            uint32_t ot = 0;
            int strip, ya, yb;
            bool ok = true;
            // a row's global inputs (skip pixel, gate's block input) are loaded ahead (three rows for
            // the skip pixel, whose DRAM latency is several rows of this epilogue; one for the gate's
            // larger input), so their latency overlaps earlier rows' epilogues
            auto prefetch = [&](EpiIn<CW> &in, EpiIn<NPAD> &inw, int o, int x) {
                if (!whole)
                    epi_prefetch<EK, CW, C0>(in, a, o, x);
                else if (C0 == 0)
                    epi_prefetch<EK, NPAD, 0>(inw, a, o, x);
            };
            constexpr int PF = EK == kEpiD2S ? 3 : 1;
            // a skip or a gate input in shared memory needs no prefetch
            const bool pf_on = !(EK == kEpiD2S && a.skip_smem) && !GATE;
            while (ok && seg.next(strip, ya, yb)) {
                const int x0 = strip * kTileM;
                const int x = x0 + q * 32 + lane;
                EpiRing<PF, EpiIn<CW>> rin;
                EpiRing<PF, EpiIn<NPAD>> rinw;
#pragma unroll
                for (int k = 0; k < PF; k++)
                    if (pf_on && ya + k < yb) prefetch(rin.e[k], rinw.e[k], ya + k, x);
                for (int o = ya; o < yb; o++, ot++) {
                    const int slot = ring_slot<S>(ot);
                    EpiIn<CW> in = rin.e[0];
                    EpiIn<NPAD> inw = rinw.e[0];
                    EpiIn<CW> nin;
                    EpiIn<NPAD> ninw;
                    if (pf_on && o + PF < yb) prefetch(nin, ninw, o + PF, x);
                    if (!(ok = dev::mbar_wait_warp(accf0 + 8 * slot, ring_phase<S>(ot), a.err, kErrEpiAccFull))) break;
                    if constexpr (EK == kEpiD2S) {
                        if (!pf_on) {
                            // the skip row landed in this output's slot (its own barrier, one phase per use)
                            if (!(ok = dev::mbar_wait_warp(skipf0 + 8 * slot, ring_phase<S>(ot), a.err, kErrEpiAccFull))) break;
                            const __half *sk = reinterpret_cast<const __half *>(sm + C::SKOFF + slot * C::SKIP_ROW);
#pragma unroll
                            for (int c3 = 0; c3 < 3; c3++) {
                                const float v = x < W ? __half2float(sk[c3 * kTileM + (x - x0)]) : 0.f;
                                in.skip[c3] = v;
                                inw.skip[c3] = v;
                            }
                        }
                    }
                    __syncwarp();
                    dev::tc_fence_after();
                    const uint32_t taddr = tmem + lanes + (uint32_t)(slot * NPAD);
                    if (!whole) {
                        float v[CW];
                        tmem_ld_cols<CW, C0>(taddr, v);
                        dev::tmem_wait_ld();
                        // hand the columns back holding the bias: the MMAs accumulate onto it
                        fill_bias(taddr);
                        dev::tmem_wait_st();
                        dev::tc_fence_before();
                        __syncwarp();
                        if (lane == 0) dev::mbar_arrive(acce0 + 8 * slot);
                        if constexpr (GATE) {
                            // the block input of this output, staged by the gate warp: this warp's
                            // chunks of its pixel, then the slot goes back
                            const uint32_t g = ot % kGateSlots;
                            if (!(ok = dev::mbar_wait_warp(gatef0 + 8 * g, (ot / kGateSlots) & 1u, a.err, kErrEpiAccFull)))
                                break;
                            const uint4 *grow = reinterpret_cast<const uint4 *>(sm + C::GOFF + g * C::GATE_ROW);
                            const int ccout = a.cout / 8;
#pragma unroll
                            for (int c = 0; c < CW / 8; c++)
                                if (C0 / 8 + c < ccout) in.gate[c] = grow[(C0 / 8 + c) * kHalo + (x - x0) + 1];
                            __syncwarp();
                            if (lane == 0) dev::mbar_arrive(gatee0 + 8 * g);
                        }
                        epi_store<EK, CW, C0>(v, a, sslope, o, x, in);
                    } else {
                        // depth-to-space by 3 only comes with 27 output channels (NPAD 32)
                        if constexpr (NPAD == 32 && EK == kEpiD2S && C0 == 0) {
                            float v[NPAD];
#pragma unroll
                            for (int c = 0; c < NPAD; c += 16) {
                                float t[16];
                                dev::tmem_ld16(taddr + c, t);
#pragma unroll
                                for (int j = 0; j < 16; j++) v[c + j] = t[j];
                            }
                            dev::tmem_wait_ld();
                            // both halves back to the bias (the other half's from shared memory)
                            fill_bias(taddr);
                            {
                                uint32_t bo[CWB];
#pragma unroll
                                for (int j = 0; j < CWB; j++) bo[j] = __float_as_uint(sbias[CWA + j]);
                                tmem_st_cols<CWB, CWA>(taddr, bo);
                            }
                            dev::tmem_wait_st();
                            dev::tc_fence_before();
                            __syncwarp();
                            if (lane == 0) dev::mbar_arrive(acce0 + 8 * slot);
                            epi_store<EK, NPAD, 0>(v, a, sslope, o, x, inw);
                        } else {
                            dev::tc_fence_before();
                            __syncwarp();
                            if (lane == 0) dev::mbar_arrive(acce0 + 8 * slot);
                        }
                    }
                    rin.push(nin);
                    rinw.push(ninw);
                }
            }
        };
        if (h == 0)
            run_half(std::integral_constant<int, CWA>{}, std::integral_constant<int, 0>{});
        else
            run_half(std::integral_constant<int, CWB>{}, std::integral_constant<int, CWA>{});
      }
    } else {
        // ================= MMA issuer (one thread). It takes a stage of RP rows per wait and
        // commit, and waits for the next stage between the rows' MMAs.
        dev::named_bar_sync(1, (kEpiWarps + 1) * 32);
        dev::tc_fence_after();
        if (lane == 0) {
            bool ok = dev::mbar_wait(wbar, 0, a.err, kErrWeights);
            // descriptor templates: the start address is the low 14 bits (16-byte units), so a byte
            // offset d is added as d >> 4
            const uint64_t bdesc0 = dev::sdesc(wbase, C::LBO_B, 128);
            const uint64_t adesc_base = dev::sdesc(abase, C::LBO_A, 128);
            // the pi-th stage fill: wait until it is full, then take its rows' plans
            static_assert(C::RP == 2, "the loop below takes stages of two rows");
            auto fetch = [&](uint32_t pi, RowPlan &p0, RowPlan &p1) -> bool {
                const uint32_t s = pi % C::NS;
                // the stage's plans (full), and where a separate warp copies the rows, the rows (landed)
                bool good = dev::mbar_wait(full0 + 8 * s, (pi / C::NS) & 1, a.err, kErrMmaFull);
                if (split_in && good) good = dev::mbar_wait(landed0 + 8 * s, (pi / C::NS) & 1, a.err, kErrMmaFull);
                p0 = plans[s * C::RP];
                p1 = plans[s * C::RP + 1];
                dev::tc_fence_after();
                return good;
            };
            // straight-line per stage; the producer's terminator stage ends the loop (so no row
            // bookkeeping here, which measured ~100 cycles a row with the tensor pipe idle)
            RowPlan c0, c1, n0, n1;
            uint32_t pi = 0;
            ok = ok && fetch(0, c0, c1);
            while (ok && c0.np != kPlanEnd) {
                const uint32_t s = pi % C::NS;
                const uint64_t adesc0 = adesc_base + (uint64_t)((s * C::STAGE) >> 4);
                // row 0, its completed outputs' commits at once (the epilogue starts on them a row
                // earlier); row 1's first tap column, then the next stage's wait and plans while
                // those MMAs run (the pipe queues only a few, so bookkeeping between two rows
                // leaves it idle), the rest of row 1 and the stage's commits
                if (c0.np) issue_plan<0, 3, C::KS, C::KC, C::NG, C::LBO_A>(adesc0, bdesc0, c0);
                if (c0.np && c0.commit_a) dev::mma_commit(c0.commit_a);
                if (c0.np && c0.commit_b) dev::mma_commit(c0.commit_b);
                if (c1.np) issue_plan<0, 1, C::KS, C::KC, C::NG, C::LBO_A>(adesc0 + (uint64_t)(C::SLOT >> 4), bdesc0, c1);
                const bool okn = fetch(pi + 1, n0, n1);
                if (c1.np) issue_plan<1, 3, C::KS, C::KC, C::NG, C::LBO_A>(adesc0 + (uint64_t)(C::SLOT >> 4), bdesc0, c1);
                dev::mma_commit(empty0 + 8 * s);
                if (c1.np && c1.commit_a) dev::mma_commit(c1.commit_a);
                if (c1.np && c1.commit_b) dev::mma_commit(c1.commit_b);
                pi++;
                ok = okn;
                c0 = n0;
                c1 = n1;
            }
            // every MMA issued has completed before TMEM can be released
            dev::mma_commit(dbar);
            dev::mbar_wait(dbar, 0, a.err, kErrDrain);
        }
        __syncwarp();
    }

    dev::tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        dev::tc_fence_after();
        dev::tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace ajib
