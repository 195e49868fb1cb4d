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
 * Feature maps live in HBM as row-chunked, padded NHWC: element (y, x, c) of a C-channel map is
 * at ((y * C/8 + c/8) * Wp + x + 1) * 8 + c % 8 (fp16), Wp = 128 * ceil(W / 128) + 2, with the
 * pad columns (x = -1 and x >= W) zero. So the staged row's 8-channel chunk k is one contiguous
 * 2080-byte run, fetched by one bulk copy (the TMA unit) with the zero padding already in place,
 * and the epilogue's stores of one chunk for 32 consecutive pixels are one coalesced 512-byte
 * write.
 *
 * A CTA is persistent on one SM and walks a contiguous run of (strip, row) tiles down a
 * 128-pixel-wide vertical strip, so each input row is fetched once. Roles:
 *   warps 0-3  producer: one thread issues the bulk copies of each input row (row-chunked
 *              inputs), or all 128 threads convert the NCHW RGB model input into the same layout;
 *   warps 4-7  epilogue: TMEM -> registers (one pixel per thread), bias, activation, SPAN gate or
 *              depth-to-space with the model-input skip, fp16 store; then zero the slot;
 *   warp 8     MMA issuer (one thread) and TMEM owner.
 * Weights for all 9 taps stay resident in shared memory for the CTA's lifetime.
 *
 * The semantics are those of the reference kernel k_conv3x3 (src/native/conv_kernels.cuh:100-350)
 * with fp32 accumulation and an fp32 epilogue instead of fp16 ones (one rounding to fp16 at the
 * store).
 */
#pragma once

#include <cuda_fp16.h>

#include "sm100.cuh"

namespace ajib {

constexpr int kTileM = 128;        // output pixels per tile (the MMA's M)
constexpr int kHalo = kTileM + 2;  // staged input pixels per row
constexpr int kTmemCols = 512;     // the whole TMEM: the accumulator ring
constexpr int kConvThreads = 288;  // 9 warps
constexpr int kMaxSmem = 227 * 1024;

// error codes written to the status word (which wait timed out)
enum { kErrProdEmpty = 101, kErrMmaFull = 102, kErrMmaAccEmpty = 103, kErrEpiAccFull = 104, kErrWeights = 105,
       kErrDrain = 106 };

struct ConvDev {
    const __half *src;    // row-chunked map [H][cin] or NCHW [3][H][W]
    const __half *resid;  // gate: row-chunked [H][cout]; depth-to-space: NCHW model input [3][H][W] or null
    __half *dst;          // row-chunked [H][cout] or NCHW [3][R*H][R*W]
    const unsigned char *wimg;  // packed B operand image, all taps
    const float *bias;    // NPAD floats
    const float *slope;   // NPAD floats or null
    int *err;             // status word
    int H, W, cin, cout;
    int in_mode, act, gate, R;  // R = 0: row-chunked output, else depth-to-space factor
    int in_norm, out_clamp;
    float in_mean[3], in_scale[3];
    int row_begin, row_end;
    int pitch;            // Wp: padded pixels per chunk row of the row-chunked maps
    int img_h;            // rows per image: H = n * img_h images stacked along H, convolved apart
};

// The input rows a segment of output rows [ya, yb) reads: one-row halos that stay inside the
// image (a stack of images of img_h rows each).
__device__ __forceinline__ void segment_rows(int ya, int yb, int img_h, int &r0, int &r1)
{
    r0 = (ya % img_h == 0) ? ya : ya - 1;
    r1 = (yb % img_h == 0) ? yb - 1 : yb;
}

// Padded pixels per chunk row of a row-chunked feature map of width W.
__host__ __device__ constexpr int feature_pitch(int W) { return (W + kTileM - 1) / kTileM * kTileM + 2; }

template <int KPAD, int NPAD>
struct ConvCfg {
    static_assert(KPAD % 16 == 0 && NPAD % 16 == 0 && KPAD <= 64 && NPAD <= 64, "padded channel counts");
    static constexpr int KC = KPAD / 8;       // 8-channel chunks per pixel
    static constexpr int KS = KPAD / 16;      // MMA K steps per tap
    static constexpr int NG = NPAD / 8;       // 8-row core-matrix groups of one tap's B
    static constexpr int S = kTmemCols / NPAD;  // accumulator ring slots
    static constexpr int LBO_A = kHalo * 16;  // bytes between K chunks of a staged row
    static constexpr int LBO_B = 3 * NG * 128;  // bytes between K chunks of a stacked-tap B
    static constexpr int SLOT = (KC * LBO_A + 1023) / 1024 * 1024;
    static constexpr int WBYTES = 9 * KPAD * NPAD * 2;
    static constexpr int AOFF = (WBYTES + 1023) / 1024 * 1024;
    static constexpr int FIXED = AOFF + 2 * 64 * 4 + 1024 + 1024;
    static constexpr int NS_FIT = (kMaxSmem - FIXED) / SLOT;
    static constexpr int NS = NS_FIT > 6 ? 6 : NS_FIT;
    static_assert(NS >= 2 && S >= 4, "pipeline depth");
    static constexpr int POFF = AOFF + NS * SLOT;  // bias[64], slope[64] floats
    static constexpr int BOFF = POFF + 2 * 64 * 4;  // mbarriers: full[NS], empty[NS], accf[S], acce[S], wbar, dbar
    static constexpr int SMEM = BOFF + 1024 + 1024;  // + alignment slack for the base
    static_assert((2 * NS + 2 * S + 2) * 8 + 8 <= 1024, "barrier area");
};

// The run of tiles a CTA owns, split into per-strip segments. All roles walk the same sequence.
struct SegIter {
    long L, L1;
    int rows, row_begin;
    __device__ SegIter(int W, int row_begin_, int row_end)
    {
        row_begin = row_begin_;
        rows = row_end - row_begin_;
        const long strips = (W + kTileM - 1) / kTileM;
        const long T = strips * rows;
        L = (long)blockIdx.x * T / gridDim.x;
        L1 = (long)(blockIdx.x + 1) * T / gridDim.x;
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

__device__ __forceinline__ uint32_t pack_h2(float a, float b)
{
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Depth-to-space by R into NCHW [3][R*H][R*W] (PixelShuffle / DepthToSpace CRD: channel
// c*R*R + ry*R + rx -> [c][R*y + ry][R*x + rx]), plus the nearest-upsampled model input when
// given, optionally clamped to [0, 1]; one rounding to fp16.
template <int R, int NPAD>
__device__ __forceinline__ void store_d2s(const float (&v)[NPAD], const ConvDev &a, int o, int x)
{
    if constexpr (3 * R * R <= NPAD) {
        const int W = a.W, H = a.H;
        const size_t OW = (size_t)R * W, OH = (size_t)R * H;
#pragma unroll
        for (int c3 = 0; c3 < 3; c3++) {
            const float add = a.resid ? __half2float(a.resid[((size_t)c3 * H + o) * W + x]) : 0.f;
#pragma unroll
            for (int ry = 0; ry < R; ry++) {
                __half *d = a.dst + ((size_t)c3 * OH + (size_t)R * o + ry) * OW + (size_t)R * x;
                float t[R];
#pragma unroll
                for (int rx = 0; rx < R; rx++) {
                    float val = v[c3 * R * R + ry * R + rx] + add;
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
}

// The ring slot of the j-th output row a CTA produces, and its mbarrier phase parity.
template <int S>
__device__ __forceinline__ int ring_slot(uint32_t j) { return S - 1 - (int)(j % S); }
template <int S>
__device__ __forceinline__ uint32_t ring_phase(uint32_t j) { return (j / S) & 1u; }

// One staged row's MMAs: for every horizontal tap dx and K step kk, one MMA per piece (a run of
// adjacent accumulators with consecutive tap rows). NP pieces, unrolled straight-line.
template <int NP, int KS, int KC, int NG, int LBO_A>
__device__ __forceinline__ void issue_row(uint64_t adesc0, uint64_t bdesc0, const uint32_t (&pd)[3],
                                          const uint32_t (&pb)[3], const uint32_t (&pi)[3])
{
#pragma unroll
    for (int dx = 0; dx < 3; dx++) {
#pragma unroll
        for (int kk = 0; kk < KS; kk++) {
            const uint64_t ad = adesc0 + (uint64_t)((kk * 2 * LBO_A + dx * 16) >> 4);
            const uint64_t bd = bdesc0 + (uint64_t)(((dx * KC + 2 * kk) * 3 * NG * 128) >> 4);
#pragma unroll
            for (int p = 0; p < NP; p++) dev::mma_f16(pd[p], ad, bd + pb[p], pi[p], 1u, 0);
        }
    }
}

template <int KPAD, int NPAD>
__global__ void __launch_bounds__(kConvThreads, 1) k_conv3x3_tc(const __grid_constant__ ConvDev a)
{
    using C = ConvCfg<KPAD, NPAD>;
    constexpr int S = C::S;
    extern __shared__ unsigned char smraw[];
    // 1024-byte aligned base (bulk-copy destinations and descriptor bases)
    unsigned char *sm = smraw + ((1024 - (dev::smem_u32(smraw) & 1023)) & 1023);
    const uint32_t sbase = dev::smem_u32(sm);
    const uint32_t wbase = sbase, abase = sbase + C::AOFF;
    float *sbias = reinterpret_cast<float *>(sm + C::POFF), *sslope = sbias + 64;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + C::BOFF);
    const uint32_t full0 = dev::smem_u32(bars), empty0 = full0 + 8 * C::NS, accf0 = empty0 + 8 * C::NS,
                   acce0 = accf0 + 8 * S, wbar = acce0 + 8 * S, dbar = wbar + 8;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 2 * C::NS + 2 * S + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool bulk_in = a.in_mode == 0;
    const int H = a.H, W = a.W;

    // ---- set-up
    if (tid == 0) {
        for (int s = 0; s < C::NS; s++) {
            dev::mbar_init(full0 + 8 * s, bulk_in ? 1 : 128);
            dev::mbar_init(empty0 + 8 * s, 1);
        }
        for (int s = 0; s < S; s++) {
            dev::mbar_init(accf0 + 8 * s, 1);
            dev::mbar_init(acce0 + 8 * s, 4);
        }
        dev::mbar_init(wbar, 1);
        dev::mbar_init(dbar, 1);
        dev::fence_mbar_init();
    }
    if (warp == 8) dev::tmem_alloc(dev::smem_u32(tslot), kTmemCols);
    // K chunks the producer never writes (channel padding) are zero for the kernel's lifetime
    {
        const int written = bulk_in ? a.cin / 8 : 1;
        const int nz = (C::KC - written) * kHalo;
        for (int s = 0; s < C::NS; s++)
            for (int i = tid; i < nz; i += kConvThreads)
                reinterpret_cast<uint4 *>(sm + C::AOFF + s * C::SLOT + written * C::LBO_A)[i] = make_uint4(0, 0, 0, 0);
    }
    for (int n = tid; n < 64; n += kConvThreads) {
        sbias[n] = n < NPAD ? a.bias[n] : 0.f;
        sslope[n] = (n < NPAD && a.slope) ? a.slope[n] : 0.f;
    }
    dev::fence_proxy_async();
    dev::tc_fence_before();
    __syncthreads();
    dev::tc_fence_after();
    const uint32_t tmem = *tslot;

    if (warp < 4) {
        // ================= producer
        if (tid == 0) {
            dev::mbar_arrive_expect_tx(wbar, C::WBYTES);
            dev::bulk_load(wbase, a.wimg, C::WBYTES, wbar);
        }
        if (bulk_in) {
            if (tid == 0) {
                const int kcin = a.cin / 8;
                const uint32_t bytes = (uint32_t)kcin * kHalo * 16;
                const size_t chunk_row = (size_t)a.pitch * 8;  // halves per chunk row
                SegIter seg(W, a.row_begin, a.row_end);
                uint32_t it = 0;
                int strip, ya, yb;
                bool ok = true;
                while (ok && seg.next(strip, ya, yb)) {
                    const int x0 = strip * kTileM;
                    int r0, r1;
                    segment_rows(ya, yb, a.img_h, r0, r1);
                    for (int r = r0; r <= r1; r++, it++) {
                        const uint32_t s = it % C::NS, ph = (it / C::NS) & 1;
                        if (!(ok = dev::mbar_wait(empty0 + 8 * s, ph ^ 1, a.err, kErrProdEmpty))) break;
                        dev::mbar_arrive_expect_tx(full0 + 8 * s, bytes);
                        const uint32_t dst = abase + s * C::SLOT;
                        // padded column x0 is pixel x0 - 1: the left halo
                        const __half *row = a.src + (size_t)r * kcin * chunk_row + (size_t)x0 * 8;
                        for (int kc = 0; kc < kcin; kc++)
                            dev::bulk_load(dst + kc * C::LBO_A, row + kc * chunk_row, kHalo * 16, full0 + 8 * s);
                    }
                }
                // on an error exit, let the last copy land before the CTA can leave
                if (!ok && it > 0) {
                    const uint32_t s = (it - 1) % C::NS, ph = ((it - 1) / C::NS) & 1;
                    dev::mbar_wait(full0 + 8 * s, ph, nullptr, 0);
                }
            }
        } else {
            // NCHW RGB model input -> chunk 0 of the staged row: {r, g, b, 0, 0, 0, 0, 0} per pixel
            SegIter seg(W, a.row_begin, a.row_end);
            uint32_t it = 0;
            int strip, ya, yb;
            bool ok = true;
            const size_t plane = (size_t)H * W;
            while (ok && seg.next(strip, ya, yb)) {
                const int x0 = strip * kTileM;
                int r0, r1;
                segment_rows(ya, yb, a.img_h, r0, r1);
                for (int r = r0; r <= r1; r++, it++) {
                    const uint32_t s = it % C::NS, ph = (it / C::NS) & 1;
                    if (!(ok = dev::mbar_wait(empty0 + 8 * s, ph ^ 1, a.err, kErrProdEmpty))) break;
                    unsigned char *dst = sm + C::AOFF + s * C::SLOT;
                    for (int p = tid; p < kHalo; p += 128) {
                        const int x = x0 - 1 + p;
                        float v[3] = {0.f, 0.f, 0.f};
                        if (x >= 0 && x < W) {
                            const __half *px = a.src + (size_t)r * W + x;
#pragma unroll
                            for (int c = 0; c < 3; c++) {
                                v[c] = __half2float(px[c * plane]);
                                if (a.in_norm) v[c] = __half2float(__float2half_rn((v[c] - a.in_mean[c]) * a.in_scale[c]));
                            }
                        }
                        uint4 q;
                        q.x = pack_h2(v[0], v[1]);
                        q.y = pack_h2(v[2], 0.f);
                        q.z = 0u;
                        q.w = 0u;
                        reinterpret_cast<uint4 *>(dst)[p] = q;
                    }
                    dev::fence_proxy_async();
                    dev::mbar_arrive(full0 + 8 * s);
                }
            }
        }
    } else if (warp < 8) {
        // ================= epilogue
        const int q = warp & 3;
        const uint32_t lanes = (uint32_t)(q * 32) << 16;
        // every ring slot starts at zero; the MMA warp waits on named barrier 1 for this
        for (int c = 0; c < S * NPAD; c += 16) dev::tmem_zero16(tmem + lanes + c);
        dev::tmem_wait_st();
        dev::tc_fence_before();
        dev::named_bar_sync(1, 160);

        const int ccout = a.cout / 8;  // row-chunked outputs: 16-byte chunks per pixel
        SegIter seg(W, a.row_begin, a.row_end);
        uint32_t ot = 0;
        int strip, ya, yb;
        bool ok = true;
        while (ok && seg.next(strip, ya, yb)) {
            const int x0 = strip * kTileM;
            const int x = x0 + q * 32 + lane;
            for (int o = ya; o < yb; o++, ot++) {
                const int slot = ring_slot<S>(ot);
                if (!(ok = dev::mbar_wait(accf0 + 8 * slot, ring_phase<S>(ot), a.err, kErrEpiAccFull))) break;
                __syncwarp();
                dev::tc_fence_after();
                float v[NPAD];
                const uint32_t taddr = tmem + lanes + (uint32_t)(slot * NPAD);
#pragma unroll
                for (int c = 0; c < NPAD / 16; c++) {
                    float t[16];
                    dev::tmem_ld16(taddr + c * 16, t);
#pragma unroll
                    for (int j = 0; j < 16; j++) v[c * 16 + j] = t[j];
                }
                dev::tmem_wait_ld();
                // hand the slot back zeroed: the MMAs accumulate into it from scratch
#pragma unroll
                for (int c = 0; c < NPAD / 16; c++) dev::tmem_zero16(taddr + c * 16);
                dev::tmem_wait_st();
                dev::tc_fence_before();
                __syncwarp();
                if (lane == 0) dev::mbar_arrive(acce0 + 8 * slot);

#pragma unroll
                for (int n = 0; n < NPAD; n += 4) {
                    const float4 b4 = *reinterpret_cast<const float4 *>(sbias + n);
                    v[n] += b4.x;
                    v[n + 1] += b4.y;
                    v[n + 2] += b4.z;
                    v[n + 3] += b4.w;
                }
                if (a.R == 0) {
                    // row-chunked output (+ activation or gate)
                    if (a.act == 1) {
#pragma unroll
                        for (int n = 0; n < NPAD; n++) v[n] = fmaxf(v[n], 0.f);
                    } else if (a.act == 2) {
#pragma unroll
                        for (int n = 0; n < NPAD; n += 4) {
                            const float4 s4 = *reinterpret_cast<const float4 *>(sslope + n);
                            v[n] = v[n] >= 0.f ? v[n] : v[n] * s4.x;
                            v[n + 1] = v[n + 1] >= 0.f ? v[n + 1] : v[n + 1] * s4.y;
                            v[n + 2] = v[n + 2] >= 0.f ? v[n + 2] : v[n + 2] * s4.z;
                            v[n + 3] = v[n + 3] >= 0.f ? v[n + 3] : v[n + 3] * s4.w;
                        }
                    } else if (a.act == 3) {
#pragma unroll
                        for (int n = 0; n < NPAD; n++) v[n] = v[n] * fmaf(0.5f, dev::tanh_fast(0.5f * v[n]), 0.5f);
                    }
                    const size_t chunk_row = (size_t)a.pitch * 8;
                    if (a.gate != 0 && x < W) {
                        const __half *xr = a.resid + (size_t)o * ccout * chunk_row + (size_t)(x + 1) * 8;
#pragma unroll
                        for (int c = 0; c < NPAD / 8; c++) {
                            if (c < ccout) {
                                const uint4 rv = __ldg(reinterpret_cast<const uint4 *>(xr + c * chunk_row));
                                const __half2 *h = reinterpret_cast<const __half2 *>(&rv);
#pragma unroll
                                for (int j = 0; j < 4; j++) {
                                    const float2 f = __half22float2(h[j]);
                                    const int n0 = c * 8 + 2 * j;
                                    if (a.gate == 1) {
                                        v[n0] = f.x + v[n0];
                                        v[n0 + 1] = f.y + v[n0 + 1];
                                    } else if (a.gate == 3) {
                                        v[n0] = (f.x + v[n0]) * (0.5f * dev::tanh_fast(0.5f * v[n0]));
                                        v[n0 + 1] = (f.y + v[n0 + 1]) * (0.5f * dev::tanh_fast(0.5f * v[n0 + 1]));
                                    }
                                }
                            }
                        }
                    }
                    // one 16-byte chunk per lane per store: 32 consecutive pixels = 512 contiguous bytes
                    if (x < W) {
                        __half *drow = a.dst + (size_t)o * ccout * chunk_row + (size_t)(x + 1) * 8;
#pragma unroll
                        for (int c = 0; c < NPAD / 8; c++) {
                            if (c < ccout) {
                                uint4 w4;
                                w4.x = pack_h2(v[c * 8 + 0], v[c * 8 + 1]);
                                w4.y = pack_h2(v[c * 8 + 2], v[c * 8 + 3]);
                                w4.z = pack_h2(v[c * 8 + 4], v[c * 8 + 5]);
                                w4.w = pack_h2(v[c * 8 + 6], v[c * 8 + 7]);
                                *reinterpret_cast<uint4 *>(drow + c * chunk_row) = w4;
                            }
                        }
                    }
                } else if (x < W) {
                    switch (a.R) {
                    case 1: store_d2s<1>(v, a, o, x); break;
                    case 2: store_d2s<2>(v, a, o, x); break;
                    case 3: store_d2s<3>(v, a, o, x); break;
                    default: store_d2s<4>(v, a, o, x); break;
                    }
                }
            }
        }
    } else {
        // ================= MMA issuer (warp 8)
        dev::named_bar_sync(1, 160);
        dev::tc_fence_after();
        if (lane == 0) {
            bool ok = dev::mbar_wait(wbar, 0, a.err, kErrWeights);
            SegIter seg(W, a.row_begin, a.row_end);
            uint32_t it = 0, ot = 0;
            int strip, ya, yb;
            // descriptor templates: the start address is the low 14 bits (16-byte units), so a byte
            // offset d is added as d >> 4
            const uint64_t bdesc0 = dev::sdesc(wbase, C::LBO_B, 128);
            const uint64_t adesc_base = dev::sdesc(abase, C::LBO_A, 128);
            while (ok && seg.next(strip, ya, yb)) {
                int r0, r1;
                segment_rows(ya, yb, a.img_h, r0, r1);
                for (int r = r0; r <= r1; r++, it++) {
                    const uint32_t s = it % C::NS, ph = (it / C::NS) & 1;
                    if (!(ok = dev::mbar_wait(full0 + 8 * s, ph, a.err, kErrMmaFull))) break;
                    // the outputs this row feeds: r+1 (tap row 0), r (1), r-1 (2), those in [ya, yb)
                    // and in r's image, grouped into pieces: runs of adjacent ring slots, one MMA each
                    const int first = r / a.img_h * a.img_h, last = first + a.img_h - 1;
                    bool v[3];
                    int sl[3];
                    v[0] = r + 1 <= last && r + 1 >= ya && r + 1 < yb;
                    v[1] = r >= ya && r < yb;
                    v[2] = r - 1 >= first && r - 1 >= ya && r - 1 < yb;
#pragma unroll
                    for (int ty = 0; ty < 3; ty++) sl[ty] = ring_slot<S>(ot + (uint32_t)(r + 1 - ty - ya));
                    // an output's first input row must find its slot free: r+1 always starts at r, and
                    // r starts at r when r is its image's first row
                    if (v[0] && ok)
                        ok = dev::mbar_wait(acce0 + 8 * sl[0], ring_phase<S>(ot + (uint32_t)(r + 1 - ya)) ^ 1u, a.err,
                                            kErrMmaAccEmpty);
                    if (v[1] && r == first && ok)
                        ok = dev::mbar_wait(acce0 + 8 * sl[1], ring_phase<S>(ot + (uint32_t)(r - ya)) ^ 1u, a.err,
                                            kErrMmaAccEmpty);
                    if (!ok) break;
                    const bool c01 = v[0] && v[1] && sl[1] == sl[0] + 1, c12 = v[1] && v[2] && sl[2] == sl[1] + 1;
                    const bool st0 = v[0], st1 = v[1] && !c01, st2 = v[2] && !c12;
                    const int len0 = 1 + (c01 ? 1 : 0) + ((c01 && c12) ? 1 : 0), len1 = 1 + (c12 ? 1 : 0);
                    // the three candidate pieces (start slot, first tap row, length)
                    const uint32_t D0 = tmem + (uint32_t)(sl[0] * NPAD), D1 = tmem + (uint32_t)(sl[1] * NPAD),
                                   D2 = tmem + (uint32_t)(sl[2] * NPAD);
                    constexpr uint32_t B1 = (uint32_t)(1 * C::NG * 128) >> 4, B2 = (uint32_t)(2 * C::NG * 128) >> 4;
                    const uint32_t I0 = dev::idesc_f16_f32(kTileM, len0 * NPAD), I1 = dev::idesc_f16_f32(kTileM, len1 * NPAD),
                                   I2 = dev::idesc_f16_f32(kTileM, NPAD);
                    uint32_t pd[3] = {D0, D1, D2}, pb[3] = {0u, B1, B2}, pi[3] = {I0, I1, I2};
                    const int mask = (st0 ? 1 : 0) | (st1 ? 2 : 0) | (st2 ? 4 : 0);
                    int np = 3;
                    switch (mask) {
                    case 1: np = 1; break;
                    case 2: pd[0] = D1; pb[0] = B1; pi[0] = I1; np = 1; break;
                    case 3: np = 2; break;
                    case 4: pd[0] = D2; pb[0] = B2; pi[0] = I2; np = 1; break;
                    case 5: pd[1] = D2; pb[1] = B2; pi[1] = I2; np = 2; break;
                    case 6: pd[0] = D1; pb[0] = B1; pi[0] = I1; pd[1] = D2; pb[1] = B2; pi[1] = I2; np = 2; break;
                    default: break;
                    }
                    dev::tc_fence_after();
                    const uint64_t adesc0 = adesc_base + (uint64_t)((s * C::SLOT) >> 4);
                    if (np == 1)
                        issue_row<1, C::KS, C::KC, C::NG, C::LBO_A>(adesc0, bdesc0, pd, pb, pi);
                    else if (np == 2)
                        issue_row<2, C::KS, C::KC, C::NG, C::LBO_A>(adesc0, bdesc0, pd, pb, pi);
                    else
                        issue_row<3, C::KS, C::KC, C::NG, C::LBO_A>(adesc0, bdesc0, pd, pb, pi);
                    dev::mma_commit(empty0 + 8 * s);
                    // outputs complete at their last input row: o + 1, or o at the image's last row
                    if (v[2]) dev::mma_commit(accf0 + 8 * sl[2]);
                    if (v[1] && r == last) dev::mma_commit(accf0 + 8 * sl[1]);
                }
                ot += (uint32_t)(yb - ya);
            }
            // every MMA issued has completed before TMEM can be released
            dev::mma_commit(dbar);
            dev::mbar_wait(dbar, 0, a.err, kErrDrain);
        }
        __syncwarp();
    }

    dev::tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        dev::tc_fence_after();
        dev::tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace ajib
