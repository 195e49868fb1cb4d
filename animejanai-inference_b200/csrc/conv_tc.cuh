/*
 * conv_tc.cuh — the fused 3x3 convolution on Blackwell tensor cores (sm_100a), device code.
 *
 * Implicit GEMM with the output pixels as M: a tile is 128 consecutive pixels of one output row,
 * N is cout (padded to a multiple of 16), K is 9 taps x cin (padded to a multiple of 16). One
 * staged input row (130 pixels: the tile plus a one-pixel halo on each side) feeds every tap of
 * the three output rows it touches: for tap (ty, tx) the A operand is the staged row starting
 * tx pixels in, which is just a 16-byte-unit shift of the shared-memory descriptor's start
 * address, because the row is staged K-major without swizzle as [cin/8][130][8 fp16].
 *
 * A CTA is persistent on one SM and walks a contiguous run of (strip, row) tiles down a
 * 128-pixel-wide vertical strip, so each input row is fetched once and used by up to three
 * output rows (A is kept in the tensor core's collector buffer across those MMAs). Roles:
 *   warps 0-3  producer: one thread issues the TMA load of each input row (NHWC inputs), or all
 *              128 threads convert the NCHW RGB model input into the same layout;
 *   warps 4-7  epilogue: TMEM -> registers (one pixel per thread), bias, activation, SPAN gate or
 *              depth-to-space with the model-input skip, fp16 store;
 *   warp 8     MMA issuer (one thread) and TMEM owner.
 * Weights for all 9 taps stay resident in shared memory for the CTA's lifetime. Accumulators are
 * fp32 in TMEM: four 128 x NPAD slots, so three output rows accumulate while the epilogue drains
 * the fourth.
 *
 * The semantics are those of the reference kernel k_conv3x3 (src/native/conv_kernels.cuh:100-350)
 * with fp32 accumulation and an fp32 epilogue instead of fp16 ones (one rounding to fp16 at the
 * store).
 */
#pragma once

#include <cuda_fp16.h>

#include "sm100.cuh"

namespace ajib {

constexpr int kTileM = 128;            // output pixels per tile (the MMA's M)
constexpr int kHalo = kTileM + 2;      // staged input pixels per row
constexpr int kAccSlots = 4;           // TMEM accumulators
constexpr int kAccStride = 64;         // TMEM columns per accumulator slot
constexpr int kConvThreads = 288;      // 9 warps
constexpr int kMaxSmem = 227 * 1024;

// error codes written to the status word (which wait timed out)
enum { kErrProdEmpty = 101, kErrMmaFull = 102, kErrMmaAccEmpty = 103, kErrEpiAccFull = 104, kErrWeights = 105,
       kErrDrain = 106 };

struct ConvDev {
    const __half *src;    // NHWC [H][W][cin] or NCHW [3][H][W]
    const __half *resid;  // gate: NHWC [H][W][cout]; depth-to-space: NCHW model input [3][H][W] or null
    __half *dst;          // NHWC [H][W][cout] or NCHW [3][R*H][R*W]
    const unsigned char *wimg;  // packed B operand image, all taps
    const float *bias;    // NPAD floats
    const float *slope;   // NPAD floats or null
    int *err;             // status word
    int H, W, cin, cout;
    int in_mode, act, gate, R;  // R = 0: NHWC output, else depth-to-space factor
    int in_norm, out_clamp;
    float in_mean[3], in_scale[3];
    int row_begin, row_end;
    int tma_split;        // 1: a 3-D tensor map, one TMA copy per 8-channel chunk
};

template <int KPAD, int NPAD>
struct ConvCfg {
    static_assert(KPAD % 16 == 0 && NPAD % 16 == 0 && KPAD <= 64 && NPAD <= 64, "padded channel counts");
    static constexpr int KC = KPAD / 8;     // 8-channel chunks per pixel
    static constexpr int KS = KPAD / 16;    // MMA K steps per tap
    static constexpr int NG = NPAD / 8;     // 8-row core-matrix groups of B
    static constexpr int LBO_A = kHalo * 16;  // bytes between K chunks of a staged row
    static constexpr int SLOT = (KC * LBO_A + 1023) / 1024 * 1024;
    static constexpr int WBYTES = 9 * KPAD * NPAD * 2;
    static constexpr int AOFF = (WBYTES + 1023) / 1024 * 1024;
    static constexpr int CC = NPAD / 8;                   // 16-byte chunks per output pixel (max)
    static constexpr int SC = (CC % 2) ? CC : CC + 1;      // staging row stride in chunks (odd: no bank conflicts)
    static constexpr int EPI_WARP = 32 * SC * 16;
    static constexpr int FIXED = AOFF + 4 * EPI_WARP + 2 * 64 * 4 + 512 + 1024;
    static constexpr int NS_FIT = (kMaxSmem - FIXED) / SLOT;
    static constexpr int NS = NS_FIT > 6 ? 6 : NS_FIT;
    static_assert(NS >= 2, "at least double-buffered input rows");
    static constexpr int EOFF = AOFF + NS * SLOT;
    static constexpr int POFF = EOFF + 4 * EPI_WARP;   // bias[64], slope[64] floats
    static constexpr int BOFF = POFF + 2 * 64 * 4;     // mbarriers
    static constexpr int SMEM = BOFF + 512 + 1024;     // + alignment slack for the base
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

template <int KPAD, int NPAD>
__global__ void __launch_bounds__(kConvThreads, 1)
    k_conv3x3_tc(const __grid_constant__ CUtensorMap tin, const __grid_constant__ ConvDev a)
{
    using C = ConvCfg<KPAD, NPAD>;
    extern __shared__ unsigned char smraw[];
    // 1024-byte aligned base (TMA destinations and descriptor bases)
    unsigned char *sm = smraw + ((1024 - (dev::smem_u32(smraw) & 1023)) & 1023);
    const uint32_t sbase = dev::smem_u32(sm);
    const uint32_t wbase = sbase, abase = sbase + C::AOFF;
    float *sbias = reinterpret_cast<float *>(sm + C::POFF), *sslope = sbias + 64;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + C::BOFF);
    // barrier indices
    const uint32_t full0 = dev::smem_u32(bars), empty0 = full0 + 8 * C::NS, accf0 = empty0 + 8 * C::NS,
                   acce0 = accf0 + 8 * kAccSlots, wbar = acce0 + 8 * kAccSlots, dbar = wbar + 8;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 2 * C::NS + 2 * kAccSlots + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool tma_in = a.in_mode == 0;
    const int H = a.H, W = a.W;

    // ---- set-up
    if (tid == 0) {
        for (int s = 0; s < C::NS; s++) {
            dev::mbar_init(full0 + 8 * s, tma_in ? 1 : 128);
            dev::mbar_init(empty0 + 8 * s, 1);
        }
        for (int s = 0; s < kAccSlots; s++) {
            dev::mbar_init(accf0 + 8 * s, 1);
            dev::mbar_init(acce0 + 8 * s, 4);
        }
        dev::mbar_init(wbar, 1);
        dev::mbar_init(dbar, 1);
        dev::fence_mbar_init();
    }
    if (warp == 8) dev::tmem_alloc(dev::smem_u32(tslot), kAccSlots * kAccStride);
    // K chunks the producer never writes (channel padding) are zero for the kernel's lifetime
    {
        const int written = tma_in ? a.cin / 8 : 1;
        const int nz = (C::KC - written) * (kHalo * 16 / 16);
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
        if (tma_in) {
            if (tid == 0) {
                dev::tma_prefetch_desc(&tin);
                dev::mbar_arrive_expect_tx(wbar, C::WBYTES);
                dev::bulk_load(wbase, a.wimg, C::WBYTES, wbar);
                const uint32_t bytes = (uint32_t)(a.cin / 8) * kHalo * 16;
                SegIter seg(W, a.row_begin, a.row_end);
                uint32_t it = 0;
                int strip, ya, yb;
                bool ok = true;
                while (ok && seg.next(strip, ya, yb)) {
                    const int x0 = strip * kTileM, r0 = max(ya - 1, 0), r1 = min(yb, H - 1);
                    for (int r = r0; r <= r1; r++, it++) {
                        const uint32_t s = it % C::NS, ph = (it / C::NS) & 1;
                        if (!(ok = dev::mbar_wait(empty0 + 8 * s, ph ^ 1, a.err, kErrProdEmpty))) break;
                        dev::mbar_arrive_expect_tx(full0 + 8 * s, bytes);
                        const uint32_t dst = abase + s * C::SLOT;
                        if (!a.tma_split) {
                            dev::tma_load_4d(dst, &tin, full0 + 8 * s, 0, x0 - 1, 0, r);
                        } else {
                            for (int kc = 0; kc < a.cin / 8; kc++)
                                dev::tma_load_3d(dst + kc * C::LBO_A, &tin, full0 + 8 * s, kc * 8, x0 - 1, r);
                        }
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
            if (tid == 0) {
                dev::mbar_arrive_expect_tx(wbar, C::WBYTES);
                dev::bulk_load(wbase, a.wimg, C::WBYTES, wbar);
            }
            SegIter seg(W, a.row_begin, a.row_end);
            uint32_t it = 0;
            int strip, ya, yb;
            bool ok = true;
            const size_t plane = (size_t)H * W;
            while (ok && seg.next(strip, ya, yb)) {
                const int x0 = strip * kTileM, r0 = max(ya - 1, 0), r1 = min(yb, H - 1);
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
        unsigned char *stage = sm + C::EOFF + q * C::EPI_WARP;
        const int ccout = a.cout / 8;  // NHWC outputs: 16-byte chunks per pixel
        SegIter seg(W, a.row_begin, a.row_end);
        uint32_t ot = 0;
        int strip, ya, yb;
        bool ok = true;
        while (ok && seg.next(strip, ya, yb)) {
            const int x0 = strip * kTileM;
            const int x = x0 + q * 32 + lane;
            for (int o = ya; o < yb; o++, ot++) {
                const uint32_t slot = ot % kAccSlots, ph = (ot / kAccSlots) & 1;
                if (!(ok = dev::mbar_wait(accf0 + 8 * slot, ph, a.err, kErrEpiAccFull))) break;
                dev::tc_fence_after();
                float v[NPAD];
                const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + slot * kAccStride;
#pragma unroll
                for (int c = 0; c < NPAD / 16; c++) {
                    float t[16];
                    dev::tmem_ld16(taddr + c * 16, t);
#pragma unroll
                    for (int j = 0; j < 16; j++) v[c * 16 + j] = t[j];
                }
                dev::tmem_wait_ld();
                dev::tc_fence_before();
                __syncwarp();
                if (lane == 0) dev::mbar_arrive(acce0 + 8 * slot);

#pragma unroll
                for (int n = 0; n < NPAD; n++) v[n] += sbias[n];
                if (a.R == 0) {
                    // NHWC output (+ activation or gate)
                    if (a.act == 1) {
#pragma unroll
                        for (int n = 0; n < NPAD; n++) v[n] = fmaxf(v[n], 0.f);
                    } else if (a.act == 2) {
#pragma unroll
                        for (int n = 0; n < NPAD; n++) v[n] = v[n] >= 0.f ? v[n] : v[n] * sslope[n];
                    } else if (a.act == 3) {
#pragma unroll
                        for (int n = 0; n < NPAD; n++) v[n] = v[n] * fmaf(0.5f, dev::tanh_fast(0.5f * v[n]), 0.5f);
                    }
                    if (a.gate != 0 && x < W) {
                        const uint4 *xr = reinterpret_cast<const uint4 *>(a.resid + ((size_t)o * W + x) * a.cout);
#pragma unroll
                        for (int c = 0; c < NPAD / 8; c++) {
                            if (c < ccout) {
                                const uint4 rv = __ldg(xr + c);
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
                    // stage [32 px][SC chunks] then copy out coalesced
                    uint4 *st = reinterpret_cast<uint4 *>(stage);
#pragma unroll
                    for (int c = 0; c < NPAD / 8; c++) {
                        if (c < ccout) {
                            uint4 w4;
                            w4.x = pack_h2(v[c * 8 + 0], v[c * 8 + 1]);
                            w4.y = pack_h2(v[c * 8 + 2], v[c * 8 + 3]);
                            w4.z = pack_h2(v[c * 8 + 4], v[c * 8 + 5]);
                            w4.w = pack_h2(v[c * 8 + 6], v[c * 8 + 7]);
                            st[lane * C::SC + c] = w4;
                        }
                    }
                    __syncwarp();
                    const int xw = x0 + q * 32;
                    uint4 *drow = reinterpret_cast<uint4 *>(a.dst + ((size_t)o * W + xw) * a.cout);
                    for (int i = lane; i < 32 * ccout; i += 32) {
                        const int p = i / ccout, c = i - p * ccout;
                        if (xw + p < W) drow[i] = st[p * C::SC + c];
                    }
                    __syncwarp();
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
        if (lane == 0) {
            constexpr uint32_t idesc = dev::idesc_f16_f32(kTileM, NPAD);
            bool ok = dev::mbar_wait(wbar, 0, a.err, kErrWeights);
            SegIter seg(W, a.row_begin, a.row_end);
            uint32_t it = 0, ot = 0;
            int strip, ya, yb;
            while (ok && seg.next(strip, ya, yb)) {
                const int r0 = max(ya - 1, 0), r1 = min(yb, H - 1);
                for (int r = r0; r <= r1 && ok; r++, it++) {
                    const uint32_t s = it % C::NS, ph = (it / C::NS) & 1;
                    if (!(ok = dev::mbar_wait(full0 + 8 * s, ph, a.err, kErrMmaFull))) break;
                    const int olo = max(r - 1, ya), ohi = min(r + 1, yb - 1);
                    // output rows whose first input row is r take a fresh accumulator
                    for (int o = olo; o <= ohi && ok; o++) {
                        if (max(o - 1, 0) == r) {
                            const uint32_t j = ot + (uint32_t)(o - ya);
                            ok = dev::mbar_wait(acce0 + 8 * (j % kAccSlots), ((j / kAccSlots) & 1) ^ 1, a.err,
                                                kErrMmaAccEmpty);
                        }
                    }
                    if (!ok) break;
                    dev::tc_fence_after();
                    const uint32_t arow = abase + s * C::SLOT;
                    const int n = ohi - olo + 1;
#pragma unroll 1
                    for (int dx = 0; dx < 3; dx++) {
#pragma unroll
                        for (int kk = 0; kk < C::KS; kk++) {
                            const uint64_t ad = dev::sdesc(arow + kk * 2 * C::LBO_A + dx * 16, C::LBO_A, 128);
                            for (int i = 0; i < n; i++) {
                                const int o = ohi - i, ty = r - o + 1, tap = ty * 3 + dx;
                                const uint64_t bd =
                                    dev::sdesc(wbase + (uint32_t)((tap * C::KC + 2 * kk) * C::NG) * 128, C::NG * 128, 128);
                                const uint32_t j = ot + (uint32_t)(o - ya);
                                const uint32_t d = tmem + (j % kAccSlots) * kAccStride;
                                const bool first = (r == max(o - 1, 0)) && dx == 0 && kk == 0;
                                const int cm = n == 1 ? 0 : (i == 0 ? 1 : (i == n - 1 ? 3 : 2));
                                dev::mma_f16(d, ad, bd, idesc, first ? 0u : 1u, cm);
                            }
                        }
                    }
                    dev::mma_commit(empty0 + 8 * s);
                    if (r - 1 >= ya && r - 1 < yb) dev::mma_commit(accf0 + 8 * ((ot + (uint32_t)(r - 1 - ya)) % kAccSlots));
                    if (r == H - 1 && r >= ya && r < yb) dev::mma_commit(accf0 + 8 * ((ot + (uint32_t)(r - ya)) % kAccSlots));
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
        dev::tmem_dealloc(tmem, kAccSlots * kAccStride);
    }
}

}  // namespace ajib
