/*
 * concat_tc.cuh — the 1x1 convolution over the concatenation of 2-4 feature maps (SPAN's
 * concat + conv), device code. The reference's k_concat1x1 (src/native/conv_kernels.cuh:351-407):
 * out = bias + sum over sources k and channels i of w[k * c + i][o] * src_k[i], no activation,
 * fp32 accumulation here, one rounding to fp16 at the store.
 *
 * GEMM with M = 128 consecutive pixels of one row, K = nsrc * c (the concatenation, padded to a
 * multiple of 16), N = c. The work is bound by HBM (for SPAN's 4 x 48 channels a 128-pixel tile
 * reads 48 KB and writes 12 KB for 2.4 MFLOP), so the design keeps many tiles in flight: each
 * source's (row, strip) block of the strip-chunked map (conv_tc.cuh) is one bulk copy, staged
 * K-major as [K/8][130][8] — the MMA's A layout, its descriptor starting past the halo column.
 * Persistent CTAs walk contiguous runs of (strip, row) tiles.
 * Roles: warp 0 producer (lane 0 arms the barriers, every lane issues copies), warp 1 MMA issuer
 * (one thread) and TMEM owner, warps 2-5
 * epilogue (TMEM lane quarter = warp % 4, one pixel per thread).
 */
#pragma once

#include <cuda_fp16.h>

#include "conv_tc.cuh"
#include "sm100.cuh"

namespace ajib {

constexpr int kCatThreads = 6 * 32;
constexpr int kCatMaxStages = 4;
constexpr int kCatSlots = 8;        // TMEM accumulator slots of 64 columns
constexpr int kCatChunkBytes = kStripW * 16;  // one 8-channel chunk of a strip, halo columns included

enum { kErrCatEmpty = 201, kErrCatFull = 202, kErrCatAccEmpty = 203, kErrCatAccFull = 204, kErrCatWeights = 205,
       kErrCatDrain = 206 };

struct CatDev {
    const __half *src[4];  // strip-chunked maps of c channels
    __half *dst;           // strip-chunked map of c channels
    const unsigned char *wimg;  // B image [kpad / 8][npad / 8][8 n][8 k]
    const float *bias;     // npad floats
    int *err;
    int nsrc, c, H, W, nstrips, kpad, row_begin, row_end;
    int ns;                // pipeline stages
};

// Shared-memory plan of k_concat1x1 for K padded to kpad and N padded to NPAD.
struct CatSmem {
    int b_bytes, stage, a_off, bias_off, bar_off, total;
    __host__ __device__ CatSmem(int kpad, int npad, int ns)
    {
        b_bytes = (kpad * npad * 2 + 1023) / 1024 * 1024;
        stage = (kpad / 8 * kCatChunkBytes + 127) / 128 * 128;
        a_off = b_bytes;
        bias_off = a_off + ns * stage;
        bar_off = bias_off + 64 * 4;
        total = bar_off + 512 + 1024;  // barriers + alignment slack
    }
};

template <int NPAD>
__global__ void __launch_bounds__(kCatThreads, 1) k_concat1x1(const __grid_constant__ CatDev a)
{
    static_assert(NPAD % 16 == 0 && NPAD >= 16 && NPAD <= 64, "N");
    extern __shared__ unsigned char smraw[];
    unsigned char *sm = smraw + ((1024 - (dev::smem_u32(smraw) & 1023)) & 1023);
    const CatSmem L(a.kpad, NPAD, a.ns);
    const uint32_t sbase = dev::smem_u32(sm), wbase = sbase, abase = sbase + L.a_off;
    float *sbias = reinterpret_cast<float *>(sm + L.bias_off);
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + L.bar_off);
    const uint32_t full0 = dev::smem_u32(bars), empty0 = full0 + 8 * kCatMaxStages, accf0 = empty0 + 8 * kCatMaxStages,
                   acce0 = accf0 + 8 * kCatSlots, wbar = acce0 + 8 * kCatSlots, dbar = wbar + 8;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 2 * kCatMaxStages + 2 * kCatSlots + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int NS = a.ns, KC = a.kpad / 8, cc = a.c / 8, kc_real = a.nsrc * cc;
    if (tid == 0) {
        for (int s = 0; s < kCatMaxStages; s++) {
            dev::mbar_init(full0 + 8 * s, 1);
            dev::mbar_init(empty0 + 8 * s, 1);
        }
        for (int s = 0; s < kCatSlots; s++) {
            dev::mbar_init(accf0 + 8 * s, 1);
            dev::mbar_init(acce0 + 8 * s, 4);
        }
        dev::mbar_init(wbar, 1);
        dev::mbar_init(dbar, 1);
        dev::fence_mbar_init();
        dev::mbar_arrive_expect_tx(wbar, (uint32_t)(a.kpad * NPAD * 2));
        dev::bulk_load(wbase, a.wimg, (uint32_t)(a.kpad * NPAD * 2), wbar);
    }
    if (warp == 1) dev::tmem_alloc(dev::smem_u32(tslot), 512);
    // K chunks past the concatenation (padding to a multiple of 16) stay zero
    for (int s = 0; s < NS; s++)
        for (int i = tid; i < (KC - kc_real) * kStripW; i += kCatThreads)
            reinterpret_cast<uint4 *>(sm + L.a_off + s * L.stage + kc_real * kCatChunkBytes)[i] = make_uint4(0, 0, 0, 0);
    for (int n = tid; n < 64; n += kCatThreads) sbias[n] = n < NPAD ? a.bias[n] : 0.f;
    dev::fence_proxy_async();
    dev::tc_fence_before();
    __syncthreads();
    dev::tc_fence_after();
    const uint32_t tmem = *tslot;
    // programmatic dependent launch: inputs are read only after the previous kernel completes
    dev::griddep_launch_dependents();
    dev::griddep_wait();

    const int H = a.H, W = a.W;
    (void)H;
    if (warp == 0) {
        // ================= producer: the whole warp walks the tiles (uniform control flow); lane 0
        // arms the stage's barrier, and the tile's (source, chunk) copies go out one per lane
        // (one thread issuing a tile's 24 copies was the kernel's bottleneck)
        SegIter seg(W, a.row_begin, a.row_end);
        uint32_t it = 0;
        int strip, ya, yb;
        bool ok = true;
        const int ncopy = a.nsrc;
        while (ok && seg.next(strip, ya, yb)) {
            for (int y = ya; y < yb; y++, it++) {
                const uint32_t s = it % NS, ph = (it / NS) & 1;
                if (!(ok = dev::mbar_wait_warp(empty0 + 8 * s, ph ^ 1, a.err, kErrCatEmpty))) break;
                if (lane == 0) dev::mbar_arrive_expect_tx(full0 + 8 * s, (uint32_t)(kc_real * kCatChunkBytes));
                __syncwarp();
                const uint32_t dst = abase + s * L.stage;
                // source k's (row, strip) block: its cc chunks, K chunks k * cc ..
                for (int k = lane; k < ncopy; k += 32)
                    dev::bulk_load(dst + k * cc * kCatChunkBytes, a.src[k] + map_at(y, strip, 0, 0, a.nstrips, cc),
                                   (uint32_t)(cc * kCatChunkBytes), full0 + 8 * s);
                __syncwarp();
            }
        }
        if (!ok && it > 0 && lane == 0) {
            const uint32_t s = (it - 1) % NS, ph = ((it - 1) / NS) & 1;
            dev::mbar_wait(full0 + 8 * s, ph, nullptr, 0);
        }
    } else if (warp == 1) {
        // ================= MMA issuer
        if (lane == 0) {
            bool ok = dev::mbar_wait(wbar, 0, a.err, kErrCatWeights);
            const uint64_t bdesc0 = dev::sdesc(wbase, (NPAD / 8) * 128, 128);
            // A starts at column 1 of each staged chunk (column 0 is the halo)
            const uint64_t adesc_base = dev::sdesc(abase + 16, kCatChunkBytes, 128);
            const uint32_t idesc = dev::idesc_f16_f32(kTileM, NPAD);
            SegIter seg(W, a.row_begin, a.row_end);
            uint32_t it = 0;
            int strip, ya, yb;
            while (ok && seg.next(strip, ya, yb)) {
                for (int y = ya; y < yb && ok; y++, it++) {
                    const uint32_t s = it % NS, slot = it % kCatSlots;
                    ok = dev::mbar_wait(full0 + 8 * s, (it / NS) & 1, a.err, kErrCatFull) &&
                         dev::mbar_wait(acce0 + 8 * slot, ((it / kCatSlots) & 1) ^ 1u, a.err, kErrCatAccEmpty);
                    if (!ok) break;
                    dev::tc_fence_after();
                    const uint64_t adesc = adesc_base + (uint64_t)((s * L.stage) >> 4);
                    for (int kk = 0; kk < KC / 2; kk++)
                        dev::mma_f16(tmem + slot * 64, adesc + (uint64_t)((kk * 2 * kCatChunkBytes) >> 4),
                                     bdesc0 + (uint64_t)((kk * 2 * (NPAD / 8) * 128) >> 4), idesc, kk > 0 ? 1u : 0u, 0);
                    dev::mma_commit(empty0 + 8 * s);
                    dev::mma_commit(accf0 + 8 * slot);
                }
            }
            dev::mma_commit(dbar);
            dev::mbar_wait(dbar, 0, a.err, kErrCatDrain);
        }
        __syncwarp();
    } else {
        // ================= epilogue: lane quarter warp % 4, one pixel per thread
        const int q = warp & 3;
        const uint32_t lanes = (uint32_t)(q * 32) << 16;
        SegIter seg(W, a.row_begin, a.row_end);
        uint32_t it = 0;
        int strip, ya, yb;
        bool ok = true;
        while (ok && seg.next(strip, ya, yb)) {
            const int x = strip * kTileM + q * 32 + lane;
            for (int y = ya; y < yb; y++, it++) {
                const uint32_t slot = it % kCatSlots;
                if (!(ok = dev::mbar_wait_warp(accf0 + 8 * slot, (it / kCatSlots) & 1, a.err, kErrCatAccFull))) break;
                __syncwarp();
                dev::tc_fence_after();
                float v[NPAD];
#pragma unroll
                for (int c0 = 0; c0 < NPAD; c0 += 16) {
                    float t[16];
                    dev::tmem_ld16(tmem + lanes + slot * 64 + c0, t);
#pragma unroll
                    for (int j = 0; j < 16; j++) v[c0 + j] = t[j];
                }
                dev::tmem_wait_ld();
                dev::tc_fence_before();
                __syncwarp();
                if (lane == 0) dev::mbar_arrive(acce0 + 8 * slot);
                if (x < W) {
#pragma unroll
                    for (int j = 0; j < NPAD / 8; j++) {
                        if (j < cc) {
                            uint4 w4;
                            w4.x = pack_h2(v[j * 8 + 0] + sbias[j * 8 + 0], v[j * 8 + 1] + sbias[j * 8 + 1]);
                            w4.y = pack_h2(v[j * 8 + 2] + sbias[j * 8 + 2], v[j * 8 + 3] + sbias[j * 8 + 3]);
                            w4.z = pack_h2(v[j * 8 + 4] + sbias[j * 8 + 4], v[j * 8 + 5] + sbias[j * 8 + 5]);
                            w4.w = pack_h2(v[j * 8 + 6] + sbias[j * 8 + 6], v[j * 8 + 7] + sbias[j * 8 + 7]);
                            store_px(a.dst, y, x, j, a.nstrips, cc, w4);
                        }
                    }
                }
            }
        }
    }

    dev::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        dev::tc_fence_after();
        dev::tmem_dealloc(tmem, 512);
    }
}

}  // namespace ajib
