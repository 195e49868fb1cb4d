/*
 * conv_pair.cuh — the fused 3x3 convolution on a pair of SMs (sm_100a), device code: one tcgen05
 * MMA of M = 256 (cta_group::2) covers a 128-pixel tile on each SM of a cluster of two CTAs.
 *
 * Why: the one-SM kernel (conv_tc.cuh) is bound by its SM's shared-memory path. Per staged row its
 * MMAs read the row (A, once per horizontal tap: 48 KB at 64 channels) and the stacked-tap weights
 * (B, 72 KB) from shared memory, near the path's 128 bytes a cycle at the tensor core's rate, and
 * the row's bulk copy and the epilogue's stores share that path. In a pair MMA each SM holds and
 * reads half of B (36 KB a row), and one issuing thread drives both SMs.
 *
 * Status: correct (the same parity tests as the one-SM kernel) but slower on B200 as built, so it
 * is off by default (ajib_conv_pair_mode). Measured on one B200, the 64-channel body conv at
 * 1080p: 0.138-0.147 ms against the one-SM kernel's 0.129-0.134 ms. With its MMAs left out the
 * rest of its pipeline (row copies, epilogue, stores) alone takes 0.104 ms, ~5.1 TB/s of HBM
 * traffic, and the six-slot ring (two of the eight 64-column TMEM slots are spares) leaves the
 * MMAs two rows of slack against that epilogue, so tensor and memory work do not overlap enough.
 *
 * The layout and the tap stacking are the one-SM kernel's: the staged row [cin/8][130][8] in
 * shared memory, dx a 16-byte shift of A's descriptor, one MMA per (dx, K step) whose N = 3 x NPAD
 * columns are the accumulators of the three output rows the input row feeds. B splits by N between
 * the two CTAs (rows [0, N/2) in the even CTA, [N/2, N) in the odd one, at the same shared-memory
 * offset), so every MMA must have the same N layout, which rules out the one-SM kernel's pieces (a
 * row's MMA split where its three accumulators wrap around the ring or where a segment starts or
 * ends, each piece another N range, each needing its own halves of B). Here every staged row issues
 * the whole window:
 *   - per segment (one strip, output rows [ya, yb) inside one image) the staged rows are
 *     ya - 1 .. yb, a row outside the image being a zero row. Staged row k (counted over the CTA's
 *     whole walk) feeds accumulators ("counters") k + 2, k + 1 and k with tap rows 0, 1 and 2, so
 *     counter c holds the output row of staged row c - 1 and is complete after staged row c. The
 *     counters that straddle a segment boundary, and those of the rows that pad the shorter run of
 *     a pair, hold no output: the epilogue hands them back unread;
 *   - the ring has S = 512 / NPAD - 2 slots in descending order (counter c in slot S - 1 - c mod S)
 *     and two spare slots after it. A window that would wrap writes its last one or two
 *     accumulators into the spares instead: counter c in slot 0 gets its second and third rows'
 *     terms in spare S, in slot 1 its third row's in spare S + 1, and the epilogue adds the spare
 *     and zeroes it.
 * The two CTAs of a pair walk their own runs of (strip, row) tiles in lockstep: staged row k of
 * both is one MMA group (the same stage buffer and TMEM columns in both).
 *
 * Roles (PairCfg::THREADS threads; an epilogue warp's index mod 4 must be its TMEM lane quarter):
 *   warp 0      copier (both CTAs): one bulk copy per staged row into its stage as soon as the
 *               stage's buffer is free, zero rows by stores;
 *   warp 2      even CTA: waits until the accumulator each row of a stage starts is free (both
 *               CTAs' epilogues free it), then arrives on the stage's barrier too;
 *   warps 4..   epilogue (both CTAs), four warps per 16 accumulator columns (16 warps at 64
 *               channels): its own TMEM lanes (its 128 pixels): tcgen05.ld (plus the spare), the
 *               bias back into the slot, activation or SPAN gate, fp16 stores; the odd CTA's warps
 *               free the slot on the even CTA's barrier;
 *   last warp   even CTA: the MMA issuer (one thread); odd CTA: relays "this CTA's rows have
 *               landed" to the even CTA's stage barriers (a bulk copy completes only on a barrier
 *               of the CTA it writes).
 * Every wait is bounded as in the one-SM kernel; both CTAs meet at a cluster barrier before the
 * TMEM is released, so neither leaves while the other's MMAs may still read its shared memory.
 */
#pragma once

#include "conv_tc.cuh"

namespace ajib {

constexpr int kPairCols = 32;  // accumulator columns an epilogue warp takes (at most)

template <int KPAD, int NPAD>
struct PairCfg {
    static_assert(KPAD % 16 == 0 && KPAD <= 64 && (NPAD == 32 || NPAD == 48 || NPAD == 64), "padded channel counts");
    static constexpr int KC = KPAD / 8;               // 8-channel chunks per pixel
    static constexpr int KS = KPAD / 16;              // MMA K steps per tap column
    static constexpr int NG = NPAD / 8;
    static constexpr int N = 3 * NPAD;                // the MMA's N: three stacked tap rows
    static constexpr int HG = 3 * NG / 2;             // 8-row groups of B in each CTA
    static constexpr int S = kTmemCols / NPAD - 2;    // ring slots; spare slots S and S + 1 follow
    static constexpr int LBO_A = kHalo * 16;          // bytes between K chunks of a staged row
    static constexpr int LBO_B = HG * 128;            // bytes between K chunks of this CTA's half of B
    static constexpr int SLOT = (KC * LBO_A + 1023) / 1024 * 1024;
    static constexpr int WBYTES = 3 * KC * LBO_B;     // this CTA's half of B, all tap columns
    static constexpr int AOFF = (WBYTES + 1023) / 1024 * 1024;
    static constexpr int RP = 2;                      // staged rows per pipeline stage
    static constexpr int STAGE = RP * SLOT;
    static constexpr int FIXED = AOFF + 2 * 64 * 4 + 1024 + 1024;
    static constexpr int NS_FIT = (kMaxSmem - FIXED) / STAGE;
    static constexpr int NS = NS_FIT > 6 ? 6 : NS_FIT;
    static_assert(NS >= 3 && S >= 4, "pipeline depth");
    // the accumulator waiter arrives on a stage's barrier at most (S - 3) / 2 stages after the
    // stage it waits for was consumed: never a phase ahead
    static_assert(2 * NS >= S - 3, "stage barrier phases");
    static constexpr int POFF = AOFF + NS * STAGE;    // bias[64], slope - 1 [64] floats
    // mbarriers: full[NS], empty[NS], accf[S], acce[S], wbar, dbar; then the TMEM base address
    static constexpr int BOFF = POFF + 2 * 64 * 4;
    static constexpr int SMEM = BOFF + 1024 + 1024;   // + alignment slack for the base
    static_assert((2 * NS + 2 * S + 2) * 8 + 8 <= 1024, "barrier area");
    static_assert(SMEM <= kMaxSmem, "shared memory budget");
    // warps: 0-3 copier / accumulator waiter / idle; then four epilogue warps (one per TMEM lane
    // quarter) per 16 accumulator columns; one idle warp; the MMA warp (index % 4 == 1: its own SM
    // sub-partition, away from the copier)
    static constexpr int EPI0 = 4;
    // accumulator columns per epilogue warp: NPAD split into the fewest groups of at most kPairCols
    static constexpr int CWP = NPAD / ((NPAD + kPairCols - 1) / kPairCols);
    static_assert(NPAD % CWP == 0 && CWP % 8 == 0, "epilogue column split");
    static constexpr int EPW = 4 * (NPAD / CWP);
    static constexpr int MMA = EPI0 + EPW + 1;
    static constexpr int THREADS = (MMA + 1) * 32;
    static_assert(MMA % 4 == 1, "MMA warp sub-partition");
};

// The rows a CTA stages, in order: per segment of its run (one strip, output rows [ya, yb), cut at
// image boundaries) the input rows ya - 1 .. yb.
struct PairWalk {
    SegIter seg;
    int img_h;
    int strip = 0, yb_seg = 0;  // the strip segment being cut at image boundaries, and its end
    int sa = 0, sb = 0, f = 0;  // the current piece [sa, sb) and the first row of its image
    int r = 1, rend = 0;        // the next staged row, and the piece's last (sb)
    __device__ PairWalk(int W, int row_begin, int row_end, int img_h_, int cta, int ncta)
        : seg(W, row_begin, row_end, cta, ncta), img_h(img_h_)
    {
    }
    // The next staged row: its strip and input row, whether that row lies in its image (else it is
    // a zero row) and whether its output row is one of the run's. False past the run's last row.
    __device__ bool next(int &s, int &row, bool &in_img, bool &out)
    {
        if (r > rend) {
            if (sb >= yb_seg) {
                int a_, b_;
                if (!seg.next(strip, a_, b_)) return false;
                sb = a_;
                yb_seg = b_;
            }
            sa = sb;
            f = sa / img_h * img_h;
            sb = min(yb_seg, f + img_h);
            r = sa - 1;
            rend = sb;
        }
        s = strip;
        row = r;
        in_img = r >= f && r < f + img_h;
        out = r >= sa && r < sb;
        r++;
        return true;
    }
};

// How many rows PairWalk yields for CTA `cta` of `ncta`.
__device__ __forceinline__ int pair_walk_rows(int W, int row_begin, int row_end, int img_h, int cta, int ncta)
{
    SegIter seg(W, row_begin, row_end, cta, ncta);
    int n = 0, s, ya, yb;
    while (seg.next(s, ya, yb))
        for (int y = ya; y < yb;) {
            const int e = min(yb, y / img_h * img_h + img_h);
            n += e - y + 2;
            y = e;
        }
    return n;
}

// f(integral_constant<CW g>) for the runtime group g in [0, G): the compile-time column offset of
// an epilogue warp's CW columns.
template <int G, int CW, typename F>
__device__ __forceinline__ void for_group(int g, F &&f)
{
    if constexpr (G > 0) {
        if (g == G - 1)
            f(std::integral_constant<int, CW * (G - 1)>{});
        else
            for_group<G - 1, CW>(g, f);
    }
}

// One output's columns [C0, C0 + CW) (v holds the sums, bias included) through the activation or
// the SPAN gate into fp16 pairs: the arithmetic of epi_store, kept apart from the stores so that
// they can issue later.
template <int EK, int CW, int C0>
__device__ __forceinline__ void pair_finish(float (&v)[CW], uint32_t (&w)[CW / 2], const ConvDev &a, const float *sslope_m1,
                                            const EpiIn<CW> &in)
{
    if constexpr (EK == kEpiAct) {
        if (a.act == 1) {
#pragma unroll
            for (int j = 0; j < CW / 2; j++) w[j] = dev::pack_relu_h2(v[2 * j], v[2 * j + 1]);
            return;
        }
        if (a.act == 2) {
#pragma unroll
            for (int n = 0; n < CW; n += 4) {
                const float4 s4 = *reinterpret_cast<const float4 *>(sslope_m1 + C0 + n);
                v[n] = fmaf(fminf(v[n], 0.f), s4.x, v[n]);
                v[n + 1] = fmaf(fminf(v[n + 1], 0.f), s4.y, v[n + 1]);
                v[n + 2] = fmaf(fminf(v[n + 2], 0.f), s4.z, v[n + 2]);
                v[n + 3] = fmaf(fminf(v[n + 3], 0.f), s4.w, v[n + 3]);
            }
        } else if (a.act == 3) {
#pragma unroll
            for (int n = 0; n < CW; n++) v[n] = v[n] * fmaf(0.5f, dev::tanh_fast(0.5f * v[n]), 0.5f);
        }
    } else {
        const int ccout = a.cout / 8;
#pragma unroll
        for (int c = 0; c < CW / 8; c++) {
            if (C0 / 8 + c >= ccout) continue;
            const __half2 *h = reinterpret_cast<const __half2 *>(&in.gate[c]);
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
#pragma unroll
    for (int j = 0; j < CW / 2; j++) w[j] = pack_h2(v[2 * j], v[2 * j + 1]);
}

// The stores of pair_finish's fp16 pairs for pixel x of output row o: one 16-byte chunk per lane
// per store, 32 consecutive pixels = 512 contiguous bytes.
template <int CW, int C0>
__device__ __forceinline__ void pair_store(const uint32_t (&w)[CW / 2], const ConvDev &a, int o, int x)
{
    if (x >= a.W) return;
    const int ccout = a.cout / 8;
#pragma unroll
    for (int c = 0; c < CW / 8; c++)
        if (C0 / 8 + c < ccout)
            store_px(a.dst, o, x, C0 / 8 + c, a.nstrips, ccout, make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]));
}

template <int KPAD, int NPAD, int EK>
__global__ void __launch_bounds__(PairCfg<KPAD, NPAD>::THREADS, 1) k_conv3x3_pair(const __grid_constant__ ConvDev a)
{
    static_assert(EK == kEpiAct || EK == kEpiGate, "epilogues of the pair kernel");
    using C = PairCfg<KPAD, NPAD>;
    constexpr int S = C::S;
    extern __shared__ unsigned char smraw[];
    // 1024-byte aligned base; the same offsets in both CTAs (the pair's MMAs address both with one
    // descriptor)
    unsigned char *sm = smraw + ((1024 - (dev::smem_u32(smraw) & 1023)) & 1023);
    const uint32_t sbase = dev::smem_u32(sm);
    const uint32_t wbase = sbase, abase = sbase + C::AOFF;
    float *sbias = reinterpret_cast<float *>(sm + C::POFF), *sslope = sbias + 64;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + C::BOFF);
    const uint32_t full0 = dev::smem_u32(bars), empty0 = full0 + 8 * C::NS, accf0 = empty0 + 8 * C::NS,
                   acce0 = accf0 + 8 * S, wbar = acce0 + 8 * S, dbar = wbar + 8;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 2 * C::NS + 2 * S + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = dev::cluster_rank();
    const bool lead = rank == 0;
    const int W = a.W, cta = blockIdx.x, ncta = gridDim.x;
    // the pair walks as many rows as the longer of its two runs
    const int K = max(pair_walk_rows(W, a.row_begin, a.row_end, a.img_h, cta, ncta),
                      pair_walk_rows(W, a.row_begin, a.row_end, a.img_h, cta ^ 1, ncta));
    const uint32_t nst = (uint32_t)((K + C::RP - 1) / C::RP);

    // ---- set-up
    if (tid == 0) {
        for (int s = 0; s < C::NS; s++) {
            // even CTA: its copier, its accumulator waiter and the odd CTA's relay
            dev::mbar_init(full0 + 8 * s, lead ? 3 : 1);
            dev::mbar_init(empty0 + 8 * s, 1);
        }
        for (int s = 0; s < S; s++) {
            dev::mbar_init(accf0 + 8 * s, 1);
            // each CTA's epilogue frees a slot with one arrival (on the even CTA's barrier)
            dev::mbar_init(acce0 + 8 * s, 2);
        }
        dev::mbar_init(wbar, lead ? 2 : 1);
        dev::mbar_init(dbar, 1);
        dev::fence_mbar_init();
        // this CTA's half of B: per (tap column, K chunk) the N rows [rank, rank + 1) x 3 NPAD / 2
        // of the stacked image [dx][kc][3 NPAD rows][8]
        dev::mbar_arrive_expect_tx(wbar, C::WBYTES);
        for (int j = 0; j < 3 * C::KC; j++)
            dev::bulk_load(wbase + j * C::LBO_B, a.wimg + ((size_t)j * 2 + rank) * C::LBO_B, C::LBO_B, wbar);
    }
    if (warp == C::MMA) dev::tmem_alloc_pair(dev::smem_u32(tslot), kTmemCols);
    {
        // K chunks past cin (channel padding) are zero for the kernel's lifetime
        const int written = a.cin / 8;
        const int nz = (C::KC - written) * kHalo;
        for (int s = 0; s < C::NS * C::RP; s++)
            for (int i = tid; i < nz; i += C::THREADS)
                reinterpret_cast<uint4 *>(sm + C::AOFF + s * C::SLOT + written * C::LBO_A)[i] = make_uint4(0, 0, 0, 0);
    }
    for (int n = tid; n < 64; n += C::THREADS) {
        sbias[n] = n < NPAD ? a.bias[n] : 0.f;
        sslope[n] = ((n < NPAD && a.slope) ? a.slope[n] : 0.f) - 1.f;
    }
    dev::fence_proxy_async();
    dev::tc_fence_before();
    __syncthreads();
    dev::tc_fence_after();
    const uint32_t tmem = *tslot;

    const bool epi = warp >= C::EPI0 && warp < C::EPI0 + C::EPW;
    const int q = warp & 3, grp = (warp - C::EPI0) >> 2;  // TMEM lane quarter; column group
    const uint32_t lanes = (uint32_t)(q * 32) << 16;
    constexpr int CW = C::CWP;
    // every ring slot starts holding the bias (the MMAs accumulate onto it), the spares zero
    if (epi)
        for_group<NPAD / CW, CW>(grp, [&](auto c0_tag) {
            constexpr int C0 = decltype(c0_tag)::value;
            uint32_t bz[CW], zz[CW];
#pragma unroll
            for (int c = 0; c < CW; c++) {
                bz[c] = __float_as_uint(sbias[C0 + c]);
                zz[c] = 0u;
            }
            for (int sl = 0; sl < S; sl++) tmem_st_cols<CW, C0>(tmem + lanes + (uint32_t)(sl * NPAD), bz);
            for (int sl = S; sl < S + 2; sl++) tmem_st_cols<CW, C0>(tmem + lanes + (uint32_t)(sl * NPAD), zz);
            dev::tmem_wait_st();
        });
    // both CTAs' barriers initialised and TMEM filled before either touches the other's
    dev::tc_fence_before();
    dev::cluster_sync();
    dev::tc_fence_after();
    // launched with programmatic stream serialisation: the previous kernel's outputs (this
    // kernel's inputs) are read only after this wait
    dev::griddep_launch_dependents();
    dev::griddep_wait();

    if (warp == 0) {
        // ================= copier: every lane walks the same rows; lane 0 copies. It waits only for
        // a free stage buffer, so rows are fetched as many stages ahead as there are buffers.
        const int kcin = a.cin / 8;
        const uint32_t bytes = (uint32_t)kcin * kHalo * 16;
        PairWalk walk(W, a.row_begin, a.row_end, a.img_h, cta, ncta);
        bool ok = true;
        uint32_t pi = 0;
        for (; pi < nst; pi++) {
            const uint32_t s = pi % C::NS, ph = (pi / C::NS) & 1;
            if (!(ok = dev::mbar_wait_warp(empty0 + 8 * s, ph ^ 1, a.err, kErrProdEmpty))) break;
            bool zeroed = false;
#pragma unroll
            for (int h = 0; h < C::RP; h++) {
                if ((int)pi * C::RP + h >= K) break;
                int st, r;
                bool in_img, out;
                // past the run: a padding row, left stale (it feeds only discarded accumulators)
                if (!walk.next(st, r, in_img, out)) continue;
                if (in_img) {
                    if (lane == 0) {
                        dev::mbar_expect_tx(full0 + 8 * s, bytes);
                        // the (row, strip) block, halo columns included: the staged row as it is
                        dev::bulk_load(abase + s * C::STAGE + h * C::SLOT, a.src + map_at(r, st, 0, 0, a.nstrips, kcin), bytes,
                                       full0 + 8 * s);
                    }
                } else {
                    // the zero padding above or below an image
                    uint4 *z = reinterpret_cast<uint4 *>(sm + C::AOFF + s * C::STAGE + h * C::SLOT);
                    for (int i = lane; i < C::KC * kHalo; i += 32) z[i] = make_uint4(0, 0, 0, 0);
                    zeroed = true;
                }
            }
            // the zero rows are read by the tensor core (the async proxy)
            if (zeroed) dev::fence_proxy_async();
            __syncwarp();
            if (lane == 0) dev::mbar_arrive(full0 + 8 * s);
        }
        // on an error exit, let the copies in flight land before the CTA can leave (the wait ends
        // at its deadline if the stage cannot complete)
        if (!ok && pi > 0 && lane == 0) dev::mbar_wait(full0 + 8 * ((pi - 1) % C::NS), ((pi - 1) / C::NS) & 1, nullptr, 0);
        __syncwarp();
    } else if (warp == 2 && lead) {
        // ================= even CTA: per stage, wait until the accumulator each of its rows starts
        // (counter k + 2) is free in both CTAs, then arrive on the stage's barrier. (Waiting in the
        // copier instead held each stage's copies back until then: with six ring slots that left
        // rows fetched one stage ahead, and the MMAs waiting on HBM latency.)
        if (lane == 0) {
            for (uint32_t pi = 0; pi < nst; pi++) {
                bool good = true;
                for (int h = 0; h < C::RP && good; h++) {
                    const int k = (int)pi * C::RP + h;
                    if (k >= K) break;
                    const uint32_t c = (uint32_t)k + 2;
                    good = dev::mbar_wait(acce0 + 8 * ring_slot<S>(c), ring_phase<S>(c) ^ 1u, a.err, kErrProdAccEmpty);
                }
                if (!good) break;
                dev::mbar_arrive(full0 + 8 * (pi % C::NS));
            }
        }
        __syncwarp();
    } else if (epi) {
        // ================= epilogue: counters 0 .. K-1 in order; counter c's output row is staged
        // row c - 1's (none for counter 0). Each warp takes 16 columns of its TMEM lane quarter:
        // four warps per SM sub-partition hide each other's TMEM, shared-memory and store
        // latencies. (With two warps of 32 columns each, a row's epilogue took ~1350 cycles, more
        // than the pair MMAs' ~1150, and set the pace.)
        for_group<NPAD / CW, CW>(grp, [&](auto c0_tag) {
            constexpr int C0 = decltype(c0_tag)::value;
            uint32_t bz[CW], zz[CW];
#pragma unroll
            for (int c = 0; c < CW; c++) {
                bz[c] = __float_as_uint(sbias[C0 + c]);
                zz[c] = 0u;
            }
            PairWalk walk(W, a.row_begin, a.row_end, a.img_h, cta, ncta);
            // the output (row o, column x of this thread) of the counter after the previous call
            auto next_out = [&](int &o, int &x) -> bool {
                int st, r;
                bool in_img, out;
                if (!walk.next(st, r, in_img, out) || !out) return false;
                o = r;
                x = st * kTileM + q * 32 + lane;
                return true;
            };
            int o = 0, x = 0;
            bool real = false;  // counter 0 holds no output
            EpiIn<CW> in;
            bool ok = true;
            for (uint32_t c = 0; ok && c < (uint32_t)K; c++) {
                // the next counter's output and its global inputs, loaded before this one's wait
                int no = 0, nx = 0;
                const bool nreal = c + 1 < (uint32_t)K && next_out(no, nx);
                EpiIn<CW> nin;
                if (nreal) epi_prefetch<EK, CW, C0>(nin, a, no, nx);
                const int slot = ring_slot<S>(c);
                ok = dev::mbar_wait_warp(accf0 + 8 * slot, ring_phase<S>(c), a.err, kErrEpiAccFull);
                if (!ok) {
                    // one verdict for all epilogue warps (they meet at the named barrier below)
                    dev::named_bar_red_and(1, C::EPW * 32, false);
                    break;
                }
                __syncwarp();
                dev::tc_fence_after();
                const uint32_t taddr = tmem + lanes + (uint32_t)(slot * NPAD);
                // slots 0 and 1 have a spare holding part of their sum
                const uint32_t saddr = tmem + lanes + (uint32_t)((S + slot) * NPAD);
                float v[CW];
                if (real) {
                    tmem_ld_cols<CW, C0>(taddr, v);
                    dev::tmem_wait_ld();
                    if (slot < 2) tmem_add_cols<CW, C0>(saddr, v);
                }
                // hand the slot back holding the bias (and its spare zero)
                tmem_st_cols<CW, C0>(taddr, bz);
                if (slot < 2) tmem_st_cols<CW, C0>(saddr, zz);
                dev::tmem_wait_st();
                dev::tc_fence_before();
                // the CTA's epilogue warps have all handed the slot back: one arrival for all of
                // them (an arrival per warp, half of them from the other CTA, made the slot's
                // barrier the bottleneck)
                if (!(ok = dev::named_bar_red_and(1, C::EPW * 32, true))) break;
                if (warp == C::EPI0 && lane == 0) {
                    if (lead)
                        dev::mbar_arrive(acce0 + 8 * slot);
                    else
                        dev::mbar_arrive_remote(dev::peer_addr(acce0 + 8 * slot, 0));
                }
                if (real) {
                    uint32_t w[CW / 2];
                    pair_finish<EK, CW, C0>(v, w, a, sslope, in);
                    pair_store<CW, C0>(w, a, o, x);
                }
                real = nreal;
                o = no;
                x = nx;
                in = nin;
            }
        });
    } else if (warp == C::MMA && !lead) {
        // ================= odd CTA: relay its weights' and stages' arrival to the even CTA
        if (lane == 0) {
            bool ok = dev::mbar_wait(wbar, 0, a.err, kErrWeights);
            if (ok) dev::mbar_arrive_remote(dev::peer_addr(wbar, 0));
            for (uint32_t pi = 0; ok && pi < nst; pi++) {
                const uint32_t s = pi % C::NS;
                if (!(ok = dev::mbar_wait(full0 + 8 * s, (pi / C::NS) & 1, a.err, kErrMmaFull))) break;
                dev::mbar_arrive_remote(dev::peer_addr(full0 + 8 * s, 0));
            }
        }
        __syncwarp();
    } else if (warp == C::MMA) {
        // ================= even CTA: the MMA issuer (one thread), a stage of two rows per wait,
        // the next stage's wait inside the second row's MMAs
        if (lane == 0) {
            bool ok = dev::mbar_wait(wbar, 0, a.err, kErrWeights);
            const uint64_t bdesc0 = dev::sdesc(wbase, C::LBO_B, 128);
            const uint64_t adesc_base = dev::sdesc(abase, C::LBO_A, 128);
            constexpr uint32_t idesc = dev::idesc_f16_f32(2 * kTileM, C::N);
            // staged row k: its window starts at counter k + 2's slot; dx columns [dx0, dx1)
            auto issue = [&](uint64_t adesc, int k, int dx0, int dx1) {
                const uint32_t d = tmem + (uint32_t)(ring_slot<S>((uint32_t)k + 2) * NPAD);
#pragma unroll
                for (int dx = 0; dx < 3; dx++) {
                    if (dx < dx0 || dx >= dx1) continue;
#pragma unroll
                    for (int kk = 0; kk < C::KS; kk++) {
                        const uint64_t ad = adesc + (uint64_t)((kk * 2 * C::LBO_A + dx * 16) >> 4);
                        const uint64_t bd = bdesc0 + (uint64_t)(((dx * C::KC + 2 * kk) * C::LBO_B) >> 4);
                        dev::mma_f16_pair(d, ad, bd, idesc, 1u);
                    }
                }
            };
            // arrive on the barrier in both CTAs when the MMAs so far are done
            auto commit2 = [&](uint32_t bar) {
                dev::mma_commit_pair(bar);
                dev::mma_commit_pair(dev::peer_addr(bar, 1));
            };
            if (ok && nst > 0) {
                ok = dev::mbar_wait(full0, 0, a.err, kErrMmaFull);
                dev::tc_fence_after();
            }
            for (uint32_t pi = 0; ok && pi < nst; pi++) {
                const uint32_t s = pi % C::NS;
                const int k0 = (int)pi * C::RP;
                const uint64_t ad0 = adesc_base + (uint64_t)((s * C::STAGE) >> 4), ad1 = ad0 + (uint64_t)(C::SLOT >> 4);
                const bool two = k0 + 1 < K;
                issue(ad0, k0, 0, 3);
                // counter k0 is complete: the epilogue starts on it a row earlier
                commit2(accf0 + 8 * ring_slot<S>((uint32_t)k0));
                if (two) issue(ad1, k0 + 1, 0, 1);
                bool okn = true;
                if (pi + 1 < nst) {
                    okn = dev::mbar_wait(full0 + 8 * ((pi + 1) % C::NS), ((pi + 1) / C::NS) & 1, a.err, kErrMmaFull);
                    dev::tc_fence_after();
                }
                if (two) issue(ad1, k0 + 1, 1, 3);
                commit2(empty0 + 8 * s);
                if (two) commit2(accf0 + 8 * ring_slot<S>((uint32_t)(k0 + 1)));
                ok = okn;
            }
            // every MMA issued has completed before the pair leaves
            dev::mma_commit_pair(dbar);
            dev::mbar_wait(dbar, 0, a.err, kErrDrain);
        }
        __syncwarp();
    }

    dev::tc_fence_before();
    dev::cluster_sync();
    if (warp == C::MMA) {
        dev::tc_fence_after();
        dev::tmem_dealloc_pair(tmem, kTmemCols);
    }
}

}  // namespace ajib
