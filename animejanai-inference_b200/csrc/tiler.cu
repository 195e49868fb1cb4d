// tiler.cu — device side of the image tiler (see tiler.h): batched tile extraction and the
// gather composition of the blended 8-bit output.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "cuctx.h"
#include "tiler.h"
#include "../../include/aji_b200.h"

namespace ajib {
namespace {

__device__ __forceinline__ int d_reflect(int i, int n)
{
    if (n == 1) return 0;
    const int period = 2 * (n - 1);
    i %= period;
    if (i < 0) i += period;
    return i < n ? i : period - i;
}

// tile k0 + blockIdx.z: pixels (x8 .. x8 + 7, y) of the reflect-padded tile, as the net's fp16
// input v * (1/255) (the reference's k_extract, src/core/tiling_gpu.cu:71-96, 3-channel model).
// Eight adjacent tile columns a thread: the row's reflection once, the columns' only where they
// leave the image, and each plane's eight values as one 16-byte store where the tile width
// allows (a warp reads 32 x 8 consecutive image pixels and writes 512 contiguous bytes a plane).
__global__ void k_extract(const uint8_t *img, int W, int H, int ci, const int *ox, const int *oy, int nx, int tw,
                          int th, int k0, int n, float inv255, __half *dst)
{
    const int x8 = (blockIdx.x * blockDim.x + threadIdx.x) * 8, y = blockIdx.y * blockDim.y + threadIdx.y, k = blockIdx.z;
    if (x8 >= tw || y >= th) return;
    const int t = k0 + k, i = t % nx, j = t / nx;
    const uint8_t *row = img + (size_t)d_reflect(oy[j] + y, H) * W * ci;
    const int gx0 = ox[i] + x8;
    const size_t plane = (size_t)n * th * tw, at = ((size_t)k * th + y) * tw + x8;
    const int g = ci == 1;
    const int nq = min(8, tw - x8);
    const bool inside = gx0 >= 0 && gx0 + 8 <= W;
    __half v[3][8];
#pragma unroll
    for (int q = 0; q < 8; q++) {
        const int gx = inside ? gx0 + q : d_reflect(gx0 + q, W);
        const uint8_t *p = row + (size_t)gx * ci;
#pragma unroll
        for (int c = 0; c < 3; c++) v[c][q] = __float2half_rn(__fmul_rn((float)p[g ? 0 : c], inv255));
    }
    if (nq == 8 && (tw & 7) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
        for (int c = 0; c < 3; c++) *reinterpret_cast<uint4 *>(dst + c * plane + at) = *reinterpret_cast<const uint4 *>(v[c]);
    } else {
#pragma unroll
        for (int q = 0; q < 8; q++)
            if (q < nq)
#pragma unroll
                for (int c = 0; c < 3; c++) dst[c * plane + at + q] = v[c][q];
    }
}

// out[Y - Y0][X][c] = u8(sum over covering tiles, tile rows then tiles, of (wy * wx) * tile), each
// multiply and add rounded on its own (the reference's k_blend + k_flush, tiling_gpu.cu:98-134),
// for output rows [Y0, Y0 + gridDim.y * kComposeBlockRows) clipped to Y1; the tiles buffer holds
// tiles [k0, k0 + ntiles) of the image's row-major tile order. A block takes kComposeBlockRows
// output rows and 64 * kComposeQ columns: it looks its rows' covering tile rows, tile-row offsets
// and vertical weights up once into shared memory, each thread looks its four adjacent columns'
// covering tiles (and, on the vector path, their tile columns and weights) up once, and then
// walks the rows, two at a time; on the vector path a pair's tile loads are asynchronous copies
// into shared memory issued while the previous pair is summed and stored. (One block per eight
// rows paid that chain of dependent table loads for every eight rows: 0.52 ms at config 2 against
// 0.33 with the block-wide tables, 0.31 with the copies one pair ahead.) Where four pixels share their covering tiles at a
// 4-aligned tile column the tile values are read 8 bytes at a time and the 8-bit output written 4
// bytes at a time. Per pixel and channel the arithmetic is the same in either path.
constexpr int kComposeQ = 4;     // output pixels per thread and row
constexpr int kComposeRows = 8;  // output rows per block (two per thread)
constexpr int kComposeMaxT = 8;  // tile rows covering one output row that the table holds
constexpr int kComposeBlockRows = 128;  // output rows per block (its row table is filled once)

__device__ __forceinline__ uint8_t to_u8(float b)
{
    const float f = __fadd_rn(__fmul_rn(b, 255.0f), 0.5f);
    return f <= 0.0f ? 0 : f >= 255.0f ? 255 : (uint8_t)f;
}

// One output row's four pixels at X0 (nq of them inside the image) into b[c][q].
__device__ __forceinline__ void compose_row(float (&b)[3][kComposeQ], const __half *tiles, size_t plane, int k0, int toh,
                                            int tow, int nx, const int *ox, const float *wx, int cols, int s, int co,
                                            int X0, int nq, const int2 (&rx)[kComposeQ], bool same, int nj,
                                            const int *jrow, const int *vrow, const float *wvrow)
{
#pragma unroll
    for (int c = 0; c < 3; c++)
#pragma unroll
        for (int q = 0; q < kComposeQ; q++) b[c][q] = 0.0f;
    for (int jj = 0; jj < nj; jj++) {
        const int j = jrow[jj], v = vrow[jj];
        const float wv = wvrow[jj];
        if (same) {
            for (int ii = 0; ii < rx[0].y; ii++) {
                const int i = rx[0].x + ii, u = X0 - __ldg(ox + i) * s, k = j * nx + i - k0;
                const float4 wq = __ldg(reinterpret_cast<const float4 *>(wx + (size_t)i * cols + u));
                const float w[4] = {__fmul_rn(wv, wq.x), __fmul_rn(wv, wq.y), __fmul_rn(wv, wq.z), __fmul_rn(wv, wq.w)};
                const size_t at = ((size_t)k * toh + v) * tow + u;
#pragma unroll
                for (int c = 0; c < 3; c++) {
                    if (c >= co) break;
                    const uint2 raw = __ldg(reinterpret_cast<const uint2 *>(tiles + (co == 1 ? 0 : c) * plane + at));
                    const float2 t01 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
                    const float2 t23 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
                    b[c][0] = __fadd_rn(b[c][0], __fmul_rn(w[0], t01.x));
                    b[c][1] = __fadd_rn(b[c][1], __fmul_rn(w[1], t01.y));
                    b[c][2] = __fadd_rn(b[c][2], __fmul_rn(w[2], t23.x));
                    b[c][3] = __fadd_rn(b[c][3], __fmul_rn(w[3], t23.y));
                }
            }
        } else {
#pragma unroll
            for (int q = 0; q < kComposeQ; q++) {
                if (q >= nq) break;
                const int X = X0 + q;
                for (int ii = 0; ii < rx[q].y; ii++) {
                    const int i = rx[q].x + ii, u = X - __ldg(ox + i) * s, k = j * nx + i - k0;
                    const float w = __fmul_rn(wv, __ldg(wx + (size_t)i * cols + u));
                    const size_t at = ((size_t)k * toh + v) * tow + u;
#pragma unroll
                    for (int c = 0; c < 3; c++) {
                        if (c >= co) break;
                        b[c][q] = __fadd_rn(b[c][q], __fmul_rn(w, __half2float(tiles[(co == 1 ? 0 : c) * plane + at])));
                    }
                }
            }
        }
    }
}

__device__ __forceinline__ void compose_store(const float (&b)[3][kComposeQ], uint8_t *o, int nq, int co, int OW)
{
    if (nq == kComposeQ && co == 3 && (OW & 3) == 0 && (reinterpret_cast<uintptr_t>(o) & 3) == 0) {
        // 12 bytes: pixel-major r, g, b of the four pixels, as three 4-byte words
        uint32_t *o4 = reinterpret_cast<uint32_t *>(o);
#pragma unroll
        for (int k = 0; k < 3; k++) {
            uint32_t wd = 0;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int flat = 4 * k + e, q = flat / 3, c = flat % 3;
                wd |= (uint32_t)to_u8(b[c][q]) << (8 * e);
            }
            o4[k] = wd;
        }
    } else if (nq == kComposeQ && co == 1 && (OW & 3) == 0 && (reinterpret_cast<uintptr_t>(o) & 3) == 0) {
        uint32_t wd = 0;
#pragma unroll
        for (int q = 0; q < kComposeQ; q++) wd |= (uint32_t)to_u8(b[0][q]) << (8 * q);
        *reinterpret_cast<uint32_t *>(o) = wd;
    } else {
#pragma unroll
        for (int q = 0; q < kComposeQ; q++)
#pragma unroll
            for (int c = 0; c < 3; c++)
                if (q < nq && c < co) o[q * co + c] = to_u8(b[c][q]);
    }
}

// The vector path where every pixel of the thread's columns and rows is covered by at most two
// tiles along each axis (every cover whose overlap is under half a tile, config 2's included):
// the thread's horizontal weights are loaded once, its tile loads for a pair of rows (up to
// 2 rows x 2 tile rows x 2 tiles x 3 channels of 4 pixels) go out together, and each pixel's sum
// runs in compose_row's order (tile rows, then tiles, each multiply and add rounded on its own).
constexpr int kComposeF = 2;

// Its tile loads are asynchronous copies (cp.async, 8 bytes each) into the thread's own slots in
// shared memory, so that a row pair's loads are in flight while the thread
// sums and stores the previous pair (the bytes a thread keeps in flight no longer wait on
// registers). Slot-major layout [slot][thread]: a warp's 32 slots of one kind are 256 contiguous
// bytes. Only the issuing thread reads its slots, after its own cp.async.wait_group.
constexpr int kComposeSlots = 2 * kComposeF * kComposeF * 3;  // per row pair
constexpr int kComposeThreads = 256;
constexpr size_t kComposeDynSmem = 2 * kComposeSlots * kComposeThreads * sizeof(uint2);

__device__ __forceinline__ void cp_async8(void *smem, const void *gmem)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)), "l"(gmem)
                 : "memory");
}

__device__ __forceinline__ int compose_slot(int r, int jj, int ii, int c) { return ((r * kComposeF + jj) * kComposeF + ii) * 3 + c; }

__device__ __forceinline__ void compose_pair_issue(uint2 *stage, int tid, const __half *tiles, size_t plane, int k0, int toh,
                                                   int tow, int nx, int i0, int ni, const int (&u)[kComposeF],
                                                   const int (&nj)[2], const int *j0, const int *v0, const int *j1,
                                                   const int *v1)
{
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const int *jr = r ? j1 : j0, *vr = r ? v1 : v0;
#pragma unroll
        for (int jj = 0; jj < kComposeF; jj++) {
#pragma unroll
            for (int ii = 0; ii < kComposeF; ii++) {
                if (jj < nj[r] && ii < ni) {
                    const int k = jr[jj] * nx + i0 + ii - k0;
                    const size_t at = ((size_t)k * toh + vr[jj]) * tow + u[ii];
#pragma unroll
                    for (int c = 0; c < 3; c++)
                        cp_async8(&stage[compose_slot(r, jj, ii, c) * kComposeThreads + tid], tiles + c * plane + at);
                }
            }
        }
    }
}

__device__ __forceinline__ void compose_pair_sum(float (&ba)[3][kComposeQ], float (&bb)[3][kComposeQ], const uint2 *stage,
                                                 int tid, int ni, const float4 (&wq)[kComposeF], const int (&nj)[2],
                                                 const float *wv0, const float *wv1)
{
#pragma unroll
    for (int r = 0; r < 2; r++) {
        float(&b)[3][kComposeQ] = r ? bb : ba;
        const float *wvr = r ? wv1 : wv0;
#pragma unroll
        for (int c = 0; c < 3; c++)
#pragma unroll
            for (int q = 0; q < kComposeQ; q++) b[c][q] = 0.0f;
#pragma unroll
        for (int jj = 0; jj < kComposeF; jj++) {
            if (jj >= nj[r]) break;
            const float wv = wvr[jj];
#pragma unroll
            for (int ii = 0; ii < kComposeF; ii++) {
                if (ii >= ni) break;
                const float w[4] = {__fmul_rn(wv, wq[ii].x), __fmul_rn(wv, wq[ii].y), __fmul_rn(wv, wq[ii].z),
                                    __fmul_rn(wv, wq[ii].w)};
#pragma unroll
                for (int c = 0; c < 3; c++) {
                    const uint2 raw = stage[compose_slot(r, jj, ii, c) * kComposeThreads + tid];
                    const float2 t01 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
                    const float2 t23 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
                    b[c][0] = __fadd_rn(b[c][0], __fmul_rn(w[0], t01.x));
                    b[c][1] = __fadd_rn(b[c][1], __fmul_rn(w[1], t01.y));
                    b[c][2] = __fadd_rn(b[c][2], __fmul_rn(w[2], t23.x));
                    b[c][3] = __fadd_rn(b[c][3], __fmul_rn(w[3], t23.y));
                }
            }
        }
    }
}

__global__ void __launch_bounds__(256, 2) k_compose(const __half *tiles, int k0, int ntiles, int toh, int tow, int nx,
                                                 const int *ox, const int *oy, const float *wx, const float *wy, int cols,
                                                 int rows, const int2 *cx, const int2 *cy, int s, int co, int OW, int Y0,
                                                 int Y1, uint8_t *out)
{
    // the block's rows: covering tile rows, their row offsets and vertical weights, looked up once
    __shared__ int s_nj[kComposeBlockRows], s_j[kComposeBlockRows][kComposeMaxT], s_v[kComposeBlockRows][kComposeMaxT];
    __shared__ float s_wv[kComposeBlockRows][kComposeMaxT];
    const int Yblk = Y0 + blockIdx.y * kComposeBlockRows;
    const int tid = threadIdx.y * blockDim.x + threadIdx.x;
    for (int r = tid; r < kComposeBlockRows; r += blockDim.x * blockDim.y) {
        const int Y = Yblk + r;
        int n = 0;
        if (Y < Y1) {
            const int2 ry = cy[Y];
            n = min(ry.y, kComposeMaxT);
            for (int jj = 0; jj < n; jj++) {
                const int j = ry.x + jj, v = Y - oy[j] * s;
                s_j[r][jj] = j;
                s_v[r][jj] = v;
                s_wv[r][jj] = wy[(size_t)j * rows + v];
            }
        }
        s_nj[r] = n;
    }
    __syncthreads();
    const int X0 = (blockIdx.x * blockDim.x + threadIdx.x) * kComposeQ;
    if (X0 >= OW) return;
    const size_t plane = (size_t)ntiles * toh * tow;
    const int nq = min(kComposeQ, OW - X0);
    // the thread's columns: their covering tiles, and for the vector path their tile columns and
    // horizontal weights (the same for every row)
    int2 rx[kComposeQ];
    bool same = nq == kComposeQ;
#pragma unroll
    for (int q = 0; q < kComposeQ; q++) {
        rx[q] = q < nq ? cx[X0 + q] : make_int2(0, 0);
        same = same && rx[q].x == rx[0].x && rx[q].y == rx[0].y;
    }
    // the vector path: every covering tile's column of X0 is 4-aligned, and so are the tile rows,
    // the weight rows and the tiles' base address (16-byte weight and 8-byte tile loads)
    same = same && (tow & 3) == 0 && (cols & 3) == 0 && (reinterpret_cast<uintptr_t>(tiles) & 7) == 0;
    if (same) {
        for (int ii = 0; ii < rx[0].y; ii++) same = same && (((X0 - __ldg(ox + rx[0].x + ii) * s) & 3) == 0);
    }
    const bool fast = same && co == 3 && rx[0].y <= kComposeF;
    int u[kComposeF];
    float4 wq[kComposeF];
#pragma unroll
    for (int ii = 0; ii < kComposeF; ii++) {
        u[ii] = 0;
        wq[ii] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (fast && ii < rx[0].y) {
            u[ii] = X0 - __ldg(ox + rx[0].x + ii) * s;
            wq[ii] = __ldg(reinterpret_cast<const float4 *>(wx + (size_t)(rx[0].x + ii) * cols + u[ii]));
        }
    }
    // rows g + ty and g + ty + blockDim.y of each group of kComposeRows: pair k = g / kComposeRows
    extern __shared__ uint2 cbuf[];  // [2 stages][kComposeSlots][kComposeThreads]
    constexpr int kPairs = kComposeBlockRows / kComposeRows;
    auto pair_rows = [&](int k, int &ra, int &rb, int &nja, int &njb) -> bool {
        if (k >= kPairs) return false;  // (the prefetch of the pair after the block's last)
        ra = k * kComposeRows + threadIdx.y;
        rb = ra + blockDim.y;
        if (Yblk + ra >= Y1) return false;
        nja = s_nj[ra];
        njb = Yblk + rb < Y1 ? s_nj[rb] : 0;
        return true;
    };
    // the pair's loads go through shared memory when the vector path serves it
    auto pair_async = [&](int nja, int njb) { return fast && nja <= kComposeF && njb <= kComposeF; };
    auto issue = [&](int k) {
        int ra, rb, nja, njb;
        if (pair_rows(k, ra, rb, nja, njb) && pair_async(nja, njb)) {
            const int nj[2] = {nja, njb};
            compose_pair_issue(cbuf + (size_t)(k & 1) * kComposeSlots * kComposeThreads, tid, tiles, plane, k0, toh, tow, nx,
                               rx[0].x, rx[0].y, u, nj, s_j[ra], s_v[ra], s_j[rb], s_v[rb]);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    issue(0);
    for (int k = 0; k < kPairs; k++) {
        int ra, rb, nja, njb;
        if (!pair_rows(k, ra, rb, nja, njb)) break;
        const int Ya = Yblk + ra, Yb2 = Yblk + rb;
        issue(k + 1);
        float ba[3][kComposeQ], bb[3][kComposeQ];
        if (pair_async(nja, njb)) {
            asm volatile("cp.async.wait_group 1;" ::: "memory");
            const int nj[2] = {nja, njb};
            compose_pair_sum(ba, bb, cbuf + (size_t)(k & 1) * kComposeSlots * kComposeThreads, tid, rx[0].y, wq, nj,
                             s_wv[ra], s_wv[rb]);
        } else {
            compose_row(ba, tiles, plane, k0, toh, tow, nx, ox, wx, cols, s, co, X0, nq, rx, same, nja, s_j[ra], s_v[ra],
                        s_wv[ra]);
            if (Yb2 < Y1)
                compose_row(bb, tiles, plane, k0, toh, tow, nx, ox, wx, cols, s, co, X0, nq, rx, same, njb, s_j[rb],
                            s_v[rb], s_wv[rb]);
        }
        compose_store(ba, out + ((size_t)(Ya - Y0) * OW + X0) * co, nq, co, OW);
        if (Yb2 < Y1) compose_store(bb, out + ((size_t)(Yb2 - Y0) * OW + X0) * co, nq, co, OW);
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// the most tiles covering one output coordinate (the compose kernel holds kComposeMaxT a row)
int max_cover(const std::vector<int2> &c)
{
    int m = 0;
    for (const int2 &e : c) m = std::max(m, e.y);
    return m;
}

// per output coordinate along one axis: the first tile covering it and how many do
std::vector<int2> cover(const std::vector<int> &org, int span, int s, int len)
{
    std::vector<int2> c((size_t)len * s);
    for (int X = 0; X < len * s; X++) {
        int first = -1, n = 0;
        for (int t = 0; t < (int)org.size(); t++)
            if (X >= org[t] * s && X < (org[t] + span) * s) {
                if (first < 0) first = t;
                n++;
            }
        c[X] = make_int2(first, n);
    }
    return c;
}

template <typename T>
bool upload(T **d, const std::vector<T> &h, size_t *bytes)
{
    if (cudaMalloc(d, h.size() * sizeof(T)) != cudaSuccess) return false;
    *bytes += h.size() * sizeof(T);
    return cudaMemcpy(*d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice) == cudaSuccess;
}

}  // namespace

DeviceTiler::~DeviceTiler()
{
    cudaFree(d_ox_);
    cudaFree(d_oy_);
    cudaFree(d_wx_);
    cudaFree(d_wy_);
    cudaFree(d_cx_);
    cudaFree(d_cy_);
}

bool DeviceTiler::init(const TileGeometry &g)
{
    g_ = g;
    const int s = g.scale;
    const int spw = std::min(g.tw, g.W), sph = std::min(g.th, g.H);
    const std::vector<int2> cy = cover(g.oy, sph, s, g.H);
    // an output row covered by more tile rows than the compose kernel's table holds: refuse
    if (max_cover(cy) > kComposeMaxT) return false;
    return upload(&d_ox_, g.ox, &bytes_) && upload(&d_oy_, g.oy, &bytes_) &&
           upload(&d_wx_, axis_weights(g.ox, g.W, g.tw, s), &bytes_) &&
           upload(&d_wy_, axis_weights(g.oy, g.H, g.th, s), &bytes_) && upload(&d_cx_, cover(g.ox, spw, s, g.W), &bytes_) &&
           upload(&d_cy_, cy, &bytes_);
}

cudaError_t DeviceTiler::extract(const uint8_t *img, int k0, int n, void *dst, cudaStream_t s) const
{
    if (n < 1) return cudaSuccess;
    const dim3 block(32, 8), grid((g_.tw + 255) / 256, (g_.th + 7) / 8, n);
    k_extract<<<grid, block, 0, s>>>(img, g_.W, g_.H, g_.ci, d_ox_, d_oy_, g_.nx(), g_.tw, g_.th, k0, n, 1.0f / 255.0f,
                                     (__half *)dst);
    return cudaGetLastError();
}

cudaError_t DeviceTiler::compose(const void *tiles, uint8_t *out, cudaStream_t st) const
{
    return compose_rows(tiles, 0, g_.count(), 0, g_.H * g_.scale, out, st);
}

cudaError_t DeviceTiler::compose_rows(const void *tiles, int k0, int ntiles, int Y0, int Y1, uint8_t *out,
                                      cudaStream_t st) const
{
    const int s = g_.scale, OW = g_.W * s;
    if (Y1 <= Y0) return cudaSuccess;
    const int cols = std::min(g_.tw, g_.W) * s, rows = std::min(g_.th, g_.H) * s;
    const int px = 64 * kComposeQ;  // output columns per block
    const dim3 block(64, kComposeRows / 2), grid((OW + px - 1) / px, (Y1 - Y0 + kComposeBlockRows - 1) / kComposeBlockRows);
    const cudaError_t ae = cudaFuncSetAttribute(k_compose, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kComposeDynSmem);
    if (ae != cudaSuccess) return ae;
    k_compose<<<grid, block, kComposeDynSmem, st>>>((const __half *)tiles, k0, ntiles, g_.th * s, g_.tw * s, g_.nx(),
                                                    d_ox_, d_oy_, d_wx_, d_wy_, cols, rows, d_cx_, d_cy_, s, g_.ci, OW,
                                                    Y0, Y1, out);
    return cudaGetLastError();
}

}  // namespace ajib

// ---------------------------------------------------------------------------------------------
// Composition that allocates no device memory (ajib_tiler_compose_static, include/aji_b200.h).
//
// For callers that may not call cudaMalloc: a host application whose device memory all comes
// from its own allocator or budget, or a real-time frame path where cudaMalloc / cudaFree would
// synchronise the device. The geometry tables that ajib_tiler_create keeps in memory it
// allocates live here in one fixed area that every GPU loading this library holds until the
// process exits. Each call rewrites every table byte it reads, so nothing has to start at zero;
// but all calls on a device share the area, so calls that overlap on the GPU race.

namespace ajib {
namespace {

constexpr size_t kStaticTableBytes = 1u << 20;  // 1 MiB: outputs up to about 24K x 24K pixels
static __device__ __align__(256) unsigned char g_tiler_tables[kStaticTableBytes];
// The host image of the tables a call uploads: file-scope, so the copy's source lives as long as
// the process whatever the copy's timing; written and copied under g_static_mu.
static unsigned char g_host_tables[kStaticTableBytes];
std::mutex g_static_mu;

// The area's device address for the current device and context. In host code g_tiler_tables names
// a host-side stand-in, not the device memory, so the address comes from cudaGetSymbolAddress:
// once per device, on the first call made with that device current, and again if that device's
// current context has changed since (a reset or a recreated primary context maps the module
// anew). The caller holds g_static_mu.
void *static_tables()
{
    static void *addr[64] = {};
    static CUcontext ctx_of[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    CUcontext cur = nullptr;
    const Driver &d = driver();
    if (!d.ok || d.ctx_get_current(&cur) != CUDA_SUCCESS) return nullptr;
    if (!addr[dev] || ctx_of[dev] != cur) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_tiler_tables) != cudaSuccess) return nullptr;
        // the lookup may have made the device's primary context current: key the cache on that
        if (d.ctx_get_current(&cur) != CUDA_SUCCESS) return nullptr;
        addr[dev] = p;
        ctx_of[dev] = cur;
    }
    return addr[dev];
}

size_t align256(size_t n) { return (n + 255) / 256 * 256; }

template <typename T>
size_t put(std::vector<unsigned char> &buf, const std::vector<T> &v)
{
    const size_t at = buf.size();
    buf.resize(align256(at + v.size() * sizeof(T)));
    std::memcpy(buf.data() + at, v.data(), v.size() * sizeof(T));
    return at;
}

}  // namespace

}  // namespace ajib

extern "C" int ajib_tiler_compose_static(int W, int H, int ci, int scale, int tile_w, int tile_h, int overlap, int even,
                                         const void *tiles, uint8_t *out, void *stream)
{
    using namespace ajib;
    if (!tiles || !out || W < 1 || H < 1 || (ci != 1 && ci != 3) || scale < 1 || tile_w < 1 || tile_h < 1 || overlap < 0)
        return AJIB_ERR_ARGS;
    try {
        const TileGeometry g = make_geometry(W, H, ci, scale, tile_w, tile_h, overlap, even != 0);
        const int s = g.scale, spw = std::min(g.tw, g.W), sph = std::min(g.th, g.H);
        // the tables of DeviceTiler::init, packed at 256-byte offsets into one host image
        std::vector<unsigned char> img;
        const size_t o_ox = put(img, g.ox), o_oy = put(img, g.oy);
        const size_t o_wx = put(img, axis_weights(g.ox, g.W, g.tw, s)), o_wy = put(img, axis_weights(g.oy, g.H, g.th, s));
        const std::vector<int2> cyv = cover(g.oy, sph, s, g.H);
        if (max_cover(cyv) > kComposeMaxT) return AJIB_ERR_UNSUPPORTED;  // more covering tile rows than the kernel holds
        const size_t o_cx = put(img, cover(g.ox, spw, s, g.W)), o_cy = put(img, cyv);
        if (img.size() > kStaticTableBytes) return AJIB_ERR_UNSUPPORTED;  // tables beyond the fixed area
        const cudaStream_t st = (cudaStream_t)stream;
        unsigned char *base = nullptr;
        {
            std::lock_guard<std::mutex> lk(g_static_mu);
            base = static_cast<unsigned char *>(static_tables());
            if (!base) return AJIB_ERR_CUDA;
            // a copy from pageable host memory: it returns once the bytes are staged (and may wait
            // for earlier work on st first), so the next call may rewrite the host image
            std::memcpy(g_host_tables, img.data(), img.size());
            if (cudaMemcpyAsync(base, g_host_tables, img.size(), cudaMemcpyHostToDevice, st) != cudaSuccess)
                return AJIB_ERR_CUDA;
        }
        const int OW = g.W * s, OH = g.H * s;
        const dim3 block(64, kComposeRows / 2),
            grid((OW + 64 * kComposeQ - 1) / (64 * kComposeQ), (OH + kComposeBlockRows - 1) / kComposeBlockRows);
        if (cudaFuncSetAttribute(k_compose, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kComposeDynSmem) != cudaSuccess)
            return AJIB_ERR_CUDA;
        k_compose<<<grid, block, kComposeDynSmem, st>>>(
            (const __half *)tiles, 0, g.count(), g.th * s, g.tw * s, g.nx(), (const int *)(base + o_ox),
            (const int *)(base + o_oy), (const float *)(base + o_wx), (const float *)(base + o_wy), spw * s, sph * s,
            (const int2 *)(base + o_cx), (const int2 *)(base + o_cy), s, g.ci, OW, 0, OH, out);
        return cudaGetLastError() == cudaSuccess ? AJIB_OK : AJIB_ERR_CUDA;
    } catch (...) {
        return AJIB_ERR_NO_MEM;
    }
}
