/*
 * selftest.cu — a one-CTA check of the tcgen05 operand encodings the conv kernels rely on:
 * K-major no-swizzle shared-memory descriptors, the f16/f32 instruction descriptor, TMEM
 * accumulator layout (row i = lane i), a start address shifted by whole 16-byte rows (how the
 * conv kernels address the three horizontal taps of one staged input row), and reuse of the A
 * operand through the collector buffer across MMAs with different B and D.
 *
 * The shared-memory regions are sized so that every address either reading of the descriptor
 * fields could produce stays inside the CTA's allocation.
 */
#include <cuda_runtime.h>

#include "sm100.cuh"
#include "../../include/aji_b200.h"

namespace ajib {
namespace {

constexpr int kRowsA = 130;       // staged rows (pixels): a 128-row operand shifted by up to 2
constexpr int kK = 32;            // two K steps of 16
constexpr int kRegionA = 48 * 1024;
constexpr int kRegionB = 32 * 1024;

__global__ void __launch_bounds__(128, 1) k_selftest(const __half *a, const __half *b, float *out, int N, int shift,
                                                     int collector, int *err)
{
    extern __shared__ __align__(1024) unsigned char sm[];
    unsigned char *sa = sm, *sb = sm + kRegionA;
    uint64_t *bar = reinterpret_cast<uint64_t *>(sm + kRegionA + kRegionB);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bar + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // A: global [130][32] row-major -> shared [kc][row][8]; B: global [2N][32] -> [kc][n][8]
    for (int i = tid; i < kRegionA / 16; i += 128) reinterpret_cast<uint4 *>(sa)[i] = make_uint4(0, 0, 0, 0);
    for (int i = tid; i < kRegionB / 16; i += 128) reinterpret_cast<uint4 *>(sb)[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();
    for (int i = tid; i < kRowsA * (kK / 8); i += 128) {
        const int r = i / (kK / 8), kc = i % (kK / 8);
        reinterpret_cast<uint4 *>(sa)[kc * kRowsA + r] = reinterpret_cast<const uint4 *>(a)[i];
    }
    for (int i = tid; i < 2 * N * (kK / 8); i += 128) {
        const int n = i / (kK / 8), kc = i % (kK / 8);
        reinterpret_cast<uint4 *>(sb)[kc * 2 * N + n] = reinterpret_cast<const uint4 *>(b)[i];
    }
    dev::fence_proxy_async();
    if (tid == 0) {
        dev::mbar_init(dev::smem_u32(bar), 1);
        dev::fence_mbar_init();
    }
    if (warp == 0) dev::tmem_alloc(dev::smem_u32(tslot), 128);
    dev::tc_fence_before();
    __syncthreads();
    dev::tc_fence_after();
    const uint32_t tmem = *tslot;

    if (tid == 0) {
        const uint32_t idesc = dev::idesc_f16_f32(128, N);
        const uint32_t lbo_a = kRowsA * 16, lbo_b = 2 * N * 16;
        for (int kk = 0; kk < kK / 16; kk++) {
            const uint64_t ad = dev::sdesc(dev::smem_u32(sa) + kk * 2 * lbo_a + shift * 16, lbo_a, 128);
            const uint64_t b0 = dev::sdesc(dev::smem_u32(sb) + kk * 2 * lbo_b, lbo_b, 128);
            const uint64_t b1 = dev::sdesc(dev::smem_u32(sb) + kk * 2 * lbo_b + N * 16, lbo_b, 128);
            dev::mma_f16(tmem, ad, b0, idesc, kk > 0, collector ? 1 : 0);
            dev::mma_f16(tmem + (uint32_t)N, ad, b1, idesc, kk > 0, collector ? 3 : 0);
        }
        dev::mma_commit(dev::smem_u32(bar));
    }
    __syncwarp();
    const bool ok = dev::mbar_wait(dev::smem_u32(bar), 0, err, 1);
    dev::tc_fence_after();
    if (ok) {
        const int row = warp * 32 + lane;
        for (int c = 0; c < 2 * N; c += 16) {
            float v[16];
            dev::tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, v);
            dev::tmem_wait_ld();
            const int which = c / N, col = c % N;
            for (int j = 0; j < 16; j++) out[((size_t)which * 128 + row) * N + col + j] = v[j];
        }
    }
    dev::tc_fence_before();
    __syncthreads();
    if (warp == 0) dev::tmem_dealloc(tmem, 128);
}

}  // namespace
}  // namespace ajib

extern "C" int ajib_selftest_umma(const void *a, const void *b, float *out, int n, int shift, int collector, int *err,
                                  void *stream)
{
    if (!a || !b || !out || (n != 16 && n != 32 && n != 48 && n != 64) || shift < 0 || shift > 2) return AJIB_ERR_ARGS;
    const int smem = ajib::kRegionA + ajib::kRegionB + 64;
    cudaError_t e = cudaFuncSetAttribute(ajib::k_selftest, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return AJIB_ERR_CUDA;
    ajib::k_selftest<<<1, 128, smem, (cudaStream_t)stream>>>((const __half *)a, (const __half *)b, out, n, shift, collector,
                                                            err);
    return cudaGetLastError() == cudaSuccess ? AJIB_OK : AJIB_ERR_CUDA;
}

// ---- the colour kernels' division by a constant (colour_math.cuh) against the IEEE division ----
#include "colour_math.cuh"

namespace ajib {
namespace {

// Every float with 2^-80 <= |a| < 2^18 (exponent field 47..144, both signs) divided by each
// given divisor (direct), or by 2 (1 - k) for each given k (the post pass's divisors of its colour
// differences): dev::div_by against __fdiv_rn. Counts the quotients that differ and records the
// first such a. Tinier dividends are outside the correction's range (below ~2^-100 its remainder
// underflows) and outside the passes': the post pass's dividends b - Y are differences of an fp16
// colour (a multiple of 2^-24) and a weighted sum of fp16 colours by fp32 coefficients (a multiple
// of 2^-52), so zero or at least 2^-52 in magnitude, and below 2^18 (fp16 colours are below
// 2^16); the pre pass's are raw - yoff (integers below 2^17) and u - coff, u an FMA chain of fp32
// filter weights (zero or above 2^-40) times integer samples below 2^16, so zero or at least 2^-63.
__global__ void k_div_check(const float *ks, int nk, int direct, unsigned long long *bad, unsigned int *first)
{
    float d[8], r[8];
    for (int j = 0; j < nk; j++) {
        d[j] = direct ? ks[j] : __fmul_rn(2.0f, __fsub_rn(1.0f, ks[j]));
        r[j] = __frcp_rn(d[j]);
    }
    const uint64_t half = (145ull - 47ull) << 23, n = 2 * half;
    unsigned long long mine = 0;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t bits = ((uint32_t)(i % half) + (47u << 23)) | (i >= half ? 0x80000000u : 0u);
        const float a = __uint_as_float(bits);
        for (int j = 0; j < nk; j++) {
            if (dev::div_by(a, d[j], r[j]) != __fdiv_rn(a, d[j])) {
                mine++;
                atomicCAS(first, 0xFFFFFFFFu, bits);
            }
        }
    }
    if (mine) atomicAdd(bad, mine);
}

}  // namespace
}  // namespace ajib

static int selftest_division(const float *k, int nk, int direct, unsigned long long *mismatches,
                             unsigned int *first_bits)
{
    if (!k || nk < 1 || nk > 8 || !mismatches || !first_bits) return AJIB_ERR_ARGS;
    float *dk = nullptr;
    unsigned long long *dbad = nullptr;
    unsigned int *dfirst = nullptr;
    cudaError_t e = cudaMalloc(&dk, 8 * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&dbad, sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMalloc(&dfirst, sizeof(unsigned int));
    if (e == cudaSuccess) e = cudaMemcpy(dk, k, nk * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(dbad, 0, sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMemset(dfirst, 0xFF, sizeof(unsigned int));
    if (e == cudaSuccess) {
        ajib::k_div_check<<<148 * 8, 256>>>(dk, nk, direct, dbad, dfirst);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(mismatches, dbad, sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(first_bits, dfirst, sizeof(unsigned int), cudaMemcpyDeviceToHost);
    cudaFree(dk);
    cudaFree(dbad);
    cudaFree(dfirst);
    return e == cudaSuccess ? AJIB_OK : AJIB_ERR_CUDA;
}

extern "C" int ajib_selftest_division(const float *k, int nk, unsigned long long *mismatches, unsigned int *first_bits)
{
    return selftest_division(k, nk, 0, mismatches, first_bits);
}

extern "C" int ajib_selftest_division_by(const float *d, int nd, unsigned long long *mismatches, unsigned int *first_bits)
{
    return selftest_division(d, nd, 1, mismatches, first_bits);
}
