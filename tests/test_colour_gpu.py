"""GPU: the colour passes (aji_run_pre / aji_run_post / 4:4:4) against the CPU oracle, bit for bit
(0 mismatches, the reference's own criterion for its fused pre-pass: sanity/pre_fusion.cu:71-99),
over formats, matrices, ranges, sitings and ragged sizes; and, when the reference's kernels were
built into oracle/_ref, against those kernels run on the same GPU."""
import ctypes as C
import os

import numpy as np
import pytest

from util import ROOT, oracle_csp, oracle_post, oracle_pre, yuv420_frame

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

REF_KERNELS = os.path.join(ROOT, "oracle", "_ref", "libref_kernels.so")

CASES = [(2, 2, 1, 1, 1920, 1080), (1, 2, 1, 1, 1280, 720), (2, 1, 2, 2, 130, 66), (1, 3, 1, 3, 62, 46),
         (2, 3, 2, 3, 258, 34), (1, 1, 2, 1, 6, 4), (2, 2, 1, 2, 2, 2)]


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16 if a.dtype == np.uint16 else np.uint8)).cuda()


def gpu_pre(fmt, y, uv, matrix, rng_, siting, filt=0, kernel=None):
    """The pre pass on the GPU; `kernel` the form the plan must choose (ajib_plan_kernel: 1
    streaming, 0 tiled; None: either)."""
    import ajib
    h, w = y.shape
    p = ajib.lib.aji_pre_plan_create(fmt, w, h, siting, filt)
    assert p
    if kernel is not None:
        assert ajib.lib.ajib_plan_kernel(p) == kernel
    dy, duv = dev(y), dev(uv)
    out = torch.empty((3, h, w), dtype=torch.float16, device="cuda")
    csp = ajib.lib.aji_make_csp(fmt, matrix, rng_)
    rc = ajib.lib.aji_run_pre(p, dy.data_ptr(), y.strides[0], duv.data_ptr(), uv.strides[0], C.byref(csp),
                              out.data_ptr(), None)
    torch.cuda.synchronize()
    ajib.lib.aji_plan_destroy(p)
    assert rc == 0
    return out.cpu().numpy().view(np.uint16)


def gpu_post(fmt, rgb_bits, matrix, rng_, siting=1, filt=0, pad=0, kernel=None):
    """The post pass on the GPU; `pad` extra elements per output row (a strided frame), `kernel` the
    form the plan must choose (ajib_plan_kernel: 1 streaming, 0 tiled; None: either)."""
    import ajib
    _, h, w = rgb_bits.shape
    p = ajib.lib.aji_post_plan_create(fmt, w, h, siting, filt)
    assert p
    if kernel is not None:
        assert ajib.lib.ajib_plan_kernel(p) == kernel
    src = torch.from_numpy(rgb_bits.view(np.float16)).cuda()
    dt = torch.int16 if fmt == 2 else torch.uint8
    # guard values around the planes: nothing outside the frame may be written
    oy = torch.full((h, w + pad), 0x5A5A if fmt == 2 else 0x5A, dtype=torch.int32, device="cuda").to(dt)
    ouv = torch.full((h // 2, w + pad), 0x5A5A if fmt == 2 else 0x5A, dtype=torch.int32, device="cuda").to(dt)
    es = 2 if fmt == 2 else 1
    csp = ajib.lib.aji_make_csp(fmt, matrix, rng_)
    rc = ajib.lib.aji_run_post(p, src.data_ptr(), C.byref(csp), oy.data_ptr(), (w + pad) * es, ouv.data_ptr(),
                               (w + pad) * es, None)
    torch.cuda.synchronize()
    ajib.lib.aji_plan_destroy(p)
    assert rc == 0
    npdt = np.uint16 if fmt == 2 else np.uint8
    y, uv = oy.cpu().numpy().view(npdt), ouv.cpu().numpy().view(npdt)
    if pad:
        guard = 0x5A5A if fmt == 2 else 0x5A
        assert (y[:, w:] == guard).all() and (uv[:, w:] == guard).all(), "stores past the frame's width"
    return y[:, :w], uv[:, :w]


@pytest.mark.parametrize("fmt,matrix,rng_,siting,w,h", CASES)
def test_pre_bit_exact(fmt, matrix, rng_, siting, w, h):
    rng = np.random.default_rng(w * 7 + h + fmt)
    y, uv = yuv420_frame(rng, w, h, fmt)
    want = oracle_pre(fmt, y, uv, matrix, rng_, siting)
    got = gpu_pre(fmt, y, uv, matrix, rng_, siting)
    assert np.array_equal(got, want), f"{int((got != want).sum())} mismatches"


@pytest.mark.parametrize("fmt,matrix,rng_,siting,w,h", CASES)
def test_post_bit_exact(fmt, matrix, rng_, siting, w, h):
    rng = np.random.default_rng(w * 3 + h + fmt)
    rgb = rng.uniform(-0.1, 1.1, size=(3, h, w)).astype(np.float16).view(np.uint16)
    wy, wuv = oracle_post(fmt, rgb, matrix, rng_, siting)
    gy, guv = gpu_post(fmt, rgb, matrix, rng_, siting)
    assert np.array_equal(gy, wy), f"luma: {int((gy != wy).sum())} mismatches"
    assert np.array_equal(guv, wuv), f"chroma: {int((guv != wuv).sum())} mismatches"


# the streaming pre kernel (k_pre_roll): config 1's frame, config 4's (a partial last strip), every
# siting, both formats, bilinear tables (2 taps), a two-row frame and a single-strip frame
STREAM_PRE_CASES = [(2, 2, 1, 1, 0, 1920, 1080), (1, 1, 2, 2, 0, 1280, 720), (2, 3, 2, 3, 0, 960, 540),
                    (1, 2, 1, 1, 1, 272, 18), (2, 1, 2, 2, 1, 144, 36), (2, 2, 1, 1, 0, 16, 2), (1, 3, 1, 3, 0, 48, 10)]


@pytest.mark.parametrize("fmt,matrix,rng_,siting,filt,w,h", STREAM_PRE_CASES)
def test_pre_streaming_bit_exact(fmt, matrix, rng_, siting, filt, w, h):
    rng = np.random.default_rng(w * 11 + h + fmt + filt)
    y, uv = yuv420_frame(rng, w, h, fmt)
    want = oracle_pre(fmt, y, uv, matrix, rng_, siting, filt)
    got = gpu_pre(fmt, y, uv, matrix, rng_, siting, filt, kernel=1)
    assert np.array_equal(got, want), f"{int((got != want).sum())} mismatches"


# the streaming post kernel (k_post_roll): the config-1 4K output, partial strips, one-step runs,
# every siting and matrix, both formats, bilinear tables (4 taps), strided outputs
STREAM_CASES = [(2, 2, 1, 1, 0, 3840, 2160, 0), (1, 1, 2, 2, 0, 136, 72, 0), (2, 3, 2, 3, 0, 264, 40, 0),
                (2, 2, 1, 1, 0, 1928, 16, 24), (1, 2, 1, 1, 0, 1280, 720, 8), (2, 1, 1, 2, 1, 520, 100, 0),
                (1, 3, 2, 3, 1, 136, 18, 16), (2, 2, 2, 1, 0, 3848, 2, 0)]


@pytest.mark.parametrize("fmt,matrix,rng_,siting,filt,w,h,pad", STREAM_CASES)
def test_post_streaming_bit_exact(fmt, matrix, rng_, siting, filt, w, h, pad):
    rng = np.random.default_rng(w * 5 + h + fmt + filt)
    rgb = rng.uniform(-0.1, 1.1, size=(3, h, w)).astype(np.float16).view(np.uint16)
    wy, wuv = oracle_post(fmt, rgb, matrix, rng_, siting, filt)
    gy, guv = gpu_post(fmt, rgb, matrix, rng_, siting, filt, pad=pad, kernel=1)
    assert np.array_equal(gy, wy), f"luma: {int((gy != wy).sum())} mismatches"
    assert np.array_equal(guv, wuv), f"chroma: {int((guv != wuv).sum())} mismatches"


@pytest.mark.parametrize("fmt", [3, 5, 6])
def test_444_bit_exact(fmt):
    import ajib
    rng = np.random.default_rng(fmt)
    h, w = 37, 53
    rgb = rng.uniform(-0.1, 1.1, size=(3, h, w)).astype(np.float16).view(np.uint16)
    o = __import__("util")._colour_sigs()
    csp_o = oracle_csp(fmt, 2, 1)
    wy, wcb, wcr = (np.zeros((h, w), np.uint16) for _ in range(3))
    o.orc_post444(fmt, w, h, rgb.ctypes.data, csp_o, wy.ctypes.data, wcb.ctypes.data, wcr.ctypes.data)
    src = torch.from_numpy(rgb.view(np.float16)).cuda()
    planes = [torch.empty((h, w), dtype=torch.int16, device="cuda") for _ in range(3)]
    csp = ajib.lib.aji_make_csp(fmt, 2, 1)
    rc = ajib.lib.aji_run_post444(fmt, w, h, src.data_ptr(), C.byref(csp), planes[0].data_ptr(), w * 2,
                                  planes[1].data_ptr(), w * 2, planes[2].data_ptr(), w * 2, None)
    assert rc == 0
    torch.cuda.synchronize()
    got = [p.cpu().numpy().view(np.uint16) for p in planes]
    for g, want in zip(got, (wy, wcb, wcr)):
        assert np.array_equal(g, want)
    # and back: 4:4:4 -> RGB
    want_rgb = np.zeros((3, h, w), np.uint16)
    o.orc_pre444(w, h, wy.ctypes.data, wcb.ctypes.data, wcr.ctypes.data, csp_o, want_rgb.ctypes.data)
    out = torch.empty((3, h, w), dtype=torch.float16, device="cuda")
    rc = ajib.lib.aji_run_pre444(w, h, planes[0].data_ptr(), w * 2, planes[1].data_ptr(), w * 2, planes[2].data_ptr(),
                                 w * 2, C.byref(csp), out.data_ptr(), None)
    assert rc == 0
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint16), want_rgb)


@pytest.mark.skipif(not os.path.exists(REF_KERNELS), reason="reference kernels not built (oracle/_ref)")
@pytest.mark.parametrize("fmt,matrix,rng_,siting,w,h", CASES[:5])
def test_against_reference_kernels(fmt, matrix, rng_, siting, w, h):
    """The reference's own src/kernels.cu, compiled for sm_100a, on the same inputs: 0 mismatches."""
    import ajib
    ref = C.CDLL(REF_KERNELS)
    ref.aji_pre_plan_create.restype = C.c_void_p
    ref.aji_post_plan_create.restype = C.c_void_p
    ref.aji_pre_plan_create.argtypes = [C.c_int] * 5
    ref.aji_post_plan_create.argtypes = [C.c_int] * 5
    ref.aji_run_pre.argtypes = [C.c_void_p, C.c_void_p, C.c_ssize_t, C.c_void_p, C.c_ssize_t, C.c_void_p, C.c_void_p,
                                C.c_void_p]
    ref.aji_run_post.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_ssize_t, C.c_void_p, C.c_ssize_t,
                                 C.c_void_p]
    ref.aji_plan_destroy.argtypes = [C.c_void_p]
    rng = np.random.default_rng(w + h)
    y, uv = yuv420_frame(rng, w, h, fmt)
    csp = ajib.lib.aji_make_csp(fmt, matrix, rng_)
    # pre
    p = ref.aji_pre_plan_create(fmt, w, h, siting, 0)
    dy, duv = dev(y), dev(uv)
    out = torch.empty((3, h, w), dtype=torch.float16, device="cuda")
    assert ref.aji_run_pre(p, dy.data_ptr(), y.strides[0], duv.data_ptr(), uv.strides[0], C.addressof(csp),
                           out.data_ptr(), None) == 0
    torch.cuda.synchronize()
    ref.aji_plan_destroy(p)
    want = out.cpu().numpy().view(np.uint16)
    got = gpu_pre(fmt, y, uv, matrix, rng_, siting)
    assert np.array_equal(got, want), f"pre: {int((got != want).sum())} mismatches vs the reference kernels"
    # post
    rgb = want
    p = ref.aji_post_plan_create(fmt, w, h, siting, 0)
    src = torch.from_numpy(rgb.view(np.float16)).cuda()
    dt = torch.int16 if fmt == 2 else torch.uint8
    es = 2 if fmt == 2 else 1
    oy = torch.empty((h, w), dtype=dt, device="cuda")
    ouv = torch.empty((h // 2, w), dtype=dt, device="cuda")
    assert ref.aji_run_post(p, src.data_ptr(), C.addressof(csp), oy.data_ptr(), w * es, ouv.data_ptr(), w * es,
                            None) == 0
    torch.cuda.synchronize()
    ref.aji_plan_destroy(p)
    npdt = np.uint16 if fmt == 2 else np.uint8
    gy, guv = gpu_post(fmt, rgb, matrix, rng_, siting)
    assert np.array_equal(gy, oy.cpu().numpy().view(npdt))
    assert np.array_equal(guv, ouv.cpu().numpy().view(npdt))


RESIZE_CASES = [(64, 36, 96, 54), (97, 41, 50, 80), (40, 30, 40, 30), (128, 72, 32, 18), (33, 17, 131, 70)]


def _resize_oracle(src_bits, sw, sh, dw, dh):
    from util import oracle
    o = oracle()
    o.orc_resize.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]
    out = np.zeros((3, dh, dw), np.uint16)
    assert o.orc_resize(np.ascontiguousarray(src_bits).ctypes.data, sw, sh, dw, dh, out.ctypes.data) == 0
    return out


def _resize_ours(src_bits, sw, sh, dw, dh):
    import ajib
    ajib.lib.aji_resize_plan_create.restype = C.c_void_p
    ajib.lib.aji_resize_plan_create.argtypes = [C.c_int] * 4
    ajib.lib.aji_run_resize.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    p = ajib.lib.aji_resize_plan_create(sw, sh, dw, dh)
    assert p
    src = torch.from_numpy(src_bits.view(np.int16)).cuda()
    out = torch.empty((3, dh, dw), dtype=torch.int16, device="cuda")
    assert ajib.lib.aji_run_resize(C.c_void_p(p), C.c_void_p(src.data_ptr()), C.c_void_p(out.data_ptr()), None) == 0
    torch.cuda.synchronize()
    ajib.lib.aji_plan_destroy(C.c_void_p(p))
    return out.cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("sw,sh,dw,dh", RESIZE_CASES)
def test_resize_spline36_against_oracle(sw, sh, dw, dh):
    rng = np.random.default_rng(sw * dh)
    src = rng.uniform(-0.1, 1.1, size=(3, sh, sw)).astype(np.float16).view(np.uint16)
    assert np.array_equal(_resize_ours(src, sw, sh, dw, dh), _resize_oracle(src, sw, sh, dw, dh))


@pytest.mark.skipif(not os.path.exists(REF_KERNELS), reason="reference kernels not built (oracle/_ref)")
@pytest.mark.parametrize("sw,sh,dw,dh", RESIZE_CASES)
def test_resize_against_reference_kernels(sw, sh, dw, dh):
    """aji_run_resize against the reference's own k_rs_h + k_rs_v on the B200: the same bits."""
    ref = C.CDLL(REF_KERNELS)
    ref.aji_resize_plan_create.restype = C.c_void_p
    ref.aji_resize_plan_create.argtypes = [C.c_int] * 4
    ref.aji_run_resize.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    ref.aji_plan_destroy.argtypes = [C.c_void_p]
    rng = np.random.default_rng(sw + sh + dw)
    src = rng.uniform(-0.1, 1.1, size=(3, sh, sw)).astype(np.float16).view(np.uint16)
    p = ref.aji_resize_plan_create(sw, sh, dw, dh)
    dsrc = torch.from_numpy(src.view(np.int16)).cuda()
    out = torch.empty((3, dh, dw), dtype=torch.int16, device="cuda")
    assert ref.aji_run_resize(p, dsrc.data_ptr(), out.data_ptr(), None) == 0
    torch.cuda.synchronize()
    ref.aji_plan_destroy(p)
    assert np.array_equal(_resize_ours(src, sw, sh, dw, dh), out.cpu().numpy().view(np.uint16))


def test_pre_division_matches_ieee():
    """The pre pass divides by the colour space's luma and chroma scales with a reciprocal and one
    FMA correction: bit-identical to the IEEE division for every float of magnitude in
    [2^-80, 2^18) (its dividends are zero or in [2^-63, 2^17)), for NV12 and P010 at both ranges."""
    import ctypes as C

    import ajib
    ds = sorted({v for fmt in (1, 2) for rng in (1, 2) for v in
                 (ajib.lib.aji_make_csp(fmt, 2, rng).yscale, ajib.lib.aji_make_csp(fmt, 2, rng).cscale)})
    assert 2 <= len(ds) <= 8
    d = (C.c_float * 8)(*ds)
    bad, first = C.c_ulonglong(), C.c_uint()
    assert ajib.lib.ajib_selftest_division_by(d, len(ds), C.byref(bad), C.byref(first)) == 0
    assert bad.value == 0, f"{bad.value} quotients differ, first dividend bits {first.value:#x}"


def test_post_division_matches_ieee():
    """The post pass divides the colour differences by 2 (1 - kb) and 2 (1 - kr) with a reciprocal
    and one FMA correction (Markstein): bit-identical to the IEEE division for every float the pass
    can divide (2^-80 <= |a| < 2^18; its dividends are zero or in [2^-52, 2^18)), for the BT.601,
    BT.709 and BT.2020 coefficients."""
    import ctypes as C

    import ajib
    ks = []
    for matrix in (1, 2, 3):
        c = ajib.lib.aji_make_csp(2, matrix, 1)
        ks += [c.kb, c.kr]
    k = (C.c_float * 8)(*ks)
    bad, first = C.c_ulonglong(), C.c_uint()
    assert ajib.lib.ajib_selftest_division(k, len(ks), C.byref(bad), C.byref(first)) == 0
    assert bad.value == 0, f"{bad.value} quotients differ, first dividend bits {first.value:#x}"
