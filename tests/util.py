"""Test helpers: the CPU oracle (oracle/liboracle.so) through ctypes, seeded inputs and weights,
and comparison metrics. The oracle is the checker only; the engine under test is libaji.so."""
import ctypes as C
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_PATH = os.path.join(ROOT, "oracle", "liboracle.so")

_orc = None


def oracle():
    global _orc
    if _orc is None:
        if not os.path.exists(ORACLE_PATH):
            raise RuntimeError(f"{ORACLE_PATH} is not built (make -C oracle)")
        o = C.CDLL(ORACLE_PATH)
        fp = C.POINTER(C.c_float)
        o.orc_conv3x3.argtypes = [C.c_int, fp, C.c_int, C.c_int, C.c_int, fp, fp, fp, C.c_int, C.c_int, C.c_int,
                                  fp, C.c_int, fp, C.c_int, fp, C.c_int]
        o.orc_conv3x3.restype = C.c_int
        o.orc_conv3x3_ex.argtypes = [C.c_int, fp, C.c_int, C.c_int, C.c_int, fp, fp, fp, C.c_int, C.c_int, C.c_int,
                                     fp, fp, fp, C.c_int, fp, C.c_int, fp, C.c_int]
        o.orc_conv3x3_ex.restype = C.c_int
        o.orc_concat1x1.argtypes = [C.POINTER(fp), C.c_int, C.c_int, C.c_int, fp, fp, fp, C.c_int]
        o.orc_concat1x1.restype = C.c_int
        o.orc_f2h.argtypes = [C.c_float]
        o.orc_f2h.restype = C.c_uint16
        o.orc_h2f.argtypes = [C.c_uint16]
        o.orc_h2f.restype = C.c_float
        _orc = o
    return _orc


def _fp(a):
    return None if a is None else a.ctypes.data_as(C.POINTER(C.c_float))


def f16r(x):
    """Round to fp16 and back (numpy's conversion is IEEE round-to-nearest-even)."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def oracle_conv(src, in_mode, H, W, cin, w, bias, slope, cout, act=0, gate=0, resid=None, R=0, model_in=None,
                out_clamp=False, nthreads=0, att=None):
    """One fused conv step on the CPU (oracle/oracle_conv.c, sanity/native_ref.h semantics).
    w: [9][cin][cout] fp16-valued float32. in_mode 2: src is the model input [3][2H][2W],
    pixel-unshuffled by 2. att: (w [cout][cout], bias [cout]) of the tanh 1x1 gate (gate 2)."""
    src = np.ascontiguousarray(src, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    slope = None if slope is None else np.ascontiguousarray(slope, dtype=np.float32)
    resid = None if resid is None else np.ascontiguousarray(resid, dtype=np.float32)
    model_in = None if model_in is None else np.ascontiguousarray(model_in, dtype=np.float32)
    aw = ab = None
    if att is not None:
        aw = np.ascontiguousarray(np.asarray(att[0], np.float32).reshape(cout, cout))
        ab = np.ascontiguousarray(att[1], dtype=np.float32)
    if R == 0:
        dst = np.zeros((H, W, cout), np.float32)
    else:
        dst = np.zeros((3, R * H, R * W), np.float32)
    rc = oracle().orc_conv3x3_ex(in_mode, _fp(src), H, W, cin, _fp(w), _fp(bias), _fp(slope), cout, act, gate,
                                 _fp(resid), _fp(aw), _fp(ab), R, _fp(model_in), 1 if out_clamp else 0, _fp(dst),
                                 nthreads)
    assert rc == 0, "oracle rejected the arguments"
    return dst


def oracle_concat(srcs, c, w, bias, nthreads=0):
    srcs = [np.ascontiguousarray(s, dtype=np.float32) for s in srcs]
    npx = srcs[0].size // c
    arr = (C.POINTER(C.c_float) * len(srcs))(*[_fp(s) for s in srcs])
    dst = np.zeros((npx, c), np.float32)
    rc = oracle().orc_concat1x1(arr, len(srcs), npx, c, _fp(np.ascontiguousarray(w, np.float32)),
                                _fp(np.ascontiguousarray(bias, np.float32)), _fp(dst), nthreads)
    assert rc == 0
    return dst


def conv_weights(rng, cin, cout, prelu=False, std=None):
    """He-init 3x3 weights as BASELINE config 0 specifies: W ~ N(0, sqrt(2/(9 cin))) rounded to
    fp16, bias ~ N(0, 0.01), PReLU slopes ~ U[0.1, 0.3]. Returns (w [9][cin][cout] fp16-valued
    float32, bias, slope or None)."""
    std = np.sqrt(2.0 / (9 * cin)) if std is None else std
    w = f16r(rng.normal(0.0, std, size=(9, cin, cout)))
    b = rng.normal(0.0, 0.01, size=cout).astype(np.float32)
    s = rng.uniform(0.1, 0.3, size=cout).astype(np.float32) if prelu else None
    return w, b, s


def to_f16_bits(x):
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def psnr(a, b, peak=1.0):
    mse = float(np.mean((np.asarray(a, np.float64) - np.asarray(b, np.float64)) ** 2))
    return float("inf") if mse == 0 else 10.0 * np.log10(peak * peak / mse)


# ---- colour oracle (oracle/oracle_colour.c) ----
def _colour_sigs():
    o = oracle()
    if getattr(o, "_colour", False):
        return o
    vp, sz = C.c_void_p, C.c_ssize_t
    o.orc_filter.argtypes = [C.c_int, C.c_int, C.c_double, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_float)]
    o.orc_filter.restype = C.c_int
    o.orc_make_csp.argtypes = [C.c_int, C.c_int, C.c_int, C.POINTER(C.c_float)]
    o.orc_make_csp.restype = None
    o.orc_pre.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, vp, sz, vp, sz, C.POINTER(C.c_float), vp]
    o.orc_pre.restype = C.c_int
    o.orc_post.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, vp, C.POINTER(C.c_float), vp, sz, vp, sz]
    o.orc_post.restype = C.c_int
    o.orc_post444.argtypes = [C.c_int, C.c_int, C.c_int, vp, C.POINTER(C.c_float), vp, vp, vp]
    o.orc_post444.restype = C.c_int
    o.orc_pre444.argtypes = [C.c_int, C.c_int, vp, vp, vp, C.POINTER(C.c_float), vp]
    o.orc_pre444.restype = C.c_int
    o._colour = True
    return o


def oracle_csp(fmt, matrix, rng_):
    o = _colour_sigs()
    c = (C.c_float * 6)()
    o.orc_make_csp(fmt, matrix, rng_, c)
    return c


def oracle_filter(src, dst, shift, filt=0):
    o = _colour_sigs()
    taps = o.orc_filter(src, dst, shift, filt, None, None)
    start = np.zeros(dst, np.int32)
    wt = np.zeros(dst * taps, np.float32)
    o.orc_filter(src, dst, shift, filt, start.ctypes.data_as(C.POINTER(C.c_int)), wt.ctypes.data_as(C.POINTER(C.c_float)))
    return taps, start, wt.reshape(dst, taps)


def oracle_pre(fmt, y, uv, matrix, rng_, siting, filt=0):
    """y: [h][w], uv: [h/2][w] interleaved (uint8 NV12 or uint16 P010). Returns fp16 bits [3][h][w]."""
    o = _colour_sigs()
    h, w = y.shape
    y = np.ascontiguousarray(y)
    uv = np.ascontiguousarray(uv)
    dst = np.zeros((3, h, w), np.uint16)
    csp = oracle_csp(fmt, matrix, rng_)
    rc = o.orc_pre(fmt, w, h, siting, filt, y.ctypes.data, y.strides[0], uv.ctypes.data, uv.strides[0], csp,
                   dst.ctypes.data)
    assert rc == 0
    return dst


def oracle_post(fmt, rgb_bits, matrix, rng_, siting=1, filt=0):
    """rgb_bits: fp16 bits [3][h][w]. Returns (y [h][w], uv [h/2][w]) uint8 or uint16."""
    o = _colour_sigs()
    _, h, w = rgb_bits.shape
    dt = np.uint16 if fmt == 2 else np.uint8
    y = np.zeros((h, w), dt)
    uv = np.zeros((h // 2, w), dt)
    src = np.ascontiguousarray(rgb_bits, np.uint16)
    csp = oracle_csp(fmt, matrix, rng_)
    rc = o.orc_post(fmt, w, h, siting, filt, src.ctypes.data, csp, y.ctypes.data, y.strides[0], uv.ctypes.data,
                    uv.strides[0])
    assert rc == 0
    return y, uv


def yuv420_frame(rng, w, h, fmt, lo=None, hi=None):
    """Random 4:2:0 planes: P010 samples are 10 bits in the high bits of 16."""
    if fmt == 2:
        lo = 0 if lo is None else lo
        hi = 1023 if hi is None else hi
        y = (rng.integers(lo, hi + 1, size=(h, w)).astype(np.uint16) << 6)
        uv = (rng.integers(lo, hi + 1, size=(h // 2, w)).astype(np.uint16) << 6)
    else:
        lo = 0 if lo is None else lo
        hi = 255 if hi is None else hi
        y = rng.integers(lo, hi + 1, size=(h, w)).astype(np.uint8)
        uv = rng.integers(lo, hi + 1, size=(h // 2, w)).astype(np.uint8)
    return y, uv


# ---- strip-chunked feature maps (the engine's layout for maps between steps) ----
STRIP_W = 130  # a strip's 128 pixels and a halo column on each side


def feature_strips(W):
    return (W + 127) // 128


def to_rows(x, pad_value=0.0):
    """NHWC [H][W][C] -> strip-chunked [H][S][C/8][130][8]: each strip's halo columns hold the
    neighbouring strips' edge pixels; the image's edge columns (column 0 of strip 0, everything
    past W) hold pad_value."""
    H, W, Cc = x.shape
    KC, S = Cc // 8, feature_strips(W)
    padded = np.full((H, S * 128 + 2, KC, 8), pad_value, dtype=np.float32)
    padded[:, 1:W + 1] = np.asarray(x, np.float32).reshape(H, W, KC, 8)
    out = np.empty((H, S, KC, STRIP_W, 8), np.float32)
    for s in range(S):
        out[:, s] = padded[:, 128 * s:128 * s + STRIP_W].transpose(0, 2, 1, 3)
    return out


def from_rows(buf, H, W, Cc):
    """The pixels of a strip-chunked map, NHWC [H][W][C]."""
    KC, S = Cc // 8, feature_strips(W)
    b = np.asarray(buf).reshape(H, S, KC, STRIP_W, 8)
    full = b[:, :, :, 1:129, :].transpose(0, 1, 3, 2, 4).reshape(H, S * 128, Cc)
    return full[:, :W]


def rows_pad_mask(H, W, Cc):
    """True at the image-edge columns of a strip-chunked map (the kernels never write them)."""
    KC, S = Cc // 8, feature_strips(W)
    m = np.zeros((H, S, KC, STRIP_W, 8), bool)
    m[:, 0, :, 0, :] = True
    for s in range(S):
        for u in range(STRIP_W):
            if 128 * s + u - 1 >= W:
                m[:, s, :, u, :] = True
    return m


def rows_halo_consistent(buf, H, W, Cc):
    """Whether every interior halo column of a strip-chunked map equals the neighbour's edge pixel."""
    KC, S = Cc // 8, feature_strips(W)
    b = np.asarray(buf).reshape(H, S, KC, STRIP_W, 8)
    for s in range(S - 1):
        if 128 * (s + 1) >= W:
            break
        if not (np.array_equal(b[:, s, :, 129], b[:, s + 1, :, 1]) and np.array_equal(b[:, s + 1, :, 0], b[:, s, :, 128])):
            return False
    return True


# ---- tiler oracle (oracle/oracle_tiling.c) ----
TILE_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_float))


def _tiling_sigs():
    o = oracle()
    if getattr(o, "_tiling", False):
        return o
    ip = C.POINTER(C.c_int)
    o.orc_tile_origins.argtypes = [C.c_int, C.c_int, C.c_int, ip, C.c_int]
    o.orc_even_origins.argtypes = [C.c_int, C.c_int, C.c_int, ip, ip, C.c_int]
    o.orc_reflect.argtypes = [C.c_int, C.c_int]
    o.orc_axis_weights.argtypes = [ip, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_float)]
    o.orc_upscale_tiled.argtypes = [TILE_FN, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                    C.c_int, C.c_int, C.c_int, C.c_ssize_t, C.c_void_p, C.c_ssize_t]
    o._tiling = True
    return o


def oracle_origins(n, tile, overlap):
    o = _tiling_sigs()
    buf = (C.c_int * 4096)()
    k = o.orc_tile_origins(n, tile, overlap, buf, 4096)
    return np.array(buf[:k], np.int32)


def oracle_even_origins(n, tile, overlap):
    o = _tiling_sigs()
    buf = (C.c_int * 4096)()
    t = C.c_int()
    k = o.orc_even_origins(n, tile, overlap, C.byref(t), buf, 4096)
    return np.array(buf[:k], np.int32), t.value


def oracle_axis_weights(org, n, tile, scale):
    o = _tiling_sigs()
    org = np.ascontiguousarray(org, np.int32)
    span = min(tile, n)
    w = np.zeros((len(org), span * scale), np.float32)
    o.orc_axis_weights(org.ctypes.data_as(C.POINTER(C.c_int)), len(org), n, tile, scale,
                       w.ctypes.data_as(C.POINTER(C.c_float)))
    return w


def oracle_upscale_tiled(model, tw, th, s, overlap, img, even=False):
    """img: uint8 [h][w][c]; model(in [3][th][tw] float32) -> [3][th*s][tw*s] float32. With even,
    tw / th are the largest tile and the tiles take the even-tile sides."""
    o = _tiling_sigs()
    h, w, c = img.shape
    img = np.ascontiguousarray(img)
    if even:
        tw0, th0 = tw, th
        tw = oracle_even_origins(w, tw0, overlap)[1]
        th = oracle_even_origins(h, th0, overlap)[1]
    out = np.zeros((h * s, w * s, c), np.uint8)

    def run(_, pin, pout):
        x = np.ctypeslib.as_array(pin, shape=(3, th, tw)).copy()
        y = np.asarray(model(x), np.float32).reshape(3 * th * s * tw * s)
        C.memmove(pout, y.ctypes.data, y.nbytes)
        return 0
    cb = TILE_FN(run)
    rc = o.orc_upscale_tiled(cb, None, tw0 if even else tw, th0 if even else th, s, overlap, int(even), img.ctypes.data,
                             w, h, c, w * c, out.ctypes.data, w * s * c)
    assert rc == 0
    return out


def oracle_resize(src_bits, sw, sh, dw, dh):
    """Spline36 resize of fp16 NCHW RGB bits [3][sh][sw] -> [3][dh][dw] (oracle/oracle_colour.c,
    the reference's k_rs_h + k_rs_v)."""
    o = oracle()
    o.orc_resize.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]
    out = np.zeros((3, dh, dw), np.uint16)
    assert o.orc_resize(np.ascontiguousarray(src_bits, dtype=np.uint16).ctypes.data, sw, sh, dw, dh, out.ctypes.data) == 0
    return out
