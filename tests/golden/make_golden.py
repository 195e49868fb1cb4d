"""Generates the golden vectors in this directory from the reference's own code, compiled from its
sources into oracle/_ref by oracle/ref/build.sh (so this runs where the reference tree is
present; the vectors are committed and the CPU tests need only them):

  conv_plans.npz   outputs of the reference's CPU reference net (sanity/native_ref.h:run_plan)
                   for small seeded plans of each family: Compact 2x, SuperUltraCompact 4x, SPAN 2x
                   (gates, SiLU, concat), SPANF3 2x (pixel-unshuffled input, tanh 1x1 gates,
                   ReLU, depth-to-space 4). Inputs and weights are regenerated from the seeds.
  resample.npz     the reference's zimg filter tables (src/resample.h:compute) for the chroma
                   passes of the BASELINE sizes and every siting, and aji_csp constants
                   (src/resample.h:make_csp) for every format / matrix / range.
  tiling.npz       the reference's tiler (src/core/tiling.cpp): tile origins, even origins, blend
                   weights, and upscale_tiled outputs with the reference test's mock models
                   (sanity/tiling_test.cpp: Nearest replication, Constant 0.6).

  python tests/golden/make_golden.py
"""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.path.join(ROOT, "oracle", "_ref")
sys.path.insert(0, os.path.join(ROOT, "animejanai-inference_b200"))
sys.path.insert(0, os.path.dirname(HERE))

# (name, builder kwargs, seed, h, w)
PLANS = [
    ("compact", dict(kind="compact", c=64, body=3, scale=2), 101, 12, 20),
    ("suc", dict(kind="compact", c=24, body=2, scale=4), 102, 9, 14),
    ("span", dict(kind="span", c=48, blocks=2, scale=2), 103, 10, 16),
    ("spanf3", dict(kind="spanf3", c=48, blocks=2), 104, 12, 20),
]
RESAMPLE = [  # (src, dst, siting, up)
    (960, 1920, 1, 1), (540, 1080, 1, 1), (960, 1920, 2, 1), (540, 1080, 3, 1), (31, 62, 1, 1),
    (3840, 1920, 1, 0), (2160, 1080, 1, 0), (3840, 1920, 2, 0), (2160, 1080, 3, 0), (62, 31, 1, 0),
]
TILE_AXES = [(2048, 512, 16), (2048, 512, 128), (100, 32, 8), (500, 512, 16), (1000, 300, 40), (33, 32, 4)]
TILED = [  # (kind, w, h, ch, tile, overlap, scale)
    (0, 100, 70, 3, 32, 8, 2), (0, 45, 61, 1, 16, 4, 4), (1, 50, 40, 3, 24, 6, 2), (0, 20, 10, 3, 32, 8, 2),
]


def plan_for(spec, seed):
    import ajib
    if spec["kind"] == "compact":
        return ajib.compact_plan(seed, c=spec["c"], body=spec["body"], scale=spec["scale"])
    if spec["kind"] == "spanf3":
        return ajib.spanf3_plan(seed, c=spec["c"], blocks=spec["blocks"])
    return ajib.span_plan(seed, c=spec["c"], blocks=spec["blocks"], scale=spec["scale"])


def plan_input(seed, h, w):
    return np.random.default_rng(seed).uniform(0, 1, size=(3, h, w)).astype(np.float16).astype(np.float32)


def main():
    import refnet
    out = {}
    for name, spec, seed, h, w in PLANS:
        plan = plan_for(spec, seed)
        x = plan_input(seed + 1, h, w)
        out[name] = refnet.run_plan(os.path.join(REF, "libref_net.so"), plan, x).astype(np.float16)
    np.savez_compressed(os.path.join(HERE, "conv_plans.npz"), **out)

    rs = C.CDLL(os.path.join(REF, "libref_resample.so"))
    rs.ref_filter.argtypes = [C.c_int, C.c_int, C.c_double, C.c_int, C.c_void_p, C.c_void_p]
    rs.ref_filter.restype = C.c_int
    rs.ref_chroma_shifts.argtypes = [C.c_int, C.c_int, C.POINTER(C.c_double), C.POINTER(C.c_double)]
    rs.ref_make_csp.argtypes = [C.c_int, C.c_int, C.c_int, C.c_void_p]
    res = {}
    for i, (src, dst, siting, up) in enumerate(RESAMPLE):
        sx, sy = C.c_double(), C.c_double()
        rs.ref_chroma_shifts(siting, up, C.byref(sx), C.byref(sy))
        shift = sx.value if src in (960, 3840, 31, 62) and dst in (1920, 62, 31) else sy.value
        taps = rs.ref_filter(src, dst, shift, 0, None, None)
        start = np.zeros(dst, np.int32)
        wt = np.zeros(dst * taps, np.float32)
        rs.ref_filter(src, dst, shift, 0, start.ctypes.data, wt.ctypes.data)
        res[f"r{i}_start"], res[f"r{i}_wt"], res[f"r{i}_shift"] = start, wt.reshape(dst, taps), np.float64(shift)
        res[f"r{i}_shifts"] = np.array([sx.value, sy.value])
    csps = []
    for fmt in (1, 2, 3, 5, 6):
        for mat in (1, 2, 3):
            for rg in (1, 2):
                c = np.zeros(6, np.float32)
                rs.ref_make_csp(fmt, mat, rg, c.ctypes.data)
                csps.append([fmt, mat, rg, *c.tolist()])
    res["csp"] = np.array(csps, np.float64)
    np.savez_compressed(os.path.join(HERE, "resample.npz"), **res)

    tl = C.CDLL(os.path.join(REF, "libref_tiling.so"))
    tl.ref_tile_origins.argtypes = [C.c_int] * 3 + [C.c_void_p, C.c_int]
    tl.ref_even_origins.argtypes = [C.c_int] * 3 + [C.c_void_p, C.c_void_p, C.c_int]
    tl.ref_axis_weights.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]
    tl.ref_reflect.argtypes = [C.c_int, C.c_int]
    tl.ref_upscale_tiled.argtypes = [C.c_int, C.c_float, C.c_void_p, C.c_void_p] + [C.c_int] * 4 + \
        [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]
    tg = {}
    for i, (n, tile, ov) in enumerate(TILE_AXES):
        o = np.zeros(256, np.int32)
        k = tl.ref_tile_origins(n, tile, ov, o.ctypes.data, 256)
        tg[f"a{i}_origins"] = o[:k].copy()
        for s in (1, 2, 4):
            span = min(tile, n)
            wbuf = np.zeros(k * span * s, np.float32)
            tl.ref_axis_weights(o.ctypes.data, k, n, tile, s, wbuf.ctypes.data)
            tg[f"a{i}_w{s}"] = wbuf.reshape(k, span * s)
        t = C.c_int()
        e = np.zeros(256, np.int32)
        k2 = tl.ref_even_origins(n, tile, ov, C.byref(t), e.ctypes.data, 256)
        tg[f"a{i}_even"] = e[:k2].copy()
        tg[f"a{i}_even_tile"] = np.int32(t.value)
    tg["reflect"] = np.array([[i, n, tl.ref_reflect(i, n)] for n in (1, 2, 5) for i in range(-12, 13)], np.int32)
    for i, (kind, w, h, ch, tile, ov, s) in enumerate(TILED):
        img = np.random.default_rng(500 + i).integers(0, 256, size=(h, w, ch)).astype(np.uint8)
        o = np.zeros((h * s, w * s, ch), np.uint8)
        rc = tl.ref_upscale_tiled(kind, C.c_float(0.6), None, None, tile, tile, s, ov, img.ctypes.data, w, h, ch,
                                  o.ctypes.data)
        assert rc == 0
        tg[f"t{i}_in"], tg[f"t{i}_out"] = img, o
    np.savez_compressed(os.path.join(HERE, "tiling.npz"), **tg)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
