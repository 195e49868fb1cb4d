"""Seeded synthetic inputs of the BASELINE configs' shapes (no public dataset is involved): P010
frames from smooth value noise spanning 10-bit 64..940 (BT.709 limited range), and uniform 8-bit
RGB noise images. Shared by the tests and bench.py."""
import numpy as np


def value_noise(rng, h, w, lo, hi, cell=32):
    """Seeded smooth value noise in [lo, hi]: random values on a coarse grid, bilinear between."""
    gh, gw = h // cell + 2, w // cell + 2
    g = rng.uniform(lo, hi, size=(gh, gw))
    ys = np.arange(h) / cell
    xs = np.arange(w) / cell
    y0, x0 = np.floor(ys).astype(int), np.floor(xs).astype(int)
    fy, fx = (ys - y0)[:, None], (xs - x0)[None, :]
    a = g[y0][:, x0]
    b = g[y0][:, x0 + 1]
    c = g[y0 + 1][:, x0]
    d = g[y0 + 1][:, x0 + 1]
    return (a * (1 - fy) * (1 - fx) + b * (1 - fy) * fx + c * fy * (1 - fx) + d * fy * fx)


def p010_frame(seed, w=1920, h=1080):
    """One P010 frame: Y [h][w] and interleaved CbCr [h/2][w] (uint16) from smooth value noise
    spanning 64..940 (10-bit), stored in the high bits of 16."""
    rng = np.random.default_rng(seed)
    y = np.rint(value_noise(rng, h, w, 64, 940)).astype(np.uint16) << 6
    u = np.rint(value_noise(rng, h // 2, w // 2, 64, 940)).astype(np.uint16) << 6
    v = np.rint(value_noise(rng, h // 2, w // 2, 64, 940)).astype(np.uint16) << 6
    uv = np.stack([u, v], axis=-1).reshape(h // 2, w)
    # the bilinear blend leaves a Fortran-ordered array: callers hand the planes' memory to the
    # engine, which reads rows
    return np.ascontiguousarray(y), np.ascontiguousarray(uv)


def rgb8_image(seed, w=2048, h=2048):
    """BASELINE config 2's input: one 8-bit RGB image [h][w][3] of uniform seeded noise."""
    return np.random.default_rng(seed).integers(0, 256, size=(h, w, 3)).astype(np.uint8)
