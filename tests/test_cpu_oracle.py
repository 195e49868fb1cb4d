"""CPU: the oracle's own consistency — fp16 conversion against numpy's IEEE conversion, the conv
step against a numpy convolution, the plan runner's shapes."""
import numpy as np

from util import conv_weights, f16r, oracle, oracle_concat, oracle_conv


def test_f2h_matches_numpy_rne():
    o = oracle()
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.normal(0, 100, 5000), rng.normal(0, 1e-5, 2000), [65504, 65520, 65519.9, -7e-8, 6e-8,
                                                                               1e-9, np.inf, -np.inf, 0.0, -0.0]])
    for x in xs.astype(np.float32):
        want = np.float32(x).astype(np.float16).view(np.uint16)
        assert o.orc_f2h(float(x)) == want, x
    for h in range(0, 65536, 7):
        v = np.uint16(h).view(np.float16)
        if np.isnan(v):
            continue
        assert o.orc_h2f(h) == np.float32(v)


def _numpy_conv(x, w, b):
    H, W, _ = x.shape
    xp = np.pad(x.astype(np.float64), ((1, 1), (1, 1), (0, 0)))
    acc = np.zeros((H, W, w.shape[2]))
    for t in range(9):
        dy, dx = divmod(t, 3)
        acc += np.einsum("hwc,cn->hwn", xp[dy:dy + H, dx:dx + W], w[t].astype(np.float64))
    return acc + b


def test_conv_matches_numpy():
    rng = np.random.default_rng(1)
    x = f16r(rng.uniform(-1, 1, size=(9, 13, 16)))
    w, b, s = conv_weights(rng, 16, 24, prelu=True)
    ref = _numpy_conv(x, w, b)
    got = oracle_conv(x, 0, 9, 13, 16, w, b, s, 24, act=2)
    want = f16r(np.where(ref >= 0, ref, ref * s).astype(np.float32))
    assert np.abs(got - want).max() <= 1e-3 * np.abs(want).max()


def test_depth_to_space_ordering():
    """PixelShuffle CRD: channel c*R*R + ry*R + rx -> [c][R*y + ry][R*x + rx] (sanity/native_ref.h:110-115)."""
    rng = np.random.default_rng(2)
    H, W, R = 3, 5, 2
    x = f16r(rng.uniform(-1, 1, size=(H, W, 8)))
    w, b, _ = conv_weights(rng, 8, 12)
    nhwc = oracle_conv(x, 0, H, W, 8, w, b, None, 12)
    d2s = oracle_conv(x, 0, H, W, 8, w, b, None, 12, R=2)
    want = nhwc.reshape(H, W, 3, R, R).transpose(2, 0, 3, 1, 4).reshape(3, H * R, W * R)
    assert np.array_equal(d2s, want)


def test_concat_matches_numpy():
    rng = np.random.default_rng(3)
    srcs = [f16r(rng.uniform(-1, 1, size=(50, 16))) for _ in range(3)]
    w = f16r(rng.normal(0, 0.1, size=(48, 16)))
    b = rng.normal(0, 0.01, size=16).astype(np.float32)
    got = oracle_concat(srcs, 16, w, b)
    want = f16r((np.concatenate(srcs, 1).astype(np.float64) @ w + b).astype(np.float32))
    assert np.abs(got - want).max() <= 1e-3
