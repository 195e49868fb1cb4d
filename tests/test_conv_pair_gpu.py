"""GPU parity of the SM-pair conv kernel (k_conv3x3_pair: one tcgen05 MMA over a cluster of two
CTAs, every staged row a whole three-tap window, ring wraps into spare TMEM slots) against the CPU
oracle, and against the one-SM kernel on the same inputs.

The pair kernel's own edge cases: runs that cross strip boundaries (junk accumulators between
segments), zero rows at image edges, pairs whose runs differ in length (padding rows), frames with
fewer tiles than CTAs (a CTA with no tiles), stacked images, row bands, and every ring position
(two spare slots) over long runs. Tolerances as in test_conv_gpu.py."""
import numpy as np
import pytest

from util import conv_weights, f16r, oracle_conv, to_f16_bits

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from test_conv_gpu import Guarded, check_close, dev_rows, run_conv  # noqa: E402


@pytest.fixture
def pairs():
    """Run with SM pairs on; restore the previous mode afterwards."""
    import ajib
    prev = ajib.pair_mode()
    ajib.pair_mode(1)
    yield ajib
    ajib.pair_mode(prev)


def _op(ajib, rng, c, act=0, gate=0):
    w, b, s = conv_weights(rng, c, c, prelu=act == 2)
    op = ajib.conv_op(ajib.Weights(to_f16_bits(w), b, s if act == 2 else None), act=act,
                      gate={3: ajib.GATE_SIGMOID_HALF, 1: ajib.GATE_RESIDUAL}.get(gate, 0))
    return op, w, b, (s if act == 2 else None)


def test_which_convs_run_on_pairs(pairs):
    ajib = pairs
    rng = np.random.default_rng(1)
    for c, act, gate, want in [(64, 2, 0, True), (48, 3, 0, True), (24, 2, 0, True), (48, 0, 3, True),
                               (24, 0, 1, True), (64, 0, 3, False), (16, 1, 0, False)]:
        op, *_ = _op(ajib, rng, c, act, gate)
        assert ajib.on_pairs(op) == want, (c, act, gate)
        ajib.pair_mode(0)
        assert not ajib.on_pairs(op)
        ajib.pair_mode(1)
    w, b, s = conv_weights(rng, 3, 64, prelu=True)
    head = ajib.conv_op(ajib.Weights(to_f16_bits(w), b, s), in_=ajib.IN_NCHW3, act=ajib.ACT_PRELU)
    assert not ajib.on_pairs(head)
    w, b, _ = conv_weights(rng, 64, 12)
    tail = ajib.conv_op(ajib.Weights(to_f16_bits(w), b), out=ajib.OUT_D2S2)
    assert not ajib.on_pairs(tail)


# (H, W): one tile (one CTA of the pair idle); tiny frames; multi-strip frames whose runs cross
# strip boundaries at many row offsets; a frame with an odd tile count (unequal runs in a pair)
SHAPES = [(1, 5), (2, 3), (19, 37), (7, 300), (130, 129), (61, 520), (300, 400), (33, 1000)]


@pytest.mark.parametrize("H,W", SHAPES)
@pytest.mark.parametrize("c,act,gate", [(64, 2, 0), (48, 3, 0), (24, 2, 0), (48, 0, 3), (24, 0, 1)])
def test_pair_against_oracle_and_single(pairs, H, W, c, act, gate):
    ajib = pairs
    rng = np.random.default_rng(H * 7919 + W * 31 + c + act + 10 * gate)
    x = f16r(rng.uniform(-1, 1, size=(H, W, c)))
    r = f16r(rng.uniform(-1, 1, size=(H, W, c))) if gate else None
    op, w, b, s = _op(ajib, rng, c, act, gate)
    assert ajib.on_pairs(op)
    want = oracle_conv(x, 0, H, W, c, w, b, s, c, act=act, gate=gate, resid=r)
    src, res = dev_rows(x), (dev_rows(r) if gate else None)
    got = run_conv(op, src, res, (H, W, c), H, W)
    check_close(got, want)
    ajib.pair_mode(0)
    single = run_conv(op, src, res, (H, W, c), H, W)
    ajib.pair_mode(1)
    check_close(single, want)
    # the same sums in another fp32 order: outputs agree to about one fp16 rounding
    d = np.abs(got - single)
    assert d.max() <= 8e-3, f"pair vs one-SM max {d.max()}"


@pytest.mark.parametrize("c,act,gate,rpc", [(64, 2, 0, 20), (48, 3, 0, 24), (48, 0, 3, 24), (24, 2, 0, 40)])
def test_pair_long_runs(pairs, c, act, gate, rpc):
    """Each CTA walks rpc rows down one strip: several turns of the ring (6 slots at 64 channels,
    8 at 48, 14 at 32) with every window position, spares included; windows of output rows at the
    top and in the middle against the oracle."""
    ajib = pairs
    rng = np.random.default_rng(900 + c + rpc + gate)
    H, W = 148 * rpc, 128
    x = f16r(rng.uniform(-1, 1, size=(H, W, c)))
    r = f16r(rng.uniform(-1, 1, size=(H, W, c))) if gate else None
    op, w, b, s = _op(ajib, rng, c, act, gate)
    got = run_conv(op, dev_rows(x), dev_rows(r) if gate else None, (H, W, c), H, W)
    for y0, y1 in [(0, 2 * rpc + 6), (H // 2 - 3, H // 2 + rpc + 3), (H - rpc - 5, H)]:
        a0, a1 = max(0, y0 - 1), min(H, y1 + 1)
        want = oracle_conv(x[a0:a1], 0, a1 - a0, W, c, w, b, s, c, act=act, gate=gate,
                           resid=None if r is None else r[a0:a1])
        k0 = y0 - a0
        check_close(got[y0:y1], want[k0:k0 + y1 - y0])


def test_pair_bands_and_stacked_images(pairs):
    """Row bands give the whole-frame result bit for bit; stacked images convolve apart."""
    ajib = pairs
    rng = np.random.default_rng(5)
    H, W, c = 45, 260, 64
    x = f16r(rng.uniform(-1, 1, size=(H, W, c)))
    op, w, b, s = _op(ajib, rng, c, act=2)
    xd = dev_rows(x)
    whole = run_conv(op, xd, None, (H, W, c), H, W)
    bands = run_conv(op, xd, None, (H, W, c), H, W, rows=[(0, 7), (7, 8), (8, 30), (30, 45)])
    assert np.array_equal(whole, bands)
    check_close(whole, oracle_conv(x, 0, H, W, c, w, b, s, c, act=2))

    n, h, W2, c2 = 5, 7, 140, 48
    x2 = f16r(rng.uniform(-1, 1, size=(n * h, W2, c2)))
    op2, w2, b2, _ = _op(ajib, rng, c2, act=3)
    want = np.concatenate([oracle_conv(x2[i * h:(i + 1) * h], 0, h, W2, c2, w2, b2, None, c2, act=3) for i in range(n)])
    s_ = torch.cuda.current_stream().cuda_stream
    src = dev_rows(x2)
    outs = []
    for bl in [[(0, 0)], [(0, 3), (3, 14), (14, 15), (15, n * h)]]:
        dst = Guarded((n * h, W2, c2), nhwc=True)
        for (a, b_) in bl:
            assert ajib.conv3x3_images(op2, src.data_ptr(), 0, dst.ptr, n, h, W2, a, b_, s_) == 0
        torch.cuda.synchronize()
        assert ajib.kernel_status() == 0
        outs.append(dst.value())
    check_close(outs[0], want)
    assert np.array_equal(outs[0], outs[1])


def test_pair_image_height_one(pairs):
    """Images of one row each (every staged window: zero row, the row, zero row)."""
    ajib = pairs
    rng = np.random.default_rng(6)
    n, W, c = 9, 200, 64
    x = f16r(rng.uniform(-1, 1, size=(n, W, c)))
    op, w, b, s = _op(ajib, rng, c, act=2)
    want = np.concatenate([oracle_conv(x[i:i + 1], 0, 1, W, c, w, b, s, c, act=2) for i in range(n)])
    dst = Guarded((n, W, c), nhwc=True)
    assert ajib.conv3x3_images(op, dev_rows(x).data_ptr(), 0, dst.ptr, n, 1, W, 0, 0,
                               torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert ajib.kernel_status() == 0
    check_close(dst.value(), want)
