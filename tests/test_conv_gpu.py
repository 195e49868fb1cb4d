"""GPU parity of the fused 3x3 conv kernels (ajib_conv3x3_launch, the tcgen05 path) against the
CPU oracle (oracle/oracle_conv.c, the reference's sanity/native_ref.h semantics).

Tolerances: the north_star's max-abs 2e-2 on every output, and the reference conv test's RMS
limit 3e-3 (sanity/native_conv_test.cu:195). Guard bands around every output catch writes out of
bounds (the reference's DevBuf pattern, native_conv_test.cu:49-76)."""
import numpy as np
import pytest

from util import (conv_weights, f16r, from_rows, oracle_concat, oracle_conv, rows_halo_consistent, rows_pad_mask,
                  to_f16_bits, to_rows)

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GUARD = 4096
GUARD_BITS = 0x7BAB  # an fp16 pattern no kernel writes


def dev_f16(x):
    """NCHW planes as they are (the model input)."""
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32).astype(np.float16)).cuda()


def dev_rows(x):
    """An NHWC map in the engine's strip-chunked layout (zero image-edge columns)."""
    return torch.from_numpy(to_rows(x).astype(np.float16)).cuda()


class Guarded:
    """A device fp16 buffer with GUARD elements of a fixed pattern on each side. An NHWC shape
    (H, W, C) is allocated strip-chunked, its image-edge columns also holding the pattern: the kernels must
    never write them."""

    def __init__(self, shape, nhwc=False):
        self.nhwc = nhwc
        self.shape = shape
        if nhwc:
            H, W, Cc = shape
            n = H * ((W + 127) // 128) * (Cc // 8) * 130 * 8
        else:
            n = int(np.prod(shape))
        self.n = n
        self.t = torch.full((n + 2 * GUARD,), 0, dtype=torch.int16, device="cuda")
        self.t.fill_(GUARD_BITS)
        self.ptr = self.t.data_ptr() + GUARD * 2

    def value(self):
        h = self.t.cpu().numpy()
        assert (h[:GUARD] == GUARD_BITS).all(), "write before the output"
        assert (h[GUARD + self.n:] == GUARD_BITS).all(), "write past the output"
        body = h[GUARD:GUARD + self.n]
        if not self.nhwc:
            return body.view(np.float16).astype(np.float32).reshape(self.shape)
        H, W, Cc = self.shape
        assert (body[rows_pad_mask(H, W, Cc).ravel()] == GUARD_BITS).all(), "write into an image-edge column"
        assert rows_halo_consistent(body, H, W, Cc), "a strip halo column differs from its neighbour's edge pixel"
        return from_rows(body.view(np.float16).astype(np.float32), H, W, Cc)


def run_conv(op, src, resid, dst_shape, H, W, rows=None):
    import ajib
    dst = Guarded(dst_shape, nhwc=op.out == ajib.OUT_NHWC)
    s = torch.cuda.current_stream().cuda_stream
    if rows is None:
        rc = ajib.conv3x3(op, src.data_ptr(), 0 if resid is None else resid.data_ptr(), dst.ptr, H, W, 0, 0, s)
        assert rc == 0, f"launch failed: {rc}"
    else:
        for (a, b) in rows:
            rc = ajib.conv3x3(op, src.data_ptr(), 0 if resid is None else resid.data_ptr(), dst.ptr, H, W, a, b, s)
            assert rc == 0, f"launch failed: {rc}"
    torch.cuda.synchronize()
    assert ajib.kernel_status() == 0, "a kernel pipeline wait timed out"
    return dst.value()


def check_close(got, want, max_abs=2e-2, rms=3e-3):
    d = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert np.isfinite(got).all()
    assert d.max() <= max_abs, f"max abs {d.max()}"
    assert np.sqrt((d ** 2).mean()) <= rms, f"rms {np.sqrt((d ** 2).mean())}"


def test_config0_conv64_prelu():
    """NCHW 1x64x128x128 U[-1,1], 3x3 64->64, W~N(0,sqrt(2/576)), b~N(0,0.01),
    PReLU slopes U[0.1,0.3]."""
    import ajib
    rng = np.random.default_rng(12345)
    H = W = 128
    x_nchw = f16r(rng.uniform(-1, 1, size=(64, H, W)))
    x = np.ascontiguousarray(x_nchw.transpose(1, 2, 0))
    w, b, s = conv_weights(rng, 64, 64, prelu=True)
    want = oracle_conv(x, 0, H, W, 64, w, b, s, 64, act=2)
    wt = ajib.Weights(to_f16_bits(w), b, s)
    op = ajib.conv_op(wt, act=ajib.ACT_PRELU)
    got = run_conv(op, dev_rows(x), None, (H, W, 64), H, W)
    check_close(got, want)


SHAPES = [(19, 37), (32, 48), (7, 300), (1, 5), (130, 129), (3, 256)]


@pytest.mark.parametrize("H,W", SHAPES)
@pytest.mark.parametrize("c,act", [(64, 2), (48, 3), (24, 2), (32, 1), (64, 0)])
def test_body(H, W, c, act):
    import ajib
    rng = np.random.default_rng(H * 1000 + W + c + act)
    x = f16r(rng.uniform(-1, 1, size=(H, W, c)))
    w, b, s = conv_weights(rng, c, c, prelu=act == 2)
    want = oracle_conv(x, 0, H, W, c, w, b, s, c, act=act)
    wt = ajib.Weights(to_f16_bits(w), b, s)
    got = run_conv(ajib.conv_op(wt, act=act), dev_rows(x), None, (H, W, c), H, W)
    check_close(got, want)


@pytest.mark.parametrize("H,W", [(19, 37), (9, 200)])
@pytest.mark.parametrize("gate", [1, 3])
@pytest.mark.parametrize("c", [48, 24])
def test_gates(H, W, gate, c):
    import ajib
    rng = np.random.default_rng(77 + gate + c + H)
    x = f16r(rng.uniform(-1, 1, size=(H, W, c)))
    r = f16r(rng.uniform(-1, 1, size=(H, W, c)))
    w, b, _ = conv_weights(rng, c, c)
    want = oracle_conv(x, 0, H, W, c, w, b, None, c, gate=gate, resid=r)
    wt = ajib.Weights(to_f16_bits(w), b)
    got = run_conv(ajib.conv_op(wt, gate=gate), dev_rows(x), dev_rows(r), (H, W, c), H, W)
    check_close(got, want)


@pytest.mark.parametrize("H,W", [(19, 37), (16, 130)])
@pytest.mark.parametrize("cout,act", [(64, 2), (48, 0), (24, 2)])
def test_head_nchw3(H, W, cout, act):
    import ajib
    rng = np.random.default_rng(5 + H + cout)
    x = f16r(rng.uniform(0, 1, size=(3, H, W)))
    w, b, s = conv_weights(rng, 3, cout, prelu=act == 2)
    want = oracle_conv(x, 1, H, W, 3, w, b, s, cout, act=act)
    wt = ajib.Weights(to_f16_bits(w), b, s)
    got = run_conv(ajib.conv_op(wt, in_=ajib.IN_NCHW3, act=act), dev_f16(x), None, (H, W, cout), H, W)
    check_close(got, want)


@pytest.mark.parametrize("H,W", [(19, 37), (8, 129)])
@pytest.mark.parametrize("cin,out,cout", [(64, 1, 12), (48, 1, 12), (24, 2, 48), (64, 2, 48), (32, 3, 3), (32, 4, 27)])
@pytest.mark.parametrize("skip", [True, False])
def test_tail_depth_to_space(H, W, cin, out, cout, skip):
    import ajib
    R = ajib.D2S_FACTOR[out]
    rng = np.random.default_rng(9 + H + cin + out)
    x = f16r(rng.uniform(-1, 1, size=(H, W, cin)))
    mi = f16r(rng.uniform(0, 1, size=(3, H, W))) if skip else None
    w, b, _ = conv_weights(rng, cin, cout)
    want = oracle_conv(x, 0, H, W, cin, w, b, None, cout, R=R, model_in=mi)
    wt = ajib.Weights(to_f16_bits(w), b)
    got = run_conv(ajib.conv_op(wt, out=out), dev_rows(x), None if mi is None else dev_f16(mi), (3, R * H, R * W), H, W)
    check_close(got, want)


def test_tail_clamp():
    import ajib
    rng = np.random.default_rng(31)
    H, W = 11, 140
    x = f16r(rng.uniform(-1, 1, size=(H, W, 64)))
    mi = f16r(rng.uniform(0, 1, size=(3, H, W)))
    w, b, _ = conv_weights(rng, 64, 12, std=0.2)
    want = oracle_conv(x, 0, H, W, 64, w, b, None, 12, R=2, model_in=mi, out_clamp=True)
    wt = ajib.Weights(to_f16_bits(w), b)
    got = run_conv(ajib.conv_op(wt, out=ajib.OUT_D2S2, out_clamp=True), dev_rows(x), dev_f16(mi), (3, 2 * H, 2 * W), H, W)
    assert got.min() >= 0 and got.max() <= 1
    check_close(got, want)


# kind, channels in/out, rows per CTA (enough for two turns of the kernel's accumulator ring:
# 8 slots at 64 padded output channels, 6 with the tanh gate, 16 at 32)
LONG = [("body", 64, 64, 20), ("body", 16, 16, 36), ("silu", 48, 48, 20), ("gate", 48, 48, 20), ("att", 48, 48, 16),
        ("head", 3, 64, 20), ("tail", 64, 12, 36), ("tail4", 24, 48, 20)]


@pytest.mark.parametrize("kind,cin,cout,rpc", LONG)
def test_long_segments(kind, cin, cout, rpc):
    """Each CTA walks rpc rows down its strip, so every CTA's accumulator ring turns at least twice
    (frames of 1080p and up give each CTA ~110 rows; the small cases above give it one or two):
    every row position in the ring, its wrap included, against the oracle on windows of output rows
    at the top of the frame and in its middle."""
    import ajib
    rng = np.random.default_rng(600 + cin + cout + rpc)
    H, W = 148 * rpc, 128
    nchw = kind == "head"
    x = f16r(rng.uniform(0 if nchw else -1, 1, size=(3, H, W) if nchw else (H, W, cin)))
    R = {"tail": 2, "tail4": 4}.get(kind, 0)
    act = {"body": 2, "silu": 3, "head": 2}.get(kind, 0)
    gate = {"gate": 3, "att": 2}.get(kind, 0)
    w, b, sl = conv_weights(rng, cin, cout, prelu=act == 2)
    r = f16r(rng.uniform(-1, 1, size=(H, W, cout))) if gate else None
    mi = f16r(rng.uniform(0, 1, size=(3, H, W))) if kind == "tail" else None
    att = None
    kw = {}
    if gate == 2:
        aw = f16r(rng.normal(0.0, np.sqrt(2.0 / cout), size=(1, cout, cout)))
        att = (aw, rng.normal(0.0, 0.01, size=cout).astype(np.float32))
        kw["att"] = ajib.Weights(to_f16_bits(aw), att[1], taps=1)
    out = {2: ajib.OUT_D2S2, 4: ajib.OUT_D2S4}.get(R, ajib.OUT_NHWC)
    op = ajib.conv_op(ajib.Weights(to_f16_bits(w), b, sl if act == 2 else None), in_=ajib.IN_NCHW3 if nchw else ajib.IN_NHWC,
                      act=act, gate={3: ajib.GATE_SIGMOID_HALF, 2: ajib.GATE_TANH1X1}.get(gate, 0), out=out, **kw)
    src = dev_f16(x) if nchw else dev_rows(x)
    resid = dev_rows(r) if gate else (dev_f16(mi) if mi is not None else None)
    got = run_conv(op, src, resid, (3, R * H, R * W) if R else (H, W, cout), H, W)
    for y0, y1 in [(0, 2 * rpc + 6), (H // 2 - 3, H // 2 + rpc + 3)]:
        a0 = max(0, y0 - 1)
        xs = x[:, a0:y1 + 1] if nchw else x[a0:y1 + 1]
        n = (y1 + 1) - a0
        want = oracle_conv(xs, 1 if nchw else 0, n, W, 3 if nchw else cin, w, b, sl if act == 2 else None, cout, act=act,
                           gate=gate, resid=None if r is None else r[a0:y1 + 1], R=R,
                           model_in=None if mi is None else mi[:, a0:y1 + 1], att=att)
        # the window's own edge rows see zero padding in the oracle: compare [y0, y1) only
        k0 = y0 - a0
        if R:
            check_close(got[:, R * y0:R * y1], want[:, R * k0:R * (k0 + y1 - y0)])
        else:
            check_close(got[y0:y1], want[k0:k0 + y1 - y0])


def test_bands_match_whole_frame():
    """Launching a frame as row bands gives exactly the whole-frame result (the band schedule)."""
    import ajib
    rng = np.random.default_rng(4)
    H, W = 45, 260
    x = dev_rows(f16r(rng.uniform(-1, 1, size=(H, W, 64))))
    w, b, s = conv_weights(rng, 64, 64, prelu=True)
    op = ajib.conv_op(ajib.Weights(to_f16_bits(w), b, s), act=ajib.ACT_PRELU)
    whole = run_conv(op, x, None, (H, W, 64), H, W)
    bands = run_conv(op, x, None, (H, W, 64), H, W, rows=[(0, 7), (7, 8), (8, 30), (30, 45)])
    assert np.array_equal(whole, bands)


@pytest.mark.parametrize("kind", ["body", "head", "tail"])
def test_stacked_images(kind):
    """Images stacked along H (the tiler's batches) convolve each on its own: equal to each image
    convolved alone, whole and as row bands that cross image boundaries."""
    import ajib
    rng = np.random.default_rng(8)
    n, h, W, c = 5, 7, 140, 48
    s_ = torch.cuda.current_stream().cuda_stream
    if kind == "head":
        x = f16r(rng.uniform(0, 1, size=(3, n * h, W)))
        w, b, sl = conv_weights(rng, 3, c, prelu=True)
        op = ajib.conv_op(ajib.Weights(to_f16_bits(w), b, sl), in_=ajib.IN_NCHW3, act=ajib.ACT_PRELU)
        src, shape = dev_f16(x), (n * h, W, c)
        want = np.concatenate([oracle_conv(np.ascontiguousarray(x[:, i * h:(i + 1) * h]), 1, h, W, 3, w, b, sl, c,
                                           act=2) for i in range(n)])
    elif kind == "body":
        x = f16r(rng.uniform(-1, 1, size=(n * h, W, c)))
        w, b, sl = conv_weights(rng, c, c, prelu=True)
        op = ajib.conv_op(ajib.Weights(to_f16_bits(w), b, sl), act=ajib.ACT_PRELU)
        src, shape = dev_rows(x), (n * h, W, c)
        want = np.concatenate([oracle_conv(x[i * h:(i + 1) * h], 0, h, W, c, w, b, sl, c, act=2) for i in range(n)])
    else:
        x = f16r(rng.uniform(-1, 1, size=(n * h, W, c)))
        R = 4
        w, b, _ = conv_weights(rng, c, 3 * R * R)
        op = ajib.conv_op(ajib.Weights(to_f16_bits(w), b), out=ajib.OUT_D2S4)
        src, shape = dev_rows(x), (3, R * n * h, R * W)
        want = np.concatenate([oracle_conv(x[i * h:(i + 1) * h], 0, h, W, c, w, b, None, 3 * R * R, R=R)
                               for i in range(n)], axis=1)
    outs = []
    for bands in [[(0, 0)], [(0, 3), (3, 14), (14, 15), (15, n * h)]]:
        dst = Guarded(shape, nhwc=op.out == ajib.OUT_NHWC)
        for (a, b_) in bands:
            assert ajib.conv3x3_images(op, src.data_ptr(), 0, dst.ptr, n, h, W, a, b_, s_) == 0
        torch.cuda.synchronize()
        assert ajib.kernel_status() == 0
        outs.append(dst.value())
    check_close(outs[0], want)
    assert np.array_equal(outs[0], outs[1])


@pytest.mark.parametrize("H,W", [(19, 37), (5, 300), (16, 128)])
@pytest.mark.parametrize("nsrc,c", [(4, 48), (2, 16), (3, 24), (4, 64), (2, 8)])
def test_concat1x1(H, W, nsrc, c):
    """SPAN's concat + 1x1 conv (reference k_concat1x1) against the oracle, whole and as bands."""
    import ajib
    rng = np.random.default_rng(H + W + nsrc + c)
    xs = [f16r(rng.uniform(-1, 1, size=(H, W, c))) for _ in range(nsrc)]
    w = f16r(rng.normal(0.0, np.sqrt(1.0 / (nsrc * c)), size=(nsrc * c, c)))
    b = rng.normal(0.0, 0.01, size=c).astype(np.float32)
    want = oracle_concat([x.reshape(-1, c) for x in xs], c, w, b).reshape(H, W, c)
    wt = ajib.Weights(to_f16_bits(w), b, taps=1)
    srcs = [dev_rows(x) for x in xs]
    s_ = torch.cuda.current_stream().cuda_stream
    outs = []
    for bands in [[(0, 0)], [(0, 2), (2, 3), (3, H)]]:
        dst = Guarded((H, W, c), nhwc=True)
        for (a, b_) in bands:
            if a >= H:
                continue
            assert ajib.concat1x1(wt, [t.data_ptr() for t in srcs], c, dst.ptr, H, W, a, b_, s_) == 0
        torch.cuda.synchronize()
        assert ajib.kernel_status() == 0
        outs.append(dst.value())
    check_close(outs[0], want)
    assert np.array_equal(outs[0], outs[1])


def test_concat1x1_refusals():
    import ajib
    rng = np.random.default_rng(0)
    w = f16r(rng.normal(0.0, 0.1, size=(96, 48)))
    wt = ajib.Weights(to_f16_bits(w), np.zeros(48, np.float32), taps=1)
    x = dev_rows(np.zeros((4, 16, 48), np.float32))
    ptrs = [x.data_ptr(), x.data_ptr()]
    dst = Guarded((4, 16, 48), nhwc=True)
    assert ajib.concat1x1(wt, ptrs, 48, dst.ptr, 4, 16) == 0
    assert ajib.concat1x1(wt, ptrs + [x.data_ptr()], 48, dst.ptr, 4, 16) == ajib.AJIB_ERR_ARGS  # weights for 2 sources
    assert ajib.concat1x1(wt, ptrs, 40, dst.ptr, 4, 16) == ajib.AJIB_ERR_ARGS
    assert ajib.concat1x1(wt, [x.data_ptr() + 2, x.data_ptr()], 48, dst.ptr, 4, 16) == ajib.AJIB_ERR_ARGS  # misaligned
    torch.cuda.synchronize()


def test_refusals():
    import ajib
    rng = np.random.default_rng(0)
    w, b, _ = conv_weights(rng, 64, 64)
    wt = ajib.Weights(to_f16_bits(w), b)
    ok, why = ajib.supported(ajib.conv_op(wt, act=ajib.ACT_PRELU))
    assert not ok and "PReLU" in why
    ok, why = ajib.supported(ajib.conv_op(wt, gate=ajib.GATE_SIGMOID_HALF, act=ajib.ACT_RELU))
    assert not ok and "activation" in why
    ok, why = ajib.supported(ajib.conv_op(wt, out=ajib.OUT_D2S2))
    assert not ok
