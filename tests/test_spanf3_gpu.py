"""GPU parity of SPANF3's two kernel features against the CPU oracle (oracle/oracle_conv.c, the
reference's sanity/native_ref.h semantics; the oracle itself is pinned to the reference's own CPU
net by tests/test_cpu_golden.py): the tanh 1x1 gate, (x + o) * tanh(att_bias + W_att^T o) with
the attention conv as a second tensor-core GEMM in the epilogue, and the model input
pixel-unshuffled by 2 as the first conv's input. Then whole SPANF3 nets (the shipping
AnimeJaNai V3.1 HD structure: b5f48 and b8f64) on the executor and through the video ABI.

Tolerances as for the other conv kernels: max-abs 2e-2 and RMS 3e-3 per kernel; nets max-abs
2e-2 (relative to the output's peak where it exceeds 1) and PSNR >= 50 dB. The random nets use
weights at 0.7 of He init, which keeps their outputs near [0, 1] and the comparison
well-conditioned (at full He init, 8 blocks of 64 channels turn a one-ulp input change into an
output change of tens)."""
import os
import tempfile

import numpy as np
import pytest

from oracle_net import run_plan
from test_conv_gpu import check_close, dev_f16, dev_rows, run_conv
from util import conv_weights, f16r, oracle_conv, oracle_post, oracle_pre, psnr, to_f16_bits, yuv420_frame

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def att_weights(rng, c):
    """The 1x1 attention conv: [1][c][c] fp16-valued, bias N(0, 0.01)."""
    w = f16r(rng.normal(0.0, np.sqrt(2.0 / c), size=(1, c, c)))
    return w, rng.normal(0.0, 0.01, size=c).astype(np.float32)


@pytest.mark.parametrize("H,W", [(19, 37), (9, 200), (4, 300), (1, 5)])
@pytest.mark.parametrize("c", [16, 32, 48, 64])
def test_tanh_gate(H, W, c):
    import ajib
    rng = np.random.default_rng(300 + c + H)
    x = f16r(rng.uniform(-1, 1, size=(H, W, c)))
    r = f16r(rng.uniform(-1, 1, size=(H, W, c)))
    w, b, _ = conv_weights(rng, c, c)
    aw, ab = att_weights(rng, c)
    want = oracle_conv(x, 0, H, W, c, w, b, None, c, gate=2, resid=r, att=(aw, ab))
    wt = ajib.Weights(to_f16_bits(w), b)
    at = ajib.Weights(to_f16_bits(aw), ab, taps=1)
    got = run_conv(ajib.conv_op(wt, gate=ajib.GATE_TANH1X1, att=at), dev_rows(x), dev_rows(r), (H, W, c), H, W)
    check_close(got, want)


def test_tanh_gate_row_bands():
    """Row ranges launched one after another give the whole-frame result exactly."""
    import ajib
    rng = np.random.default_rng(41)
    H, W, c = 23, 140, 48
    x, r = dev_rows(f16r(rng.uniform(-1, 1, size=(H, W, c)))), dev_rows(f16r(rng.uniform(-1, 1, size=(H, W, c))))
    w, b, _ = conv_weights(rng, c, c)
    aw, ab = att_weights(rng, c)
    op = ajib.conv_op(ajib.Weights(to_f16_bits(w), b), gate=ajib.GATE_TANH1X1, att=ajib.Weights(to_f16_bits(aw), ab, taps=1))
    whole = run_conv(op, x, r, (H, W, c), H, W)
    bands = run_conv(op, x, r, (H, W, c), H, W, rows=[(0, 7), (7, 8), (8, 23)])
    assert np.array_equal(whole, bands)


@pytest.mark.parametrize("H,W", [(19, 37), (8, 130), (1, 3)])
@pytest.mark.parametrize("cout,act", [(48, 0), (64, 1), (32, 2), (16, 0)])
@pytest.mark.parametrize("norm", [False, True])
def test_head_unshuffle(H, W, cout, act, norm):
    """The first conv of an unshuffled model: the input [3][2H][2W] read as 12 channels at H x W."""
    import ajib
    rng = np.random.default_rng(500 + H + cout + act + norm)
    x = f16r(rng.uniform(0, 1, size=(3, 2 * H, 2 * W)))
    w, b, s = conv_weights(rng, 12, cout, prelu=act == 2)
    mean, scale = (0.4488, 0.4371, 0.4040), (1.7, 1.1, 0.9)
    xin = x
    if norm:
        xin = f16r((x - np.asarray(mean, np.float32)[:, None, None]) * np.asarray(scale, np.float32)[:, None, None])
    want = oracle_conv(xin, 2, H, W, 12, w, b, s, cout, act=act)
    wt = ajib.Weights(to_f16_bits(w), b, s)
    op = ajib.conv_op(wt, in_=ajib.IN_NCHW3_UNSHUFFLE2, act=act, in_norm=(mean, scale) if norm else None)
    got = run_conv(op, dev_f16(x), None, (H, W, cout), H, W)
    check_close(got, want)


@pytest.mark.parametrize("H,W", [(7, 37), (5, 140)])
def test_unshuffle_to_depth_to_space(H, W):
    """One conv from the unshuffled input straight to depth-to-space 4 (a 2x model of one conv)."""
    import ajib
    rng = np.random.default_rng(61 + H)
    x = f16r(rng.uniform(0, 1, size=(3, 2 * H, 2 * W)))
    w, b, _ = conv_weights(rng, 12, 48)
    want = oracle_conv(x, 2, H, W, 12, w, b, None, 48, R=4)
    op = ajib.conv_op(ajib.Weights(to_f16_bits(w), b), in_=ajib.IN_NCHW3_UNSHUFFLE2, out=ajib.OUT_D2S4)
    got = run_conv(op, dev_f16(x), None, (3, 4 * H, 4 * W), H, W)
    check_close(got, want)


def test_refusals():
    import ajib
    rng = np.random.default_rng(3)
    w, b, _ = conv_weights(rng, 48, 48)
    wt = ajib.Weights(to_f16_bits(w), b)
    assert not ajib.supported(ajib.conv_op(wt, gate=ajib.GATE_TANH1X1))[0]  # no attention weights
    aw, ab = att_weights(rng, 32)
    bad = ajib.conv_op(wt, gate=ajib.GATE_TANH1X1, att=ajib.Weights(to_f16_bits(aw), ab, taps=1))
    ok, why = ajib.supported(bad)
    assert not ok and "attention" in why
    w12, b12, _ = conv_weights(rng, 3, 48)
    ok, why = ajib.supported(ajib.conv_op(ajib.Weights(to_f16_bits(w12), b12), in_=ajib.IN_NCHW3_UNSHUFFLE2))
    assert not ok and "12 channels" in why


def run_exec(plan, x, bands=1):
    import ajib
    _, h, w = x.shape
    m = ajib.Model(plan)
    assert m.scale == 2
    ex = ajib.Exec(m, w, h, bands=bands)
    src = torch.from_numpy(x.astype(np.float16)).cuda()
    dst = torch.empty((3, 2 * h, 2 * w), dtype=torch.float16, device="cuda")
    assert ex.run(src.data_ptr(), dst.data_ptr(), 0) == 0
    torch.cuda.synchronize()
    assert ajib.kernel_status() == 0
    return dst.float().cpu().numpy()


def check_net(got, want):
    assert np.isfinite(got).all()
    peak = max(1.0, float(np.abs(want).max()))
    err = np.abs(got - want).max() / peak
    assert err <= 2e-2, f"max abs {err} of peak {peak}"
    assert psnr(got / peak, want / peak) >= 50.0


@pytest.mark.parametrize("c,blocks,h,w", [(48, 5, 48, 300), (64, 8, 30, 96), (16, 2, 10, 22)])
def test_spanf3_net(c, blocks, h, w):
    import ajib
    plan = ajib.spanf3_plan(70 + c, c=c, blocks=blocks, gain=0.7)
    x = f16r(np.random.default_rng(c).uniform(0, 1, size=(3, h, w)))
    check_net(run_exec(plan, x), run_plan(plan, x))


def test_spanf3_bands_bit_identical():
    import ajib
    plan = ajib.spanf3_plan(71, c=48, blocks=2, gain=0.7)
    x = f16r(np.random.default_rng(8).uniform(0, 1, size=(3, 64, 140)))
    assert np.array_equal(run_exec(plan, x, bands=1), run_exec(plan, x, bands=3))


def test_spanf3_odd_size_refused():
    import ajib
    m = ajib.Model(ajib.spanf3_plan(72, c=16, blocks=1))
    with pytest.raises(ajib.AjibError) as e:
        ajib.Exec(m, 31, 20)
    assert "even" in str(e.value)


def test_video_spanf3():
    """aji_infer with an unshuffled 2x model: P010 in, P010 out at twice the size, against the
    oracle's pre -> net -> post."""
    import ajib
    w, h = 128, 72
    plan = ajib.spanf3_plan(73, c=48, blocks=2, gain=0.7)
    d = tempfile.mkdtemp()
    path = os.path.join(d, "spanf3.ajnm")
    with open(path, "wb") as f:
        f.write(ajib.model_bytes(plan))
    vid = ajib.Video(path, w, h)
    ow, oh = vid.configure(w, h)
    assert (ow, oh) == (2 * w, 2 * h)
    rng = np.random.default_rng(9)
    y, uv = yuv420_frame(rng, w, h, 2, lo=64, hi=940)
    dy = torch.from_numpy(y.view(np.int16)).cuda()
    duv = torch.from_numpy(uv.view(np.int16)).cuda()
    oy = torch.empty((oh, ow), dtype=torch.int16, device="cuda")
    ouv = torch.empty((oh // 2, ow), dtype=torch.int16, device="cuda")
    fin = ajib.frame(w, h, ajib.FMT_P010, [dy.data_ptr(), duv.data_ptr()], [w * 2, w * 2])
    fout = ajib.frame(ow, oh, ajib.FMT_P010, [oy.data_ptr(), ouv.data_ptr()], [ow * 2, ow * 2])
    assert vid.infer(fin, fout, 0) == 0, vid.error()
    t = vid.flush(0)
    assert t > 0 and vid.wait(t) == 0
    rgb = oracle_pre(2, y, uv, 2, 1, 1).view(np.float16).astype(np.float32)
    net = run_plan(plan, rgb)
    wy, wuv = oracle_post(2, net.astype(np.float16).view(np.uint16), 2, 1, 1)
    gy = oy.cpu().numpy().view(np.uint16) >> 6
    guv = ouv.cpu().numpy().view(np.uint16) >> 6
    assert np.abs(gy.astype(int) - (wy >> 6).astype(int)).max() <= 3
    assert np.abs(guv.astype(int) - (wuv >> 6).astype(int)).max() <= 3
    vid.close()


def test_image_spanf3_against_oracle():
    """aji_img_upscale with an unshuffled 2x model: even tiles of the model input, 2x output."""
    import ctypes as C

    import ajib
    from util import oracle_upscale_tiled
    plan = ajib.spanf3_plan(74, c=48, blocks=2, gain=0.7)
    d = tempfile.mkdtemp()
    path = os.path.join(d, "spanf3.ajnm")
    with open(path, "wb") as f:
        f.write(ajib.model_bytes(plan))
    ctx = ajib.Image()
    m = ctx.load(path, tile=64, overlap=16)
    info = ajib.ImgModelInfo()
    assert ajib.lib.aji_img_model_info_get(m, C.byref(info)) == 0 and info.scale == 2
    W, H = 150, 100
    img = np.random.default_rng(W).integers(0, 256, size=(H, W, 3)).astype(np.uint8)
    rc, got = ctx.upscale(m, img, 2)
    assert rc == 0, ctx.error()
    want = oracle_upscale_tiled(lambda x: run_plan(plan, x.astype(np.float16).astype(np.float32)), 64, 64, 2, 16, img)
    diff = np.abs(got.astype(int) - want.astype(int))
    assert diff.max() <= 3, diff.max()
    ajib.lib.aji_img_release(C.byref(m))
    # an odd tile size cannot be unshuffled
    with pytest.raises(ajib.AjibError) as e:
        ctx.load(path, tile=63, overlap=16)
    assert "even" in str(e.value)
    ctx.close()
