"""GPU: parity at the BASELINE configs' own sizes, through the engine's C ABIs.

- Config 1: one 1920x1080 P010 frame through aji_infer with the full 16-body Compact 2x.
- Config 2: one 2048x2048 8-bit RGB image through aji_img_upscale with SuperUltraCompact 4x,
  tiles of 512 with 16 px overlap (25 tiles).
- Config 3: SPAN 48x6 2x at 1920x1080.
- Config 4: two Compact nets chained by an animejanai.conf, 960x540 -> 1920x1080 -> 3840x2160.

Each network output is checked three ways:
- the whole frame against a plain PyTorch fp32 reference of the plan (tests/torch_ref.py);
- windows of rows (top, middle across CTA-run seams and accumulator ring wraps, bottom) against the
  C oracle (sanity/native_ref.h:run_plan semantics), run on the input rows the window's receptive
  field reaches. The windows span the full width, so every strip seam is inside them;
- the P010 video output, bit for bit, against the oracle's post pass applied to the executor's own
  fp16 output. The pre and post passes are bit-exact, so this pins aji_infer's colour passes and
  chaining at full size.

Tolerances are the north_star's: max-abs 2e-2 on a [0,1] scale and PSNR >= 50 dB for network
outputs; P010 within that tolerance in 10-bit codes (18) with a mean under one code and
PSNR >= 50 dB against the oracle's own chain; bytes within 3 codes for the 8-bit image.
Depth-to-space indexing is pinned bit for bit by one-hot weights, against the reference's own
k_conv3x3 recompiled for sm_100a (oracle/_ref)."""
import ctypes as C
import os
import tempfile

import numpy as np
import pytest

from oracle_net import run_plan
from synth import p010_frame, rgb8_image
from torch_ref import run_plan_torch
from util import ROOT, f16r, oracle_post, oracle_pre, oracle_upscale_tiled, psnr, to_rows

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

P010, BT709, LIMITED, LEFT = 2, 2, 1, 1
REF_CONV = os.path.join(ROOT, "oracle", "_ref", "libref_conv.so")


def _model_file(plan, d=None, name="m.ajnm"):
    import ajib
    d = d or tempfile.mkdtemp()
    path = os.path.join(d, name)
    with open(path, "wb") as f:
        f.write(ajib.model_bytes(plan))
    return path


def receptive_radius(plan):
    """An upper bound on how many input rows away an output row can depend: one per 3x3 step."""
    return sum(1 for s in plan["steps"] if np.asarray(s["w"]).shape[0] == 9)


def exec_gpu(plan, x):
    """The plan on the executor (ajib_exec_run): x NCHW fp16-valued [3][h][w] (numpy or a CUDA
    tensor) -> the fp16 output as a CUDA tensor."""
    import ajib
    xt = x if isinstance(x, torch.Tensor) else torch.from_numpy(np.asarray(x, np.float32))
    xt = xt.cuda().half().contiguous()
    _, h, w = xt.shape
    m = ajib.Model(plan)
    ex = ajib.Exec(m, w, h)
    R = m.scale
    out = torch.empty((3, R * h, R * w), dtype=torch.float16, device="cuda")
    assert ex.run(xt.data_ptr(), out.data_ptr(), 0) == 0
    torch.cuda.synchronize()
    assert ajib.kernel_status() == 0
    return out


def check_net(got, want, what):
    """got, want: tensors (same device) of fp16-valued outputs on a [0,1] scale."""
    got, want = got.float(), want.float()
    assert torch.isfinite(got).all(), what
    err = float((got - want).abs().max())
    mse = float(((got.double() - want.double()) ** 2).mean())
    p = float("inf") if mse == 0 else 10.0 * np.log10(1.0 / mse)
    assert err <= 2e-2, f"{what}: max abs {err}"
    assert p >= 50.0, f"{what}: psnr {p}"
    return err, p


def check_windows(plan, x, got, windows):
    """Rows [a, b) of the conv-resolution output of `plan` on x (NCHW numpy) against the C oracle
    run on input rows [a - r, b + r) (clipped to the frame), r = the receptive radius; got: the
    engine's whole output (CUDA tensor)."""
    _, H, W = x.shape
    R = got.shape[1] // H
    r = receptive_radius(plan)
    for a, b in windows:
        c0, c1 = max(0, a - r), min(H, b + r)
        want = run_plan(plan, np.ascontiguousarray(x[:, c0:c1]))
        g = got[:, R * a:R * b].float().cpu().numpy()
        wnt = want[:, R * (a - c0):R * (b - c0)]
        err = np.abs(g - wnt).max()
        assert err <= 2e-2, f"rows {a}..{b}: max abs {err}"
        assert psnr(g, wnt) >= 50.0, f"rows {a}..{b}: psnr {psnr(g, wnt)}"


def infer_p010(vid, w, h, ow, oh, y, uv):
    """aji_infer on one P010 frame in device memory; returns the P010 output planes (uint16)."""
    import ajib
    dy = torch.from_numpy(y.view(np.int16)).cuda()
    duv = torch.from_numpy(uv.view(np.int16)).cuda()
    oy = torch.empty((oh, ow), dtype=torch.int16, device="cuda")
    ouv = torch.empty((oh // 2, ow), dtype=torch.int16, device="cuda")
    fin = ajib.frame(w, h, ajib.FMT_P010, [dy.data_ptr(), duv.data_ptr()], [w * 2, w * 2])
    fout = ajib.frame(ow, oh, ajib.FMT_P010, [oy.data_ptr(), ouv.data_ptr()], [ow * 2, ow * 2])
    assert vid.infer(fin, fout, 0) == 0, vid.error()
    t = vid.flush(0)
    assert t > 0 and vid.wait(t) == 0, vid.error()
    return oy.cpu().numpy().view(np.uint16), ouv.cpu().numpy().view(np.uint16)


# The network tolerance (max-abs 2e-2 on [0, 1]) in 10-bit limited-range codes (876 levels).
P010_MAX_CODES = 18


def check_p010(gy, guv, net_out, ref_out):
    """The video output against (1) the oracle's post pass on the engine's own net output, bit for
    bit, and (2) the oracle's post pass on the fp32 reference's output, within the network's
    tolerance carried into codes (max 18, PSNR >= 50 dB) and a mean under one code."""
    bits = net_out.cpu().numpy().view(np.uint16)
    wy, wuv = oracle_post(P010, bits, BT709, LIMITED, LEFT)
    assert np.array_equal(gy, wy), "luma differs from the post pass of the net output"
    assert np.array_equal(guv, wuv), "chroma differs from the post pass of the net output"
    ry, ruv = oracle_post(P010, ref_out.half().cpu().numpy().view(np.uint16), BT709, LIMITED, LEFT)
    for g, r in ((gy, ry), (guv, ruv)):
        d = np.abs((g >> 6).astype(int) - (r >> 6).astype(int))
        assert d.max() <= P010_MAX_CODES, d.max()
        assert d.mean() < 1.0, d.mean()
        assert psnr((g >> 6) / 1023.0, (r >> 6) / 1023.0) >= 50.0


def test_config1_compact_1080p_p010():
    """BASELINE config 1 at full size: bench.py's model (seed 1) and a 1080p value-noise frame."""
    import ajib
    plan = ajib.compact_plan(1)
    w, h = 1920, 1080
    y, uv = p010_frame(11, w, h)
    vid = ajib.Video(_model_file(plan), w, h)
    ow, oh = vid.configure(w, h)
    assert (ow, oh) == (2 * w, 2 * h)
    gy, guv = infer_p010(vid, w, h, ow, oh, y, uv)
    vid.close()
    x = oracle_pre(P010, y, uv, BT709, LIMITED, LEFT).view(np.float16).astype(np.float32)
    net = exec_gpu(plan, x)
    ref = run_plan_torch(plan, x)
    check_net(net, ref, "Compact 1080p whole frame")
    check_windows(plan, x, net, [(0, 16), (536, 568), (1064, 1080)])
    check_p010(gy, guv, net, ref)


def test_config3_span_1080p():
    """BASELINE config 3's net (SPAN 48 features x 6 blocks) at 1920x1080."""
    import ajib
    plan = ajib.span_plan(1, c=48, blocks=6)
    y, uv = p010_frame(12)
    x = oracle_pre(P010, y, uv, BT709, LIMITED, LEFT).view(np.float16).astype(np.float32)
    net = exec_gpu(plan, x)
    check_net(net, run_plan_torch(plan, x), "SPAN 1080p whole frame")
    check_windows(plan, x, net, [(0, 12), (530, 546), (1068, 1080)])


def test_config3_spanf3_1080p():
    """The shipping SPANF3 structure (pixel-unshuffled input, tanh gates) at 1920x1080."""
    import ajib
    plan = ajib.spanf3_plan(1, c=48, blocks=5, gain=0.7)
    y, uv = p010_frame(13)
    x = oracle_pre(P010, y, uv, BT709, LIMITED, LEFT).view(np.float16).astype(np.float32)
    net = exec_gpu(plan, x)
    check_net(net, run_plan_torch(plan, x), "SPANF3 1080p whole frame")
    # windows in conv-resolution rows (the unshuffled input is 540 rows high)
    u = plan["unshuffle"]
    r = receptive_radius(plan)
    for a, b in [(0, 8), (266, 276), (532, 540)]:
        c0, c1 = max(0, a - r), min(540, b + r)
        want = run_plan(plan, np.ascontiguousarray(x[:, u * c0:u * c1]))
        R = plan["depth_to_space"]
        g = net[:, R * a:R * b].float().cpu().numpy()
        wnt = want[:, R * (a - c0):R * (b - c0)]
        assert np.abs(g - wnt).max() <= 2e-2 and psnr(g, wnt) >= 50.0, (a, b)


def test_config4_chain_960x540():
    """two Compact nets (seeds 1 and 2, as bench.py) chained through an
    animejanai.conf, 960x540 P010 -> 3840x2160 P010. Each net is checked on the input the engine
    gave it, so a tolerance-sized difference in the first does not compound into the second."""
    import ajib
    plans = [ajib.compact_plan(1), ajib.compact_plan(2)]
    d = tempfile.mkdtemp()
    for k, pl in enumerate(plans):
        _model_file(pl, d, f"m{k + 1}.ajnm")
    conf = os.path.join(d, "animejanai.conf")
    with open(conf, "w") as f:
        f.write("[global]\nlogging=no\n\n[slot_1]\nprofile_name=t\nchain_1_model_1_name=m1\nchain_1_model_2_name=m2\n")
    vid = ajib.Video.from_conf(conf, d, slot=1)
    w, h = 960, 540
    ow, oh = vid.configure(w, h)
    assert (ow, oh) == (4 * w, 4 * h), vid.log()
    y, uv = p010_frame(14, w, h)
    gy, guv = infer_p010(vid, w, h, ow, oh, y, uv)
    vid.close()
    x = oracle_pre(P010, y, uv, BT709, LIMITED, LEFT).view(np.float16).astype(np.float32)
    mid = exec_gpu(plans[0], x)
    ref_mid = run_plan_torch(plans[0], x)
    check_net(mid, ref_mid, "chain net 1 (960x540)")
    check_windows(plans[0], x, mid, [(0, 10), (264, 276), (530, 540)])
    out = exec_gpu(plans[1], mid)
    ref = run_plan_torch(plans[1], mid.float())
    check_net(out, ref, "chain net 2 (1920x1080)")
    check_windows(plans[1], mid.float().cpu().numpy(), out, [(540, 556)])
    # the video output is the post pass of exactly these two nets
    check_p010(gy, guv, out, run_plan_torch(plans[1], ref_mid))


def test_config2_suc_2048_tiled():
    """a 2048x2048 8-bit RGB image, SuperUltraCompact 4x (24 x 8), tiles 512
    with 16 px overlap, through aji_img_upscale, against the oracle tiler driving the oracle net."""
    import ajib
    plan = ajib.compact_plan(21, c=24, body=8, scale=4)
    ctx = ajib.Image()
    m = ctx.load(_model_file(plan), tile=512, overlap=16)
    img = rgb8_image(31)
    rc, got = ctx.upscale(m, img, 4)
    assert rc == 0, ctx.error()
    ajib.lib.aji_img_release(C.byref(m))
    ctx.close()
    assert got.shape == (8192, 8192, 3)
    want = oracle_upscale_tiled(lambda t: run_plan(plan, t.astype(np.float16).astype(np.float32)), 512, 512, 4, 16,
                                img)
    d = np.abs(got.astype(np.int16) - want.astype(np.int16))
    assert d.max() <= 3, d.max()
    assert psnr(got / 255.0, want / 255.0) >= 50.0


def _ref_conv_lib():
    ref = C.CDLL(REF_CONV)
    ref.ref_conv_upload.restype = C.c_void_p
    ref.ref_conv_upload.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int]
    ref.ref_conv_launch.argtypes = [C.c_void_p] + [C.c_int] * 6 + [C.c_void_p] * 3 + [C.c_int] * 3 + [C.c_void_p]
    ref.ref_conv_release.argtypes = [C.c_void_p]
    return ref


@pytest.mark.parametrize("R,cin,H,W,clamp", [(2, 64, 37, 150, False), (2, 64, 64, 256, True), (4, 24, 33, 200, False),
                                             (4, 24, 40, 128, True)])
def test_depth_to_space_index_bit_exact(R, cin, H, W, clamp):
    """Pixel-shuffle indexing, bit for bit: one-hot weights (each output channel = one input
    channel at the centre tap + another at the right tap) on inputs that are multiples of 1/256,
    so every value is exact in fp16 and fp32. The output [c][R*y+ry][R*x+rx] is channel
    c*R*R + ry*R + rx plus the nearest model-input skip, against the host permutation and the
    reference's own k_conv3x3 (conv_kernels.cuh:315-346) on the B200."""
    import ajib
    from util import to_f16_bits
    rng = np.random.default_rng(R * 100 + H)
    cout = 3 * R * R
    a = rng.integers(0, cin, size=cout)
    b = rng.integers(0, cin, size=cout)
    w = np.zeros((9, cin, cout), np.float32)
    w[4, a, np.arange(cout)] = 1.0   # centre tap
    w[5, b, np.arange(cout)] = 1.0   # right tap (x + 1)
    bias = np.zeros(cout, np.float32)
    x = rng.integers(0, 256, size=(H, W, cin)).astype(np.float32) / 256.0
    skip = rng.integers(0, 256, size=(3, H, W)).astype(np.float32) / 256.0
    # the host's answer
    xr = np.concatenate([x[:, 1:], np.zeros((H, 1, cin), np.float32)], axis=1)
    conv = x[:, :, a] + xr[:, :, b]                       # [H][W][cout]
    want = np.zeros((3, R * H, R * W), np.float32)
    for n in range(cout):
        c3, ry, rx = n // (R * R), (n // R) % R, n % R
        want[c3, ry::R, rx::R] = conv[:, :, n] + skip[c3]
    if clamp:
        want = np.clip(want, 0.0, 1.0)
    want = want.astype(np.float16)
    # this engine
    wt = ajib.Weights(to_f16_bits(w), bias, None)
    op = ajib.conv_op(wt, out={2: ajib.OUT_D2S2, 4: ajib.OUT_D2S4}[R], out_clamp=clamp)
    src = torch.from_numpy(to_rows(x).astype(np.float16)).cuda()
    dskip = torch.from_numpy(skip.astype(np.float16)).cuda()
    dst = torch.zeros((3, R * H, R * W), dtype=torch.float16, device="cuda")
    assert ajib.conv3x3(op, src.data_ptr(), dskip.data_ptr(), dst.data_ptr(), H, W, 0, 0, 0) == 0
    torch.cuda.synchronize()
    assert ajib.kernel_status() == 0
    got = dst.cpu().numpy()
    assert np.array_equal(got.view(np.uint16), want.view(np.uint16))
    # the reference's kernel (no clamp option in its launch: compare the unclamped case)
    if not clamp and os.path.exists(REF_CONV):
        ref = _ref_conv_lib()
        wbits = to_f16_bits(w)  # kept alive while the library reads it
        hw = ref.ref_conv_upload(wbits.ctypes.data, bias.ctypes.data, None, cin, cin, cout, (cout + 15) // 16 * 16)
        assert hw
        rsrc = torch.from_numpy(x.astype(np.float16)).cuda()
        rdst = torch.zeros_like(dst)
        rc = ref.ref_conv_launch(hw, 0, 0, 0, {2: 1, 4: 2}[R], cin, cout, rsrc.data_ptr(), dskip.data_ptr(),
                                 rdst.data_ptr(), H, W, -1, None)
        torch.cuda.synchronize()
        ref.ref_conv_release(hw)
        assert rc == 0, "the reference kernel refused the op"
        assert torch.equal(rdst.view(torch.int16), dst.view(torch.int16))
