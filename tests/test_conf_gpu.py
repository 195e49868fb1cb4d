"""GPU: conf mode (animejanai.conf chains of native model files) and aji_resize_frame.

A chain runs its steps in order on the stream: the pre-pass at the input size, each model (with a
Spline36 resize before it when the chain asks for one) at the size the previous step produced,
the post-pass at the chain's output size (src/aji_trt.cpp:1407-1455 for the chain's sizes). The
oracle runs the same steps on the CPU: oracle pre-pass, oracle resize, the plan oracle per model,
oracle post-pass; the nets' fp16 tolerance can move a quantised sample by a level or two."""
import ctypes as C
import os
import tempfile

import numpy as np
import pytest

from oracle_net import run_plan
from util import oracle_post, oracle_pre, oracle_resize, psnr, yuv420_frame

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def model_dir(plans):
    import ajib
    d = tempfile.mkdtemp()
    for name, plan in plans.items():
        with open(os.path.join(d, name + ".ajnm"), "wb") as f:
            f.write(ajib.model_bytes(plan))
    return d


def write_conf(d, text):
    path = os.path.join(d, "animejanai.conf")
    with open(path, "w") as f:
        f.write(text)
    return path


CONF = """[global]
logging=yes

[slot_1]
profile_name=Chains
chain_1_max_resolution=100x70
chain_1_model_1_name=m1
chain_1_model_2_name=m2
chain_2_min_resolution=100x70
chain_2_model_1_resize_factor_before_upscale=50
chain_2_model_1_name=m1

[slot_2]
profile_name=Missing
chain_1_model_1_name=not_there
"""


def run_frame(vid, w, h, ow, oh, seed):
    import ajib
    rng = np.random.default_rng(seed)
    y, uv = yuv420_frame(rng, w, h, 2, lo=64, hi=940)
    dy, duv = torch.from_numpy(y.view(np.int16)).cuda(), torch.from_numpy(uv.view(np.int16)).cuda()
    oy = torch.empty((oh, ow), dtype=torch.int16, device="cuda")
    ouv = torch.empty((oh // 2, ow), dtype=torch.int16, device="cuda")
    fin = ajib.frame(w, h, ajib.FMT_P010, [dy.data_ptr(), duv.data_ptr()], [w * 2, w * 2])
    fout = ajib.frame(ow, oh, ajib.FMT_P010, [oy.data_ptr(), ouv.data_ptr()], [ow * 2, ow * 2])
    assert vid.infer(fin, fout, 0) == 0, vid.error()
    t = vid.flush(0)
    assert t > 0 and vid.wait(t) == 0
    return y, uv, oy.cpu().numpy().view(np.uint16) >> 6, ouv.cpu().numpy().view(np.uint16) >> 6


def check_yuv(gy, guv, wy, wuv):
    assert np.abs(gy.astype(int) - (wy >> 6).astype(int)).max() <= 3
    assert np.abs(guv.astype(int) - (wuv >> 6).astype(int)).max() <= 3
    assert psnr(gy / 1023.0, (wy >> 6) / 1023.0) >= 50.0


def f16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def test_two_model_chain():
    """BASELINE config 4's structure (two 2x Compact nets in a chain), at a small size."""
    import ajib
    m1, m2 = ajib.compact_plan(31, body=2), ajib.compact_plan(32, body=2)
    d = model_dir({"m1": m1, "m2": m2})
    vid = ajib.Video.from_conf(write_conf(d, CONF), slot=1)
    w, h = 80, 48
    ow, oh = vid.configure(w, h)
    assert (ow, oh) == (4 * w, 4 * h)
    assert "Applied Model: m1" in vid.log() and "Applied Model: m2" in vid.log()
    y, uv, gy, guv = run_frame(vid, w, h, ow, oh, 1)
    rgb = oracle_pre(2, y, uv, 2, 1, 1).view(np.float16).astype(np.float32)
    net = run_plan(m2, f16(run_plan(m1, rgb)))
    wy, wuv = oracle_post(2, net.astype(np.float16).view(np.uint16), 2, 1, 1)
    check_yuv(gy, guv, wy, wuv)
    vid.close()


def test_resize_before_upscale():
    import ajib
    m1 = ajib.compact_plan(33, body=2)
    d = model_dir({"m1": m1, "m2": ajib.compact_plan(34, body=1)})
    vid = ajib.Video.from_conf(write_conf(d, CONF), slot=1)
    w, h = 120, 72  # beyond chain 1's window: chain 2, resize to 50 % then m1
    ow, oh = vid.configure(w, h)
    assert (ow, oh) == (w, h)
    assert "Resize Factor Before Upscale: 50%" in vid.log()
    y, uv, gy, guv = run_frame(vid, w, h, ow, oh, 2)
    rgb = oracle_pre(2, y, uv, 2, 1, 1)
    small = oracle_resize(rgb, w, h, w // 2, h // 2).view(np.float16).astype(np.float32)
    net = run_plan(m1, small)
    wy, wuv = oracle_post(2, net.astype(np.float16).view(np.uint16), 2, 1, 1)
    check_yuv(gy, guv, wy, wuv)
    vid.close()


def test_missing_model_is_passthrough():
    import ajib
    d = model_dir({})
    vid = ajib.Video.from_conf(write_conf(d, CONF), slot=2)
    ow, oh = vid.configure(64, 48, allow_passthrough=True)
    assert (ow, oh) == (64, 48)
    assert "model not found" in vid.log()
    vid.close()


@pytest.mark.parametrize("w,h,ow,oh", [(96, 64, 50, 40), (64, 48, 130, 96)])
def test_resize_frame(w, h, ow, oh):
    """aji_resize_frame: P010 -> fp16 RGB -> Spline36 -> P010, bit-exact with the oracle's steps."""
    import ajib
    m1 = ajib.compact_plan(35, body=1)
    d = model_dir({"m1": m1})
    vid = ajib.Video.from_conf(write_conf(d, CONF), slot=1)
    rng = np.random.default_rng(w + ow)
    y, uv = yuv420_frame(rng, w, h, 2, lo=64, hi=940)
    dy, duv = torch.from_numpy(y.view(np.int16)).cuda(), torch.from_numpy(uv.view(np.int16)).cuda()
    oy = torch.empty((oh, ow), dtype=torch.int16, device="cuda")
    ouv = torch.empty((oh // 2, ow), dtype=torch.int16, device="cuda")
    fin = ajib.frame(w, h, ajib.FMT_P010, [dy.data_ptr(), duv.data_ptr()], [w * 2, w * 2])
    fout = ajib.frame(ow, oh, ajib.FMT_P010, [oy.data_ptr(), ouv.data_ptr()], [ow * 2, ow * 2])
    for _ in range(2):  # the second call reuses the plans and buffers of the first
        assert vid.resize_frame(fin, fout, 0) == 0, vid.error()
        torch.cuda.synchronize()
    rgb = oracle_pre(2, y, uv, 2, 1, 1)
    wy, wuv = oracle_post(2, oracle_resize(rgb, w, h, ow, oh), 2, 1, 1)
    assert np.array_equal(oy.cpu().numpy().view(np.uint16), wy)
    assert np.array_equal(ouv.cpu().numpy().view(np.uint16), wuv)
    vid.close()


def test_onnx_models_run_like_their_native_files():
    """An ONNX model (lowered when loaded) gives the same bytes as the native file of the same plan:
    video conf mode looking up <name>.onnx, and the image ABI loading the .onnx path."""
    import sys
    sys.path.insert(0, os.path.dirname(__file__))
    from onnx_writer import export
    import ajib
    m1 = ajib.compact_plan(36, body=2)
    d_native = model_dir({"m1": m1, "m2": ajib.compact_plan(37, body=1)})
    d_onnx = tempfile.mkdtemp()
    with open(os.path.join(d_onnx, "m1.onnx"), "wb") as f:
        f.write(export(m1))
    conf = CONF.replace("chain_1_model_2_name=m2\n", "")
    outs = []
    for d in (d_native, d_onnx):
        vid = ajib.Video.from_conf(write_conf(d, conf), slot=1)
        w, h = 80, 48
        ow, oh = vid.configure(w, h)
        assert (ow, oh) == (2 * w, 2 * h), vid.log()
        outs.append(run_frame(vid, w, h, ow, oh, 3)[2:])
        vid.close()
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])
    # the image ABI on the .onnx file
    img = np.random.default_rng(9).integers(0, 256, size=(70, 90, 3)).astype(np.uint8)
    res = []
    for path in (os.path.join(d_native, "m1.ajnm"), os.path.join(d_onnx, "m1.onnx")):
        ctx = ajib.Image()
        m = ctx.load(path, tile=48, overlap=8)
        rc, out = ctx.upscale(m, img, 2)
        assert rc == 0, ctx.error()
        ajib.lib.aji_img_release(C.byref(m))
        ctx.close()
        res.append(out)
    assert np.array_equal(res[0], res[1])
