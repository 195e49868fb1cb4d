"""GPU: whole nets on the executor (ajib_exec_*) and through the video ABI (aji_infer) against the
CPU oracle's plan runner (sanity/native_ref.h:run_plan semantics). Tolerances from the
north_star: max-abs 2e-2 on a [0,1] scale and PSNR >= 50 dB."""
import os
import tempfile

import numpy as np
import pytest

from oracle_net import run_plan
from util import f16r, oracle_post, oracle_pre, psnr, yuv420_frame

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def run_exec(plan, x, bands=1):
    import ajib
    _, h, w = x.shape
    m = ajib.Model(plan)
    ex = ajib.Exec(m, w, h, bands=bands)
    src = torch.from_numpy(x.astype(np.float16)).cuda()
    R = m.scale
    dst = torch.empty((3, R * h, R * w), dtype=torch.float16, device="cuda")
    assert ex.run(src.data_ptr(), dst.data_ptr(), 0) == 0
    torch.cuda.synchronize()
    assert ajib.kernel_status() == 0
    return dst.float().cpu().numpy()


def check(got, want):
    assert np.isfinite(got).all()
    err = np.abs(got - want).max()
    p = psnr(got, want)
    assert err <= 2e-2, f"max abs {err}"
    assert p >= 50.0, f"psnr {p}"


@pytest.mark.parametrize("h,w", [(24, 40), (37, 150)])
def test_compact_full_depth(h, w):
    import ajib
    plan = ajib.compact_plan(11)
    x = f16r(np.random.default_rng(1).uniform(0, 1, size=(3, h, w)))
    check(run_exec(plan, x), run_plan(plan, x))


def test_compact_bands_bit_identical():
    import ajib
    plan = ajib.compact_plan(12, body=6)
    x = f16r(np.random.default_rng(2).uniform(0, 1, size=(3, 61, 140)))
    a = run_exec(plan, x, bands=1)
    b = run_exec(plan, x, bands=5)
    assert np.array_equal(a, b)


def test_super_ultra_compact_4x():
    import ajib
    plan = ajib.compact_plan(13, c=24, body=8, scale=4)
    x = f16r(np.random.default_rng(3).uniform(0, 1, size=(3, 33, 70)))
    check(run_exec(plan, x), run_plan(plan, x))


@pytest.mark.parametrize("c,blocks,scale", [(48, 6, 2), (16, 2, 4)])
def test_span(c, blocks, scale):
    """SPAN (BASELINE config 3's architecture at 48 channels, 6 blocks): SiLU convs, sigmoid gates,
    the concat + 1x1 conv, depth-to-space."""
    import ajib
    plan = ajib.span_plan(15 + c, c=c, blocks=blocks, scale=scale)
    x = f16r(np.random.default_rng(6).uniform(0, 1, size=(3, 29, 150)))
    check(run_exec(plan, x), run_plan(plan, x))


def test_span_bands_bit_identical():
    import ajib
    plan = ajib.span_plan(16, c=16, blocks=2)
    x = f16r(np.random.default_rng(7).uniform(0, 1, size=(3, 40, 70)))
    assert np.array_equal(run_exec(plan, x, bands=1), run_exec(plan, x, bands=4))


def test_video_p010_chain():
    """aji_infer (pre -> net -> post) against oracle pre -> oracle net -> oracle post. The net's
    fp16 tolerance can move a quantised sample by a level or two; everything else is exact."""
    import ajib
    w, h = 96, 64
    plan = ajib.compact_plan(14, body=4)
    d = tempfile.mkdtemp()
    path = os.path.join(d, "m.ajnm")
    with open(path, "wb") as f:
        f.write(ajib.model_bytes(plan))
    vid = ajib.Video(path, w, h)
    ow, oh = vid.configure(w, h)
    assert (ow, oh) == (2 * w, 2 * h)
    rng = np.random.default_rng(5)
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
    # the net's 2e-2 tolerance is ~17 luma levels of 10-bit limited range; require far less
    assert np.abs(gy.astype(int) - (wy >> 6).astype(int)).max() <= 3
    assert np.abs(guv.astype(int) - (wuv >> 6).astype(int)).max() <= 3
    assert psnr(gy / 1023.0, (wy >> 6) / 1023.0) >= 50.0
    # errors surface as status codes, not crashes
    bad = ajib.frame(w + 2, h, ajib.FMT_P010, [dy.data_ptr(), duv.data_ptr()], [w * 2, w * 2])
    assert vid.infer(bad, fout, 0) == -2
    assert "do not match" in vid.error()
    vid.close()


@pytest.mark.parametrize("net,fmt,norm,w,h", [("compact", 2, False, 200, 72), ("compact", 1, False, 200, 72),
                                              ("compact", 2, True, 200, 72), ("compact", 2, False, 272, 40),
                                              ("compact", 1, True, 272, 40), ("spanf3", 2, False, 272, 40),
                                              ("spanf3", 1, True, 272, 40), ("spanf3", 2, True, 200, 72)])
def test_fused_pre_pack_matches_separate_passes(net, fmt, norm, w, h):
    """aji_infer fuses the first net's input pack into the colour pre pass (the pre pass writes the
    head's strip-chunked map as well as the NCHW RGB; for SPANF3's 2x pixel-unshuffled head, the
    16-channel map at half size). Its output must equal, bit for bit, the unfused chain:
    aji_run_pre, the executor with its own pack, aji_run_post, on the same frame. Widths that are
    multiples of 16 take the streaming pre kernel, the others the tiled one (for the unshuffled
    head followed by the executor's pack)."""
    import ctypes as C
    import ajib
    plan = ajib.compact_plan(41, body=3) if net == "compact" else ajib.spanf3_plan(43, c=16, blocks=2, gain=0.7)
    if norm:
        plan["steps"][0]["in_norm"] = ((0.45, 0.5, 0.4), (2.0, 1.9, 2.1))
    d = tempfile.mkdtemp()
    path = os.path.join(d, "m.ajnm")
    with open(path, "wb") as f:
        f.write(ajib.model_bytes(plan))
    vid = ajib.Video(path, w, h)
    ow, oh = vid.configure(w, h)
    rng = np.random.default_rng(fmt * 10 + norm)
    y, uv = yuv420_frame(rng, w, h, fmt)
    es = 2 if fmt == 2 else 1
    tdt = torch.int16 if fmt == 2 else torch.uint8
    view = np.int16 if fmt == 2 else np.uint8
    dy, duv = torch.from_numpy(y.view(view)).cuda(), torch.from_numpy(uv.view(view)).cuda()
    oy, ouv = torch.empty((oh, ow), dtype=tdt, device="cuda"), torch.empty((oh // 2, ow), dtype=tdt, device="cuda")
    fin = ajib.frame(w, h, fmt, [dy.data_ptr(), duv.data_ptr()], [w * es, w * es])
    fout = ajib.frame(ow, oh, fmt, [oy.data_ptr(), ouv.data_ptr()], [ow * es, ow * es])
    assert vid.infer(fin, fout, 0) == 0, vid.error()
    torch.cuda.synchronize()
    vid.close()
    # the same three passes, unfused
    csp = ajib.lib.aji_make_csp(fmt, ajib.MATRIX_BT709, ajib.RANGE_LIMITED)
    pre = ajib.lib.aji_pre_plan_create(fmt, w, h, ajib.SITING_LEFT, 0)
    rgb = torch.empty((3, h, w), dtype=torch.float16, device="cuda")
    assert ajib.lib.aji_run_pre(pre, dy.data_ptr(), w * es, duv.data_ptr(), w * es, C.byref(csp), rgb.data_ptr(), None) == 0
    ex = ajib.Exec(ajib.Model(plan), w, h)
    out = torch.empty((3, oh, ow), dtype=torch.float16, device="cuda")
    assert ex.run(rgb.data_ptr(), out.data_ptr(), 0) == 0
    post = ajib.lib.aji_post_plan_create(fmt, ow, oh, ajib.SITING_LEFT, 0)
    py, puv = torch.empty_like(oy), torch.empty_like(ouv)
    assert ajib.lib.aji_run_post(post, out.data_ptr(), C.byref(csp), py.data_ptr(), ow * es, puv.data_ptr(), ow * es,
                                 None) == 0
    torch.cuda.synchronize()
    ajib.lib.aji_plan_destroy(pre)
    ajib.lib.aji_plan_destroy(post)
    assert torch.equal(oy, py) and torch.equal(ouv, puv)
