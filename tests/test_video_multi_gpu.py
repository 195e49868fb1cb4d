"""GPU: one video stream over several devices (ajib_video_create_multi). Frame k runs on device
k mod n with its own context; every output must equal, bit for bit, what a one-device aji_infer
gives for the same frame, and tickets complete in submission order. On a one-GPU box the ring
logic (slot reuse, in-order completion) runs with n = 1 at several ring depths; the two-device
case runs where the box has two GPUs."""
import os
import tempfile

import numpy as np
import pytest

from synth import p010_frame

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

W, H = 192, 108


def _model(plan):
    import ajib
    d = tempfile.mkdtemp()
    path = os.path.join(d, "m.ajnm")
    with open(path, "wb") as f:
        f.write(ajib.model_bytes(plan))
    return path


def _single(path, frames):
    """The outputs of a one-device video context (device memory frames), in order."""
    import ajib
    vid = ajib.Video(path, W, H)
    ow, oh = vid.configure(W, H)
    outs = []
    for y, uv in frames:
        dy = torch.from_numpy(y.view(np.int16)).cuda()
        duv = torch.from_numpy(uv.view(np.int16)).cuda()
        oy = torch.empty((oh, ow), dtype=torch.int16, device="cuda")
        ouv = torch.empty((oh // 2, ow), dtype=torch.int16, device="cuda")
        fin = ajib.frame(W, H, ajib.FMT_P010, [dy.data_ptr(), duv.data_ptr()], [W * 2, W * 2])
        fout = ajib.frame(ow, oh, ajib.FMT_P010, [oy.data_ptr(), ouv.data_ptr()], [ow * 2, ow * 2])
        assert vid.infer(fin, fout, 0) == 0, vid.error()
        torch.cuda.synchronize()
        outs.append((oy.cpu().numpy().view(np.uint16), ouv.cpu().numpy().view(np.uint16)))
    vid.close()
    return outs


def _multi(path, devices, depth, frames, pinned):
    import ajib
    m = ajib.VideoMulti(devices, model_path=path, max_w=W, max_h=H, depth=depth)
    ow, oh = m.configure(W, H)
    assert (ow, oh) == (2 * W, 2 * H)
    ins, outs, tickets = [], [], []
    for y, uv in frames:
        ty, tuv = torch.from_numpy(y.view(np.int16)), torch.from_numpy(uv.view(np.int16))
        oy, ouv = torch.zeros((oh, ow), dtype=torch.int16), torch.zeros((oh // 2, ow), dtype=torch.int16)
        if pinned:
            ty, tuv, oy, ouv = ty.pin_memory(), tuv.pin_memory(), oy.pin_memory(), ouv.pin_memory()
        ins.append((ty, tuv))
        outs.append((oy, ouv))
        fin = ajib.frame(W, H, ajib.FMT_P010, [ty.data_ptr(), tuv.data_ptr()], [W * 2, W * 2])
        fout = ajib.frame(ow, oh, ajib.FMT_P010, [oy.data_ptr(), ouv.data_ptr()], [ow * 2, ow * 2])
        t = m.submit(fin, fout)
        assert t == len(tickets) + 1, m.error()
        tickets.append(t)
    # completion in order: once the last ticket is waited for, every earlier one reports done
    assert m.wait(tickets[-1]) == 0, m.error()
    assert all(m.done(t) == 1 for t in tickets)
    got = [(oy.numpy().view(np.uint16).copy(), ouv.numpy().view(np.uint16).copy()) for oy, ouv in outs]
    m.close()
    return got


@pytest.mark.parametrize("depth,pinned", [(1, True), (2, True), (3, False)])
def test_one_device_ring_matches_single_context(depth, pinned):
    import ajib
    path = _model(ajib.compact_plan(31, body=3))
    frames = [p010_frame(100 + i, W, H) for i in range(7)]
    want = _single(path, frames)
    got = _multi(path, [0], depth, frames, pinned)
    for k, ((gy, guv), (wy, wuv)) in enumerate(zip(got, want)):
        assert np.array_equal(gy, wy) and np.array_equal(guv, wuv), f"frame {k}"


def test_refusals_and_errors():
    import ajib
    path = _model(ajib.compact_plan(32, body=1))
    with pytest.raises(ajib.AjibError):
        ajib.VideoMulti([0, 0], model_path=path, max_w=W, max_h=H)
    with pytest.raises(ajib.AjibError):
        ajib.VideoMulti([0], model_path=path, max_w=W, max_h=H, depth=0)
    m = ajib.VideoMulti([0], model_path=path, max_w=W, max_h=H)
    # submit before configure, then a frame of the wrong size
    y = torch.zeros((H, W), dtype=torch.int16)
    fin = ajib.frame(W, H, ajib.FMT_P010, [y.data_ptr(), y.data_ptr()], [W * 2, W * 2])
    assert m.submit(fin, fin) < 0 and "configure" in m.error()
    ow, oh = m.configure(W, H)
    assert m.submit(fin, fin) == ajib.AJIB_ERR_ARGS and "do not match" in m.error()
    assert m.wait(5) == ajib.AJIB_ERR_ARGS
    m.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_devices_match_single_context_and_time_both():
    import ajib
    path = _model(ajib.compact_plan(33, body=3))
    frames = [p010_frame(200 + i, W, H) for i in range(9)]
    want = _single(path, frames)
    got = _multi(path, [0, 1], 2, frames, True)
    for k, ((gy, guv), (wy, wuv)) in enumerate(zip(got, want)):
        assert np.array_equal(gy, wy) and np.array_equal(guv, wuv), f"frame {k}"
    # device timing: both devices ran frames
    m = ajib.VideoMulti([0, 1], model_path=path, max_w=W, max_h=H)
    ow, oh = m.configure(W, H)
    assert m.timing(True) == 0
    y, uv = (torch.from_numpy(a.view(np.int16)).pin_memory() for a in frames[0])
    oy, ouv = torch.zeros((oh, ow), dtype=torch.int16).pin_memory(), torch.zeros((oh // 2, ow), dtype=torch.int16).pin_memory()
    fin = ajib.frame(W, H, ajib.FMT_P010, [y.data_ptr(), uv.data_ptr()], [W * 2, W * 2])
    outs = [(torch.zeros_like(oy).pin_memory(), torch.zeros_like(ouv).pin_memory()) for _ in range(4)]
    t = 0
    for o in outs:
        fout = ajib.frame(ow, oh, ajib.FMT_P010, [o[0].data_ptr(), o[1].data_ptr()], [ow * 2, ow * 2])
        t = m.submit(fin, fout)
    assert m.wait(t) == 0
    ms = m.device_ms()
    assert len(ms) == 2 and all(v > 0 for v in ms)
    m.close()
