"""GPU: the still-image path. The tiler kernels bit for bit against the CPU tiler oracle (which is
pinned to the reference's upscale_tiled) and against the reference's own GPU tiler kernels
(src/core/tiling_gpu.cu, compiled into oracle/_ref); then aji_img_upscale end to end with a
SuperUltraCompact net against the oracle (tiler + reference-semantics net), within the net's
fp16 tolerance."""
import ctypes as C
import os
import tempfile

import numpy as np
import pytest

from oracle_net import run_plan
from util import ROOT, oracle_axis_weights, oracle_origins, oracle_upscale_tiled, psnr

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

REF_TGPU = os.path.join(ROOT, "oracle", "_ref", "libref_tiling_gpu.so")


def make_tiler(W, H, ci, s, tile, overlap, even=0):
    import ajib
    t = C.c_void_p()
    assert ajib.lib.ajib_tiler_create(W, H, ci, s, tile, tile, overlap, even, C.byref(t)) == 0
    nx, ny, tw, th = C.c_int(), C.c_int(), C.c_int(), C.c_int()
    ajib.lib.ajib_tiler_info(t, C.byref(nx), C.byref(ny), C.byref(tw), C.byref(th))
    return t, nx.value, ny.value, tw.value, th.value


def reflect(i, n):
    if n == 1:
        return 0
    p = 2 * (n - 1)
    i %= p
    return i if i < n else p - i


@pytest.mark.parametrize("W,H,ci,tile,ov,s", [(100, 70, 3, 32, 8, 2), (45, 61, 1, 16, 4, 4), (20, 10, 3, 32, 8, 2),
                                             (300, 129, 3, 64, 16, 4)])
def test_tiler_extract_and_compose_bit_exact(W, H, ci, tile, ov, s):
    import ajib
    rng = np.random.default_rng(W + H)
    img = rng.integers(0, 256, size=(H, W, ci)).astype(np.uint8)
    t, nx, ny, tw, th = make_tiler(W, H, ci, s, tile, ov)
    n = nx * ny
    dimg = torch.from_numpy(img.reshape(-1)).cuda()
    tin = torch.empty((3, n * th, tw), dtype=torch.float16, device="cuda")
    assert ajib.lib.ajib_tiler_extract(t, dimg.data_ptr(), 0, n, tin.data_ptr(), None) == 0
    torch.cuda.synchronize()
    got = tin.cpu().numpy()
    ox, oy = oracle_origins(W, tile, ov), oracle_origins(H, tile, ov)
    inv = np.float32(1.0) / np.float32(255.0)
    for k in range(n):
        j, i = divmod(k, nx)
        ys = [reflect(oy[j] + y, H) for y in range(th)]
        xs = [reflect(ox[i] + x, W) for x in range(tw)]
        patch = img[np.ix_(ys, xs)].astype(np.float32) * inv
        want = patch if ci == 3 else np.repeat(patch, 3, axis=2)
        assert np.array_equal(got[:, k * th:(k + 1) * th, :], want.transpose(2, 0, 1).astype(np.float16))
    # compose random model outputs, against the oracle tiler driven by the same outputs
    touts = rng.uniform(-0.05, 1.05, size=(n, 3, th * s, tw * s)).astype(np.float16)
    dt = torch.from_numpy(np.ascontiguousarray(touts.transpose(1, 0, 2, 3))).cuda()
    out = torch.empty(H * s * W * s * ci, dtype=torch.uint8, device="cuda")
    assert ajib.lib.ajib_tiler_compose(t, dt.data_ptr(), out.data_ptr(), None) == 0
    torch.cuda.synchronize()
    calls = iter(range(n))
    want = oracle_upscale_tiled(lambda x: touts[next(calls)].astype(np.float32), tw, th, s, ov, img)
    assert np.array_equal(out.cpu().numpy().reshape(H * s, W * s, ci), want)
    ajib.lib.ajib_tiler_release(C.byref(t))


def test_tiler_compose_unaligned_buffers():
    """ajib_tiler_compose with the tile stack one fp16 element and the output one byte past an
    aligned address (any device pointers a caller holds): the vector loads and stores are left
    for per-element ones, and the bytes equal the aligned call's. The geometry is one the vector
    path serves when the buffers are aligned (4-aligned tile columns, RGB)."""
    import ajib
    W, H, ci, tile, ov, s = 256, 192, 3, 64, 16, 4
    rng = np.random.default_rng(5)
    t, nx, ny, tw, th = make_tiler(W, H, ci, s, tile, ov)
    n = nx * ny
    touts = rng.uniform(-0.05, 1.05, size=(3, n, th * s, tw * s)).astype(np.float16)
    flat = np.ascontiguousarray(touts).reshape(-1)
    nbytes = H * s * W * s * ci
    dt = torch.from_numpy(flat).cuda()
    dt1 = torch.empty(flat.size + 1, dtype=torch.float16, device="cuda")
    dt1[1:] = dt
    out = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    out1 = torch.zeros(nbytes + 1, dtype=torch.uint8, device="cuda")
    assert ajib.lib.ajib_tiler_compose(t, dt.data_ptr(), out.data_ptr(), None) == 0
    assert ajib.lib.ajib_tiler_compose(t, dt1.data_ptr() + 2, out1.data_ptr() + 1, None) == 0
    torch.cuda.synchronize()
    assert np.array_equal(out1.cpu().numpy()[1:], out.cpu().numpy())
    assert int(out1[0].item()) == 0
    ajib.lib.ajib_tiler_release(C.byref(t))


@pytest.mark.skipif(not os.path.exists(REF_TGPU), reason="reference GPU tiler not built (oracle/_ref)")
def test_tiler_matches_reference_gpu_kernels():
    """The reference's own extract / blend / band flush on the B200: same bytes."""
    import ajib
    ref = C.CDLL(REF_TGPU)
    W, H, ci, tile, ov, s = 150, 90, 3, 64, 16, 2
    rng = np.random.default_rng(9)
    img = rng.integers(0, 256, size=(H, W, ci)).astype(np.uint8)
    t, nx, ny, tw, th = make_tiler(W, H, ci, s, tile, ov)
    n = nx * ny
    ox, oy = oracle_origins(W, tile, ov), oracle_origins(H, tile, ov)
    dimg = torch.from_numpy(img.reshape(-1)).cuda()
    # extract: ours batched vs the reference tile by tile
    tin = torch.empty((3, n * th, tw), dtype=torch.float16, device="cuda")
    assert ajib.lib.ajib_tiler_extract(t, dimg.data_ptr(), 0, n, tin.data_ptr(), None) == 0
    one = torch.empty((3, th, tw), dtype=torch.float16, device="cuda")
    for k in range(n):
        j, i = divmod(k, nx)
        assert ref.ref_tile_extract_f16(C.c_void_p(dimg.data_ptr()), W, H, ci, int(ox[i]), int(oy[j]), tw, th,
                                        C.c_void_p(one.data_ptr()), None) == 0
        torch.cuda.synchronize()
        assert torch.equal(one, tin[:, k * th:(k + 1) * th, :])
    # compose vs blend into a full-height band + one flush
    touts = torch.from_numpy(rng.uniform(-0.05, 1.05, size=(3, n * th * s, tw * s)).astype(np.float16)).cuda()
    out = torch.empty(H * s * W * s * ci, dtype=torch.uint8, device="cuda")
    assert ajib.lib.ajib_tiler_compose(t, touts.data_ptr(), out.data_ptr(), None) == 0
    OW, OH = W * s, H * s
    band = torch.zeros(ci * OH * OW, dtype=torch.float32, device="cuda")
    wx = torch.from_numpy(oracle_axis_weights(ox, W, tile, s).reshape(-1)).cuda()
    wy = torch.from_numpy(oracle_axis_weights(oy, H, tile, s).reshape(-1)).cuda()
    cols, rows = min(tile, W) * s, min(tile, H) * s
    for k in range(n):
        j, i = divmod(k, nx)
        tile_k = touts[:, k * th * s:(k + 1) * th * s, :].contiguous()
        assert ref.ref_tile_blend_f16(C.c_void_p(tile_k.data_ptr()), tw * s, th * s,
                                      C.c_void_p(wx.data_ptr() + 4 * i * cols), C.c_void_p(wy.data_ptr() + 4 * j * rows),
                                      cols, rows, int(ox[i]) * s, int(oy[j]) * s, C.c_void_p(band.data_ptr()), ci, OH, OW,
                                      None) == 0
        torch.cuda.synchronize()
    ref_out = torch.empty(OH * OW * ci, dtype=torch.uint8, device="cuda")
    assert ref.ref_band_flush(C.c_void_p(band.data_ptr()), ci, OH, OW, 0, OH, C.c_void_p(ref_out.data_ptr()), None) == 0
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out)
    ajib.lib.ajib_tiler_release(C.byref(t))


def _model_file(plan):
    import ajib
    d = tempfile.mkdtemp()
    path = os.path.join(d, "m.ajnm")
    with open(path, "wb") as f:
        f.write(ajib.model_bytes(plan))
    return path


@pytest.mark.parametrize("W,H,ci,tile,ov,even", [(150, 100, 3, 64, 16, 0), (90, 70, 1, 48, 8, 0), (130, 77, 3, 64, 16, 1)])
def test_upscale_suc_against_oracle(W, H, ci, tile, ov, even):
    """aji_img_upscale with a SuperUltraCompact 4x net (BASELINE config 2's architecture)."""
    import ajib
    plan = ajib.compact_plan(21, c=24, body=8, scale=4)
    path = _model_file(plan)
    ctx = ajib.Image()
    m = ctx.load(path, tile=tile, overlap=ov, flags=ajib.IMG_LOAD_EVEN_TILES if even else 0)
    info = ajib.ImgModelInfo()
    assert ajib.lib.aji_img_model_info_get(m, C.byref(info)) == 0 and info.scale == 4
    img = np.random.default_rng(W).integers(0, 256, size=(H, W, ci)).astype(np.uint8)
    rc, got = ctx.upscale(m, img, 4)
    assert rc == 0, ctx.error()
    want = oracle_upscale_tiled(lambda x: run_plan(plan, x.astype(np.float16).astype(np.float32)), tile, tile, 4, ov,
                                img, even=bool(even))
    d = np.abs(got.astype(int) - want.astype(int))
    assert d.max() <= 3, d.max()
    assert psnr(got / 255.0, want / 255.0) >= 50.0
    ajib.lib.aji_img_release(C.byref(m))
    ctx.close()


def test_even_tiles_of_changing_width():
    """Even tiles narrower than the model's tile, then at another width, with one model: the
    executor's maps change pitch between the runs and their pad columns must read as zero again."""
    import ajib
    plan = ajib.compact_plan(23, c=24, body=3, scale=4)
    path = _model_file(plan)
    ctx = ajib.Image()
    m = ctx.load(path, tile=64, overlap=8, flags=ajib.IMG_LOAD_EVEN_TILES)
    # even tile widths 48 (65 and 45 wide), 64 (100 wide), then 48 again
    for W, H in [(65, 77), (100, 90), (45, 50)]:
        img = np.random.default_rng(W * H).integers(0, 256, size=(H, W, 3)).astype(np.uint8)
        rc, got = ctx.upscale(m, img, 4)
        assert rc == 0, ctx.error()
        want = oracle_upscale_tiled(lambda x: run_plan(plan, x.astype(np.float16).astype(np.float32)), 64, 64, 4, 8,
                                    img, even=True)
        assert np.abs(got.astype(int) - want.astype(int)).max() <= 3, (W, H)
    ajib.lib.aji_img_release(C.byref(m))
    ctx.close()


def test_waves_progress_and_strided_output():
    """The image path's waves (tile rows composed and downloaded while later ones compute):
    progress reports rise to the total and do not change the bytes; a host output with a row
    stride wider than a row gets the same rows, its padding untouched; the result matches the
    oracle tiler."""
    import ajib
    plan = ajib.compact_plan(24, c=24, body=2, scale=4)
    path = _model_file(plan)
    ctx = ajib.Image()
    m = ctx.load(path, tile=32, overlap=8)
    H, W = 150, 70  # seven tile rows: four waves of one or two
    img = np.random.default_rng(9).integers(0, 256, size=(H, W, 3)).astype(np.uint8)
    rc, plain = ctx.upscale(m, img, 4)
    assert rc == 0, ctx.error()
    seen = []

    def watch(_, done, total):
        seen.append((done, total))
        return 0
    rc, got = ctx.upscale(m, img, 4, progress=watch)
    assert rc == 0, ctx.error()
    assert np.array_equal(got, plain)
    assert len(seen) >= 2 and all(t == seen[-1][1] for _, t in seen)
    assert all(a < b for (a, _), (b, _) in zip(seen, seen[1:])) and seen[-1][0] == seen[-1][1]
    # a padded host output (row stride 40 bytes wider than a row)
    OW, OH = 4 * W, 4 * H
    big = np.full((OH, OW * 3 + 40), 0xA5, np.uint8)
    bi = ajib.img_buffer(np.ascontiguousarray(img))
    bo = ajib.ImgBuffer()
    bo.width, bo.height, bo.channels = OW, OH, 3
    bo.stride = big.shape[1]
    bo.data = big.ctypes.data
    assert ajib.lib.aji_img_upscale(m, C.byref(bi), C.byref(bo), ajib.PROGRESS_FN(), None) == 0, ctx.error()
    assert np.array_equal(big[:, :OW * 3].reshape(OH, OW, 3), plain)
    assert (big[:, OW * 3:] == 0xA5).all()
    want = oracle_upscale_tiled(lambda x: run_plan(plan, x.astype(np.float16).astype(np.float32)), 32, 32, 4, 8, img)
    assert np.abs(plain.astype(int) - want.astype(int)).max() <= 3
    ajib.lib.aji_img_release(C.byref(m))
    ctx.close()


def test_image_api_errors_and_progress():
    import ajib
    plan = ajib.compact_plan(22, c=24, body=2, scale=4)
    path = _model_file(plan)
    ctx = ajib.Image()
    m = ctx.load(path, tile=32, overlap=8)
    img = np.zeros((70, 50, 3), np.uint8)
    # wrong output size
    bi = ajib.img_buffer(img)
    bad = np.zeros((70 * 2, 50 * 2, 3), np.uint8)
    bo = ajib.img_buffer(bad)
    assert ajib.lib.aji_img_upscale(m, C.byref(bi), C.byref(bo), ajib.PROGRESS_FN(), None) == ajib.IMG_ERR_ARGS
    assert "output must be" in ctx.error()
    # progress and cancellation
    seen = []

    def cancel(_, done, total):
        seen.append((done, total))
        return 1
    rc, _ = ctx.upscale(m, img, 4, progress=cancel)
    assert rc == ajib.IMG_CANCELLED and seen and seen[0][1] >= 1
    # memory report, probe, enumeration
    mem = ajib.ImgMemory()
    assert ajib.lib.aji_img_memory_get(ctx.handle, m, C.byref(mem)) == 0
    assert mem.device_total > mem.device_free > 0 and mem.model_weights > 0
    mp = ajib.ImgModelParams()
    mp.onnx_path = path.encode()
    mp.tile_w = mp.tile_h = 64
    assert ajib.lib.aji_img_native_probe(ctx.handle, C.byref(mp), C.byref(mem)) == 0
    devs = (ajib.ImgDevice * 8)()
    n = ajib.lib.aji_img_enum_devices(ajib.IMG_TENSORRT, devs, 8)
    assert n >= 1 and devs[0].sm_major == 10 and devs[0].id >> 63 == 1
    assert ajib.lib.aji_img_enum_devices(ajib.IMG_DIRECTML, devs, 8) < 0
    ajib.lib.aji_img_release(C.byref(m))
    ctx.close()


def _device_ids():
    import ajib
    devs = (ajib.ImgDevice * 16)()
    n = ajib.lib.aji_img_enum_devices(ajib.IMG_TENSORRT, devs, 16)
    return [devs[i].id for i in range(n)]


def _upscale(ctx, path, img, tile, ov):
    m = ctx.load(path, tile=tile, overlap=ov)
    rc, out = ctx.upscale(m, img, 4)
    assert rc == 0, ctx.error()
    import ajib
    ajib.lib.aji_img_release(C.byref(m))
    return out


def test_multi_context_one_device_equals_single():
    import ajib
    path = _model_file(ajib.compact_plan(23, c=24, body=2, scale=4))
    img = np.random.default_rng(4).integers(0, 256, size=(150, 120, 3)).astype(np.uint8)
    a = ajib.Image()
    want = _upscale(a, path, img, 48, 8)
    a.close()
    b = ajib.Image(device_ids=[_device_ids()[0]])
    got = _upscale(b, path, img, 48, 8)
    b.close()
    assert np.array_equal(got, want)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_multi_device_bands_equal_single():
    """Bands on two (or more) GPUs: the same bytes as one GPU, for a tall image of several tile rows."""
    import ajib
    path = _model_file(ajib.compact_plan(24, c=24, body=2, scale=4))
    img = np.random.default_rng(5).integers(0, 256, size=(300, 90, 3)).astype(np.uint8)
    a = ajib.Image()
    want = _upscale(a, path, img, 64, 16)
    a.close()
    ids = _device_ids()[:min(4, torch.cuda.device_count())]
    b = ajib.Image(device_ids=ids)
    got = _upscale(b, path, img, 64, 16)
    b.close()
    assert np.array_equal(got, want)
    # duplicates are refused
    with pytest.raises(ajib.AjibError):
        ajib.Image(device_ids=[ids[0], ids[0]])
