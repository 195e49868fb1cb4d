"""GPU: ajib_tiler_compose_static, the tile composition that allocates no device memory.

It is meant for callers that may not call cudaMalloc (a host application that owns all device
memory through its own allocator, or a real-time frame path where an allocation would stall the
device). Its tables live in a fixed area inside the library that every call shares, so the test
makes two calls in a row with different image shapes: the second must not see the first one's
tables, both with the host waiting between the calls and with both enqueued back to back on one
stream (the second call's table upload is ordered after the first call's kernel by the stream).
Each result must equal, byte for byte, what ajib_tiler_create + ajib_tiler_compose give (the
tiler's own tolerance is exact). This file sorts last so that a run stopping at the first
failure has run every other test before it; it also passes on its own in a fresh process."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def compose_both(W, H, ci, s, tile, ov, even, seed):
    import ajib
    lib = ajib.lib
    lib.ajib_tiler_compose_static.argtypes = [C.c_int] * 8 + [C.c_void_p, C.c_void_p, C.c_void_p]
    lib.ajib_tiler_compose_static.restype = C.c_int
    t = C.c_void_p()
    assert lib.ajib_tiler_create(W, H, ci, s, tile, tile, ov, even, C.byref(t)) == 0
    nx, ny, tw, th = C.c_int(), C.c_int(), C.c_int(), C.c_int()
    lib.ajib_tiler_info(t, C.byref(nx), C.byref(ny), C.byref(tw), C.byref(th))
    n = nx.value * ny.value
    rng = np.random.default_rng(seed)
    tiles = torch.from_numpy(rng.uniform(-0.05, 1.05, size=(3, n * th.value * s, tw.value * s)).astype(np.float16)).cuda()
    want = torch.zeros(H * s * W * s * ci, dtype=torch.uint8, device="cuda")
    got = torch.full_like(want, 77)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.ajib_tiler_compose(t, C.c_void_p(tiles.data_ptr()), C.c_void_p(want.data_ptr()), C.c_void_p(stream)) == 0
    rc = lib.ajib_tiler_compose_static(W, H, ci, s, tile, tile, ov, even, C.c_void_p(tiles.data_ptr()),
                                       C.c_void_p(got.data_ptr()), C.c_void_p(stream))
    assert rc == 0
    torch.cuda.synchronize()
    lib.ajib_tiler_release(C.byref(t))
    return got.cpu().numpy(), want.cpu().numpy()


def test_compose_static_matches_allocating_compose_twice():
    # first a large shape (many tiles, big tables), then a small one reusing the same area
    got1, want1 = compose_both(700, 260, 3, 4, 128, 16, 0, seed=1)
    got2, want2 = compose_both(90, 70, 1, 2, 32, 8, 1, seed=2)
    assert np.array_equal(got1, want1)
    assert np.array_equal(got2, want2)


def test_compose_static_refuses_oversized_tables():
    import ajib
    lib = ajib.lib
    lib.ajib_tiler_compose_static.argtypes = [C.c_int] * 8 + [C.c_void_p, C.c_void_p, C.c_void_p]
    lib.ajib_tiler_compose_static.restype = C.c_int
    # 20000 x 20000 at scale 4: the per-column and per-row tables alone pass 1 MiB, so the call is
    # refused on the host before anything runs (the small buffers below are never touched)
    tiles = torch.zeros(64, dtype=torch.float16, device="cuda")
    out = torch.zeros(64, dtype=torch.uint8, device="cuda")
    rc = lib.ajib_tiler_compose_static(20000, 20000, 3, 4, 512, 512, 16, 0, C.c_void_p(tiles.data_ptr()),
                                       C.c_void_p(out.data_ptr()), None)
    assert rc == -3  # AJIB_ERR_UNSUPPORTED


def test_compose_static_back_to_back_on_one_stream():
    """Two static composes of different shapes enqueued on one stream with no host wait between
    them, then both outputs against the allocating compose."""
    import ajib
    lib = ajib.lib
    lib.ajib_tiler_compose_static.argtypes = [C.c_int] * 8 + [C.c_void_p, C.c_void_p, C.c_void_p]
    lib.ajib_tiler_compose_static.restype = C.c_int
    shapes = [(700, 260, 3, 4, 128, 16, 0, 3), (90, 70, 1, 2, 32, 8, 1, 4)]
    stream = torch.cuda.Stream()
    sp = C.c_void_p(stream.cuda_stream)
    runs = []
    for W, H, ci, s, tile, ov, even, seed in shapes:
        t = C.c_void_p()
        assert lib.ajib_tiler_create(W, H, ci, s, tile, tile, ov, even, C.byref(t)) == 0
        nx, ny, tw, th = C.c_int(), C.c_int(), C.c_int(), C.c_int()
        lib.ajib_tiler_info(t, C.byref(nx), C.byref(ny), C.byref(tw), C.byref(th))
        n = nx.value * ny.value
        rng = np.random.default_rng(seed)
        tiles = torch.from_numpy(rng.uniform(-0.05, 1.05, size=(3, n * th.value * s, tw.value * s))
                                 .astype(np.float16)).cuda()
        want = torch.zeros(H * s * W * s * ci, dtype=torch.uint8, device="cuda")
        assert lib.ajib_tiler_compose(t, C.c_void_p(tiles.data_ptr()), C.c_void_p(want.data_ptr()), None) == 0
        torch.cuda.synchronize()
        lib.ajib_tiler_release(C.byref(t))
        runs.append((W, H, ci, s, tile, ov, even, tiles, want, torch.full_like(want, 77)))
    for W, H, ci, s, tile, ov, even, tiles, _, got in runs:
        assert lib.ajib_tiler_compose_static(W, H, ci, s, tile, tile, ov, even, C.c_void_p(tiles.data_ptr()),
                                             C.c_void_p(got.data_ptr()), sp) == 0
    stream.synchronize()
    for *_, want, got in runs:
        assert torch.equal(got, want)
