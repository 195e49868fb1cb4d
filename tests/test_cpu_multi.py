"""CPU, two gloo ranks: the several-GPU image path's split (ajib_img_shares, used by
ajib_img_create_multi's upscale). Each rank takes its band of output rows, blends only the tile
rows the split gives it (the oracle tiler, src/core/tiling.cpp:115-289, with a mock model whose
other tiles are zero), and the gathered bands equal the one-process result byte for byte: the
split's bands partition the output and every tile touching a band is in its tile rows."""
import ctypes as C
import os
import socket

import numpy as np
import pytest

from util import ROOT, oracle_origins, oracle_upscale_tiled

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

CASES = [  # W, H, ci, scale, tile, overlap, even
    (150, 200, 3, 2, 48, 8, 0),
    (90, 333, 1, 4, 64, 16, 0),
    (120, 260, 3, 2, 64, 16, 1),
]


def lib():
    l = C.CDLL(os.path.join(ROOT, "animejanai-inference_b200", "libaji.so"))
    l.ajib_img_shares.argtypes = [C.c_int] * 9 + [C.POINTER(C.c_int)] * 4
    l.ajib_img_shares.restype = C.c_int
    return l


def shares(W, H, ci, s, tile, ov, even, ndev):
    arr = [(C.c_int * ndev)() for _ in range(4)]
    n = lib().ajib_img_shares(W, H, ci, s, tile, tile, ov, even, ndev, *arr)
    assert n >= 1
    return [(arr[0][d], arr[1][d], arr[2][d], arr[3][d]) for d in range(n)]


def mock_model(tile_rows, nx, s):
    """A model that upsamples nearest and marks each tile, or outputs zeros for tile rows outside
    tile_rows (tiles arrive in row-major order)."""
    count = [0]

    def run(x):
        k = count[0]
        count[0] += 1
        j = k // nx
        y = np.repeat(np.repeat(x, s, axis=1), s, axis=2) * np.float32(0.9) + np.float32(0.03 * (k % 5))
        return y if tile_rows is None or tile_rows[0] <= j <= tile_rows[1] else np.zeros_like(y)
    return run


def band_result(case, rank, world):
    W, H, ci, s, tile, ov, even = case
    img = np.random.default_rng(W * H).integers(0, 256, size=(H, W, ci)).astype(np.uint8)
    sh = shares(W, H, ci, s, tile, ov, even, world)
    if even:
        from util import oracle_even_origins
        nx = len(oracle_even_origins(W, tile, ov)[0])
    else:
        nx = len(oracle_origins(W, tile, ov))
    if rank >= len(sh):
        return np.zeros((0, W * s, ci), np.uint8), img
    y0, y1, j0, j1 = sh[rank]
    out = oracle_upscale_tiled(mock_model((j0, j1), nx, s), tile, tile, s, ov, img, even=bool(even))
    return out[y0:y1], img


def worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        for ci_, case in enumerate(CASES):
            band, _ = band_result(case, rank, world)
            sizes = [None] * world
            dist.all_gather_object(sizes, band.shape[0])
            t = torch.from_numpy(np.ascontiguousarray(band)).reshape(-1)
            maxn = max(sizes) * band.shape[1] * band.shape[2]
            buf = torch.zeros(maxn, dtype=torch.uint8)
            buf[:t.numel()] = t
            gathered = [torch.zeros(maxn, dtype=torch.uint8) for _ in range(world)]
            dist.all_gather(gathered, buf)
            if rank == 0:
                rows = [g[:sizes[r] * band.shape[1] * band.shape[2]].numpy().reshape(sizes[r], band.shape[1], band.shape[2])
                        for r, g in enumerate(gathered)]
                q.put((ci_, np.concatenate(rows, axis=0)))
    finally:
        dist.destroy_process_group()


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shares_partition_rows_and_cover_tiles():
    for (W, H, ci, s, tile, ov, even) in CASES:
        for ndev in (1, 2, 3, 8):
            sh = shares(W, H, ci, s, tile, ov, even, ndev)
            assert sh[0][0] == 0 and sh[-1][1] == H * s
            for a, b in zip(sh, sh[1:]):
                assert a[1] == b[0] and a[0] < a[1]


def test_two_rank_bands_equal_one_process():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in CASES:
        ci_, arr = q.get(timeout=300)
        results[ci_] = arr
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for ci_, case in enumerate(CASES):
        W, H, ci, s, tile, ov, even = case
        img = np.random.default_rng(W * H).integers(0, 256, size=(H, W, ci)).astype(np.uint8)
        if even:
            from util import oracle_even_origins
            nx = len(oracle_even_origins(W, tile, ov)[0])
        else:
            nx = len(oracle_origins(W, tile, ov))
        full = oracle_upscale_tiled(mock_model(None, nx, s), tile, tile, s, ov, img, even=bool(even))
        assert np.array_equal(results[ci_], full), f"case {case}"
