"""CPU: the tiler oracle (oracle/oracle_tiling.c) against the reference tiler's golden vectors
(src/core/tiling.cpp run on the reference test's mock models, sanity/tiling_test.cpp: Nearest
replication must reproduce an exact nearest upscale, Constant 0.6 must give 153), and the
engine's host-side tile geometry against the same vectors."""
import os

import numpy as np

from util import oracle_axis_weights, oracle_even_origins, oracle_origins, oracle_upscale_tiled, _tiling_sigs

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _mg():
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLD, "make_golden.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def test_origins_and_weights_match_reference():
    g = np.load(os.path.join(GOLD, "tiling.npz"))
    for i, (n, tile, ov) in enumerate(_mg().TILE_AXES):
        org = oracle_origins(n, tile, ov)
        assert np.array_equal(org, g[f"a{i}_origins"]), (n, tile, ov)
        for s in (1, 2, 4):
            assert np.array_equal(oracle_axis_weights(org, n, tile, s), g[f"a{i}_w{s}"]), (n, tile, ov, s)
        e, t = oracle_even_origins(n, tile, ov)
        assert np.array_equal(e, g[f"a{i}_even"]) and t == int(g[f"a{i}_even_tile"])
    o = _tiling_sigs()
    for i, n, want in g["reflect"]:
        assert o.orc_reflect(int(i), int(n)) == want


def test_baseline_config2_geometry():
    """2048 wide, tile 512, overlap 16 -> origins {0, 496, 992, 1488, 1536}."""
    assert list(oracle_origins(2048, 512, 16)) == [0, 496, 992, 1488, 1536]


def _nearest(s):
    def model(x):
        return np.repeat(np.repeat(x, s, axis=1), s, axis=2)
    return model


def _constant(s, v=0.6):
    def model(x):
        return np.full((3, x.shape[1] * s, x.shape[2] * s), v, np.float32)
    return model


def test_upscale_tiled_matches_reference_mock_models():
    g = np.load(os.path.join(GOLD, "tiling.npz"))
    for i, (kind, w, h, ch, tile, ov, s) in enumerate(_mg().TILED):
        img = g[f"t{i}_in"]
        model = _nearest(s) if kind == 0 else _constant(s)
        got = oracle_upscale_tiled(model, tile, tile, s, ov, img)
        assert np.array_equal(got, g[f"t{i}_out"]), (kind, w, h, ch, tile, ov, s)
        if kind == 0:  # the reference's own known answer: an exact nearest upscale
            assert np.array_equal(got, np.repeat(np.repeat(img, s, axis=0), s, axis=1))
        else:
            assert (got == 153).all()
