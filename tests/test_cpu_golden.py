"""CPU: the oracle pinned to golden vectors the reference's own code produced (tests/golden,
made by tests/golden/make_golden.py from the reference sources compiled into oracle/_ref), and the
engine's host-side tables checked against the same vectors. Where oracle/_ref is present, the
oracle is also compared with the reference live on fresh seeds."""
import os

import numpy as np
import pytest

from util import ROOT, oracle_csp, oracle_filter

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
REF_NET = os.path.join(ROOT, "oracle", "_ref", "libref_net.so")


def _plans():
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLD, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg


@pytest.mark.parametrize("idx", [0, 1, 2, 3])
def test_oracle_net_matches_reference_golden(idx):
    from oracle_net import run_plan
    mg = _plans()
    name, spec, seed, h, w = mg.PLANS[idx]
    plan = mg.plan_for(spec, seed)
    x = mg.plan_input(seed + 1, h, w)
    want = np.load(os.path.join(GOLD, "conv_plans.npz"))[name].astype(np.float32)
    got = run_plan(plan, x)
    assert np.array_equal(got.astype(np.float16), want.astype(np.float16)), name


@pytest.mark.skipif(not os.path.exists(REF_NET), reason="oracle/_ref not built")
@pytest.mark.parametrize("seed", [7, 8])
def test_oracle_net_matches_reference_live(seed):
    import ajib
    import refnet
    from oracle_net import run_plan
    for plan in (ajib.compact_plan(seed, body=2), ajib.span_plan(seed, c=16, blocks=2),
                 ajib.compact_plan(seed, c=24, body=1, scale=4), ajib.spanf3_plan(seed, c=16, blocks=2)):
        # an unshuffled model takes even sizes
        h, w = (12, 18) if plan.get("unshuffle", 1) == 2 else (11, 17)
        x = np.random.default_rng(seed).uniform(0, 1, size=(3, h, w)).astype(np.float16).astype(np.float32)
        assert np.array_equal(run_plan(plan, x), refnet.run_plan(REF_NET, plan, x))


def test_filter_tables_match_reference_golden():
    import ajib
    mg = _plans()
    g = np.load(os.path.join(GOLD, "resample.npz"))
    for i, (src, dst, siting, up) in enumerate(mg.RESAMPLE):
        shift = float(g[f"r{i}_shift"])
        taps, start, wt = oracle_filter(src, dst, shift)
        assert np.array_equal(start, g[f"r{i}_start"]) and np.array_equal(wt, g[f"r{i}_wt"]), (src, dst, siting)
        taps2, start2, wt2 = ajib.filter_table(src, dst, shift)
        assert np.array_equal(start2, g[f"r{i}_start"]) and np.array_equal(wt2, g[f"r{i}_wt"]), (src, dst, siting)


def test_csp_matches_reference_golden():
    import ajib
    g = np.load(os.path.join(GOLD, "resample.npz"))
    for row in g["csp"]:
        fmt, mat, rg = (int(v) for v in row[:3])
        want = np.asarray(row[3:], np.float32)
        assert np.array_equal(np.frombuffer(bytes(oracle_csp(fmt, mat, rg)), np.float32), want)
        c = ajib.lib.aji_make_csp(fmt, mat, rg)
        got = np.array([c.kr, c.kb, c.yoff, c.yscale, c.coff, c.cscale], np.float32)
        assert np.array_equal(got, want), (fmt, mat, rg)
