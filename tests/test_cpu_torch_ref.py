"""The PyTorch fp32 reference of a plan (tests/torch_ref.py), which the GPU tests use for whole
frames at BASELINE sizes, checked on the CPU against the C oracle (sanity/native_ref.h:run_plan
semantics) for every plan form: Compact / SuperUltraCompact, SPAN, SPANF3. Both are fp32 with
fp16-rounded maps; they differ only in accumulation order (the oracle accumulates in double), so
an fp16 rounding boundary may differ by one unit in the last place."""
import numpy as np
import pytest

import ajib_plans as P
from oracle_net import run_plan
from torch_ref import run_plan_torch
from util import f16r

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("name,plan,h,w", [
    ("compact", P.compact_plan(3, c=16, body=3), 19, 37),
    ("suc", P.compact_plan(4, c=24, body=2, scale=4), 13, 21),
    ("span", P.span_plan(5, c=16, blocks=2), 17, 30),
    ("spanf3", P.spanf3_plan(6, c=16, blocks=2, gain=0.7), 18, 26),
])
def test_torch_reference_matches_oracle(name, plan, h, w):
    x = f16r(np.random.default_rng(len(name)).uniform(0, 1, size=(3, h, w)))
    want = run_plan(plan, x)
    got = run_plan_torch(plan, x, device="cpu").numpy()
    assert got.shape == want.shape
    assert np.abs(got - want).max() <= 2e-3, name
