"""The CPU oracle for a whole plan: sanity/native_ref.h:24-122 (ajiref::run_plan) restated, one
step at a time through oracle/liboracle.so. Test infrastructure only (the checker)."""
import numpy as np

from util import oracle_concat, oracle_conv

MODEL_INPUT, MODEL_OUTPUT = -2, -3
D2S = {0: 0, 1: 2, 2: 4, 3: 1, 4: 3}


def _att(s):
    """The tanh gate's 1x1 weights as [cout][cout] fp16-valued floats and the bias."""
    w, b = s["att"][0], s["att"][1]
    return np.asarray(w, np.float32).astype(np.float16).astype(np.float32).reshape(s["cout"], s["cout"]), b


def run_plan(plan, x, nthreads=0):
    """x: NCHW float32 [3][h][w] (fp16-valued). Returns NCHW [3][R*h/u][R*w/u] float32 (fp16-valued),
    u the plan's pixel-unshuffle factor (the conv resolution is h/u x w/u)."""
    u = plan.get("unshuffle", 1)
    _, h, w = x.shape
    h, w = h // u, w // u
    feats = {}
    out = None
    for s in plan["steps"]:
        wq = np.asarray(s["w"], np.float32).astype(np.float16).astype(np.float32)
        if s["kind"] == 1:
            srcs = [feats[t].reshape(-1, s["c"]) for t in s["srcs"]]
            y = oracle_concat(srcs, s["c"], wq.reshape(-1, s["c"]), s["bias"], nthreads)
            feats[s["dst"]] = y.reshape(h, w, s["c"])
            continue
        src = x if s["src"] == MODEL_INPUT else feats[s["src"]]
        in_mode = (2 if s.get("in_", 1) == 2 else 1) if s["src"] == MODEL_INPUT else 0
        R = D2S[s.get("out", 0)]
        resid = None
        model_in = None
        if s.get("gate", 0):
            resid = feats[s["resid"]]
        if R and s.get("resid", -1) == MODEL_INPUT:
            model_in = x
        y = oracle_conv(src, in_mode, h, w, s["cin"], wq, s["bias"], s.get("slope"), s["cout"], act=s.get("act", 0),
                        gate=s.get("gate", 0), resid=resid, R=R, model_in=model_in,
                        out_clamp=bool(s.get("out_clamp")), nthreads=nthreads,
                        att=_att(s) if s.get("gate", 0) == 2 else None)
        if s["dst"] == MODEL_OUTPUT:
            out = y
        else:
            feats[s["dst"]] = y
    return out
