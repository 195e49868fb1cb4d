"""CPU: ONNX models lowered to native plans (csrc/onnx.cpp + csrc/lower.cpp, the reference's
src/native/onnx_graph.cpp + lower.cpp rules). Graphs are written here (tests/onnx_writer.py) the
way the supported families export, from a plan; the lowering must give that plan back, step for
step and weight for weight, and the same bytes as the reference's own lowering (compiled from its
sources into oracle/_ref/libref_lower.so by oracle/ref/build.sh) where that is present. Graphs the
kernels cannot run are refused with a reason."""
import ctypes as C
import os

import numpy as np
import pytest

from onnx_writer import Graph, export, export_span, export_spanf3
from util import ROOT

REF_LOWER = os.path.join(ROOT, "oracle", "_ref", "libref_lower.so")


def lowered(onnx_bytes):
    import ajib
    return ajib.parse_model_bytes(ajib.model_from_bytes(onnx_bytes))


def ref_lowered(onnx_bytes):
    ref = C.CDLL(REF_LOWER)
    ref.ref_lower.argtypes = [C.c_char_p, C.c_size_t, C.c_void_p, C.c_size_t, C.POINTER(C.c_size_t), C.c_char_p,
                              C.c_size_t]
    n = C.c_size_t()
    why = C.create_string_buffer(512)
    assert ref.ref_lower(onnx_bytes, len(onnx_bytes), None, 0, C.byref(n), why, 512) == 0, why.value.decode()
    buf = C.create_string_buffer(n.value)
    assert ref.ref_lower(onnx_bytes, len(onnx_bytes), buf, n.value, C.byref(n), why, 512) == 0
    return buf.raw[:n.value]


def same_plan(got, want, norm=None, clamp=False, f16_params=False):
    assert got["depth_to_space"] == want["depth_to_space"]
    assert list(got["channels"]) == list(want["channels"])
    assert len(got["steps"]) == len(want["steps"])
    for i, (g, w) in enumerate(zip(got["steps"], want["steps"])):
        for k in ("kind", "act", "gate", "out", "src", "resid", "dst"):
            assert g[k] == w.get(k, {"kind": 0, "act": 0, "gate": 0, "out": 0, "src": -1, "resid": -1}.get(k)), (i, k)
        if w["kind"] == 1:
            assert g["srcs"] == list(w["srcs"]) and g["c"] == w["c"] and g["nsrc"] == len(w["srcs"])
        else:
            assert g["in_"] == w.get("in_", 0) and g["cin"] == w["cin"] and g["cout"] == w["cout"]
        # weights: the fp16 values the plan carries, bias and slopes as given
        assert np.array_equal(g["w"].astype(np.float16).view(np.uint16),
                              np.asarray(w["w"], np.float32).astype(np.float16).view(np.uint16)), i
        # a file with fp16 parameters stores bias and slopes at fp16 too
        rnd = (lambda a: np.asarray(a, np.float32).astype(np.float16).astype(np.float32)) if f16_params else \
            (lambda a: np.asarray(a, np.float32))
        assert np.array_equal(g["bias"], rnd(w["bias"])), i
        if w.get("slope") is not None:
            assert np.array_equal(g["slope"], rnd(w["slope"])), i
        if w.get("gate", 0) == 2:
            aw = np.asarray(w["att"][0], np.float32)
            assert np.array_equal(g["att"][0].astype(np.float16).view(np.uint16),
                                  aw.reshape(g["att"][0].shape).astype(np.float16).view(np.uint16)), i
            assert np.array_equal(g["att"][1], rnd(w["att"][1])), i
    assert got.get("unshuffle", 1) == want.get("unshuffle", 1)
    first = got["steps"][0]
    if norm is not None:
        mean, scale = norm
        assert "in_norm" in first
        assert np.allclose(first["in_norm"][0], mean) and np.allclose(first["in_norm"][1], scale)
    assert bool(got["steps"][-1].get("out_clamp")) == clamp


@pytest.mark.parametrize("kw", [{}, {"d2s_mode": "DCR"}, {"skip_form": "half_pixel"}, {"clip": True},
                                {"shape_plumbing": True}, {"wdtype": 10}])
def test_compact_forms(kw):
    import ajib
    plan = ajib.compact_plan(41, body=3)
    same_plan(lowered(export(plan, **kw)), plan, clamp=kw.get("clip", False), f16_params=kw.get("wdtype") == 10)


def test_super_ultra_compact_4x():
    import ajib
    plan = ajib.compact_plan(42, c=24, body=4, scale=4)
    same_plan(lowered(export(plan)), plan)


def test_leaky_relu_and_relu():
    import ajib
    plan = ajib.compact_plan(43, body=2)
    for s in plan["steps"]:
        if s.get("act") == 2:
            s["slope"] = np.full(s["cout"], 0.2, np.float32)
    got = lowered(export(plan, act_form="leaky"))
    same_plan(got, plan)
    for s in plan["steps"]:
        if s.get("act") == 2:
            s["act"], s["slope"] = 1, None
    same_plan(lowered(export(plan)), plan)


@pytest.mark.parametrize("merged", [False, True])
def test_span(merged):
    import ajib
    plan = ajib.span_plan(44, c=48, blocks=3)
    onnx = export_span(plan) if merged else export(plan)
    same_plan(lowered(onnx), plan)


@pytest.mark.parametrize("s2d", [False, True])
@pytest.mark.parametrize("c,blocks", [(48, 5), (64, 8), (16, 2)])
def test_spanf3(s2d, c, blocks):
    """SPANF3 with the 2x pixel-unshuffle (Reshape/Transpose or SpaceToDepth), the input Pad and
    output Slice computed from the input's shape, tanh gates, ReLU convs, depth-to-space 4."""
    import ajib
    plan = ajib.spanf3_plan(60 + c, c=c, blocks=blocks)
    got = lowered(export_spanf3(plan, space_to_depth=s2d))
    same_plan(got, plan)
    assert len(got["steps"]) == 3 * blocks + 3 and got["depth_to_space"] == 4 and got["unshuffle"] == 2
    assert got["steps"][0]["in_"] == 2 and got["steps"][0]["cin"] == 12


def test_fixed_pad_and_crop_refused():
    import ajib
    plan = ajib.spanf3_plan(61, c=16, blocks=1)
    onnx = export_spanf3(plan)
    # the same graph with a Pad by a constant amount
    g = Graph()
    rng = np.random.default_rng(1)
    w = rng.normal(0, 0.1, size=(9, 3, 12)).astype(np.float32)
    p = g.node("Pad", ["input", g.init(np.array([0, 0, 1, 1, 0, 0, 1, 1]), "p", dtype=7)])
    o = g.conv(p, w, np.zeros(12, np.float32), 3)
    g.node("DepthToSpace", [o], ["output"], blocksize=2, mode="CRD")
    _refused(g.model(), "Pad by a fixed amount")
    assert lowered(onnx)["unshuffle"] == 2


def test_input_normalisation():
    import ajib
    plan = ajib.span_plan(45, c=16, blocks=2)
    mean, scale = (0.4488, 0.4371, 0.4040), (255.0, 255.0, 255.0)
    got = lowered(export(plan, norm=(mean, scale)))
    same_plan(got, plan, norm=(mean, scale))


@pytest.mark.skipif(not os.path.exists(REF_LOWER), reason="reference lowering not built (oracle/_ref)")
@pytest.mark.parametrize("which", ["compact", "suc", "span", "span_merged", "compact_dcr_clip", "spanf3",
                                   "spanf3_s2d"])
def test_against_reference_lowering(which):
    """The same ONNX bytes through the reference's lowering: the same plan, byte for byte (the
    name aside)."""
    import ajib
    if which == "compact":
        onnx = export(ajib.compact_plan(46, body=3))
    elif which == "suc":
        onnx = export(ajib.compact_plan(47, c=24, body=3, scale=4))
    elif which == "span":
        onnx = export(ajib.span_plan(48, c=48, blocks=2))
    elif which == "span_merged":
        onnx = export_span(ajib.span_plan(49, c=48, blocks=2))
    elif which == "spanf3":
        onnx = export_spanf3(ajib.spanf3_plan(51, c=48, blocks=2))
    elif which == "spanf3_s2d":
        onnx = export_spanf3(ajib.spanf3_plan(52, c=64, blocks=2), space_to_depth=True)
    else:
        onnx = export(ajib.compact_plan(50, body=2), d2s_mode="DCR", clip=True)
    ours = ajib.parse_model_bytes(ajib.model_from_bytes(onnx))
    ref = ajib.parse_model_bytes(ref_lowered(onnx))
    assert len(ours["steps"]) == len(ref["steps"])
    assert list(ours["channels"]) == list(ref["channels"]) and ours["depth_to_space"] == ref["depth_to_space"]
    for a, b in zip(ours["steps"], ref["steps"]):
        for k in ("kind", "in_", "act", "gate", "out", "cin", "cout", "src", "resid", "dst", "c", "nsrc", "srcs",
                  "out_clamp"):
            assert a.get(k) == b.get(k), k
        assert np.array_equal(a["w"], b["w"]) and np.array_equal(a["bias"], b["bias"])
        assert (a.get("slope") is None) == (b.get("slope") is None)
        if a.get("slope") is not None:
            assert np.array_equal(a["slope"], b["slope"])
        assert ("att" in a) == ("att" in b)
        if "att" in a:
            assert all(np.array_equal(u, v) for u, v in zip(a["att"][:2], b["att"][:2]))
    assert ours["unshuffle"] == ref["unshuffle"]


def _refused(onnx, what):
    import ajib
    with pytest.raises(ajib.AjibError) as e:
        ajib.model_from_bytes(onnx)
    assert what in str(e.value), str(e.value)


def test_refusals():
    import ajib
    rng = np.random.default_rng(0)
    w = rng.normal(0, 0.1, size=(9, 3, 12)).astype(np.float32)
    # a strided conv
    g = Graph()
    W = w.reshape(3, 3, 3, 12).transpose(3, 2, 0, 1)
    o = g.node("Conv", ["input", g.init(W), g.init(np.zeros(12, np.float32), "b")], kernel_shape=[3, 3],
               pads=[1, 1, 1, 1], strides=[2, 2])
    g.node("DepthToSpace", [o], ["output"], blocksize=2, mode="CRD")
    _refused(g.model(), "strided")
    # an op the kernels do not run
    g = Graph()
    o = g.conv("input", w, np.zeros(12, np.float32), 3)
    o = g.node("Softmax", [o], axis=1)
    g.node("DepthToSpace", [o], ["output"], blocksize=2, mode="CRD")
    _refused(g.model(), "Softmax")
    # not ONNX at all
    _refused(b"\x01\x02garbage", "ONNX")
    # a Resize of the input that is not pixel replication
    g = Graph()
    o = g.conv("input", w, np.zeros(12, np.float32), 3)
    o = g.node("DepthToSpace", [o], blocksize=2, mode="CRD")
    rz = g.node("Resize", ["input", "", g.init(np.array([1, 1, 2, 2], np.float32), "sc")], mode="linear")
    g.node("Add", [o, rz], ["output"])
    _refused(g.model(), "upsampled model input")
