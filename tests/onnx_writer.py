"""A minimal ONNX model writer for the lowering tests: protobuf wire format by hand (the public
onnx.proto field numbers), no onnx package. Builds the graphs the supported families export
(SRVGG Compact / SuperUltraCompact, SPAN) from a plan dict of animejanai-inference_b200/ajib.py,
so the lowering can be checked against the plan that made the graph."""
import struct

import numpy as np


def _varint(v):
    out = bytearray()
    v &= (1 << 64) - 1
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field, wt):
    return _varint(field << 3 | wt)


def _ld(field, payload):
    return _key(field, 2) + _varint(len(payload)) + payload


def _str(field, s):
    return _ld(field, s.encode())


def _int(field, v):
    return _key(field, 0) + _varint(v)


def tensor(name, arr, dtype=1):
    """TensorProto: FLOAT (1) or FLOAT16 (10) as raw_data, INT64 (7) as raw_data."""
    arr = np.asarray(arr)
    b = b"".join(_int(1, int(d)) for d in arr.shape)
    b += _int(2, dtype) + _str(8, name)
    if dtype == 1:
        raw = arr.astype("<f4").tobytes()
    elif dtype == 10:
        raw = arr.astype("<f2").tobytes()
    elif dtype == 7:
        raw = arr.astype("<i8").tobytes()
    else:
        raise ValueError(dtype)
    return b + _ld(9, raw)


def attr(name, value):
    """AttributeProto of an int, float, string, ints or floats."""
    b = _str(1, name)
    if isinstance(value, bool) or isinstance(value, int):
        return b + _int(3, int(value)) + _int(20, 2)
    if isinstance(value, float):
        return b + _key(2, 5) + struct.pack("<f", value) + _int(20, 1)
    if isinstance(value, str):
        return b + _ld(4, value.encode()) + _int(20, 3)
    if isinstance(value, (list, tuple)) and all(isinstance(v, int) for v in value):
        return b + _ld(8, b"".join(_varint(v) for v in value)) + _int(20, 7)
    if isinstance(value, (list, tuple)):
        return b + _ld(7, struct.pack(f"<{len(value)}f", *value)) + _int(20, 6)
    raise ValueError(value)


class Graph:
    def __init__(self, wdtype=1):
        self.nodes, self.inits, self.n = [], [], 0
        self.wdtype = wdtype

    def name(self, p="t"):
        self.n += 1
        return f"{p}{self.n}"

    def init(self, arr, p="w", dtype=None):
        n = self.name(p)
        self.inits.append(tensor(n, arr, self.wdtype if dtype is None else dtype))
        return n

    def node(self, op, ins, outs=None, **attrs):
        outs = outs or [self.name()]
        b = b"".join(_str(1, i) for i in ins) + b"".join(_str(2, o) for o in outs) + _str(3, self.name("n"))
        b += _str(4, op) + b"".join(_ld(5, attr(k, v)) for k, v in attrs.items())
        self.nodes.append(b)
        return outs[0] if len(outs) == 1 else outs

    def conv(self, x, w, bias, k):
        """w: [taps][cin][cout] (the plan's layout) -> ONNX [cout][cin][k][k]."""
        w = np.asarray(w, np.float32)
        taps, cin, cout = w.shape
        W = w.reshape(k, k, cin, cout).transpose(3, 2, 0, 1)
        p = k // 2
        return self.node("Conv", [x, self.init(W), self.init(np.asarray(bias, np.float32), "b")],
                         kernel_shape=[k, k], pads=[p, p, p, p], strides=[1, 1])

    def model(self, inp="input", out="output", opset=17):
        def vi(n):
            return _str(1, n)
        g = b"".join(_ld(1, n) for n in self.nodes) + _str(2, "g")
        g += b"".join(_ld(5, t) for t in self.inits) + _ld(11, vi(inp)) + _ld(12, vi(out))
        return _int(1, 8) + _ld(8, _str(1, "") + _int(2, opset)) + _ld(7, g)


def export(plan, wdtype=1, d2s_mode="CRD", act_form="prelu", skip_form="asymmetric", norm=None, clip=False,
           shape_plumbing=False):
    """The ONNX graph of a Compact / SPAN plan dict, written the way PyTorch exports those nets.
    act_form: "prelu" (PRelu with [C,1,1] slopes) or "leaky" (LeakyRelu; the plan's slopes must
    be one value). norm: (mean, scale) per channel, applied as Sub then Mul to the input."""
    g = Graph(wdtype)
    x = "input"
    if shape_plumbing:
        shp = g.node("Shape", [x])
        g.node("Gather", [shp, g.init(np.array([2]), "i", dtype=7)], axis=0)
    if norm is not None:
        mean, scale = norm
        x = g.node("Sub", [x, g.init(np.asarray(mean, np.float32).reshape(1, 3, 1, 1), "m", dtype=1)])
        x = g.node("Mul", [x, g.init(np.asarray(scale, np.float32).reshape(1, 3, 1, 1), "s", dtype=1)])
    t = {-2: x}
    steps = plan["steps"]
    for s in steps:
        if s["kind"] == 1:
            cat = g.node("Concat", [t[f] for f in s["srcs"]], axis=1)
            w = np.asarray(s["w"], np.float32)
            t[s["dst"]] = g.conv(cat, w, s["bias"], 1)
            continue
        src = t[s["src"]]
        w, bias = np.asarray(s["w"], np.float32), np.asarray(s["bias"], np.float32)
        r = {1: 2, 2: 4, 3: 1, 4: 3}.get(s.get("out", 0), 1)
        if s.get("out", 0) and d2s_mode == "DCR" and r > 1:
            # DCR reads conv channel q * 3 + c where CRD (the plan's order) reads c * r * r + q
            perm = [(k % 3) * r * r + k // 3 for k in range(3 * r * r)]
            w, bias = w[:, :, perm], bias[perm]
        o = g.conv(src, w, bias, 3)
        if s.get("out", 0):
            if r > 1:
                o = g.node("DepthToSpace", [o], blocksize=r, mode=d2s_mode)
            if s.get("resid", -1) == -2:
                if skip_form == "asymmetric":
                    rz = g.node("Resize", ["input", "", g.init(np.array([1, 1, r, r], np.float32), "sc", dtype=1)],
                                mode="nearest", coordinate_transformation_mode="asymmetric", nearest_mode="floor")
                else:
                    rz = g.node("Resize", ["input", "", g.init(np.array([1, 1, r, r], np.float32), "sc", dtype=1)],
                                mode="nearest", coordinate_transformation_mode="half_pixel",
                                nearest_mode="round_prefer_floor")
                o = g.node("Add", [o, rz])
            if clip:
                o = g.node("Clip", [o, g.init(np.array(0.0, np.float32), "lo", dtype=1),
                                    g.init(np.array(1.0, np.float32), "hi", dtype=1)])
            g.node("Identity", [o], ["output"])
            continue
        act, gate = s.get("act", 0), s.get("gate", 0)
        if act == 1:
            o = g.node("Relu", [o])
        elif act == 2:
            sl = np.asarray(s["slope"], np.float32)
            if act_form == "leaky":
                o = g.node("LeakyRelu", [o], alpha=float(sl[0]))
            else:
                o = g.node("PRelu", [o, g.init(sl.reshape(-1, 1, 1), "sl")])
        elif act == 3:
            sig = g.node("Sigmoid", [o])
            o = g.node("Mul", [o, sig])
        if gate == 3:
            xin = t[s["resid"]]
            add = g.node("Add", [xin, o])
            sig = g.node("Sigmoid", [o])
            sub = g.node("Sub", [sig, g.init(np.array(0.5, np.float32), "h", dtype=1)])
            o = g.node("Mul", [add, sub])
        elif gate == 1:
            o = g.node("Add", [t[s["resid"]], o])
        t[s["dst"]] = o
    return g.model()


def export_span(plan, **kw):
    """SPAN exports one conv for the last block's c1: its raw output feeds the concat, its SiLU the
    block. The plan carries that conv twice (a plain step, then the SiLU step); merge them back."""
    steps = list(plan["steps"])
    merged, alias = [], {}
    i = 0
    while i < len(steps):
        s = steps[i]
        n = steps[i + 1] if i + 1 < len(steps) else None
        if (n is not None and s["kind"] == 0 and n["kind"] == 0 and s.get("act", 0) == 0 and n.get("act", 0) == 3
                and s["src"] == n["src"] and np.array_equal(s["w"], n["w"])):
            merged.append(dict(n, raw_dst=s["dst"]))
            i += 2
            continue
        merged.append(s)
        i += 1
    g = Graph(kw.get("wdtype", 1))
    t = {-2: "input"}
    for s in merged:
        if s["kind"] == 1:
            cat = g.node("Concat", [t[f] for f in s["srcs"]], axis=1)
            t[s["dst"]] = g.conv(cat, np.asarray(s["w"], np.float32), s["bias"], 1)
            continue
        o = g.conv(t[s["src"]], s["w"], s["bias"], 3)
        if "raw_dst" in s:
            t[s["raw_dst"]] = o
        if s.get("out", 0):
            r = {1: 2, 2: 4, 3: 1, 4: 3}[s["out"]]
            o = g.node("DepthToSpace", [o], blocksize=r, mode="CRD") if r > 1 else o
            g.node("Identity", [o], ["output"])
            continue
        if s.get("act", 0) == 3:
            o = g.node("Mul", [o, g.node("Sigmoid", [o])])
        if s.get("gate", 0) == 3:
            add = g.node("Add", [t[s["resid"]], o])
            sub = g.node("Sub", [g.node("Sigmoid", [o]), g.init(np.array(0.5, np.float32), "h", dtype=1)])
            o = g.node("Mul", [add, sub])
        t[s["dst"]] = o
    return g.model()


def export_spanf3(plan, space_to_depth=False, wdtype=1):
    """A SPANF3 plan (animejanai-inference_b200/ajib.py spanf3_plan) as PyTorch exports the
    network: the input padded to the unshuffle factor and the output cropped back (both by
    amounts computed from the input's Shape), the 2x pixel-unshuffle as Reshape -> Transpose ->
    Reshape (or SpaceToDepth, whose DCR channel order the head conv's weights follow), each block's
    gate as Add(x, c3) * Tanh(Conv1x1(c3)), and the last step's DepthToSpace 4."""
    g = Graph(wdtype)
    steps = plan["steps"]
    shp = g.node("Shape", ["input"])
    hdim = g.node("Gather", [shp, g.init(np.array([2]), "i", dtype=7)], axis=0)
    padded = g.node("Pad", ["input", hdim], mode="reflect")
    head = steps[0]
    w0 = np.asarray(head["w"], np.float32)
    if space_to_depth:
        u = g.node("SpaceToDepth", [padded], blocksize=2)
        # ONNX channel j = (ry * 2 + rx) * 3 + c holds the plan's channel k = c * 4 + ry * 2 + rx
        perm = np.zeros(12, np.int64)
        for k in range(12):
            perm[((k % 4) // 2 * 2 + k % 2) * 3 + k // 4] = k
        w0 = w0[:, perm, :]
    else:
        r1 = g.node("Reshape", [padded, shp])
        tr = g.node("Transpose", [r1], perm=[0, 1, 3, 5, 2, 4])
        u = g.node("Reshape", [tr, shp])
    t = {head["dst"]: g.conv(u, w0, head["bias"], 3)}
    for s in steps[1:]:
        if s["kind"] == 1:
            cat = g.node("Concat", [t[f] for f in s["srcs"]], axis=1)
            t[s["dst"]] = g.conv(cat, np.asarray(s["w"], np.float32), s["bias"], 1)
            continue
        o = g.conv(t[s["src"]], s["w"], s["bias"], 3)
        if s.get("out", 0):
            d = g.node("DepthToSpace", [o], blocksize=4, mode="CRD")
            g.node("Slice", [d, g.init(np.array([0]), "z", dtype=7), hdim], ["output"])
            continue
        if s.get("act", 0) == 1:
            o = g.node("Relu", [o])
        if s.get("gate", 0) == 2:
            add = g.node("Add", [t[s["resid"]], o])
            att = g.node("Tanh", [g.conv(o, s["att"][0], s["att"][1], 1)])
            o = g.node("Mul", [add, att])
        t[s["dst"]] = o
    return g.model()
