"""Native model files and the seeded model architectures of the BASELINE configs, in pure numpy.

A plan is a dict {name, steps, channels, depth_to_space[, unshuffle]} of fused conv steps: the
structure the reference's lowering produces (src/native/lower.h:38-77; sanity/native_lower_test.cpp
compact() / span_s() / spanf3). model_bytes / parse_model_bytes write and read this engine's model
file (layout documented in csrc/model.cpp). This module loads no library, so the CPU baseline and
the oracle tests can build plans without the engine.
"""
import struct

import numpy as np

# op vocabulary (reference src/native/ops.h:13-21; the same integer values as include/aji_b200.h)
IN_NHWC, IN_NCHW3, IN_NCHW3_UNSHUFFLE2 = 0, 1, 2
ACT_NONE, ACT_RELU, ACT_PRELU, ACT_SILU = 0, 1, 2, 3
GATE_NONE, GATE_RESIDUAL, GATE_TANH1X1, GATE_SIGMOID_HALF = 0, 1, 2, 3
OUT_NHWC, OUT_D2S2, OUT_D2S4, OUT_D2S1, OUT_D2S3 = 0, 1, 2, 3, 4

MODEL_INPUT, MODEL_OUTPUT = -2, -3


def _conv_step(w, bias, slope=None, in_=IN_NHWC, act=ACT_NONE, gate=GATE_NONE, out=OUT_NHWC, src=-1, resid=-1,
               dst=-1, out_clamp=False, in_norm=None):
    """w: [9][cin][cout] float (rounded to fp16 when written)."""
    w = np.asarray(w, np.float32)
    return dict(kind=0, in_=in_, act=act, gate=gate, out=out, cin=w.shape[1], cout=w.shape[2], src=src, resid=resid,
                dst=dst, w=w, bias=np.asarray(bias, np.float32), slope=None if slope is None else np.asarray(slope, np.float32),
                out_clamp=out_clamp, in_norm=in_norm)


def _concat_step(w, bias, srcs, c, dst):
    return dict(kind=1, c=c, nsrc=len(srcs), srcs=list(srcs), dst=dst, w=np.asarray(w, np.float32).reshape(1, len(srcs) * c, c),
                bias=np.asarray(bias, np.float32), slope=None)


def model_bytes(plan):
    """Serialise a plan dict {name, steps, channels, depth_to_space} to the native model format."""
    out = [b"AJNM", struct.pack("<I", 1)]
    name = plan.get("name", "").encode()
    out.append(struct.pack("<IIIII", len(plan["steps"]), len(plan["channels"]), plan.get("unshuffle", 1),
                           plan["depth_to_space"], len(name)))
    out.append(name)
    out.append(np.asarray(plan["channels"], np.int32).tobytes())

    def weights(w, b, s):
        taps, cin, cout = w.shape
        parts = [struct.pack("<iii", taps, cin, cout), w.astype(np.float16).view(np.uint16).tobytes(),
                 np.asarray(b, np.float32).tobytes(), struct.pack("<i", 0 if s is None else 1)]
        if s is not None:
            parts.append(np.asarray(s, np.float32).tobytes())
        return b"".join(parts)

    for s in plan["steps"]:
        srcs = list(s.get("srcs", [])) + [-1] * (4 - len(s.get("srcs", [])))
        norm = s.get("in_norm")
        mean, scale = (norm if norm is not None else ((0.0, 0.0, 0.0), (1.0, 1.0, 1.0)))
        out.append(struct.pack("<12i4i", s["kind"], s.get("in_", 0), s.get("act", 0), s.get("gate", 0), s.get("out", 0),
                               s.get("cin", 0), s.get("cout", 0), s.get("src", -1), s.get("resid", -1), s["dst"],
                               s.get("c", 0), s.get("nsrc", 0), *srcs))
        out.append(struct.pack("<i3f3fi", 1 if norm is not None else 0, *mean, *scale, 1 if s.get("out_clamp") else 0))
        out.append(weights(s["w"], s["bias"], s.get("slope")))
        if s["kind"] == 0 and s.get("gate", 0) == GATE_TANH1X1:
            aw = np.asarray(s["att"][0], np.float32)
            out.append(weights(aw.reshape(1, aw.shape[-2], aw.shape[-1]), s["att"][1], None))
    return b"".join(out)


def parse_model_bytes(b):
    """The plan dict of a native model file (the inverse of model_bytes)."""
    assert b[:4] == b"AJNM"
    at = 8
    nsteps, nfeat, unshuffle, d2s, name_len = struct.unpack_from("<IIIII", b, at)
    at += 20
    name = b[at:at + name_len].decode()
    at += name_len
    channels = list(np.frombuffer(b, np.int32, nfeat, at))
    at += 4 * nfeat

    def weights():
        nonlocal at
        taps, cin, cout = struct.unpack_from("<iii", b, at)
        at += 12
        w = np.frombuffer(b, np.uint16, taps * cin * cout, at).view(np.float16).astype(np.float32).reshape(taps, cin, cout)
        at += 2 * taps * cin * cout
        bias = np.frombuffer(b, np.float32, cout, at).copy()
        at += 4 * cout
        (has,) = struct.unpack_from("<i", b, at)
        at += 4
        slope = None
        if has:
            slope = np.frombuffer(b, np.float32, cout, at).copy()
            at += 4 * cout
        return w, bias, slope

    steps = []
    for _ in range(nsteps):
        f = struct.unpack_from("<12i4i", b, at)
        at += 64
        norm_flag, m0, m1, m2, s0, s1, s2, clamp = struct.unpack_from("<i3f3fi", b, at)
        at += 32
        w, bias, slope = weights()
        s = dict(kind=f[0], in_=f[1], act=f[2], gate=f[3], out=f[4], cin=f[5], cout=f[6], src=f[7], resid=f[8],
                 dst=f[9], c=f[10], nsrc=f[11], srcs=[x for x in f[12:16] if x != -1], w=w, bias=bias)
        if slope is not None:
            s["slope"] = slope
        if norm_flag:
            s["in_norm"] = ((m0, m1, m2), (s0, s1, s2))
        if clamp:
            s["out_clamp"] = True
        if f[0] == 0 and f[3] == 2:
            s["att"] = weights()
        steps.append(s)
    return dict(name=name, steps=steps, channels=channels, depth_to_space=d2s, unshuffle=unshuffle)



def _he(rng, cin, cout, taps=9):
    return (rng.normal(0.0, np.sqrt(2.0 / (taps * cin)), size=(taps, cin, cout))).astype(np.float16).astype(np.float32)


def compact_plan(seed, c=64, body=16, scale=2, name=None):
    """SRVGGNetCompact: conv_first 3->c + PReLU, `body` x (c->c + PReLU), c->3*scale^2,
    pixel_shuffle(scale), + nearest-upsampled input. He-init weights, bias N(0, 0.01), PReLU
    slopes U[0.1, 0.3], all from `seed`."""
    rng = np.random.default_rng(seed)
    steps = []

    def bias(n):
        return rng.normal(0.0, 0.01, size=n).astype(np.float32)

    def slope(n):
        return rng.uniform(0.1, 0.3, size=n).astype(np.float32)

    steps.append(_conv_step(_he(rng, 3, c), bias(c), slope(c), in_=IN_NCHW3, act=ACT_PRELU, src=MODEL_INPUT, dst=0))
    for i in range(body):
        steps.append(_conv_step(_he(rng, c, c), bias(c), slope(c), act=ACT_PRELU, src=i, dst=i + 1))
    out_mode = {1: OUT_D2S1, 2: OUT_D2S2, 3: OUT_D2S3, 4: OUT_D2S4}[scale]
    steps.append(_conv_step(_he(rng, c, 3 * scale * scale), bias(3 * scale * scale), out=out_mode, src=body,
                            resid=MODEL_INPUT, dst=MODEL_OUTPUT))
    return dict(name=name or f"compact-{c}x{body}-{scale}x", steps=steps, channels=[c] * (body + 1),
                depth_to_space=scale)


def span_plan(seed, c=48, blocks=6, scale=2, name=None):
    """SPAN: conv_first 3->c; `blocks` SPABs (c1+SiLU, c2+SiLU, c3 with (c3 + x)(sigmoid(c3) - 0.5));
    conv_2; concat[feat, conv_2, block 1 out, last block's c1 pre-activation] -> 1x1 4c->c;
    c->3*scale^2 3x3; pixel_shuffle(scale). The last block's c1 is recomputed as a plain conv for the
    concat, as the reference's lowering does (23 steps for 6 blocks)."""
    rng = np.random.default_rng(seed)
    steps, channels = [], []

    def bias(n):
        return rng.normal(0.0, 0.01, size=n).astype(np.float32)

    def new_feat():
        channels.append(c)
        return len(channels) - 1

    feat = new_feat()
    steps.append(_conv_step(_he(rng, 3, c), bias(c), in_=IN_NCHW3, src=MODEL_INPUT, dst=feat))
    x, out_b1, mid = feat, None, None
    for b in range(blocks):
        w1, b1 = _he(rng, c, c), bias(c)
        if b == blocks - 1:
            mid = new_feat()
            steps.append(_conv_step(w1, b1, src=x, dst=mid))
        a1 = new_feat()
        steps.append(_conv_step(w1, b1, act=ACT_SILU, src=x, dst=a1))
        a2 = new_feat()
        steps.append(_conv_step(_he(rng, c, c), bias(c), act=ACT_SILU, src=a1, dst=a2))
        o = new_feat()
        steps.append(_conv_step(_he(rng, c, c), bias(c), gate=GATE_SIGMOID_HALF, src=a2, resid=x, dst=o))
        x = o
        if b == 0:
            out_b1 = o
    o2 = new_feat()
    steps.append(_conv_step(_he(rng, c, c), bias(c), src=x, dst=o2))
    cat = new_feat()
    steps.append(_concat_step(_he(rng, 4 * c, c, taps=1), bias(c), [feat, o2, out_b1, mid], c, cat))
    out_mode = {1: OUT_D2S1, 2: OUT_D2S2, 3: OUT_D2S3, 4: OUT_D2S4}[scale]
    steps.append(_conv_step(_he(rng, c, 3 * scale * scale), bias(3 * scale * scale), out=out_mode, src=cat,
                            dst=MODEL_OUTPUT))
    return dict(name=name or f"span-{c}x{blocks}-{scale}x", steps=steps, channels=channels, depth_to_space=scale)


def spanf3_plan(seed, c=48, blocks=5, name=None, gain=1.0):
    """SPANF3 2x with the 2x pixel-unshuffled input (the shipping AnimeJaNai V3.1 HD Performance /
    Balanced structure, b5f48 / b8f64): conv_first 12->c at half resolution; `blocks` blocks of
    c1+ReLU, c2+ReLU, c3 with the tanh gate (c3 + x) * tanh(att(c3)), att a 1x1 c->c conv; concat
    [feat, last block, first block, the last block's ReLU(c1)] -> 1x1 4c->c; c->48 3x3;
    depth-to-space 4 (2x overall). The plan the reference's lowering gives such a graph
    (sanity/native_lower_test.cpp spanf3: 3 * blocks + 3 steps). gain scales every He-init weight
    (below 1 the random net stays well-conditioned at depth: 8 blocks of 64 at gain 1 amplify a
    one-ulp input change a hundredfold)."""
    rng = np.random.default_rng(seed)
    steps, channels = [], []

    def _he(rng_, cin, cout, taps=9):
        w = rng_.normal(0.0, gain * np.sqrt(2.0 / (taps * cin)), size=(taps, cin, cout))
        return w.astype(np.float16).astype(np.float32)

    def bias(n):
        return rng.normal(0.0, 0.01, size=n).astype(np.float32)

    def new_feat():
        channels.append(c)
        return len(channels) - 1

    feat = new_feat()
    steps.append(_conv_step(_he(rng, 12, c), bias(c), in_=IN_NCHW3_UNSHUFFLE2, src=MODEL_INPUT, dst=feat))
    x, out_b1, mid = feat, None, None
    for b in range(blocks):
        a1 = new_feat()
        steps.append(_conv_step(_he(rng, c, c), bias(c), act=ACT_RELU, src=x, dst=a1))
        a2 = new_feat()
        steps.append(_conv_step(_he(rng, c, c), bias(c), act=ACT_RELU, src=a1, dst=a2))
        o = new_feat()
        st = _conv_step(_he(rng, c, c), bias(c), gate=GATE_TANH1X1, src=a2, resid=x, dst=o)
        st["att"] = (_he(rng, c, c, taps=1), bias(c))
        steps.append(st)
        x, mid = o, a1
        if b == 0:
            out_b1 = o
    cat = new_feat()
    steps.append(_concat_step(_he(rng, 4 * c, c, taps=1), bias(c), [feat, x, out_b1, mid], c, cat))
    steps.append(_conv_step(_he(rng, c, 48), bias(48), out=OUT_D2S4, src=cat, dst=MODEL_OUTPUT))
    return dict(name=name or f"spanf3-{c}x{blocks}-unshuffle", steps=steps, channels=channels, depth_to_space=4,
                unshuffle=2)
