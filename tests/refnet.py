"""The reference's own CPU reference net (sanity/native_ref.h:run_plan), compiled from the
reference sources into oracle/_ref/libref_net.so by oracle/ref/build.sh, driven from a plan dict.
Test and CPU-baseline infrastructure only."""
import ctypes as C

import numpy as np

MODEL_INPUT, MODEL_OUTPUT = -2, -3
_libs = {}


class RefStep(C.Structure):
    _fields_ = [("kind", C.c_int), ("in_", C.c_int), ("act", C.c_int), ("gate", C.c_int), ("out", C.c_int),
                ("cin", C.c_int), ("cout", C.c_int), ("src", C.c_int), ("resid", C.c_int), ("dst", C.c_int),
                ("c", C.c_int), ("nsrc", C.c_int), ("srcs", C.c_int * 4), ("taps", C.c_int),
                ("w", C.c_void_p), ("bias", C.c_void_p), ("slope", C.c_void_p), ("att_w", C.c_void_p),
                ("att_bias", C.c_void_p)]


def _lib(path):
    if path not in _libs:
        lib = C.CDLL(path)
        lib.ref_run_plan.argtypes = [C.POINTER(RefStep), C.c_int, C.POINTER(C.c_int), C.c_int, C.c_int, C.c_int,
                                     C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        lib.ref_run_plan.restype = C.c_int
        lib.ref_threads.restype = C.c_int
        _libs[path] = lib
    return _libs[path]


def threads(path, nthreads=0):
    return _lib(path).ref_threads()


def plan_struct(plan):
    """The plan as the shims' ref_step array (oracle/ref/refplan.h) and the channel list; the third
    element keeps the weight arrays alive while the structures point at them."""
    keep = []
    steps = (RefStep * len(plan["steps"]))()
    for i, s in enumerate(plan["steps"]):
        r = steps[i]
        w = np.ascontiguousarray(np.asarray(s["w"], np.float32).astype(np.float16).view(np.uint16))
        b = np.ascontiguousarray(s["bias"], np.float32)
        sl = None if s.get("slope") is None else np.ascontiguousarray(s["slope"], np.float32)
        keep += [w, b, sl]
        r.kind = s["kind"]
        r.in_, r.act, r.gate, r.out = s.get("in_", 0), s.get("act", 0), s.get("gate", 0), s.get("out", 0)
        r.cin, r.cout = s.get("cin", 0), s.get("cout", 0)
        r.src, r.resid, r.dst = s.get("src", -1), s.get("resid", -1), s["dst"]
        r.c, r.nsrc = s.get("c", 0), s.get("nsrc", 0)
        srcs = list(s.get("srcs", [])) + [-1] * (4 - len(s.get("srcs", [])))
        for k in range(4):
            r.srcs[k] = srcs[k]
        r.taps = w.shape[0]
        r.w, r.bias = w.ctypes.data, b.ctypes.data
        r.slope = None if sl is None else sl.ctypes.data
        r.att_w = r.att_bias = None
        if s.get("gate", 0) == 2:
            aw = np.ascontiguousarray(np.asarray(s["att"][0], np.float32).astype(np.float16).view(np.uint16))
            ab = np.ascontiguousarray(s["att"][1], np.float32)
            keep += [aw, ab]
            r.att_w, r.att_bias = aw.ctypes.data, ab.ctypes.data
    ch = (C.c_int * len(plan["channels"]))(*plan["channels"])
    return steps, ch, keep


def run_plan(path, plan, x, nthreads=0):
    """x: NCHW float32 [3][h][w]. Returns the reference's NCHW output [3][R*h/u][R*w/u]."""
    lib = _lib(path)
    steps, ch, keep = plan_struct(plan)
    x = np.ascontiguousarray(x, np.float32)
    _, h, wd = x.shape
    R, u = plan["depth_to_space"], plan.get("unshuffle", 1)
    out = np.zeros((3, R * h // u, R * wd // u), np.float32)
    rc = lib.ref_run_plan(steps, len(plan["steps"]), ch, len(plan["channels"]), R, u, x.ctypes.data, wd, h,
                          out.ctypes.data)
    assert rc == 0
    return out


class RefExec:
    """The reference's own GPU executor (src/native/executor.cpp, its k_conv3x3 / k_concat1x1
    kernels for sm_100a) for a plan at w x h, from oracle/_ref/libref_exec.so."""

    def __init__(self, path, plan, w, h, stream=None):
        lib = C.CDLL(path)
        lib.ref_exec_create.restype = C.c_void_p
        lib.ref_exec_create.argtypes = [C.POINTER(RefStep), C.c_int, C.POINTER(C.c_int), C.c_int, C.c_int, C.c_int,
                                        C.c_int, C.c_int, C.c_void_p, C.c_char_p, C.c_int]
        lib.ref_exec_run.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        lib.ref_exec_run.restype = C.c_int
        lib.ref_exec_release.argtypes = [C.c_void_p]
        self.lib = lib
        steps, ch, keep = plan_struct(plan)
        err = C.create_string_buffer(512)
        self.handle = lib.ref_exec_create(steps, len(plan["steps"]), ch, len(plan["channels"]), plan["depth_to_space"],
                                          plan.get("unshuffle", 1), w, h, stream, err, 512)
        if not self.handle:
            raise RuntimeError("reference executor refused the plan: " + err.value.decode())

    def run(self, src, dst, stream=None):
        return self.lib.ref_exec_run(self.handle, src, dst, stream)

    def close(self):
        if self.handle:
            self.lib.ref_exec_release(self.handle)
            self.handle = None
