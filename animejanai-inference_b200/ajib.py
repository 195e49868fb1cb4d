"""ctypes binding of libaji.so (include/aji.h, include/aji_image.h, include/aji_b200.h).

This is how the tests and bench.py call the engine: through the same C ABI a player or image
tool binds (the reference's callers load libaji.so with dlopen/dlsym; see INTEGRATION.md for the
cgo/ctypes stubs). Device buffers are passed as integer device addresses (from torch tensors in
the tests). There is no fallback: importing this module without the built library raises.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libaji.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is not built: run __graft_entry__.build() (make -C csrc)")

lib = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)

# ---- status codes (aji_b200.h) ----
AJIB_OK, AJIB_ERR, AJIB_ERR_ARGS, AJIB_ERR_UNSUPPORTED, AJIB_ERR_CUDA, AJIB_ERR_NO_MEM, AJIB_ERR_TIMEOUT = (
    0, -1, -2, -3, -4, -5, -6)

# op vocabulary (reference src/native/ops.h:13-21)
IN_NHWC, IN_NCHW3 = 0, 1
ACT_NONE, ACT_RELU, ACT_PRELU, ACT_SILU = 0, 1, 2, 3
GATE_NONE, GATE_RESIDUAL, GATE_TANH1X1, GATE_SIGMOID_HALF = 0, 1, 2, 3
OUT_NHWC, OUT_D2S2, OUT_D2S4, OUT_D2S1, OUT_D2S3 = 0, 1, 2, 3, 4
D2S_FACTOR = {OUT_NHWC: 0, OUT_D2S2: 2, OUT_D2S4: 4, OUT_D2S1: 1, OUT_D2S3: 3}


class ConvOp(C.Structure):
    """struct ajib_conv (aji_b200.h)."""
    _fields_ = [
        ("in_", C.c_int), ("act", C.c_int), ("gate", C.c_int), ("out", C.c_int),
        ("cin", C.c_int), ("cout", C.c_int),
        ("w", C.c_void_p), ("att", C.c_void_p),
        ("in_norm", C.c_int), ("in_mean", C.c_float * 3), ("in_scale", C.c_float * 3),
        ("out_clamp", C.c_int),
    ]


_vp = C.c_void_p
lib.ajib_weights_upload.argtypes = [C.POINTER(_vp), _vp, _vp, _vp, C.c_int, C.c_int, C.c_int]
lib.ajib_weights_upload.restype = C.c_int
lib.ajib_weights_release.argtypes = [C.POINTER(_vp)]
lib.ajib_weights_release.restype = None
lib.ajib_weights_bytes.argtypes = [_vp]
lib.ajib_weights_bytes.restype = C.c_size_t
lib.ajib_conv_supported.argtypes = [C.POINTER(ConvOp), C.c_char_p, C.c_size_t]
lib.ajib_conv_supported.restype = C.c_int
lib.ajib_conv3x3_launch.argtypes = [C.POINTER(ConvOp), _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp]
lib.ajib_conv3x3_launch.restype = C.c_int
lib.ajib_kernel_status.argtypes = [C.c_int]
lib.ajib_kernel_status.restype = C.c_int
lib.ajib_selftest_umma.argtypes = [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _vp, _vp]
lib.ajib_selftest_umma.restype = C.c_int


class AjibError(RuntimeError):
    pass


def check(rc, what):
    if rc != AJIB_OK:
        raise AjibError(f"{what} failed with status {rc}")
    return rc


class Weights:
    """Packed conv weights on the current device (ajib_weights_upload)."""

    def __init__(self, w_f16_bits, bias, slope=None, taps=9):
        import numpy as np
        w = np.ascontiguousarray(w_f16_bits, dtype=np.uint16)
        b = np.ascontiguousarray(bias, dtype=np.float32)
        s = None if slope is None else np.ascontiguousarray(slope, dtype=np.float32)
        cin, cout = w.shape[-2], w.shape[-1]
        self.handle = _vp()
        check(lib.ajib_weights_upload(C.byref(self.handle), w.ctypes.data, b.ctypes.data,
                                      None if s is None else s.ctypes.data, taps, cin, cout),
              "ajib_weights_upload")
        self.cin, self.cout, self.taps = cin, cout, taps

    def release(self):
        if self.handle:
            lib.ajib_weights_release(C.byref(self.handle))

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


def conv_op(w, in_=IN_NHWC, act=ACT_NONE, gate=GATE_NONE, out=OUT_NHWC, in_norm=None, out_clamp=False):
    op = ConvOp()
    op.in_, op.act, op.gate, op.out = in_, act, gate, out
    op.cin, op.cout = w.cin, w.cout
    op.w = w.handle
    op.att = None
    if in_norm is not None:
        op.in_norm = 1
        mean, scale = in_norm
        for i in range(3):
            op.in_mean[i] = mean[i]
            op.in_scale[i] = scale[i]
    else:
        op.in_norm = 0
        for i in range(3):
            op.in_mean[i] = 0.0
            op.in_scale[i] = 1.0
    op.out_clamp = 1 if out_clamp else 0
    # the op holds only the raw handle: keep the Weights (which frees the device copy when it is
    # collected) alive as long as the op
    op._weights = w
    return op


def supported(op):
    why = C.create_string_buffer(256)
    ok = lib.ajib_conv_supported(C.byref(op), why, 256)
    return bool(ok), why.value.decode()


def conv3x3(op, src, resid, dst, H, W, row_begin=0, row_end=0, stream=0):
    return lib.ajib_conv3x3_launch(C.byref(op), src, resid, dst, H, W, row_begin, row_end, stream)


def kernel_status(clear=True):
    return lib.ajib_kernel_status(1 if clear else 0)
