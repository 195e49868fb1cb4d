"""ctypes binding of libaji.so (include/aji.h, include/aji_image.h, include/aji_b200.h).

This is how the tests and bench.py call the engine: through the same C ABI a player or image
tool binds (the reference's callers load libaji.so with dlopen/dlsym). Device buffers are passed
as integer device addresses (from torch tensors in the tests). There is no fallback: importing
this module without the built library raises.
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
IN_NHWC, IN_NCHW3, IN_NCHW3_UNSHUFFLE2 = 0, 1, 2
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
lib.ajib_conv3x3_launch_images.argtypes = [C.POINTER(ConvOp), _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                           _vp]
lib.ajib_conv3x3_launch_images.restype = C.c_int
lib.ajib_feature_strips.argtypes = [C.c_int]
lib.ajib_feature_strips.restype = C.c_int
lib.ajib_feature_bytes.argtypes = [C.c_int, C.c_int, C.c_int]
lib.ajib_feature_bytes.restype = C.c_size_t
lib.ajib_kernel_status.argtypes = [C.c_int]
lib.ajib_kernel_status.restype = C.c_int
lib.ajib_conv_pair_mode.argtypes = [C.c_int]
lib.ajib_conv_pair_mode.restype = C.c_int
lib.ajib_conv_on_pairs.argtypes = [C.POINTER(ConvOp)]
lib.ajib_conv_on_pairs.restype = C.c_int
lib.ajib_conv_pair_clusters.argtypes = []
lib.ajib_conv_pair_clusters.restype = C.c_int
lib.ajib_selftest_umma.argtypes = [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _vp, _vp]
lib.ajib_selftest_umma.restype = C.c_int
lib.ajib_selftest_division.argtypes = [_vp, C.c_int, _vp, _vp]
lib.ajib_selftest_division.restype = C.c_int
lib.ajib_selftest_division_by.argtypes = [_vp, C.c_int, _vp, _vp]
lib.ajib_selftest_division_by.restype = C.c_int


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


def conv_op(w, in_=IN_NHWC, act=ACT_NONE, gate=GATE_NONE, out=OUT_NHWC, in_norm=None, out_clamp=False, att=None):
    """att: the tanh gate's 1x1 attention Weights (taps 1, cout -> cout)."""
    op = ConvOp()
    op.in_, op.act, op.gate, op.out = in_, act, gate, out
    op.cin, op.cout = w.cin, w.cout
    op.w = w.handle
    op.att = None if att is None else att.handle
    op._att = att
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


lib.ajib_concat1x1_launch.argtypes = [_vp, C.c_int, C.POINTER(_vp), C.c_int, _vp, C.c_int, C.c_int, C.c_int, C.c_int,
                                      _vp]
lib.ajib_concat1x1_launch.restype = C.c_int


def concat1x1(w, srcs, c, dst, H, W, row_begin=0, row_end=0, stream=0):
    """SPAN's concat + 1x1 conv on strip-chunked maps (ajib_concat1x1_launch); w: Weights(taps=1)."""
    arr = (_vp * len(srcs))(*srcs)
    return lib.ajib_concat1x1_launch(w.handle, len(srcs), arr, c, dst, H, W, row_begin, row_end, stream)


def conv3x3_images(op, src, resid, dst, nimg, img_h, W, row_begin=0, row_end=0, stream=0):
    return lib.ajib_conv3x3_launch_images(C.byref(op), src, resid, dst, nimg, img_h, W, row_begin, row_end, stream)


def kernel_status(clear=True):
    return lib.ajib_kernel_status(1 if clear else 0)


def pair_mode(mode=-1):
    """Whether eligible convs run on SM pairs (ajib_conv_pair_mode): 1 / 0 sets, -1 queries;
    returns the mode in force."""
    return lib.ajib_conv_pair_mode(mode)


def on_pairs(op):
    """True when op runs on the SM-pair kernel in the current mode (ajib_conv_on_pairs)."""
    return bool(lib.ajib_conv_on_pairs(C.byref(op)))


# ---------------------------------------------------------------------------------------------
# native model files and the seeded BASELINE architectures live in ajib_plans (pure numpy, no
# library load); re-exported here for callers of this binding.
from ajib_plans import (MODEL_INPUT, MODEL_OUTPUT, compact_plan, model_bytes, parse_model_bytes,  # noqa: E402,F401
                        span_plan, spanf3_plan)


def model_from_bytes(b):
    """ajib_model_from_memory on native or ONNX bytes; returns the model's native file bytes."""
    h = _vp()
    err = C.create_string_buffer(512)
    rc = lib.ajib_model_from_memory(b, len(b), C.byref(h), err, 512)
    if rc != 0:
        raise AjibError(err.value.decode())
    n = C.c_size_t()
    lib.ajib_model_save(h, None, 0, C.byref(n))
    buf = C.create_string_buffer(n.value)
    assert lib.ajib_model_save(h, buf, n.value, C.byref(n)) == 0
    lib.ajib_model_release(C.byref(h))
    return buf.raw[:n.value]


lib.ajib_model_load.argtypes = [C.c_char_p, C.POINTER(_vp), C.c_char_p, C.c_size_t]
lib.ajib_model_load.restype = C.c_int
lib.ajib_model_from_memory.argtypes = [C.c_char_p, C.c_size_t, C.POINTER(_vp), C.c_char_p, C.c_size_t]
lib.ajib_model_from_memory.restype = C.c_int
lib.ajib_model_release.argtypes = [C.POINTER(_vp)]
lib.ajib_model_release.restype = None
lib.ajib_model_info.argtypes = [_vp, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_double), C.c_char_p,
                                C.c_size_t]
lib.ajib_model_info.restype = C.c_int
lib.ajib_exec_create.argtypes = [_vp, C.c_int, C.c_int, C.POINTER(_vp), C.c_char_p, C.c_size_t]
lib.ajib_exec_create.restype = C.c_int
lib.ajib_exec_release.argtypes = [C.POINTER(_vp)]
lib.ajib_exec_release.restype = None
lib.ajib_exec_run.argtypes = [_vp, _vp, _vp, _vp]
lib.ajib_exec_run.restype = C.c_int
lib.ajib_exec_profile.argtypes = [_vp, C.c_int]
lib.ajib_exec_profile.restype = C.c_int
lib.ajib_exec_profile_read.argtypes = [_vp, C.POINTER(C.c_double), C.POINTER(C.c_int), C.c_int]
lib.ajib_exec_profile_read.restype = C.c_int
lib.ajib_exec_run_images.argtypes = [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _vp]
lib.ajib_exec_run_images.restype = C.c_int
lib.ajib_exec_set_bands.argtypes = [_vp, C.c_int]
lib.ajib_exec_set_bands.restype = C.c_int
lib.ajib_exec_info.argtypes = [_vp, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t), C.POINTER(C.c_int)]
lib.ajib_exec_info.restype = C.c_int


class Model:
    def __init__(self, plan=None, path=None):
        self.handle = _vp()
        err = C.create_string_buffer(512)
        if path is not None:
            rc = lib.ajib_model_load(path.encode(), C.byref(self.handle), err, 512)
        else:
            data = model_bytes(plan)
            rc = lib.ajib_model_from_memory(data, len(data), C.byref(self.handle), err, 512)
        if rc != AJIB_OK:
            raise AjibError(f"model load failed: {err.value.decode()}")
        scale, steps, fpp = C.c_int(), C.c_int(), C.c_double()
        desc = C.create_string_buffer(256)
        lib.ajib_model_info(self.handle, C.byref(scale), C.byref(steps), C.byref(fpp), desc, 256)
        self.scale, self.steps, self.flops_per_px, self.desc = scale.value, steps.value, fpp.value, desc.value.decode()

    def __del__(self):
        try:
            if self.handle:
                lib.ajib_model_release(C.byref(self.handle))
        except Exception:
            pass


class Exec:
    def __init__(self, model, w, h, bands=1):
        self.handle = _vp()
        self.model = model
        err = C.create_string_buffer(512)
        rc = lib.ajib_exec_create(model.handle, w, h, C.byref(self.handle), err, 512)
        if rc != AJIB_OK:
            raise AjibError(f"executor creation failed: {err.value.decode()}")
        if bands != 1:
            check(lib.ajib_exec_set_bands(self.handle, bands), "ajib_exec_set_bands")
        self.w, self.h = w, h

    def run(self, src, dst, stream=0):
        return lib.ajib_exec_run(self.handle, src, dst, stream)

    def run_images(self, src, dst, w, img_h, nimg, stream=0):
        return lib.ajib_exec_run_images(self.handle, src, dst, w, img_h, nimg, stream)

    def profile(self, on):
        return lib.ajib_exec_profile(self.handle, 1 if on else 0)

    def profile_read(self, nsteps):
        import numpy as np
        ms = np.zeros(nsteps)
        n = np.zeros(nsteps, np.int32)
        check(lib.ajib_exec_profile_read(self.handle, ms.ctypes.data_as(C.POINTER(C.c_double)),
                                         n.ctypes.data_as(C.POINTER(C.c_int)), nsteps), "ajib_exec_profile_read")
        return ms, n

    def info(self):
        a, b, n = C.c_size_t(), C.c_size_t(), C.c_int()
        lib.ajib_exec_info(self.handle, C.byref(a), C.byref(b), C.byref(n))
        return dict(device_bytes=a.value, weight_bytes=b.value, launches=n.value)

    def __del__(self):
        try:
            if self.handle:
                lib.ajib_exec_release(C.byref(self.handle))
        except Exception:
            pass


# ---------------------------------------------------------------------------------------------
# the video ABI (include/aji.h)

AJI_API_VERSION = 9
FMT_NV12, FMT_P010, FMT_YUV444P16, FMT_RGB10A2, FMT_YUV444P10MSB, FMT_YUV444P12MSB = 1, 2, 3, 4, 5, 6
MATRIX_BT601, MATRIX_BT709, MATRIX_BT2020 = 1, 2, 3
RANGE_LIMITED, RANGE_FULL = 1, 2
SITING_LEFT, SITING_CENTER, SITING_TOPLEFT = 1, 2, 3
AJI_OK, AJI_ERR = 0, -1

LOG_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_int, C.c_char_p)


class CreateParams(C.Structure):
    _fields_ = [("api_version", C.c_uint32), ("cuda_context", C.c_void_p), ("conf_path", C.c_char_p),
                ("model_dir", C.c_char_p), ("trtexec", C.c_char_p), ("trtexec_env", C.c_char_p), ("slot", C.c_int),
                ("rife_model_dir", C.c_char_p), ("async_build", C.c_int), ("d3d11_device", C.c_void_p),
                ("engine_path", C.c_char_p), ("max_width", C.c_int), ("max_height", C.c_int), ("log", LOG_FN),
                ("log_opaque", C.c_void_p)]


class Frame(C.Structure):
    _fields_ = [("width", C.c_int), ("height", C.c_int), ("format", C.c_int), ("matrix", C.c_int), ("range", C.c_int),
                ("siting", C.c_int), ("plane", C.c_void_p * 3), ("stride", C.c_ssize_t * 3)]


def frame(w, h, fmt, planes, strides, matrix=MATRIX_BT709, range_=RANGE_LIMITED, siting=SITING_LEFT):
    f = Frame()
    f.width, f.height, f.format, f.matrix, f.range, f.siting = w, h, fmt, matrix, range_, siting
    for i in range(3):
        f.plane[i] = planes[i] if i < len(planes) else None
        f.stride[i] = strides[i] if i < len(strides) else 0
    return f


lib.aji_create.argtypes = [C.POINTER(CreateParams)]
lib.aji_create.restype = C.c_void_p
lib.aji_configure.argtypes = [_vp, C.c_int, C.c_int, C.c_double, C.POINTER(C.c_int), C.POINTER(C.c_int)]
lib.aji_configure.restype = C.c_int
lib.aji_infer.argtypes = [_vp, C.POINTER(Frame), C.POINTER(Frame), _vp]
lib.aji_infer.restype = C.c_int
lib.aji_flush.argtypes = [_vp, _vp]
lib.aji_flush.restype = C.c_uint64
lib.aji_done.argtypes = [_vp, C.c_uint64]
lib.aji_done.restype = C.c_int
lib.aji_wait.argtypes = [_vp, C.c_uint64]
lib.aji_wait.restype = C.c_int
lib.aji_last_error.argtypes = [_vp]
lib.aji_last_error.restype = C.c_char_p
lib.aji_current_log.argtypes = [_vp]
lib.aji_current_log.restype = C.c_char_p
lib.aji_scale_factor.argtypes = [_vp]
lib.aji_scale_factor.restype = C.c_int
lib.aji_destroy.argtypes = [C.POINTER(_vp)]
lib.aji_destroy.restype = None


class Video:
    """A direct-mode aji_ctx on a native model file."""

    def __init__(self, model_path, max_w, max_h, cuda_context=None):
        p = CreateParams()
        p.api_version = AJI_API_VERSION
        p.cuda_context = cuda_context
        p.engine_path = model_path.encode()
        p.max_width, p.max_height = max_w, max_h
        self._p = p
        h = lib.aji_create(C.byref(p))
        if not h:
            raise AjibError("aji_create failed")
        self.handle = _vp(h)

    @classmethod
    def from_conf(cls, conf_path, model_dir=None, slot=1, cuda_context=None):
        """A conf-mode aji_ctx: animejanai.conf chains of native model files (<model_dir>/<name>.ajnm)."""
        self = cls.__new__(cls)
        p = CreateParams()
        p.api_version = AJI_API_VERSION
        p.cuda_context = cuda_context
        p.conf_path = conf_path.encode()
        p.model_dir = None if model_dir is None else model_dir.encode()
        p.slot = slot
        self._p = p
        h = lib.aji_create(C.byref(p))
        if not h:
            raise AjibError("aji_create (conf mode) failed")
        self.handle = _vp(h)
        return self

    def configure(self, w, h, fps=24.0, allow_passthrough=False):
        ow, oh = C.c_int(), C.c_int()
        rc = lib.aji_configure(self.handle, w, h, fps, C.byref(ow), C.byref(oh))
        if rc != 1 and not (allow_passthrough and rc == 0):
            raise AjibError(f"aji_configure: {rc} {self.error()}")
        return ow.value, oh.value

    def log(self):
        return (lib.aji_current_log(self.handle) or b"").decode()

    def resize_frame(self, fin, fout, stream=0):
        return lib.aji_resize_frame(self.handle, C.byref(fin), C.byref(fout), stream)

    def infer(self, fin, fout, stream=0):
        return lib.aji_infer(self.handle, C.byref(fin), C.byref(fout), stream)

    def flush(self, stream=0):
        return lib.aji_flush(self.handle, stream)

    def wait(self, ticket):
        return lib.aji_wait(self.handle, ticket)

    def error(self):
        return (lib.aji_last_error(self.handle) or b"").decode()

    def close(self):
        if self.handle:
            lib.aji_destroy(C.byref(self.handle))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


lib.ajib_video_create_multi.argtypes = [C.POINTER(CreateParams), C.POINTER(C.c_int), C.c_int, C.c_int, C.c_char_p,
                                        C.c_size_t]
lib.ajib_video_create_multi.restype = C.c_void_p
lib.ajib_video_multi_configure.argtypes = [_vp, C.c_int, C.c_int, C.c_double, C.POINTER(C.c_int), C.POINTER(C.c_int)]
lib.ajib_video_multi_configure.restype = C.c_int
lib.ajib_video_multi_submit.argtypes = [_vp, C.POINTER(Frame), C.POINTER(Frame)]
lib.ajib_video_multi_submit.restype = C.c_int64
lib.ajib_video_multi_wait.argtypes = [_vp, C.c_int64]
lib.ajib_video_multi_wait.restype = C.c_int
lib.ajib_video_multi_done.argtypes = [_vp, C.c_int64]
lib.ajib_video_multi_done.restype = C.c_int
lib.ajib_video_multi_devices.argtypes = [_vp]
lib.ajib_video_multi_devices.restype = C.c_int
lib.ajib_video_multi_error.argtypes = [_vp]
lib.ajib_video_multi_error.restype = C.c_char_p
lib.ajib_video_multi_destroy.argtypes = [C.POINTER(_vp)]
lib.ajib_video_multi_destroy.restype = None
lib.ajib_video_multi_timing.argtypes = [_vp, C.c_int]
lib.ajib_video_multi_timing.restype = C.c_int
lib.ajib_video_multi_device_ms.argtypes = [_vp, C.POINTER(C.c_double), C.c_int]
lib.ajib_video_multi_device_ms.restype = C.c_int
lib.ajib_selftest_frame_order.argtypes = [C.c_int, C.c_int, C.c_int, _vp, _vp, _vp, _vp, _vp]
lib.ajib_selftest_frame_order.restype = C.c_int


class VideoMulti:
    """One stream over several GPUs (ajib_video_create_multi): host frames in and out, frame k on
    device k mod n, results in submission order. model_path: direct mode; conf_path: conf mode."""

    def __init__(self, devices, model_path=None, max_w=0, max_h=0, conf_path=None, model_dir=None, slot=1, depth=2):
        p = CreateParams()
        p.api_version = AJI_API_VERSION
        if conf_path is not None:
            p.conf_path = conf_path.encode()
            p.model_dir = None if model_dir is None else model_dir.encode()
            p.slot = slot
        else:
            p.engine_path = model_path.encode()
            p.max_width, p.max_height = max_w, max_h
        self._p = p
        ids = (C.c_int * len(devices))(*devices)
        err = C.create_string_buffer(512)
        h = lib.ajib_video_create_multi(C.byref(p), ids, len(devices), depth, err, 512)
        if not h:
            raise AjibError("ajib_video_create_multi: " + err.value.decode())
        self.handle = _vp(h)

    def configure(self, w, h, fps=24.0):
        ow, oh = C.c_int(), C.c_int()
        rc = lib.ajib_video_multi_configure(self.handle, w, h, fps, C.byref(ow), C.byref(oh))
        if rc != 0:
            raise AjibError(f"ajib_video_multi_configure: {rc} {self.error()}")
        return ow.value, oh.value

    def submit(self, fin, fout):
        return lib.ajib_video_multi_submit(self.handle, C.byref(fin), C.byref(fout))

    def wait(self, ticket):
        return lib.ajib_video_multi_wait(self.handle, ticket)

    def done(self, ticket):
        return lib.ajib_video_multi_done(self.handle, ticket)

    def timing(self, on):
        return lib.ajib_video_multi_timing(self.handle, 1 if on else 0)

    def device_ms(self):
        n = lib.ajib_video_multi_devices(self.handle)
        ms = (C.c_double * n)()
        check(lib.ajib_video_multi_device_ms(self.handle, ms, n), "ajib_video_multi_device_ms")
        return list(ms)

    def error(self):
        return (lib.ajib_video_multi_error(self.handle) or b"").decode()

    def close(self):
        if self.handle:
            lib.ajib_video_multi_destroy(C.byref(self.handle))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def frame_order(ndev, depth, finish_order):
    """ajib_selftest_frame_order: (device_of, slot_of, reuse_of, completed_after)."""
    import numpy as np
    n = len(finish_order)
    fo = np.ascontiguousarray(finish_order, np.int64)
    dev = np.zeros(n, np.int32)
    slot = np.zeros(n, np.int32)
    reuse = np.zeros(n, np.int64)
    comp = np.zeros(n, np.int64)
    check(lib.ajib_selftest_frame_order(ndev, depth, n, fo.ctypes.data, dev.ctypes.data, slot.ctypes.data,
                                        reuse.ctypes.data, comp.ctypes.data), "ajib_selftest_frame_order")
    return dev, slot, reuse, comp


# colour passes (aji_b200.h, named as the reference's src/kernels.h)
class Csp(C.Structure):
    _fields_ = [("kr", C.c_float), ("kb", C.c_float), ("yoff", C.c_float), ("yscale", C.c_float), ("coff", C.c_float),
                ("cscale", C.c_float)]


lib.aji_make_csp.argtypes = [C.c_int, C.c_int, C.c_int]
lib.aji_make_csp.restype = Csp
for _n in ("aji_pre_plan_create", "aji_post_plan_create"):
    getattr(lib, _n).argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
    getattr(lib, _n).restype = C.c_void_p
lib.aji_plan_destroy.argtypes = [_vp]
lib.aji_plan_destroy.restype = None
lib.aji_run_pre.argtypes = [_vp, _vp, C.c_ssize_t, _vp, C.c_ssize_t, C.POINTER(Csp), _vp, _vp]
lib.aji_run_pre.restype = C.c_int
lib.aji_run_post.argtypes = [_vp, _vp, C.POINTER(Csp), _vp, C.c_ssize_t, _vp, C.c_ssize_t, _vp]
lib.aji_run_post.restype = C.c_int
lib.aji_run_post444.argtypes = [C.c_int, C.c_int, C.c_int, _vp, C.POINTER(Csp), _vp, C.c_ssize_t, _vp, C.c_ssize_t,
                                _vp, C.c_ssize_t, _vp]
lib.aji_run_post444.restype = C.c_int
lib.aji_run_pre444.argtypes = [C.c_int, C.c_int, _vp, C.c_ssize_t, _vp, C.c_ssize_t, _vp, C.c_ssize_t, C.POINTER(Csp),
                               _vp, _vp]
lib.aji_run_pre444.restype = C.c_int
lib.ajib_plan_table.argtypes = [_vp, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_float), C.c_int]
lib.ajib_plan_table.restype = C.c_int
lib.ajib_plan_kernel.argtypes = [_vp]
lib.ajib_plan_kernel.restype = C.c_int
lib.ajib_filter_table.argtypes = [C.c_int, C.c_int, C.c_double, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_float)]
lib.ajib_filter_table.restype = C.c_int


def filter_table(src, dst, shift, filt=0):
    import numpy as np
    taps = lib.ajib_filter_table(src, dst, shift, filt, None, None)
    start = np.zeros(dst, np.int32)
    wt = np.zeros(dst * taps, np.float32)
    lib.ajib_filter_table(src, dst, shift, filt, start.ctypes.data_as(C.POINTER(C.c_int)),
                          wt.ctypes.data_as(C.POINTER(C.c_float)))
    return taps, start, wt.reshape(dst, taps)


# ---------------------------------------------------------------------------------------------
# the image ABI (include/aji_image.h) and the GPU tiler (aji_b200.h, ajib_tiler_*)

AJI_IMAGE_API_VERSION = 1
IMG_TENSORRT, IMG_DIRECTML, IMG_TENSORRT_RTX, IMG_VULKAN = 1, 2, 3, 4
IMG_OK, IMG_ERR, IMG_ERR_ARGS, IMG_NOT_READY, IMG_CANCELLED, IMG_ERR_NO_MEM = 0, -1, -2, -3, -4, -5
IMG_LOAD_EVEN_TILES = 2
IMG_LOG_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_int, C.c_char_p)
PROGRESS_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int, C.c_int)


class ImgDevice(C.Structure):
    _fields_ = [("id", C.c_uint64), ("name", C.c_char * 128), ("vram_bytes", C.c_uint64), ("sm_major", C.c_int),
                ("sm_minor", C.c_int)]


class ImgCreateParams(C.Structure):
    _fields_ = [("api_version", C.c_uint32), ("backend", C.c_int), ("device_id", C.c_uint64), ("cache_dir", C.c_char_p),
                ("trtexec", C.c_char_p), ("trtexec_env", C.c_char_p), ("log", IMG_LOG_FN), ("log_opaque", C.c_void_p)]


class ImgModelParams(C.Structure):
    _fields_ = [("onnx_path", C.c_char_p), ("tile_w", C.c_int), ("tile_h", C.c_int), ("overlap", C.c_int),
                ("flags", C.c_int)]


class ImgModelInfo(C.Structure):
    _fields_ = [("scale", C.c_int), ("in_channels", C.c_int), ("out_channels", C.c_int), ("tile_w", C.c_int),
                ("tile_h", C.c_int), ("overlap", C.c_int)]


class ImgBuffer(C.Structure):
    _fields_ = [("width", C.c_int), ("height", C.c_int), ("channels", C.c_int), ("stride", C.c_ssize_t),
                ("data", C.c_void_p)]


class ImgMemory(C.Structure):
    _fields_ = [("device_free", C.c_uint64), ("device_total", C.c_uint64), ("ctx_activations", C.c_uint64),
                ("ctx_scratch", C.c_uint64), ("model_weights", C.c_uint64), ("model_activations", C.c_uint64),
                ("model_buffers", C.c_uint64), ("activations_shared", C.c_int)]


lib.aji_img_enum_devices.argtypes = [C.c_int, C.POINTER(ImgDevice), C.c_int]
lib.aji_img_enum_devices.restype = C.c_int
lib.aji_img_create.argtypes = [C.POINTER(ImgCreateParams), C.c_char_p, C.c_size_t]
lib.aji_img_create.restype = C.c_void_p
lib.aji_img_load.argtypes = [_vp, C.POINTER(ImgModelParams)]
lib.aji_img_load.restype = C.c_void_p
lib.aji_img_model_state.argtypes = [_vp]
lib.aji_img_model_state.restype = C.c_int
lib.aji_img_model_info_get.argtypes = [_vp, C.POINTER(ImgModelInfo)]
lib.aji_img_model_info_get.restype = C.c_int
lib.aji_img_upscale.argtypes = [_vp, C.POINTER(ImgBuffer), C.POINTER(ImgBuffer), PROGRESS_FN, C.c_void_p]
lib.aji_img_upscale.restype = C.c_int
lib.aji_img_release.argtypes = [C.POINTER(_vp)]
lib.aji_img_release.restype = None
lib.aji_img_last_error.argtypes = [_vp]
lib.aji_img_last_error.restype = C.c_char_p
lib.aji_img_destroy.argtypes = [C.POINTER(_vp)]
lib.aji_img_destroy.restype = None
lib.aji_img_release_device.argtypes = [C.c_int, C.c_uint64]
lib.aji_img_release_device.restype = C.c_int
lib.aji_img_memory_get.argtypes = [_vp, _vp, C.POINTER(ImgMemory)]
lib.aji_img_memory_get.restype = C.c_int
lib.aji_img_native_probe.argtypes = [_vp, C.POINTER(ImgModelParams), C.POINTER(ImgMemory)]
lib.aji_img_native_probe.restype = C.c_int
lib.ajib_img_create_multi.argtypes = [C.POINTER(ImgCreateParams), C.POINTER(C.c_uint64), C.c_int, C.c_char_p, C.c_size_t]
lib.ajib_img_create_multi.restype = C.c_void_p
lib.ajib_model_save.argtypes = [_vp, _vp, C.c_size_t, C.POINTER(C.c_size_t)]
lib.ajib_model_save.restype = C.c_int
lib.ajib_tiler_create.argtypes = [C.c_int] * 8 + [C.POINTER(_vp)]
lib.ajib_tiler_create.restype = C.c_int
lib.ajib_tiler_info.argtypes = [_vp] + [C.POINTER(C.c_int)] * 4
lib.ajib_tiler_info.restype = C.c_int
lib.ajib_tiler_extract.argtypes = [_vp, _vp, C.c_int, C.c_int, _vp, _vp]
lib.ajib_tiler_extract.restype = C.c_int
lib.ajib_tiler_compose.argtypes = [_vp, _vp, _vp, _vp]
lib.ajib_tiler_compose.restype = C.c_int
lib.ajib_tiler_release.argtypes = [C.POINTER(_vp)]
lib.ajib_tiler_release.restype = None


def img_buffer(arr):
    """An aji_img_buffer over a uint8 numpy array [h][w][c] (kept alive by the caller)."""
    h, w, c = arr.shape
    b = ImgBuffer()
    b.width, b.height, b.channels = w, h, c
    b.stride = arr.strides[0]
    b.data = arr.ctypes.data
    return b


class Image:
    """An aji_img_ctx (CUDA backend) on device `device_id` (0 = first)."""

    def __init__(self, device_id=0, device_ids=None):
        """device_ids: a list of aji_img_device ids for a context over several GPUs
        (ajib_img_create_multi)."""
        p = ImgCreateParams()
        p.api_version = AJI_IMAGE_API_VERSION
        p.backend = IMG_TENSORRT
        p.device_id = device_id
        err = C.create_string_buffer(512)
        if device_ids is not None:
            ids = (C.c_uint64 * len(device_ids))(*device_ids)
            h = lib.ajib_img_create_multi(C.byref(p), ids, len(device_ids), err, 512)
        else:
            h = lib.aji_img_create(C.byref(p), err, 512)
        if not h:
            raise AjibError(f"aji_img_create: {err.value.decode()}")
        self.handle = _vp(h)

    def load(self, path, tile=512, overlap=0, flags=0):
        mp = ImgModelParams()
        mp.onnx_path = path.encode()
        mp.tile_w = mp.tile_h = tile
        mp.overlap = overlap
        mp.flags = flags
        m = lib.aji_img_load(self.handle, C.byref(mp))
        if not m:
            raise AjibError(f"aji_img_load: {self.error()}")
        return _vp(m)

    def upscale(self, model, img, scale, progress=None):
        h, w, c = img.shape
        img = np.ascontiguousarray(img)
        out = np.zeros((h * scale, w * scale, c), np.uint8)
        bi, bo = img_buffer(img), img_buffer(out)
        cb = PROGRESS_FN(progress) if progress else PROGRESS_FN()
        rc = lib.aji_img_upscale(model, C.byref(bi), C.byref(bo), cb, None)
        return rc, out

    def error(self):
        return (lib.aji_img_last_error(self.handle) or b"").decode()

    def close(self):
        if self.handle:
            lib.aji_img_destroy(C.byref(self.handle))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


import numpy as np  # noqa: E402  (used by the helpers above)
