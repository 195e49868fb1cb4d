"""CPU: libaji.so loads and exports every function include/*.h declares (what a dlopen/dlsym
caller such as the reference's dispatcher needs, src/aji_dispatch.cpp:186-228), and the host-only
parts of the engine (model file parsing and plan checks) behave."""
import ctypes as C
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = ["aji.h", "aji_image.h", "aji_b200.h"]

# the reference dispatcher's required symbols (src/aji_dispatch.cpp:186-228, aji_img_dispatch.cpp:105-124)
REQUIRED_VIDEO = ["aji_create", "aji_set_slot", "aji_configure", "aji_infer", "aji_flush", "aji_done", "aji_wait",
                  "aji_current_log", "aji_scale_factor", "aji_rife_factor", "aji_rife_before_upscale",
                  "aji_pre_resize", "aji_resize", "aji_poll", "aji_infer_rife", "aji_temporal_radius", "aji_ingest",
                  "aji_infer_seq", "aji_temporal_reset", "aji_last_error", "aji_destroy"]
REQUIRED_IMAGE = ["aji_img_enum_devices", "aji_img_create", "aji_img_load", "aji_img_model_state",
                  "aji_img_model_info_get", "aji_img_upscale", "aji_img_release", "aji_img_last_error",
                  "aji_img_destroy"]


def declared(header):
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = "\n".join(line for line in text.splitlines() if not line.lstrip().startswith("#"))
    return re.findall(r"(?:AJI_EXPORT|AJI_IMG_EXPORT|AJIB_EXPORT)[^;(]*?\b(\w+)\s*\(", text)


def test_library_exports_every_declared_symbol():
    import ajib
    names = [n for h in HEADERS for n in declared(h)]
    assert len(names) > 40
    missing = [n for n in names if not hasattr(ajib.lib, n)]
    assert not missing, f"declared but not exported: {missing}"


@pytest.mark.parametrize("name", REQUIRED_VIDEO)
def test_reference_required_video_symbols(name):
    import ajib
    assert hasattr(ajib.lib, name)


@pytest.mark.parametrize("name", REQUIRED_IMAGE)
def test_reference_required_image_symbols(name):
    import ajib
    assert hasattr(ajib.lib, name)


def test_model_roundtrip_and_info():
    import ajib
    m = ajib.Model(ajib.compact_plan(1))
    assert m.steps == 18 and m.scale == 2
    assert m.flops_per_px == 1196928.0  # 1,196,928 FLOP per input pixel
    s = ajib.Model(ajib.span_plan(1))
    assert s.steps == 23 and s.scale == 2
    assert s.flops_per_px == 819360.0 + 41472.0  # + the recomputed c1 of the last block
    u = ajib.Model(ajib.compact_plan(1, c=24, body=8, scale=4))
    assert u.steps == 10 and u.scale == 4 and u.flops_per_px == 104976.0


def test_model_refusals():
    import ajib
    good = ajib.model_bytes(ajib.compact_plan(1, body=2))
    for bad, why in [(b"XXXX" + good[4:], "magic"), (good[:-7], "truncated"), (good + b"\0", "trailing")]:
        with pytest.raises(ajib.AjibError, match=why):
            _load_bytes(bad)
    plan = ajib.compact_plan(1, body=2)
    plan["steps"][1]["src"] = 5  # reads a tensor nobody wrote
    with pytest.raises(ajib.AjibError, match="source"):
        ajib.Model(plan)
    plan = ajib.compact_plan(1, body=2)
    plan["steps"][1]["slope"] = None  # PReLU without slopes
    with pytest.raises(ajib.AjibError, match="PReLU"):
        ajib.Model(plan)


def _load_bytes(data):
    import ajib
    h = C.c_void_p()
    err = C.create_string_buffer(512)
    rc = ajib.lib.ajib_model_from_memory(data, len(data), C.byref(h), err, 512)
    if rc != 0:
        raise ajib.AjibError(err.value.decode())
    ajib.lib.ajib_model_release(C.byref(h))


def test_video_create_refuses_bad_params():
    import ajib
    p = ajib.CreateParams()
    p.api_version = 8
    assert not ajib.lib.aji_create(C.byref(p))
    p.api_version = ajib.AJI_API_VERSION
    # direct mode without a model file, and (here, without a GPU) conf mode too, give no context
    assert not ajib.lib.aji_create(C.byref(p))
    p.conf_path = b"/nonexistent/animejanai.conf"
    assert not ajib.lib.aji_create(C.byref(p))


def test_csp_constants():
    """aji_make_csp against the standard BT constants (reference src/resample.h:100-129)."""
    import ajib
    c = ajib.lib.aji_make_csp(ajib.FMT_P010, ajib.MATRIX_BT709, ajib.RANGE_LIMITED)
    assert (c.kr, c.kb) == (np.float32(0.2126), np.float32(0.0722))
    assert (c.yoff, c.yscale, c.coff, c.cscale) == (4096.0, 56064.0, 32768.0, 57344.0)
    c = ajib.lib.aji_make_csp(ajib.FMT_NV12, ajib.MATRIX_BT601, ajib.RANGE_FULL)
    assert (c.yoff, c.yscale, c.coff, c.cscale) == (0.0, 255.0, 128.0, 255.0)
    c = ajib.lib.aji_make_csp(ajib.FMT_YUV444P12MSB, ajib.MATRIX_BT2020, ajib.RANGE_FULL)
    assert (c.yscale, c.coff) == (65520.0, 32768.0)
