"""Benchmark: BASELINE config 1 — SRVGGNetCompact 2x video, 1920x1080 P010 -> 3840x2160 P010,
fp16 net with random-init seeded weights, through the engine's video C ABI (include/aji.h:
aji_create / aji_configure / aji_infer).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|refgpu] [--model M]

A step is one frame through pre-pass -> 18 fused convs -> post-pass. `value` is frames/s over all
ranks with frames already resident in HBM (device-timed with CUDA events on the launching
stream, max over ranks). N > 1: one process per GPU (torchrun), each rank upscales its own
frames, no collectives on the data path ("scaling": "weak"); a gloo group only carries barriers
and the max of the per-rank times. `e2e` is the product's own multi-GPU path: rank 0 drives
ajib_video_create_multi over devices 0..N-1 (frame k on device k mod N, results in submission
order) with the frames in pinned host memory, each frame's upload and download inside the
device-timed region (max over the GPUs).

--impl reference times the reference's own CPU implementation of this path (the fp32 reference
net sanity/native_ref.h:run_plan, compiled from the reference sources into oracle/_ref) on the
host cores, on a bounded sample of the same frame (a band of rows through all 18 steps); where
that build is absent, the oracle's restatement of it.

--model spanf3 runs the same video path with the shipping AnimeJaNai V3.1 HD "Performance"
structure instead (SPANF3, 48 features x 5 blocks, 2x pixel-unshuffled input, tanh 1x1 gates,
depth-to-space 4): not a BASELINE config, but the reference publishes a number for it
(2.02-2.06 ms per 1080p chain on an RTX 5090).
"""
import argparse
import atexit
import ctypes as C
import datetime
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "animejanai-inference_b200"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

from synth import p010_frame  # noqa: E402  (seeded synthetic frames, shared with the tests)

W_IN, H_IN, SCALE = 1920, 1080, 2
MODEL_SEED = 1
METRIC = "frames/s 1080p->4K 2x Compact fp16 at 1/2/4/8 B200; % tensor-core peak"
SPANF3_PUBLISHED_MS = 2.02  # the reference on an RTX 5090, Linux (BENCHMARKS.md:257)

# The workloads: BASELINE config 1 (the headline, default), config 3 (SPAN), config 4 (a chain of
# two Compact nets, 960x540 -> 1920x1080 -> 3840x2160, through animejanai.conf), and the shipping
# SPANF3 structure. Each runs through the video ABI on P010 frames.
MODELS = {
    "compact": dict(metric=METRIC, w=1920, h=1080,
                    workload="BASELINE config 1: Compact 2x video, 1920x1080 P010 BT.709 limited -> 3840x2160 P010",
                    model="SRVGGNetCompact 64 feat x 16 body, PReLU, pixel_shuffle 2, random-init (seed 1)",
                    kernel="k_conv3x3_tc<64,64> (body conv 64->64 + PReLU, 1920x1080)"),
    "span": dict(metric="frames/s 1080p->4K 2x SPAN-S 48x6 fp16 (BASELINE config 3)", w=1920, h=1080,
                 workload="BASELINE config 3: SPAN 2x video, 1920x1080 P010 BT.709 limited -> 3840x2160 P010",
                 model="SPAN 48 feat x 6 blocks (SiLU, sigmoid gates, concat 1x1), pixel_shuffle 2, random-init (seed 1)",
                 kernel="k_conv3x3_tc<48,48> (SPAN body convs 48->48, SiLU / sigmoid gate, 1920x1080)"),
    "chain": dict(metric="frames/s 960x540->1080p->4K two-model Compact chain fp16 (BASELINE config 4)", w=960, h=540,
                  workload="BASELINE config 4: two Compact 2x nets chained by animejanai.conf, 960x540 P010 -> "
                           "3840x2160 P010 (a stream of frames, frame-parallel over ranks)",
                  model="2 x SRVGGNetCompact 64x16 2x, random-init (seeds 1, 2)",
                  kernel="k_conv3x3_tc<64,64> (second net's body conv 64->64 + PReLU, 1920x1080)"),
    "suc-image": dict(metric="images/s 2048x2048->8192x8192 4x SuperUltraCompact 24x8 fp16, tiles 512 overlap 16 "
                               "(BASELINE config 2)", w=2048, h=2048,
                      workload="BASELINE config 2: one 2048x2048 8-bit RGB image, SuperUltraCompact 4x, tiled on the "
                               "device as 25 tiles of 512 with 16 px overlap and linear blending -> 8192x8192 8-bit RGB",
                      model="SRVGGNetCompact 24 feat x 8 body (SuperUltraCompact), PReLU, pixel_shuffle 4, random-init "
                            "(seed 1)",
                      kernel="k_conv3x3_tc<32,32> (SUC body conv 24->24 + PReLU over the 25 stacked 512x512 tiles)"),
    "spanf3": dict(metric="frames/s 1080p->4K 2x SPANF3 b5f48 unshuffle fp16 (video chain)", w=1920, h=1080,
                   workload="SPANF3 b5f48 2x video (2x pixel-unshuffle, tanh gates), 1920x1080 P010 BT.709 limited -> "
                            "3840x2160 P010",
                   model="SPANF3 48 feat x 5 blocks, unshuffle 2, depth-to-space 4, random-init (seed 1, 0.7 He)",
                   kernel="k_conv3x3_tc<48,48> (SPANF3 body convs 48->48, ReLU / tanh gate, 960x540)"),
}


def bench_plans(model):
    """The model's plans, in chain order (pure numpy: ajib_plans loads no library)."""
    import ajib_plans as P
    if model == "spanf3":
        return [P.spanf3_plan(MODEL_SEED, c=48, blocks=5, gain=0.7)]
    if model == "span":
        return [P.span_plan(MODEL_SEED, c=48, blocks=6)]
    if model == "chain":
        return [P.compact_plan(MODEL_SEED), P.compact_plan(MODEL_SEED + 1)]
    if model == "suc-image":
        return [P.compact_plan(MODEL_SEED, c=24, body=8, scale=4)]
    return [P.compact_plan(MODEL_SEED)]


def plan_scale(plan):
    return plan["depth_to_space"] // plan.get("unshuffle", 1)
# DRAM bytes (read + write) of one body-conv launch at 1920x1080, from the ncu capture summarised
# in profiles/conv3x3_body_64x64_1080p.txt (the roofline's "traffic")
BODY_TRAFFIC_BYTES = 501.0e6


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p.get("bf16_tflops_sustained", p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms, started before the warm-up
    steps so that it is sampling when the timed region begins. stop(t0, t1) keeps the samples
    taken inside the timed region [t0, t1] (host wall clock); a region shorter than the sampling
    period may hold none, and then the last sample taken before it ended (under the warm-up
    steps' load) stands in, marked by "window"."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            atexit.register(self._end)  # an exception before stop() must not leave it sampling
        except Exception:
            self.proc = None

    def _end(self):
        if self.proc and self.proc.poll() is None:
            self.proc.kill()

    def wait_first(self, timeout=5.0):
        """Wait (at most `timeout` seconds) until the first sample has been written."""
        t_end = time.time() + timeout
        while self.proc and time.time() < t_end:
            if os.path.getsize(self.path) > 0:
                return
            time.sleep(0.02)

    def stop(self, t0=None, t1=None):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        rows = []  # (time, sm MHz, max MHz, reasons)
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 8:
                    continue
                try:
                    ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f")
                except ValueError:
                    ts = None  # an unexpected timestamp format: the sample counts as inside
                try:
                    row = (ts, float(parts[1]), float(parts[2]),
                           {n for n, v in zip(names, parts[4:8]) if v.lower() == "active"})
                except ValueError:
                    continue
                rows.append(row)
        os.unlink(self.path)
        window = "timed region"
        if t0 is not None and t1 is not None:
            inside = [r for r in rows if r[0] is None or t0 <= r[0] <= t1]
            if not inside:
                inside, window = [r for r in rows if r[0] <= t1][-1:], "last sample before the timed region ended"
            rows = inside
        if not rows:
            return None
        reasons = set().union(*(r[3] for r in rows))
        return {"sm_mhz": float(np.median([r[1] for r in rows])), "sm_max_mhz": max(r[2] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows), "window": window}


CPU_BAND_ROWS = 16  # the CPU baseline's sample: a band of this many input rows of the frame


def cpu_baseline_sample(rows=CPU_BAND_ROWS, nthreads=0, model="compact"):
    """The reference CPU path on a bounded sample: a band of `rows` input rows of a P010 frame
    through the colour pre pass, the net(s) (every step; a chain's second net on the first's
    output band) and the colour post pass, timed on the host cores. The net is the reference's own
    run_plan (sanity/native_ref.h) compiled from its sources into oracle/_ref when built, else the
    oracle's restatement; the colour passes are the oracle's restatement of src/kernels.cu (the
    reference has no CPU colour code). Loads neither libaji.so nor the GPU.
    Returns (frames/s extrapolated from the band, band seconds, cores, kind, sample)."""
    from util import oracle_post, oracle_pre
    spec = MODELS[model]
    plans = bench_plans(model)
    u = plans[0].get("unshuffle", 1)
    rows = max(rows, 2 * u)
    y, uv = p010_frame(7, spec["w"], rows)
    ref_lib = os.path.join(ROOT, "oracle", "_ref", "libref_net.so")
    if os.path.exists(ref_lib):
        import refnet

        def net(plan, x):
            return refnet.run_plan(ref_lib, plan, x, nthreads)
        cores, kind = refnet.threads(ref_lib, nthreads), "reference"
    else:
        import oracle_net

        def net(plan, x):
            return oracle_net.run_plan(plan, x, nthreads)
        cores, kind = (nthreads if nthreads > 0 else os.cpu_count()), "port"
    t0 = time.perf_counter()
    x = oracle_pre(2, y, uv, 2, 1, 1).view(np.float16).astype(np.float32)
    for plan in plans:
        x = net(plan, x)
    oracle_post(2, x.astype(np.float16).view(np.uint16), 2, 1, 1)
    dt = time.perf_counter() - t0
    fps = rows / spec["h"] / dt
    nsteps = sum(len(p["steps"]) for p in plans)
    return fps, dt, cores, kind, (f"a {spec['w']}x{rows} P010 band of the {spec['w']}x{spec['h']} frame: colour pre "
                                  f"pass, all {nsteps} net steps ({kind} run_plan), colour post pass; "
                                  f"{dt:.2f} s per band, frames/s = {rows}/{spec['h']} frame / band time")


def run_reference(args, rank, world):
    """The reference's CPU implementation of the path on the host cores, on rank 0 only. A step is
    one band sample (cpu_baseline_sample); value = frames/s extrapolated from the bands."""
    if rank != 0:
        return
    bands = []
    info = None
    for i in range(args.warmup + args.steps):
        fps, dt, cores, kind, sample = cpu_baseline_sample(model=args.model)
        if i >= args.warmup:
            bands.append(dt)
        info = (cores, kind, sample)
    band_s = float(np.mean(bands))
    spec = MODELS[args.model]
    rows = max(CPU_BAND_ROWS, 2 * bench_plans(args.model)[0].get("unshuffle", 1))
    v = rows / spec["h"] / band_s
    line = {"impl": "reference", "metric": spec["metric"], "value": v, "unit": "frames/s",
            "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * band_s, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": spec["workload"] + ", reference CPU path on band samples", "model": spec["model"],
                       "step": f"one {spec['w']}x{rows} band of the frame through the whole path (ms_per_step is "
                               f"the band's time); value = {rows}/{spec['h']} frame per step / ms_per_step, "
                               "an extrapolation to whole frames"},
            "cpu_baseline": {"value": v, "unit": "frames/s", "cores": info[0], "kind": info[1], "sample": info[2]},
            "e2e": {"value": v, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


class RefCsp(C.Structure):
    _fields_ = [("kr", C.c_float), ("kb", C.c_float), ("yoff", C.c_float), ("yscale", C.c_float),
                ("coff", C.c_float), ("cscale", C.c_float)]


def reference_gpu_bar(args, plans, spec, frames_in, stream, dev):
    """The reference's own native video path on this B200, on the same frames: its colour kernels
    (src/kernels.cu aji_run_pre / aji_run_post) and its executor (src/native/executor.cpp, one
    mma.sync k_conv3x3 / k_concat1x1 launch per plan step), all compiled for sm_100a from its
    sources into oracle/_ref. K frames timed with CUDA events on the launching stream, as this
    engine's frames are; plus the reference's body conv (64 -> 64 + PReLU at the frame's size)
    alone. Returns (fields for the JSON line, the P010 output of frame 0)."""
    import torch
    import refnet
    kern = os.path.join(ROOT, "oracle", "_ref", "libref_kernels.so")
    exe = os.path.join(ROOT, "oracle", "_ref", "libref_exec.so")
    if not (os.path.exists(kern) and os.path.exists(exe)):
        return {"unavailable": "the reference's GPU kernels are not built (oracle/_ref)"}, None
    ref = C.CDLL(kern)
    ref.aji_pre_plan_create.restype = C.c_void_p
    ref.aji_post_plan_create.restype = C.c_void_p
    ref.aji_pre_plan_create.argtypes = [C.c_int] * 5
    ref.aji_post_plan_create.argtypes = [C.c_int] * 5
    ref.aji_run_pre.argtypes = [C.c_void_p, C.c_void_p, C.c_ssize_t, C.c_void_p, C.c_ssize_t, C.c_void_p, C.c_void_p,
                                C.c_void_p]
    ref.aji_run_post.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_ssize_t, C.c_void_p, C.c_ssize_t,
                                 C.c_void_p]
    ref.aji_make_csp.restype = RefCsp
    ref.aji_make_csp.argtypes = [C.c_int] * 3
    ref.aji_plan_destroy.argtypes = [C.c_void_p]
    sp = stream.cuda_stream
    W, H = spec["w"], spec["h"]
    csp = ref.aji_make_csp(2, 2, 1)
    sizes, cw, ch = [], W, H
    for pl in plans:
        sizes.append((cw, ch))
        cw, ch = cw * plan_scale(pl), ch * plan_scale(pl)
    OW, OH = cw, ch
    execs = [refnet.RefExec(exe, pl, w_, h_, sp) for pl, (w_, h_) in zip(plans, sizes)]
    bufs = [torch.empty((3, h_, w_), dtype=torch.float16, device=dev) for (w_, h_) in sizes]
    bufs.append(torch.empty((3, OH, OW), dtype=torch.float16, device=dev))
    pre = ref.aji_pre_plan_create(2, W, H, 1, 0)
    post = ref.aji_post_plan_create(2, OW, OH, 1, 0)
    oy = torch.empty((OH, OW), dtype=torch.int16, device=dev)
    ouv = torch.empty((OH // 2, OW), dtype=torch.int16, device=dev)

    def frame(i):
        yi, uvi = frames_in[i % len(frames_in)]
        assert ref.aji_run_pre(pre, yi.data_ptr(), W * 2, uvi.data_ptr(), W * 2, C.byref(csp), bufs[0].data_ptr(),
                               sp) == 0
        for k, e in enumerate(execs):
            assert e.run(bufs[k].data_ptr(), bufs[k + 1].data_ptr(), sp) == 0
        assert ref.aji_run_post(post, bufs[-1].data_ptr(), C.byref(csp), oy.data_ptr(), OW * 2, ouv.data_ptr(),
                                OW * 2, sp) == 0

    n = max(3, min(args.steps, 50))
    for i in range(3):
        frame(i)
    stream.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(n):
        frame(i)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / n
    frame(0)
    stream.synchronize()
    out0 = (oy.cpu().numpy().view(np.uint16).copy(), ouv.cpu().numpy().view(np.uint16).copy())
    for e in execs:
        e.close()
    ref.aji_plan_destroy(pre)
    ref.aji_plan_destroy(post)
    fields = {"what": "the reference's native video path (aji_run_pre -> Executor::run, one mma.sync k_conv3x3 per "
                      "step -> aji_run_post) compiled for sm_100a from its own sources, same frames, same GPU",
              "frames": n, "ms_per_frame": ms, "frames_per_s": 1000.0 / ms}
    # the reference's body conv alone (the kernel to beat), where the model has one of 64 channels
    conv_lib = os.path.join(ROOT, "oracle", "_ref", "libref_conv.so")
    body = [st for st in plans[-1]["steps"] if st["kind"] == 0 and st.get("in_", 0) == 0 and st.get("out", 0) == 0]
    if os.path.exists(conv_lib) and body and body[0]["cin"] == 64 and body[0]["cout"] == 64:
        from util import conv_weights, to_f16_bits
        rc_ = C.CDLL(conv_lib)
        rc_.ref_conv_upload.restype = C.c_void_p
        rc_.ref_conv_upload.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int]
        rc_.ref_conv_launch.argtypes = [C.c_void_p] + [C.c_int] * 6 + [C.c_void_p] * 3 + [C.c_int] * 3 + [C.c_void_p]
        rc_.ref_conv_release.argtypes = [C.c_void_p]
        bw, bh = sizes[-1]
        rng = np.random.default_rng(0)
        w, b, sl = conv_weights(rng, 64, 64, prelu=True)
        wb = to_f16_bits(w)
        hw = rc_.ref_conv_upload(wb.ctypes.data, b.ctypes.data, sl.ctypes.data, 64, 64, 64, 64)
        src = torch.from_numpy(rng.uniform(-1, 1, size=(bh, bw, 64)).astype(np.float16)).to(dev)
        dst = torch.empty_like(src)

        def launch():
            assert rc_.ref_conv_launch(hw, 0, 2, 0, 0, 64, 64, src.data_ptr(), None, dst.data_ptr(), bh, bw, -1, sp) == 0
        for _ in range(3):
            launch()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        for _ in range(20):
            launch()
        c1.record(stream)
        c1.synchronize()
        fields["body_conv_ms"] = c0.elapsed_time(c1) / 20
        fields["body_conv"] = f"reference k_conv3x3<64,64,PReLU> at {bw}x{bh} alone, its own tile pick"
        rc_.ref_conv_release(hw)
    return fields, out0


def oracle_window_check(plan, y, uv, gy, guv, W, H):
    """The frame's P010 output on a window of rows against the oracle's own chain (pre pass, the
    net on the input rows the window's receptive field reaches, post pass), within the tests'
    3 codes of 10 bits. Untimed; for single-model workloads."""
    from oracle_net import run_plan
    from util import oracle_post, oracle_pre
    u = plan.get("unshuffle", 1)
    R = plan_scale(plan)
    radius = u * sum(1 for st in plan["steps"] if np.asarray(st["w"]).shape[0] == 9)
    a = (H // 2 - 4) // (2 * u) * (2 * u)
    b = a + 8
    # 8 more input rows each side: the post pass's 12-tap vertical chroma filter reaches 6 output rows
    c0, c1 = max(0, a - radius - 8) // (2 * u) * (2 * u), min(H, b + radius + 8)
    x = oracle_pre(2, y, uv, 2, 1, 1).view(np.float16).astype(np.float32)
    t0 = time.perf_counter()
    net = run_plan(plan, np.ascontiguousarray(x[:, c0:c1]))
    wy, wuv = oracle_post(2, net.astype(np.float16).view(np.uint16), 2, 1, 1)
    dt = time.perf_counter() - t0
    ly = (wy[R * (a - c0):R * (b - c0)] >> 6).astype(int)
    luv = (wuv[R * (a - c0) // 2:R * (b - c0) // 2] >> 6).astype(int)
    dy = int(np.abs((gy[R * a:R * b] >> 6).astype(int) - ly).max())
    duv = int(np.abs((guv[R * a // 2:R * b // 2] >> 6).astype(int) - luv).max())
    return {"input_rows": [a, b], "oracle_rows": [c0, c1], "max_code_diff_y": dy, "max_code_diff_uv": duv,
            "ok": dy <= 3 and duv <= 3, "oracle_s": dt}


CHAIN_STREAM_FRAMES = 240  # a stream of 240 frames through the two-model chain


def run_e2e_multi(args, world, plans, mdir, W, H, depth=2):
    """The e2e leg: the workload through ajib_video_create_multi over devices 0..world-1 from this
    one process, host frames in pinned memory. config 4 (chain) is its 240-frame stream; the other
    workloads run `steps` frames per GPU. Returns the line's e2e object."""
    import torch
    import ajib
    devices = list(range(world))
    if len(plans) == 1:
        vm = ajib.VideoMulti(devices, model_path=os.path.join(mdir, "m1.ajnm"), max_w=W, max_h=H, depth=depth)
    else:
        vm = ajib.VideoMulti(devices, conf_path=os.path.join(mdir, "animejanai.conf"), model_dir=mdir, slot=1,
                             depth=depth)
    ow, oh = vm.configure(W, H)
    nin = 2 * world
    hin = []
    for i in range(nin):
        y, uv = p010_frame(5000 + i, W, H)
        hin.append((torch.from_numpy(y.view(np.int16)).pin_memory(), torch.from_numpy(uv.view(np.int16)).pin_memory()))
    nout = 2 * depth * world  # output buffers in flight: one is reused once its frame has finished
    hout = [(torch.empty((oh, ow), dtype=torch.int16).pin_memory(),
             torch.empty((oh // 2, ow), dtype=torch.int16).pin_memory()) for _ in range(nout)]
    fin = [ajib.frame(W, H, ajib.FMT_P010, [y.data_ptr(), uv.data_ptr()], [W * 2, W * 2]) for y, uv in hin]
    fout = [ajib.frame(ow, oh, ajib.FMT_P010, [y.data_ptr(), uv.data_ptr()], [ow * 2, ow * 2]) for y, uv in hout]
    tickets = []

    def submit(i):
        if i >= nout:
            assert vm.wait(tickets[i - nout]) == 0, vm.error()
        t = vm.submit(fin[i % nin], fout[i % nout])
        if t <= 0:
            raise RuntimeError(f"ajib_video_multi_submit failed: {t} {vm.error()}")
        tickets.append(t)

    for i in range(max(3, args.warmup) * world):
        submit(i)
    assert vm.wait(tickets[-1]) == 0, vm.error()
    nframes = CHAIN_STREAM_FRAMES if args.model == "chain" else args.steps * world
    tickets.clear()
    assert vm.timing(True) == 0, vm.error()
    t0 = time.perf_counter()
    for i in range(nframes):
        submit(i)
    assert vm.wait(tickets[-1]) == 0, vm.error()
    host_s = time.perf_counter() - t0
    ms = vm.device_ms()
    vm.close()
    t_ms = max(ms)
    h2d = (hin[0][0].numel() + hin[0][1].numel()) * 2
    d2h = (hout[0][0].numel() + hout[0][1].numel()) * 2
    return {"value": nframes / (t_ms / 1000.0), "unit": "frames/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "frames": nframes, "api": f"ajib_video_create_multi over {world} GPU(s) "
            f"(ring depth {depth}), pinned host frames, submission-order completion",
            "device_ms_max": t_ms, "device_ms": ms, "host_wall_s": host_s}


def current_context():
    """The CUDA driver context torch made current on this rank's device (passed to aji_create)."""
    import torch
    torch.cuda.current_stream().synchronize()
    cuda = C.CDLL("libcuda.so.1")
    ctx = C.c_void_p()
    cuda.cuCtxGetCurrent(C.byref(ctx))
    return ctx.value


def run_ours(args, rank, world, local_rank, dist):
    import torch
    import ajib

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    hbm_peak, tflops_burst, tflops_sus, peak_src = load_peaks()

    # model files (seeded random init); a chain through animejanai.conf
    spec = MODELS[args.model]
    W_IN, H_IN = spec["w"], spec["h"]
    plans = bench_plans(args.model)
    plan = plans[-1]  # the profiled (last) model
    spanf3 = args.model == "spanf3"
    mdir = tempfile.mkdtemp(prefix="ajib_bench_")
    for k, pl in enumerate(plans):
        with open(os.path.join(mdir, f"m{k + 1}.ajnm"), "wb") as f:
            f.write(ajib.model_bytes(pl))
    torch.zeros(1, device=dev)
    if args.bands > 1:
        os.environ["AJIB_BANDS"] = str(args.bands)  # read by aji_create
    if len(plans) == 1:
        vid = ajib.Video(os.path.join(mdir, "m1.ajnm"), W_IN, H_IN, cuda_context=current_context())
    else:
        conf = os.path.join(mdir, "animejanai.conf")
        with open(conf, "w") as f:
            f.write("[global]\nlogging=no\n\n[slot_1]\nprofile_name=bench\n" +
                    "".join(f"chain_1_model_{k + 1}_name=m{k + 1}\n" for k in range(len(plans))))
        vid = ajib.Video.from_conf(conf, mdir, slot=1, cuda_context=current_context())
    ow, oh = vid.configure(W_IN, H_IN)

    nfr = 4
    frames_in = []
    for i in range(nfr):
        y, uv = p010_frame(1000 * rank + i, W_IN, H_IN)
        frames_in.append((torch.from_numpy(y.view(np.int16)).to(dev), torch.from_numpy(uv.view(np.int16)).to(dev)))
    outs = [(torch.empty((oh, ow), dtype=torch.int16, device=dev), torch.empty((oh // 2, ow), dtype=torch.int16, device=dev))
            for _ in range(2)]
    stream = torch.cuda.Stream(device=dev)
    sp = stream.cuda_stream

    def fr(i):
        yi, uvi = frames_in[i % nfr]
        return ajib.frame(W_IN, H_IN, ajib.FMT_P010, [yi.data_ptr(), uvi.data_ptr()], [W_IN * 2, W_IN * 2])

    def fo(i):
        yo, uvo = outs[i % 2]
        return ajib.frame(ow, oh, ajib.FMT_P010, [yo.data_ptr(), uvo.data_ptr()], [ow * 2, ow * 2])

    fins = [fr(i) for i in range(nfr)]
    fouts = [fo(i) for i in range(2)]

    def step(i):
        rc = vid.infer(fins[i % nfr], fouts[i % 2], sp)
        if rc != 0:
            raise RuntimeError(f"aji_infer failed: {rc} {vid.error()}")

    def barrier():
        if dist is not None:
            dist.barrier()

    clocks = ClockSampler(local_rank)
    clocks.start()
    clocks.wait_first()
    for i in range(args.warmup):
        step(i)
    stream.synchronize()
    assert ajib.kernel_status() == 0, "a kernel pipeline wait timed out during warm-up"

    # ---- device-timed region (frames resident in HBM); no per-step events inside it (they would
    # split the programmatic overlap of consecutive kernels)
    prof = args.bands <= 1
    barrier()
    torch.cuda.synchronize()
    t0 = datetime.datetime.now()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    e1.synchronize()
    torch.cuda.synchronize()
    t1 = datetime.datetime.now()
    clk = clocks.stop(t0, t1)
    barrier()
    t_ms = e0.elapsed_time(e1)
    assert ajib.kernel_status() == 0, "a kernel pipeline wait timed out"
    # per-kernel times for the roofline: a separate run of the same frames with a CUDA-event pair
    # around every launch on the launching stream (ajib_video_profile)
    step_ms = np.zeros(64)
    step_n = np.zeros(64, dtype=np.int32)
    if prof:
        ajib.lib.ajib_video_profile(vid.handle, 1)
        for i in range(min(args.steps, 32)):
            step(i)
        stream.synchronize()
        ajib.lib.ajib_video_profile_read(vid.handle, step_ms.ctypes.data_as(C.POINTER(C.c_double)),
                                         step_n.ctypes.data_as(C.POINTER(C.c_int)), 64)
        ajib.lib.ajib_video_profile(vid.handle, 0)

    # ---- e2e through the product's multi-device entry point (ajib_video_create_multi), driven by
    # rank 0 over devices 0..N-1 while the other ranks wait: host frames in pinned memory, frame k
    # on device k mod N, each device uploading, upscaling and downloading on its own streams, the
    # results completing in submission order. Device-timed per GPU from its first upload's start
    # to its last download's end; the max over the GPUs is the time.
    barrier()
    e2e_info = None
    if rank == 0:
        e2e_info = run_e2e_multi(args, world, plans, mdir, W_IN, H_IN)
    barrier()

    # ---- untimed: the output of frame 0 (checksum, and a window of rows against the oracle's own
    # chain), and the reference's own GPU path on the same frames (N = 1 only)
    check = None
    ref_gpu = None
    if world == 1 and not args.no_check:
        step(0)
        stream.synchronize()
        gy = outs[0][0].cpu().numpy().view(np.uint16)
        guv = outs[0][1].cpu().numpy().view(np.uint16)
        import hashlib
        check = {"frame": 0, "p010_sha256": hashlib.sha256(gy.tobytes() + guv.tobytes()).hexdigest()}
        if len(plans) == 1:
            y0, uv0 = p010_frame(1000 * rank + 0, W_IN, H_IN)
            check["oracle_window"] = oracle_window_check(plan, y0, uv0, gy, guv, W_IN, H_IN)
        ref_gpu, rout = reference_gpu_bar(args, plans, spec, frames_in, stream, dev)
        if rout is not None:
            ref_gpu["speedup_frame"] = ref_gpu["ms_per_frame"] / (t_ms / args.steps)
            ref_gpu["max_code_diff_vs_this_engine"] = int(max(
                np.abs((rout[0] >> 6).astype(int) - (gy >> 6).astype(int)).max(),
                np.abs((rout[1] >> 6).astype(int) - (guv >> 6).astype(int)).max()))

    # max over ranks
    times = np.array([t_ms], dtype=np.float64)
    if dist is not None:
        import torch as _t
        tt = _t.from_numpy(times)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        times = tt.numpy()
    t_ms = float(times[0])

    if rank != 0:
        vid.close()
        return
    frames_total = args.steps * world
    value = frames_total / (t_ms / 1000.0)

    # roofline of the dominant kernel: the body convs (Compact: 16 x 64 -> 64 + PReLU; SPANF3:
    # 15 x 48 -> 48, ReLU or the tanh gate with its 1x1 attention GEMM), FLOPs at conv resolution
    u = plan.get("unshuffle", 1)
    pw, ph = W_IN, H_IN  # the profiled model's input size
    for pl in plans[:-1]:
        pw, ph = pw * plan_scale(pl), ph * plan_scale(pl)
    cpx = (pw // u) * (ph // u)
    body = [k for k, st in enumerate(plan["steps"])
            if st["kind"] == 0 and st.get("in_", 0) == 0 and st.get("out", 0) == 0]
    flops_steps = [2.0 * 9 * plan["steps"][k]["cin"] * plan["steps"][k]["cout"] * cpx +
                   (2.0 * plan["steps"][k]["cout"] ** 2 * cpx if plan["steps"][k].get("gate", 0) == 2 else 0.0)
                   for k in body]
    body_ms = None
    if prof and all(step_n[k] > 0 for k in body):
        body_ms = float(sum(step_ms[k] / step_n[k] for k in body) / len(body))
    roof = None
    if body_ms:
        # the kernel time comes from a short per-launch event pass (at most 32 frames, well under a
        # second), so the burst peak is the denominator; the sustained fraction is reported beside it
        flops_body = float(np.mean(flops_steps))
        achieved = flops_body / (body_ms / 1000.0) / 1e12
        frame_tf = chain_flops(plans, W_IN, H_IN) / (t_ms / args.steps / 1000.0) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": tflops_burst, "unit": "TFLOP/s",
                "frac": achieved / tflops_burst,
                "traffic": BODY_TRAFFIC_BYTES if args.model in ("compact", "chain") else None,
                "kernel": spec["kernel"],
                "kernel_ms": body_ms, "peak_source": f"{peak_src} bf16 burst (MEASURED_PEAKS.json)",
                "frac_of_sustained": achieved / tflops_sus, "flops_per_launch": flops_body,
                "frame_tflops": frame_tf, "frame_frac_of_burst": frame_tf / tflops_burst}

    nsteps = sum(len(pl["steps"]) for pl in plans)
    workload, model = spec["workload"], spec["model"]
    line = {"metric": spec["metric"], "value": value, "unit": "frames/s", "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": (value / world) / (1000.0 / SPANF3_PUBLISHED_MS) if spanf3 else None,
            "dtype": "f16", "data": "synthetic",
            "config": {"workload": workload, "model": model,
                       "global_batch": world, "parallelism": f"frame-parallel x{world} (replicas, no collectives)",
                       "l2": "inputs larger than L2 (activation buffers of 66-265 MB per frame)",
                       "bands": args.bands},
            "roofline": roof,
            "e2e": e2e_info,
            # in the timed region: pre, per net its input pack (fused into the pre pass for a first
            # net whose head reads the plain NCHW input) and steps, post
            "gpu_launches": args.steps * (2 + (nsteps + len(plans) - fused_pack(plans)) * max(1, args.bands)),
            "clocks": clk}
    if check is not None:
        line["check"] = check
    if ref_gpu is not None:
        if body_ms and "body_conv_ms" in ref_gpu and args.model in ("compact", "chain"):
            ref_gpu["speedup_body_conv"] = ref_gpu["body_conv_ms"] / body_ms
        line["reference_gpu"] = ref_gpu
    if spanf3:
        line["config"]["published"] = (f"reference {SPANF3_PUBLISHED_MS} ms per 1080p chain on an RTX 5090 "
                                       "(BENCHMARKS.md:257); vs_baseline is per GPU")
    if world == 1 and not args.no_cpu_baseline:
        fps, _, cores, kind, sample = cpu_baseline_sample(model=args.model)
        line["cpu_baseline"] = {"value": fps, "unit": "frames/s", "cores": cores, "kind": kind, "sample": sample}
    vid.close()
    print(json.dumps(line), flush=True)


def run_kernel(args):
    """The dominant kernel alone: the body conv (64 -> 64 + PReLU) at --size, K launches timed with
    CUDA events on the launching stream. --impl ours: this engine's tcgen05 kernel through
    ajib_conv3x3_launch; --impl refgpu: the reference's k_conv3x3 (mma.sync, fp16 accumulation)
    compiled for sm_100a from its own sources (oracle/_ref/libref_conv.so) with its own tile pick,
    the GPU bar the new kernel is measured against."""
    import torch
    import ajib
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from util import conv_weights, to_f16_bits, to_rows
    w_, h_ = (int(v) for v in args.size.split("x"))
    hbm_peak, tflops_burst, tflops_sus, peak_src = load_peaks()
    if args.kernel in ("pre", "post"):
        run_colour_kernel(args, torch.cuda.current_stream(), hbm_peak, peak_src)
        return
    rng = np.random.default_rng(0)
    x = rng.uniform(-1, 1, size=(h_, w_, 64)).astype(np.float16).astype(np.float32)
    w, b, sl = conv_weights(rng, 64, 64, prelu=True)
    s = torch.cuda.current_stream()
    if args.impl == "refgpu":
        ref = C.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref_conv.so"))
        ref.ref_conv_upload.restype = C.c_void_p
        ref.ref_conv_upload.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int]
        ref.ref_conv_launch.argtypes = [C.c_void_p] + [C.c_int] * 6 + [C.c_void_p] * 3 + [C.c_int] * 3 + [C.c_void_p]
        wb = to_f16_bits(w)
        hw = ref.ref_conv_upload(wb.ctypes.data, b.ctypes.data, sl.ctypes.data, 64, 64, 64, 64)
        src = torch.from_numpy(x.astype(np.float16)).cuda()
        dst = torch.empty_like(src)

        def launch():
            return ref.ref_conv_launch(hw, 0, 2, 0, 0, 64, 64, src.data_ptr(), None, dst.data_ptr(), h_, w_, -1,
                                       s.cuda_stream)
        kname = "reference k_conv3x3<64,64,...,PReLU> (mma.sync m16n8k16 fp16-acc) recompiled for sm_100a"
    elif args.kernel in ("conv48", "conv24"):
        # the SPAN (48) and SuperUltraCompact (24) body convs: same-width 3x3 with --act
        cw = int(args.kernel[4:])
        wk, bk, sk = conv_weights(rng, cw, cw, prelu=True)
        wt = ajib.Weights(to_f16_bits(wk), bk, sk)
        op = ajib.conv_op(wt, act={"none": ajib.ACT_NONE, "relu": ajib.ACT_RELU, "prelu": ajib.ACT_PRELU,
                                    "silu": ajib.ACT_SILU}[args.act])
        xc = rng.uniform(-1, 1, size=(h_, w_, cw)).astype(np.float16).astype(np.float32)
        src = torch.from_numpy(to_rows(xc).astype(np.float16)).cuda()
        dst = torch.zeros_like(src)

        def launch():
            return ajib.conv3x3(op, src.data_ptr(), 0, dst.data_ptr(), h_, w_, 0, 0, s.cuda_stream)
        kname = f"k_conv3x3_tc<{cw},{cw}> {args.act} (tcgen05, fp32 TMEM accumulation)"
    elif args.kernel == "conv64":
        wt = ajib.Weights(to_f16_bits(w), b, sl)
        op = ajib.conv_op(wt, act=ajib.ACT_PRELU)
        src = torch.from_numpy(to_rows(x).astype(np.float16)).cuda()
        dst = torch.zeros_like(src)

        def launch():
            return ajib.conv3x3(op, src.data_ptr(), 0, dst.data_ptr(), h_, w_, 0, 0, s.cuda_stream)
        kname = ("k_conv3x3_pair<64,64> (tcgen05 cta_group::2 over an SM pair, fp32 TMEM accumulation)" if ajib.on_pairs(op)
                 else "k_conv3x3_tc<64,64> (tcgen05, fp32 TMEM accumulation)")
    else:
        # the frame's other convs: head 3->64 from NCHW planes (or from an 8-channel row-chunked
        # map, "head8"), tail 64->12 with depth-to-space 2 and the model-input skip
        cin = {"head": 3, "head8": 8, "tail": 64}[args.kernel]
        cout = 12 if args.kernel == "tail" else 64
        wk, bk, sk = conv_weights(rng, cin, cout, prelu=args.kernel != "tail")
        wt = ajib.Weights(to_f16_bits(wk), bk, sk)
        mi = None
        if args.kernel == "head":
            op = ajib.conv_op(wt, in_=ajib.IN_NCHW3, act=ajib.ACT_PRELU)
            src = torch.from_numpy(rng.uniform(0, 1, size=(3, h_, w_)).astype(np.float16)).cuda()
            dst = torch.zeros(ajib.lib.ajib_feature_bytes(h_, w_, 64) // 2, dtype=torch.float16, device="cuda")
        elif args.kernel == "head8":
            op = ajib.conv_op(wt, act=ajib.ACT_PRELU)
            src = torch.from_numpy(to_rows(rng.uniform(0, 1, size=(h_, w_, 8)).astype(np.float32)).astype(np.float16)).cuda()
            dst = torch.zeros(ajib.lib.ajib_feature_bytes(h_, w_, 64) // 2, dtype=torch.float16, device="cuda")
        else:
            op = ajib.conv_op(wt, out=ajib.OUT_D2S2)
            src = torch.from_numpy(to_rows(x).astype(np.float16)).cuda()
            mi = torch.from_numpy(rng.uniform(0, 1, size=(3, h_, w_)).astype(np.float16)).cuda()
            dst = torch.zeros((3, 2 * h_, 2 * w_), dtype=torch.float16, device="cuda")

        def launch():
            return ajib.conv3x3(op, src.data_ptr(), 0 if mi is None else mi.data_ptr(), dst.data_ptr(), h_, w_, 0, 0,
                                s.cuda_stream)
        kname = f"k_conv3x3_tc {args.kernel} ({cin}->{cout})"
    for _ in range(args.warmup):
        assert launch() == 0
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(args.steps):
        assert launch() == 0
    e1.record(s)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    if args.kernel in ("conv64", None) or args.impl == "refgpu":
        flops, nbytes = 2.0 * 9 * 64 * 64 * w_ * h_, 2 * 2 * 64 * w_ * h_
    elif args.kernel in ("conv48", "conv24"):
        cw = int(args.kernel[4:])
        flops, nbytes = 2.0 * 9 * cw * cw * w_ * h_, 2 * 2 * cw * w_ * h_
    elif args.kernel in ("head", "head8"):
        flops, nbytes = 2.0 * 9 * 3 * 64 * w_ * h_, (3 * 2 + 64 * 2) * w_ * h_
    else:
        flops, nbytes = 2.0 * 9 * 64 * 12 * w_ * h_, (64 * 2 + 3 * 2 + 12 * 2) * w_ * h_
    tf = flops / (ms / 1000.0) / 1e12
    print(json.dumps({"kernel": kname, "impl": args.impl, "size": args.size, "ms_per_launch": ms, "tflops": tf,
                      "frac_of_burst_peak": tf / tflops_burst, "peak_source": peak_src,
                      "algorithmic_bytes": nbytes, "hbm_gbs_algorithmic": nbytes / (ms / 1000.0) / 1e9,
                      "frac_of_hbm_peak": nbytes / (ms / 1000.0) / 1e9 / hbm_peak}), flush=True)


def run_colour_kernel(args, s, hbm_peak, peak_src):
    """A colour pass alone, config 1's: `pre` converts a --size P010 frame (BT.709 limited, left
    siting) to fp16 NCHW RGB, `post` converts the 2x model output (fp16 NCHW RGB at twice --size)
    back to P010. K launches timed with CUDA events on the launching stream; algorithmic bytes are
    the frame's planes read and written once."""
    import torch
    import ajib
    w_, h_ = (int(v) for v in args.size.split("x"))
    rng = np.random.default_rng(0)
    fmt = 2
    csp = ajib.lib.aji_make_csp(fmt, 2, 1)
    if args.kernel == "pre":
        p = ajib.lib.aji_pre_plan_create(fmt, w_, h_, 1, 0)
        y = torch.from_numpy((rng.integers(64, 941, size=(h_, w_)).astype(np.uint16) << 6).view(np.int16)).cuda()
        uv = torch.from_numpy((rng.integers(64, 961, size=(h_ // 2, w_)).astype(np.uint16) << 6).view(np.int16)).cuda()
        out = torch.empty((3, h_, w_), dtype=torch.float16, device="cuda")

        def launch():
            return ajib.lib.aji_run_pre(p, y.data_ptr(), 2 * w_, uv.data_ptr(), 2 * w_, C.byref(csp), out.data_ptr(),
                                        s.cuda_stream)
        nbytes = 2 * w_ * h_ * 3 // 2 + 2 * 3 * w_ * h_
    else:
        w_, h_ = 2 * w_, 2 * h_
        p = ajib.lib.aji_post_plan_create(fmt, w_, h_, 1, 0)
        src = torch.from_numpy(rng.uniform(0, 1, size=(3, h_, w_)).astype(np.float16)).cuda()
        y = torch.empty((h_, w_), dtype=torch.int16, device="cuda")
        uv = torch.empty((h_ // 2, w_), dtype=torch.int16, device="cuda")

        def launch():
            return ajib.lib.aji_run_post(p, src.data_ptr(), C.byref(csp), y.data_ptr(), 2 * w_, uv.data_ptr(), 2 * w_,
                                         s.cuda_stream)
        nbytes = 2 * 3 * w_ * h_ + 2 * w_ * h_ * 3 // 2
    assert p
    form = ajib.lib.ajib_plan_kernel(p)
    for _ in range(args.warmup):
        assert launch() == 0
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(args.steps):
        assert launch() == 0
    e1.record(s)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    ajib.lib.aji_plan_destroy(p)
    gbs = nbytes / (ms / 1000.0) / 1e9
    print(json.dumps({"kernel": f"colour {args.kernel} ({'streaming' if form == 1 else 'tiled'} form)",
                      "size": f"{w_}x{h_}", "ms_per_launch": ms, "algorithmic_bytes": nbytes,
                      "hbm_gbs_algorithmic": gbs, "frac_of_hbm_peak": gbs / hbm_peak, "peak_source": peak_src}),
          flush=True)


IMG_TILE, IMG_OVERLAP = 512, 16


def run_image(args, rank, world, local_rank, dist):
    """the still-image path. `value`: images/s with the image resident in HBM,
    a step being the tiler's extract of all 25 tiles, the net over the 25 stacked tiles (one launch
    per step, ajib_exec_run_images) and the gather composition into the 8-bit output, device-timed
    with CUDA events, max over ranks (each rank its own images). `e2e`: aji_img_upscale (the image
    ABI, blocking) from host memory to host memory, on rank 0 over devices 0..N-1
    (ajib_img_create_multi when N > 1: output-row bands per GPU), host wall clock around each
    blocking call (its copies included). Roofline: the body conv, bound by HBM at 24 channels."""
    import torch
    import ajib
    from synth import rgb8_image
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    hbm_peak, tflops_burst, tflops_sus, peak_src = load_peaks()
    spec = MODELS[args.model]
    plan = bench_plans(args.model)[0]
    W, H, S = spec["w"], spec["h"], plan["depth_to_space"]
    torch.zeros(1, device=dev)
    t = C.c_void_p()
    ajib.check(ajib.lib.ajib_tiler_create(W, H, 3, S, IMG_TILE, IMG_TILE, IMG_OVERLAP, 0, C.byref(t)), "ajib_tiler_create")
    nx, ny, tw, th = C.c_int(), C.c_int(), C.c_int(), C.c_int()
    ajib.lib.ajib_tiler_info(t, C.byref(nx), C.byref(ny), C.byref(tw), C.byref(th))
    n, tw, th = nx.value * ny.value, tw.value, th.value
    model = ajib.Model(plan)
    ex = ajib.Exec(model, tw, th * n)
    img = rgb8_image(31 + rank, W, H)
    d_img = torch.from_numpy(img.reshape(-1)).to(dev)
    d_tin = torch.empty((3, n * th, tw), dtype=torch.float16, device=dev)
    d_tout = torch.empty((3, n * th * S, tw * S), dtype=torch.float16, device=dev)
    d_out = torch.empty(H * S * W * S * 3, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)
    sp = stream.cuda_stream

    def extract():
        ajib.check(ajib.lib.ajib_tiler_extract(t, C.c_void_p(d_img.data_ptr()), 0, n, C.c_void_p(d_tin.data_ptr()),
                                               C.c_void_p(sp)), "ajib_tiler_extract")

    def net():
        ajib.check(ex.run_images(d_tin.data_ptr(), d_tout.data_ptr(), tw, th, n, sp), "ajib_exec_run_images")

    def compose():
        ajib.check(ajib.lib.ajib_tiler_compose(t, C.c_void_p(d_tout.data_ptr()), C.c_void_p(d_out.data_ptr()),
                                               C.c_void_p(sp)), "ajib_tiler_compose")

    def step():
        extract()
        net()
        compose()

    def barrier():
        if dist is not None:
            dist.barrier()

    clocks = ClockSampler(local_rank)
    clocks.start()
    clocks.wait_first()
    for _ in range(args.warmup):
        step()
    stream.synchronize()
    assert ajib.kernel_status() == 0
    barrier()
    torch.cuda.synchronize()
    t0 = datetime.datetime.now()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    e1.synchronize()
    t1 = datetime.datetime.now()
    clk = clocks.stop(t0, t1)
    barrier()
    t_ms = e0.elapsed_time(e1)
    assert ajib.kernel_status() == 0

    # per-kernel times (a separate pass): extract and compose by events, the net's steps by the
    # executor's per-step events
    def timed(fn, reps=10):
        a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_.record(stream)
        for _ in range(reps):
            fn()
        b_.record(stream)
        b_.synchronize()
        return a_.elapsed_time(b_) / reps
    extract_ms, compose_ms = timed(extract), timed(compose)
    ex.profile(True)
    for _ in range(10):
        net()
    stream.synchronize()
    step_ms, step_n = ex.profile_read(len(plan["steps"]))
    ex.profile(False)
    body = [k for k, st in enumerate(plan["steps"]) if st.get("in_", 0) == 0 and st.get("out", 0) == 0]
    body_ms = float(np.mean([step_ms[k] / max(1, step_n[k]) for k in body]))
    net_ms = float(np.sum(step_ms / np.maximum(1, step_n)))
    px = n * th * tw
    body_bytes = 2.0 * px * 24 * 2   # read and write one 24-channel fp16 map of the stacked tiles
    body_flops = 2.0 * 9 * 24 * 24 * px
    extract_bytes = W * H * 3 + n * 3 * th * tw * 2
    compose_bytes = n * 3 * th * S * tw * S * 2 + W * S * H * S * 3

    # e2e through the image ABI, rank 0 over all the GPUs
    barrier()
    e2e = None
    if rank == 0:
        mdir = tempfile.mkdtemp(prefix="ajib_bench_")
        path = os.path.join(mdir, "suc.ajnm")
        with open(path, "wb") as f:
            f.write(ajib.model_bytes(plan))
        ctx = ajib.Image(device_ids=None) if world == 1 else ajib.Image(device_ids=_img_device_ids(world))
        mh = ctx.load(path, tile=IMG_TILE, overlap=IMG_OVERLAP)
        hin = torch.from_numpy(img).pin_memory()
        hout = torch.empty((H * S, W * S, 3), dtype=torch.uint8).pin_memory()
        bi, bo = ajib.img_buffer(hin.numpy()), ajib.img_buffer(hout.numpy())
        for _ in range(max(1, args.warmup)):
            assert ajib.lib.aji_img_upscale(mh, C.byref(bi), C.byref(bo), ajib.PROGRESS_FN(), None) == 0, ctx.error()
        reps = max(3, min(args.steps, 20))
        w0 = time.perf_counter()
        for _ in range(reps):
            assert ajib.lib.aji_img_upscale(mh, C.byref(bi), C.byref(bo), ajib.PROGRESS_FN(), None) == 0, ctx.error()
        wall = (time.perf_counter() - w0) / reps
        ajib.lib.aji_img_release(C.byref(mh))
        ctx.close()
        e2e = {"value": 1.0 / wall, "unit": "images/s", "h2d_bytes_per_step": W * H * 3,
               "d2h_bytes_per_step": W * S * H * S * 3, "api": f"aji_img_upscale over {world} GPU(s)"
               + (" (ajib_img_create_multi)" if world > 1 else "") + ", pinned host buffers",
               "timing": f"host wall clock around {reps} blocking calls"}
    barrier()
    times = np.array([t_ms], dtype=np.float64)
    if dist is not None:
        tt = torch.from_numpy(times)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        times = tt.numpy()
    t_ms = float(times[0])
    ajib.lib.ajib_tiler_release(C.byref(t))
    launches_net = ex.info()["launches"]  # the net's launches per run (the head's input pack included)
    if rank != 0:
        return
    achieved = body_bytes / (body_ms / 1000.0) / 1e9
    roof = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
            "traffic": None, "kernel": spec["kernel"], "kernel_ms": body_ms, "bytes_per_launch": body_bytes,
            "peak_source": f"{peak_src} HBM copy (MEASURED_PEAKS.json)",
            "tensor_tflops": body_flops / (body_ms / 1000.0) / 1e12,
            "tensor_frac_of_burst": body_flops / (body_ms / 1000.0) / 1e12 / tflops_burst,
            "extract": {"ms": extract_ms, "bytes": extract_bytes,
                        "frac_of_hbm": extract_bytes / (extract_ms / 1000.0) / 1e9 / hbm_peak},
            "compose": {"ms": compose_ms, "bytes": compose_bytes,
                        "frac_of_hbm": compose_bytes / (compose_ms / 1000.0) / 1e9 / hbm_peak},
            "net_ms": net_ms, "net_tflops": chain_flops([plan], tw, th * n) / (net_ms / 1000.0) / 1e12}
    value = args.steps * world / (t_ms / 1000.0)
    line = {"metric": spec["metric"], "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": spec["workload"], "model": spec["model"], "global_batch": world,
                       "parallelism": f"image-parallel x{world} (replicas) for value; e2e splits one image's output "
                                      "rows over the GPUs", "tiles_per_net_launch": n,
                       "l2": "inputs larger than L2 (629 MB of stacked tile outputs per image)"},
            "roofline": roof, "e2e": e2e,
            "gpu_launches": args.steps * (2 + launches_net), "clocks": clk}
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_image_sample(plan)
    print(json.dumps(line), flush=True)


def _img_device_ids(n):
    """The image ABI's device ids (aji_img_enum_devices) of CUDA devices 0..n-1."""
    import ajib
    devs = (ajib.ImgDevice * 64)()
    k = ajib.lib.aji_img_enum_devices(ajib.IMG_TENSORRT, devs, 64)
    return [devs[i].id for i in range(min(n, k))]


def cpu_image_sample(plan, nthreads=0):
    """The reference CPU path for config 2 on a bounded sample: one 512x512 tile of the image
    through the reference net (run_plan, oracle/_ref) on all host cores, scaled to the 25 tiles
    of a 2048x2048 image (the tiler's host-side blend is a small part of it)."""
    from synth import rgb8_image
    ref_lib = os.path.join(ROOT, "oracle", "_ref", "libref_net.so")
    x = (rgb8_image(31, IMG_TILE, IMG_TILE).astype(np.float32) / 255.0).transpose(2, 0, 1).copy()
    t0 = time.perf_counter()
    if os.path.exists(ref_lib):
        import refnet
        refnet.run_plan(ref_lib, plan, x, nthreads)
        cores, kind = refnet.threads(ref_lib, nthreads), "reference"
    else:
        import oracle_net
        oracle_net.run_plan(plan, x, nthreads)
        cores, kind = (nthreads if nthreads > 0 else os.cpu_count()), "port"
    dt = time.perf_counter() - t0
    return {"value": 1.0 / (25 * dt), "unit": "images/s", "cores": cores, "kind": kind,
            "sample": f"one 512x512 tile through the {kind} run_plan ({dt:.2f} s), x 25 tiles per image"}


def fused_pack(plans):
    """1 when the video path fuses the first net's input pack into the colour pre pass (its head
    reads the NCHW RGB input, plain or 2x pixel-unshuffled; the unshuffled map is written by the
    streaming pre kernel, which every bench frame width, a multiple of 16, takes), else 0."""
    import ajib
    head = plans[0]["steps"][0]
    return 1 if head["kind"] == 0 and head.get("in_", 0) in (ajib.IN_NCHW3, ajib.IN_NCHW3_UNSHUFFLE2) else 0


def chain_flops(plans, w, h):
    """Algorithmic FLOPs of one frame of w x h through the chain: every step's 2 * taps * cin * cout
    (plus a tanh gate's 2 * cout^2) per conv-resolution pixel."""
    total = 0.0
    for plan in plans:
        u = plan.get("unshuffle", 1)
        per_px = 0.0
        for s in plan["steps"]:
            per_px += 2.0 * s["w"].shape[0] * s["w"].shape[1] * s["w"].shape[2]
            if s["kind"] == 0 and s.get("gate", 0) == 2:
                per_px += 2.0 * s["cout"] ** 2
        total += per_px * (w // u) * (h // u)
        w, h = w * plan_scale(plan), h * plan_scale(plan)
    return total


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "refgpu"])
    ap.add_argument("--kernel", default=None,
                    choices=[None, "conv64", "conv48", "conv24", "head", "head8", "tail", "pre", "post"],
                    help="time the dominant kernel alone instead of the whole frame")
    ap.add_argument("--size", default="1920x1080")
    ap.add_argument("--act", default="prelu", choices=["none", "relu", "prelu", "silu"],
                    help="--kernel conv48 / conv24: the activation")
    ap.add_argument("--bands", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-check", action="store_true",
                    help="skip the untimed output check and the reference GPU bar")
    ap.add_argument("--model", default="compact", choices=list(MODELS),
                    help="compact: BASELINE config 1 (the headline); span: config 3; chain: config 4; "
                         "spanf3: the shipping SPANF3 structure")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.kernel:
        run_kernel(args)
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as td
        td.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
        dist = td
    try:
        if args.model == "suc-image":
            run_image(args, rank, world, local_rank, dist)
        else:
            run_ours(args, rank, world, local_rank, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
