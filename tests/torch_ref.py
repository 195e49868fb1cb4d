"""A plain PyTorch fp32 reference of a whole plan (the semantics of sanity/native_ref.h:24-122,
ajiref::run_plan, as oracle/oracle_conv.c restates them): every conv in fp32 from fp16-valued
inputs and weights, activations and gates in fp32, each stored feature map rounded to fp16, the
depth-to-space output rounded once after the model-input skip is added. It runs on any torch
device, so the tests can check whole frames at BASELINE sizes on the GPU (TF32 off); the C oracle
stays the pinned checker on windows of rows. Test infrastructure only."""
import numpy as np

MODEL_INPUT, MODEL_OUTPUT = -2, -3
D2S = {0: 0, 1: 2, 2: 4, 3: 1, 4: 3}


def _f16r(t):
    return t.half().float()


def _conv_w(torch, w, dev):
    """[taps][cin][cout] -> torch [cout][cin][k][k], rounded to fp16 values."""
    w = np.asarray(w, np.float32).astype(np.float16).astype(np.float32)
    taps, cin, cout = w.shape
    k = 3 if taps == 9 else 1
    return torch.from_numpy(np.ascontiguousarray(w.reshape(k, k, cin, cout).transpose(3, 2, 0, 1))).to(dev)


def run_plan_torch(plan, x, device="cuda"):
    """x: NCHW [3][h][w] (numpy or torch, fp16-valued). Returns the NCHW fp32 output as a torch
    tensor on `device` (fp16-valued)."""
    import torch
    import torch.nn.functional as F
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    x = torch.as_tensor(np.asarray(x, np.float32) if not isinstance(x, torch.Tensor) else x).to(device).float()
    x = x.unsqueeze(0)
    u = plan.get("unshuffle", 1)
    feats = {}
    out = None
    with torch.no_grad():
        for s in plan["steps"]:
            bias = torch.from_numpy(np.asarray(s["bias"], np.float32)).to(device)
            if s["kind"] == 1:
                cat = torch.cat([feats[t] for t in s["srcs"]], dim=1)
                w = _conv_w(torch, s["w"], device)
                feats[s["dst"]] = _f16r(F.conv2d(cat, w, bias))
                continue
            if s["src"] == MODEL_INPUT:
                src = F.pixel_unshuffle(x, 2) if s.get("in_", 1) == 2 else x
            else:
                src = feats[s["src"]]
            v = F.conv2d(src, _conv_w(torch, s["w"], device), bias, padding=1)
            act = s.get("act", 0)
            if act == 1:
                v = torch.clamp_min(v, 0.0)
            elif act == 2:
                sl = torch.from_numpy(np.asarray(s["slope"], np.float32)).to(device).view(1, -1, 1, 1)
                v = torch.where(v >= 0, v, v * sl)
            elif act == 3:
                v = v / (1.0 + torch.exp(-v))
            gate = s.get("gate", 0)
            if gate == 1:
                v = feats[s["resid"]] + v
            elif gate == 2:
                aw = _conv_w(torch, np.asarray(s["att"][0], np.float32).reshape(1, s["cout"], s["cout"]), device)
                ab = torch.from_numpy(np.asarray(s["att"][1], np.float32)).to(device)
                o16 = _f16r(v)
                v = (feats[s["resid"]] + o16) * torch.tanh(F.conv2d(o16, aw, ab))
            elif gate == 3:
                v = (feats[s["resid"]] + v) * (torch.sigmoid(v) - 0.5)
            R = D2S[s.get("out", 0)]
            if R == 0:
                feats[s["dst"]] = _f16r(v)
                continue
            y = F.pixel_shuffle(v[:, :3 * R * R], R)
            if s.get("resid", -1) == MODEL_INPUT and u == 1:
                y = y + F.interpolate(x, scale_factor=R, mode="nearest")
            if s.get("out_clamp"):
                y = torch.clamp(y, 0.0, 1.0)
            out = _f16r(y)[0]
    return out
