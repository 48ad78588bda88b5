"""Golden fixtures (reference onnxruntime outputs), as the reference's
tests/Sdcb.SimdGcdrNet.Tests/GoldenData.cs and tests/GoldenDerive.cs load and
derive them.  The stored tensors are NCHW [1,3,h,w]; helpers here return
NHWC views, which is the layout of both the oracle and the CUDA backend.
"""
from __future__ import annotations

import json
import os

import numpy as np

DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
MODEL_DIR = os.path.join(DIR, "models")
GC_PATH = os.path.join(MODEL_DIR, "gcdrnet_gcnet_sim.onnx")
DR_PATH = os.path.join(MODEL_DIR, "gcdrnet_drnet_sim.onnx")
TAGS = ("small", "pad", "mid")


def manifest():
    with open(os.path.join(DIR, "manifest.json")) as fh:
        return json.load(fh)


def dims(tag):
    """(h, w, ph, pw, oh, ow) as GoldenData.Dims."""
    e = manifest()[tag]
    return e["h"], e["w"], e["ph"], e["pw"], e["orig_h"], e["orig_w"]


def bgr(tag) -> np.ndarray:
    """Tight BGR24 pixels [oh][ow][3] of {tag}_src.png (GoldenData.Bgr)."""
    from PIL import Image
    im = Image.open(os.path.join(DIR, f"{tag}_src.png")).convert("RGB")
    rgb = np.asarray(im, dtype=np.uint8)
    return np.ascontiguousarray(rgb[:, :, ::-1])


def f32_nchw(tag, name) -> np.ndarray:
    h, w, *_ = dims(tag)
    a = np.fromfile(os.path.join(DIR, f"{tag}_{name}.f32"), dtype="<f4")
    return a.reshape(1, 3, h, w)


def f32_nhwc(tag, name) -> np.ndarray:
    """ORT output ("shadow" = GC-Net, "output" = DR-Net) as NHWC [h][w][3]."""
    return np.ascontiguousarray(f32_nchw(tag, name)[0].transpose(1, 2, 0))


def input_nhwc(tag) -> np.ndarray:
    """GoldenDerive.Input: tight BGR / 255, top/left edge replicate pad, NHWC."""
    h, w, ph, pw, oh, ow = dims(tag)
    b = bgr(tag).astype(np.float32) / np.float32(255.0)
    ys = np.maximum(np.arange(h) - ph, 0)
    xs = np.maximum(np.arange(w) - pw, 0)
    return np.ascontiguousarray(b[ys][:, xs])


def dr_in_nhwc(tag) -> np.ndarray:
    """GoldenDerive.DrIn on the golden shadow: [x ; clamp(x / max(s,1e-6), 0, 1)]."""
    x = input_nhwc(tag)
    s = f32_nhwc(tag, "shadow")
    r = np.clip(x / np.maximum(s, np.float32(1e-6)), 0.0, 1.0).astype(np.float32)
    return np.ascontiguousarray(np.concatenate([x, r], axis=2))


def final_u8(tag) -> np.ndarray:
    """GoldenDerive.FinalU8: (int)(output*255) clamped, top/left pad cropped, [oh][ow][3]."""
    h, w, ph, pw, oh, ow = dims(tag)
    out = f32_nhwc(tag, "output").astype(np.float64) * 255.0
    v = np.clip(np.trunc(out), 0, 255).astype(np.uint8)
    return np.ascontiguousarray(v[ph:, pw:])
